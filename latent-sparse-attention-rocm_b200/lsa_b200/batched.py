"""Batched decode over sequences of different lengths (the 128k batched-decode configuration).

The reference selects per sequence (its gates build one index per sequence,
``src/lsa_rocm_lab/port/gates.py:59``) and reads a batch with per-row lists
(``read_kernel_tiled.py:92-156``). Here every sequence keeps its own buckets; the tables are
concatenated, and ONE launch (``lsa_select_batched``) selects for all rows, row r reading
rows ``[table_off[r], table_off[r] + table_rows[r])``. Row r's lists equal ``flat_select``
on its own sequence's buckets, byte for byte. The read is the ordinary batched sparse read
over ``k``/``v`` ``[B, T_max, Hkv, Dh]`` (positions past a sequence's length are never listed).

Multi-GPU: sequences are independent units, so ranks take contiguous sequence ranges
(``shard_rows``) with no collective on the data path.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, pipeline
from ._lib import check, lib, ptr, require_cuda, stream_of


@dataclass
class BatchedBuckets:
    """Concatenated per-sequence bucket tables."""

    centroids: torch.Tensor  # [sum rows, d] bf16
    members: torch.Tensor  # [sum rows, cap] int32, positions within each row's sequence
    table_off: torch.Tensor  # [B] int64 first table row of each sequence
    table_rows: torch.Tensor  # [B] int32 bucket rows of each sequence
    max_rows: int
    centroids_f32: torch.Tensor | None = None


def concat_buckets(per_sequence: list) -> BatchedBuckets:
    """Per-sequence ``pipeline.Buckets`` -> one concatenated table set."""
    if not per_sequence:
        raise ValueError("concat_buckets needs at least one sequence")
    dev = per_sequence[0].centroids.device
    rows = [b.rows for b in per_sequence]
    off = [0]
    for n in rows[:-1]:
        off.append(off[-1] + n)
    f32 = None
    if all(b.centroids_f32 is not None for b in per_sequence):
        f32 = torch.cat([b.centroids_f32 for b in per_sequence]).contiguous()
    return BatchedBuckets(
        centroids=torch.cat([b.centroids for b in per_sequence]).contiguous(),
        members=torch.cat([b.members for b in per_sequence]).contiguous(),
        table_off=torch.tensor(off, dtype=torch.int64, device=dev),
        table_rows=torch.tensor(rows, dtype=torch.int32, device=dev),
        max_rows=max(rows),
        centroids_f32=f32,
    )


def build_batched_buckets(index_keys: list, config) -> BatchedBuckets:
    """``build_buckets_gpu`` per sequence (index keys ``[T_b, d]`` each), concatenated."""
    return concat_buckets([pipeline.build_buckets_gpu(ik, config) for ik in index_keys])


def batched_select(index_queries, positions, bb: BatchedBuckets, config, top_k=None, score_dtype="bf16"):
    """One row per sequence: (lists int32 [B, top_k + window + sink], lengths int32 [B])."""
    require_cuda(index_queries, positions, what="batched_select")
    top_k = config.top_k if top_k is None else int(top_k)
    if positions.shape[0] != index_queries.shape[0] or bb.table_off.shape[0] != index_queries.shape[0]:
        raise ValueError("batched_select: one index query, one position and one bucket table per sequence")
    if score_dtype == "fp32" and bb.centroids_f32 is None:
        raise ValueError("batched_select(score_dtype='fp32') needs fp32 centroids")
    q, q_code, c = pipeline._scoring_operands(index_queries, bb.centroids, bb.centroids_f32, score_dtype)
    R, d = q.shape
    dev = q.device
    width = top_k + config.window_size + config.sink_size
    lists = torch.empty(R, width, dtype=torch.int32, device=dev)
    lengths = torch.empty(R, dtype=torch.int32, device=dev)
    if R == 0:
        return lists, lengths
    pos = positions.to(torch.int32).contiguous()
    L = lib()
    sc = _lib.scratch(L.lsa_select_batched_scratch(R, bb.max_rows), dev)
    ct = _lib.counters(R + 1, dev)  # tickets + the status word
    check(L.lsa_select_batched(ptr(q), q_code, R, d, ptr(c), _lib.DTYPE_CODE[c.dtype], d,
                               ptr(bb.table_off), ptr(bb.table_rows), bb.max_rows, ptr(pos),
                               config.cluster_block_size, config.block_bucket_count, ptr(bb.members),
                               bb.members.shape[1], config.top_p, config.window_size, config.sink_size, top_k,
                               ptr(lists), ptr(lengths), ptr(sc), sc.numel(), ptr(ct), ct.numel(), -1, stream_of(q)),
          "batched_select")
    _lib.after_call(dev, "batched_select")
    return lists, lengths


def batched_decode(q, k, v, index_queries, positions, bb: BatchedBuckets, config, scale=None):
    """Select + read for one decoded token per sequence: q [B, 1, Hq, Dh] -> out like q."""
    lists, lengths = batched_select(index_queries, positions, bb, config)
    return pipeline.lsa_read(q, k, v, lists[:, None], lengths[:, None], scale)


def head_sharded_select(index_queries, positions, bb: BatchedBuckets, config, gather, top_k=None):
    """Head sharding without a replicated selection: this rank selects only its share of
    the sequences (``bb`` / ``index_queries`` / ``positions`` hold that share, equal shares
    on every rank), and one all-gather hands every rank every sequence's read list - the
    rank then reads its own KV heads of all sequences. ``gather`` maps x [...] to
    [world, ...] (``seqshard.all_gather_fn()`` over NCCL). Returns (lists [B, width],
    lengths [B]) with B = world x this rank's share, in rank order."""
    lists, lengths = batched_select(index_queries, positions, bb, config, top_k)
    # one exchange: each row's length rides as a last column of its list
    packed = gather(torch.cat([lists, lengths[:, None]], dim=1))  # [world, share, width + 1]
    packed = packed.reshape(-1, lists.shape[-1] + 1)
    return packed[:, :-1], packed[:, -1].contiguous()


def shard_rows(B: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous sequence range [start, end) of ``rank``: sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(B, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)
