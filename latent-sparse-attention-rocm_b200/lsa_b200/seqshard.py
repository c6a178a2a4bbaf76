"""Sequence-sharded tree decode (the 1M-context tree configuration over several GPUs).

The reference decodes a sequence on one device (``src/lsa_rocm_lab/port/_tree.py:318-373``
beam, ``pipeline.py:269`` expansion, ``read_kernel_tiled.py:41-89`` read). Here a sequence's
positions are split into contiguous, block-aligned shards, one per rank; every rank builds
the buckets and node hierarchy of its own shard. A decode step has one exchange per stage:

1. candidates: each rank runs the beam on its shard (``lsa_tree_select_keys``) and emits its
   best ``top_p`` packed keys with GLOBAL bucket ids (score bits unchanged);
2. exchange: all-gather of the candidate keys (top_p x 8 bytes per rank and sequence);
3. selection: every rank takes the same best ``top_p`` of all candidates
   (``lsa_best_first_keys``: packed-key order, ties to the lower global bucket) and walks the
   expansion over the global member table (all-gathered once at build time, 4 bytes per
   member), so every rank holds the same read list;
4. partial read: each rank reads the listed keys that fall in its shard
   (``lsa_sparse_read_partial``: fp32 output + log2-sum-exp per row and head);
5. exchange: all-gather of the partials, and the log-sum-exp merge (``lsa_merge_partials``).

The exchanges go through ``gather`` callables: ``peer_gather_fn`` (stores into the peers' memory
over NVLink, ``lsa_b200.peer``), ``torch.distributed.all_gather_into_tensor``
(NCCL over NVLink) across ranks, or a plain concatenation when one process emulates several
shards. With one shard the procedure is exactly the single-GPU tree decode.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, pipeline
from ._lib import check, lib, ptr, require_cuda, stream_of


def shard_bounds(C: int, world: int, rank: int, block: int) -> tuple[int, int]:
    """[start, end) of ``rank``'s positions: contiguous, whole cluster blocks, sizes within a block."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    blocks = (C + block - 1) // block
    base, extra = divmod(blocks, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return min(b0 * block, C), min(b1 * block, C)


@dataclass
class ShardIndex:
    start: int  # first global position of the shard
    length: int  # positions in the shard
    buckets: pipeline.Buckets  # member ids are shard-local positions
    hierarchy: pipeline.Hierarchy
    bucket_offset: int  # global id of the shard's bucket 0
    members_global: torch.Tensor | None = None  # [all buckets, cap] int32 global positions


def build_shard_index(index_keys: torch.Tensor, start: int, config) -> ShardIndex:
    """The shard's buckets and hierarchy from its index keys ``[length, d]`` (global ids later)."""
    buckets = pipeline.build_buckets_gpu(index_keys, config)
    hierarchy = pipeline.build_hierarchy_gpu(index_keys, buckets, config)
    return ShardIndex(start, index_keys.shape[0], buckets, hierarchy, 0)


def globalise(shards: list[ShardIndex], gathered_members: list[torch.Tensor] | None = None) -> None:
    """Set every shard's bucket offset and the global member table (in shard order).

    ``gathered_members``: the per-shard global member tables when the shards live on other
    ranks (see ``local_global_members``); None when every shard is in this process."""
    off = 0
    for s in shards:
        s.bucket_offset = off
        off += s.buckets.rows
    tables = gathered_members if gathered_members is not None else [local_global_members(s) for s in shards]
    table = torch.cat(tables).contiguous()
    for s in shards:
        s.members_global = table


def local_global_members(s: ShardIndex) -> torch.Tensor:
    """The shard's member table in global positions (-1 pads kept)."""
    m = s.buckets.members
    return torch.where(m >= 0, m + s.start, m).to(torch.int32).contiguous()


def _local_position(s: ShardIndex, pos: torch.Tensor) -> torch.Tensor:
    """Global decode positions -> the shard-local position the beam sees: a shard wholly
    before the query sees all its closed blocks; the query's shard sees its own prefix."""
    local = (pos.to(torch.int64) - s.start).clamp(max=s.length)
    return local.clamp(min=0).to(torch.int32).contiguous()


def shard_candidates(index_queries, positions, s: ShardIndex, config, local_positions=None) -> torch.Tensor:
    """The shard's best ``top_p`` packed keys [R, top_p] int64 with global bucket ids.
    ``local_positions``: the shard-local positions when already computed (shards alike)."""
    require_cuda(index_queries, positions, what="shard_candidates")
    if s.buckets.centroids_f32 is None:
        raise ValueError("the shard's tree scores buckets with centroids_f32")
    q = index_queries.float().contiguous()
    pos = _local_position(s, positions) if local_positions is None else local_positions
    R, d = q.shape
    dev = q.device
    levels = s.hierarchy.levels
    n = len(levels)
    picks = torch.empty(R, config.top_p, dtype=torch.int32, device=dev)
    keys = torch.empty(R, config.top_p, dtype=torch.int64, device=dev)
    if R == 0:
        return keys
    counts = (ctypes.c_int64 * max(n, 1))(*[lv.centroids.shape[0] for lv in levels])
    cents = [lv.centroids.float().contiguous() for lv in levels]
    kids = [lv.children.to(torch.int64).contiguous() for lv in levels]
    cptrs = (ctypes.c_void_p * max(n, 1))(*[c.data_ptr() for c in cents])
    kptrs = (ctypes.c_void_p * max(n, 1))(*[c.data_ptr() for c in kids])
    L = lib()
    sb, nc = ctypes.c_int64(), ctypes.c_int64()
    check(L.lsa_tree_plan(R, n, counts, config.beam_width, config.node_bucket_size, config.node_cluster_block_size,
                          config.block_bucket_count, config.top_p, ctypes.byref(sb), ctypes.byref(nc)),
          "shard_candidates")
    sc = _lib.scratch(sb.value, dev)
    ct = _lib.counters(nc.value, dev)
    bc = s.buckets.centroids_f32.float().contiguous()
    check(L.lsa_tree_select_keys(ptr(q), R, d, ptr(pos), config.cluster_block_size, config.block_bucket_count,
                                 s.buckets.rows, n, cptrs, kptrs, counts, ptr(bc), config.node_bucket_size,
                                 config.node_cluster_block_size, config.top_level, config.beam_width, config.top_p,
                                 ptr(picks), ptr(keys), s.bucket_offset, ptr(sc), sc.numel(), ptr(ct), ct.numel(),
                                 stream_of(q)), "shard_candidates")
    _lib.after_call(dev, "shard_candidates")
    return keys


def select_from_candidates(all_keys, positions, members_global, config, top_k=None):
    """All ranks' candidates [R, ranks * top_p] -> the read lists every rank shares."""
    best = pipeline.best_first_keys(all_keys.contiguous(), config.top_p)
    return expand_from_best(best, positions, members_global, config, top_k)


def expand_from_best(best, positions, members_global, config, top_k=None):
    """The expansion walk straight from the ordered packed keys [R, top_p] (no unpack pass)."""
    top_k = config.top_k if top_k is None else int(top_k)
    best = best.contiguous()
    R, P = best.shape
    width = top_k + config.window_size + config.sink_size
    lists = torch.empty(R, width, dtype=torch.int32, device=best.device)
    lengths = torch.empty(R, dtype=torch.int32, device=best.device)
    if R:
        mem = members_global.to(torch.int32).contiguous()
        pos = positions.to(torch.int32).contiguous()
        check(lib().lsa_expand_from_keys(ptr(best), R, P, P, ptr(mem), mem.shape[0], mem.shape[1], ptr(pos),
                                         config.window_size, config.sink_size, top_k, ptr(lists), ptr(lengths),
                                         stream_of(best)), "expand_from_best")
    return lists, lengths


def shard_partial_read(q, k_shard, v_shard, lists, lengths, start: int, scale=None):
    """This shard's part of the read: (fp32 output [R, Hq, D], log2-sum-exp [R, Hq])."""
    assert q.is_cuda and k_shard.is_cuda and v_shard.is_cuda, "the sparse read is a GPU kernel"
    B, Tq, Hq, D = q.shape
    Tk, Hkv = k_shard.shape[1], k_shard.shape[2]
    q, k_shard, v_shard = q.contiguous(), k_shard.contiguous(), v_shard.contiguous()
    width = lists.shape[-1]
    ids = lists.reshape(-1, width).to(torch.int32).contiguous()
    lens = lengths.reshape(-1).to(torch.int32).contiguous()
    out = torch.empty(B * Tq, Hq, D, dtype=torch.float32, device=q.device)
    lse = torch.empty(B * Tq, Hq, dtype=torch.float32, device=q.device)
    L = lib()
    splits, sb, nc = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    check(L.lsa_sparse_read_plan(B, Tq, Hq, Hkv, D, width, 0, ctypes.byref(splits), ctypes.byref(sb),
                                 ctypes.byref(nc)), "shard_partial_read")
    sc = _lib.scratch(sb.value, q.device)
    ct = _lib.counters(nc.value, q.device)
    scale = D ** -0.5 if scale is None else float(scale)
    check(L.lsa_sparse_read_partial(ptr(q), ptr(k_shard), ptr(v_shard), _lib.DTYPE_CODE[q.dtype], ptr(ids), ptr(lens),
                                    B, Tq, Tk, Hq, Hkv, D, width, scale, start, ptr(out), ptr(lse), ptr(sc),
                                    sc.numel(), ptr(ct), ct.numel(), 0, stream_of(q)), "shard_partial_read")
    _lib.after_call(q.device, "shard_partial_read")
    return out, lse


def merge_partials(outs: torch.Tensor, lses: torch.Tensor, dtype, shape):
    """[P, n, D] fp32 outputs + [P, n] log2-sum-exp -> the read over all shards, ``shape``/``dtype``."""
    outs, lses = outs.float().contiguous(), lses.float().contiguous()
    P, n, D = outs.shape
    res = torch.empty(n, D, dtype=dtype, device=outs.device)
    check(lib().lsa_merge_partials(ptr(outs), ptr(lses), P, n, D, _lib.DTYPE_CODE[dtype], ptr(res),
                                   stream_of(outs)), "merge_partials")
    return res.view(shape)


def all_gather_fn(group=None):
    """A gather over ranks: x [...] -> [world, ...] (torch.distributed, NCCL on GPUs)."""
    import torch.distributed as dist

    def gather(x: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(group)
        x = x.contiguous().reshape((-1,) + tuple(x.shape[1:])) if x.dim() else x.reshape(1)
        out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x, group=group)
        return out.view((world,) + tuple(x.shape))

    return gather


def peer_gather_fn(group=None):
    """A gather over ranks with the contract of ``all_gather_fn``, over peer memory: every rank
    stores its chunk into every peer's arena over NVLink and waits for their flags (two small
    kernels, ``lsa_b200.peer.PeerGather``; a collective to construct)."""
    from .peer import PeerGather

    return PeerGather(group)


def seqshard_decode(q, k_shard, v_shard, index_queries, positions, s: ShardIndex, config, gather, scale=None):
    """One decode step of a sequence sharded over ranks: q [1, R, Hq, D] (R query rows of the
    sequence), this rank's k/v shard [1, length, Hkv, D]. Every rank returns the full output."""
    keys = shard_candidates(index_queries, positions, s, config)  # [R, top_p]
    all_keys = gather(keys)  # [world, R, top_p]
    R = keys.shape[0]
    lists, lengths = select_from_candidates(all_keys.permute(1, 0, 2).reshape(R, -1), positions, s.members_global,
                                            config)
    out, lse = shard_partial_read(q, k_shard, v_shard, lists[None], lengths[None], s.start, scale)
    outs, lses = gather(out), gather(lse)  # [world, R, Hq, D], [world, R, Hq]
    Hq, D = out.shape[1], out.shape[2]
    return merge_partials(outs.reshape(outs.shape[0], -1, D), lses.reshape(lses.shape[0], -1), q.dtype, q.shape)


_SIDE_STREAMS: dict = {}


def _fan_out(fns, device):
    """Run each callable on its own side stream forked from the current one (an event wait,
    so it also forks a CUDA graph being captured), then join them back; the callables'
    tensors are marked as used by the current stream. Each side stream keeps its own
    workspaces (the package caches scratch and counters per stream)."""
    main = torch.cuda.current_stream(device)
    key = (device.index, len(fns))
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = [torch.cuda.Stream(device) for _ in fns]
    out = []
    for fn, st in zip(fns, _SIDE_STREAMS[key]):
        st.wait_stream(main)
        with torch.cuda.stream(st):
            out.append(fn())
    for st in _SIDE_STREAMS[key]:
        main.wait_stream(st)
    for r in out:
        for t in (r if isinstance(r, tuple) else (r,)):
            t.record_stream(main)
    return out


def one_shard_decode_batch(q, k, v, index_queries, positions, shards, config, scale=None):
    """``seqshard_decode_batch`` when one GPU holds every sequence whole (a single shard that
    starts at position 0): there is nothing to exchange, so each sequence's read lists come
    from its one-launch tree select (the beam and the expansion, ``lsa_tree_select_lists``;
    a side stream each) and one read covers all sequences. The lists equal the sharded
    procedure's with one shard (the beam's visible count is clamped to the shard's buckets
    either way); the output is one read instead of a partial read and a log-sum-exp merge,
    equal within the read's tolerance. Shapes as ``seqshard_decode_batch``."""
    B = len(shards)
    if q.shape[0] != B or k.shape[0] != B or v.shape[0] != B:
        raise ValueError("one_shard_decode_batch: one q / k / v batch row per shard index")
    if any(s.start != 0 or s.length != k.shape[1] for s in shards):
        raise ValueError("one_shard_decode_batch: every shard must hold its whole sequence from position 0")
    dev = q.device
    walks = _fan_out([lambda b=b: pipeline.tree_select(index_queries[b], positions, shards[b].buckets,
                                                       shards[b].hierarchy, config) for b in range(B)], dev)
    lists = torch.stack([w[0] for w in walks])
    lengths = torch.stack([w[1] for w in walks])
    return pipeline.lsa_read(q, k, v, lists, lengths, scale)


def seqshard_decode_batch(q, k, v, index_queries, positions, shards, config, gather, scale=None):
    """One decode step of several sharded sequences with TWO exchanges in all: the candidate
    keys of every sequence in one all-gather, the partial outputs and log2-sum-exps of every
    sequence in a second one, then one log-sum-exp merge over all of them. The partial reads
    of all sequences are ONE read call (the sequences as its batch rows).

    q [B, R, Hq, D]; this rank's shard of every sequence k / v [B, length, Hkv, D] (every
    sequence sharded alike: the shards start at the same position and hold as many
    positions); index_queries[b] [R, d];
    shards[b] the sequence's ShardIndex; positions [R] shared. Returns [B, R, Hq, D] in q's
    dtype, matching ``seqshard_decode`` sequence by sequence."""
    B = len(shards)
    if q.shape[0] != B or k.shape[0] != B or v.shape[0] != B:
        raise ValueError("seqshard_decode_batch: one q / k / v batch row per shard index")
    if any(s.start != shards[0].start for s in shards):
        raise ValueError("seqshard_decode_batch: every sequence's shard must start at the same position")
    if any(s.length != shards[0].length for s in shards):
        raise ValueError("seqshard_decode_batch: every sequence's shard must hold the same positions")
    local = _local_position(shards[0], positions)  # the same for every sequence
    dev = q.device
    # the sequences' beams are independent chains of small launches: one side stream each
    keys = torch.stack(_fan_out([lambda b=b: shard_candidates(index_queries[b], positions, shards[b], config, local)
                                 for b in range(B)], dev))
    all_keys = gather(keys)  # [world, B, R, top_p]
    R = keys.shape[1]
    # the best top_p of every sequence's candidates in one launch, then each sequence's walk
    best = pipeline.best_first_keys(all_keys.permute(1, 2, 0, 3).reshape(B * R, -1).contiguous(), config.top_p)
    walks = _fan_out([lambda b=b: expand_from_best(best[b * R:(b + 1) * R], positions, shards[b].members_global,
                                                    config) for b in range(B)], dev)
    lists, lengths = [w[0] for w in walks], [w[1] for w in walks]
    out, lse = shard_partial_read(q, k, v, torch.stack(lists), torch.stack(lengths), shards[0].start, scale)
    D = out.shape[-1]
    packed = torch.cat([out.reshape(-1, D), lse.reshape(-1, 1)], dim=1)  # [B R Hq, D + 1]
    g = gather(packed)  # [world, B R Hq, D + 1]
    return merge_partials(g[..., :D].contiguous(), g[..., D].contiguous(), q.dtype, tuple(q.shape))
