"""The LSA select + read pipeline on B200 - drop-in for ``lsa_rocm_lab.port.pipeline``.

Same names, arguments, outputs and errors as the reference module
(AIwork4me/latent-sparse-attention-rocm, ``src/lsa_rocm_lab/port/pipeline.py``), every
stage a hand-written sm_100a kernel behind the C-ABI in ``liblsa_b200.so``:

- ``build_buckets_gpu`` (ref ``:71-116``): pools, spherical Ward merge, members and
  centroids in four kernels (``lsa_build_buckets``);
- ``build_hierarchy_gpu`` (ref ``:153-181``): node-bucket pairing by halvings
  (``lsa_pair_to_size``) and normalised node centroids;
- ``flat_select`` (ref ``:274-316``) with the ``LSA_SELECT_IMPL`` switch, read per call:
  ``reference`` = the unfused kernel chain (scores, listing, best-first top-k, unpack,
  expansion), ``fused_unpack`` = the chain with the unpack folded into the walk,
  ``fused`` = ONE launch from index queries to read lists. All arms are byte-identical;
- ``tree_select`` (ref ``:319-337``), ``lsa_read`` (ref ``:373-375``),
  ``position_buckets`` (ref ``:378-403``), ``visible_counts``, ``best_first_keys``;
- ``dense_read`` (ref ``:340-370``) stays the torch SDPA baseline, as in the reference.

Selection arithmetic is canonical and deterministic (fixed-order fp32 dot, packed int64
keys with the lower column winning ties), so the lists are reproducible bit for bit.
Outputs are fresh tensors on the inputs' device; inputs are never mutated. Calls launch
on torch's current stream and do not synchronise, except the index builds, which read a
device status word to raise on an infeasible Ward merge.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _lib
from ._lib import BF16, F32, check, lib, ptr, require_cuda, stream_of
from .read_kernel_tiled import sparse_read_auto as sparse_read

EMPTY = torch.iinfo(torch.int64).min  # the empty packed key: sorts after every real key
WHOLE = 4  # the reference listing's whole-path factor (columns <= WHOLE * top_p)

SELECT_IMPLS = ("reference", "fused", "fused_unpack")


@dataclass(frozen=True)
class PortConfig:
    """The design's knobs (ref ``pipeline.py:32-54``)."""

    cluster_block_size: int = 512  # keys per Ward block; blocks become visible once closed
    pool_size: int = 4
    bucket_size: int = 8
    bucket_cap: int = 16
    top_p: int = 1024
    top_k: int = 4096
    window_size: int = 512
    sink_size: int = 4
    node_bucket_size: int = 4
    top_level: int = 3
    node_cluster_block_size: int = 64
    beam_width: int = 64
    start_nodes: int | None = None

    @property
    def block_bucket_count(self) -> int:
        return self.cluster_block_size // self.bucket_size


@dataclass
class Buckets:
    """A cache's buckets on the GPU (ref ``pipeline.py:57-68``) plus their fp32 key sums."""

    centroids: torch.Tensor  # [rows, index_dim] bf16, the scoring operand of the selects
    members: torch.Tensor  # [rows, bucket_cap] int32, absolute positions, -1 padded
    sizes: torch.Tensor  # [rows] int32
    centroids_f32: torch.Tensor | None = None  # [rows, index_dim] fp32
    key_sums: torch.Tensor | None = None  # [rows, index_dim] fp32, the hierarchy's pairing input

    @property
    def rows(self) -> int:
        return self.centroids.shape[0]


@dataclass
class NodeLevel:
    centroids: torch.Tensor  # [N, index_dim] fp32
    children: torch.Tensor  # [N, node_bucket_size] int64 - rows of the level below
    key_sums: torch.Tensor  # [N, index_dim] fp32


@dataclass
class Hierarchy:
    levels: list[NodeLevel] = field(default_factory=list)
    bucket_key_sums: torch.Tensor | None = None


# ------------------------------------------------------------------ builds


def _validate_build(config: PortConfig, index_dim: int) -> None:
    block, pool, cap, bpb = config.cluster_block_size, config.pool_size, config.bucket_cap, config.block_bucket_count
    if block % pool or block % config.bucket_size:
        raise ValueError("pool_size and bucket_size must divide cluster_block_size")
    if block // pool > 128:
        raise ValueError(f"{block // pool} pools per block: the Ward kernel keeps at most 128 (raise pool_size)")
    if index_dim % 8 or index_dim > 2048:
        raise ValueError(f"index_dim {index_dim} must be a multiple of 8 and at most 2048")
    if cap * (bpb + 1) < 2 * block:
        raise ValueError(f"bucket_cap {cap} cannot hold {block} keys in {bpb} buckets (cap * (bpb + 1) < 2 * block)")


def _status(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def _raise_status(status: torch.Tensor, what: str) -> None:
    code = int(status.item())
    if code:
        check(code, what)


def build_buckets_gpu(index_keys: torch.Tensor, config: PortConfig) -> Buckets:
    """Cluster every closed cluster block into buckets (ref ``pipeline.py:71-116``)."""
    require_cuda(index_keys, what="build_buckets_gpu")
    keys = index_keys.float().contiguous()
    T, d = keys.shape
    _validate_build(config, d)
    block, pool, bpb, cap = config.cluster_block_size, config.pool_size, config.block_bucket_count, config.bucket_cap
    rows = (T // block) * bpb
    dev = keys.device
    cf = torch.empty(rows, d, dtype=torch.float32, device=dev)
    cb = torch.empty(rows, d, dtype=torch.bfloat16, device=dev)
    members = torch.empty(rows, cap, dtype=torch.int32, device=dev)
    sizes = torch.empty(rows, dtype=torch.int32, device=dev)
    sums = torch.empty(rows, d, dtype=torch.float32, device=dev)
    if rows:
        L = lib()
        nbytes = L.lsa_build_buckets_workspace(T, d, block, pool)
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        status = _status(dev)
        check(L.lsa_build_buckets(ptr(keys), T, d, block, pool, bpb, cap, ptr(cf), ptr(cb), ptr(members),
                                  ptr(sizes), ptr(sums), ptr(ws), nbytes, ptr(status), stream_of(keys)),
              "build_buckets_gpu")
        _raise_status(status, "build_buckets_gpu")
    return Buckets(cb, members, sizes, centroids_f32=cf, key_sums=sums)


def position_buckets(index_keys: torch.Tensor, config: PortConfig) -> Buckets:
    """Positional block-sparse buckets: runs of ``bucket_size`` keys (ref ``pipeline.py:378-403``)."""
    require_cuda(index_keys, what="position_buckets")
    keys = index_keys.float().contiguous()
    T, d = keys.shape
    block, size, cap, bpb = config.cluster_block_size, config.bucket_size, config.bucket_cap, config.block_bucket_count
    if block % size or cap < size or d % 8:
        raise ValueError("bucket_size must divide cluster_block_size and fit bucket_cap; index_dim % 8 == 0")
    rows = (T // block) * bpb
    dev = keys.device
    cf = torch.empty(rows, d, dtype=torch.float32, device=dev)
    cb = torch.empty(rows, d, dtype=torch.bfloat16, device=dev)
    members = torch.empty(rows, cap, dtype=torch.int32, device=dev)
    sizes = torch.empty(rows, dtype=torch.int32, device=dev)
    sums = torch.empty(rows, d, dtype=torch.float32, device=dev)
    if rows:
        status = _status(dev)
        check(lib().lsa_position_buckets(ptr(keys), T, d, block, size, cap, ptr(cf), ptr(cb), ptr(members),
                                         ptr(sizes), ptr(sums), ptr(status), stream_of(keys)), "position_buckets")
        _raise_status(status, "position_buckets")
    return Buckets(cb, members, sizes, centroids_f32=cf, key_sums=sums)


def positional_picks(positions: torch.Tensor, buckets: Buckets, config: PortConfig, first: int = 4,
                     last: int = 4) -> torch.Tensor:
    """cfg 2's positional arm: first/last visible buckets plus strided ones, [R, top_p] int32."""
    require_cuda(positions, what="positional_picks")
    pos = positions.to(torch.int32).contiguous()
    picks = torch.empty(pos.shape[0], config.top_p, dtype=torch.int32, device=pos.device)
    check(lib().lsa_positional_picks(ptr(pos), pos.shape[0], config.cluster_block_size, config.block_bucket_count,
                                     buckets.rows, config.top_p, first, last, ptr(picks), stream_of(pos)),
          "positional_picks")
    return picks


def positional_select(positions, buckets: Buckets, config: PortConfig, top_k=None, first: int = 4, last: int = 4):
    """The positional decode arm over ``position_buckets``: static picks, the same expansion."""
    top_k = config.top_k if top_k is None else top_k
    picks = positional_picks(positions, buckets, config, first, last)
    return expand_in_order(picks, buckets.members, positions, config.window_size, config.sink_size, top_k)


def _normalize(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(x)
    if x.shape[0]:
        check(lib().lsa_normalize_rows(ptr(x), x.shape[0], x.shape[1], ptr(out), None, stream_of(x)), "normalize")
    return out


def _pair_to_size(sums: torch.Tensor, size: int):
    """One level's pairing (ref ``pipeline.py:136-150``): [blocks, n, d] -> labels [blocks, n],
    children order [blocks * n] int64 (absolute rows in node order), node sums."""
    blocks, n, d = sums.shape
    dev = sums.device
    labels = torch.empty(blocks, n, dtype=torch.int32, device=dev)
    order = torch.empty(blocks * n, dtype=torch.int64, device=dev)
    node_sums = torch.empty(blocks, n // size, d, dtype=torch.float32, device=dev)
    if blocks:
        L = lib()
        nbytes = L.lsa_pair_to_size_workspace(blocks, n, d)
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        status = _status(dev)
        check(L.lsa_pair_to_size(ptr(sums.contiguous()), blocks, n, d, size, ptr(labels), ptr(order),
                                 ptr(node_sums), ptr(ws), nbytes, ptr(status), stream_of(sums)), "pair_to_size")
        _raise_status(status, "pair_to_size")
    return labels, order, node_sums


def build_hierarchy_gpu(index_keys: torch.Tensor, buckets: Buckets, config: PortConfig) -> Hierarchy:
    """Pair every full node cluster block of every level (ref ``pipeline.py:153-181``)."""
    require_cuda(index_keys, what="build_hierarchy_gpu")
    size, block_size = config.node_bucket_size, config.node_cluster_block_size
    if size & (size - 1) or block_size % size or block_size > 128:
        raise ValueError("node_bucket_size must be a power of two dividing node_cluster_block_size (<= 128)")
    key_sums = buckets.key_sums
    if key_sums is None:
        raise ValueError("buckets carry no key_sums: build them with build_buckets_gpu / position_buckets")
    hierarchy = Hierarchy(bucket_key_sums=key_sums)
    while True:
        blocks = key_sums.shape[0] // block_size
        if not blocks or len(hierarchy.levels) >= config.top_level:
            break
        count = blocks * block_size
        _, order, node_sums = _pair_to_size(key_sums[:count].reshape(blocks, block_size, -1), size)
        key_sums = node_sums.reshape(-1, key_sums.shape[1])
        hierarchy.levels.append(NodeLevel(_normalize(key_sums), order.view(-1, size), key_sums.clone()))
    return hierarchy


# ------------------------------------------------------------------ select


def visible_counts(positions: torch.Tensor, buckets: Buckets, config: PortConfig) -> torch.Tensor:
    """Buckets each query sees: the closed blocks before its own (ref ``pipeline.py:184-186``)."""
    require_cuda(positions, what="visible_counts")
    pos = positions.to(torch.int32).contiguous()
    out = torch.empty(pos.shape[0], dtype=torch.int32, device=pos.device)
    check(lib().lsa_visible_counts(ptr(pos), pos.shape[0], config.cluster_block_size, config.block_bucket_count,
                                   buckets.rows, ptr(out), stream_of(pos)), "visible_counts")
    return out


def best_first_keys(keys: torch.Tensor, top_p: int, counts: torch.Tensor | None = None) -> torch.Tensor:
    """The best ``top_p`` packed keys per row, best first (ref ``pipeline.py:189-214``).

    ``counts`` masks slots at or past each row's count to EMPTY before the top-k (upstream
    ``TopK.best()``'s ``~listed`` mask)."""
    require_cuda(keys, what="best_first_keys")
    keys = keys.contiguous()
    R, N = keys.shape
    k = min(top_p, N)
    out = torch.empty(R, k, dtype=torch.int64, device=keys.device)
    cnt = None if counts is None else counts.to(torch.int32).contiguous()
    if R and k:
        check(lib().lsa_best_first_keys(ptr(keys), R, N, N, k, ptr(cnt), ptr(out), k, stream_of(keys)),
              "best_first_keys")
    return out


def unpack_ids(keys: torch.Tensor) -> torch.Tensor:
    """Packed keys -> bucket ids, -1 where EMPTY (upstream ``keys.unpack_ids``)."""
    require_cuda(keys, what="unpack_ids")
    keys = keys.contiguous()
    ids = torch.empty(keys.shape, dtype=torch.int32, device=keys.device)
    if keys.numel():
        check(lib().lsa_unpack_ids(ptr(keys), keys.numel(), ptr(ids), stream_of(keys)), "unpack_ids")
    return ids


def pack_keys(scores: torch.Tensor, lengths: torch.Tensor) -> torch.Tensor:
    """The whole-path listing: every column packed, EMPTY at or past the row's length."""
    require_cuda(scores, what="pack_keys")
    R, N = scores.shape
    keys = torch.empty(R, N, dtype=torch.int64, device=scores.device)
    s = scores.contiguous()
    ln = lengths.to(torch.int32).contiguous()
    if R * N:
        check(lib().lsa_pack_keys(ptr(s), R, N, N, ptr(ln), ptr(keys), N, stream_of(s)), "pack_keys")
    return keys


def bucket_scores(queries: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    """scores [R, N] fp32 = canonical fp32 dot of each query with each centroid."""
    require_cuda(queries, centroids, what="bucket_scores")
    q = queries.contiguous()
    c = centroids.contiguous()
    R, d = q.shape
    N = c.shape[0]
    out = torch.empty(R, N, dtype=torch.float32, device=q.device)
    if R and N:
        check(lib().lsa_bucket_scores(ptr(q), _lib.DTYPE_CODE[q.dtype], R, d, ptr(c), _lib.DTYPE_CODE[c.dtype], N, d,
                                      ptr(out), N, stream_of(q)), "bucket_scores")
    return out


def _production_scores(index_queries, positions, buckets, config, score_dtype):
    """The scoring every select arm shares (ref ``pipeline.py:217-232``)."""
    if positions.shape[0] != index_queries.shape[0]:
        raise ValueError(
            f"a position a query: {index_queries.shape[0]} queries, {positions.shape[0]} positions"
        )
    counts = visible_counts(positions, buckets, config)
    if score_dtype == "fp32":
        scores = bucket_scores(index_queries.float(), buckets.centroids_f32)
    else:
        scores = bucket_scores(index_queries.to(torch.bfloat16), buckets.centroids)
    return scores, counts


def _mask_for(scores: torch.Tensor, config: PortConfig, listed: torch.Tensor) -> torch.Tensor | None:
    """Counts ``best_first_keys`` masks by (ref ``pipeline.py:235-245``): None on the whole path.

    This build's listing always writes EMPTY past each row's length, so the mask is a
    no-op either way; the rule is kept so the reference chain's op sequence is the same."""
    return None if scores.shape[1] <= WHOLE * config.top_p else listed


def expand_in_order(picked: torch.Tensor, members: torch.Tensor, positions: torch.Tensor, window_size: int,
                    sink_size: int, top_k: int):
    """Rank-order expansion from picked bucket ids (upstream ``expand_in_order``)."""
    require_cuda(picked, members, positions, what="expand_in_order")
    picked = picked.to(torch.int32).contiguous()
    R, P = picked.shape
    width = top_k + window_size + sink_size
    lists = torch.empty(R, width, dtype=torch.int32, device=picked.device)
    lengths = torch.empty(R, dtype=torch.int32, device=picked.device)
    if R:
        mem = members.to(torch.int32).contiguous()
        pos = positions.to(torch.int32).contiguous()
        check(lib().lsa_expand_in_order(ptr(picked), R, P, P, ptr(mem), mem.shape[0], mem.shape[1], ptr(pos),
                                        window_size, sink_size, top_k, ptr(lists), ptr(lengths), stream_of(picked)),
              "expand_in_order")
    return lists, lengths


def flat_select_reference(index_queries, positions, buckets, config, top_k=None, score_dtype="bf16"):
    """The unfused select chain (ref ``pipeline.py:248-271``): scores, listing, best-first
    top-k, unpack, expansion - five kernels, the A/B oracle for the fused arms."""
    require_cuda(index_queries, positions, what="flat_select")
    top_k = config.top_k if top_k is None else top_k
    scores, counts = _production_scores(index_queries, positions, buckets, config, score_dtype)
    keys = pack_keys(scores, counts)
    picked = unpack_ids(best_first_keys(keys, config.top_p, counts=_mask_for(scores, config, counts)))
    return expand_in_order(picked, buckets.members, positions, config.window_size, config.sink_size, top_k)


def _scoring_operands(index_queries, centroids_bf16, centroids_f32, score_dtype):
    """(queries, query dtype code, centroids) of a fused select: "fp32" scores fp32 queries on
    the fp32 centroids; "bf16" scores bf16(queries) on the bf16 centroids - an fp32 query
    goes in as is with code F32_AS_BF16 (the kernel rounds it on load: no cast launch)."""
    if score_dtype == "fp32":
        return index_queries.float().contiguous(), _lib.F32, centroids_f32
    if index_queries.dtype == torch.float32:
        return index_queries.contiguous(), _lib.F32_AS_BF16, centroids_bf16
    q = index_queries.to(torch.bfloat16).contiguous()
    return q, _lib.BF16, centroids_bf16


def _select_fused(index_queries, positions, buckets, config, top_k, score_dtype):
    """One launch from index queries to read lists (``lsa_select_fused``)."""
    if positions.shape[0] != index_queries.shape[0]:
        raise ValueError(
            f"a position a query: {index_queries.shape[0]} queries, {positions.shape[0]} positions"
        )
    c = buckets.centroids_f32 if score_dtype == "fp32" else buckets.centroids
    # lsa_select_fused through the torch op (current stream; fp32 queries on bf16 centroids are
    # rounded in-kernel - query code 3)
    lists, lengths = _lib.torch_ops().select_fused(index_queries, positions, c, buckets.members,
                                                   config.cluster_block_size, config.block_bucket_count, config.top_p,
                                                   config.window_size, config.sink_size, top_k)
    _lib.after_call(index_queries.device, "flat_select(fused)")
    return lists, lengths


def flat_select(index_queries, positions, buckets, config, top_k=None, score_dtype="bf16"):
    """Select each query's keys - the production composition, implementation-switched.

    ``LSA_SELECT_IMPL`` picks the implementation (default ``reference``), read per call:
    ``reference`` is the unfused kernel chain (``flat_select_reference``); ``fused`` is
    one launch from index queries to read lists; ``fused_unpack`` keeps the listing and
    top-k kernels and folds the unpack into the expansion walk. All arms reproduce the
    reference output byte-exactly; unknown values fail loudly.
    """
    impl = os.environ.get("LSA_SELECT_IMPL", "reference")
    if impl not in SELECT_IMPLS:
        raise ValueError(f"LSA_SELECT_IMPL must be reference|fused|fused_unpack, got {impl!r}")
    require_cuda(index_queries, positions, what="flat_select")
    if impl == "reference":
        return flat_select_reference(index_queries, positions, buckets, config, top_k, score_dtype)
    top_k = config.top_k if top_k is None else top_k
    if impl == "fused":
        return _select_fused(index_queries, positions, buckets, config, top_k, score_dtype)
    from . import select_fused

    scores, counts = _production_scores(index_queries, positions, buckets, config, score_dtype)
    keys = pack_keys(scores, counts)
    ordered = best_first_keys(keys, config.top_p, counts=_mask_for(scores, config, counts))
    return select_fused.expand_in_order_from_keys(ordered, buckets.members, positions.int(), config.window_size,
                                                  config.sink_size, top_k)


def select_from_queries(q, positions, buckets, config, top_k=None, score_dtype="bf16"):
    """``make_index_space`` + ``flat_select`` (fused) from raw queries, for decode steps.

    q [R, Hq, D] (one row per decoding sequence, Hq a multiple of the index's KV heads):
    the index query of each row (the group mean of every KV head's query heads) is built
    inside the decode select kernel, so one launch goes from the model's query to the read
    lists - the same lists as ``flat_select(regroup_rows(q, ...)[0], ...)`` byte for byte.
    Rows the one-cluster decode select does not take are regrouped first (on the GPU) and go
    the fused two-step way. Reference: ``src/lsa_rocm_lab/port/gates.py:50-59`` (the index
    space) and ``src/lsa_rocm_lab/port/pipeline.py:274-316`` (the fused select).
    """
    require_cuda(q, positions, what="select_from_queries")
    if q.dim() != 3:
        raise ValueError(f"raw queries are [R, Hq, D], got shape {tuple(q.shape)}")
    if positions.shape[0] != q.shape[0]:
        raise ValueError(f"a position a query: {q.shape[0]} queries, {positions.shape[0]} positions")
    top_k = config.top_k if top_k is None else top_k
    c = buckets.centroids_f32 if score_dtype == "fp32" else buckets.centroids
    lists, lengths = _lib.torch_ops().select_fused(q, positions, c, buckets.members, config.cluster_block_size,
                                                   config.block_bucket_count, config.top_p, config.window_size,
                                                   config.sink_size, top_k)
    _lib.after_call(q.device, "select_from_queries")
    return lists, lengths


def tree_select(index_queries, positions, buckets, hierarchy, config, top_k=None):
    """Select each query's keys by a beam down the levels (ref ``pipeline.py:319-337``)."""
    from ._tree import tree_select_batched

    return tree_select_batched(index_queries, positions, buckets, hierarchy, config, top_k)


def decode_fused(q, k, v, index_queries, positions, buckets, config, scale=None, return_lists=False):
    """flat_select + lsa_read for the decode rows of one sequence in ONE launch.

    q [1, R, Hq, 128] (R <= 4 rows at ``positions``), k/v [1, Tk, Hkv, 128] bf16/fp16,
    index_queries [R, d]. Same lists as ``flat_select`` (bf16 scoring), same read as
    ``lsa_read``; ``return_lists`` also returns (lists, lengths)."""
    require_cuda(q, k, v, index_queries, positions, what="decode_fused")
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("decode_fused reads bf16 or fp16 q/k/v")
    B, R, Hq, D = q.shape
    if B != 1 or k.shape[0] != 1:
        raise ValueError("decode_fused decodes rows of one sequence (batch 1)")
    Tk, Hkv = k.shape[1], k.shape[2]
    iq = index_queries.to(torch.bfloat16).contiguous()
    c = buckets.centroids.contiguous()
    N, d = c.shape
    width = config.top_k + config.window_size + config.sink_size
    dev = q.device
    out = torch.empty_like(q)
    lists = torch.empty(R, width, dtype=torch.int32, device=dev) if return_lists else None
    lengths = torch.empty(R, dtype=torch.int32, device=dev) if return_lists else None
    L = lib()
    sb, nc = ctypes.c_int64(), ctypes.c_int64()
    check(L.lsa_decode_fused_plan(R, Hq, Hkv, N, buckets.members.shape[1], width, ctypes.byref(sb),
                                  ctypes.byref(nc)), "decode_fused")
    sc = _lib.scratch(sb.value, dev)
    ct = _lib.counters(nc.value, dev)
    pos = positions.to(torch.int32).contiguous()
    scale = D ** -0.5 if scale is None else float(scale)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    check(L.lsa_decode_fused(ptr(iq), R, d, ptr(c), N, d, ptr(buckets.members), buckets.members.shape[1], ptr(pos),
                             config.cluster_block_size, config.block_bucket_count, config.top_p, config.window_size,
                             config.sink_size, config.top_k, ptr(qc), ptr(kc), ptr(vc), _lib.DTYPE_CODE[q.dtype], Tk,
                             Hq, Hkv, D, scale, ptr(out), ptr(lists), ptr(lengths), ptr(sc), sc.numel(), ptr(ct),
                             ct.numel(), stream_of(q)), "decode_fused")
    _lib.after_call(dev, "decode_fused")
    return (out, lists, lengths) if return_lists else out


# ------------------------------------------------------------------ read


def dense_read(q, k, v, scale):
    """The dense causal baseline - torch SDPA (ref ``pipeline.py:340-370``).

    Square -> fused causal; one query row -> unmasked over the whole cache; a chunk ->
    explicit bottom-right causal mask; ``q_len > kv_len`` -> ValueError."""
    heads_q, heads_kv = q.shape[2], k.shape[2]
    q_len, kv_len = q.shape[1], k.shape[1]
    if q_len > kv_len:
        raise ValueError(f"query rows {q_len} exceed the cache {kv_len}: no causal read exists")
    queries, keys, values = q.permute(0, 2, 1, 3), k.permute(0, 2, 1, 3), v.permute(0, 2, 1, 3)
    gqa = heads_q != heads_kv
    if q_len == kv_len:
        out = F.scaled_dot_product_attention(queries, keys, values, is_causal=True, scale=scale, enable_gqa=gqa)
    elif q_len == 1:
        out = F.scaled_dot_product_attention(queries, keys, values, scale=scale, enable_gqa=gqa)
    else:
        causal = torch.arange(kv_len, device=q.device)[None, :] <= torch.arange(
            kv_len - q_len, kv_len, device=q.device
        )[:, None]
        out = F.scaled_dot_product_attention(queries, keys, values, attn_mask=causal, scale=scale, enable_gqa=gqa)
    return out.permute(0, 2, 1, 3)


def lsa_read(q, k, v, read_lists, lengths, scale):
    """The sparse read over selected lists (ref ``pipeline.py:373-375``)."""
    return sparse_read(q, k, v, read_lists, lengths, scale)
