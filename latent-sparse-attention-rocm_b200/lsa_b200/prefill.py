"""The prefill arm: per-tile selection and the tensor-core sparse prefill read.

The reference selects per query row (``src/lsa_rocm_lab/port/pipeline.py:248-316``) and
reads per row (``read_kernel_tiled.py:41-89``); at prefill it spends most of its time in
that read (``docs/OPTIMIZATION_v0.3.md:94-96``). Here a 64-query tile shares one list:

* ``tile_select`` scores each tile's fp32 sum of bf16 index queries against the bucket
  centroids, keeps the best ``top_p`` buckets of the blocks closed before the tile, and
  walks them into ``top_k`` key ids followed by the sinks below the tile's block
  (``lsa_tile_select``: the fused selection over tile rows).
* ``sparse_prefill`` reads, for each query row, its tile's list and then its own open
  block ``[block_start, row]`` causally (``lsa_sparse_prefill``: tcgen05 MMAs with S and O
  in tensor memory). Shapes the tensor-core kernel does not take (head groups other than
  4/8/16, head dim other than 128, fp32) go through the general sparse read over the
  equivalent per-row lists (``prefill_row_lists``) - also a CUDA kernel.

Row t's keys are exactly ``prefill_row_lists``'s row t, so both paths agree with the
general read (and with the CPU checker's ``sparse_read``) on the same lists.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_of

TILE = 64
_TC_GROUPS = (4, 8, 16)


def tile_queries(index_queries: torch.Tensor, tile: int = TILE) -> torch.Tensor:
    """[T, d] index queries -> [ceil(T / tile), d] fp32 sums of the bf16-rounded rows."""
    require_cuda(index_queries, what="tile_queries")
    iq = index_queries if index_queries.dtype in (torch.float32, torch.bfloat16) else index_queries.float()
    iq = iq.contiguous()
    T, d = iq.shape
    out = torch.empty((T + tile - 1) // tile, d, dtype=torch.float32, device=iq.device)
    check(lib().lsa_tile_queries(ptr(iq), _lib.DTYPE_CODE[iq.dtype], T, d, d, tile, ptr(out), stream_of(iq)),
          "tile_queries")
    return out


def tile_select(index_queries: torch.Tensor, buckets, config, tile: int = TILE, top_k: int | None = None):
    """Per-tile lists: (int32 [tiles, top_k + sink] -1 padded, int32 [tiles])."""
    require_cuda(index_queries, what="tile_select")
    top_k = config.top_k if top_k is None else int(top_k)
    if config.cluster_block_size % tile:
        raise ValueError(f"the tile ({tile}) must divide the cluster block ({config.cluster_block_size})")
    iq = index_queries if index_queries.dtype in (torch.float32, torch.bfloat16) else index_queries.float()
    iq = iq.contiguous()
    T, d = iq.shape
    c = buckets.centroids.contiguous()
    N = c.shape[0]
    dev = iq.device
    tiles = (T + tile - 1) // tile
    width = top_k + config.sink_size
    lists = torch.empty(tiles, width, dtype=torch.int32, device=dev)
    lengths = torch.empty(tiles, dtype=torch.int32, device=dev)
    if tiles == 0:
        return lists, lengths
    L = lib()
    sc = _lib.scratch(L.lsa_tile_select_scratch(T, tile, d, N), dev)
    ct = _lib.counters(tiles, dev)
    check(L.lsa_tile_select(ptr(iq), _lib.DTYPE_CODE[iq.dtype], T, d, tile, ptr(c), _lib.DTYPE_CODE[c.dtype], N, d,
                            config.cluster_block_size, config.block_bucket_count, ptr(buckets.members),
                            buckets.members.shape[1], config.top_p, config.sink_size, top_k, ptr(lists),
                            ptr(lengths), ptr(sc), sc.numel(), ptr(ct), ct.numel(), stream_of(iq)), "tile_select")
    _lib.after_call(dev, "tile_select")
    return lists, lengths


def prefill_row_lists(tile_lists: torch.Tensor, tile_lengths: torch.Tensor, T: int, block: int, tile: int = TILE):
    """Per-row read lists of the prefill arm on the GPU: the tile's list, then [block_start, row].

    Returns (int32 [T, tile_width + block] -1 padded, int32 [T])."""
    dev = tile_lists.device
    tw = tile_lists.shape[-1]
    rows = torch.arange(T, device=dev, dtype=torch.int64)
    tl = tile_lists[rows // tile].to(torch.int32)
    tlen = tile_lengths[rows // tile].to(torch.int64).clamp(0, tw)
    bs = rows // block * block
    local_n = rows - bs + 1
    width = tw + block
    col = torch.arange(width, device=dev, dtype=torch.int64)[None, :]
    from_tile = col < tlen[:, None]
    in_local = (col >= tlen[:, None]) & (col < (tlen + local_n)[:, None])
    tl_full = torch.nn.functional.pad(tl, (0, block), value=-1)
    local_ids = bs[:, None] + (col - tlen[:, None])
    lists = torch.where(from_tile, tl_full.to(torch.int64), torch.where(in_local, local_ids, torch.full_like(col, -1)))
    return lists.to(torch.int32), (tlen + local_n).to(torch.int32)


def sparse_prefill(q, k, v, tile_lists, tile_lengths, block: int, scale=None, tile: int = TILE):
    """Prefill attention of every row over its tile's list and its open block.

    q [B, T, Hq, D]; k, v [B, Tk, Hkv, D] with Tk >= T (row t's keys live at positions
    < t + 1); tile_lists [B, tiles, W] or [tiles, W] int32 (-1 padded), tile_lengths
    [B, tiles] or [tiles]. Output like q."""
    assert q.is_cuda and k.is_cuda and v.is_cuda, "the sparse prefill read is a GPU kernel"
    B, T, Hq, D = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    assert Hq % Hkv == 0, "query heads must group evenly onto KV heads"
    if Tk < T:
        raise ValueError(f"prefill needs the keys of every query row: Tk={Tk} < T={T}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"q, k, v must share a dtype, got {q.dtype}/{k.dtype}/{v.dtype}")
    scale = D ** -0.5 if scale is None else float(scale)
    tiles = (T + tile - 1) // tile
    tl = tile_lists.reshape(-1, tiles, tile_lists.shape[-1]).to(torch.int32)
    tn = tile_lengths.reshape(-1, tiles).to(torch.int32)
    if tl.shape[0] == 1 and B > 1:
        tl, tn = tl.expand(B, -1, -1), tn.expand(B, -1)
    G = Hq // Hkv
    tc_ok = (D == 128 and G in _TC_GROUPS and q.dtype in (torch.bfloat16, torch.float16)
             and tile % (256 // G) == 0 and block % tile == 0)
    if not tc_ok:
        from .read_kernel_tiled import _read

        lists, lengths = [], []
        for b in range(B):
            li, ln = prefill_row_lists(tl[b], tn[b], T, block, tile)
            lists.append(li)
            lengths.append(ln)
        return _read(q, k, v, torch.stack(lists), torch.stack(lengths), scale)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    tl, tn = tl.contiguous(), tn.contiguous()
    out = torch.empty_like(q)
    if B * T == 0:
        return out
    st = _lib.status_word(q.device)
    check(lib().lsa_sparse_prefill(ptr(q), ptr(k), ptr(v), _lib.DTYPE_CODE[q.dtype], ptr(tl), ptr(tn), tl.shape[-1],
                                   B, T, Tk, Hq, Hkv, D, tile, block, scale, ptr(out), ptr(st), stream_of(q)),
          "sparse_prefill")
    _lib.after_call(q.device, "sparse_prefill")
    return out


def status(device) -> int:
    """The device status word (0, or LSA_ERR_TIMEOUT after a bounded wait expired); syncs."""
    return int(_lib.status_word(torch.device(device)).item())


def lsa_prefill(q, k, v, index_queries, buckets, config, scale=None, tile: int = TILE, top_k=None):
    """Select per tile, then read: the whole prefill arm for batch row 0's index."""
    lists, lengths = tile_select(index_queries, buckets, config, tile, top_k)
    return sparse_prefill(q, k, v, lists, lengths, config.cluster_block_size, scale, tile)
