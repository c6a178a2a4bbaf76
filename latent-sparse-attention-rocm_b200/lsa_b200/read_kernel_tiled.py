"""The sparse read - drop-in for ``lsa_rocm_lab.port.read_kernel_tiled``.

Reference: AIwork4me/latent-sparse-attention-rocm, ``src/lsa_rocm_lab/port/read_kernel_tiled.py``
(numerics ``:41-89``, wrapper ``:92-136``, dispatch ``:144-156``).

One B200 entry point (``lsa_sparse_read``, registered as the torch op ``lsa::sparse_read``)
serves every launch shape, picking its kernel by the shape (decode rows: one cluster per row
and KV head; batches: the persistent read; the rest: split-K), so ``tile_rows``, ``chunk`` and
``num_warps`` - the reference's Triton tunables - are accepted and have no effect. Same contract: q [B, Tq, Hq, Dh],
k/v [B, Tk, Hkv, Dh], read_ids [B, Tq, width] int32 (-1 padded), lengths [B, Tq];
lengths are clamped to the width; rows with no listed key read as zeros; duplicates
count per occurrence; the output has q's shape, dtype and device. Ids outside [0, Tk)
are skipped (never dereferenced).
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_of

DECODE_ROW_LIMIT = 32


def _read(q, k, v, read_ids, lengths, scale, splits: int = 0):
    assert q.is_cuda and k.is_cuda and v.is_cuda, "the sparse read is a GPU kernel"
    B, Tq, Hq, D = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    assert Hq % Hkv == 0, "query heads must group evenly onto KV heads"
    if q.dtype not in _lib.DTYPE_CODE or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"q, k, v must share one of fp32/fp16/bf16, got {q.dtype}/{k.dtype}/{v.dtype}")
    if splits == 0:  # lsa_sparse_read through the torch op, on the current stream
        out = _lib.torch_ops().sparse_read(q, k, v, read_ids, lengths, D ** -0.5 if scale is None else float(scale))
        _lib.after_call(q.device, "sparse_read")
        return out
    # a forced split count (tests of the split plans): the C ABI directly
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    width = read_ids.shape[-1]
    ids = read_ids.reshape(-1, width).to(torch.int32).contiguous()
    lens = lengths.reshape(-1).to(torch.int32).contiguous()
    out = torch.empty_like(q)
    if B * Tq == 0:
        return out
    L = lib()
    import ctypes

    s_out, sb, nc = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    check(L.lsa_sparse_read_plan(B, Tq, Hq, Hkv, D, width, splits, ctypes.byref(s_out), ctypes.byref(sb),
                                 ctypes.byref(nc)), "sparse_read")
    sc = _lib.scratch(sb.value, q.device)
    ct = _lib.counters(nc.value, q.device)
    scale = D ** -0.5 if scale is None else float(scale)
    check(L.lsa_sparse_read(ptr(q), ptr(k), ptr(v), _lib.DTYPE_CODE[q.dtype], ptr(ids), ptr(lens), B, Tq, Tk, Hq, Hkv,
                            D, width, scale, ptr(out), ptr(sc), sc.numel(), ptr(ct), ct.numel(), splits,
                            stream_of(q)), "sparse_read")
    _lib.after_call(q.device, "sparse_read")
    return out


def sparse_read_tiled(q, k, v, read_ids, lengths, scale=None, tile_rows: int = 4, chunk: int = 64,
                      num_warps: int = 4):
    """Attention over each query row's read list (ref ``read_kernel_tiled.py:92-136``)."""
    del tile_rows, chunk, num_warps  # Triton tunables of the reference; one B200 kernel here
    return _read(q, k, v, read_ids, lengths, scale)


def sparse_read_auto(q, k, v, read_ids, lengths, scale=None):
    """The production sparse read entry (ref ``read_kernel_tiled.py:147-156``)."""
    return _read(q, k, v, read_ids, lengths, scale)
