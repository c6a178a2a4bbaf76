"""Fused selection operators - drop-in for ``lsa_rocm_lab.port.select_fused``.

Reference: AIwork4me/latent-sparse-attention-rocm, ``src/lsa_rocm_lab/port/select_fused.py``.

``select_topk_scores`` (ref ``:83-137``) packs each score row in-register and keeps the
``min(top_p, N)`` greatest packed keys sorted descending, in one kernel, for ANY width:
the exact best-k of the live columns, which is what the reference's whole-path kernel and
its wide-row fallback both compute. There is no fallback here (the kernel handles every
width), so no UserWarning is raised. Output [R, K2], K2 = next_pow2(min(top_p, N)), EMPTY
past the first min(top_p, N) keys.

``expand_in_order_from_keys`` (ref ``:217-280``) walks ordered packed keys with the unpack
fused into the walk. Like the reference it refuses a non-power-of-two ``bucket_cap``.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_of

WHOLE_FACTOR = 4


def _next_pow2(x: int) -> int:
    p = 1
    while p < x:
        p <<= 1
    return p


def select_topk_scores(scores: torch.Tensor, lengths: torch.Tensor, top_p: int) -> torch.Tensor:
    """Scores [R, N] fp32 + live columns [R] -> ordered packed keys [R, K2] int64."""
    if scores.device.type != "cuda":
        raise ValueError(f"select_topk_scores is a B200 kernel, got device {scores.device}")
    if scores.dtype != torch.float32:
        raise ValueError(f"scores must be the GEMM's fp32 output, got {scores.dtype}")
    rows, columns = scores.shape
    keep = min(top_p, columns)
    k2 = _next_pow2(keep) if keep else 1
    out = torch.empty(rows, k2, device=scores.device, dtype=torch.int64)
    if rows:
        s = scores.contiguous()
        ln = lengths.to(torch.int32).contiguous()
        check(lib().lsa_select_topk_scores(ptr(s), rows, columns, columns, ptr(ln), top_p, ptr(out), k2,
                                           stream_of(s)), "select_topk_scores")
    return out


def expand_in_order_from_keys(ordered_keys: torch.Tensor, bucket_members: torch.Tensor, positions: torch.Tensor,
                              window_size: int, sink_size: int, top_k: int):
    """Read lists [R, top_k + window + sink] int32 (-1 padded) and lengths [R] int32."""
    if ordered_keys.device.type != "cuda":
        raise ValueError(f"expand_in_order_from_keys is a B200 kernel, got device {ordered_keys.device}")
    bucket_cap = bucket_members.size(1)
    if bucket_cap & (bucket_cap - 1):
        raise ValueError(
            f"bucket_cap {bucket_cap} is not a power of two - the reference's walk tile needs a "
            "power-of-two bucket_cap (production: 16), and this drop-in keeps that contract"
        )
    keys = ordered_keys.contiguous()
    R, P = keys.shape
    width = top_k + window_size + sink_size
    out = torch.empty(R, width, device=keys.device, dtype=torch.int32)
    lengths = torch.empty(R, device=keys.device, dtype=torch.int32)
    if R:
        mem = bucket_members.to(torch.int32).contiguous()
        pos = positions.to(torch.int32).contiguous()
        check(lib().lsa_expand_from_keys(ptr(keys), R, P, P, ptr(mem), mem.shape[0], bucket_cap, ptr(pos),
                                         window_size, sink_size, top_k, ptr(out), ptr(lengths), stream_of(keys)),
              "expand_in_order_from_keys")
    return out, lengths


__all__ = ["select_topk_scores", "expand_in_order_from_keys", "WHOLE_FACTOR", "_lib"]
