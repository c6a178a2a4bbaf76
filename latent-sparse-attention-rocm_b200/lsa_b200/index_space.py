"""The GQA -> index-space collapse (the reference's ``make_index_space``).

Reference: AIwork4me/latent-sparse-attention-rocm, ``src/lsa_rocm_lab/port/gates.py:50-59``,
which calls upstream ``lsa.core.index_space.regroup`` (absent from the reference).
Definition used here (one ``lsa_regroup`` kernel, fp32 out): the index query of position t
is, per KV head, the mean of its query group's vectors, concatenated over KV heads; the
index key is the unit row of the KV heads' keys concatenated. index_dim = Hkv * Dh.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_of


def regroup_rows(q: torch.Tensor, k: torch.Tensor):
    """q [T, Hq, D], k [T, Hkv, D] of one sequence -> (index queries, index keys) [T, Hkv * D] fp32."""
    require_cuda(q, k, what="make_index_space")
    if q.dtype != k.dtype or q.dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"q and k must share one of fp32/fp16/bf16, got {q.dtype}/{k.dtype}")
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must group evenly onto KV heads")
    q, k = q.contiguous(), k.contiguous()
    iq = torch.empty(T, Hkv * D, dtype=torch.float32, device=q.device)
    ik = torch.empty(T, Hkv * D, dtype=torch.float32, device=q.device)
    if T:
        check(lib().lsa_regroup(ptr(q), ptr(k), _lib.DTYPE_CODE[q.dtype], T, Hq, Hkv, D, ptr(iq), ptr(ik),
                                stream_of(q)), "make_index_space")
    return iq, ik


def make_index_space(q: torch.Tensor, k: torch.Tensor):
    """q [B, T, Hq, D], k [B, T, Hkv, D] -> (index_queries [T, d], index_keys [T, d]) of batch row 0."""
    return regroup_rows(q[0], k[0])


def index_keys(k: torch.Tensor) -> torch.Tensor:
    """k [T, Hkv, D] of one sequence -> unit-row index keys [T, Hkv * D] fp32."""
    return regroup_rows(k, k)[1]


def index_queries(q: torch.Tensor, Hkv: int) -> torch.Tensor:
    """q [T, Hq, D] -> index queries [T, Hkv * D] fp32 (group means, unnormalised)."""
    return regroup_rows(q, q[:, :Hkv])[0]
