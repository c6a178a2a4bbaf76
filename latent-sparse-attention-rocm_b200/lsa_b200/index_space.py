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
    return _lib.torch_ops().regroup(q, k)  # lsa_regroup on the current stream


def regroup_project_rows(q: torch.Tensor, k: torch.Tensor, projection: torch.Tensor):
    """regroup_rows through a D-LSA projection map ``projection`` [d_out, Hkv * D] (fp32, one row
    per output dim): index queries = group means projected, index keys = the concatenated key
    rows projected then normalised -> [T, d_out] fp32 each (``lsa_regroup_project``)."""
    require_cuda(q, k, projection, what="make_index_space")
    if q.dtype != k.dtype or q.dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"q and k must share one of fp32/fp16/bf16, got {q.dtype}/{k.dtype}")
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must group evenly onto KV heads")
    W = projection.float().contiguous()
    if W.dim() != 2 or W.shape[1] != Hkv * D:
        raise ValueError(f"projection must be [d_out, {Hkv * D}], got {tuple(W.shape)}")
    d_out = W.shape[0]
    q, k = q.contiguous(), k.contiguous()
    iq = torch.empty(T, d_out, dtype=torch.float32, device=q.device)
    ik = torch.empty(T, d_out, dtype=torch.float32, device=q.device)
    if T:
        check(lib().lsa_regroup_project(ptr(q), ptr(k), _lib.DTYPE_CODE[q.dtype], T, Hq, Hkv, D, ptr(W), d_out,
                                        ptr(iq), ptr(ik), stream_of(q)), "make_index_space(projection)")
    return iq, ik


def make_index_space(q: torch.Tensor, k: torch.Tensor, projection: torch.Tensor | None = None):
    """q [B, T, Hq, D], k [B, T, Hkv, D] -> (index_queries [T, d], index_keys [T, d]) of batch row 0;
    with a D-LSA ``projection`` map [d_out, Hkv * D] the index space is d_out wide."""
    if projection is not None:
        return regroup_project_rows(q[0], k[0], projection)
    return regroup_rows(q[0], k[0])


def index_keys(k: torch.Tensor, projection: torch.Tensor | None = None) -> torch.Tensor:
    """k [T, Hkv, D] of one sequence -> unit-row index keys [T, d] fp32 (d = Hkv * D, or the
    projection's d_out)."""
    if projection is not None:
        return regroup_project_rows(k, k, projection)[1]
    return regroup_rows(k, k)[1]


def index_queries(q: torch.Tensor, Hkv: int, projection: torch.Tensor | None = None) -> torch.Tensor:
    """q [T, Hq, D] -> index queries [T, d] fp32 (group means, unnormalised; projected with a map)."""
    if projection is not None:
        return regroup_project_rows(q, q[:, :Hkv], projection)[0]
    return regroup_rows(q, q[:, :Hkv])[0]
