"""The v1 sparse-read entry - drop-in for ``lsa_rocm_lab.port.read_kernel``.

Reference: AIwork4me/latent-sparse-attention-rocm, ``src/lsa_rocm_lab/port/read_kernel.py:80-120``.
Same signature and contract, served by the one B200 read kernel. One deliberate
difference: a row with no listed key reads as zeros here, where the reference's v1
kernel divides 0 by 0 (NaN) - the hazard its tiled kernel fixed (``read_kernel_tiled.py:20-22``).
"""

from __future__ import annotations

from .read_kernel_tiled import _read


def sparse_read(q, k, v, read_ids, lengths, scale=None, block: int = 64):
    """Attention over each query row's read list (``block`` is the reference's Triton tunable)."""
    del block
    return _read(q, k, v, read_ids, lengths, scale)
