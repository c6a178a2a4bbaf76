"""Shared test setup: paths, the ``gpu`` marker, seeded inputs, oracle <-> torch helpers.

``-m "not gpu"`` runs on a CPU-only machine: the oracle against the reference's golden
vectors and known answers, host logic, the C-ABI library's exports, and the multi-rank
logic on gloo. ``-m gpu`` runs the CUDA kernels through the C-ABI against the oracle.
"""

import os
import pathlib
import sys

import numpy as np
import pytest
import torch

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "latent-sparse-attention-rocm_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

SEED = 20261105
# checked mode: every entry point synchronises after its launch and raises if a bounded
# wait expired or a counter was left off zero (lsa_b200.check_status)
os.environ.setdefault("LSA_CHECK_STATUS", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a); runs the kernels via the C-ABI")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible: GPU parity tests run on the B200 box")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def lsa():
    import lsa_b200

    return lsa_b200


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def oracle_buckets_to_gpu(ob, device="cuda"):
    """Oracle buckets -> the package's Buckets on the GPU (identical bits)."""
    from lsa_b200.pipeline import Buckets

    return Buckets(
        torch.from_numpy(ob.centroids_bf16).to(device).to(torch.bfloat16),
        torch.from_numpy(ob.members).to(device),
        torch.from_numpy(ob.sizes).to(device),
        centroids_f32=torch.from_numpy(ob.centroids_f32).to(device),
        key_sums=torch.from_numpy(ob.key_sums).to(device),
    )


def drift_keys(rng: np.random.Generator, T: int, Hkv: int, D: int, amp: float = 0.5) -> np.ndarray:
    """Keys with a per-position low-rank drift: k[t,h] = n[t,h] + amp * sum_r c_r(t) U_r, with a
    rank-8 Gaussian basis U ~ N(0,1)/sqrt(8) per KV head and c_r(t) = sin(2 pi t / P_r + phi_r),
    P_r log-spaced over [256, T], phi_r ~ U(0, 2 pi)."""
    rank = 8
    U = rng.standard_normal((Hkv, rank, D)).astype(np.float32) / np.sqrt(rank)
    periods = np.geomspace(256, max(T, 257), rank)
    phase = rng.uniform(0, 2 * np.pi, rank)
    t = np.arange(T)[:, None]
    c = np.sin(2 * np.pi * t / periods[None, :] + phase[None, :]).astype(np.float32)  # [T, rank]
    n = rng.standard_normal((T, Hkv, D)).astype(np.float32)
    return n + amp * np.einsum("tr,hrd->thd", c, U).astype(np.float32)
