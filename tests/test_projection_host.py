"""D-LSA projection maps on the host: the checker's projected index space (an identity map
reproduces the plain regroup; the projected keys are unit rows), the training-free PCA map
(orthonormal rows, ordered by captured energy; full width keeps every dot product), and the
per-layer map container's save / load round trip."""

import numpy as np
import torch


def test_identity_map_reproduces_regroup(oracle):
    rng = np.random.default_rng(3)
    q = rng.standard_normal((9, 12, 64)).astype(np.float32)
    k = rng.standard_normal((9, 4, 64)).astype(np.float32)
    iq, ik = oracle.regroup(q, k)
    pq, pk = oracle.regroup_project(q, k, np.eye(256, dtype=np.float32))
    assert np.array_equal(iq, pq) and np.array_equal(ik, pk)


def test_projected_keys_are_unit_rows(oracle):
    rng = np.random.default_rng(4)
    q = rng.standard_normal((7, 8, 64)).astype(np.float32)
    k = rng.standard_normal((7, 2, 64)).astype(np.float32)
    W = rng.standard_normal((32, 128)).astype(np.float32)
    iq, ik = oracle.regroup_project(q, k, W)
    assert iq.shape == (7, 32) and ik.shape == (7, 32)
    assert np.allclose(np.linalg.norm(ik, axis=1), 1.0, atol=1e-5)
    want_q = q.reshape(7, 2, 4, 64).mean(2).reshape(7, 128) @ W.T
    assert np.allclose(iq, want_q, atol=1e-4)


def test_pca_map_is_orthonormal_and_ordered():
    from lsa_b200.projection import pca_map

    g = torch.Generator().manual_seed(5)
    basis = torch.linalg.qr(torch.randn(64, 64, generator=g))[0]
    keys = torch.randn(2000, 64, generator=g) * torch.linspace(3.0, 0.1, 64) @ basis.T
    W = pca_map(keys, 16)
    assert W.shape == (16, 64) and W.dtype == torch.float32
    assert torch.allclose(W @ W.T, torch.eye(16), atol=1e-4)
    energy = ((keys @ W.T) ** 2).sum(0)
    assert bool((energy[:-1] >= energy[1:] - 1e-3).all())  # largest directions first
    full = pca_map(keys, 64)
    assert torch.allclose((keys @ full.T) @ full, keys, atol=1e-3)  # full width keeps every dot


def test_maps_save_and_load(tmp_path):
    from lsa_b200.projection import ProjectionMaps

    maps = ProjectionMaps([torch.randn(32, 128), torch.randn(64, 128)])
    maps.save(tmp_path / "maps.npz")
    back = ProjectionMaps.load(tmp_path / "maps.npz")
    assert len(back) == 2 and all(torch.equal(a, b) for a, b in zip(maps.maps, back.maps))
