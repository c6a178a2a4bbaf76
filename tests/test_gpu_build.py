"""GPU parity of the index builds and the tree beam vs the oracle (bit-exact).

Index space (regroup), bucket build (pools -> Ward merge -> members -> centroids), the
positional arm, the node hierarchy (children, key sums, centroids) and the tree select's
read lists. Mirrors the reference's gates A / A2 / C (src/lsa_rocm_lab/port/gates.py:114-260)
but with exact equality: the kernels follow the oracle's operation sequence.
"""

import numpy as np
import pytest
import torch

from conftest import drift_keys, oracle_buckets_to_gpu

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(t):
    return t.detach().cpu().numpy()


def _bits_equal(a, b):
    return a.shape == b.shape and (a.view(np.int32) == b.view(np.int32)).all()


@pytest.mark.parametrize("T,Hq,Hkv,D,dtype", [(300, 8, 2, 64, torch.float32), (512, 32, 8, 128, torch.bfloat16),
                                               (64, 12, 4, 64, torch.float16), (1, 32, 8, 128, torch.bfloat16),
                                               (3, 16, 16, 128, torch.bfloat16), (5, 64, 4, 64, torch.float16),
                                               (2000, 8, 2, 64, torch.float32)])
def test_regroup_exact(oracle, lsa, T, Hq, Hkv, D, dtype):
    """Bit-exact against the checker: one CTA per row up to 1024 rows (G <= 8, d <= 2048),
    one warp per row beyond (and for larger groups)."""
    rng = np.random.default_rng(T)
    q = torch.from_numpy(rng.standard_normal((1, T, Hq, D)).astype(np.float32)).to(dtype)
    k = torch.from_numpy(rng.standard_normal((1, T, Hkv, D)).astype(np.float32)).to(dtype)
    iq, ik = lsa.make_index_space(q.to(DEV), k.to(DEV))
    wq, wk = oracle.regroup(q[0].float().numpy(), k[0].float().numpy())
    assert _bits_equal(_np(iq), wq) and _bits_equal(_np(ik), wk)


CONFIGS = [
    dict(cluster_block_size=128, pool_size=4, bucket_size=8, bucket_cap=16),       # gate geometry
    dict(cluster_block_size=64, pool_size=4, bucket_size=64, bucket_cap=64),       # cfg 1
    dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128),     # cfg 2 / 3
    dict(cluster_block_size=1024, pool_size=8, bucket_size=128, bucket_cap=256),   # cfg 5
    dict(cluster_block_size=512, pool_size=4, bucket_size=8, bucket_cap=16),       # reference default
]


@pytest.mark.parametrize("cfg", CONFIGS)
def test_bucket_build_exact(oracle, lsa, cfg):
    rng = np.random.default_rng(cfg["cluster_block_size"] + cfg["bucket_size"])
    T, Hkv, D = 4 * cfg["cluster_block_size"] + 37, 2, 64
    q = rng.standard_normal((T, 8, D)).astype(np.float32)
    k = drift_keys(rng, T, Hkv, D)
    _, ik = oracle.regroup(q, k)
    ob = oracle.build_buckets(ik, oracle.Config(**cfg))
    gb = lsa.build_buckets_gpu(torch.from_numpy(ik).to(DEV), lsa.PortConfig(**cfg))
    assert (_np(gb.members) == ob.members).all()
    assert (_np(gb.sizes) == ob.sizes).all()
    assert _bits_equal(_np(gb.key_sums), ob.key_sums)
    assert _bits_equal(_np(gb.centroids_f32), ob.centroids_f32)
    assert _bits_equal(_np(gb.centroids.float()), ob.centroids_bf16)
    pb = lsa.position_buckets(torch.from_numpy(ik).to(DEV), lsa.PortConfig(**cfg))
    op = oracle.position_buckets(ik, oracle.Config(**cfg))
    assert (_np(pb.members) == op.members).all() and _bits_equal(_np(pb.centroids_f32), op.centroids_f32)


def test_infeasible_cap_is_refused(lsa):
    with pytest.raises(ValueError):
        lsa.build_buckets_gpu(torch.zeros(1024, 64, device=DEV),
                              lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=64))


TREE_CONFIGS = [
    (dict(cluster_block_size=512, pool_size=4, bucket_size=8, bucket_cap=16, top_p=1024, top_k=4096,
          window_size=512, sink_size=4, node_bucket_size=4, top_level=3, node_cluster_block_size=64,
          beam_width=64), 2048),  # tests/test_tree_batched_pages.py geometry
    (dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
          window_size=64, sink_size=4, node_bucket_size=4, top_level=3, node_cluster_block_size=64,
          beam_width=16), 32768),  # cfg 2 tree arm
    (dict(cluster_block_size=1024, pool_size=8, bucket_size=128, bucket_cap=256, top_p=64, top_k=8192,
          window_size=128, sink_size=4, node_bucket_size=16, top_level=2, node_cluster_block_size=64,
          beam_width=64), 1 << 17),  # cfg 5 geometry at 128k
]


@pytest.mark.parametrize("cfg,T", TREE_CONFIGS)
def test_hierarchy_and_tree_select_exact(oracle, lsa, cfg, T):
    rng = np.random.default_rng(T)
    Hkv, D = (2, 64) if T <= 4096 else (8, 128)
    k = drift_keys(rng, T, Hkv, D)
    q = rng.standard_normal((T, 4 * Hkv, D)).astype(np.float32)
    iq, ik = oracle.regroup(q, k)
    ocfg = oracle.Config(**cfg)
    ob = oracle.build_buckets(ik, ocfg)
    oh = oracle.build_hierarchy(ob, ocfg)
    gb = oracle_buckets_to_gpu(ob)
    pcfg = lsa.PortConfig(**cfg)
    gh = lsa.build_hierarchy_gpu(torch.from_numpy(ik).to(DEV), gb, pcfg)
    assert len(gh.levels) == len(oh.levels) > 0
    for gl, ol in zip(gh.levels, oh.levels):
        assert (_np(gl.children) == ol.children).all()
        assert _bits_equal(_np(gl.key_sums), ol.key_sums)
        assert _bits_equal(_np(gl.centroids), ol.centroids)
    rows = np.unique(np.concatenate([rng.integers(0, T, 48), [T - 1, T - 2, 0, 511, 512, 4095, 4096]]))
    rows = rows[rows < T]
    want_l, want_n = oracle.tree_select(iq[rows], rows, ob, oh, ocfg)
    got_l, got_n = lsa.tree_select(torch.from_numpy(iq[rows]).to(DEV), torch.from_numpy(rows).to(DEV), gb, gh, pcfg)
    assert (_np(got_n) == want_n).all()
    assert (_np(got_l) == want_l).all()
