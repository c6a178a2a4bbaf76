"""D-LSA projection maps on the GPU: lsa_regroup_project bit-exact against the checker
(dtypes, group sizes, position counts off the 8-position CTA tile, narrow and full output
widths), and the whole selection on a projected index - a training-free PCA map, the Ward
build and the one-launch select in the d_out-wide space - bit-exact against the checker."""

import numpy as np
import pytest
import torch


pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bits(a, b):
    return a.shape == b.shape and (a.view(np.int32) == b.view(np.int32)).all()


@pytest.mark.parametrize("T,Hq,Hkv,D,d_out,dtype", [(1, 32, 8, 128, 256, torch.bfloat16),
                                                    (13, 8, 2, 64, 64, torch.float32),
                                                    (70, 12, 4, 64, 256, torch.float16),
                                                    (9, 16, 16, 128, 2048, torch.bfloat16),
                                                    (300, 32, 8, 128, 1024, torch.bfloat16)])
def test_regroup_project_exact(oracle, lsa, T, Hq, Hkv, D, d_out, dtype):
    from lsa_b200.index_space import regroup_project_rows

    rng = np.random.default_rng(T + d_out)
    q = torch.from_numpy(rng.standard_normal((T, Hq, D)).astype(np.float32)).to(dtype)
    k = torch.from_numpy(rng.standard_normal((T, Hkv, D)).astype(np.float32)).to(dtype)
    W = rng.standard_normal((d_out, Hkv * D)).astype(np.float32) / np.sqrt(Hkv * D)
    iq, ik = regroup_project_rows(q.to(DEV), k.to(DEV), torch.from_numpy(W).to(DEV))
    wq, wk = oracle.regroup_project(q.float().numpy(), k.float().numpy(), W)
    assert _bits(iq.cpu().numpy(), wq) and _bits(ik.cpu().numpy(), wk)


def test_selection_on_a_pca_projected_index(oracle, lsa, monkeypatch):
    from lsa_b200.projection import pca_map

    rng = np.random.default_rng(11)
    T, Hq, Hkv, D, d_out = 4096, 32, 8, 128, 256
    q = torch.from_numpy(rng.standard_normal((1, T, Hq, D)).astype(np.float32)).bfloat16().to(DEV)
    k = torch.from_numpy(rng.standard_normal((1, T, Hkv, D)).astype(np.float32)).bfloat16().to(DEV)
    _, plain_keys = lsa.make_index_space(q, k)
    W = pca_map(plain_keys, d_out)
    iq, ik = lsa.make_index_space(q, k, projection=W)
    cfg = dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
               window_size=64, sink_size=4)
    buckets = lsa.build_buckets_gpu(ik, lsa.PortConfig(**cfg))
    ocfg = oracle.Config(**cfg)
    wq, wk = oracle.regroup_project(q[0].float().cpu().numpy(), k[0].float().cpu().numpy(), W.cpu().numpy())
    assert _bits(ik.cpu().numpy(), wk) and _bits(iq.cpu().numpy(), wq)
    ob = oracle.build_buckets(wk, ocfg)
    assert np.array_equal(buckets.members.cpu().numpy(), ob.members)
    rows = np.array([T - 1, 2600, 1023])
    monkeypatch.setenv("LSA_SELECT_IMPL", "fused")
    lists, lengths = lsa.flat_select(iq[rows], torch.from_numpy(rows).to(DEV), buckets, lsa.PortConfig(**cfg))
    want_l, want_n = oracle.flat_select(wq[rows], rows, ob, ocfg)
    assert np.array_equal(lists.cpu().numpy(), want_l) and np.array_equal(lengths.cpu().numpy(), want_n)
