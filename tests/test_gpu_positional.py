"""cfg 2's positional block-sparse decode arm: the static picks (first 4 + last 4 + strided
visible buckets) and the expansion over positional buckets (src/lsa_rocm_lab/port/
pipeline.py:378-403) bit-exact against the CPU checker, and the read within tolerance."""

import numpy as np
import pytest
import torch

from conftest import drift_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"
CFG2 = dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
            window_size=64, sink_size=4)


def _np(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def test_positional_picks_match_oracle(oracle, lsa):
    cfg = lsa.PortConfig(**CFG2)
    ocfg = oracle.Config(**CFG2)
    pos = np.array([0, 511, 512, 2047, 4096, 4607, 9000, 20000, 32767], dtype=np.int32)
    rows = 512
    from lsa_b200.pipeline import Buckets

    fake = Buckets(torch.zeros(rows, 8, dtype=torch.bfloat16, device=DEV),
                   torch.zeros(rows, 128, dtype=torch.int32, device=DEV),
                   torch.zeros(rows, dtype=torch.int32, device=DEV))
    got = lsa.pipeline.positional_picks(torch.from_numpy(pos).to(DEV), fake, cfg)
    want = oracle.positional_picks(pos, rows, ocfg)
    assert np.array_equal(_np(got), want)
    full = want[-1]
    assert (full[:4] == [0, 1, 2, 3]).all() and (full[-4:] == [500, 501, 502, 503]).all()
    assert (np.diff(full) > 0).all() and full.size == 32


def test_positional_arm_32k_vs_oracle(oracle, lsa):
    from lsa_b200.index_space import index_keys, index_queries

    rng = np.random.default_rng(20261105 + 2)
    T, Hq, Hkv = 32768, 32, 8
    k = torch.from_numpy(drift_keys(rng, T, Hkv, 128)).to(DEV).to(torch.bfloat16)[None]
    v = torch.from_numpy(rng.standard_normal((1, T, Hkv, 128)).astype(np.float32)).to(DEV).to(torch.bfloat16)
    q = torch.from_numpy(rng.standard_normal((1, 1, Hq, 128)).astype(np.float32)).to(DEV).to(torch.bfloat16)
    cfg = lsa.PortConfig(**CFG2)
    ik = index_keys(k[0])
    pb = lsa.position_buckets(ik, cfg)
    ob = oracle.position_buckets(_np(ik), oracle.Config(**CFG2))
    pos = torch.tensor([T - 1], dtype=torch.int32, device=DEV)
    gl, gn = lsa.pipeline.positional_select(pos, pb, cfg)
    wl, wn = oracle.positional_select([T - 1], ob, oracle.Config(**CFG2))
    assert np.array_equal(_np(gl), wl) and np.array_equal(_np(gn), wn)
    assert int(gn[0]) == 32 * 64 - 4 + 64 + 4  # bucket 0 holds the sinks, which the walk lists once, last
    out = lsa.lsa_read(q, k, v, gl[None], gn[None], 128 ** -0.5)
    want = oracle.sparse_read(_np(q), _np(k), _np(v), wl[None], wn[None], 128 ** -0.5)
    assert float(np.abs(_np(out) - want).max()) <= 2e-2
    del index_queries
