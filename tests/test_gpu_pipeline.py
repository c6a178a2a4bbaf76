"""End-to-end parity at the BASELINE configurations (select bit-exact, read within tolerance).

cfg 1: the CPU-oracle flat decode (B=1, pos 2047, Hq 8 / Hkv 2, Dh 64, fp32, 64-token
buckets, top-8 + the most recent bucket as the window) - selected indices bit-exact,
output within 1e-5. cfg 2: decode at 32k (Hq 32 / Hkv 8, Dh 128, bf16, drift keys,
64-token buckets, top-32 buckets) through every select arm - lists bit-exact, output
within 2e-2. Plus the reference's gate E (a decode step equals the prefill row) and a
size-independent property at full size: every listed id is causal, unique and visible.
"""

import numpy as np
import pytest
import torch

from conftest import drift_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"

CFG1 = dict(cluster_block_size=64, pool_size=4, bucket_size=64, bucket_cap=64, top_p=8, top_k=512,
            window_size=64, sink_size=0)
CFG2 = dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
            window_size=64, sink_size=4)


def _np(t):
    return t.detach().cpu().numpy()


def test_config1_cpu_oracle_flat_decode(oracle, lsa):
    rng = np.random.default_rng(20261105)
    T, Hq, Hkv, D = 2048, 8, 2, 64
    q = rng.standard_normal((1, T, Hq, D)).astype(np.float32)
    k = rng.standard_normal((1, T, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((1, T, Hkv, D)).astype(np.float32)
    iq, ik = oracle.regroup(q[0], k[0])
    ocfg = oracle.Config(**CFG1)
    ob = oracle.build_buckets(ik, ocfg)
    pos = np.array([T - 1])
    want_l, want_n = oracle.flat_select(iq[-1:], pos, ob, ocfg, score_dtype="fp32")
    want_o = oracle.sparse_read(q[:, -1:], k, v, want_l[None], want_n[None], D ** -0.5)
    assert want_n[0] == 8 * 64 + 64  # eight buckets of 64 keys and the window
    tq, tk, tv = (torch.from_numpy(x).to(DEV) for x in (q, k, v))
    giq, gik = lsa.make_index_space(tq, tk)
    pcfg = lsa.PortConfig(**CFG1)
    gb = lsa.build_buckets_gpu(gik, pcfg)
    for impl in ("reference", "fused", "fused_unpack"):
        import os

        os.environ["LSA_SELECT_IMPL"] = impl
        try:
            gl, gn = lsa.flat_select(giq[-1:], torch.tensor([T - 1], device=DEV), gb, pcfg, score_dtype="fp32")
        finally:
            os.environ.pop("LSA_SELECT_IMPL", None)
        assert (_np(gl) == want_l).all() and (_np(gn) == want_n).all(), impl
        out = lsa.lsa_read(tq[:, -1:], tk, tv, gl[None], gn[None], D ** -0.5)
        assert float(np.abs(_np(out) - want_o).max()) <= 1e-5


def _cfg2_inputs(seed=20261105 + 32768, T=32768):
    rng = np.random.default_rng(seed)
    Hq, Hkv, D = 32, 8, 128
    q = torch.from_numpy(rng.standard_normal((1, T, Hq, D)).astype(np.float32)).bfloat16()
    k = torch.from_numpy(drift_keys(rng, T, Hkv, D)[None]).bfloat16()
    v = torch.from_numpy(rng.standard_normal((1, T, Hkv, D)).astype(np.float32)).bfloat16()
    return q, k, v


@pytest.mark.parametrize("impl", ["reference", "fused", "fused_unpack"])
def test_config2_decode_32k_exact(oracle, lsa, monkeypatch, impl):
    q, k, v = _cfg2_inputs()
    T = q.shape[1]
    tq, tk, tv = q.to(DEV), k.to(DEV), v.to(DEV)
    giq, gik = lsa.make_index_space(tq, tk)
    pcfg = lsa.PortConfig(**CFG2)
    gb = lsa.build_buckets_gpu(gik, pcfg)
    # the oracle on the same bits: index space, buckets and selection
    iq, ik = oracle.regroup(q[0].float().numpy(), k[0].float().numpy())
    assert (iq.view(np.int32) == _np(giq).view(np.int32)).all()
    ob = oracle.build_buckets(ik, oracle.Config(**CFG2))
    assert (_np(gb.members) == ob.members).all()
    pos = np.array([T - 1])
    want_l, want_n = oracle.flat_select(iq[-1:], pos, ob, oracle.Config(**CFG2))
    monkeypatch.setenv("LSA_SELECT_IMPL", impl)
    gl, gn = lsa.flat_select(giq[-1:], torch.tensor([T - 1], device=DEV), gb, pcfg)
    assert (_np(gl) == want_l).all() and (_np(gn) == want_n).all()
    out = lsa.lsa_read(tq[:, -1:], tk, tv, gl[None], gn[None], 128 ** -0.5)
    want_o = oracle.sparse_read(q[:, -1:].float().numpy(), k.float().numpy(), v.float().numpy(), want_l[None],
                                want_n[None])
    assert float(np.abs(_np(out.float()) - want_o).max()) <= 2e-2


def test_gate_e_decode_step_equals_prefill_row(lsa):
    """src/lsa_rocm_lab/port/gates.py:332-354 on the gate geometry."""
    torch.manual_seed(20261105)
    T = 512
    cfg = lsa.PortConfig(cluster_block_size=128, bucket_size=8, bucket_cap=16, top_p=16, top_k=64, window_size=128,
                         sink_size=4, node_bucket_size=4, top_level=2, node_cluster_block_size=64, beam_width=4)
    q = torch.randn(1, T, 4, 64, device=DEV) * 0.2
    k = torch.randn(1, T, 2, 64, device=DEV) * 0.2
    v = torch.randn(1, T, 2, 64, device=DEV) * 0.2
    iq, ik = lsa.make_index_space(q, k)
    b = lsa.build_buckets_gpu(ik, cfg)
    pos = torch.arange(T, device=DEV)
    wl, wn = lsa.flat_select(iq, pos, b, cfg)
    whole = lsa.lsa_read(q, k, v, wl[None], wn[None], 0.125)
    sl, sn = lsa.flat_select(iq[-1:], pos[-1:], b, cfg)
    step = lsa.lsa_read(q[:, -1:], k, v, sl[None], sn[None], 0.125)
    assert torch.equal(sl[0], wl[-1]) and torch.equal(sn[0], wn[-1])
    assert float((step - whole[:, -1:]).abs().max()) < 5e-3


def test_full_size_lists_are_causal_unique_visible(lsa, monkeypatch):
    """Size-independent properties of a full 32k prefill-row select (every row, every arm)."""
    q, k, _ = _cfg2_inputs(seed=7)
    T = q.shape[1]
    giq, gik = lsa.make_index_space(q.to(DEV), k.to(DEV))
    pcfg = lsa.PortConfig(**CFG2)
    gb = lsa.build_buckets_gpu(gik, pcfg)
    pos = torch.arange(0, T, 97, device=DEV)
    res = {}
    for impl in ("reference", "fused", "fused_unpack"):
        monkeypatch.setenv("LSA_SELECT_IMPL", impl)
        res[impl] = lsa.flat_select(giq[pos], pos, gb, pcfg)
    for impl in ("fused", "fused_unpack"):
        assert torch.equal(res[impl][0], res["reference"][0]) and torch.equal(res[impl][1], res["reference"][1])
    lists, lengths = res["reference"]
    L, N = _np(lists), _np(lengths)
    P = _np(pos)
    for r in range(len(P)):
        ids = L[r, : N[r]]
        assert (ids >= 0).all() and (ids <= P[r]).all(), "causal"
        assert len(np.unique(ids)) == len(ids), "no id read twice"
        assert (L[r, N[r]:] == -1).all()
        sel = ids[: max(0, N[r] - min(64, P[r] + 1) - min(4, max(0, P[r] + 1 - 64)))]
        closed = P[r] // 512 * 512
        assert (sel < closed).all(), "selected ids come from closed blocks only"
