"""GPU parity: scoring, packed-key top-k, expansion and the three select arms vs the oracle.

Bit-exact: scores (canonical fp32 dot), packed keys, best-first keys, read lists and
lengths. Cases mirror the reference's select tests (AIwork4me/latent-sparse-attention-rocm,
tests/test_select_fusion.py, test_select_topk.py, test_select_wide_adversarial.py).
"""

import os

import numpy as np
import pytest
import torch

from conftest import oracle_buckets_to_gpu

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIME = 20261108


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("R,N,d", [(1, 504, 1024), (5, 300, 128), (3, 77, 256), (2, 1000, 2048), (9, 16, 8)])
@pytest.mark.parametrize("kind", ["bf16", "fp32", "fp32xbf16"])
def test_scores_bit_exact(oracle, lsa, R, N, d, kind):
    rng = np.random.default_rng(R * 1000 + N + d)
    q = rng.standard_normal((R, d)).astype(np.float32)
    c = rng.standard_normal((N, d)).astype(np.float32)
    if kind != "fp32":
        c = oracle.bf16_round(c)
    if kind == "bf16":
        q = oracle.bf16_round(q)
    tq = torch.from_numpy(q).to(DEV)
    tc = torch.from_numpy(c).to(DEV)
    if kind == "bf16":
        tq = tq.bfloat16()
    if kind != "fp32":
        tc = tc.bfloat16()
    got = _np(lsa.pipeline.bucket_scores(tq, tc))
    want = oracle.scores(q, c)
    assert (got.view(np.int32) == want.view(np.int32)).all()


@pytest.mark.parametrize("rows,width,top_p,lengths_kind", [
    (64, 4096, 1024, "full"), (8, 4096, 1024, "ragged"), (64, 1024, 1024, "full"), (7, 300, 128, "ragged"),
    (5, 192, 1024, "full"), (3, 64, 64, "zeros"), (16, 2048, 512, "mix0"), (4, 16384, 256, "ragged"),
    (2, 12000, 1000, "full"), (1, 504, 32, "full"),
])
def test_select_topk_scores_and_best_first_exact(oracle, lsa, rows, width, top_p, lengths_kind):
    """tests/test_select_fusion.py:111-134 + test_select_wide_adversarial.py:143-198 (any width)."""
    rng = np.random.default_rng(TIME + width + rows)
    s = rng.standard_normal((rows, width)).astype(np.float32)
    if lengths_kind == "full":
        ln = np.full(rows, width, np.int32)
    elif lengths_kind == "ragged":
        ln = rng.integers(1, width + 1, rows).astype(np.int32)
    elif lengths_kind == "zeros":
        ln = np.zeros(rows, np.int32)
    else:
        ln = rng.integers(0, width + 1, rows).astype(np.int32)
    k = min(top_p, width)
    want = oracle.best_first(oracle.pack_keys(s, ln), k, ln)
    ts, tl = torch.from_numpy(s).to(DEV), torch.from_numpy(ln).to(DEV)
    got = _np(lsa.select_fused.select_topk_scores(ts, tl, top_p))
    assert (got[:, :k] == want).all()
    assert (got[:, k:] == oracle.EMPTY).all()
    keys = lsa.pipeline.pack_keys(ts, tl)
    assert (_np(keys) == oracle.pack_keys(s, ln)).all()
    # the reference chain's best-first keys, with and without the listing mask
    assert (_np(lsa.pipeline.best_first_keys(keys, top_p, counts=tl)) == want).all()
    assert (_np(lsa.pipeline.best_first_keys(keys, top_p)) == want).all()


def test_tied_denormal_nan_scores(oracle, lsa):
    """tests/test_select_fusion.py:137-174: ties -> lowest column; +-0, denormals, inf, NaN."""
    rng = np.random.default_rng(TIME + 5)
    s = rng.standard_normal((8, 1024)).astype(np.float32)
    s *= np.array([-1e30, -1e-30, 0.0, 1e-30, 1e30, -0.0, 1.0, -1.0], np.float32)[:, None]
    s[0, ::7] = np.nan
    s[1, :3] = -0.0
    s[2] = 0.0
    s[3, ::5] = np.inf
    s[4, ::3] = -np.inf
    s[5, 1::2] = -np.float32("nan")
    ln = np.full(8, 1024, np.int32)
    want = oracle.best_first(oracle.pack_keys(s, ln), 256, ln)
    got = _np(lsa.select_fused.select_topk_scores(torch.from_numpy(s).to(DEV), torch.from_numpy(ln).to(DEV), 256))
    assert (got == want).all()
    assert (oracle.unpack(got[2:3, :128]) == np.arange(128)).all()


def _members(rows, cap, seed, hi=997):
    g = np.random.default_rng(seed)
    m = (g.random((rows, cap)) * hi).astype(np.int32)
    m[g.random((rows, cap)) < 0.15] = -1
    return m


@pytest.mark.parametrize("rows,width,window,sink,top_k,positions_kind,cap", [
    (1, 1024, 512, 4, 4096, "last", 16), (32, 1024, 512, 4, 4096, "ragged", 16), (8, 256, 512, 4, 4096, "early", 16),
    (4, 256, 512, 4, 4096, "boundary", 16), (4, 128, 512, 4, 64, "last", 16), (4, 128, 8, 2, 4096, "last", 16),
    (2, 4096, 512, 4, 4096, "last", 16), (8, 512, 512, 4, 4096, "ragged", 8), (8, 512, 512, 4, 4096, "ragged", 32),
    (8, 512, 512, 4, 4096, "ragged", 64), (3, 504, 64, 4, 2048, "last", 128), (2, 512, 64, 0, 512, "last", 64),
])
def test_expand_exact(oracle, lsa, rows, width, window, sink, top_k, positions_kind, cap):
    """tests/test_select_fusion.py:196-240 and test_select_wide_adversarial.py:212-233."""
    rng = np.random.default_rng(TIME + width + top_k + cap)
    s = rng.standard_normal((rows, width)).astype(np.float32)
    ln = np.full(rows, width, np.int32)
    kk = min(1024, width)
    ordered = oracle.best_first(oracle.pack_keys(s, ln), kk)
    members = _members(width, cap, TIME + cap, hi=5000)
    if positions_kind == "last":
        pos = np.full(rows, 4096, np.int32)
    elif positions_kind == "ragged":
        pos = np.array([1, 511, 512, 513, 1023, 1024, 2047, 4095] * 4, np.int32)[:rows]
    elif positions_kind == "early":
        pos = np.arange(rows, dtype=np.int32)
    else:
        pos = np.array([511, 512, 513, 1024], np.int32)[:rows]
    want_l, want_n = oracle.expand(oracle.unpack(ordered), members, pos, window, sink, top_k)
    tk, tm, tp = (torch.from_numpy(x).to(DEV) for x in (ordered, members, pos))
    got_l, got_n = lsa.select_fused.expand_in_order_from_keys(tk, tm, tp, window, sink, top_k)
    assert (_np(got_l) == want_l).all() and (_np(got_n) == want_n).all()
    got_l, got_n = lsa.pipeline.expand_in_order(lsa.pipeline.unpack_ids(tk), tm, tp, window, sink, top_k)
    assert (_np(got_l) == want_l).all() and (_np(got_n) == want_n).all()


def test_non_pow2_bucket_cap_fails_loudly(lsa):
    """tests/test_select_wide_adversarial.py:243-253."""
    ordered = torch.full((4, 64), lsa.pipeline.EMPTY, device=DEV, dtype=torch.int64)
    members = torch.zeros(64, 24, dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError, match="power-of-two"):
        lsa.select_fused.expand_in_order_from_keys(ordered, members, torch.full((4,), 64, device=DEV), 64, 4, 128)


def _workspace(oracle, context, cfg, seed=TIME):
    rng = np.random.default_rng(seed + context)
    q = (rng.standard_normal((context, 8, 64)) * 0.2).astype(np.float32)
    k = (rng.standard_normal((context, 2, 64)) * 0.2).astype(np.float32)
    iq, ik = oracle.regroup(oracle.bf16_round(q), oracle.bf16_round(k))
    return iq, oracle.build_buckets(ik, cfg)


@pytest.mark.parametrize("context", [512, 1536, 2048, 8192])
@pytest.mark.parametrize("impl", ["reference", "fused", "fused_unpack"])
def test_switched_flat_select_exact_vs_oracle(oracle, lsa, monkeypatch, context, impl):
    """tests/test_select_fusion.py:257-270 - every arm equals the oracle byte for byte."""
    from oracle.oracle import Config

    cfg = Config()
    iq, ob = _workspace(oracle, context, cfg)
    want_l, want_n = oracle.flat_select(iq, np.arange(context), ob, cfg)
    b = oracle_buckets_to_gpu(ob)
    pcfg = lsa.PortConfig()
    monkeypatch.setenv("LSA_SELECT_IMPL", impl)
    got_l, got_n = lsa.flat_select(torch.from_numpy(iq).to(DEV), torch.arange(context, device=DEV), b, pcfg)
    assert (_np(got_l) == want_l).all() and (_np(got_n) == want_n).all()


@pytest.mark.parametrize("impl", ["reference", "fused", "fused_unpack"])
@pytest.mark.parametrize("score_dtype", ["bf16", "fp32"])
def test_decode_ragged_and_score_dtypes(oracle, lsa, monkeypatch, impl, score_dtype):
    """tests/test_select_fusion.py:275-313."""
    from oracle.oracle import Config

    cfg = Config()
    iq, ob = _workspace(oracle, 2048, cfg)
    b = oracle_buckets_to_gpu(ob)
    monkeypatch.setenv("LSA_SELECT_IMPL", impl)
    for pos in ([2047], [0], [0, 1, 511, 512, 513, 1024, 1536, 2045, 2047] * 3 + [2047, 2047, 2047, 2047, 2044]):
        pos = np.array(pos)
        want = oracle.flat_select(iq[pos], pos, ob, cfg, score_dtype=score_dtype)
        got = lsa.flat_select(torch.from_numpy(iq[pos]).to(DEV), torch.from_numpy(pos).to(DEV), b,
                              lsa.PortConfig(), score_dtype=score_dtype)
        assert (_np(got[0]) == want[0]).all() and (_np(got[1]) == want[1]).all()


def test_fused_deterministic_and_replayable(oracle, lsa, monkeypatch):
    """tests/test_select_fusion.py:318-332, plus the ticket reset: repeated launches agree."""
    from oracle.oracle import Config

    cfg = Config()
    iq, ob = _workspace(oracle, 2048, cfg)
    b = oracle_buckets_to_gpu(ob)
    monkeypatch.setenv("LSA_SELECT_IMPL", "fused")
    q = torch.from_numpy(iq[::8]).to(DEV)
    pos = torch.arange(2048, device=DEV)[::8]
    first = lsa.flat_select(q, pos, b, lsa.PortConfig())
    for _ in range(5):
        again = lsa.flat_select(q, pos, b, lsa.PortConfig())
        assert torch.equal(first[0], again[0]) and torch.equal(first[1], again[1])


def test_switch_rejects_unknown_impl(lsa, monkeypatch):
    monkeypatch.setenv("LSA_SELECT_IMPL", "bogus")
    with pytest.raises(ValueError, match="LSA_SELECT_IMPL"):
        lsa.flat_select(torch.zeros(2, 8, device=DEV), torch.tensor([7, 7], device=DEV), None, lsa.PortConfig())


@pytest.mark.parametrize("P,cap,top_k", [(300, 6, 1024), (100, 12, 512), (4096, 16, 4096), (1024, 16, 16384)])
def test_expand_staging_paths(oracle, lsa, P, cap, top_k):
    """The expansion's three ways of reaching the member rows: staged with 16-byte copies
    (cap % 4 == 0), staged with plain loads (cap % 4 != 0: 6), and the tiled walk from global
    memory when the rows and the gathered list outgrow shared memory (4096 picks x 16; a
    16384-id list) - all equal the checker's walk."""
    rng = np.random.default_rng(P + cap)
    rows = 3
    member_rows = 5000
    members = _members(member_rows, cap, P * 7 + cap, hi=60000)
    picks = np.stack([rng.permutation(member_rows)[:P] for _ in range(rows)]).astype(np.int32)
    picks[0, -5:] = -1  # short pick lists pad with -1
    pos = np.array([60000, 30000, 511], np.int32)
    want_l, want_n = oracle.expand(picks, members, pos, 64, 4, top_k)
    tp, tm, tpos = (torch.from_numpy(x).to(DEV) for x in (picks, members, pos))
    got_l, got_n = lsa.pipeline.expand_in_order(tp, tm, tpos, 64, 4, top_k)
    assert (_np(got_l) == want_l).all() and (_np(got_n) == want_n).all()


@pytest.mark.parametrize("R,N,top_p,cap,d", [(1, 504, 32, 128, 1024), (3, 40, 8, 32, 128), (2, 1500, 64, 64, 256),
                                             (40, 300, 16, 16, 128)])
def test_fp32_queries_read_as_bf16_equal_cast_queries(lsa, R, N, top_p, cap, d):
    """Query code 3 (fp32 storage, rounded to bf16 on load) gives byte-identical lists to the
    same queries cast to bf16 first (code 2), on the decode, cluster, streaming and per-row
    paths of lsa_select_fused."""
    from lsa_b200 import _lib

    rng = np.random.default_rng(N + top_p)
    block, bpb = 512, 8
    T = (N // bpb + 1) * block
    c = torch.from_numpy(rng.standard_normal((N, d)).astype(np.float32)).to(DEV).bfloat16()
    members = torch.from_numpy(rng.integers(-1, T, (N, cap)).astype(np.int32)).to(DEV)
    q32 = torch.from_numpy(rng.standard_normal((R, d)).astype(np.float32)).to(DEV)
    pos = torch.from_numpy(rng.integers(T // 2, T, R).astype(np.int32)).to(DEV)
    top_k, window, sink = 4 * cap, 64, 4
    width = top_k + window + sink
    L = _lib.lib()
    outs = []
    for q, code in ((q32, _lib.F32_AS_BF16), (q32.bfloat16().contiguous(), _lib.BF16)):
        lists = torch.empty(R, width, dtype=torch.int32, device=DEV)
        lengths = torch.empty(R, dtype=torch.int32, device=DEV)
        sc = torch.empty(L.lsa_select_fused_scratch(R, N) + 256, dtype=torch.uint8, device=DEV)
        ct = torch.zeros(R + 1, dtype=torch.int32, device=DEV)
        rc = L.lsa_select_fused(_lib.ptr(q), code, R, d, _lib.ptr(c), _lib.BF16, N, d, _lib.ptr(pos), block, bpb,
                                _lib.ptr(members), cap, top_p, window, sink, top_k, _lib.ptr(lists),
                                _lib.ptr(lengths), _lib.ptr(sc), sc.numel(), _lib.ptr(ct), ct.numel(), -1,
                                _lib.stream_of(q))
        assert rc == 0
        outs.append((_np(lists), _np(lengths)))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


SFQ_CFG = dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
               window_size=64, sink_size=4)


@pytest.mark.parametrize("dtype,Hq,Hkv,D,score_dtype", [
    ("bf16", 32, 8, 128, "bf16"), ("fp16", 8, 2, 64, "fp32"), ("fp32", 16, 1, 128, "bf16"),
    ("bf16", 4, 4, 32, "bf16"), ("bf16", 16, 2, 64, "fp32"),
])
def test_select_from_queries_equals_regroup_then_select(oracle, lsa, dtype, Hq, Hkv, D, score_dtype):
    """One launch from the model's raw queries (the index query built inside the decode select)
    gives the lists of regroup + the fused select, byte for byte, and the checker's lists;
    the 300-row batch goes the regroup-first way (more rows than the decode select takes)."""
    from lsa_b200.index_space import regroup_rows

    T = 4096
    rng = np.random.default_rng(Hq * 100 + D)
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]
    q = torch.from_numpy(rng.standard_normal((T, Hq, D)).astype(np.float32)).to(DEV).to(tdt)
    from conftest import drift_keys

    k = torch.from_numpy(drift_keys(rng, T, Hkv, D)).to(DEV).to(tdt)
    iq_np, ik_np = oracle.regroup(q.float().cpu().numpy(), k.float().cpu().numpy())
    ocfg = oracle.Config(**SFQ_CFG)
    ob = oracle.build_buckets(ik_np, ocfg)
    b = oracle_buckets_to_gpu(ob)
    pcfg = lsa.PortConfig(**SFQ_CFG)
    iq, _ = regroup_rows(q, k)
    assert (iq.cpu().numpy().view(np.uint32) == iq_np.view(np.uint32)).all()
    for pos in ([T - 1], [0], [0, 1, 511, 512, 513, 1024, 2047, 3000, T - 1], list(range(T - 300, T))):
        pos_np = np.array(pos)
        pt = torch.from_numpy(pos_np).to(DEV)
        got = lsa.select_from_queries(q[pt], pt, b, pcfg, score_dtype=score_dtype)
        two = lsa.pipeline._select_fused(iq[pt], pt, b, pcfg, pcfg.top_k, score_dtype)
        assert torch.equal(got[0], two[0]) and torch.equal(got[1], two[1])
        want = oracle.flat_select(iq_np[pos_np], pos_np, ob, ocfg, score_dtype=score_dtype)
        assert (_np(got[0]) == want[0]).all() and (_np(got[1]) == want[1]).all()


def test_select_from_queries_rejects_bad_shapes(lsa):
    b = lsa.Buckets(torch.zeros(4, 64, device=DEV, dtype=torch.bfloat16), torch.zeros(4, 8, device=DEV,
                    dtype=torch.int32), torch.zeros(4, device=DEV, dtype=torch.int32))
    pos = torch.tensor([7], device=DEV)
    with pytest.raises(ValueError, match="raw queries"):
        lsa.select_from_queries(torch.zeros(1, 64, device=DEV), pos, b, lsa.PortConfig())
    with pytest.raises(RuntimeError, match="Hkv"):  # 64 index dims do not split into heads of 48
        lsa.select_from_queries(torch.zeros(1, 4, 48, device=DEV), pos, b, lsa.PortConfig())
