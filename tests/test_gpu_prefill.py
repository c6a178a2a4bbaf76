"""GPU parity of the prefill arm: per-tile selection bit-exact vs the CPU checker, the
tensor-core prefill read within tolerance of the checker's read over the same per-row
lists, and size-independent properties at the 32k prefill configuration.

The tile arm is not in the reference (it selects per row); the checker defines it
(oracle.tile_select / oracle.prefill_row_lists) and the read numerics follow
src/lsa_rocm_lab/port/read_kernel_tiled.py:41-89. Tolerances (max abs): bf16 2e-2,
fp16 5e-3 (src/lsa_rocm_lab/port/gates.py:41-45).
"""

import numpy as np
import pytest
import torch

from conftest import drift_keys, oracle_buckets_to_gpu

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float16: 5e-3, torch.bfloat16: 2e-2}
CFG = dict(cluster_block_size=256, pool_size=4, bucket_size=64, bucket_cap=128, top_p=4, top_k=256,
           window_size=64, sink_size=4)


def _np(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def _qkv(rng, T, Hq, Hkv, D, dtype):
    q = (rng.standard_normal((1, T, Hq, D)) * 0.3).astype(np.float32)
    k = drift_keys(rng, T, Hkv, D)[None].astype(np.float32) * 0.3
    v = rng.standard_normal((1, T, Hkv, D)).astype(np.float32)
    t = [torch.from_numpy(x).to(DEV).to(dtype) for x in (q, k, v)]
    return t, [_np(x) for x in t]


def test_tile_queries_bit_exact(oracle, lsa):
    rng = np.random.default_rng(1)
    for T, d in ((1000, 256), (64, 1024), (130, 8)):
        iq = rng.standard_normal((T, d)).astype(np.float32)
        got = lsa.prefill.tile_queries(torch.from_numpy(iq).to(DEV))
        want = oracle.tile_queries(oracle.bf16_round(iq), 64)
        assert got.shape == want.shape and np.array_equal(_np(got).view(np.int32), want.view(np.int32))


@pytest.mark.parametrize("T", [2048, 1000])
def test_tile_select_bit_exact(oracle, lsa, T):
    rng = np.random.default_rng(T)
    (tq, tk, _), _ = _qkv(rng, T, 8, 2, 64, torch.float32)
    iq, ik = lsa.make_index_space(tq, tk)
    ocfg = oracle.Config(**CFG)
    ob = oracle.build_buckets(_np(ik), ocfg)
    want_l, want_n = oracle.tile_select(_np(iq), ob, ocfg)
    gl, gn = lsa.prefill.tile_select(iq, oracle_buckets_to_gpu(ob), lsa.PortConfig(**CFG))
    assert np.array_equal(_np(gl), want_l) and np.array_equal(_np(gn), want_n)
    # the first block's tiles see nothing; later tiles read top_p full buckets + sinks
    assert (want_n[: CFG["cluster_block_size"] // 64] == 0).all()
    assert want_n.max() == CFG["top_k"] + CFG["sink_size"]


def _prefill_case(oracle, lsa, rng, T, Hq, Hkv, dtype, block=256, corrupt=False):
    (tq, tk, tv), (q, k, v) = _qkv(rng, T, Hq, Hkv, 128, dtype)
    tiles = (T + 63) // 64
    width = 300
    lists = np.full((tiles, width), -1, np.int32)
    lengths = np.zeros(tiles, np.int32)
    for t in range(tiles):
        bs = t * 64 // block * block
        if bs == 0:
            continue
        n = int(rng.integers(1, width + 1))
        lists[t, :n] = rng.integers(0, bs, n)
        lengths[t] = n
        if corrupt and n > 4:  # ids the read skips: pads and other negatives
            lists[t, 0], lists[t, 1], lists[t, 3] = -1, -7, -1
    rl, rn = oracle.prefill_row_lists(lists, lengths, T, oracle.Config(cluster_block_size=block))
    want = oracle.sparse_read(q, k, v, rl[None], rn[None], 128 ** -0.5)
    got = lsa.prefill.sparse_prefill(tq, tk, tv, torch.from_numpy(lists).to(DEV), torch.from_numpy(lengths).to(DEV),
                                     block)
    return got, want


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(8, 2), (16, 2), (32, 2)])
def test_sparse_prefill_vs_oracle(oracle, lsa, dtype, hq, hkv):
    rng = np.random.default_rng(hq * 31 + (dtype == torch.float16))
    got, want = _prefill_case(oracle, lsa, rng, 1024, hq, hkv, dtype)
    err = float(np.abs(_np(got) - want).max())
    assert err <= TOL[dtype], err
    assert lsa.prefill.status(DEV) == 0


def test_sparse_prefill_ragged_and_skipped_ids(oracle, lsa):
    rng = np.random.default_rng(7)
    got, want = _prefill_case(oracle, lsa, rng, 1000, 8, 2, torch.bfloat16, corrupt=True)  # T % 64 != 0
    assert torch.isfinite(got).all()
    assert float(np.abs(_np(got) - want).max()) <= TOL[torch.bfloat16]


def test_sparse_prefill_general_path_shapes(oracle, lsa):
    """Head groups / dims the tensor-core kernel does not take go through the general read."""
    rng = np.random.default_rng(8)
    for hq, hkv, dtype in ((4, 2, torch.bfloat16), (8, 8, torch.float32)):
        (tq, tk, tv), (q, k, v) = _qkv(rng, 512, hq, hkv, 128, dtype)
        lists = np.full((8, 40), -1, np.int32)
        lengths = np.zeros(8, np.int32)
        for t in range(4, 8):
            lists[t, :40] = rng.integers(0, 256, 40)
            lengths[t] = 40
        rl, rn = oracle.prefill_row_lists(lists, lengths, 512, oracle.Config(cluster_block_size=256))
        want = oracle.sparse_read(q, k, v, rl[None], rn[None], 128 ** -0.5)
        got = lsa.prefill.sparse_prefill(tq, tk, tv, torch.from_numpy(lists).to(DEV),
                                         torch.from_numpy(lengths).to(DEV), 256)
        tol = 1e-5 if dtype == torch.float32 else TOL[dtype]
        assert float(np.abs(_np(got) - want).max()) <= tol


def test_prefill_with_every_closed_key_is_dense_causal(lsa):
    """Tile lists holding every key of the closed blocks make the read dense causal attention."""
    torch.manual_seed(5)
    T, block = 2048, 512
    for dtype in (torch.bfloat16, torch.float16):
        q = (torch.randn(1, T, 32, 128, device=DEV) * 0.3).to(dtype)
        k = (torch.randn(1, T, 8, 128, device=DEV) * 0.3).to(dtype)
        v = torch.randn(1, T, 8, 128, device=DEV).to(dtype)
        tiles = T // 64
        lists = torch.full((tiles, T), -1, dtype=torch.int32, device=DEV)
        bs = torch.arange(tiles, device=DEV) * 64 // block * block
        col = torch.arange(T, device=DEV)
        lists = torch.where(col[None, :] < bs[:, None], col[None, :].expand(tiles, T), lists).to(torch.int32)
        got = lsa.prefill.sparse_prefill(q, k, v, lists, bs.to(torch.int32), block)
        dense = lsa.dense_read(q, k, v, 128 ** -0.5)
        err = float((got.float() - dense.float()).abs().max())
        assert err <= TOL[dtype], (dtype, err)


def test_prefill_32k_sampled_rows(oracle, lsa):
    """cfg 3 at full size (T 32768, Hq 32 / Hkv 8, Dh 128, bf16, drift keys, 64-token
    buckets, top-32 per 64-query tile): sampled rows against the checker's read of the
    same per-row lists; every tile list causal, unique and below its block."""
    rng = np.random.default_rng(20261105 + 3)
    T, Hq, Hkv, D = 32768, 32, 8, 128
    (tq, tk, tv), _ = _qkv(rng, T, Hq, Hkv, D, torch.bfloat16)
    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
                         window_size=64, sink_size=4)
    iq, ik = lsa.make_index_space(tq, tk)
    gb = lsa.build_buckets_gpu(ik, cfg)
    tl, tn = lsa.prefill.tile_select(iq, gb, cfg)
    out = lsa.prefill.sparse_prefill(tq, tk, tv, tl, tn, cfg.cluster_block_size)
    assert lsa.prefill.status(DEV) == 0
    tl_np, tn_np = _np(tl), _np(tn)
    for t in range(tl_np.shape[0]):
        bs = t * 64 // 512 * 512
        ids = tl_np[t, : tn_np[t]]
        assert (ids >= 0).all() and (ids < max(bs, 1)).all() and np.unique(ids).size == ids.size
    rows = np.array([0, 63, 511, 512, 4095, 17000, 32767])
    rl, rn = oracle.prefill_row_lists(tl_np, tn_np, T, oracle.Config(cluster_block_size=512))
    q_s = _np(tq)[:, rows]
    want = oracle.sparse_read(q_s, _np(tk), _np(tv), rl[rows][None], rn[rows][None], D ** -0.5)
    err = float(np.abs(_np(out)[:, rows] - want).max())
    assert err <= TOL[torch.bfloat16], err
