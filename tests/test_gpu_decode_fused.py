"""The fused decode (one cooperative launch: scoring, grid barrier, top-32 + expansion in
every CTA, split read, ticket merge) against the two-launch path and the CPU checker:
lists bit-equal to flat_select, output within the bf16/fp16 tolerance of lsa_read and of
the checker's read (src/lsa_rocm_lab/port/gates.py:41-45 tolerances)."""

import os

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


def _setup(lsa, T, Hq, Hkv, positions, dtype, seed, cfg):
    from lsa_b200.index_space import index_keys, index_queries

    rng = np.random.default_rng(seed)
    k = torch.from_numpy(drift_keys(rng, T, Hkv, 128)).to(DEV).to(dtype)[None]
    v = torch.from_numpy(rng.standard_normal((1, T, Hkv, 128)).astype(np.float32)).to(DEV).to(dtype)
    q = torch.from_numpy(rng.standard_normal((1, len(positions), Hq, 128)).astype(np.float32)).to(DEV).to(dtype)
    iq = index_queries(q[0], Hkv)
    pcfg = lsa.PortConfig(**cfg)
    buckets = lsa.build_buckets_gpu(index_keys(k[0]), pcfg)
    pos = torch.tensor(positions, dtype=torch.int32, device=DEV)
    return q, k, v, iq, pos, pcfg, buckets


@pytest.mark.parametrize("positions", [[32767], [20000, 31000, 32767], [300, 511, 512, 16000]])
def test_fused_decode_cfg2(oracle, lsa, positions):
    q, k, v, iq, pos, pcfg, buckets = _setup(lsa, 32768, 32, 8, positions, torch.bfloat16, 41, CFG2)
    out, lists, lengths = lsa.pipeline.decode_fused(q, k, v, iq, pos, buckets, pcfg, return_lists=True)
    for impl in ("fused", "reference"):
        os.environ["LSA_SELECT_IMPL"] = impl
        try:
            wl, wn = lsa.flat_select(iq, pos, buckets, pcfg)
        finally:
            os.environ.pop("LSA_SELECT_IMPL", None)
        assert torch.equal(lists, wl) and torch.equal(lengths, wn), impl
    ref = lsa.lsa_read(q, k, v, wl[None], wn[None], 128 ** -0.5)
    assert float((out.float() - ref.float()).abs().max()) <= 2e-2
    # the read itself against the checker, for the last row
    want = oracle.sparse_read(_np(q)[:, -1:], _np(k), _np(v), _np(wl)[None, -1:], _np(wn)[None, -1:], 128 ** -0.5)
    assert float(np.abs(_np(out)[:, -1:] - want).max()) <= 2e-2
    assert lsa.prefill.status(DEV) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_decode_group8_and_fp16(lsa, dtype):
    cfg = dict(CFG2, top_p=16, top_k=1024)
    q, k, v, iq, pos, pcfg, buckets = _setup(lsa, 8192, 64, 8, [8191, 4000], dtype, 43, cfg)
    out, lists, lengths = lsa.pipeline.decode_fused(q, k, v, iq, pos, buckets, pcfg, return_lists=True)
    wl, wn = lsa.flat_select(iq, pos, buckets, pcfg)
    assert torch.equal(lists, wl) and torch.equal(lengths, wn)
    ref = lsa.lsa_read(q, k, v, wl[None], wn[None], 128 ** -0.5)
    tol = 5e-3 if dtype == torch.float16 else 2e-2
    assert float((out.float() - ref.float()).abs().max()) <= tol


def test_fused_decode_repeats_and_rejects(lsa):
    q, k, v, iq, pos, pcfg, buckets = _setup(lsa, 4096, 32, 8, [4095], torch.bfloat16, 45, CFG2)
    a = lsa.pipeline.decode_fused(q, k, v, iq, pos, buckets, pcfg)
    b = lsa.pipeline.decode_fused(q, k, v, iq, pos, buckets, pcfg)  # counters left at rest
    assert torch.equal(a, b)
    with pytest.raises(ValueError):  # five rows: beyond the fused path
        q5 = torch.zeros(1, 5, 32, 128, dtype=torch.bfloat16, device=DEV)
        lsa.pipeline.decode_fused(q5, k, v, iq.repeat(5, 1), pos.repeat(5), buckets, pcfg)
