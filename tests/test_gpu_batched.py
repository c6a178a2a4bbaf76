"""Batched decode (one row per sequence, ragged lengths): the one-launch batched selection
equals flat_select on each sequence's own buckets byte for byte, and the batched read
matches the CPU checker's read. Shapes follow the 128k batched-decode configuration scaled
down (Hq 64 / Hkv 8 / Dh 128, top-64 buckets) plus a small GQA case."""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def _case(lsa, lengths, Hq, Hkv, D, cfg, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    B, Tmax = len(lengths), max(lengths)
    q = torch.randn(B, 1, Hq, D, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(B, Tmax, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, Tmax, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    from lsa_b200.index_space import index_keys, index_queries

    iqs, per_seq = [], []
    for b, L in enumerate(lengths):
        iqs.append(index_queries(q[b], Hkv))
        per_seq.append(lsa.build_buckets_gpu(index_keys(k[b, :L]), cfg))
    pos = torch.tensor([L - 1 for L in lengths], dtype=torch.int32, device=DEV)
    return q, k, v, torch.cat(iqs), pos, per_seq


@pytest.mark.parametrize("impl", ["fused", "reference"])
def test_batched_select_equals_per_sequence(lsa, impl):
    from lsa_b200 import batched

    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=8, top_k=512,
                         window_size=64, sink_size=4)
    lengths = [2300, 4096, 1024, 3333, 511]
    q, k, v, iq, pos, per_seq = _case(lsa, lengths, 8, 2, 64, cfg, 11)
    bb = batched.concat_buckets(per_seq)
    gl, gn = batched.batched_select(iq, pos, bb, cfg)
    os.environ["LSA_SELECT_IMPL"] = impl
    try:
        for b in range(len(lengths)):
            wl, wn = lsa.flat_select(iq[b:b + 1], pos[b:b + 1], per_seq[b], cfg)
            assert torch.equal(gl[b:b + 1], wl) and torch.equal(gn[b:b + 1], wn), b
    finally:
        os.environ.pop("LSA_SELECT_IMPL", None)
    assert int(gn[4]) == 64 + 4  # a sequence shorter than a block: window + sinks only


def test_batched_decode_cfg4_shape_vs_oracle(oracle, lsa):
    """Hq 64 / Hkv 8 / Dh 128, top-64 buckets of 64 tokens (4096-token budget), ragged lengths."""
    from lsa_b200 import batched

    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=64, top_k=4096,
                         window_size=64, sink_size=4)
    rng = np.random.default_rng(20261105 + 4)
    lengths = [int(x) for x in rng.integers(8192, 16385, 6)]
    q, k, v, iq, pos, per_seq = _case(lsa, lengths, 64, 8, 128, cfg, 12)
    bb = batched.concat_buckets(per_seq)
    lists, lens = batched.batched_select(iq, pos, bb, cfg)
    for b in range(len(lengths)):
        wl, wn = lsa.flat_select(iq[b:b + 1], pos[b:b + 1], per_seq[b], cfg)
        assert torch.equal(lists[b:b + 1], wl) and torch.equal(lens[b:b + 1], wn), b
        ids = _np(lists[b, : lens[b]])
        assert (ids >= 0).all() and (ids < lengths[b]).all() and np.unique(ids).size == ids.size
    out = batched.batched_decode(q, k, v, iq, pos, bb, cfg, 128 ** -0.5)
    want = oracle.sparse_read(_np(q), _np(k), _np(v), _np(lists)[:, None], _np(lens)[:, None], 128 ** -0.5)
    assert float(np.abs(_np(out) - want).max()) <= 2e-2


def test_batched_select_rejects_mismatched_tables(lsa):
    from lsa_b200 import batched

    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=8, top_k=512,
                         window_size=64, sink_size=4)
    q, k, v, iq, pos, per_seq = _case(lsa, [2048, 2048], 8, 2, 64, cfg, 13)
    bb = batched.concat_buckets(per_seq[:1])
    with pytest.raises(ValueError):
        batched.batched_select(iq, pos, bb, cfg)


STREAM_CASES = [
    # (Hkv, D, bucket, cap, top_p, top_k): index width d = Hkv * D sets the columns per 32 KB stage
    (8, 128, 64, 128, 64, 4096),  # the 128k configuration: d = 1024, 16 columns per stage
    (2, 64, 32, 64, 128, 4096),  # d = 128: one 128-column item per stage, top-128 lists
    (4, 64, 64, 128, 32, 2048),  # d = 256, top-32
]


@pytest.mark.parametrize("Hkv,D,bucket,cap,top_p,top_k", STREAM_CASES)
def test_batched_select_wide_rows_stream_kernel(lsa, Hkv, D, bucket, cap, top_p, top_k):
    """Rows wider than one cluster (> 1024 visible buckets) take the persistent streaming
    kernel: every row equals the reference arm of flat_select on its own sequence, byte for
    byte, including a sequence shorter than a block and lengths off the block grid; the
    fused flat_select of one wide row (the same kernel, R = 1) agrees too; a replay gives
    the same lists (the tickets return to zero)."""
    from lsa_b200 import batched

    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=bucket, bucket_cap=cap, top_p=top_p,
                         top_k=top_k, window_size=64, sink_size=4)
    lengths = [70001, 131072, 300, 99999, 66560]
    q, k, v, iq, pos, per_seq = _case(lsa, lengths, Hkv * 2, Hkv, D, cfg, 21)
    bb = batched.concat_buckets(per_seq)
    assert bb.max_rows > 1024
    gl, gn = batched.batched_select(iq, pos, bb, cfg)
    gl2, gn2 = batched.batched_select(iq, pos, bb, cfg)
    assert torch.equal(gl, gl2) and torch.equal(gn, gn2)
    for impl in ("reference", "fused"):
        os.environ["LSA_SELECT_IMPL"] = impl
        try:
            for b in range(len(lengths)):
                wl, wn = lsa.flat_select(iq[b:b + 1], pos[b:b + 1], per_seq[b], cfg)
                assert torch.equal(gl[b:b + 1], wl) and torch.equal(gn[b:b + 1], wn), (impl, b)
        finally:
            os.environ.pop("LSA_SELECT_IMPL", None)
    assert int(gn[2]) == 64 + 4  # shorter than a block: window + sinks only


def test_batched_select_narrow_rows_wide_batch(lsa):
    """Rows that each fit one cluster but, together, enough columns to fill the GPU (at least
    8192 row-columns) take the streaming scorer too: every row equals the reference arm of
    flat_select on its own sequence."""
    from lsa_b200 import batched

    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
                         window_size=64, sink_size=4)
    rng = np.random.default_rng(77)
    lengths = [int(x) for x in rng.integers(12000, 16385, 40)]
    lengths[3] = 200  # shorter than a block
    q, k, v, iq, pos, per_seq = _case(lsa, lengths, 4, 2, 64, cfg, 31)
    bb = batched.concat_buckets(per_seq)
    assert len(lengths) * bb.max_rows >= 8192 and bb.max_rows <= 1024
    gl, gn = batched.batched_select(iq, pos, bb, cfg)
    os.environ["LSA_SELECT_IMPL"] = "reference"
    try:
        for b in range(len(lengths)):
            wl, wn = lsa.flat_select(iq[b:b + 1], pos[b:b + 1], per_seq[b], cfg)
            assert torch.equal(gl[b:b + 1], wl) and torch.equal(gn[b:b + 1], wn), b
    finally:
        os.environ.pop("LSA_SELECT_IMPL", None)
