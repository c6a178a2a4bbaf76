"""GPU parity of the sparse read vs the oracle and the reference's golden vectors.

Tolerances (max abs): fp32 1e-5, fp16 5e-3, bf16 2e-2 - the north-star's fp32/bf16 bars
and the reference's fp16 gate (src/lsa_rocm_lab/port/gates.py:41-45). Cases mirror the
reference's read tests (tests/test_read_kernel_tiled.py): GQA/MQA, batches and ragged
rows, long decode rows (many splits), pads and boundary ids, duplicates, zero-length
rows, full causal == SDPA.
"""

import pathlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float32: 1e-5, torch.float16: 5e-3, torch.bfloat16: 2e-2}
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "read_golden.npz"


def _case(oracle, B, Tq, Tk, Hq, Hkv, D, width, dtype, seed, lengths=None, ids=None):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((B, Tq, Hq, D)) * 0.2).astype(np.float32)
    k = (rng.standard_normal((B, Tk, Hkv, D)) * 0.2).astype(np.float32)
    v = (rng.standard_normal((B, Tk, Hkv, D)) * 0.2).astype(np.float32)
    if dtype != torch.float32:
        q, k, v = (torch.from_numpy(x).to(dtype).float().numpy() for x in (q, k, v))
    if ids is None:
        ids = rng.integers(0, Tk, (B, Tq, width)).astype(np.int32)
    if lengths is None:
        lengths = np.full((B, Tq), width, np.int32)
    want = oracle.sparse_read(q, k, v, ids, lengths)
    tq, tk, tv = (torch.from_numpy(x).to(DEV).to(dtype) for x in (q, k, v))
    return tq, tk, tv, torch.from_numpy(ids).to(DEV), torch.from_numpy(lengths).to(DEV), want


def _check(got, want, dtype):
    err = float(np.abs(got.float().cpu().numpy() - want).max())
    assert err <= TOL[dtype], err


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("hq,hkv,D", [(8, 2, 64), (4, 1, 64), (2, 2, 64), (32, 8, 128), (64, 8, 128), (12, 4, 128)])
def test_read_gqa_vs_oracle(oracle, lsa, dtype, hq, hkv, D):
    tq, tk, tv, ids, ln, want = _case(oracle, 1, 5, 384, hq, hkv, D, 300, dtype, hq * 7 + D)
    _check(lsa.read_kernel_tiled.sparse_read_auto(tq, tk, tv, ids, ln, D ** -0.5), want, dtype)


@pytest.mark.parametrize("splits", [1, 3, 8, 16, 17, 40, 0])
def test_decode_row_splits_vs_oracle(oracle, lsa, splits):
    """A 2116-id decode row (cfg-2 width) through forced split counts; 0 = automatic."""
    from lsa_b200.read_kernel_tiled import _read

    tq, tk, tv, ids, ln, want = _case(oracle, 1, 1, 4096, 32, 8, 128, 2116, torch.bfloat16, 11)
    _check(_read(tq, tk, tv, ids, ln, 128 ** -0.5, splits=splits), want, torch.bfloat16)
    tq, tk, tv, ids, ln, want = _case(oracle, 1, 1, 4096, 32, 8, 128, 2116, torch.float32, 12)
    _check(_read(tq, tk, tv, ids, ln, 128 ** -0.5, splits=splits), want, torch.float32)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("width", [40, 200, 2116, 3000, 4000])
@pytest.mark.parametrize("hq,hkv,D", [(32, 8, 128), (8, 1, 64), (2, 2, 128), (16, 2, 64)])
def test_decode_read_shapes_vs_oracle(oracle, lsa, dtype, width, hq, hkv, D):
    """The decode-sized read (fewer than 16 (row, KV head) units, one cluster per unit):
    one CTA (40 ids) up to 16 CTAs of 8-32 slots per warp (4000 ids); out-of-range ids, -1
    pads and a length below the width are skipped."""
    rng = np.random.default_rng(width + hq + D)
    Tk = 4096
    ids = rng.integers(-1, Tk + 5, (1, 1, width)).astype(np.int32)
    lengths = np.array([[width - 3]], np.int32)
    tq, tk, tv, i, ln, want = _case(oracle, 1, 1, Tk, hq, hkv, D, width, dtype, width, lengths=lengths, ids=ids)
    _check(lsa.read_kernel_tiled.sparse_read_auto(tq, tk, tv, i, ln, D ** -0.5), want, dtype)


def test_decode_partial_read_vs_oracle(oracle, lsa):
    """The sequence-shard partial read of a decode row: fp32 output and log2-sum-exp over
    this shard's keys (global ids offset by the shard start) match the oracle's read."""
    from lsa_b200 import seqshard

    rng = np.random.default_rng(5)
    Tk, start, width = 2048, 1024, 2116
    ids = (rng.integers(0, Tk, (1, 1, width)) + start).astype(np.int32)
    tq, tk, tv, i, ln, _ = _case(oracle, 1, 1, Tk, 32, 8, 128, width, torch.bfloat16, 6, ids=ids - start)
    out, lse = seqshard.shard_partial_read(tq, tk, tv, torch.from_numpy(ids).to(DEV), ln, start, 128 ** -0.5)
    want = oracle.sparse_read(tq.float().cpu().numpy(), tk.float().cpu().numpy(), tv.float().cpu().numpy(),
                              ids - start, ln.cpu().numpy())
    assert float(np.abs(out.view(1, 1, 32, 128).cpu().numpy() - want).max()) <= TOL[torch.bfloat16]
    assert torch.isfinite(lse).all()


def test_batch_ragged_pad_boundary(oracle, lsa):
    rng = np.random.default_rng(3)
    B, T, width = 3, 13, 128
    ids = rng.integers(-1, T, (B, T, width)).astype(np.int32)  # -1 pads mixed in
    ids[0, :, 0], ids[0, :, 1] = 0, T - 1
    lengths = rng.integers(0, width + 1, (B, T)).astype(np.int32)
    lengths[1, 3] = width + 40  # claims past the width are clamped
    tq, tk, tv, i, ln, want = _case(oracle, B, T, T, 8, 2, 64, width, torch.bfloat16, 4, lengths=np.minimum(
        lengths, width), ids=ids)
    ln[1, 3] = width + 40
    _check(lsa.read_kernel.sparse_read(tq, tk, tv, i, ln, 0.125), want, torch.bfloat16)


def test_zero_length_and_duplicates(oracle, lsa):
    rng = np.random.default_rng(5)
    ids = rng.integers(0, 64, (1, 64, 32)).astype(np.int32)
    ids[0, 0, :2] = 5
    lengths = np.full((1, 64), 32, np.int32)
    lengths[0, 1::2] = 0
    lengths[0, 0] = 2
    tq, tk, tv, i, ln, want = _case(oracle, 1, 64, 64, 8, 2, 64, 32, torch.bfloat16, 6, lengths=lengths, ids=ids)
    got = lsa.read_kernel_tiled.sparse_read_tiled(tq, tk, tv, i, ln, 0.125)
    assert torch.isfinite(got).all()
    assert got[0, 1::2].float().abs().max() == 0.0
    _check(got, want, torch.bfloat16)
    for h in range(8):  # duplicated key -> that key's value row
        assert torch.allclose(got[0, 0, h].float(), tv[0, 5, h // 4].float(), atol=1e-2)


def test_full_causal_matches_dense_sdpa(lsa):
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        torch.manual_seed(20261106)
        T = 256
        q = (torch.randn(1, T, 8, 64, device=DEV) * 0.2).to(dtype)
        k = (torch.randn(1, T, 2, 64, device=DEV) * 0.2).to(dtype)
        v = (torch.randn(1, T, 2, 64, device=DEV) * 0.2).to(dtype)
        row = torch.arange(T, device=DEV, dtype=torch.int32)
        ids = torch.where(row[None, :] <= row[:, None], row[None, :].expand(T, T), torch.tensor(-1, device=DEV,
                                                                                                 dtype=torch.int32))
        got = lsa.read_kernel_tiled.sparse_read_tiled(q, k, v, ids.view(1, T, T), (row + 1).view(1, T), 0.125)
        dense = lsa.dense_read(q, k, v, 0.125)
        tol = {torch.float32: 1e-4, torch.float16: 5e-3, torch.bfloat16: 2e-2}[dtype]
        assert torch.allclose(got.float(), dense.float(), atol=tol, rtol=tol), dtype


def test_golden_vectors_through_cuda(lsa):
    """The reference Triton kernels' own outputs (tests/golden) reproduced by the B200 kernel."""
    blob = np.load(GOLDEN)
    for name in [str(c) for c in blob["cases"]]:
        g = {k.split("/", 1)[1]: blob[k] for k in blob.files if k.startswith(name + "/")}
        dtype = torch.bfloat16 if str(g["dtype"]) == "bfloat16" else torch.float32
        q, k, v = (torch.from_numpy(g[x]).to(DEV).to(dtype) for x in ("q", "k", "v"))
        got = lsa.read_kernel_tiled.sparse_read_auto(q, k, v, torch.from_numpy(g["ids"]).to(DEV),
                                                     torch.from_numpy(g["lengths"]).to(DEV), float(g["scale"]))
        err = float((got.float().cpu() - torch.from_numpy(g["tiled_tm4_cn32"])).abs().max())
        assert err <= TOL[dtype], (name, err)


def test_read_rejects_cpu_and_bad_groups(lsa):
    q = torch.zeros(1, 1, 6, 64)
    with pytest.raises(AssertionError):
        lsa.read_kernel_tiled.sparse_read_auto(q, q[:, :, :2], q[:, :, :2], torch.zeros(1, 1, 4, dtype=torch.int32),
                                               torch.zeros(1, 1, dtype=torch.int32))
    qg = torch.zeros(1, 1, 6, 64, device=DEV)
    kg = torch.zeros(1, 4, 4, 64, device=DEV)
    with pytest.raises(AssertionError):
        lsa.read_kernel_tiled.sparse_read_auto(qg, kg, kg, torch.zeros(1, 1, 4, dtype=torch.int32, device=DEV),
                                               torch.zeros(1, 1, dtype=torch.int32, device=DEV))


@pytest.mark.parametrize("dtype,B,Tq,hq,hkv,D,width", [
    (torch.bfloat16, 40, 1, 64, 8, 128, 2112),  # batched decode rows: 320 (row, KV head) units
    (torch.float16, 24, 3, 32, 8, 64, 1100),  # 576 units, D = 64, G = 4
    (torch.bfloat16, 3, 100, 8, 2, 128, 700),  # prefill-like rows: 600 units, G = 4
])
def test_persistent_read_vs_oracle(oracle, lsa, dtype, B, Tq, hq, hkv, D, width):
    """Batches with at least two (row, KV head) units per SM take the persistent read (16-bit
    inputs; fp32 keeps the split kernel with ticket merges): ragged lengths (zero, partial,
    full), -1 pads, out-of-range ids and duplicates, against the oracle."""
    rng = np.random.default_rng(B * 31 + Tq)
    Tk = 4096
    ids = rng.integers(-1, Tk + 3, (B, Tq, width)).astype(np.int32)  # -1 pads and ids >= Tk are skipped
    ids[..., 5:9] = ids[..., 1:5]  # duplicates count per occurrence
    lengths = rng.integers(0, width + 1, (B, Tq)).astype(np.int32)
    lengths.flat[0] = 0
    lengths.flat[-1] = width
    ids_ok = np.where((ids >= 0) & (ids < Tk), ids, -1).astype(np.int32)  # the checker's view of skipped ids
    tq, tk, tv, _, ln, want = _case(oracle, B, Tq, Tk, hq, hkv, D, width, dtype, B + Tq, lengths=lengths, ids=ids_ok)
    got = lsa.read_kernel_tiled.sparse_read_auto(tq, tk, tv, torch.from_numpy(ids).to(DEV), ln, D ** -0.5)
    _check(got, want, dtype)
    if dtype == torch.bfloat16:  # the fp32 inputs of the same case: split kernel, ticket merges
        f = lambda x: x.float()
        _check(lsa.read_kernel_tiled.sparse_read_auto(f(tq), f(tk), f(tv), torch.from_numpy(ids).to(DEV), ln,
                                                      D ** -0.5), want, torch.bfloat16)


def test_persistent_partial_reads_merge_to_full(lsa):
    """Partial reads (fp32 output + log2-sum-exp, global ids with an id base) over two halves
    of the keys, each through the persistent kernel, merge to the full read."""
    from lsa_b200 import seqshard

    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    B, Hq, Hkv, D, Tk, width = 48, 32, 8, 128, 2048, 1500
    q = torch.randn(B, 1, Hq, D, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(B, Tk, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, Tk, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    ids = torch.randint(0, Tk, (B, 1, width), generator=g, device=DEV, dtype=torch.int32)
    lens = torch.randint(0, width + 1, (B, 1), generator=g, device=DEV, dtype=torch.int32)
    full = lsa.read_kernel_tiled.sparse_read_auto(q, k, v, ids, lens, D ** -0.5).float()
    half = Tk // 2
    parts = [seqshard.shard_partial_read(q, k[:, lo:lo + half].contiguous(), v[:, lo:lo + half].contiguous(), ids,
                                         lens, lo, D ** -0.5) for lo in (0, half)]
    outs = torch.stack([p[0] for p in parts])
    lses = torch.stack([p[1] for p in parts])
    merged = seqshard.merge_partials(outs.reshape(2, -1, D), lses.reshape(2, -1), torch.float32, q.shape)
    assert float((merged - full).abs().max()) <= 2e-2
