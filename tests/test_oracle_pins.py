"""Pin the CPU oracle before trusting it (CPU only).

1. The read oracle against the reference's OWN Triton read kernels, whose outputs were
   generated in the Triton interpreter (tests/golden/make_golden.py -> read_golden.npz).
2. The key / top-k / expansion contract against the known answers the reference's own
   tests assert (AIwork4me/latent-sparse-attention-rocm, tests/test_select_topk.py,
   tests/test_select_fusion.py, tests/test_select_wide_adversarial.py,
   tests/test_read_kernel_tiled.py), restated on the oracle.
3. The C expansion walk against a literal pure-Python restatement of the reference's
   tiled walk (src/lsa_rocm_lab/port/select_fused.py:172-214) on small cases.
"""

import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "read_golden.npz"
TOL = {"float32": 1e-5, "bfloat16": 2e-2}


def _cases():
    blob = np.load(GOLDEN)
    return blob, [str(c) for c in blob["cases"]]


@pytest.mark.parametrize("name", _cases()[1])
def test_read_oracle_matches_reference_triton_kernels(oracle, name):
    blob, _ = _cases()
    g = {k.split("/", 1)[1]: blob[k] for k in blob.files if k.startswith(name + "/")}
    dtype = str(g["dtype"])
    out = oracle.sparse_read(g["q"], g["k"], g["v"], g["ids"], g["lengths"], float(g["scale"]))
    if dtype == "bfloat16":
        out = oracle.bf16_round(out)
    for which in ("tiled_tm4_cn32", "tiled_tm1_cn64"):
        ref = g[which]
        assert np.isfinite(ref).all()
        err = float(np.abs(out - ref).max())
        assert err <= TOL[dtype], f"{name}/{which}: max abs {err}"
    # v1 agrees wherever it is defined (its zero-length rows are 0/0 = NaN)
    v1 = g["v1"]
    live = np.isfinite(v1)
    assert np.abs(out[live] - v1[live]).max() <= TOL[dtype]
    zero_rows = (g["lengths"] == 0)
    if zero_rows.any():
        assert np.isnan(v1[zero_rows]).all(), "the reference v1 kernel's documented NaN hazard"
        assert (out[zero_rows] == 0).all(), "zero-length rows read as zeros (the tiled contract)"


def test_duplicates_collapse_to_the_value_row(oracle):
    """tests/test_read_kernel_tiled.py:154-168 - a duplicated id weighs 2p/2p: the value row."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 1, 8, 64)).astype(np.float32)
    k = rng.standard_normal((1, 16, 2, 64)).astype(np.float32)
    v = rng.standard_normal((1, 16, 2, 64)).astype(np.float32)
    ids = np.full((1, 1, 8), -1, np.int32)
    ids[0, 0, :2] = 5
    out = oracle.sparse_read(q, k, v, ids, np.array([[2]], np.int32))
    for h in range(8):
        np.testing.assert_allclose(out[0, 0, h], v[0, 5, h // 4], atol=1e-6)


def test_full_causal_lists_equal_dense_attention(oracle):
    """The D2 anchor (port/gates.py:300-329): full causal lists reproduce dense causal attention."""
    import torch

    rng = np.random.default_rng(2)
    T, Hq, Hkv, D = 48, 4, 2, 64
    q = (rng.standard_normal((1, T, Hq, D)) * 0.2).astype(np.float32)
    k = (rng.standard_normal((1, T, Hkv, D)) * 0.2).astype(np.float32)
    v = (rng.standard_normal((1, T, Hkv, D)) * 0.2).astype(np.float32)
    row = np.arange(T)
    ids = np.where(row[None, :] <= row[:, None], row[None, :], -1).astype(np.int32)[None]
    out = oracle.sparse_read(q, k, v, ids, (row + 1).astype(np.int32)[None])
    tq = torch.from_numpy(q).permute(0, 2, 1, 3).double()
    tk = torch.from_numpy(k).permute(0, 2, 1, 3).double().repeat_interleave(Hq // Hkv, 1)
    tv = torch.from_numpy(v).permute(0, 2, 1, 3).double().repeat_interleave(Hq // Hkv, 1)
    dense = torch.nn.functional.scaled_dot_product_attention(tq, tk, tv, is_causal=True).permute(0, 2, 1, 3)
    np.testing.assert_allclose(out, dense.float().numpy(), atol=1e-6)


# ------------------------------------------------------------------ keys / top-k


def test_ordered_bits_preserve_order(oracle):
    vals = np.array([-np.inf, -1e30, -1.0, -1e-30, -0.0, 0.0, 1e-30, 1.0, 1e30, np.inf], np.float32)
    ob = oracle.ordered_bits(vals)
    assert (np.diff(ob.astype(np.int64)) > 0).all()
    rng = np.random.default_rng(3)
    x = rng.standard_normal(10000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 10000)
    x = x.astype(np.float32)
    order = np.argsort(x, kind="stable")
    ob = oracle.ordered_bits(x[order]).astype(np.int64)
    assert (np.diff(ob) >= 0).all()
    # defined NaN placement: +NaN above +inf, -NaN below -inf
    nan = np.array([np.float32("nan")], np.float32)
    neg_nan = (-nan).astype(np.float32)
    assert oracle.ordered_bits(nan)[0] > oracle.ordered_bits(np.array([np.inf], np.float32))[0]
    assert oracle.ordered_bits(neg_nan)[0] < oracle.ordered_bits(np.array([-np.inf], np.float32))[0]
    # the C scalar agrees with the vectorised form
    L = oracle.lib()
    for f in [-2.5, -0.0, 0.0, 3.25, float("inf")]:
        assert L.ora_ordered_bits(f) == int(oracle.ordered_bits(np.array([f], np.float32))[0])


def test_pack_unpack_round_trip(oracle):
    rng = np.random.default_rng(4)
    s = rng.standard_normal((3, 50)).astype(np.float32)
    keys = oracle.pack_keys(s, np.array([50, 20, 0], np.int32))
    ids = oracle.unpack(keys)
    assert (ids[0] == np.arange(50)).all()
    assert (ids[1, :20] == np.arange(20)).all() and (ids[1, 20:] == -1).all()
    assert (keys[2] == oracle.EMPTY).all()
    packed = oracle.pack_keys_of(s, np.arange(50)[None, :].repeat(3, 0))
    assert ((keys == packed) | (keys == oracle.EMPTY)).all()


@pytest.mark.parametrize("rows,width,top_p", [(64, 4096, 1024), (64, 1024, 1024), (7, 300, 128)])
def test_topk_equals_sort_slice(oracle, rows, width, top_p):
    """tests/test_select_topk.py:51-61: unique packed keys => top-k == sort-slice."""
    rng = np.random.default_rng(20261107)
    s = rng.standard_normal((rows, width)).astype(np.float32)
    keys = oracle.pack_keys(s, np.full(rows, width, np.int32))
    got = oracle.best_first(keys, top_p)
    want = np.sort(keys, axis=1)[:, ::-1][:, :top_p]
    assert want.shape == got.shape and (got == want).all()


def test_tied_scores_resolve_to_lowest_column(oracle):
    """tests/test_select_fusion.py:137-147: every score tied -> picks are 0, 1, 2, ..."""
    keys = oracle.pack_keys(np.zeros((4, 512), np.float32), np.full(4, 512, np.int32))
    picks = oracle.unpack(oracle.best_first(keys, 128))
    assert (picks == np.arange(128)[None, :]).all()


def test_empty_keys_sort_last_and_zero_visibility_is_all_empty(oracle):
    """tests/test_select_topk.py:73-82 and test_select_fusion.py:72-88."""
    rng = np.random.default_rng(2)
    s = rng.standard_normal((4, 64)).astype(np.float32)
    lengths = np.array([64, 40, 8, 0], np.int32)
    got = oracle.best_first(oracle.pack_keys(s, lengths), 8)
    assert (got[3] == oracle.EMPTY).all()
    assert (got[2, :8] != oracle.EMPTY).all()
    ids = oracle.unpack(got)
    assert (ids[1] < 40).all() and (ids[2] < 8).all()
    assert (np.diff(got.astype(object), axis=1) <= 0).all()


def test_unlisted_slots_are_masked(oracle):
    """tests/test_select_wide_adversarial.py:76-113: slots past a row's count never win."""
    rng = np.random.default_rng(5)
    rows, width = 6, 2048
    s = rng.standard_normal((rows, width)).astype(np.float32)
    counts = np.sort(rng.integers(0, width + 1, rows)).astype(np.int32)
    keys = oracle.pack_keys(s, counts)
    poison = np.where(np.arange(width)[None, :] >= counts[:, None], np.int64(2**63 - 2), keys)
    got = oracle.best_first(poison, 1024, counts)
    want = oracle.best_first(keys, 1024)
    assert (got == want).all()
    assert (oracle.best_first(keys, 1024, counts) == want).all(), "whole-path byte freeze"


# ------------------------------------------------------------------ expansion


def _walk_reference_style(picked, members, positions, window, sink, top_k, tile):
    """Literal restatement of the reference's tiled walk (select_fused.py:172-214) plus the
    window/sink tail this build defines (window ascending, then sinks below window_start)."""
    R, P = picked.shape
    cap = members.shape[1]
    width = top_k + window + sink
    out = np.full((R, width), -1, np.int64)
    lengths = np.zeros(R, np.int64)
    for r in range(R):
        pos = int(positions[r])
        ws = max(0, pos + 1 - window)
        slot = np.arange(tile * cap)
        filled = 0
        for first in range(0, P, tile):
            pick = first + slot // cap
            live = (pick < P) & (filled < top_k)
            bucket = np.where(live, picked[r, np.minimum(pick, P - 1)], -1)
            ids = np.where(bucket >= 0, members[np.maximum(bucket, 0), slot % cap], -1)
            valid = (bucket >= 0) & (ids >= sink) & (ids < ws)
            at = filled + np.cumsum(valid) - 1
            stored = valid & (at < top_k)
            out[r, at[stored]] = ids[stored]
            filled += int(valid.sum())
        filled = min(filled, top_k)
        n = filled
        for idx in range(ws, pos + 1):
            out[r, n] = idx
            n += 1
        for idx in range(min(sink, ws)):
            out[r, n] = idx
            n += 1
        lengths[r] = n
    return out, lengths


@pytest.mark.parametrize("positions,window,sink,top_k", [
    ([4096], 512, 4, 4096),
    ([1, 511, 512, 513, 1023, 1024, 2047, 4095], 512, 4, 4096),
    (list(range(8)), 512, 4, 4096),
    ([511, 512, 513, 1024], 512, 4, 4096),
    ([4096] * 4, 512, 4, 64),
    ([4096] * 4, 8, 2, 4096),
])
@pytest.mark.parametrize("tile", [1, 4, 64])
def test_expand_matches_reference_walk(oracle, positions, window, sink, top_k, tile):
    """The expansion edge matrix of tests/test_select_fusion.py:196-225 on the oracle."""
    rng = np.random.default_rng(20261108 + top_k + len(positions))
    width = 256
    members = (rng.random((width, 16)) * 997).astype(np.int32)
    members[rng.random((width, 16)) < 0.15] = -1
    s = rng.standard_normal((len(positions), width)).astype(np.float32)
    picked = oracle.unpack(oracle.best_first(oracle.pack_keys(s, np.full(len(positions), width, np.int32)), 128))
    picked[:, 100:] = -1  # an EMPTY tail contributes nothing
    pos = np.array(positions, np.int32)
    got_l, got_n = oracle.expand(picked, members, pos, window, sink, top_k)
    want_l, want_n = _walk_reference_style(picked, members, pos, window, sink, top_k, tile)
    assert (got_l == want_l).all() and (got_n == want_n).all()


def test_positional_picks_pattern(oracle):
    """The static positional arm: all visible buckets when few, else first 4, last 4 and
    24 strided between them, ascending and unique."""
    cfg = oracle.Config(cluster_block_size=512, bucket_size=64, top_p=32)
    p = oracle.positional_picks([100, 2047, 3000, 32767], 512, cfg)
    assert (p[0] == -1).all()  # nothing closed yet
    assert (p[1][:24] == np.arange(24)).all() and (p[1][24:] == -1).all()  # 24 visible: all of them
    for row, v in ((p[2], 40), (p[3], 504)):
        assert row.size == 32 and (np.diff(row) > 0).all() and (row >= 0).all()
        assert list(row[:4]) == [0, 1, 2, 3] and list(row[-4:]) == [v - 4, v - 3, v - 2, v - 1]


def test_oracle_map_slots_semantics(oracle):
    """The MAP_SLOTS restatement: mapped entries below the length, -1 elsewhere, -1 for ids
    outside the table and for slot rows outside it."""
    table = np.array([[10, 11, 12, 13], [20, 21, 22, 23]], np.int32)
    lists = np.array([[0, 3, 2, -1, 1], [3, 9, 0, 1, 2], [0, 1, 2, 3, 0]], np.int32)
    lengths = np.array([4, 3, 5], np.int32)
    got = oracle.map_slots(lists, lengths, table, np.array([1, 0, 5], np.int32))
    assert got.tolist() == [[20, 23, 22, -1, -1], [13, -1, 10, -1, -1], [-1, -1, -1, -1, -1]]
