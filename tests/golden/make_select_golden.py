"""Generate tests/golden/select_golden.npz: selection and tree fixtures produced by the
reference's OWN code, run here on CPU.

The reference (AIwork4me/latent-sparse-attention-rocm) keeps its selection and tree logic
in src/lsa_rocm_lab/port/: the fused pack + top-k kernel ``_select_topk_scores``
(select_fused.py:52-80) and the rank-order walk ``_expand_in_order_keys``
(select_fused.py:141-214), both ``@triton.jit`` and run here under TRITON_INTERPRET=1;
``best_first_keys`` (pipeline.py:189-214) in torch; the tree's growth replay
``_growth_replay`` (_tree.py:100-142) and its beam ``_beam_pick_rows`` (_tree.py:318-373)
in torch. Those files import a few names from the upstream package ``lsa``
(Prefrontal-AI/latent-sparse-attention @ 5ebea732), which the reference does not ship;
they are stubbed here with this repository's documented definitions (the ones oracle/
restates and the CUDA kernels follow):

* ``keys.EMPTY`` = INT64_MIN; ``keys.ordered_bits`` = the order-preserving fp32 -> int32
  map (b >= 0 ? b : b ^ 0x7FFFFFFF); ``keys.key_bucket`` = 0x7FFFFFFF - (key & 0xFFFFFFFF);
* ``expansion._row_budget`` = (TOP_K, TOP_P) from EARLY_POSITION on (the callers pass 0);
  ``expansion._append_window_and_sink`` = the window [window_start, position] ascending,
  then the sinks [0, min(sink, window_start)); length = filled + both;
* ``hierarchy.Growth`` = a record of (covered_buckets, made, closed).

(Triton version shim: tl.topk gains the 3.8 ``descending=`` keyword, see _topk_compat.)
Everything else - the packing, the top-k order and its EMPTY tail, the walk's tiles,
masks, cumsum compaction and budget cap, the topk mask, the replay's block arithmetic,
the beam's candidate sort, first-occurrence dedup, stable descending order and lower-row
ties - is the reference's own code, loaded from its files unchanged. The fixtures
therefore pin oracle/ (and through the parity tests the CUDA kernels) to the reference's
selection logic; the stubbed definitions stay "unpinned vs upstream".

Usage (needs the reference checkout; the committed .npz is what the tests read):
    python tests/golden/make_select_golden.py /path/to/latent-sparse-attention-rocm
"""

from __future__ import annotations

import dataclasses
import importlib.util
import os
import pathlib
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "select_golden.npz"
EMPTY = -(2 ** 63)


# ------------------------------------------------------------------ upstream stubs


@triton.jit
def _ordered_bits(x):
    b = x.to(tl.int32, bitcast=True)
    return tl.where(b >= 0, b, b ^ 0x7FFFFFFF)


@triton.jit
def _key_bucket(key):
    return (0x7FFFFFFF - (key & 0xFFFFFFFF)).to(tl.int32)


@triton.jit
def _row_budget(position, TOP_K: tl.constexpr, TOP_P: tl.constexpr, EARLY_POSITION: tl.constexpr,
                EARLY_TOP_K: tl.constexpr, EARLY_TOP_P: tl.constexpr):
    early = position < EARLY_POSITION
    return tl.where(early, EARLY_TOP_K, TOP_K), tl.where(early, EARLY_TOP_P, TOP_P)


@triton.jit
def _append_window_and_sink(out_ptr, slot_ptr, position, window_start, filled, WINDOW_SIZE: tl.constexpr,
                            SINK_SIZE: tl.constexpr, LOCAL_BLOCK: tl.constexpr, MAP_SLOTS: tl.constexpr):
    i = tl.arange(0, LOCAL_BLOCK)
    nwin = position - window_start + 1
    nsink = tl.minimum(window_start, SINK_SIZE)
    ids = tl.where(i < nwin, window_start + i, i - nwin)
    keep = i < nwin + nsink
    if MAP_SLOTS:
        ids = tl.load(slot_ptr + ids, mask=keep, other=-1)
    tl.store(out_ptr + filled + i, ids, mask=keep)
    return filled + nwin + nsink


def _pack_keys_torch(scores, ids):
    bits = scores.float().contiguous().view(torch.int32).to(torch.int64)
    ob = torch.where(bits >= 0, bits, bits ^ 0x7FFFFFFF)
    key = (ob << 32) | (0x7FFFFFFF - ids.to(torch.int64).clamp_min(0))
    return torch.where(ids >= 0, key, torch.full_like(key, EMPTY))


@dataclasses.dataclass
class _Growth:
    covered_buckets: int
    made: list
    closed: list


# The reference targets Triton 3.8, whose tl.topk takes ``descending=``; Triton 3.6 (this
# image) always returns the top k descending and has no such keyword. Same semantics,
# keyword accepted.
from triton.language import standard as _tl_standard  # noqa: E402


@triton.jit
def _topk_compat(x, k: tl.constexpr, dim: tl.constexpr = None, descending: tl.constexpr = True):
    return _tl_standard.sort_impl(x, k=k, dim=dim, descending=descending)


def _install_stubs():
    tl.topk = _topk_compat

    def mod(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        sys.modules[name] = m
        return m

    mod("lsa")
    mod("lsa.core")
    mod("lsa.core.kernels")
    mod("lsa.core.kernels.triton")
    mod("lsa.core.kernels.triton.keys", EMPTY=EMPTY, ordered_bits=_ordered_bits, key_bucket=_key_bucket,
        pack_keys=_pack_keys_torch, unpack_ids=lambda k: torch.where(k == EMPTY, -1, 0x7FFFFFFF - (k & 0xFFFFFFFF)))
    mod("lsa.core.kernels.triton.expansion", _append_window_and_sink=_append_window_and_sink, _row_budget=_row_budget)
    mod("lsa.core.hierarchy", Growth=_Growth, growth_at=None, Hierarchy=object)
    mod("lsa_rocm_lab")
    mod("lsa_rocm_lab.port", HIP_PRECISION="ieee", triton_expansion=types.SimpleNamespace(),
        triton_top_k=types.SimpleNamespace(WHOLE=4), triton_ward=types.SimpleNamespace())


def _load(ref_root: pathlib.Path, name: str):
    path = ref_root / "src" / "lsa_rocm_lab" / "port" / f"{name}.py"
    spec = importlib.util.spec_from_file_location(f"lsa_rocm_lab.port.{name}", path)
    m = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = m
    spec.loader.exec_module(m)
    setattr(sys.modules["lsa_rocm_lab.port"], name, m)
    return m


# ------------------------------------------------------------------ cases


def _topk_cases(rng):
    """(name, scores [R, N] fp32, lengths [R] int32, top_p): the reference's kernel-A matrix
    (tests/test_select_fusion.py:112-173) at interpreter-sized widths, plus the decode rows of
    configurations 1 and 2."""
    cases = []

    def lens(kind, R, N):
        if kind == "full":
            return np.full(R, N, np.int32)
        if kind == "ragged":
            return rng.integers(1, N + 1, R).astype(np.int32)
        if kind == "zeros":
            return np.zeros(R, np.int32)
        return rng.integers(0, N + 1, R).astype(np.int32)

    for name, R, N, top_p, kind in [("cfg2_row", 4, 504, 32, "full"), ("cfg1_row", 3, 31, 8, "full"),
                                    ("k_eq_width", 4, 256, 256, "full"), ("nonpow2_ragged", 7, 300, 128, "ragged"),
                                    ("k_gt_width", 5, 192, 1024, "full"), ("zero_rows", 3, 64, 64, "zeros"),
                                    ("mixed_zero", 6, 512, 64, "mix0")]:
        cases.append((name, rng.standard_normal((R, N)).astype(np.float32), lens(kind, R, N), top_p))
    cases.append(("tied", np.zeros((4, 512), np.float32), np.full(4, 512, np.int32), 128))
    sc = rng.standard_normal((8, 1024)).astype(np.float32)
    sc *= np.array([-1e30, -1e-30, 0.0, 1e-30, 1e30, -0.0, 1.0, -1.0], np.float32)[:, None]
    cases.append(("neg_denormal", sc, np.full(8, 1024, np.int32), 256))
    sc = rng.standard_normal((4, 512)).astype(np.float32)
    sc[0, ::7] = np.nan
    sc[1] = np.nan
    sc[2, :3] = -0.0
    sc[3, ::5] = np.inf
    cases.append(("nan_inf_negzero", sc, np.full(4, 512, np.int32), 128))
    return cases


def _run_topk(sf, scores, lengths, top_p):
    R, N = scores.shape
    keep = min(top_p, N)
    k2 = triton.next_power_of_2(keep)
    out = torch.empty(R, k2, dtype=torch.int64)
    s = torch.from_numpy(scores)
    sf._select_topk_scores[(R,)](s, torch.from_numpy(lengths), out, s.stride(0), out.stride(0), N,
                                 BLOCK=triton.next_power_of_2(N), K2=k2)
    return out.numpy()


def _members(rng, rows, cap, hi=997):
    m = rng.integers(0, hi, (rows, cap)).astype(np.int32)
    m[rng.random((rows, cap)) < 0.15] = -1
    return m


def _run_expand(sf, keys, members, positions, window, sink, top_k):
    R, top_p = keys.shape
    cap = members.shape[1]
    decoding = R <= 32
    tile = max(1, (4096 if decoding else 1024) // cap)
    width = top_k + window + sink
    out = torch.empty(R, width, dtype=torch.int32)
    lengths = torch.empty(R, dtype=torch.int32)
    kt, mt, pt = torch.from_numpy(keys), torch.from_numpy(members), torch.from_numpy(positions)
    sf._expand_in_order_keys[(R,)](kt, mt, pt, out, lengths, mt, pt, kt.stride(0), width, 0, TOP_P=top_p,
                                   BUCKET_CAP=cap, TILE=tile, WINDOW_SIZE=window, SINK_SIZE=sink, TOP_K=top_k,
                                   WIDTH=width, PAD_BLOCK=triton.next_power_of_2(width),
                                   LOCAL_BLOCK=triton.next_power_of_2(window + sink), MAP_SLOTS=False,
                                   EARLY_POSITION=0, EARLY_TOP_K=0, EARLY_TOP_P=0)
    return out.numpy(), lengths.numpy()


def _expand_cases(rng, sf):
    """The reference's expansion matrix (tests/test_select_fusion.py:197-251) at interpreter
    sizes, plus configuration 2's decode geometry (cap 128, top-32, budget 2048, window 64)."""
    cases = []
    for name, R, N, window, sink, top_k, kind in [
            ("decode_last", 1, 512, 512, 4, 4096, "last"), ("ragged", 8, 512, 512, 4, 4096, "ragged"),
            ("early", 8, 256, 512, 4, 4096, "early"), ("boundary", 4, 256, 512, 4, 4096, "boundary"),
            ("tiny_topk", 4, 128, 512, 4, 64, "last"), ("tiny_window_sink", 4, 128, 8, 2, 4096, "last")]:
        scores = rng.standard_normal((R, N)).astype(np.float32)
        keys = _run_topk(sf, scores, np.full(R, N, np.int32), min(1024, N))
        members = _members(rng, N, 16)
        if kind == "last":
            pos = np.full(R, 4096, np.int32)
        elif kind == "ragged":
            pos = np.array([1, 511, 512, 513, 1023, 1024, 2047, 4095][:R], np.int32)
        elif kind == "early":
            pos = np.arange(R, dtype=np.int32)
        else:
            pos = np.array([511, 512, 513, 1024][:R], np.int32)
        cases.append((name, keys, members, pos, window, sink, top_k))
    # short rows: an EMPTY-heavy key tail (3 live columns, then none)
    keys = _run_topk(sf, rng.standard_normal((2, 64)).astype(np.float32), np.array([3, 0], np.int32), 64)
    cases.append(("empty_picks", keys, _members(rng, 64, 16), np.array([500, 500], np.int32), 64, 4, 128))
    # configuration 2: 504 visible buckets of a 32k cache, members within their 512-blocks
    keys = _run_topk(sf, rng.standard_normal((2, 504)).astype(np.float32), np.full(2, 504, np.int32), 32)
    mem = np.full((512, 128), -1, np.int32)
    for b in range(512):
        n = int(rng.integers(40, 90))
        mem[b, :n] = np.sort(rng.choice(64 * 8, n, replace=False)[:n] % 512 + (b // 8) * 512)
    cases.append(("cfg2_decode", keys, mem, np.array([32767, 32700], np.int32), 64, 4, 2048))
    return cases


def _tree_geometries():
    return {
        # the reference's own gate geometry (gates.py:448-457), pools of 4
        "gate": dict(cluster_block_size=128, pool_size=4, bucket_size=8, bucket_cap=16, top_p=16, top_k=64,
                     window_size=128, sink_size=4, node_bucket_size=4, top_level=2, node_cluster_block_size=64,
                     beam_width=4),
        # two levels with a wider beam (the shape of configuration 5, scaled down)
        "two_level": dict(cluster_block_size=256, pool_size=4, bucket_size=32, bucket_cap=64, top_p=32,
                          top_k=1024, window_size=128, sink_size=4, node_bucket_size=4, top_level=2,
                          node_cluster_block_size=16, beam_width=8),
    }


def main(ref_root: pathlib.Path) -> None:
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O

    O.build()
    _install_stubs()
    _load(ref_root, "read_kernel_tiled")
    pipe = _load(ref_root, "pipeline")
    sf = _load(ref_root, "select_fused")
    tree = _load(ref_root, "_tree")
    rng = np.random.default_rng(20261105)
    out: dict = {}

    # A: fused pack + top-k (select_fused.py:52-80)
    names = []
    for name, scores, lengths, top_p in _topk_cases(rng):
        out[f"topk/{name}/scores"] = scores
        out[f"topk/{name}/lengths"] = lengths
        out[f"topk/{name}/top_p"] = np.int64(top_p)
        out[f"topk/{name}/keys"] = _run_topk(sf, scores, lengths, top_p)
        names.append(name)
    out["topk/names"] = np.array(names)

    # B: the rank-order walk over packed keys (select_fused.py:141-214)
    names = []
    for name, keys, members, pos, window, sink, top_k in _expand_cases(rng, sf):
        lists, lengths = _run_expand(sf, keys, members, pos, window, sink, top_k)
        for k, v in dict(keys=keys, members=members, positions=pos, window=np.int64(window), sink=np.int64(sink),
                         top_k=np.int64(top_k), lists=lists, lengths=lengths).items():
            out[f"expand/{name}/{k}"] = v
        names.append(name)
    out["expand/names"] = np.array(names)

    # C: best_first_keys with the listing mask (pipeline.py:189-214)
    keys = rng.integers(-(2 ** 62), 2 ** 62, (6, 300), dtype=np.int64)
    keys[:, ::9] = EMPTY
    counts = np.array([300, 0, 17, 150, 299, 64], np.int32)
    out["best_first/keys"] = keys
    out["best_first/counts"] = counts
    out["best_first/top_p"] = np.int64(64)
    out["best_first/masked"] = pipe.best_first_keys(torch.from_numpy(keys), 64, torch.from_numpy(counts)).numpy()
    out["best_first/unmasked"] = pipe.best_first_keys(torch.from_numpy(keys), 64).numpy()

    # D + E: the growth replay (_tree.py:100-142) and the beam (_tree.py:318-373)
    names = []
    for gname, g in _tree_geometries().items():
        cfg = pipe.PortConfig(**g)
        pages = list(range(0, 97))
        covered, made, closed = tree._growth_replay(pages, cfg)
        out[f"growth/{gname}/pages"] = np.array(pages, np.int64)
        out[f"growth/{gname}/covered"] = np.array(covered, np.int64)
        out[f"growth/{gname}/made"] = np.array(made, np.int64)
        out[f"growth/{gname}/closed"] = np.array(closed, np.int64)
        # an index: drift-free random keys through the checker's build (the tree walk reads
        # only centroids and children, so any valid index serves)
        T = g["cluster_block_size"] * 24  # (index width 32: the walk does not depend on it)
        d = 32
        ik = O.normalize_rows(rng.standard_normal((T, d)).astype(np.float32))
        iq = rng.standard_normal((T, d)).astype(np.float32)
        ocfg = O.Config(**g)
        ob = O.build_buckets(ik, ocfg)
        oh = O.build_hierarchy(ob, ocfg)
        positions = np.unique(np.concatenate([rng.integers(0, T, 48), [0, T - 1, g["cluster_block_size"] * 8,
                                                                        g["cluster_block_size"] * 8 - 1]])).astype(np.int64)
        buckets = pipe.Buckets(torch.from_numpy(ob.centroids_bf16).bfloat16(), torch.from_numpy(ob.members),
                               torch.from_numpy(ob.sizes), centroids_f32=torch.from_numpy(ob.centroids_f32))
        hier = pipe.Hierarchy(levels=[pipe.NodeLevel(torch.from_numpy(lv.centroids), torch.from_numpy(lv.children),
                                                     torch.from_numpy(lv.key_sums)) for lv in oh.levels])
        picks = np.full((len(positions), g["top_p"]), -1, np.int64)
        page_of = positions // g["cluster_block_size"]
        for page in np.unique(page_of).tolist():
            rows = np.nonzero(page_of == page)[0]
            cv, md, cl = tree._growth_replay([page], cfg)
            growth = _Growth(cv[0], md[0], cl[0])
            picks[rows] = tree._beam_pick_rows(torch.from_numpy(iq[positions[rows]]), torch.from_numpy(positions[rows]),
                                               buckets, hier, growth, cfg).numpy()
        out[f"beam/{gname}/keys"] = ik
        out[f"beam/{gname}/queries"] = iq[positions]
        out[f"beam/{gname}/positions"] = positions
        out[f"beam/{gname}/picks"] = picks
        names.append(gname)
    out["tree/names"] = np.array(names)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB, {len(out)} arrays)")


if __name__ == "__main__":
    main(pathlib.Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LSA_REFERENCE_ROOT", "")))
