"""The checker (oracle/) against selection and tree outputs of the reference's own code.

tests/golden/select_golden.npz was produced by tests/golden/make_select_golden.py, which
runs the reference's files unchanged - the fused pack + top-k and the rank-order walk
(src/lsa_rocm_lab/port/select_fused.py:52-80, 141-214) in the Triton interpreter,
best_first_keys (pipeline.py:189-214), the growth replay and the tree beam
(_tree.py:100-142, 318-373) in torch - with only the absent upstream names stubbed by this
repository's documented definitions (EMPTY, ordered_bits, key_bucket, the window/sink
tail, the row budget, the Growth record). Bit-exact throughout: packed keys, read lists,
lengths, growth counts and tree picks.
"""

import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "select_golden.npz"
EMPTY = np.int64(-(2 ** 63))
TREE_GEOMETRIES = {
    "gate": dict(cluster_block_size=128, pool_size=4, bucket_size=8, bucket_cap=16, top_p=16, top_k=64,
                 window_size=128, sink_size=4, node_bucket_size=4, top_level=2, node_cluster_block_size=64,
                 beam_width=4),
    "two_level": dict(cluster_block_size=256, pool_size=4, bucket_size=32, bucket_cap=64, top_p=32, top_k=1024,
                      window_size=128, sink_size=4, node_bucket_size=4, top_level=2, node_cluster_block_size=16,
                      beam_width=8),
}


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def _names(g, group):
    return [str(n) for n in g[f"{group}/names"]]


def test_fixture_covers_the_reference_matrices(g):
    assert len(_names(g, "topk")) >= 10 and len(_names(g, "expand")) >= 8 and len(_names(g, "tree")) == 2


def test_fused_topk_keys_match_the_reference_kernel(oracle, g):
    for name in _names(g, "topk"):
        scores, lengths = g[f"topk/{name}/scores"], g[f"topk/{name}/lengths"]
        top_p, want = int(g[f"topk/{name}/top_p"]), g[f"topk/{name}/keys"]
        keep = min(top_p, scores.shape[1])
        got = oracle.best_first(oracle.pack_keys(scores, lengths), keep)
        assert np.array_equal(got, want[:, :keep]), name
        assert (want[:, keep:] == EMPTY).all(), name  # the kernel's K2 tail


def test_walk_lists_match_the_reference_kernel(oracle, g):
    for name in _names(g, "expand"):
        p = f"expand/{name}/"
        lists, lengths = oracle.expand(oracle.unpack(g[p + "keys"]), g[p + "members"], g[p + "positions"],
                                       int(g[p + "window"]), int(g[p + "sink"]), int(g[p + "top_k"]))
        assert np.array_equal(lists, g[p + "lists"]), name
        assert np.array_equal(lengths, g[p + "lengths"]), name


def test_best_first_with_and_without_the_listing_mask(oracle, g):
    keys, counts, k = g["best_first/keys"], g["best_first/counts"], int(g["best_first/top_p"])
    assert np.array_equal(oracle.best_first(keys, k, counts), g["best_first/masked"])
    assert np.array_equal(oracle.best_first(keys, k), g["best_first/unmasked"])


@pytest.mark.parametrize("geometry", sorted(TREE_GEOMETRIES))
def test_growth_replay_matches_the_reference(oracle, g, geometry):
    cfg = oracle.Config(**TREE_GEOMETRIES[geometry])
    p = f"growth/{geometry}/"
    for i, page in enumerate(g[p + "pages"].tolist()):
        covered, made, closed = oracle.growth_at(page, cfg)
        assert covered == int(g[p + "covered"][i]), (geometry, page)
        assert list(made) == g[p + "made"][i].tolist(), (geometry, page)
        assert list(closed) == g[p + "closed"][i].tolist(), (geometry, page)


@pytest.mark.parametrize("geometry", sorted(TREE_GEOMETRIES))
def test_tree_picks_match_the_reference_beam(oracle, g, geometry):
    cfg = oracle.Config(**TREE_GEOMETRIES[geometry])
    p = f"beam/{geometry}/"
    ob = oracle.build_buckets(g[p + "keys"], cfg)
    oh = oracle.build_hierarchy(ob, cfg)
    got = oracle.tree_picks(g[p + "queries"], g[p + "positions"], ob, oh, cfg)
    assert np.array_equal(got, g[p + "picks"]), geometry
