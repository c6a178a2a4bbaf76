"""The CUDA selection kernels against outputs of the reference's own selection code.

Same fixtures as tests/test_oracle_select_golden.py (tests/golden/select_golden.npz, made
by running the reference's select_fused.py / pipeline.py / _tree.py with only the absent
upstream names stubbed): the fused top-k (lsa_select_topk_scores), the walk from packed
keys (lsa_expand_from_keys), best_first_keys with and without the listing mask, and the
tree beam's picks (lsa_tree_select) on an index the GPU builds from the fixtures' keys.
Bit-exact.
"""

import pathlib

import numpy as np
import pytest
import torch

from test_oracle_select_golden import EMPTY, TREE_GEOMETRIES

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "select_golden.npz"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _names(g, group):
    return [str(n) for n in g[f"{group}/names"]]


def test_cuda_topk_matches_the_reference_kernel(lsa, g):
    for name in _names(g, "topk"):
        p = f"topk/{name}/"
        got = lsa.select_fused.select_topk_scores(_t(g[p + "scores"]), _t(g[p + "lengths"]), int(g[p + "top_p"]))
        want = g[p + "keys"]
        got = got.cpu().numpy()
        k = min(got.shape[1], want.shape[1])
        assert np.array_equal(got[:, :k], want[:, :k]), name
        assert (got[:, k:] == EMPTY).all() and (want[:, k:] == EMPTY).all(), name


def test_cuda_walk_matches_the_reference_kernel(lsa, g):
    for name in _names(g, "expand"):
        p = f"expand/{name}/"
        lists, lengths = lsa.select_fused.expand_in_order_from_keys(_t(g[p + "keys"]), _t(g[p + "members"]),
                                                                    _t(g[p + "positions"]), int(g[p + "window"]),
                                                                    int(g[p + "sink"]), int(g[p + "top_k"]))
        assert np.array_equal(lists.cpu().numpy(), g[p + "lists"]), name
        assert np.array_equal(lengths.cpu().numpy(), g[p + "lengths"]), name


def test_cuda_best_first_matches_the_reference(lsa, g):
    keys, counts, k = _t(g["best_first/keys"]), _t(g["best_first/counts"]), int(g["best_first/top_p"])
    assert np.array_equal(lsa.best_first_keys(keys, k, counts=counts).cpu().numpy(), g["best_first/masked"])
    assert np.array_equal(lsa.best_first_keys(keys, k).cpu().numpy(), g["best_first/unmasked"])


@pytest.mark.parametrize("geometry", sorted(TREE_GEOMETRIES))
def test_cuda_tree_picks_match_the_reference_beam(lsa, g, geometry):
    from lsa_b200 import _tree

    cfg = lsa.PortConfig(**TREE_GEOMETRIES[geometry])
    p = f"beam/{geometry}/"
    keys = _t(g[p + "keys"])
    buckets = lsa.build_buckets_gpu(keys, cfg)
    hierarchy = lsa.build_hierarchy_gpu(keys, buckets, cfg)
    picks = _tree.tree_picks(_t(g[p + "queries"]), _t(g[p + "positions"]), buckets, hierarchy, cfg)
    assert np.array_equal(picks.long().cpu().numpy(), g[p + "picks"]), geometry
