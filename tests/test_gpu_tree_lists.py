"""The tree select's read lists from one call (lsa_tree_select_lists) against the two-step
form: the beam's picks (lsa_tree_select), then the expansion kernel (lsa_expand_in_order).

The reference's tree_select (src/lsa_rocm_lab/port/_tree.py:34-60) is exactly that two-step
form. lsa_tree_select_lists expands inside the beam's launch when its cluster form takes the
rows and the picked member rows fit its shared memory; otherwise it runs the two steps.
Each case here checks byte-equal lists and lengths on both paths, twice in a row (the second
call reuses the cached scratch and counters). The oracle parity of tree_select itself is in
test_gpu_build.py.
"""

import numpy as np
import pytest
import torch

from conftest import drift_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"

CFG2 = dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
            window_size=64, sink_size=4, node_bucket_size=4, top_level=3, node_cluster_block_size=64,
            beam_width=64)
# top_p * bucket_cap = 32768 member slots = 128 KB: past the one-launch staging budget
WIDE = dict(cluster_block_size=1024, pool_size=8, bucket_size=128, bucket_cap=256, top_p=128, top_k=16384,
            window_size=128, sink_size=4, node_bucket_size=16, top_level=2, node_cluster_block_size=64,
            beam_width=128)

CASES = [
    ("one decode row (one launch)", CFG2, 32768, 1),
    ("48 rows (one launch)", CFG2, 32768, 48),
    ("70 rows (per-level launches, then the expansion kernel)", CFG2, 32768, 70),
    ("members past the staging budget (beam, then the expansion kernel)", WIDE, 32768, 8),
]

_INDEX = {}


def _index(lsa, cfg, T):
    key = (tuple(sorted(cfg.items())), T)
    if key not in _INDEX:
        rng = np.random.default_rng(T + cfg["top_p"])
        Hkv, D = 8, 128
        k = torch.from_numpy(drift_keys(rng, T, Hkv, D)).to(DEV)
        q = torch.from_numpy(rng.standard_normal((T, 4 * Hkv, D)).astype(np.float32)).to(DEV)
        iq, ik = lsa.make_index_space(q[None], k[None])
        pcfg = lsa.PortConfig(**cfg)
        buckets = lsa.build_buckets_gpu(ik, pcfg)
        hierarchy = lsa.build_hierarchy_gpu(ik, buckets, pcfg)
        _INDEX.clear()
        _INDEX[key] = (iq, buckets, hierarchy, pcfg)
    return _INDEX[key]


@pytest.mark.parametrize("name,cfg,T,nrows", CASES, ids=[c[0] for c in CASES])
def test_tree_lists_equal_picks_then_expansion(lsa, name, cfg, T, nrows):
    from lsa_b200 import _tree, pipeline

    iq, buckets, hierarchy, pcfg = _index(lsa, cfg, T)
    rng = np.random.default_rng(nrows)
    rows = np.unique(np.concatenate([[T - 1], rng.integers(cfg["cluster_block_size"], T, 4 * nrows)]))[:nrows]
    pos = torch.from_numpy(rows.astype(np.int32)).to(DEV)
    q = iq[torch.from_numpy(rows).to(DEV)]
    picks = _tree.tree_picks(q, pos, buckets, hierarchy, pcfg)
    want_l, want_n = pipeline.expand_in_order(picks, buckets.members, pos, pcfg.window_size, pcfg.sink_size,
                                              pcfg.top_k)
    for _ in range(2):
        got_l, got_n = lsa.tree_select(q, pos, buckets, hierarchy, pcfg)
        torch.cuda.synchronize()
        assert torch.equal(got_n, want_n)
        assert torch.equal(got_l, want_l)
    assert int(want_n.min()) > pcfg.window_size  # the walk kept picked members, not only the tail
