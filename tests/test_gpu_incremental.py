"""Incremental index maintenance: the buckets and node hierarchy kept current by appends equal
a full rebuild (build_buckets_gpu + build_hierarchy_gpu on every key so far) bit for bit,
after every append - single positions, partial blocks, several blocks at once, appends that
complete node blocks at two levels."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _equal_index(state, keys, cfg, lsa):
    full_b = lsa.build_buckets_gpu(keys, cfg)
    inc_b = state.buckets
    for name in ("centroids", "members", "sizes", "centroids_f32", "key_sums"):
        a, b = getattr(inc_b, name), getattr(full_b, name)
        assert a.shape == b.shape and torch.equal(a, b), name
    full_h = lsa.build_hierarchy_gpu(keys, full_b, cfg)
    inc_h = state.hierarchy
    assert len(inc_h.levels) == len(full_h.levels)
    for lv_i, lv_f in zip(inc_h.levels, full_h.levels):
        for name in ("centroids", "children", "key_sums"):
            assert torch.equal(getattr(lv_i, name), getattr(lv_f, name)), name


@pytest.mark.parametrize("node_size", [4, 16])
def test_incremental_index_equals_rebuild(lsa, node_size):
    from lsa_b200.incremental import IndexState
    from lsa_b200.index_space import index_keys
    from lsa_b200.synthetic import drift_keys

    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
                         window_size=64, sink_size=4, node_bucket_size=node_size, node_cluster_block_size=64,
                         top_level=3)
    T = 70001
    g = torch.Generator(device=DEV)
    g.manual_seed(node_size)
    keys = index_keys(drift_keys(T, 2, 64, g, DEV)[0].to(torch.bfloat16))
    state = IndexState(keys.shape[1], cfg, DEV)
    rng = np.random.default_rng(node_size)
    sizes = [1, 1, 510, 37, 4096, 513, 511, 1, 8192, 16384]
    at, checks = 0, 0
    while at < T:
        n = sizes[checks] if checks < len(sizes) else int(rng.integers(1, 6000))
        n = min(n, T - at)
        state.append(keys[at:at + n])
        at += n
        checks += 1
        assert state.positions == at and state.closed == at // 512 * 512
        if checks <= len(sizes) or checks % 4 == 0 or at == T:
            _equal_index(state, keys[:at], cfg, lsa)
    assert len(state.hierarchy.levels) >= 2
    # selection over the maintained index equals selection over the rebuilt one
    iq = keys[-1:].clone()
    pos = torch.tensor([T - 1], dtype=torch.int32, device=DEV)
    full_b = lsa.build_buckets_gpu(keys, cfg)
    full_h = lsa.build_hierarchy_gpu(keys, full_b, cfg)
    a = lsa.tree_select(iq, pos, state.buckets, state.hierarchy, cfg)
    b = lsa.tree_select(iq, pos, full_b, full_h, cfg)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().view(np.uint32)


def test_incremental_index_equals_oracle(lsa, oracle):
    """The maintained index against the CPU checker's full build (oracle.build_buckets +
    oracle.build_hierarchy over every key so far), bit for bit, at several checkpoints."""
    from lsa_b200.incremental import IndexState
    from lsa_b200.index_space import index_keys
    from lsa_b200.synthetic import drift_keys

    cfg = dict(cluster_block_size=256, pool_size=4, bucket_size=32, bucket_cap=64, top_p=8, top_k=512,
               window_size=64, sink_size=4, node_bucket_size=4, node_cluster_block_size=32, top_level=2)
    T = 9000
    g = torch.Generator(device=DEV)
    g.manual_seed(7)
    keys = index_keys(drift_keys(T, 2, 32, g, DEV)[0].to(torch.bfloat16))
    state = IndexState(keys.shape[1], lsa.PortConfig(**cfg), DEV)
    ocfg = oracle.Config(**cfg)
    at = 0
    for n in (1, 300, 211, 1024, 2000, 5, 2459, 3000):
        n = min(n, T - at)
        state.append(keys[at:at + n])
        at += n
        if at < cfg["cluster_block_size"]:
            continue
        ob = oracle.build_buckets(keys[:at].float().cpu().numpy(), ocfg)
        b = state.buckets
        assert (b.members.cpu().numpy() == ob.members).all() and (b.sizes.cpu().numpy() == ob.sizes).all()
        assert (_bits(b.centroids_f32) == ob.centroids_f32.view(np.uint32)).all()
        assert (_bits(b.centroids) == ob.centroids_bf16.astype(np.float32).view(np.uint32)).all()
        assert (_bits(b.key_sums) == ob.key_sums.view(np.uint32)).all()
        oh = oracle.build_hierarchy(ob, ocfg)
        assert len(state.hierarchy.levels) == len(oh.levels)
        for lv, ol in zip(state.hierarchy.levels, oh.levels):
            assert (lv.children.cpu().numpy() == ol.children).all()
            assert (_bits(lv.centroids) == ol.centroids.view(np.uint32)).all()
            assert (_bits(lv.key_sums) == ol.key_sums.view(np.uint32)).all()
    assert at == T and len(state.hierarchy.levels) >= 1
