"""Bucket build, pairing and growth on the oracle (CPU only).

The Ward merge and the node pairing come from the absent upstream package; this build
defines their rules (oracle/lsa_oracle.c). These tests hold the C oracle to an
independent pure-Python statement of those rules on small blocks, check the structural
guarantees the reference relies on (a partition of every block into exactly bpb buckets
under the cap; node pairing into exact pairs), and check the closed-form growth the CUDA
tree kernel uses against the reference's replay loop (src/lsa_rocm_lab/port/_tree.py:100-142).
"""

import numpy as np
import pytest


def _ob(x: np.float32) -> int:
    b = int(np.array([x], np.float32).view(np.int32)[0])
    return b if b >= 0 else b ^ 0x7FFFFFFF


def _key(cost: np.float32, idx: int) -> int:
    return ((_ob(cost) & 0xFFFFFFFF) << 32 | idx) - (1 << 64 if _ob(cost) < 0 else 0)


def ward_python(oracle, s, sizes, target, cap):
    """Pure-Python statement of the merge rules (float32 scalars, same op order)."""
    f = np.float32
    P = s.shape[0]
    G = np.zeros((P, P), np.float32)
    for i in range(P):
        for j in range(i, P):
            G[i, j] = G[j, i] = oracle.cdot(s[i], s[j])
    alive = [True] * P
    sz = list(map(int, sizes))
    root = list(range(P))
    count = P
    while count > target:
        norm = [np.sqrt(G[i, i], dtype=np.float32) if alive[i] else f(0) for i in range(P)]
        nn, nk = [-1] * P, [None] * P
        for i in range(P):
            if not alive[i]:
                continue
            for j in range(P):
                if j == i or not alive[j] or sz[i] + sz[j] > cap:
                    continue
                merged = f(f(G[i, i] + G[j, j]) + f(f(2) * G[i, j]))
                cost = f(f(norm[i] + norm[j]) - np.sqrt(max(merged, f(0)), dtype=np.float32))
                k = _key(cost, j)
                if nk[i] is None or k < nk[i]:
                    nk[i] = k
            if nk[i] is not None:
                nn[i] = nk[i] & 0xFFFFFFFF
        pairs = [(i, nn[i]) for i in range(P) if alive[i] and nn[i] > i and nn[nn[i]] == i]
        if not pairs:
            return None
        pk = sorted(((nk[i] >> 32) << 32 | i, i, j) for i, j in pairs)
        take = pk[: count - target]
        partner = {i: j for _, i, j in take}
        dying = set(partner.values())
        Gn = G.copy()
        surv = [i for i in range(P) if alive[i] and i not in dying]
        for ai, A in enumerate(surv):
            for C in surv[ai:]:
                b, d = partner.get(A, -1), partner.get(C, -1)
                if b < 0 and d < 0:
                    continue
                if A == C:
                    v = f(f(G[A, A] + G[A, b]) + f(G[b, A] + G[b, b]))
                elif b >= 0 and d >= 0:
                    v = f(f(G[A, C] + G[A, d]) + f(G[b, C] + G[b, d]))
                elif b >= 0:
                    v = f(G[A, C] + G[b, C])
                else:
                    v = f(G[A, C] + G[A, d])
                Gn[A, C] = Gn[C, A] = v
        G = Gn
        for a, b in partner.items():
            sz[a] += sz[b]
            alive[b] = False
            root = [a if r == b else r for r in root]
        count -= len(partner)
    rank = {i: n for n, i in enumerate(i for i in range(P) if alive[i])}
    return np.array([rank[root[p]] for p in range(P)], np.int32)


@pytest.mark.parametrize("P,d,target,cap,pool", [(16, 16, 1, 64, 4), (16, 32, 4, 32, 4), (24, 8, 3, 40, 4),
                                                  (32, 64, 4, 48, 4), (12, 16, 6, 2, 1)])
def test_ward_c_matches_python_rules(oracle, P, d, target, cap, pool):
    rng = np.random.default_rng(P * 31 + d)
    s = rng.standard_normal((P, d)).astype(np.float32)
    sizes = np.full(P, pool, np.int32)
    want = ward_python(oracle, s, sizes, target, cap)
    got = np.empty(P, np.int32)
    status = oracle.lib().ora_ward_block(oracle._p(s), P, d, oracle._p(sizes), target, cap, oracle._p(got))
    assert status == 0 and want is not None
    assert (got == want).all()


@pytest.mark.parametrize("block,pool,bsize,cap,d", [(512, 4, 64, 128, 128), (128, 4, 8, 16, 64),
                                                    (64, 4, 64, 64, 128), (1024, 8, 128, 256, 64)])
def test_bucket_build_partitions_every_block(oracle, block, pool, bsize, cap, d):
    from oracle.oracle import Config

    rng = np.random.default_rng(block + d)
    T = 3 * block + 17  # a ragged tail block stays unbuilt
    keys = oracle.normalize_rows(rng.standard_normal((T, d)).astype(np.float32))
    cfg = Config(cluster_block_size=block, pool_size=pool, bucket_size=bsize, bucket_cap=cap)
    b = oracle.build_buckets(keys, cfg)
    bpb = block // bsize
    assert b.rows == 3 * bpb
    for g in range(3):
        m = b.members[g * bpb:(g + 1) * bpb]
        live = np.sort(m[m >= 0])
        assert (live == np.arange(g * block, (g + 1) * block)).all(), "each block is partitioned exactly"
        assert (b.sizes[g * bpb:(g + 1) * bpb] > 0).all() and (b.sizes <= cap).all()
        assert (b.sizes[g * bpb:(g + 1) * bpb] % pool == 0).all(), "buckets are unions of whole pools"
    for row in range(b.rows):
        m = b.members[row, : b.sizes[row]]
        assert (np.diff(m) > 0).all() and (b.members[row, b.sizes[row]:] == -1).all()
        want = np.zeros(d, np.float32)
        for t in m:
            want = (want + keys[t]).astype(np.float32)
        assert (b.key_sums[row] == want).all()
    norms = np.linalg.norm(b.centroids_f32.astype(np.float64), axis=1)
    np.testing.assert_allclose(norms, 1.0, atol=1e-5)


def test_bucket_build_is_deterministic_and_positional_arm(oracle):
    from oracle.oracle import Config

    rng = np.random.default_rng(7)
    keys = oracle.normalize_rows(rng.standard_normal((1024, 64)).astype(np.float32))
    cfg = Config(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128)
    a, b = oracle.build_buckets(keys, cfg), oracle.build_buckets(keys, cfg)
    assert (a.members == b.members).all() and (a.centroids_f32 == b.centroids_f32).all()
    p = oracle.position_buckets(keys, cfg)
    assert (p.members[:, :64] == np.arange(1024).reshape(16, 64)).all() and (p.members[:, 64:] == -1).all()


def test_pairing_makes_exact_pairs(oracle):
    rng = np.random.default_rng(9)
    sums = rng.standard_normal((3, 64, 32)).astype(np.float32)
    labels, node_sums = oracle.pair_to_size(sums, 4)
    for g in range(3):
        assert (np.bincount(labels[g], minlength=16) == 4).all()
        for n in range(16):
            kids = np.nonzero(labels[g] == n)[0]
            np.testing.assert_allclose(node_sums[g, n], sums[g, kids].sum(0), atol=1e-5)


def _growth_closed_form(page, cfg):
    """The closed form tree.cu evaluates on the device."""
    bpb, nb, size = cfg.block_bucket_count, cfg.node_cluster_block_size, cfg.node_bucket_size
    covered = page * bpb // nb * nb
    made, closed = [0] * cfg.top_level, [0] * cfg.top_level
    m = covered // size
    for level in range(cfg.top_level):
        made[level] = m
        if level + 1 < cfg.top_level:
            closed[level] = m // nb * nb
            m = closed[level] // size
    return covered, made, closed


@pytest.mark.parametrize("block,bsize,nb,size,top", [(512, 8, 64, 4, 3), (512, 64, 64, 4, 3), (1024, 128, 64, 16, 2),
                                                     (128, 8, 64, 4, 2), (512, 4, 64, 2, 4), (256, 2, 32, 8, 3)])
def test_growth_closed_form_equals_replay_loop(oracle, block, bsize, nb, size, top):
    from oracle.oracle import Config

    cfg = Config(cluster_block_size=block, bucket_size=bsize, node_cluster_block_size=nb, node_bucket_size=size,
                 top_level=top)
    for page in range(0, 600):
        assert oracle.growth_at(page, cfg) == _growth_closed_form(page, cfg), page
