"""Sequence-sharded tree decode, all shards emulated in one process (the exchanges are
concatenations): the selection equals the CPU checker's restatement of the sharded
procedure byte for byte, the merged read matches the checker's read of the same lists over
the whole sequence, and with one shard the procedure is exactly the single-GPU tree decode.
Configuration: the 1M tree config's knobs (1024-token blocks, 128-token buckets, nodes of
16, two levels, beam 64) at a 32k context, pools of 8 (a 1024-token block of pools of 4
would exceed the Ward merge's 128 pools per block)."""

import numpy as np
import pytest
import torch

from conftest import drift_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"
CFG = dict(cluster_block_size=1024, pool_size=8, bucket_size=128, bucket_cap=256, top_p=16, top_k=2048,
           window_size=128, sink_size=4, node_bucket_size=16, top_level=2, node_cluster_block_size=64,
           beam_width=64)


def _np(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def _setup(lsa, oracle, C, world, seed=7):
    from lsa_b200 import seqshard
    from lsa_b200.index_space import index_keys, index_queries

    rng = np.random.default_rng(seed)
    Hq, Hkv, D = 8, 2, 128
    k = torch.from_numpy(drift_keys(rng, C, Hkv, D) * 0.3).to(DEV).to(torch.bfloat16)[None]
    v = torch.from_numpy(rng.standard_normal((1, C, Hkv, D)).astype(np.float32)).to(DEV).to(torch.bfloat16)
    q = torch.from_numpy(rng.standard_normal((1, 1, Hq, D)).astype(np.float32) * 0.3).to(DEV).to(torch.bfloat16)
    iq = index_queries(q[0], Hkv)
    pcfg = lsa.PortConfig(**CFG)
    ocfg = oracle.Config(**CFG)
    shards, ora_shards = [], []
    for r in range(world):
        s0, s1 = seqshard.shard_bounds(C, world, r, CFG["cluster_block_size"])
        ik = index_keys(k[0, s0:s1])
        shards.append(seqshard.build_shard_index(ik, s0, pcfg))
        ob = oracle.build_buckets(_np(ik), ocfg)
        ora_shards.append((s0, s1 - s0, ob, oracle.build_hierarchy(ob, ocfg)))
    seqshard.globalise(shards)
    return q, k, v, iq, pcfg, ocfg, shards, ora_shards


def _run(q, k, v, iq, pos, shards, pcfg):
    from lsa_b200 import seqshard

    cands = [seqshard.shard_candidates(iq, pos, s, pcfg) for s in shards]
    lists, lengths = seqshard.select_from_candidates(torch.cat(cands, dim=1), pos, shards[0].members_global, pcfg)
    parts = [seqshard.shard_partial_read(q, k[:, s.start:s.start + s.length], v[:, s.start:s.start + s.length],
                                         lists[None], lengths[None], s.start) for s in shards]
    outs = torch.stack([p[0] for p in parts]).reshape(len(shards), -1, q.shape[-1])
    lses = torch.stack([p[1] for p in parts]).reshape(len(shards), -1)
    return lists, lengths, seqshard.merge_partials(outs, lses, q.dtype, q.shape)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_seqshard_matches_oracle(lsa, oracle, world):
    C = 32768
    q, k, v, iq, pcfg, ocfg, shards, ora_shards = _setup(lsa, oracle, C, world)
    pos = torch.tensor([C - 1], dtype=torch.int32, device=DEV)
    lists, lengths, out = _run(q, k, v, iq, pos, shards, pcfg)
    want_l, want_n = oracle.seqshard_select(_np(iq), [C - 1], ora_shards, ocfg)
    assert np.array_equal(_np(lists), want_l) and np.array_equal(_np(lengths), want_n)
    want = oracle.sparse_read(_np(q), _np(k), _np(v), want_l[None], want_n[None], 128 ** -0.5)
    assert float(np.abs(_np(out) - want).max()) <= 2e-2
    assert lsa.prefill.status(DEV) == 0


def test_one_shard_is_the_single_gpu_tree_decode(lsa, oracle):
    C = 32768
    q, k, v, iq, pcfg, ocfg, shards, ora_shards = _setup(lsa, oracle, C, 1, seed=9)
    pos = torch.tensor([C - 1], dtype=torch.int32, device=DEV)
    lists, lengths, out = _run(q, k, v, iq, pos, shards, pcfg)
    s = shards[0]
    tl, tn = lsa.tree_select(iq, pos, s.buckets, s.hierarchy, pcfg)
    assert torch.equal(lists, tl) and torch.equal(lengths, tn)
    ref = lsa.lsa_read(q, k, v, tl[None], tn[None], 128 ** -0.5)
    assert float((out.float() - ref.float()).abs().max()) <= 2e-2


def test_partial_read_lse_and_empty_shard(lsa):
    """A shard holding none of the row's keys contributes lse = -inf and weight 0."""
    from lsa_b200 import seqshard

    torch.manual_seed(3)
    q = torch.randn(1, 1, 8, 128, device=DEV).to(torch.bfloat16)
    k = torch.randn(1, 4096, 2, 128, device=DEV).to(torch.bfloat16)
    v = torch.randn(1, 4096, 2, 128, device=DEV).to(torch.bfloat16)
    lists = torch.arange(0, 1024, dtype=torch.int32, device=DEV)[None, None]
    lengths = torch.tensor([[1024]], dtype=torch.int32, device=DEV)
    o_a, l_a = seqshard.shard_partial_read(q, k[:, :2048], v[:, :2048], lists, lengths, 0)
    o_b, l_b = seqshard.shard_partial_read(q, k[:, 2048:], v[:, 2048:], lists, lengths, 2048)
    assert torch.isinf(l_b).all() and (l_b < 0).all() and o_b.abs().max() == 0
    merged = seqshard.merge_partials(torch.stack([o_a, o_b]).reshape(2, -1, 128),
                                     torch.stack([l_a, l_b]).reshape(2, -1), q.dtype, q.shape)
    ref = lsa.lsa_read(q, k, v, lists, lengths, 128 ** -0.5)
    assert float((merged.float() - ref.float()).abs().max()) <= 2e-2


def test_batched_step_equals_per_sequence(lsa, oracle):
    """The two-exchange step over several sequences (candidates of all sequences in one
    gather, one partial read for all of them, all partials in a second gather, one merge)
    matches the per-sequence step, here with one rank (the gather adds the rank axis)."""
    from lsa_b200 import seqshard

    C = 16384
    seqs = [_setup(lsa, oracle, C, 1, seed=s) for s in (21, 22, 23)]
    pos = torch.tensor([C - 1], dtype=torch.int32, device=DEV)
    gather = lambda x: x[None]
    pcfg = seqs[0][4]
    want = [seqshard.seqshard_decode(s[0], s[1], s[2], s[3], pos, s[6][0], pcfg, gather) for s in seqs]
    got = seqshard.seqshard_decode_batch(torch.cat([s[0] for s in seqs]), torch.cat([s[1] for s in seqs]),
                                         torch.cat([s[2] for s in seqs]), [s[3] for s in seqs], pos,
                                         [s[6][0] for s in seqs], pcfg, gather)
    assert got.shape == (3,) + tuple(seqs[0][0].shape[1:])
    for b in range(3):  # one batched read against three single-row reads: same lists, same keys
        assert float((got[b].float() - want[b][0].float()).abs().max()) <= 2e-2


def test_batched_step_in_cuda_graph(lsa, oracle):
    """The batched step captured in a CUDA graph (side-stream fork / join, graph-pool outputs,
    per-stream scratch sized in the eager warm-up) replays to the eager step's output, byte
    for byte, and replays again after the inputs change in place."""
    from lsa_b200 import seqshard

    C = 16384
    seqs = [_setup(lsa, oracle, C, 1, seed=s) for s in (31, 32)]
    pos = torch.tensor([C - 1], dtype=torch.int32, device=DEV)
    gather = lambda x: x[None]
    pcfg = seqs[0][4]
    q = torch.cat([s[0] for s in seqs])
    k = torch.cat([s[1] for s in seqs])
    v = torch.cat([s[2] for s in seqs])
    iqs = [s[3] for s in seqs]
    shards = [s[6][0] for s in seqs]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        step = lambda: seqshard.seqshard_decode_batch(q, k, v, iqs, pos, shards, pcfg, gather)
        eager = step().clone()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            out = step()
        g.replay()
        stream.synchronize()
        assert torch.equal(out, eager)
        q.mul_(0.5)  # new queries in place: the replay must follow them
        eager2 = step().clone()
        g.replay()
        stream.synchronize()
        assert torch.equal(out, eager2) and not torch.equal(eager2, eager)
    del g


def test_one_shard_batch_equals_the_sharded_step(lsa, oracle):
    """With one GPU holding every sequence whole, one_shard_decode_batch (the one-launch tree
    select per sequence, one read) matches the sharded step with one rank within the read
    tolerance, eagerly and replayed from a CUDA graph (byte for byte against its own eager
    output)."""
    from lsa_b200 import seqshard

    C = 16384
    seqs = [_setup(lsa, oracle, C, 1, seed=s) for s in (41, 42, 43)]
    pos = torch.tensor([C - 1], dtype=torch.int32, device=DEV)
    pcfg = seqs[0][4]
    q = torch.cat([s[0] for s in seqs])
    k = torch.cat([s[1] for s in seqs])
    v = torch.cat([s[2] for s in seqs])
    iqs = [s[3] for s in seqs]
    shards = [s[6][0] for s in seqs]
    want = seqshard.seqshard_decode_batch(q, k, v, iqs, pos, shards, pcfg, lambda x: x[None])
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        step = lambda: seqshard.one_shard_decode_batch(q, k, v, iqs, pos, shards, pcfg)
        eager = step().clone()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            out = step()
        g.replay()
        stream.synchronize()
        assert torch.equal(out, eager)
    del g
    assert eager.shape == want.shape
    assert float((eager.float() - want.float()).abs().max()) <= 2e-2
    with pytest.raises(ValueError):  # a shard that does not start at position 0 is not a whole sequence
        bad = seqshard.ShardIndex(1024, shards[0].length, shards[0].buckets, shards[0].hierarchy, 0)
        seqshard.one_shard_decode_batch(q[:1], k[:1], v[:1], iqs[:1], pos, [bad], pcfg)
