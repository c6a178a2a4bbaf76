"""The sequence-sharded decode's exchanges on CPU (gloo, world size 2): each rank builds the
CPU checker's index of its own block-aligned shard, computes its candidate keys, and the
package's all-gather (lsa_b200.seqshard.all_gather_fn) exchanges candidates and member
tables; the merged selection equals the single-process sharded selection on every rank."""

import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(cluster_block_size=256, pool_size=4, bucket_size=32, bucket_cap=64, top_p=6, top_k=160, window_size=32,
           sink_size=4, node_bucket_size=4, top_level=2, node_cluster_block_size=8, beam_width=8)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(C, d):
    rng = np.random.default_rng(31)
    keys = rng.standard_normal((C, d)).astype(np.float32)
    keys /= np.linalg.norm(keys, axis=1, keepdims=True)
    q = rng.standard_normal((2, d)).astype(np.float32)
    return keys, q


def _worker(rank, world, port, C, q_out):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "latent-sparse-attention-rocm_b200"))
    import torch
    import torch.distributed as dist

    from lsa_b200.seqshard import all_gather_fn, shard_bounds
    from oracle import oracle as O

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = O.Config(**CFG)
    keys, q = _inputs(C, 64)
    pos = np.array([C - 1, C - 200])
    s0, s1 = shard_bounds(C, world, rank, CFG["cluster_block_size"])
    b = O.build_buckets(keys[s0:s1], cfg)
    h = O.build_hierarchy(b, cfg)
    gather = all_gather_fn()
    rows = gather(torch.tensor([b.rows], dtype=torch.int64))[:, 0].tolist()
    offset = sum(rows[:rank])
    cand = O.shard_candidate_keys(q, pos, s0, s1 - s0, b, h, offset, cfg)
    all_cand = gather(torch.from_numpy(cand))  # [world, R, top_p]
    all_cand = all_cand.permute(1, 0, 2).reshape(cand.shape[0], -1).numpy()
    mine = np.where(b.members >= 0, b.members + s0, b.members).astype(np.int32)
    pad = max(rows) - mine.shape[0]
    padded = np.concatenate([mine, np.full((pad, mine.shape[1]), -1, np.int32)])
    tables = gather(torch.from_numpy(padded)).numpy()
    members = np.concatenate([tables[r][: rows[r]] for r in range(world)])
    lists, lengths = O.merge_shard_candidates(all_cand, pos, members, cfg)
    q_out.put((rank, lists.tolist(), lengths.tolist()))
    dist.destroy_process_group()


def test_seqshard_exchange_gloo():
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "latent-sparse-attention-rocm_b200"))
    from lsa_b200.seqshard import shard_bounds
    from oracle import oracle as O

    C, world = 2048, 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, C, q_out)) for r in range(world)]
    for p in ps:
        p.start()
    got = {}
    import queue
    import time

    deadline = time.time() + 300
    while len(got) < world and time.time() < deadline:
        try:
            r, l, n = q_out.get(timeout=2)
            got[r] = (l, n)
        except queue.Empty:
            assert all(p.exitcode in (None, 0) for p in ps), [p.exitcode for p in ps]
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert len(got) == world
    cfg = O.Config(**CFG)
    keys, q = _inputs(C, 64)
    shards = []
    for r in range(world):
        s0, s1 = shard_bounds(C, world, r, CFG["cluster_block_size"])
        b = O.build_buckets(keys[s0:s1], cfg)
        shards.append((s0, s1 - s0, b, O.build_hierarchy(b, cfg)))
    want_l, want_n = O.seqshard_select(q, np.array([C - 1, C - 200]), shards, cfg)
    for r in range(world):
        assert np.array_equal(np.array(got[r][0]), want_l) and np.array_equal(np.array(got[r][1]), want_n)
    assert (want_n > CFG["window_size"]).all()  # picks from both shards were walked


def test_shard_bounds_block_aligned():
    sys.path.insert(0, os.path.join(ROOT, "latent-sparse-attention-rocm_b200"))
    from lsa_b200.seqshard import shard_bounds

    for C, world, block in ((1 << 20, 8, 1024), (10000, 3, 512), (512, 4, 512)):
        bounds = [shard_bounds(C, world, r, block) for r in range(world)]
        assert bounds[0][0] == 0 and bounds[-1][1] == C
        for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
            assert a1 == b0 and a0 % block == 0
    with pytest.raises(ValueError):
        shard_bounds(100, 2, 2, 64)


def test_one_shard_batch_refuses_partial_shards_on_cpu():
    """one_shard_decode_batch serves a GPU that holds every sequence whole: a shard that starts
    past position 0, one shorter than the cache, or a batch without one shard per sequence is
    refused before any kernel runs."""
    sys.path.insert(0, os.path.join(ROOT, "latent-sparse-attention-rocm_b200"))
    import torch

    from lsa_b200 import pipeline
    from lsa_b200.seqshard import ShardIndex, one_shard_decode_batch

    q = torch.zeros(1, 1, 8, 64)
    k = torch.zeros(1, 2048, 2, 64)
    cfg = pipeline.PortConfig()
    whole = ShardIndex(0, 2048, None, None, 0)
    late = ShardIndex(1024, 1024, None, None, 0)
    short = ShardIndex(0, 1024, None, None, 0)
    pos = torch.tensor([2047], dtype=torch.int32)
    for shards in ([late], [short], [whole, whole]):
        with pytest.raises(ValueError):
            one_shard_decode_batch(q, k, k, [q[0, :, :2].reshape(1, -1)], pos, shards, cfg)
