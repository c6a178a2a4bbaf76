"""Host-side sharding of the batched decode over ranks (gloo, world size 2, CPU): every
sequence is owned by exactly one rank, ranges are contiguous and balanced."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, B, q):
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "latent-sparse-attention-rocm_b200"))
    from lsa_b200.batched import shard_rows

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    start, end = shard_rows(B, world, rank)
    owned = torch.zeros(B, dtype=torch.int64)
    owned[start:end] = 1
    dist.all_reduce(owned)
    sizes = [None] * world
    dist.all_gather_object(sizes, end - start)
    if rank == 0:
        q.put((owned.tolist(), sizes))
    dist.destroy_process_group()


@pytest.mark.parametrize("B", [64, 5, 1])
def test_shard_rows_covers_batch_once(B):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, B, q)) for r in range(2)]
    for p in ps:
        p.start()
    owned, sizes = q.get(timeout=120)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert owned == [1] * B
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == B
