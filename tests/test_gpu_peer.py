"""The all-gather over peer memory (lsa_b200.peer.PeerGather) against NCCL's all-gather, on
two GPUs (two spawned ranks): byte-equal results for several sizes and dtypes (16-byte
multiples and a padded odd size), repeated so both receive buffers and the epoch advance are
exercised, and replayed from a CUDA graph with the input changed in place. Skipped with fewer
than two GPUs."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [((4, 1, 64), torch.int64), ((128, 129), torch.float32), ((1000, 33), torch.bfloat16), ((3,), torch.int32),
          ((1 << 18,), torch.int32)]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, errors):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "latent-sparse-attention-rocm_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    import lsa_b200
    from lsa_b200.peer import PeerGather

    try:
        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        pg = PeerGather()
        g = torch.Generator(device="cuda")
        for it in range(4):
            for shape, dt in SHAPES:
                g.manual_seed(1000 * it + 10 * rank + len(shape))
                x = (torch.randn(shape, generator=g, device="cuda") * 1000).to(dt)
                got = pg(x)
                want = torch.empty((world,) + tuple(shape), dtype=dt, device="cuda")
                dist.all_gather_into_tensor(want.view(-1), x.reshape(-1))
                assert got.shape == want.shape and torch.equal(got, want)
        lsa_b200.check_status()
        # graph replay: the captured gather follows in-place changes of its input
        x = torch.zeros(128, 129, device="cuda")
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            pg(x)
            s.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                out = pg(x)
            for step in range(3):
                x.fill_(rank * 10 + step)
                graph.replay()
                s.synchronize()
                want = torch.stack([torch.full((128, 129), float(r * 10 + step), device="cuda") for r in range(world)])
                assert torch.equal(out, want)
        del graph
        lsa_b200.check_status()
        torch.cuda.synchronize()
        dist.barrier()
        pg.close()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        errors.put(f"rank {rank}: {type(exc).__name__}: {exc}")
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="the peer gather test needs two GPUs")
def test_peer_gather_equals_nccl_all_gather():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    world = 2
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, "; ".join(msgs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
