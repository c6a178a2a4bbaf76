"""Benchmark: LSA decode select+read at 32k context, bf16, on B200.

Workload ("decode32k"): B=1, one query token, Hq=32, Hkv=8, Dh=128, bf16, drift keys,
64-token buckets in 512-token cluster blocks (8 per block, cap 128, pools of 4), top-32
buckets (2048-token budget), window 64, sinks 4 - the D-LSA Flat arm: the one-launch select
(LSA_SELECT_IMPL=fused) and the sparse read. A STEP is one decoded token through LAYERS = 32
layers, each layer its own independent 32k KV cache (4.3 GB of K/V in all), so one step
touches 32 x ~9.7 MB, more than twice the 126 MB L2, before any cache is revisited: no L2
flush is needed. The select+read index (buckets) is built before timing, as in the
reference's bench (src/lsa_rocm_lab/port/bench.py:113-154 times select+read on a prebuilt
index).

Before any number is printed, layer 0's read lists are checked bit-exactly and its output
within 2e-2 against the CPU checker (oracle/); a mismatch exits non-zero without a line (the
reference refuses to benchmark when its gates fail, src/lsa_rocm_lab/kernel_adapter.py:177-186).

value = algorithmic bytes of the step / step time, in GB/s (whole job: summed over the
N ranks, max time over ranks); us_per_select_read = step time / LAYERS. The device-timed
region replays a CUDA graph of one step K times with inputs resident, an event after every
replay: ``timing`` holds p50 / p95 / min / max / MAD over those K steps
(src/lsa_rocm_lab/port/bench.py:51-64). ``e2e`` is the same metric through the public
Python API with host buffers: every step copies the 32 layers' query rows from pinned host
memory, runs make_index_space + flat_select + lsa_read per layer, and copies the outputs
back - the step captured once in a CUDA graph whose replays include both copies
(``eager_*`` keys: the same step launched eagerly from Python, host-bound).

The other configurations ride in the same line: ``prefill`` (configs[2], one GPU),
``sharded`` (configs[3] batched 128k decode sharded by KV head, configs[4] tree decode of
1M-token sequences sharded by sequence - on every GPU count, so the N-GPU runs carry their
scaling) and ``cpu_baselines`` (the CPU checker on this box's host cores for configs 1-5,
bounded samples).

``--impl reference`` times the reference's CPU path for this workload on the host cores:
the CPU checker (oracle/, a restatement of the reference's select + read; the reference's
own path needs the absent upstream package and a ROCm GPU) builds the index and runs a
bounded sample of select+reads per step, one worker process per core; it loads no CUDA
library of this repository.

Multi-GPU (--gpus N under torchrun): the decode of one sequence does not shard, so the
headline runs N independent replicas (scaling "weak"; no collective on its data path);
``sharded`` runs the two configurations that do shard, with their NCCL exchanges.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
PKG = ROOT / "latent-sparse-attention-rocm_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode select+read µs/step & HBM GB/s @32k bf16; prefill select+read tok/s vs dense"
T_CTX, HQ, HKV, DH = 32768, 32, 8, 128
LAYERS = 32
CFG = dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=2048,
           window_size=64, sink_size=4)
SEED = 20261105


def _load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _profile_field(name: str, field: str):
    """A `field: value` number recorded in the committed ncu summary (profiles/), else None."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith(field + ":"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def _traffic_from_profile(name: str):
    """dram bytes per launch recorded in the committed ncu summary (profiles/), else None."""
    return _profile_field(name, "traffic_bytes_per_launch")


def _dist(ms: list) -> dict:
    """p50 / p95 / min / max / MAD of per-step times (ms), as the reference's summarize
    (src/lsa_rocm_lab/port/bench.py:51-64)."""
    xs = sorted(ms)
    n = len(xs)
    if not n:
        return {}
    p50 = statistics.median(xs)
    p95 = xs[min(n - 1, int(math.ceil(0.95 * n)) - 1)]
    mad = statistics.median([abs(x - p50) for x in xs])
    return {"samples": n, "p50_ms": round(p50, 5), "p95_ms": round(p95, 5), "min_ms": round(xs[0], 5),
            "max_ms": round(xs[-1], 5), "mad_ms": round(mad, 5)}


def _lscpu_model() -> str:
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return "unknown"


class GateError(RuntimeError):
    """The timed path disagrees with the CPU checker: no number may be reported."""


def gate_decode(L, lists, lengths, out) -> dict:
    """Layer 0 of the decode step against the CPU checker on the same index: the read lists
    bit-exact, the output within 2e-2 (bf16)."""
    import numpy as np

    from oracle import oracle as O

    b = L["buckets"]
    ob = O.Buckets(b.centroids_f32.cpu().numpy(), b.centroids.float().cpu().numpy(), b.members.cpu().numpy(),
                   b.sizes.cpu().numpy(), b.key_sums.cpu().numpy())
    want_l, want_n = O.flat_select(L["iq"].float().cpu().numpy(), np.array([T_CTX - 1]), ob, O.Config(**CFG))
    got_l, got_n = lists.cpu().numpy(), lengths.cpu().numpy()
    if not (np.array_equal(got_l, want_l) and np.array_equal(got_n, want_n)):
        raise GateError("decode32k layer 0: read lists differ from the CPU checker")
    want_o = O.sparse_read(L["q"].float().cpu().numpy(), L["k"].float().cpu().numpy(), L["v"].float().cpu().numpy(),
                           want_l[None], want_n[None], DH ** -0.5)
    err = float(np.abs(out.float().cpu().numpy() - want_o).max())
    if not err <= 2e-2:
        raise GateError(f"decode32k layer 0: output max abs err {err} > 2e-2")
    return {"lists_bit_exact": True, "output_max_abs_err": err, "tolerance": 2e-2, "checker": "oracle/ (CPU)"}


# --------------------------------------------------------------------------- B200 arm


def decode_config(world, decode_impl="split"):
    """The decode32k line's config (the same dict on the B200 and the reference arms)."""
    return {"workload": "decode32k", "layers_per_step": LAYERS, "context": T_CTX, "batch": 1, "heads_q": HQ,
            "heads_kv": HKV, "head_dim": DH, "bucket_size": CFG["bucket_size"], "top_p_buckets": CFG["top_p"],
            "budget_tokens": CFG["top_k"], "window": CFG["window_size"], "sink": CFG["sink_size"],
            "decode_impl": decode_impl, "parallelism": f"replicas{world}",
            "l2": "no flush: 32 independent 32k caches, each step touches 32 x ~9.7 MB > 2x L2"}


def build_layers(dev, lsa, arms=False):
    """LAYERS independent caches: K/V, the decode row's q and index query, the Ward buckets
    (and with ``arms`` the node hierarchy and the positional buckets)."""
    import torch

    from lsa_b200.index_space import regroup_rows
    from lsa_b200.synthetic import drift_keys

    pcfg = lsa.PortConfig(**CFG)
    layers = []
    for layer in range(LAYERS):
        gen = torch.Generator(device=dev)
        gen.manual_seed(SEED + T_CTX + layer)
        k = drift_keys(T_CTX, HKV, DH, gen, dev).to(torch.bfloat16)
        v = torch.randn(1, T_CTX, HKV, DH, generator=gen, device=dev).to(torch.bfloat16)
        q = torch.randn(1, 1, HQ, DH, generator=gen, device=dev).to(torch.bfloat16)
        _, ik = regroup_rows(k[0], k[0])  # index keys (the query half of this call is unused)
        buckets = lsa.build_buckets_gpu(ik, pcfg)
        # the other decode arms of the configuration: the tree over these buckets, and the
        # positional block-sparse buckets
        hierarchy = lsa.build_hierarchy_gpu(ik, buckets, pcfg) if arms else None
        pbuckets = lsa.position_buckets(ik, pcfg) if arms else None
        del ik
        iq, _ = regroup_rows(q[0], k[0, -1:])
        layers.append(dict(k=k, v=v, q=q, iq=iq.to(torch.bfloat16), iq32=iq, buckets=buckets, hierarchy=hierarchy,
                           pbuckets=pbuckets, pos=torch.tensor([T_CTX - 1], device=dev, dtype=torch.int32)))
    torch.cuda.synchronize(dev)
    return pcfg, layers


def exchange_fn(world):
    """The sharded legs' all-gather and its name: NCCL by default, or over peer memory (stores
    into the peers' arenas over NVLink, lsa_b200.peer) with LSA_EXCHANGE=peer. Measured at two
    GPUs: tree1m 168.5 us/step with NCCL, 176.5 with the peer gather; the batched split
    selection 233 vs 242 us - the step's exchanges are latency-bound either way."""
    from lsa_b200 import seqshard

    if world == 1:
        return (lambda x: x[None]), "none"
    if os.environ.get("LSA_EXCHANGE", "nccl") == "peer":
        return seqshard.peer_gather_fn(), "peer-memory"
    return seqshard.all_gather_fn(), "NCCL"


def run_b200(args, rank, world, dev):
    import torch

    import lsa_b200 as lsa
    from lsa_b200 import pipeline

    os.environ["LSA_SELECT_IMPL"] = "fused"
    scale = DH ** -0.5
    pcfg, layers = build_layers(dev, lsa, arms=not args.quick)
    stream = torch.cuda.Stream(dev)

    def select(L):
        return pipeline._select_fused(L["iq"], L["pos"], L["buckets"], pcfg, pcfg.top_k, "bf16")

    def read(L, lists, lengths):
        return lsa.lsa_read(L["q"], L["k"], L["v"], lists[None], lengths[None], scale)

    def fused(L):
        return pipeline.decode_fused(L["q"], L["k"], L["v"], L["iq"], L["pos"], L["buckets"], pcfg, scale)

    def split_step():
        outs = []
        for L in layers:
            lists, lengths = select(L)
            outs.append(read(L, lists, lengths))
        return outs

    def step():
        if args.decode_impl == "split":
            return split_step()
        return [fused(L) for L in layers]

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
        sel = [select(L) for L in layers]
        out0 = read(layers[0], *sel[0])
        stream.synchronize()
    gate = gate_decode(layers[0], sel[0][0], sel[0][1], out0)  # raises GateError on a mismatch
    lengths_all = [int(s[1].item()) for s in sel]
    n_ids = sum(lengths_all)
    members_bytes = LAYERS * CFG["top_p"] * CFG["bucket_cap"] * 4
    visible = min((T_CTX - 1) // CFG["cluster_block_size"] * (CFG["cluster_block_size"] // CFG["bucket_size"]),
                  layers[0]["buckets"].rows)
    centroid_bytes = LAYERS * visible * HKV * DH * 2
    kv_bytes = n_ids * HKV * DH * 2 * 2
    small = LAYERS * (HQ * DH * 2 * 2 + HKV * DH * 2 + (CFG["top_k"] + CFG["window_size"] + CFG["sink_size"]) * 4 * 2)
    step_bytes = centroid_bytes + members_bytes + kv_bytes + small
    read_bytes_per_launch = (kv_bytes + n_ids * 4) / LAYERS + HQ * DH * 2 * 2

    # one graph holding one step (LAYERS select+read pairs), replayed K times
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    split_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(split_graph, stream=stream):
        for _ in range(args.steps):
            split_step()
    fused_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for L in layers:
            fused(L)
        stream.synchronize()
    with torch.cuda.graph(fused_graph, stream=stream):
        for _ in range(args.steps):
            for L in layers:
                fused(L)
    read_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(read_graph, stream=stream):
        for _ in range(args.steps):
            for L, (ls, ln) in zip(layers, sel):
                read(L, ls, ln)
    select_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(select_graph, stream=stream):
        for _ in range(args.steps):
            for L in layers:
                select(L)
    # the select from the model's raw query (index query built in the kernel): the e2e step's
    select_q_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(select_q_graph, stream=stream):
        for _ in range(args.steps):
            for L in layers:
                lsa.select_from_queries(L["q"][0], L["pos"], L["buckets"], pcfg)

    def timed(g, reps=1):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 3)):
                g.replay()
            stream.synchronize()
            if world > 1:
                torch.distributed.barrier()
            torch.cuda.synchronize(dev)
            ev0.record(stream)
            for _ in range(reps):
                g.replay()
            ev1.record(stream)
            stream.synchronize()
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        return ev0.elapsed_time(ev1) / reps

    def timed_steps(g, steps):
        """K replays of a one-step graph between a barrier and synchronisations; an event
        after every replay gives the per-step distribution."""
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 3)):
                g.replay()
            stream.synchronize()
            if world > 1:
                torch.distributed.barrier()
            torch.cuda.synchronize(dev)
            evs[0].record(stream)
            for i in range(steps):
                g.replay()
                evs[i + 1].record(stream)
            stream.synchronize()
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        per = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
        return evs[0].elapsed_time(evs[-1]), per

    with ClockSampler(dev.index) as clocks:
        ms_total, per_step = timed_steps(graph, args.steps)
    ms_read = timed(read_graph)
    ms_select = timed(select_graph)
    ms_select_q = timed(select_q_graph)
    ms_split = timed(split_graph)
    ms_fused = timed(fused_graph)
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_per_step = ms_total / args.steps
    value = world * step_bytes / (ms_per_step / 1e3) / 1e9
    us_read = ms_read / args.steps / LAYERS * 1e3
    us_select = ms_select / args.steps / LAYERS * 1e3

    # end to end through the public API with host buffers
    q_host = torch.stack([L["q"] for L in layers]).cpu().pin_memory()
    k_last = [L["k"][0, -1:] for L in layers]
    out_host = torch.empty(LAYERS, 1, 1, HQ, DH, dtype=torch.bfloat16).pin_memory()
    from lsa_b200.index_space import regroup_rows

    def e2e_step():
        qd = q_host.to(dev, non_blocking=True)
        outs = []
        for i, L in enumerate(layers):
            if args.decode_impl == "split":
                # the index query is built inside the select from the model's query
                lists, lengths = lsa.select_from_queries(qd[i, 0], L["pos"], L["buckets"], pcfg)
                outs.append(lsa.lsa_read(qd[i], L["k"], L["v"], lists[None], lengths[None], scale))
            else:
                iq, _ = regroup_rows(qd[i, 0], k_last[i])
                outs.append(pipeline.decode_fused(qd[i], L["k"], L["v"], iq, L["pos"], L["buckets"], pcfg, scale))
        out_host.copy_(torch.stack(outs), non_blocking=True)

    e2e_ms, us_dense, us_tree, us_positional = float("nan"), float("nan"), float("nan"), float("nan")
    e2e_eager_ms = float("nan")
    ms_batch = float("nan")
    index_maint = None
    if not args.quick:
        with torch.cuda.stream(stream):
            for _ in range(3):
                e2e_step()
            stream.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            torch.cuda.nvtx.range_push("e2e_eager")  # launch lists: ncu --nvtx --nvtx-include e2e_eager/
            for _ in range(args.steps):
                e2e_step()
            torch.cuda.nvtx.range_pop()
            ev1.record(stream)
            stream.synchronize()
            e2e_eager_ms = ev0.elapsed_time(ev1) / args.steps
            # the same public-API step captured once in a CUDA graph, as a serving loop would
            # run it: every replay copies the step's q from pinned host memory and the outputs
            # back (the copies are nodes of the graph), only the host's launch work is gone
            e2e_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(e2e_graph, stream=stream):
                e2e_step()
            for _ in range(3):
                e2e_graph.replay()
            stream.synchronize()
            ev0.record(stream)
            for _ in range(args.steps):
                e2e_graph.replay()
            ev1.record(stream)
            stream.synchronize()
            del e2e_graph
        e2e_ms = ev0.elapsed_time(ev1) / args.steps
        t = torch.tensor([e2e_ms, e2e_eager_ms], device=dev, dtype=torch.float64)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms, e2e_eager_ms = float(t[0].item()), float(t[1].item())

        # dense decode baseline (SDPA over the whole cache) on the same rotation
        dense_graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for L in layers:
                lsa.dense_read(L["q"], L["k"], L["v"], scale)
            stream.synchronize()
        with torch.cuda.graph(dense_graph, stream=stream):
            for L in layers:
                lsa.dense_read(L["q"], L["k"], L["v"], scale)
        us_dense = timed(dense_graph, reps=2) / LAYERS * 1e3

        # the configuration's other arms on the same rotation: D-LSA Tree and positional
        def arm_ms(select_fn):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                for L in layers:
                    ls, ln = select_fn(L)
                    read(L, ls, ln)
                stream.synchronize()
            with torch.cuda.graph(gr, stream=stream):
                for L in layers:
                    ls, ln = select_fn(L)
                    read(L, ls, ln)
            return timed(gr, reps=2) / LAYERS * 1e3

        us_tree = arm_ms(lambda L: lsa.tree_select(L["iq32"], L["pos"], L["buckets"], L["hierarchy"], pcfg))
        us_positional = arm_ms(lambda L: pipeline.positional_select(L["pos"], L["pbuckets"], pcfg))

        # the same LAYERS caches decoded as ONE batch of LAYERS sequences (one batched select
        # launch + one batched read launch): the bandwidth view of this decode
        from lsa_b200 import batched

        kb = torch.cat([L["k"] for L in layers])
        vb = torch.cat([L["v"] for L in layers])
        qb = torch.cat([L["q"] for L in layers])
        iqb = torch.cat([L["iq"] for L in layers])
        posb = torch.cat([L["pos"] for L in layers])
        bb = batched.concat_buckets([L["buckets"] for L in layers])
        bgraph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            batched.batched_decode(qb, kb, vb, iqb, posb, bb, pcfg, scale)
            stream.synchronize()
        with torch.cuda.graph(bgraph, stream=stream):
            for _ in range(args.steps):
                batched.batched_decode(qb, kb, vb, iqb, posb, bb, pcfg, scale)
        ms_batch = timed(bgraph) / args.steps
        del kb, vb, bgraph

        # index maintenance on layer 0's keys: a decode appends one position per step and a
        # cluster block closes every 512 of them; the incremental index builds only that block
        # (and any node block it completes) - against the full rebuild of the 32k index
        from lsa_b200.incremental import IndexState
        from lsa_b200.index_space import index_keys

        ik0 = index_keys(layers[0]["k"][0])
        blk = CFG["cluster_block_size"]
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            st_ix = IndexState(ik0.shape[1], pcfg, dev)
            at = T_CTX - 4 * blk
            st_ix.append(ik0[:at])
            close_us, open_us = [], []
            for _ in range(4):  # four block closes: positions up to the close, then the closing one
                stream.synchronize()
                ev0.record(stream)
                for i in range(at, at + blk - 1):
                    st_ix.append(ik0[i:i + 1])
                ev1.record(stream)
                stream.synchronize()
                open_us.append(ev0.elapsed_time(ev1) * 1e3 / (blk - 1))
                ev0.record(stream)
                st_ix.append(ik0[at + blk - 1:at + blk])
                ev1.record(stream)
                stream.synchronize()
                close_us.append(ev0.elapsed_time(ev1) * 1e3)
                at += blk
            ev0.record(stream)
            for _ in range(3):
                fb = lsa.build_buckets_gpu(ik0, pcfg)
                lsa.build_hierarchy_gpu(ik0, fb, pcfg)
            ev1.record(stream)
            stream.synchronize()
            us_rebuild = ev0.elapsed_time(ev1) / 3 * 1e3
        index_maint = {"us_per_block_close": round(sorted(close_us)[len(close_us) // 2], 1),
                       "us_per_open_append": round(sorted(open_us)[len(open_us) // 2], 2),
                       "us_full_rebuild_32k": round(us_rebuild, 1), "block_closes": len(close_us),
                       "note": "host-driven eager appends on layer 0's keys; a close builds one 512-position "
                               "block (and any node block it completes)"}
        del ik0, st_ix

    hbm, tflops, peak_kind = _load_peaks()
    read_gbs = read_bytes_per_launch / (us_read * 1e-6) / 1e9
    fused_impl = args.decode_impl != "split"
    if fused_impl:  # the step is one fused kernel per layer: its bytes over its time
        roof = {"bound": "hbm", "kernel": "lsa::fused_decode_kernel", "achieved": round(value / world, 1),
                "peak": hbm, "unit": "GB/s", "frac": round(value / world / hbm, 4), "peak_kind": peak_kind,
                "traffic": _traffic_from_profile("fused_decode_32k.md"),
                "bytes_per_launch": round(step_bytes / LAYERS)}
    else:
        roof = {"bound": "hbm", "kernel": "lsa::decode_read_kernel", "achieved": round(read_gbs, 1),
                "peak": hbm, "unit": "GB/s", "frac": round(read_gbs / hbm, 4), "peak_kind": peak_kind,
                "traffic": _traffic_from_profile("decode_read_32k.md"),
                "bytes_per_launch": round(read_bytes_per_launch)}
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded drift keys, N(0,1) q/v)",
        "config": decode_config(world, args.decode_impl),
        "timing": {**_dist(per_step), "note": "per step (LAYERS select+read pairs), this rank"},
        "gate": gate,
        "us_per_select_read": round(ms_per_step / LAYERS * 1e3, 3),
        "us_per_select_read_split": round(ms_split / args.steps / LAYERS * 1e3, 3),
        "us_per_select_read_fused": round(ms_fused / args.steps / LAYERS * 1e3, 3),
        "us_per_select": round(us_select, 3), "us_per_read": round(us_read, 3),
        "us_per_select_from_queries": round(ms_select_q / args.steps / LAYERS * 1e3, 3),
        "read_roofline": {"kernel": "lsa::decode_read_kernel", "achieved": round(read_gbs, 1), "unit": "GB/s",
                          "frac": round(read_gbs / hbm, 4)},
        "select_roofline": {"kernel": "lsa::select_decode_kernel", "unit": "GB/s",
                            "bytes_per_launch": round((centroid_bytes + members_bytes) / LAYERS),
                            "achieved": round((centroid_bytes + members_bytes) / LAYERS / (us_select * 1e-6) / 1e9, 1),
                            "frac": round((centroid_bytes + members_bytes) / LAYERS / (us_select * 1e-6) / 1e9 / hbm,
                                          4)},
        "dense_us_per_decode": round(us_dense, 3),
        "batch_decode": None if ms_batch != ms_batch else {
            "sequences": LAYERS, "us_per_batch": round(ms_batch * 1e3, 2), "gbs": round(step_bytes / (ms_batch * 1e-3) / 1e9, 1),
            "hbm_frac": round(step_bytes / (ms_batch * 1e-3) / 1e9 / hbm, 4),
            "note": "the LAYERS caches decoded as one batch (batched select + batched read)"},
        "index_maintenance": index_maint,
        "arms_us_per_decode": None if us_tree != us_tree else {
            "flat": round(ms_split / args.steps / LAYERS * 1e3, 3), "tree": round(us_tree, 3),
            "positional": round(us_positional, 3), "dense": round(us_dense, 3)},
        "speedup_vs_dense_decode": (round(us_dense / (ms_per_step / LAYERS * 1e3), 3)
                                    if us_dense == us_dense else None),
        "bytes_per_step": step_bytes, "keys_read_per_step": n_ids,
        "gpu_launches": args.steps * LAYERS * (1 if fused_impl else 2),
        "roofline": roof,
        "step_roofline_frac": round(value / world / hbm, 4),
        "e2e": None if e2e_ms != e2e_ms else {"value": round(world * step_bytes / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": int(q_host.numel() * 2),
                "d2h_bytes_per_step": int(out_host.numel() * 2), "cuda_graph": True,
                "eager_ms_per_step": round(e2e_eager_ms, 4),
                "eager_value": round(world * step_bytes / (e2e_eager_ms / 1e3) / 1e9, 2)},
        "clocks": clocks.summary(),
    }
    return result, layers


# --------------------------------------------------------------------------- prefill leg


def run_prefill(args, dev, dump=None):
    """cfg 3: prefill select+read at T tokens (default 32k), bf16, per-64-query-tile top-32.

    Times, on inputs resident in HBM (q 268 MB + K/V 134 MB at 32k, larger than L2, so
    no flush): the tile selection, the tensor-core prefill read, select+read together, and
    dense causal SDPA with the cuDNN backend forced. tok/s = T / (select+read time)."""
    import torch
    from torch.nn.attention import SDPBackend, sdpa_kernel

    import lsa_b200 as lsa
    from lsa_b200 import prefill, synthetic

    T = args.prefill_T
    q, k, v = synthetic.qkv(T, HQ, HKV, DH, SEED + 3, dev)
    pcfg = lsa.PortConfig(**CFG)
    iq, ik = lsa.make_index_space(q, k)
    buckets = lsa.build_buckets_gpu(ik, pcfg)
    scale = DH ** -0.5
    stream = torch.cuda.Stream(dev)

    def timed(fn, reps):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                fn()
            stream.synchronize()
            ev0.record(stream)
            for _ in range(reps):
                fn()
            ev1.record(stream)
            stream.synchronize()
        return ev0.elapsed_time(ev1) / reps

    with torch.cuda.stream(stream):
        tl, tn = prefill.tile_select(iq, buckets, pcfg)
        stream.synchronize()
    reps = max(args.steps, 1)
    ms_select = timed(lambda: prefill.tile_select(iq, buckets, pcfg), reps)
    ms_read = timed(lambda: prefill.sparse_prefill(q, k, v, tl, tn, pcfg.cluster_block_size, scale), reps)
    with ClockSampler(dev.index) as clocks:
        ms_total = timed(lambda: prefill.lsa_prefill(q, k, v, iq, buckets, pcfg, scale), reps)
    status = prefill.status(dev)
    # algorithmic work: every row's keys = its tile's list + its open block [bs, t]
    rows = torch.arange(T, device=dev)
    keys_per_row = tn.long()[rows // 64] + (rows % pcfg.cluster_block_size) + 1
    total_keys = int(keys_per_row.sum().item())
    flops = 4 * DH * HQ * total_keys
    dense_flops = 4 * DH * HQ * T * (T + 1) // 2
    ms_dense = float("nan")
    if not args.quick:
        qt, kt, vt = (x.transpose(1, 2) for x in (q, k, v))

        def dense():
            with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                return torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=True, scale=scale,
                                                                        enable_gqa=True)

        ms_dense = timed(dense, max(2, reps // 2))
    if dump is not None and T >= 64 * 401:  # the CPU baseline's sample: a tile in the last quarter
        import numpy as np

        t = 400
        path = os.path.join(dump["dir"], "prefill.npz")
        np.savez(path, **_np_buckets(buckets), iq=iq.float().cpu().numpy(),
                 q=q[:, t * 64:(t + 1) * 64].float().cpu().numpy(), k=k.float().cpu().numpy(),
                 v=v.float().cpu().numpy(), tile=np.int64(t))
        dump["prefill"] = path
    hbm, tflops, peak_kind = _load_peaks()
    achieved = flops / (ms_read * 1e-3) / 1e12
    return {
        "workload": f"prefill{T // 1024}k", "tokens": T, "heads_q": HQ, "heads_kv": HKV, "head_dim": DH,
        "tile_queries": 64, "top_p_buckets_per_tile": CFG["top_p"], "budget_tokens": CFG["top_k"],
        "sink": CFG["sink_size"], "l2": "no flush: q + K/V of one step exceed L2",
        "tok_per_s": round(T / (ms_total * 1e-3), 1),
        "ms_select_read": round(ms_total, 4), "ms_select": round(ms_select, 4), "ms_read": round(ms_read, 4),
        "ms_dense_cudnn": round(ms_dense, 4) if ms_dense == ms_dense else None,
        "dense_tok_per_s": round(T / (ms_dense * 1e-3), 1) if ms_dense == ms_dense else None,
        "speedup_vs_dense": round(ms_dense / ms_total, 3) if ms_dense == ms_dense else None,
        "keys_read": total_keys, "flops": flops, "dense_flops": dense_flops, "status": status,
        "roofline": {"bound": "tensor", "kernel": "lsa::sparse_prefill_kernel", "achieved": round(achieved, 1),
                     "peak": tflops, "unit": "TFLOP/s", "frac": round(achieved / tflops, 4), "peak_kind": peak_kind,
                     "traffic": _traffic_from_profile("sparse_prefill_32k.md")},
        "clocks": clocks.summary(),
        "gpu_launches_per_step": 3,  # tile queries, the one-CTA-per-tile fused select, the tcgen05 read
    }


# --------------------------------------------------------------------------- batched 128k decode


BATCH_CFG = dict(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=64, top_k=4096,
                 window_size=64, sink_size=4)


def run_batched(args, rank, world, dev, mode=None, dump=None):
    """cfg 4: B = 64 sequences, lengths ~ U[65536, 131072] (seeded), Hq 64 / Hkv 8 / Dh 128,
    bf16, q/k/v ~ N(0, 1), top-64 buckets (4096-token budget), window 64, sinks 4.
    Sharding (total work fixed -> "strong"):
      heads (default, the configuration's own): rank r holds KV heads [r Hkv/N, (r+1) Hkv/N)
        of all 64 sequences and the index of its share of the sequences; it selects that
        share, one NCCL all-gather gives every rank every sequence's read list, and it reads
        its heads of all sequences (batched.head_sharded_select);
      heads_replicated: as heads, but every rank holds the whole index and selects for all
        64 sequences (no collective; the selection is repeated on every rank);
      sequences: rank r owns sequences shard_rows(64, N, r) with all their heads.
    A step = one token for every sequence: select (+ the gather) + one read launch,
    replayed from a CUDA graph. One step reads ~1.1 GB of K/V at N = 1 (> L2): no flush."""
    import torch

    import lsa_b200 as lsa
    from lsa_b200 import batched, seqshard
    from lsa_b200.index_space import index_keys, index_queries

    mode = mode or args.batched_shard
    B, HQB = args.batched_seqs, 64
    len_lo, len_hi = (int(x) for x in args.batched_len.split(","))
    if mode != "sequences" and HKV % world:
        raise ValueError(f"head sharding needs {HKV} KV heads to divide over {world} ranks")
    if mode == "heads" and B % world:
        mode = "heads_replicated"  # equal selection shares are needed for the all-gather
    gen = torch.Generator(device="cpu")
    gen.manual_seed(SEED + 4)
    lengths_all = torch.randint(len_lo, len_hi + 1, (B,), generator=gen).tolist()
    seq0, seq1 = (0, B) if mode != "sequences" else batched.shard_rows(B, world, rank)  # K/V held
    sel0, sel1 = batched.shard_rows(B, world, rank) if mode != "heads_replicated" else (0, B)  # selected
    h0, h1 = (rank * HKV // world, (rank + 1) * HKV // world) if mode != "sequences" else (0, HKV)
    lengths = lengths_all[seq0:seq1]
    G = HQB // HKV
    pcfg = lsa.PortConfig(**BATCH_CFG)
    Tmax = max(lengths) if lengths else 1
    nb = len(lengths)
    q = torch.empty(nb, 1, (h1 - h0) * G, DH, dtype=torch.bfloat16, device=dev)
    k = torch.empty(nb, Tmax, h1 - h0, DH, dtype=torch.bfloat16, device=dev)
    v = torch.empty(nb, Tmax, h1 - h0, DH, dtype=torch.bfloat16, device=dev)
    iqs, per_seq = [], []
    for i, L in enumerate(lengths):  # per sequence (seeded by the sequence, not the rank)
        sid = seq0 + i
        g = torch.Generator(device=dev)
        g.manual_seed(SEED + 4 + 1000 * sid)
        qf = torch.randn(1, HQB, DH, generator=g, device=dev).to(torch.bfloat16)
        kf = torch.randn(Tmax, HKV, DH, generator=g, device=dev).to(torch.bfloat16)
        q[i] = qf[:, h0 * G:h1 * G]
        k[i] = kf[:, h0:h1]
        v[i] = torch.randn(Tmax, HKV, DH, generator=g, device=dev).to(torch.bfloat16)[:, h0:h1]
        if sel0 <= sid < sel1:
            iqs.append(index_queries(qf, HKV))
            per_seq.append(lsa.build_buckets_gpu(index_keys(kf[:L]), pcfg))
        del kf
    iq = torch.cat(iqs)
    bb = batched.concat_buckets(per_seq)
    pos = torch.tensor([L - 1 for L in lengths_all[sel0:sel1]], dtype=torch.int32, device=dev)
    if dump is not None and world == 1:  # the CPU baseline's sample: sequence 0, the rows its list reads
        import numpy as np

        l0, n0 = lsa.flat_select(iq[:1], pos[:1], per_seq[0], pcfg)
        ids = l0[0, : int(n0[0])]
        rows = torch.unique(ids[ids >= 0]).long()
        path = os.path.join(dump["dir"], "batched.npz")
        np.savez(path, **_np_buckets(per_seq[0]), iq=iq[:1].cpu().numpy(), pos=pos[:1].cpu().numpy(),
                 q=q[:1].float().cpu().numpy(), k=k[:1, rows].float().cpu().numpy(),
                 v=v[:1, rows].float().cpu().numpy(), rows=rows.cpu().numpy().astype(np.int64))
        vis0 = min((lengths_all[0] - 1) // 512 * 8, per_seq[0].rows)
        nbytes = (vis0 * HKV * DH * 2 + pcfg.top_p * pcfg.bucket_cap * 4 + int(n0[0]) * HKV * DH * 2 * 2
                  + HQB * DH * 2 * 2)
        dump["batched"] = (path, nbytes)
    del per_seq
    scale = DH ** -0.5
    stream = torch.cuda.Stream(dev)
    hkv_r = h1 - h0
    gather, exchange = exchange_fn(world)

    def select():
        if mode == "heads":
            return batched.head_sharded_select(iq, pos, bb, pcfg, gather)
        return batched.batched_select(iq, pos, bb, pcfg)

    def step():
        lists, lens = select()
        return lsa.lsa_read(q, k, v, lists[:, None], lens[:, None], scale)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        lists, lens = select()
        stream.synchronize()
    n_ids = int(lens.long().sum().item())
    own = lengths_all[sel0:sel1]
    vis = [min((L - 1) // 512 * 8, int(r)) for L, r in zip(own, bb.table_rows.tolist())]
    # the selection's bytes count once per step over the job (a replicated selection is not
    # extra work): the rows this rank selects, except replicas beyond rank 0
    sel_bytes = sum(vis) * HKV * DH * 2 + len(own) * pcfg.top_p * pcfg.bucket_cap * 4 + len(own) * lists.shape[1] * 4
    if mode == "heads_replicated" and rank != 0:
        sel_bytes = 0
    step_bytes = sel_bytes + n_ids * hkv_r * DH * 2 * 2 + nb * (hkv_r * G * DH * 2 * 2 + HKV * DH * 4)

    def graph_of(fn, n):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn()
            stream.synchronize()
        with torch.cuda.graph(gr, stream=stream):
            for _ in range(n):
                fn()
        return gr

    graph = graph_of(step, 1)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        with ClockSampler(dev.index) as clocks:
            evs[0].record(stream)
            for i in range(args.steps):
                graph.replay()
                evs[i + 1].record(stream)
            stream.synchronize()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    ms = evs[0].elapsed_time(evs[-1]) / args.steps
    per_step = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    del graph

    def graph_ms(fn):
        gr = graph_of(fn, args.steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            gr.replay()
            if world > 1:
                stream.synchronize()
                torch.distributed.barrier()
            e0.record(stream)
            gr.replay()
            e1.record(stream)
            stream.synchronize()
        del gr
        return e0.elapsed_time(e1) / args.steps

    us_select = graph_ms(select) * 1e3
    us_read = graph_ms(lambda: lsa.lsa_read(q, k, v, lists[:, None], lens[:, None], scale)) * 1e3
    tot = torch.tensor([ms, float(step_bytes), float(len(own) if mode != "heads_replicated" else nb)], device=dev,
                       dtype=torch.float64)
    if world > 1:
        t_max = tot[:1].clone()
        torch.distributed.all_reduce(t_max, op=torch.distributed.ReduceOp.MAX)
        sums = tot[1:].clone()
        torch.distributed.all_reduce(sums)
        ms, all_bytes, all_seqs = float(t_max.item()), float(sums[0].item()), int(sums[1].item())
        if mode == "heads_replicated":
            all_seqs = B
    else:
        all_bytes, all_seqs = float(step_bytes), B
    hbm, tflops, peak_kind = _load_peaks()
    value = all_bytes / (ms * 1e-3) / 1e9
    # the dominant kernel: the read (persistent grid from 16 (row, KV head) units up)
    read_bytes = n_ids * hkv_r * DH * 2 * 2 + nb * hkv_r * G * DH * 2 * 2 + n_ids * 4
    persist = nb * hkv_r >= 16
    read_gbs = read_bytes / (us_read * 1e-6) / 1e9
    prof = _traffic_from_profile("sparse_read_persist_batched.md")
    traffic = None
    if prof is not None and persist:  # the profiled launch's DRAM bytes per algorithmic byte, at this size
        ratio = _profile_field("sparse_read_persist_batched.md", "traffic_per_algorithmic_byte")
        traffic = round(read_bytes * ratio) if ratio else None
    roof = {"bound": "hbm", "kernel": "lsa::sparse_read_persist_kernel" if persist else "lsa::sparse_read_kernel",
            "achieved": round(read_gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(read_gbs / hbm, 4),
            "peak_kind": peak_kind, "traffic": traffic, "bytes_per_launch": int(read_bytes)}
    return {
        "metric": f"batched decode select+read GB/s @128k bf16 ({B} sequences)", "value": round(value, 2),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic (seeded N(0,1) q/k/v, lengths U[{len_lo}, {len_hi}])",
        "config": {"workload": "batched128k", "batch": B, "sequences_selected_per_rank": len(own),
                   "sequences_read_per_rank": nb, "heads_q": HQB, "heads_kv": HKV, "heads_kv_per_rank": hkv_r,
                   "head_dim": DH, "top_p_buckets": BATCH_CFG["top_p"], "budget_tokens": BATCH_CFG["top_k"],
                   "lengths": [len_lo, len_hi],
                   "parallelism": {"heads": f"kv-head-shard{world} (selection split + {exchange} all-gather of the lists)",
                                   "heads_replicated": f"kv-head-shard{world} (selection replicated)",
                                   "sequences": f"sequence-shard{world}"}[mode],
                   "l2": "no flush: one step reads > 1 GB of K/V"},
        "us_per_step": round(ms * 1e3, 2), "us_select": round(us_select, 2), "us_read": round(us_read, 2),
        "timing": {**_dist(per_step), "note": "per step, rank 0"},
        "sequences": all_seqs, "bytes_per_step": int(all_bytes),
        "roofline": roof,
        # per step: the selection - one launch, or two (streaming scorer + per-row finish) when
        # the widest row has more than 1024 buckets - and the read
        "gpu_launches": args.steps * (1 + (2 if bb.max_rows > 1024 or len(own) * bb.max_rows >= 8192 else 1)),
        "step_roofline_frac": round(value / (world * hbm), 4), "peak_kind": peak_kind,
        "clocks": clocks.summary(),
    }


# --------------------------------------------------------------------------- tree 1M decode


TREE_CFG = dict(cluster_block_size=1024, pool_size=8, bucket_size=128, bucket_cap=256, top_p=64, top_k=8192,
                window_size=128, sink_size=4, node_bucket_size=16, top_level=2, node_cluster_block_size=64,
                beam_width=64)


def run_tree1m(args, rank, world, dev, dump=None):
    """cfg 5: B = 4 sequences of 1,048,576 tokens, Hq 32 / Hkv 8 / Dh 128, bf16, drift keys,
    128-token buckets (8 per 1024-token block), nodes of 16 buckets, two levels, beam 64,
    top-64 buckets (8192-token budget), window 128, sinks 4; pools of 8 (a 1024-token block
    of pools of 4 would exceed the Ward merge's 128 pools). Each rank holds a contiguous,
    block-aligned 1/N of every sequence and its shard index; a step decodes one token per
    sequence through lsa_b200.seqshard (candidate all-gather, best-first merge, partial
    reads, log-sum-exp merge over NCCL). Total work fixed -> "strong". Two independent sets
    of queries and caches alternate step by step, so a step's ~136 MB of listed K/V rows is
    not left in L2 by the step before. Each set's step is one CUDA graph (holding the NCCL
    all-gathers when N > 1), timed with CUDA events, max over ranks."""
    import torch

    import lsa_b200 as lsa
    from lsa_b200 import seqshard, synthetic
    from lsa_b200.index_space import index_keys, index_queries

    B, C = 4, args.tree_ctx
    pcfg = lsa.PortConfig(**TREE_CFG)
    s0, s1 = seqshard.shard_bounds(C, world, rank, TREE_CFG["cluster_block_size"])
    n = s1 - s0
    gather, exchange = exchange_fn(world)
    # the index build's one-time exchanges (member tables, MBs) go through NCCL
    build_gather = seqshard.all_gather_fn() if world > 1 else (lambda x: x[None])
    pos = torch.full((1,), C - 1, dtype=torch.int32, device=dev)
    scale = DH ** -0.5
    sets = []
    for which in range(2):
        g = torch.Generator(device=dev)
        g.manual_seed(SEED + 5 + 100 * which + rank)
        q = torch.randn(B, 1, HQ, DH, generator=g, device=dev).to(torch.bfloat16)
        k = torch.empty(B, n, HKV, DH, dtype=torch.bfloat16, device=dev)
        v = torch.empty(B, n, HKV, DH, dtype=torch.bfloat16, device=dev)
        shards = []
        for b in range(B):
            k[b] = synthetic.drift_keys(n, HKV, DH, g, dev)[0].to(torch.bfloat16)
            v[b] = torch.randn(n, HKV, DH, generator=g, device=dev).to(torch.bfloat16)
            si = seqshard.build_shard_index(index_keys(k[b]), s0, pcfg)
            rows = build_gather(torch.tensor([si.buckets.rows], dtype=torch.int64, device=dev))[:, 0].tolist()
            mine = seqshard.local_global_members(si)
            padded = torch.full((max(rows), mine.shape[1]), -1, dtype=torch.int32, device=dev)
            padded[: mine.shape[0]] = mine
            tables = build_gather(padded)
            si.bucket_offset = sum(rows[:rank])
            si.members_global = torch.cat([tables[r][: rows[r]] for r in range(len(rows))]).contiguous()
            shards.append(si)
        # a 1-GPU run holds the whole sequence: its queries decode the last position
        iq = [index_queries(q[b], HKV) for b in range(B)]
        sets.append((q, k, v, iq, shards))

    if dump is not None and world == 1:  # the CPU baseline's sample: sequence 0 of set 0, its list's rows
        import numpy as np

        q0, k0, v0, iq0, sh0 = sets[0]
        si = sh0[0]
        l0, n0 = lsa.tree_select(iq0[0], pos, si.buckets, si.hierarchy, pcfg)
        ids = l0[0, : int(n0[0])]
        rows = torch.unique(ids[ids >= 0]).long()
        lv = {}
        for i, level in enumerate(si.hierarchy.levels):
            lv[f"lc{i}"] = level.centroids.float().cpu().numpy()
            lv[f"lk{i}"] = level.children.cpu().numpy().astype(np.int64)
            lv[f"ls{i}"] = level.key_sums.float().cpu().numpy()
        path = os.path.join(dump["dir"], "tree.npz")
        np.savez(path, **_np_buckets(si.buckets), **lv, nlev=np.int64(len(si.hierarchy.levels)),
                 iq=iq0[0].cpu().numpy(), pos=pos.cpu().numpy(), q=q0[:1].float().cpu().numpy(),
                 k=k0[:1, rows].float().cpu().numpy(), v=v0[:1, rows].float().cpu().numpy(),
                 rows=rows.cpu().numpy().astype(np.int64))
        dump["tree"] = path

    def step(which):  # all sequences' candidates in one all-gather, one partial read, all partials in a second
        q, k, v, iq, shards = sets[which]
        if world == 1:  # one GPU holds every sequence whole: nothing to exchange
            return seqshard.one_shard_decode_batch(q, k, v, iq, pos, shards, pcfg, scale)
        return seqshard.seqshard_decode_batch(q, k, v, iq, pos, shards, pcfg, gather, scale)

    for _ in range(args.warmup):
        step(0)
        step(1)
    torch.cuda.synchronize(dev)
    # each set's step captured in a CUDA graph (the step is a chain of small launches:
    # replaying removes the host's launch overhead); with several ranks the graph holds the
    # two all-gathers too
    use_graph = not args.tree_eager
    graphs = [None, None]
    stream = torch.cuda.Stream(dev)
    if use_graph:
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            for which in range(2):
                step(which)
                stream.synchronize()
                graphs[which] = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graphs[which], stream=stream):
                    step(which)
        torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with torch.cuda.stream(stream), ClockSampler(dev.index) as clocks:
        evs[0].record(stream)
        for i in range(args.steps):
            if graphs[i % 2] is not None:
                graphs[i % 2].replay()
            else:
                step(i % 2)
            evs[i + 1].record(stream)
        stream.synchronize()
    torch.cuda.synchronize(dev)
    ms = evs[0].elapsed_time(evs[-1]) / args.steps
    per_step = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    del graphs  # a graph holding NCCL calls goes before the process group does
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    # algorithmic bytes of a step over all ranks: listed K/V rows + scored centroids (beam)
    width_ids = TREE_CFG["top_k"] + TREE_CFG["window_size"] + TREE_CFG["sink_size"]
    kv_bytes = B * width_ids * HKV * DH * 2 * 2
    levels_rows = sum(lv.centroids.shape[0] for si in sets[0][4] for lv in si.hierarchy.levels)
    cand_bytes = B * (TREE_CFG["beam_width"] * TREE_CFG["node_bucket_size"] * 2 + TREE_CFG["node_cluster_block_size"])
    cand_bytes *= HKV * DH * 4 * world
    step_bytes = kv_bytes + cand_bytes
    hbm, tflops, peak_kind = _load_peaks()
    value = step_bytes / (ms * 1e-3) / 1e9
    return {
        "metric": "tree decode select+read µs/step @1M bf16 (4 sequences)", "value": round(ms * 1e3, 2),
        "unit": "us/step", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded drift keys, N(0,1) q/v)",
        "config": {"workload": "tree1m", "batch": B, "context": C, "heads_q": HQ, "heads_kv": HKV, "head_dim": DH,
                   "shard_tokens": n, "parallelism": f"sequence-shard{world}", "exchange": f"{exchange} all-gather x2/step (candidates, partials)" if world > 1 else "none (one shard: the one-launch tree select per sequence, one read)",
                   "cuda_graph": use_graph, "rotation": "2 query/cache sets alternate step by step",
                   **{k2: TREE_CFG[k2] for k2 in ("bucket_size", "top_p", "top_k", "beam_width")},
                   "l2": "no flush: 2 sets of 4 x 1M-token caches (32 GiB) >> L2, consecutive steps read different sets"},
        "us_per_step": round(ms * 1e3, 2), "timing": {**_dist(per_step), "note": "per step, rank 0"},
        "effective_gbs": round(value, 2), "step_roofline_frac": round(value / (world * hbm), 4),
        "bytes_per_step": step_bytes, "hierarchy_nodes": levels_rows, "peak_kind": peak_kind,
        "clocks": clocks.summary(),
    }


# --------------------------------------------------------------------------- CPU baselines
#
# The CPU checker (oracle/: C + numpy, single-threaded per process) timed on this box's host
# cores: one spawn worker per core, every worker running the same bounded sample, so the
# rate is cores x one worker's rate. Samples are saved as .npz by the GPU legs (the index
# built by the GPU build kernels, bit-identical to the checker's own build - the parity
# tests pin that); the timed work is the configuration's select + read on the checker.
# K/V of the long-context configurations (128k, 1M) are saved as the rows the row's list
# reads (ids remapped to them), so a worker holds megabytes instead of gigabytes; the read's
# row count and arithmetic are the configuration's.


def _cpu_worker(payload):
    """One worker: `n` samples of one configuration on the checker -> (seconds, n, info)."""
    import numpy as np

    from oracle import oracle as O

    kind, path, n = payload
    blob = dict(np.load(path))
    t0 = time.perf_counter()
    info = 0
    for _ in range(n):
        if kind == "cfg1":  # the whole decode on the checker, ctx 2048 fp32
            cfg = O.Config(**CFG1)
            ob = O.Buckets(blob["cf"], blob["cb"], blob["members"], blob["sizes"], blob["sums"])
            lists, lengths = O.flat_select(blob["iq"], blob["pos"], ob, cfg, score_dtype="fp32")
            O.sparse_read(blob["q"], blob["k"], blob["v"], lists[None], lengths[None], blob["scale"].item())
            info = int(lengths[0])
        elif kind == "decode32k":
            ob = O.Buckets(blob["cf"], blob["cb"], blob["members"], blob["sizes"], blob["sums"])
            lists, lengths = O.flat_select(blob["iq"], np.array([T_CTX - 1]), ob, O.Config(**CFG))
            O.sparse_read(blob["q"], blob["k"], blob["v"], lists[None], lengths[None], DH ** -0.5)
            info = int(lengths[0])
        elif kind == "prefill":  # the select of every tile, then the read of one tile's rows
            cfg = O.Config(**CFG)
            ob = O.Buckets(blob["cf"], blob["cb"], blob["members"], blob["sizes"], blob["sums"])
            tl, tn = O.tile_select(blob["iq"], ob, cfg, 64)
            t = int(blob["tile"])
            rl, rn = O.prefill_row_lists(tl, tn, (t + 1) * 64, cfg, 64)
            O.sparse_read(blob["q"], blob["k"], blob["v"], rl[None, t * 64:], rn[None, t * 64:], DH ** -0.5)
            info = int(rn[t * 64:].sum())
        elif kind in ("batched", "tree"):
            cfg = O.Config(**(BATCH_CFG if kind == "batched" else TREE_CFG))
            ob = O.Buckets(blob["cf"], blob["cb"], blob["members"], blob["sizes"], blob["sums"])
            if kind == "batched":
                lists, lengths = O.flat_select(blob["iq"], blob["pos"], ob, cfg)
            else:
                levels = [O.Level(blob[f"lc{i}"], blob[f"lk{i}"], blob[f"ls{i}"]) for i in range(int(blob["nlev"]))]
                lists, lengths = O.tree_select(blob["iq"], blob["pos"], ob, O.Hierarchy(levels), cfg)
            # the read over the saved rows: ids remapped to their row in the saved K/V
            rows = blob["rows"]
            local = np.where(lists >= 0, np.searchsorted(rows, np.maximum(lists, 0)), -1).astype(np.int32)
            O.sparse_read(blob["q"], blob["k"], blob["v"], local[None], lengths[None], DH ** -0.5)
            info = int(lengths[0])
    return time.perf_counter() - t0, n, info


def _pool_rate(kind, path, seconds=8.0, cores=None):
    """Time `kind` on every host core for about `seconds`: (samples per second, cores, info, s/sample)."""
    import multiprocessing as mp

    cores = cores or os.cpu_count() or 1
    dt1, _, info = _cpu_worker((kind, path, 1))  # one sample in this process: the per-worker size
    per_worker = max(1, int(seconds / max(dt1, 1e-3)))
    ctx = mp.get_context("spawn")  # this process holds a CUDA context: never fork it
    with ctx.Pool(cores) as pool:
        pool.map(_cpu_worker, [(kind, path, 1)] * cores)  # imports and first touches, untimed
        res = pool.map(_cpu_worker, [(kind, path, per_worker)] * cores)
    # the workers run side by side: samples over the slowest worker's compute time (the
    # sample's file load is outside each worker's clock)
    n = sum(r[1] for r in res)
    return n / max(r[0] for r in res), cores, info, dt1


def _np_buckets(b):
    return dict(cf=b.centroids_f32.cpu().numpy(), cb=b.centroids.float().cpu().numpy(), members=b.members.cpu().numpy(),
                sizes=b.sizes.cpu().numpy(), sums=b.key_sums.cpu().numpy())


def _dump_layer_for_cpu(L, path):
    import numpy as np

    np.savez(path, **_np_buckets(L["buckets"]), iq=L["iq"].float().cpu().numpy(), q=L["q"].float().cpu().numpy(),
             k=L["k"].float().cpu().numpy(), v=L["v"].float().cpu().numpy())


def _bytes_per_select_read(length: int) -> int:
    """Algorithmic bytes of one decode select+read (same count as the B200 arm's step / LAYERS)."""
    visible = (T_CTX - 1) // CFG["cluster_block_size"] * (CFG["cluster_block_size"] // CFG["bucket_size"])
    width = CFG["top_k"] + CFG["window_size"] + CFG["sink_size"]
    return (visible * HKV * DH * 2 + CFG["top_p"] * CFG["bucket_cap"] * 4 + length * HKV * DH * 2 * 2
            + HQ * DH * 2 * 2 + HKV * DH * 2 + width * 4 * 2)


def cpu_baseline(path, seconds=10.0):
    """cfg 2 on the checker, every host core: the B200 line's cpu_baseline."""
    rate, cores, length, dt1 = _pool_rate("decode32k", path, seconds)
    return {"value": round(rate * _bytes_per_select_read(length) / 1e9, 4), "unit": "GB/s", "cores": cores,
            "kind": "port", "cpu_model": _lscpu_model(),
            "sample": f"decode32k select+read on the checker (oracle/, C + numpy), one spawn worker per core, "
                      f"{dt1 * 1e3:.1f} ms per select+read per worker, {rate:.2f} select+reads/s in all"}


CFG1 = dict(cluster_block_size=64, pool_size=4, bucket_size=64, bucket_cap=64, top_p=8, top_k=512, window_size=64,
            sink_size=0)


def _cfg1_sample(path):
    """cfg 1 (the reference's CPU-runnable case): ctx 2048, Hq 8 / Hkv 2 / Dh 64, fp32,
    64-token buckets, top-8 + the most recent bucket as the window; the index is built by
    the checker."""
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(SEED + 1)
    T, H, K, D = 2048, 8, 2, 64
    q = rng.standard_normal((1, T, H, D)).astype(np.float32)
    k = rng.standard_normal((1, T, K, D)).astype(np.float32)
    v = rng.standard_normal((1, T, K, D)).astype(np.float32)
    iq, ik = O.regroup(q[0], k[0])
    ob = O.build_buckets(ik, O.Config(**CFG1))
    np.savez(path, cf=ob.centroids_f32, cb=ob.centroids_bf16, members=ob.members, sizes=ob.sizes, sums=ob.key_sums,
             iq=iq[-1:], pos=np.array([T - 1], np.int32), q=q[:, -1:], k=k, v=v, scale=np.float32(D ** -0.5))


def cpu_baselines(tmp, samples: dict) -> dict:
    """configs 1, 3, 4, 5 on the checker (bounded samples, every host core)."""
    out = {"cpu_model": _lscpu_model()}
    p1 = os.path.join(tmp, "cfg1.npz")
    _cfg1_sample(p1)
    rate, cores, length, dt1 = _pool_rate("cfg1", p1, 4.0)
    out["cfg1_decode2k_fp32"] = {"value": round(dt1 * 1e6, 1), "unit": "us per select+read (one core)",
                                 "decodes_per_s": round(rate, 1), "cores": cores, "keys_read": length,
                                 "sample": "whole decode (select + read) of one query at ctx 2048 on the checker"}
    if "prefill" in samples:
        rate, cores, keys, dt1 = _pool_rate("prefill", samples["prefill"], 10.0)
        # one sample = the select of all 512 tiles + the read of one tile (64 rows): per tile,
        # a 512th of the select plus one tile's read
        out["cfg3_prefill32k"] = {"value": round(64 * rate, 1), "unit": "tok/s (lower estimate: the select of "
                                  "all 512 tiles is repeated in every 64-row sample)", "cores": cores,
                                  "sample": "tile select of all 512 tiles + the read of one 64-row tile per sample "
                                            f"({dt1:.2f} s per sample per worker); tok/s = 64 x samples/s"}
    if "batched" in samples:
        path, nbytes = samples["batched"]
        rate, cores, length, dt1 = _pool_rate("batched", path, 8.0)
        out["cfg4_batched128k"] = {"value": round(rate * nbytes / 1e9, 4), "unit": "GB/s", "cores": cores,
                                   "sequences_per_s": round(rate, 2),
                                   "sample": f"one 128k sequence's select + read (top-64, {length} ids, 8 KV heads) "
                                             f"per sample, {dt1 * 1e3:.1f} ms per worker"}
    if "tree" in samples:
        path = samples["tree"]
        rate, cores, length, dt1 = _pool_rate("tree", path, 8.0)
        out["cfg5_tree1m"] = {"value": round(4 / rate * 1e6, 1), "unit": "us per step (4 sequences, all cores)",
                              "cores": cores, "sample": f"one 1M-token sequence's tree select (2 levels, beam 64) + "
                              f"read of {length} ids per sample, {dt1 * 1e3:.1f} ms per worker; a step = 4 sequences"}
    return out


def run_reference(args, rank, world):
    """--impl reference: the CPU path of the reference for this workload, all host cores.

    The checker builds the index (oracle.build_buckets) and runs the select + read; this
    process loads no CUDA library of this repository. Same config as the B200 line."""
    if rank != 0:
        return None
    import tempfile

    import numpy as np

    from oracle import oracle as O

    O.build()
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "layer0.npz")
        g = np.random.default_rng(SEED + T_CTX)
        kk = O.bf16_round(g.standard_normal((T_CTX, HKV, DH)).astype(np.float32))
        vv = O.bf16_round(g.standard_normal((1, T_CTX, HKV, DH)).astype(np.float32))
        qq = O.bf16_round(g.standard_normal((1, HQ, DH)).astype(np.float32))
        _, ik = O.regroup(kk, kk)
        ob = O.build_buckets(ik, O.Config(**CFG))
        iq, _ = O.regroup(qq, kk[-1:])
        np.savez(path, cf=ob.centroids_f32, cb=ob.centroids_bf16, members=ob.members, sizes=ob.sizes, sums=ob.key_sums,
                 iq=O.bf16_round(iq), q=qq[None], k=kk[None], v=vv)
        cores = os.cpu_count() or 1
        samples, lengths = [], 0
        for i in range(args.warmup + args.steps):
            rate, cores, lengths, dt1 = _pool_rate("decode32k", path, 2.0, cores)
            if i >= args.warmup:
                samples.append(rate)
    rate = statistics.mean(samples)
    value = rate * _bytes_per_select_read(lengths) / 1e9
    ms_per_step = LAYERS / rate * 1e3  # a step of the B200 line: LAYERS select+reads
    return {"metric": METRIC, "value": round(value, 4), "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded drift keys, N(0,1) q/v)", "config": decode_config(world),
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                             "cpu_model": _lscpu_model(),
                             "sample": f"about 2 s of decode32k select+reads per worker per step, {cores} spawn "
                                       "workers, oracle/ (C + numpy), index built by the checker"},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# --------------------------------------------------------------------------- main


def main() -> int:
    global LAYERS
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", default="b200", choices=["b200", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--layers", type=int, default=LAYERS, help="independent 32k caches per step")
    parser.add_argument("--quick", action="store_true", help="skip e2e, dense and CPU legs (profiling runs)")
    parser.add_argument("--prefill-T", type=int, default=T_CTX, help="prefill leg tokens (0: skip the leg)")
    parser.add_argument("--only-prefill", action="store_true", help="run the prefill leg alone (profiling runs)")
    parser.add_argument("--workload", default="decode32k", choices=["decode32k", "batched128k", "tree1m"],
                        help="decode32k (default: + prefill leg), the 64-sequence 128k batched decode, or the "
                             "sequence-sharded 1M tree decode")
    parser.add_argument("--tree-ctx", type=int, default=1 << 20, help="tree1m context length")
    parser.add_argument("--tree-eager", action="store_true", help="tree1m: time eager launches, no CUDA graph")
    parser.add_argument("--decode-impl", default="split", choices=["split", "fused"],
                        help="decode32k step: the select and read launches (default), or one fused launch")
    parser.add_argument("--batched-seqs", type=int, default=64, help="batched128k sequences (profiling: fewer)")
    parser.add_argument("--batched-len", default="65536,131072",
                        help="batched128k sequence length range min,max (profiling: shorter)")
    parser.add_argument("--batched-shard", default="heads", choices=["heads", "heads_replicated", "sequences"],
                        help="batched128k over ranks: by KV head with the selection split (default) or "
                             "replicated, or by sequence")
    parser.add_argument("--no-sharded", action="store_true", help="skip the batched128k / tree1m legs")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    LAYERS = args.layers
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    import torch

    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return 0

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime

        # communicator set-up lines (ranks, devices, transports) on stderr, so a run's log
        # shows every rank joining; stdout keeps the one JSON line. A bare version request
        # (NCCL_DEBUG=VERSION, some launchers' default) is raised to the INIT lines.
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def finish(out):
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        if rank == 0 and out is not None:
            print(json.dumps(out), flush=True)
        return 0

    if args.workload in ("batched128k", "tree1m"):
        return finish((run_batched if args.workload == "batched128k" else run_tree1m)(args, rank, world, dev))
    if args.only_prefill:
        return finish(run_prefill(args, dev) if rank == 0 else None)
    import tempfile

    tmp = tempfile.TemporaryDirectory()
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline and not args.quick
    dump = {"dir": tmp.name} if want_cpu else None
    try:
        result, layers = run_b200(args, rank, world, dev)
    except GateError as e:
        print(f"bench: refusing to report: {e}", file=sys.stderr, flush=True)
        return 3
    if want_cpu:
        _dump_layer_for_cpu(layers[0], os.path.join(tmp.name, "layer0.npz"))
    del layers
    torch.cuda.empty_cache()
    if args.prefill_T > 0 and rank == 0 and world == 1:
        result["prefill"] = run_prefill(args, dev, dump)
        torch.cuda.empty_cache()
    if not args.no_sharded and not args.quick:
        # the configurations that shard, on every GPU count (their scaling rides in this line)
        split = run_batched(args, rank, world, dev, dump=dump)
        torch.cuda.empty_cache()
        result["sharded"] = {"batched128k": split}
        if world > 1:
            # head sharding two ways: the selection split over the ranks (+ one NCCL all-gather of
            # the lists) or repeated on every rank; the faster one heads the key, the other beside
            repl = run_batched(args, rank, world, dev, mode="heads_replicated")
            torch.cuda.empty_cache()
            best, other = (split, repl) if split["ms_per_step"] <= repl["ms_per_step"] else (repl, split)
            result["sharded"]["batched128k"] = best
            result["sharded"]["batched128k_other_head_sharding"] = other
        result["sharded"]["tree1m"] = run_tree1m(args, rank, world, dev, dump=dump)
        torch.cuda.empty_cache()
    result["cpu_baseline"] = None
    if want_cpu:
        result["cpu_baseline"] = cpu_baseline(os.path.join(tmp.name, "layer0.npz"))
        result["cpu_baselines"] = cpu_baselines(tmp.name, dump)
    tmp.cleanup()
    lsa_check = __import__("lsa_b200").check_status
    lsa_check(dev, "bench")  # no bounded wait expired anywhere in the run
    return finish(result)


if __name__ == "__main__":
    sys.exit(main())
