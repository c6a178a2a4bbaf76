"""Benchmark: LSA decode select+read at 32k context, bf16, on B200.

Workload ("decode32k"): B=1, one query token, Hq=32, Hkv=8, Dh=128, bf16, drift keys,
64-token buckets in 512-token cluster blocks (8 per block, cap 128, pools of 4), top-32
buckets (2048-token budget), window 64, sinks 4 - the D-LSA Flat arm through the fused
select (LSA_SELECT_IMPL=fused: one launch from index query to read lists) and the split-K
TMA-gather read. A STEP is one decoded token through LAYERS = 32 layers, each layer its
own independent 32k KV cache (4.3 GB of K/V in all), so one step touches 32 x ~9.7 MB,
more than twice the 126 MB L2, before any cache is revisited: no L2 flush is needed.
The select+read index (buckets) is built before timing, as in the reference's bench
(src/lsa_rocm_lab/port/bench.py:113-154 times select+read on a prebuilt index).

value = algorithmic bytes of the step / step time, in GB/s (whole job: summed over the
N replica ranks, max time over ranks); us_per_select_read = step time / LAYERS. The
device-timed region replays one CUDA graph of the K steps' kernels with inputs resident.
``e2e`` is the same metric through the public Python API with host buffers: every step
copies the 32 layers' query rows from pinned host memory, runs make_index_space +
flat_select + lsa_read per layer, and copies the outputs back - the step captured once in a
CUDA graph whose replays include both copies (``eager_*`` keys: the same step launched
eagerly from Python, host-bound).

``--impl reference`` times the reference's CPU path for this workload on the host cores:
the CPU checker (oracle/, a restatement of the reference's select + read; the reference's
own path needs the absent upstream package and a ROCm GPU) over a bounded sample of
select+reads per step, with one worker process per core.

Multi-GPU (--gpus N under torchrun): the decode of one sequence does not shard, so the N
ranks run independent replicas (scaling "weak"); no collective is on the data path.
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


# --------------------------------------------------------------------------- B200 arm


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
        stream.synchronize()
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

    # one graph holding K steps (LAYERS select+read pairs each)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(args.steps):
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

    with ClockSampler(dev.index) as clocks:
        ms_total = timed(graph)
    ms_read = timed(read_graph)
    ms_select = timed(select_graph)
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
            iq, _ = regroup_rows(qd[i, 0], k_last[i])
            if args.decode_impl == "split":
                lists, lengths = lsa.flat_select(iq, L["pos"], L["buckets"], pcfg)
                outs.append(lsa.lsa_read(qd[i], L["k"], L["v"], lists[None], lengths[None], scale))
            else:
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
            for _ in range(args.steps):
                e2e_step()
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
        roof = {"bound": "hbm", "kernel": "lsa::sparse_read_kernel", "achieved": round(read_gbs, 1),
                "peak": hbm, "unit": "GB/s", "frac": round(read_gbs / hbm, 4), "peak_kind": peak_kind,
                "traffic": _traffic_from_profile("sparse_read_decode32k.md"),
                "bytes_per_launch": round(read_bytes_per_launch)}
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded drift keys, N(0,1) q/v)",
        "config": {"workload": "decode32k", "layers_per_step": LAYERS, "context": T_CTX, "batch": 1,
                   "heads_q": HQ, "heads_kv": HKV, "head_dim": DH, "bucket_size": CFG["bucket_size"],
                   "top_p_buckets": CFG["top_p"], "budget_tokens": CFG["top_k"], "window": CFG["window_size"],
                   "sink": CFG["sink_size"], "decode_impl": args.decode_impl, "parallelism": f"replicas{world}",
                   "l2": "no flush: 32 independent 32k caches, each step touches 32 x ~9.7 MB > 2x L2"},
        "us_per_select_read": round(ms_per_step / LAYERS * 1e3, 3),
        "us_per_select_read_split": round(ms_split / args.steps / LAYERS * 1e3, 3),
        "us_per_select_read_fused": round(ms_fused / args.steps / LAYERS * 1e3, 3),
        "us_per_select": round(us_select, 3), "us_per_read": round(us_read, 3),
        "read_roofline": {"kernel": "lsa::sparse_read_kernel", "achieved": round(read_gbs, 1), "unit": "GB/s",
                          "frac": round(read_gbs / hbm, 4)},
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


def run_prefill(args, dev):
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


def run_batched(args, rank, world, dev):
    """cfg 4: B = 64 sequences, lengths ~ U[65536, 131072] (seeded), Hq 64 / Hkv 8 / Dh 128,
    bf16, q/k/v ~ N(0, 1), top-64 buckets (4096-token budget), window 64, sinks 4.
    Sharding (no collective either way; total work fixed -> "strong"):
      heads (default, the configuration's own): every rank holds all 64 sequences' index
        (centroids and members, replicated) and selects for all of them - the selection is
        shared by the heads - then reads only its Hkv / N KV heads (and their q heads);
      sequences: rank r owns sequences shard_rows(64, world, r) with all their heads.
    A step = one token for every sequence: one batched-select launch + one read launch,
    replayed from a CUDA graph. One step reads ~1.1 GB of K/V at N = 1 (> L2): no flush."""
    import torch

    import lsa_b200 as lsa
    from lsa_b200 import batched
    from lsa_b200.index_space import index_keys, index_queries

    B, HQB = args.batched_seqs, 64
    len_lo, len_hi = (int(x) for x in args.batched_len.split(","))
    by_heads = args.batched_shard == "heads"
    if by_heads and HKV % world:
        raise ValueError(f"head sharding needs {HKV} KV heads to divide over {world} ranks")
    gen = torch.Generator(device="cpu")
    gen.manual_seed(SEED + 4)
    lengths_all = torch.randint(len_lo, len_hi + 1, (B,), generator=gen).tolist()
    start, end = (0, B) if by_heads else batched.shard_rows(B, world, rank)
    lengths = lengths_all[start:end]
    h0, h1 = (rank * HKV // world, (rank + 1) * HKV // world) if by_heads else (0, HKV)
    G = HQB // HKV
    pcfg = lsa.PortConfig(**BATCH_CFG)
    Tmax = max(lengths) if lengths else 1
    nb = len(lengths)
    q = torch.empty(nb, 1, (h1 - h0) * G, DH, dtype=torch.bfloat16, device=dev)
    k = torch.empty(nb, Tmax, h1 - h0, DH, dtype=torch.bfloat16, device=dev)
    v = torch.empty(nb, Tmax, h1 - h0, DH, dtype=torch.bfloat16, device=dev)
    iqs, per_seq = [], []
    for i, L in enumerate(lengths):  # per sequence (seeded by the sequence, not the rank)
        g = torch.Generator(device=dev)
        g.manual_seed(SEED + 4 + 1000 * (start + i))
        qf = torch.randn(1, HQB, DH, generator=g, device=dev).to(torch.bfloat16)
        kf = torch.randn(Tmax, HKV, DH, generator=g, device=dev).to(torch.bfloat16)
        q[i] = qf[:, h0 * G:h1 * G]
        k[i] = kf[:, h0:h1]
        v[i] = torch.randn(Tmax, HKV, DH, generator=g, device=dev).to(torch.bfloat16)[:, h0:h1]
        iqs.append(index_queries(qf, HKV))
        per_seq.append(lsa.build_buckets_gpu(index_keys(kf[:L]), pcfg))
        del kf
    iq = torch.cat(iqs)
    bb = batched.concat_buckets(per_seq)
    del per_seq
    pos = torch.tensor([L - 1 for L in lengths], dtype=torch.int32, device=dev)
    scale = DH ** -0.5
    stream = torch.cuda.Stream(dev)
    hkv_r = h1 - h0

    def step():
        lists, lens = batched.batched_select(iq, pos, bb, pcfg)
        return lsa.lsa_read(q, k, v, lists[:, None], lens[:, None], scale)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        lists, lens = batched.batched_select(iq, pos, bb, pcfg)
        stream.synchronize()
    n_ids = int(lens.long().sum().item())
    vis = [min((L - 1) // 512 * 8, int(r)) for L, r in zip(lengths, bb.table_rows.tolist())]
    # the selection's bytes count once per step (replicated selections are not extra work)
    sel_bytes = sum(vis) * HKV * DH * 2 + nb * pcfg.top_p * pcfg.bucket_cap * 4 + nb * lists.shape[1] * 4
    if by_heads and rank != 0:
        sel_bytes = 0
    step_bytes = sel_bytes + n_ids * hkv_r * DH * 2 * 2 + nb * (hkv_r * G * DH * 2 * 2 + HKV * DH * 4)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(args.steps):
            step()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        stream.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        with ClockSampler(dev.index) as clocks:
            ev0.record(stream)
            graph.replay()
            ev1.record(stream)
            stream.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    del graph

    def graph_ms(fn):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for _ in range(args.steps):
                fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            gr.replay()
            e0.record(stream)
            gr.replay()
            e1.record(stream)
            stream.synchronize()
        return e0.elapsed_time(e1) / args.steps

    us_select = graph_ms(lambda: batched.batched_select(iq, pos, bb, pcfg)) * 1e3
    us_read = graph_ms(lambda: lsa.lsa_read(q, k, v, lists[:, None], lens[:, None], scale)) * 1e3
    tot = torch.tensor([ms, float(step_bytes), float(nb)], device=dev, dtype=torch.float64)
    if world > 1:
        t_max = tot[:1].clone()
        torch.distributed.all_reduce(t_max, op=torch.distributed.ReduceOp.MAX)
        sums = tot[1:].clone()
        torch.distributed.all_reduce(sums)
        ms, all_bytes, all_seqs = float(t_max.item()), float(sums[0].item()), int(sums[1].item())
    else:
        all_bytes, all_seqs = float(step_bytes), nb
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
        "config": {"workload": "batched128k", "batch": B, "sequences_per_rank": nb, "heads_q": HQB,
                   "heads_kv": HKV, "heads_kv_per_rank": hkv_r, "head_dim": DH, "top_p_buckets": BATCH_CFG["top_p"],
                   "budget_tokens": BATCH_CFG["top_k"],
                   "lengths": [len_lo, len_hi],
                   "parallelism": f"{'kv-head' if by_heads else 'sequence'}-shard{world}",
                   "l2": "no flush: one step reads > 1 GB of K/V"},
        "us_per_step": round(ms * 1e3, 2), "us_select": round(us_select, 2), "us_read": round(us_read, 2),
        "sequences": all_seqs, "bytes_per_step": int(all_bytes),
        # per step: the read, and the selection - one launch, or two (streaming scorer + per-row
        # finish) when the widest row has more than 1024 buckets (more than one cluster)
        "roofline": roof,
        "gpu_launches": args.steps * (1 + (2 if bb.max_rows > 1024 or nb * bb.max_rows >= 8192 else 1)),
        "step_roofline_frac": round(value / world / hbm, 4), "peak_kind": peak_kind,
        "clocks": clocks.summary(),
    }


# --------------------------------------------------------------------------- tree 1M decode


TREE_CFG = dict(cluster_block_size=1024, pool_size=8, bucket_size=128, bucket_cap=256, top_p=64, top_k=8192,
                window_size=128, sink_size=4, node_bucket_size=16, top_level=2, node_cluster_block_size=64,
                beam_width=64)


def run_tree1m(args, rank, world, dev):
    """cfg 5: B = 4 sequences of 1,048,576 tokens, Hq 32 / Hkv 8 / Dh 128, bf16, drift keys,
    128-token buckets (8 per 1024-token block), nodes of 16 buckets, two levels, beam 64,
    top-64 buckets (8192-token budget), window 128, sinks 4; pools of 8 (a 1024-token block
    of pools of 4 would exceed the Ward merge's 128 pools). Each rank holds a contiguous,
    block-aligned 1/N of every sequence and its shard index; a step decodes one token per
    sequence through lsa_b200.seqshard (candidate all-gather, best-first merge, partial
    reads, log-sum-exp merge over NCCL). Total work fixed -> "strong". Eager launches and
    collectives, timed with CUDA events, max over ranks."""
    import torch

    import lsa_b200 as lsa
    from lsa_b200 import seqshard, synthetic
    from lsa_b200.index_space import index_keys, index_queries

    B, C = 4, args.tree_ctx
    pcfg = lsa.PortConfig(**TREE_CFG)
    s0, s1 = seqshard.shard_bounds(C, world, rank, TREE_CFG["cluster_block_size"])
    n = s1 - s0
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 5 + rank)
    q = torch.randn(B, 1, HQ, DH, generator=g, device=dev).to(torch.bfloat16)
    k = torch.empty(B, n, HKV, DH, dtype=torch.bfloat16, device=dev)
    v = torch.empty(B, n, HKV, DH, dtype=torch.bfloat16, device=dev)
    gather = seqshard.all_gather_fn() if world > 1 else (lambda x: x[None])
    shards = []
    for b in range(B):
        k[b] = synthetic.drift_keys(n, HKV, DH, g, dev)[0].to(torch.bfloat16)
        v[b] = torch.randn(n, HKV, DH, generator=g, device=dev).to(torch.bfloat16)
        si = seqshard.build_shard_index(index_keys(k[b]), s0, pcfg)
        rows = gather(torch.tensor([si.buckets.rows], dtype=torch.int64, device=dev))[:, 0].tolist()
        mine = seqshard.local_global_members(si)
        padded = torch.full((max(rows), mine.shape[1]), -1, dtype=torch.int32, device=dev)
        padded[: mine.shape[0]] = mine
        tables = gather(padded)
        si.bucket_offset = sum(rows[:rank])
        si.members_global = torch.cat([tables[r][: rows[r]] for r in range(len(rows))]).contiguous()
        shards.append(si)
    # a 1-GPU run holds the whole sequence: its queries decode the last position
    iq = [index_queries(q[b], HKV) for b in range(B)]
    pos = torch.full((1,), C - 1, dtype=torch.int32, device=dev)
    scale = DH ** -0.5

    def step():  # all sequences' candidates in one all-gather, one partial read, all partials in a second
        return seqshard.seqshard_decode_batch(q, k, v, iq, pos, shards, pcfg, gather, scale)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    # one step captured in a CUDA graph (the step is a chain of small launches: replaying it
    # removes the host's launch overhead); with several ranks the graph holds the two NCCL
    # all-gathers too (measured at 2 GPUs: 365 us/step in the graph against 1008 us eager)
    use_graph = not args.tree_eager
    graph = None
    if use_graph:
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            step()
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step()
        torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        ev0.record()
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step()
        ev1.record()
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    del graph  # a graph holding NCCL calls goes before the process group does
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    # algorithmic bytes of a step over all ranks: listed K/V rows + scored centroids (beam)
    width_ids = TREE_CFG["top_k"] + TREE_CFG["window_size"] + TREE_CFG["sink_size"]
    kv_bytes = B * width_ids * HKV * DH * 2 * 2
    levels_rows = sum(lv.centroids.shape[0] for si in shards for lv in si.hierarchy.levels)
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
                   "shard_tokens": n, "parallelism": f"sequence-shard{world}", "exchange": "NCCL all-gather x2/step (candidates, partials)",
                   "cuda_graph": use_graph,
                   **{k2: TREE_CFG[k2] for k2 in ("bucket_size", "top_p", "top_k", "beam_width")},
                   "l2": "no flush: 4 x 1M-token caches (16 GiB) >> L2"},
        "effective_gbs": round(value, 2), "step_roofline_frac": round(value / world / hbm, 4),
        "bytes_per_step": step_bytes, "hierarchy_nodes": levels_rows, "peak_kind": peak_kind,
        "clocks": clocks.summary(),
    }


# --------------------------------------------------------------------------- CPU baseline


def _cpu_sample(payload):
    """One worker: time select+read on the checker for `n` decode rows of one cache."""
    import numpy as np

    from oracle import oracle as O

    path, n = payload
    blob = np.load(path)
    ob = O.Buckets(blob["cf"], blob["cb"], blob["members"], blob["sizes"], blob["sums"])
    cfg = O.Config(**CFG)
    t0 = time.perf_counter()
    length = 0
    for _ in range(n):
        lists, lengths = O.flat_select(blob["iq"], np.array([T_CTX - 1]), ob, cfg)
        O.sparse_read(blob["q"], blob["k"], blob["v"], lists[None], lengths[None], DH ** -0.5)
        length = int(lengths[0])
    return time.perf_counter() - t0, n, length


def _dump_layer_for_cpu(L, path):
    import numpy as np

    b = L["buckets"]
    np.savez(path, cf=b.centroids_f32.cpu().numpy(), cb=b.centroids.float().cpu().numpy(),
             members=b.members.cpu().numpy(), sizes=b.sizes.cpu().numpy(), sums=b.key_sums.cpu().numpy(),
             iq=L["iq"].float().cpu().numpy(), q=L["q"].float().cpu().numpy(), k=L["k"].float().cpu().numpy(),
             v=L["v"].float().cpu().numpy())


def _bytes_per_select_read(length: int) -> int:
    """Algorithmic bytes of one decode select+read (same count as the B200 arm's step / LAYERS)."""
    visible = (T_CTX - 1) // CFG["cluster_block_size"] * (CFG["cluster_block_size"] // CFG["bucket_size"])
    width = CFG["top_k"] + CFG["window_size"] + CFG["sink_size"]
    return (visible * HKV * DH * 2 + CFG["top_p"] * CFG["bucket_cap"] * 4 + length * HKV * DH * 2 * 2
            + HQ * DH * 2 * 2 + HKV * DH * 2 + width * 4 * 2)


def cpu_baseline(layer, seconds=10.0):
    """The checker's select+read on this box's host, single core: a bounded sample."""
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "layer0.npz")
        _dump_layer_for_cpu(layer, path)
        dt, n, _ = _cpu_sample((path, 1))
        reps = max(1, min(64, int(seconds / max(dt, 1e-3))))
        dt, n, length = _cpu_sample((path, reps))
    per = dt / n
    return {"value": round(_bytes_per_select_read(length) / per / 1e9, 4), "unit": "GB/s", "cores": 1,
            "kind": "port",
            "sample": f"{n} decode select+read on one 32k cache (oracle/, C + numpy), {per * 1e3:.2f} ms each"}


def run_reference(args, rank, world):
    """--impl reference: the CPU path of the reference for this workload, all host cores.

    The index is built on the GPU when one is visible (bit-identical to the checker's own
    build, which the parity tests pin), else by the checker; only select+read is timed."""
    if rank != 0:
        return None
    import multiprocessing as mp
    import tempfile

    import numpy as np
    import torch

    cores = os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "layer0.npz")
        if torch.cuda.is_available():
            import lsa_b200 as lsa
            from lsa_b200.index_space import regroup_rows
            from lsa_b200.synthetic import drift_keys

            dev = torch.device("cuda:0")
            gen = torch.Generator(device=dev)
            gen.manual_seed(SEED + T_CTX)
            k = drift_keys(T_CTX, HKV, DH, gen, dev).to(torch.bfloat16)
            v = torch.randn(1, T_CTX, HKV, DH, generator=gen, device=dev).to(torch.bfloat16)
            q = torch.randn(1, 1, HQ, DH, generator=gen, device=dev).to(torch.bfloat16)
            _, ik = regroup_rows(k[0], k[0])
            buckets = lsa.build_buckets_gpu(ik, lsa.PortConfig(**CFG))
            iq, _ = regroup_rows(q[0], k[0, -1:])
            _dump_layer_for_cpu(dict(k=k, v=v, q=q, iq=iq.to(torch.bfloat16), buckets=buckets), path)
        else:
            from oracle import oracle as O

            g = np.random.default_rng(SEED)
            kk = O.bf16_round(g.standard_normal((T_CTX, HKV, DH)).astype(np.float32))
            qq = O.bf16_round(g.standard_normal((1, HQ, DH)).astype(np.float32))
            _, ik = O.regroup(kk, kk)
            ob = O.build_buckets(ik, O.Config(**CFG))
            iq, _ = O.regroup(qq, kk[-1:])
            np.savez(path, cf=ob.centroids_f32, cb=ob.centroids_bf16, members=ob.members, sizes=ob.sizes,
                     sums=ob.key_sums, iq=O.bf16_round(iq), q=qq[None], k=kk[None],
                     v=O.bf16_round(g.standard_normal((1, T_CTX, HKV, DH)).astype(np.float32)))
        dt1, _, length = _cpu_sample((path, 1))
        per_worker = max(1, int(2.0 / max(dt1, 1e-3)))  # about 2 s of work per worker per step
        ctx = mp.get_context("spawn")
        with ctx.Pool(cores) as pool:
            samples = []
            for i in range(args.warmup + args.steps):
                t0 = time.perf_counter()
                res = pool.map(_cpu_sample, [(path, per_worker)] * cores)
                wall = time.perf_counter() - t0
                if i >= args.warmup:
                    samples.append((wall, sum(r[1] for r in res)))
    wall = sum(w for w, _ in samples)
    n_sr = sum(n for _, n in samples)
    value = n_sr * _bytes_per_select_read(length) / wall / 1e9
    ms_per_step = wall / len(samples) * 1e3
    return {"metric": METRIC, "value": round(value, 4), "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded)", "config": {"workload": "decode32k", "select_impl": "reference-cpu"},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{per_worker} decode select+read per worker per step, {cores} spawn "
                                       "workers, oracle/ (C + numpy)"},
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
    parser.add_argument("--batched-shard", default="heads", choices=["heads", "sequences"],
                        help="batched128k over ranks: by KV head (selection replicated) or by sequence")
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

        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"  # keep stdout to the one JSON line

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if args.workload in ("batched128k", "tree1m"):
        out = (run_batched if args.workload == "batched128k" else run_tree1m)(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(out), flush=True)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return 0
    if args.only_prefill:
        if rank == 0:
            print(json.dumps(run_prefill(args, dev)), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    result, layers = run_b200(args, rank, world, dev)
    if args.prefill_T > 0 and rank == 0 and world == 1:
        del layers[1:]  # free the rotation's caches before the prefill leg
        torch.cuda.empty_cache()
        result["prefill"] = run_prefill(args, dev)
    if rank == 0:
        if not args.no_cpu_baseline and not args.quick and world == 1:
            result["cpu_baseline"] = cpu_baseline(layers[0])
        else:
            result["cpu_baseline"] = None
        print(json.dumps(result), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
