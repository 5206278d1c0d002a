"""Benchmark of the tree-sparse verify-attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

One JSON line on rank 0.  A "step" is one call of the hot path on one batch of
synthetic input: metadata build from the tree mask + prefix sweep + CSR tree
walk + normalise (``run_tree_sparse_kernel``'s work), for the workload that
the headline metric is quoted on (Llama-3-8B GQA shapes: B=1, 32 q-heads /
8 kv-heads, head_dim 128, prefix 4096, 64-node draft tree, BLOCK 64x64).

* ``value``: algorithmic HBM bytes of the whole problem (Q + K + V + O, each
  touched once) / device time per step.  With N GPUs the problem's (batch,
  kv-head) units are sharded over the ranks (``tsfa_shard``: contiguous
  balanced ranges, no collective on the path) -- strong scaling of one
  problem -- and the step time is the max over ranks.  Inputs are resident in
  HBM.  The K timed steps run back to back from CUDA graphs between one pair
  of CUDA events, cycling over enough input sets (> 1.5x the 126 MB L2 per
  rank) that every step reads its inputs from HBM.  ``isolated`` gives the
  same op timed one step at a time (256 MB L2 flush, then an event pair).
* ``gather``: the optional NCCL all-gather of the output shards
  (``tsfa_shard.gather``), timed apart and not part of ``value``.
* ``e2e``: the same metric through the public API with host buffers: pinned
  host -> device copies of the rank's Q/K/V slices and the mask, the call, and
  a device -> host copy of the output, all inside the timed region, every
  step; the steps are pipelined over two sets of device buffers (one step's
  host -> device copies overlap the previous step's call and read-back), and
  the same steps on one stream are reported beside (``serial_us_per_call``);
  the copies and the call are also timed apart with CUDA events (``breakdown``).
* ``roofline``: the op's forward kernel alone (prebuilt metadata: the same
  instantiation and plan as in the op), timed with CUDA events on its
  launching stream, against the measured HBM copy bandwidth; ``tensor_frac``
  against the measured bf16 GEMM rate.
* ``configs``: the tensor-bound benchmark configurations 3 (batched serving,
  Llama-3-70B heads) and 4 (long context), sharded the same way: us/call,
  tokens/s, HBM and tensor fractions.
* ``comparators``: torch SDPA on the same input sets with the tree as an
  additive mask (a library kernel, not this package), timed the same way.
* ``cpu_baseline``: the numpy oracle (a restatement of the reference's
  dense+mask path and metadata builder) on the whole op, rank 0, N=1.
* ``--impl reference``: the reference's CPU path (same oracle port, whole
  op, every host core) on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "eagle3-tree-sparse-flashattn_b200"))

import tsfa_trees as trees  # noqa: E402

METRIC = "tree-attn fwd µs/call & achieved HBM TB/s, 8B-GQA prefix 4K tree 64"
L2_BYTES = 126 * 1000 * 1000
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0
SUBCONFIGS = ("cfg3_serving_70b", "cfg4_long_ctx")


def workload_bytes(c) -> int:
    B, Hq, Hkv, D, P, T = c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"]
    return 2 * B * Hq * T * D * 2 + 2 * 2 * B * Hkv * (P + T) * D


def workload_flops(c, mask) -> dict:
    B, Hq, D, P, T, BM, BN = c["B"], c["Hq"], c["D"], c["P"], c["T"], c["BM"], c["BN"]
    nqb, ntb = -(-T // BM), -(-T // BN)
    pad = np.zeros((nqb * BM, ntb * BN), bool)
    pad[:T, :T] = mask
    nnz = int(pad.reshape(nqb, BM, ntb, BN).any(axis=(1, 3)).sum())
    return {"prefix": 4 * B * Hq * T * P * D, "tree_executed": 4 * B * Hq * D * nnz * BM * BN,
            "tree_useful": 4 * B * Hq * D * int(mask.sum())}


def peaks():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured")
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_TFLOPS_SUSTAINED, "fallback"


def cpu_info():
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return model


def use_all_cores() -> int:
    """Every host core for the CPU legs (torchrun sets OMP_NUM_THREADS=1)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n)
    except Exception:
        pass
    try:
        import torch

        torch.set_num_threads(n)
    except Exception:
        pass
    return n


# --------------------------------------------------------------------------- CPU legs
def time_oracle(c, mask, seed: int, budget_s: float, min_reps: int = 2):
    """Oracle metadata build + dense+mask fp32 attention over the whole op,
    on host cores; returns (median seconds, bytes of the op, repetitions)."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import torch

    import tsfa_oracle as orc

    gen = torch.Generator().manual_seed(seed)
    B, Hq, Hkv, D, P, T = c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"]
    q = torch.randn((B, Hq, T, D), generator=gen).to(torch.bfloat16).float().numpy()
    k = torch.randn((B, Hkv, P + T, D), generator=gen).to(torch.bfloat16).float().numpy()
    v = torch.randn((B, Hkv, P + T, D), generator=gen).to(torch.bfloat16).float().numpy()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        orc.prepare_tree_sparse_metadata(mask, P, c["BM"], c["BN"])
        orc.dense_tree_attention(q, k, v, mask, P)
        times.append(time.perf_counter() - t0)
    return statistics.median(times), workload_bytes(c), len(times)


def run_reference_arm(args, c, mask, rank):
    if rank != 0:
        return
    cores = use_all_cores()
    model = cpu_info()
    for _ in range(args.warmup):
        time_oracle(c, mask, 1, 0.0, min_reps=1)
    times = []
    for _ in range(args.steps):
        t, nbytes, _ = time_oracle(c, mask, 1, 0.0, min_reps=1)
        times.append(t)
    t = statistics.mean(times)
    value = workload_bytes(c) / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), bf16-rounded)",
        "config": {"workload": args.config, "B": c["B"], "Hq": c["Hq"], "Hkv": c["Hkv"], "head_dim": c["D"],
                   "prefix_len": c["P"], "tree_nodes": c["T"], "block_m": c["BM"], "block_n": c["BN"]},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": cores, "kind": "port",
                         "sample": f"the whole {args.config} op per step: numpy oracle metadata build + dense+mask "
                                   f"fp32 attention over every (batch, kv-head); CPU {model}"},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


class Timing:
    """CUDA-graph replay and CUDA-event timing on one side stream."""

    def __init__(self, torch, dev, world):
        self.torch, self.dev, self.world = torch, dev, world
        self.stream = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))

    def graphs_of(self, fn, n, chunk):
        """CUDA graphs running fn(0 .. n-1) in order: full chunks + remainder."""
        torch = self.torch
        out, i = [], 0
        while i < n:
            cnt = min(chunk, n - i)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                for j in range(i, i + cnt):
                    fn(j)
            out.append(g)
            i += cnt
        return out

    def run(self, gs):
        with self.torch.cuda.stream(self.stream):
            for g in gs:
                g.replay()

    def back_to_back(self, gs, n):
        """Device time per step (ms) of n steps replayed back to back: one event pair."""
        torch = self.torch
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            e0.record(self.stream)
            for g in gs:
                g.replay()
            e1.record(self.stream)
        torch.cuda.synchronize(self.dev)
        return e0.elapsed_time(e1) / n

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()
        self.torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, values):
        if self.world == 1:
            return list(values)
        import torch.distributed as dist

        t = self.torch.tensor(list(values), dtype=self.torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()


def device_inputs(torch, c, dev, seed):
    """Q/K/V ~ N(0, 1) in bf16, drawn on the device from a seeded generator:
    every rank draws the same problem."""
    g = torch.Generator(device=dev).manual_seed(seed)
    B, Hq, Hkv, D, P, T = c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"]
    return tuple(torch.randn(s, generator=g, device=dev).to(torch.bfloat16)
                 for s in ((B, Hq, T, D), (B, Hkv, P + T, D), (B, Hkv, P + T, D)))


def shard_bytes(c, shard) -> int:
    """Algorithmic bytes of one rank's units (its share of workload_bytes)."""
    units = max(shard.units, 0)
    return workload_bytes(c) * units // max(c["B"] * c["Hkv"], 1)


def subconfig_record(torch, tm, name, args, rank, world, hbm_gbs, tc_burst, tc_sus):
    """A tensor-bound benchmark configuration through the same sharded op:
    device time per call back to back (max over ranks), tokens/s, HBM and
    tensor fractions."""
    import tsfa_shard

    c = trees.CONFIGS[name]
    mask = trees.config_tree(c, seed=0)
    m = torch.from_numpy(mask).to(tm.dev)
    shard = tsfa_shard.plan(c["B"], c["Hkv"], world, rank)
    per_rank = max(shard_bytes(c, shard), 1)
    nsets = max(1, math.ceil(1.5 * L2_BYTES / per_rank))
    sets = [device_inputs(torch, c, tm.dev, 3000 + i) for i in range(nsets)]
    outs = [torch.empty_like(s[0]) for s in sets]

    def step(i=0):
        q, k, v = sets[i % nsets]
        tsfa_shard.run_shard(q, k, v, m, outs[i % nsets], shard, block_m=c["BM"], block_n=c["BN"])

    n = max(5, min(args.steps, 200))
    with torch.cuda.stream(tm.stream):
        for i in range(nsets):
            step(i)
    gs = tm.graphs_of(step, n, max(nsets, 16))
    tm.run(gs)
    tm.barrier()
    t_ms = tm.back_to_back(gs, n)
    tm.barrier()
    (t_ms,) = tm.max_over_ranks([t_ms])
    t = t_ms / 1e3
    fl = workload_flops(c, mask)
    flops = fl["prefix"] + fl["tree_executed"]
    nbytes = workload_bytes(c)
    del sets, outs, gs
    torch.cuda.empty_cache()
    return {
        "shape": {k: c[k] for k in ("B", "Hq", "Hkv", "D", "P", "T", "BM", "BN")},
        "us_per_call": t * 1e6, "steps": n, "tokens_per_s": c["B"] * c["T"] / t,
        # fractions per GPU: the whole job's rate over world x one GPU's peak
        "hbm_tbs": nbytes / t / 1e12, "hbm_frac": nbytes / t / 1e9 / hbm_gbs / world,
        "tensor_tflops": flops / t / 1e12, "tensor_frac_sustained": flops / t / 1e12 / tc_sus / world,
        "tensor_frac_burst": flops / t / 1e12 / tc_burst / world,
        "flops": {"prefix": fl["prefix"], "tree_executed": fl["tree_executed"], "tree_useful": fl["tree_useful"]},
        "bytes_per_call": nbytes, "units_per_rank_max": tsfa_shard.max_units(c["B"], c["Hkv"], world),
        "l2": f"{nsets} input set(s) of the whole problem; each rank reads {per_rank / 2**20:.0f} MiB per call",
    }


def sdpa_comparator(torch, tm, sets, m, P, T, nsets, steps, step):
    """torch SDPA with an additive [T, P + T] mask (0 visible, -inf not) on the
    bench's input sets: device time per call back to back, and its largest
    difference from this package's output on set 0."""
    import torch.nn.functional as F

    q0 = sets[0][0]
    add = torch.zeros((T, P + T), dtype=q0.dtype, device=q0.device)
    add[:, P:].masked_fill_(m.to(torch.bool).logical_not(), float("-inf"))

    def call(i):
        qi, ki, vi = sets[i % nsets]
        return F.scaled_dot_product_attention(qi, ki, vi, attn_mask=add, enable_gqa=True)

    try:
        diff = float((call(0).float() - step(0).float()).abs().max())
        n = max(10, min(steps, 2000))
        gs = tm.graphs_of(call, n, nsets * max(1, 256 // nsets))
        tm.run(gs)
        t_ms = tm.back_to_back(gs, n)
    except Exception as e:  # a comparator that cannot run is reported, not fatal
        return {"torch_sdpa_additive_mask": {"unavailable": f"{type(e).__name__}: {e}"[:200]}}
    return {"torch_sdpa_additive_mask": {"us_per_call": t_ms * 1e3, "steps": n, "max_abs_diff_vs_op": diff,
                                         "how": "F.scaled_dot_product_attention(enable_gqa=True) with a [T, P+T] "
                                                "additive mask, same rotating input sets, back to back"}}


def run_ours(args, c, mask, rank, world, local_rank):
    import torch

    import eagle_tree_sparse_bridge as br
    import tree_sparse_flashattn as tsfa
    import tsfa_native as nat
    import tsfa_shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    nat.require_cuda(dev)
    tm = Timing(torch, dev, world)
    B, Hq, Hkv, D, P, T = c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"]
    G = Hq // Hkv
    shard = tsfa_shard.plan(B, Hkv, world, rank)
    per_rank = max(shard_bytes(c, shard), 1)
    gen = torch.Generator().manual_seed(1000)  # the same problem on every rank
    q_h = torch.randn((B, Hq, T, D), generator=gen).to(torch.bfloat16)
    k_h = torch.randn((B, Hkv, P + T, D), generator=gen).to(torch.bfloat16)
    v_h = torch.randn((B, Hkv, P + T, D), generator=gen).to(torch.bfloat16)
    m_h = torch.from_numpy(mask)
    q, k, v, m = (x.to(dev) for x in (q_h, k_h, v_h, m_h))

    # Input sets cycled through by consecutive steps: what one rank reads over
    # all of them is more than 1.5x the 126 MB L2, so every step reads its
    # Q/K/V from HBM although the steps run back to back (no flush kernel and
    # no event pair between them).
    nsets = max(2, math.ceil(1.5 * L2_BYTES / per_rank))
    sets = [(q, k, v)] + [device_inputs(torch, c, dev, 2000 + i) for i in range(nsets - 1)]
    meta = tsfa.prepare_tree_sparse_metadata(m, P, c["BM"], c["BN"])
    o_sets = [torch.empty_like(q) for _ in range(nsets)]
    calls = shard.calls()

    def step(i=0):
        """One call of the op on this rank's units (the whole op at N = 1)."""
        qi, ki, vi = sets[i % nsets]
        if world == 1:
            return br.run_tree_sparse_kernel(qi, ki, vi, m, block_m=c["BM"], block_n=c["BN"])
        tsfa_shard.run_shard(qi, ki, vi, m, o_sets[i % nsets], shard, block_m=c["BM"], block_n=c["BN"])
        return o_sets[i % nsets]

    def kernel_only_cluster(i=0):
        """The forward forced onto the cluster merge, alone over prebuilt metadata."""
        nat.force_cluster_merge(True)
        try:
            kernel_only(i)
        finally:
            nat.force_cluster_merge(False)

    def kernel_only(i=0):
        """The forward alone over prebuilt metadata, on this rank's units."""
        qi, ki, vi = sets[i % nsets]
        oi = o_sets[i % nsets]
        for b0, b1, h0, h1 in calls:
            nat.fwd_with_metadata(qi[b0:b1, h0 * G:h1 * G], ki[b0:b1, h0:h1], vi[b0:b1, h0:h1],
                                  oi[b0:b1, h0 * G:h1 * G], meta, prefix_len=P)

    with torch.cuda.stream(tm.stream):
        for i in range(nsets):
            step(i)
            op_plan = nat.last_plan()  # the op's forward plan (the roofline leg should run the same)
            kernel_only(i)
            kernel_plan = nat.last_plan()
    torch.cuda.synchronize(dev)
    chunk = nsets * max(1, 256 // nsets)
    g_warm = tm.graphs_of(lambda j: (step(j), kernel_only(j)), max(args.warmup, 3), chunk)
    g_step = tm.graphs_of(step, args.steps, chunk)
    g_kern = tm.graphs_of(kernel_only, args.steps, chunk)
    g_kern_cl = tm.graphs_of(kernel_only_cluster, args.steps, chunk)
    g_spin = tm.graphs_of(lambda j: (step(j), kernel_only(j)), 128, chunk)
    torch.cuda.synchronize(dev)

    visible = [x.strip() for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip()]
    sampler = ClockSampler(visible[local_rank] if local_rank < len(visible) else local_rank)
    tm.run(g_warm)
    # the first replay of a graph also uploads it to the device: replay the
    # timed graphs once, untimed, so the timed region holds only the steps
    tm.run(g_step)
    tm.run(g_kern)
    tm.run(g_kern_cl)
    tm.run(g_spin)
    tm.barrier()
    sampler.start()
    time.sleep(0.3)
    # Untimed steps right before each timed leg (a few ms of work): a GPU
    # that has sat idle (the clock sampler's start-up) is back at full clocks
    # when the events start.
    tm.run(g_spin)
    tm.barrier()
    wall0 = time.perf_counter()
    t_step_ms = tm.back_to_back(g_step, args.steps)
    tm.barrier()
    wall1 = time.perf_counter()
    tm.run(g_spin)
    t_kern_ms = tm.back_to_back(g_kern, args.steps)
    tm.barrier()
    tm.run(g_spin)
    t_kern_cl_ms = tm.back_to_back(g_kern_cl, args.steps)
    tm.barrier()

    # The same op timed in isolation: L2 flushed by a 256 MB write before each
    # step and a CUDA event pair around each step (adds the ~5 us floor of an
    # event-timed launch on these boxes).
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    g1_step, g1_kern = tm.graphs_of(step, 1, 1)[0], tm.graphs_of(kernel_only, 1, 1)[0]

    def timed(fn, n, with_flush=True):
        st = tm.stream
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        with torch.cuda.stream(st):
            for i in range(n):
                if with_flush:
                    flush.fill_(i & 0xFF)
                ev[i][0].record(st)
                fn()
                ev[i][1].record(st)
        torch.cuda.synchronize(dev)
        return [a.elapsed_time(b) for a, b in ev]

    iso_steps = max(10, min(args.steps, 300))
    with torch.cuda.stream(tm.stream):
        g1_step.replay()
        g1_kern.replay()
    tm.run(g_spin)
    iso_step_ms = statistics.mean(timed(g1_step.replay, iso_steps))
    tm.run(g_spin)
    iso_kern_ms = statistics.mean(timed(g1_kern.replay, iso_steps))
    tm.barrier()

    # The optional output gather (NCCL all_gather over NVLink), timed apart.
    gather = None
    if world > 1:
        out_full = o_sets[0]
        tsfa_shard.gather(out_full, shard)
        tm.barrier()
        gt = []
        for _ in range(20):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            tsfa_shard.gather(out_full, shard)
            e1.record()
            torch.cuda.synchronize(dev)
            gt.append(e0.elapsed_time(e1))
        (g_ms,) = tm.max_over_ranks([statistics.median(gt)])
        gather = {"us_per_call": g_ms * 1e3, "how": "torch.distributed.all_gather (NCCL) of the ranks' output "
                                                    "shards into a full output on every rank; median of 20, max "
                                                    "over ranks; not part of value"}

    # Comparator (a library kernel, not this package's path): torch SDPA on the
    # same input sets with the tree as an additive mask over [P + T] keys and
    # the kv-heads shared by enable_gqa, timed like the op (N = 1 only).
    sdpa = None
    if world == 1:
        sdpa = sdpa_comparator(torch, tm, sets, m, P, T, nsets, args.steps, step)
    tm.barrier()

    # end to end through the public API with host buffers: this rank's slices
    q_p, k_p, v_p, m_p = (x.pin_memory() for x in (q_h, k_h, v_h, m_h))
    out_p = torch.empty(q_h.shape, dtype=q_h.dtype).pin_memory()
    cs = torch.cuda.current_stream(dev)
    e2e_parts = []

    def e2e_step(record=False):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if record:
            ev[0].record(cs)
        if world == 1:
            qd = q_p.to(dev, non_blocking=True)
            kd = k_p.to(dev, non_blocking=True)
            vd = v_p.to(dev, non_blocking=True)
            md = m_p.to(dev, non_blocking=True)
            if record:
                ev[1].record(cs)
            o = br.run_tree_sparse_kernel(qd, kd, vd, md, block_m=c["BM"], block_n=c["BN"])
            if record:
                ev[2].record(cs)
            out_p.copy_(o, non_blocking=True)
        else:
            md = m_p.to(dev, non_blocking=True)
            views = [(b0, b1, h0, h1, q_p[b0:b1, h0 * G:h1 * G].to(dev, non_blocking=True),
                      k_p[b0:b1, h0:h1].to(dev, non_blocking=True), v_p[b0:b1, h0:h1].to(dev, non_blocking=True))
                     for b0, b1, h0, h1 in calls]
            if record:
                ev[1].record(cs)
            outs = [(b0, b1, h0, h1, br.run_tree_sparse_kernel(qd, kd, vd, md, block_m=c["BM"], block_n=c["BN"]))
                    for b0, b1, h0, h1, qd, kd, vd in views]
            if record:
                ev[2].record(cs)
            for b0, b1, h0, h1, o in outs:
                out_p[b0:b1, h0 * G:h1 * G].copy_(o, non_blocking=True)
        if record:
            ev[3].record(cs)
            e2e_parts.append(ev)

    # K steps back to back between one event pair (the pinned copies, the
    # call and the read-back of each step queue behind the previous step's on
    # one stream), after untimed steps that bring the host->device path up to
    # its sustained rate
    with torch.cuda.stream(tm.stream):
        for _ in range(10):
            e2e_step()
    torch.cuda.synchronize(dev)
    e2e_steps = max(10, min(args.steps, 200))
    e2e_t0, e2e_t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(tm.stream):
        e2e_t0.record(tm.stream)
        for _ in range(e2e_steps):
            e2e_step()
        e2e_t1.record(tm.stream)
    torch.cuda.synchronize(dev)
    e2e_serial_ms = e2e_t0.elapsed_time(e2e_t1) / e2e_steps

    # The same steps pipelined over two sets of device input buffers: step
    # i's host->device copies run on a copy stream while step i-1's call and
    # its device->host read-back run on the op's stream (PCIe is full duplex),
    # the way a serving loop feeds the op.  Every step still copies all of its
    # inputs in and its output out inside the timed region.
    s_h2d, s_op = torch.cuda.Stream(dev), tm.stream
    pviews = list(calls) if world > 1 else [None]

    def host_slices(v):
        if v is None:
            return q_p, k_p, v_p
        b0, b1, h0, h1 = v
        return q_p[b0:b1, h0 * G:h1 * G], k_p[b0:b1, h0:h1], v_p[b0:b1, h0:h1]

    dbuf = [[tuple(torch.empty(x.shape, dtype=x.dtype, device=dev) for x in host_slices(v)) for v in pviews]
            for _ in range(2)]
    dmask = [torch.empty(m_p.shape, dtype=m_p.dtype, device=dev) for _ in range(2)]
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    op_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_pipe_step(i):
        j = i & 1
        with torch.cuda.stream(s_h2d):
            s_h2d.wait_event(op_done[j])  # step i - 2's call has read these buffers
            for v, bufs in zip(pviews, dbuf[j]):
                for d, h in zip(bufs, host_slices(v)):
                    d.copy_(h, non_blocking=True)
            dmask[j].copy_(m_p, non_blocking=True)
            h2d_done[j].record(s_h2d)
        with torch.cuda.stream(s_op):
            s_op.wait_event(h2d_done[j])
            for v, (qd, kd, vd) in zip(pviews, dbuf[j]):
                o = br.run_tree_sparse_kernel(qd, kd, vd, dmask[j], block_m=c["BM"], block_n=c["BN"])
                if v is None:
                    out_p.copy_(o, non_blocking=True)
                else:
                    b0, b1, h0, h1 = v
                    out_p[b0:b1, h0 * G:h1 * G].copy_(o, non_blocking=True)
            op_done[j].record(s_op)

    for i in range(10):
        e2e_pipe_step(i)
    torch.cuda.synchronize(dev)
    p_t0, p_t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_t0.record(s_h2d)
    for i in range(e2e_steps):
        e2e_pipe_step(i)
    s_h2d.wait_event(op_done[(e2e_steps - 1) & 1])
    p_t1.record(s_h2d)
    torch.cuda.synchronize(dev)
    e2e_ms = p_t0.elapsed_time(p_t1) / e2e_steps
    del dbuf, dmask
    for _ in range(10):
        e2e_step(record=True)
    torch.cuda.synchronize(dev)
    parts = np.array([[ev[i].elapsed_time(ev[i + 1]) for i in range(3)] for ev in e2e_parts])
    h2d_us, call_us, d2h_us = (float(x) * 1e3 for x in np.median(parts, axis=0))
    tm.barrier()

    hbm_gbs, tc_burst, tc_sus, src = peaks()
    configs = {}
    if not args.no_subconfigs:
        del sets, o_sets, g_step, g_kern, g_kern_cl, g_spin, g_warm
        torch.cuda.empty_cache()
        for name in SUBCONFIGS:
            configs[name] = subconfig_record(torch, tm, name, args, rank, world, hbm_gbs, tc_burst, tc_sus)
    time.sleep(0.2)
    clocks = sampler.stop()

    nbytes = workload_bytes(c)
    t_step, t_kern, t_kern_cl, t_e2e, t_e2e_serial, t_iso_step, t_iso_kern, h2d_us, call_us, d2h_us = \
        tm.max_over_ranks([t_step_ms / 1e3, t_kern_ms / 1e3, t_kern_cl_ms / 1e3, e2e_ms / 1e3, e2e_serial_ms / 1e3,
                           iso_step_ms / 1e3, iso_kern_ms / 1e3, h2d_us, call_us, d2h_us])
    if rank != 0:
        return
    flops = workload_flops(c, mask)
    achieved = nbytes / t_kern / 1e9
    traffic = None
    tpath = os.path.join(HERE, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            tj = json.load(f)
        if tj.get("workload") == args.config and world == 1:
            traffic = tj.get("dram_bytes_per_launch")
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cores = use_all_cores()
        t_cpu, cpu_bytes, reps = time_oracle(c, mask, 1, args.cpu_budget)
        cpu = {"value": cpu_bytes / t_cpu / 1e12, "unit": "TB/s", "cores": cores, "kind": "port",
               "sample": f"the whole {args.config} op, median of {reps} runs (~{args.cpu_budget:.0f} s): numpy "
                         f"oracle metadata build + dense+mask fp32 attention; CPU {cpu_info()}"}
    h2d_bytes = sum(x.numel() * x.element_size() for x in (q_h, k_h, v_h)) * per_rank // max(nbytes, 1) \
        + m_h.numel() * m_h.element_size()
    line = {
        "metric": METRIC,
        "value": nbytes / t_step / 1e12,
        "unit": "TB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": t_step * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16; seeded random draft tree)",
        "config": {"workload": args.config, "global_batch": B, "Hq": Hq, "Hkv": Hkv, "head_dim": D,
                   "prefix_len": P, "tree_nodes": T, "block_m": c["BM"], "block_n": c["BN"],
                   "parallelism": (f"{world} ranks over the {B * Hkv} (batch, kv-head) units "
                                   f"(<= {tsfa_shard.max_units(B, Hkv, world)} per rank), no collective on the path"
                                   if world > 1 else "one GPU"),
                   "l2": f"steps back to back over {nsets} rotating input sets ({nsets * per_rank / 2**20:.0f} MiB "
                         f"read per rank > 126 MB L2): every step reads HBM"},
        "us_per_call": t_step * 1e6,
        "kernel_us": t_kern * 1e6,
        "tokens_per_s": B * T / t_step,
        "isolated": {"us_per_call": t_iso_step * 1e6, "kernel_us": t_iso_kern * 1e6, "steps": iso_steps,
                     "how": "256 MB L2 flush + CUDA event pair around each step"},
        "gather": gather,
        "configs": configs,
        "comparators": sdpa,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_gbs, "unit": "GB/s",
                     "frac": achieved / hbm_gbs, "traffic": traffic, "peak_source": src,
                     "kernel": "the whole op's forward (prefix sweep + tree walk + split merge through L2): "
                               "the instantiation and plan the op launches behind its metadata kernel, alone "
                               "over prebuilt metadata",
                     "op_plan": op_plan, "kernel_plan": kernel_plan,
                     "bytes_per_launch": nbytes, "tensor_tflops": flops["prefix"] / t_kern / 1e12,
                     "tensor_frac": flops["prefix"] / t_kern / 1e12 / tc_burst,
                     "cluster_merge": {"kernel": "the same forward with the thread-block-cluster merge (the "
                                                 "per-batch op's), alone over prebuilt metadata",
                                       "kernel_us": t_kern_cl * 1e6, "achieved": nbytes / t_kern_cl / 1e9,
                                       "frac": nbytes / t_kern_cl / 1e9 / hbm_gbs}},
        "cpu_baseline": cpu,
        "e2e": {"value": nbytes / t_e2e / 1e12, "unit": "TB/s", "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": q_h.numel() * q_h.element_size() * per_rank // max(nbytes, 1),
                "us_per_call": t_e2e * 1e6, "steps": e2e_steps,
                "how": "the steps pipelined over two sets of device input buffers (step i's host->device copies on "
                       "a copy stream beside step i-1's call and read-back on the op's stream), between one CUDA "
                       "event pair, after 10 untimed",
                "serial_us_per_call": t_e2e_serial * 1e6,
                "serial_how": "the same steps on one stream (copies, call, read-back in turn), one event pair",
                "breakdown_us": {"h2d": h2d_us, "call": call_us, "d2h": d2h_us,
                                 "how": "median of 10 steps, CUDA events between the pinned copies and the call"}},
        "gpu_launches": 2 * args.steps * len(calls),  # per step and call: metadata build + forward
        "clocks": clocks,
        "wall_s_timed_steps": wall1 - wall0,
    }
    print(json.dumps(line), flush=True)


def run_profile_case(args, c, mask):
    """Small eager case for profiler captures (ncu): the op and the forward
    over prebuilt metadata, `--steps` times each on one input set, no graphs,
    no timing.  Prints one line when done."""
    import torch

    import eagle_tree_sparse_bridge as br
    import tree_sparse_flashattn as tsfa
    import tsfa_native as nat

    dev = torch.device("cuda", 0)
    q, k, v = device_inputs(torch, c, dev, 4000)
    m = torch.from_numpy(mask).to(dev)
    meta = tsfa.prepare_tree_sparse_metadata(m, c["P"], c["BM"], c["BN"])
    o = torch.empty_like(q)
    for _ in range(max(args.steps, 1)):
        br.run_tree_sparse_kernel(q, k, v, m, block_m=c["BM"], block_n=c["BN"])
    for _ in range(max(args.steps, 1)):
        nat.fwd_with_metadata(q, k, v, o, meta, prefix_len=c["P"])
    torch.cuda.synchronize(dev)
    print(f"profile case {args.config}: {args.steps} op calls, {args.steps} forward calls", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="cfg2_llama3_8b", choices=sorted(trees.CONFIGS))
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subconfigs", action="store_true", help="skip the configuration 3 / 4 records")
    ap.add_argument("--profile-case", action="store_true",
                    help="run the op and the forward --steps times eagerly for a profiler capture; no timing")
    args = ap.parse_args()
    c = trees.CONFIGS[args.config]
    mask = trees.config_tree(c, seed=0)
    if args.profile_case:
        run_profile_case(args, c, mask)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, c, mask, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, c, mask, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
