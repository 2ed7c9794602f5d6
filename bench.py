"""Training-throughput benchmark: tinytrain's training step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config llama-1b]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference ...      # the reference's CPU build

One step = one AdamW optimizer step over the global batch: n_micro
micro-batches of 16 x 2048 tokens per rank (gradient accumulation), forward,
fused cross-entropy, backward, bucketed NCCL gradient all-reduce overlapped
with the last backward (N > 1), global-norm clipping folded into the fused
AdamW kernel. Weights are fp32 ~ N(0, 0.02), tokens uniform in [0, 32000)
(synthetic: no dataset). The global batch is fixed (256 x 2048 for llama-1b),
so scaling is strong.

value: tokens/s with the token ids already in HBM (tt_trainer_step_device),
timed with CUDA events on the launching stream, max over ranks.
e2e: the same through the public C ABI with host buffers
(tt_trainer_step_submit / tt_trainer_step_result: each step's host ids
uploaded and its loss read back inside the timed region, the next step
submitted before the previous result is collected).
roofline: the dominant kernel (the tcgen05 GEMM with the bf16x3 operand
split) timed live over the timed region (events around each launch);
achieved = algorithmic FLOPs (2*M*N*K per GEMM) / kernel time; traffic = the
average DRAM bytes per GEMM launch of one llama-1b micro-batch step, from the
ncu capture summarized in profiles/gemm_traffic_llama1b_microbatch.md.
graph (--graph, one GPU): the same step replayed from a CUDA graph
(tt_trainer_step_graph), timed after the e2e region.
"""
from __future__ import annotations

import argparse
import atexit
import ctypes as C
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

def gemm_traffic(model):
    """DRAM bytes per GEMM launch from the committed ncu summary (llama-1b)."""
    if model != "llama-1b":
        return None
    try:
        with open(os.path.join(ROOT, "profiles", "gemm_traffic_llama1b_microbatch.md")) as f:
            for ln in f:
                if ln.startswith("traffic_bytes_per_launch:"):
                    return float(ln.split(":", 1)[1])
    except OSError:
        pass
    return None


WORKLOADS = {
    "llama-1b": dict(model="llama-1b", vocab=32000, dim=2048, layers=16, heads=16, ffn=5632,
                     max_seq=2048, global_batch=256, seq=2048, micro=16),
    "llama-110m": dict(model="llama-110m", vocab=32000, dim=768, layers=12, heads=12, ffn=2048,
                       max_seq=1024, global_batch=64, seq=1024, micro=64),
    "llama-13m": dict(model="llama-13m", vocab=32000, dim=256, layers=6, heads=8, ffn=768,
                      max_seq=256, global_batch=16, seq=128, micro=16),
}
# The reference's CPU micro-step sample per config (B, T): the config's own
# sequence length. At 1B one 1 x 2048 micro-step takes ~10 min on 8 cores and
# more than 62 GB of host memory at full depth, so the sample is taken at
# depths 1 and 2 of the same width and extrapolated (reference_micro_step).
CPU_SAMPLE = {"llama-1b": (1, 2048), "llama-110m": (1, 1024), "llama-13m": (16, 128)}
SAMPLE_DEPTHS = (1, 2)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def flops_per_token(w):
    d, L, f, V, T = w["dim"], w["layers"], w["ffn"], w["vocab"], w["seq"]
    linear = L * (4 * d * d + 3 * d * f) + d * V
    return 6 * linear + 6 * T * d * L


def n_params(w):
    d, L, f, V = w["dim"], w["layers"], w["ffn"], w["vocab"]
    return V * d + L * (2 * d + 4 * d * d + 3 * d * f) + d


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons, one process per
    node (local rank 0) for all of the node's GPUs in the run.

    The sampler starts before the warm-up steps, so nvidia-smi's own start-up
    (driver queries on every GPU) overlaps the warm-up and leaves the device
    busy, and it runs until the last region ends. Each sample carries its
    timestamp; summary(t0, t1) keeps the samples taken between two instants
    recorded with now() at a region's start and end."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus, active=True):
        self.gpus = gpus
        self.active = active
        self.proc = None
        self.f = None
        self.path = None

    def start(self):
        if not self.active:
            return self
        try:
            d = tempfile.mkdtemp(prefix="bench_clocks_")
            self.path = os.path.join(d, f"clocks_{os.getpid()}.csv")
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", ",".join(str(g) for g in self.gpus)],
                stdout=self.f, stderr=subprocess.DEVNULL)
            atexit.register(self.stop)
        except Exception:
            self.proc = None
        return self

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.proc = None
        if self.f:
            self.f.close()
            self.f = None

    @staticmethod
    def now():
        return datetime.datetime.now()

    @staticmethod
    def parse(lines, t0, t1):
        """Median SM clock, max SM clock and the active throttle reasons of
        the CSV sample lines stamped within [t0, t1]."""
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for line in lines:
            p = [x.strip() for x in line.split(",")]
            if len(p) < 10:
                continue
            try:
                clk, cmax = float(p[2]), float(p[3])
            except ValueError:
                continue
            try:
                ts = datetime.datetime.strptime(p[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                ts = None
            rows.append((ts, clk, cmax, p))
        # Samples whose timestamp does not parse are kept only if none parses
        # (an unexpected nvidia-smi format then gives the whole run's samples).
        windowed = any(r[0] is not None for r in rows)
        for ts, clk, cmax, p in rows:
            if windowed and (ts is None or ts < t0 or ts > t1):
                continue
            sm.append(clk)
            smax.append(cmax)
            for n, v in zip(names, p[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}

    def summary(self, t0, t1):
        if not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        with open(self.path) as f:
            lines = f.readlines()
        r = self.parse(lines, t0, t1)
        if r["sm_mhz"] is None:
            # a region shorter than the 200 ms sampling period: the samples
            # within half a second of it
            pad = datetime.timedelta(seconds=0.5)
            r = self.parse(lines, t0 - pad, t1 + pad)
            r["window"] = "region +- 0.5 s (region shorter than the sampling period)"
        return r


def reference_micro_step(w):
    """The reference CPU build's training throughput on the workload, from a
    bounded sample (oracle/_ref: the reference's src/*.cpp compiled unchanged,
    all host threads).

    The sample is one micro-step of CPU_SAMPLE tokens at the config's width
    and sequence length: forward, cross-entropy and backward of the
    reference's GPTModel, timed at depth 1 and at depth 2, each after one
    untimed micro-step (the first step of a process pays page faults and
    allocator growth: 77 s against 51 s warm at depth 1 of the 1B width). The
    reference runs its layers one after another with the same ops, so a
    full-depth micro-step costs base + L * per_layer with per_layer = t(2) -
    t(1) and base = t(1) - per_layer. Measured at the 1B width on 8 cores, a
    third layer added 53 s against 57 s for the second: the per-layer cost is
    flat to slightly falling, so the estimate is at most a few percent off. The
    optimizer step (clip + AdamW, linear in the parameter count) is timed on
    the depth-2 model, scaled to the full parameter count, and amortized over
    the micro-steps of one global batch, as gradient accumulation does.
    Returns a dict with tokens/s and the parts.
    """
    from oracle import refbind as rb
    if not rb.available():
        return None
    B, T = CPU_SAMPLE[w["model"]]
    d1, d2 = SAMPLE_DEPTHS
    t, opt, reps = {}, {}, {}
    for d in (d1, d2):
        c = rb.cfg(vocab=w["vocab"], dim=w["dim"], layers=d, heads=w["heads"], ffn=w["ffn"],
                   max_seq=max(w["max_seq"], T))
        t[d], opt[d] = rb.time_phases(c, B, T, 1, 1)
        reps[d] = 1
        if t[d] < 1.0:
            # A small model's micro-step is short against timer and load
            # noise: average enough of them for about two seconds.
            reps[d] = min(20, int(2.0 / max(t[d], 1e-3)) + 1)
            t[d], opt[d] = rb.time_phases(c, B, T, 1, reps[d])
    per_layer = (t[d2] - t[d1]) / (d2 - d1)
    if per_layer <= 0.0:
        # Noise larger than a layer's cost (tiny models only): charge the
        # whole depth-d2 time to its layers.
        per_layer = t[d2] / d2
    rest = max(t[d1] - d1 * per_layer, 0.0)
    micro = rest + w["layers"] * per_layer
    w2 = dict(w, layers=d2)
    opt_full = opt[d2] * n_params(w) / n_params(w2)
    n_micro = w["global_batch"] * w["seq"] / (B * T)
    step = n_micro * micro + opt_full
    tps = w["global_batch"] * w["seq"] / step
    sample = (f"reference train step at the {w['model']} width, one micro-step of {B} x {T} "
              f"tokens (forward, cross-entropy, backward) timed at depth {d1} ({t[d1]:.1f} s) and "
              f"depth {d2} ({t[d2]:.1f} s), each after one untimed micro-step"
              f"{' (means over %d and %d micro-steps)' % (reps[d1], reps[d2]) if reps[d1] > 1 or reps[d2] > 1 else ''}: "
              f"{per_layer:.1f} s per layer + {rest:.1f} s base, "
              f"{micro:.0f} s per full-depth ({w['layers']} layers) micro-step; clip + AdamW "
              f"{opt_full:.1f} s (timed at depth {d2}, scaled to {n_params(w)} parameters) "
              f"amortized over the {n_micro:.0f} micro-steps of a {w['global_batch']} x {w['seq']} "
              f"global batch; {os.cpu_count()} host threads")
    return {"tokens_per_s": tps, "micro_s": micro, "per_layer_s": per_layer, "rest_s": rest,
            "opt_s": opt_full, "sample": sample, "timed": {str(d): t[d] for d in t}}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args, w, rank, world):
    """--impl reference: the reference's own CPU implementation (oracle/_ref,
    the reference sources compiled unchanged), all host threads, rank 0 only.
    One full-depth micro-step of the workload takes minutes on the CPU, so the
    arm times the two depth samples of reference_micro_step (two timed
    micro-steps whatever --steps asks; "steps" reports them)."""
    if rank != 0:
        return
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count()))
    from oracle import refbind as rb
    if not rb.available():
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref/libttref.so was not built"}))
        return
    t0 = time.time()
    r = reference_micro_step(w)
    tps = r["tokens_per_s"]
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count()))
    ms_step = w["global_batch"] * w["seq"] / tps * 1e3
    print(json.dumps({
        "impl": "reference", "metric": "train tokens/sec", "value": tps, "unit": "tokens/s",
        "n_gpus": world, "steps": 2, "steps_requested": args.steps, "warmup": 0,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(w, world),
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "reference",
                         "cpu": cpu_model(), "sample": r["sample"]},
        "reference_parts": {k: r[k] for k in ("micro_s", "per_layer_s", "rest_s", "opt_s",
                                              "timed")},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "wall_s": time.time() - t0}))


def workload_config(w, world):
    return {"workload": f"{w['model']} training step: dim {w['dim']}, {w['layers']} layers, "
                        f"{w['heads']} heads, ffn {w['ffn']}, vocab {w['vocab']}, tied "
                        f"embeddings, global batch {w['global_batch']} x {w['seq']} tokens "
                        f"in micro-batches of {w['micro']} x {w['seq']}, AdamW + clip 1.0",
            "model": w["model"], "params": n_params(w), "global_batch": w["global_batch"],
            "seq_len": w["seq"], "micro_batch": w["micro"], "parallelism": f"dp{world}",
            "l2": "no flush: every step streams > 10 GB (weights, moments, activations) "
                  "through a 126 MB L2"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="llama-1b", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="override the config's global batch (sequences), e.g. one "
                         "micro-batch per step for an ncu launch list")
    ap.add_argument("--micro", type=int, default=None,
                    help="sequences per micro-batch (gradient accumulation unit); "
                         "the global batch and so the optimizer step are unchanged")
    ap.add_argument("--graph", action="store_true",
                    help="also time the step replayed from a CUDA graph (one GPU; reported "
                         "under 'graph', after the e2e region)")
    args = ap.parse_args()
    w = dict(WORKLOADS[args.config])
    if args.global_batch:
        w["global_batch"] = args.global_batch
    if args.micro:
        w["micro"] = args.micro
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, w, rank, world)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    from tinytrain_b200 import _ttk
    from tinytrain_b200 import trainer as trn

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    stream = torch.cuda.current_stream()
    trn.set_stream(stream.cuda_stream)
    # Freed blocks are handed back out by the library instead of returning
    # to the device pool: a training loop repeats its allocation pattern
    # every step, and without the cache the pool's map / unmap calls into
    # the driver stalled the host for 0.5-2 s at the start of some steps.
    _ttk.call("ttk_set_block_cache", 1)

    if w["global_batch"] % world:
        raise SystemExit("global batch must split evenly across ranks")
    # Micro-batch: the config's, or the rank's whole share when that is smaller.
    w["micro"] = min(w["micro"], w["global_batch"] // world)
    if (w["global_batch"] // world) % w["micro"]:
        raise SystemExit("rank share must split into whole micro-batches")
    n_micro = w["global_batch"] // (w["micro"] * world)
    B, T = w["micro"], w["seq"]
    tokens_rank = n_micro * B * T

    cfgm = {k: w[k] for k in ("vocab", "dim", "layers", "heads", "ffn", "max_seq")}
    tr = trn.Trainer(cfgm, seed=1234, host_init=False)
    tr.init_normal(0.02, seed=1234)
    tr.set_optimizer(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, clip=1.0)
    if world > 1:
        uid = trn.dist_unique_id() if rank == 0 else b"\0" * 128
        obj = [uid]
        dist.broadcast_object_list(obj, src=0)
        tr.dist_init(rank, world, obj[0], bucket_bytes=64 << 20)

    # Synthetic tokens: each rank its own disjoint stream of windows.
    g = np.random.default_rng(10_000 + rank)
    n_sets = 4
    host_idx = [g.integers(0, w["vocab"], tokens_rank, dtype=np.int64) for _ in range(n_sets)]
    host_tgt = [g.integers(0, w["vocab"], tokens_rank, dtype=np.int64) for _ in range(n_sets)]
    dev_idx = [torch.from_numpy(x).to(dev) for x in host_idx]
    dev_tgt = [torch.from_numpy(x).to(dev) for x in host_tgt]
    pin_idx = [torch.from_numpy(x).pin_memory() for x in host_idx]
    pin_tgt = [torch.from_numpy(x).pin_memory() for x in host_tgt]

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def max_each_over_ranks(vs):
        if world == 1:
            return list(vs)
        t = torch.tensor(vs, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(x) for x in t.tolist()]

    # One clock sampler per node (local rank 0) over the node's GPUs of this
    # run, started before the warm-up and stopped after the e2e region.
    clk = ClockSampler([local] if world == 1 else list(range(world)), active=local == 0).start()

    # ---- warm-up (device-resident ids). The last warm-up step runs with the
    # GEMM timing on, so the timed steps find its CUDA events already
    # created: creating the ~10k events of a first timed step cost 0.4 s of
    # device time (9.40 s against 8.99 s for the next steps).
    # The all-reduce timing events (N > 1) are warmed the same way.
    for i in range(args.warmup):
        if i == args.warmup - 1:
            _ttk.call("ttk_profile_enable", 1)
            if world > 1:
                tr.comm_profile(True)
        tr.step_device(dev_idx[i % n_sets].data_ptr(), dev_tgt[i % n_sets].data_ptr(), B, T,
                       n_micro, 3e-4)
    barrier()
    _ttk.call("ttk_profile_read", None, None, None)  # discard; returns the events to the pool
    if world > 1:
        tr.comm_stats()  # discard, likewise

    # ---- timed region: value
    _ttk.call("ttk_pool_high_water", None, None, 1)
    _ttk.call("ttk_profile_enable", 1)
    if world > 1:
        tr.comm_profile(True)
    l0 = trn.kernel_launches()
    # One event per step boundary on the launching stream: the first and last
    # bracket the timed region, the ones between give each step's time.
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    e0, e1 = ev[0], ev[-1]
    barrier()
    c0 = clk.now()
    e0.record(stream)
    for i in range(args.steps):
        tr.step_device(dev_idx[i % n_sets].data_ptr(), dev_tgt[i % n_sets].data_ptr(), B, T,
                       n_micro, 3e-4)
        ev[i + 1].record(stream)
    barrier()
    c1 = clk.now()
    launches = trn.kernel_launches() - l0
    rh, uh = C.c_size_t(0), C.c_size_t(0)
    _ttk.call("ttk_pool_high_water", C.byref(rh), C.byref(uh), 0)
    free_b, total_b = torch.cuda.mem_get_info()
    memory = {"pool_reserved_high_gb": rh.value / 1e9, "pool_used_high_gb": uh.value / 1e9,
              "device_free_gb": free_b / 1e9, "device_total_gb": total_b / 1e9}
    comm = None
    if world > 1:
        tr.comm_profile(False)
        busy, tail, n_ar, n_st = tr.comm_stats()
        busy, tail = max_over_ranks(busy), max_over_ranks(tail)
        comm = {"allreduce_ms_per_step": busy / args.steps,
                "exposed_tail_ms_per_step": tail / args.steps,
                "allreduces_per_step": n_ar / max(n_st, 1),
                "bytes_per_step": n_params(w) * 4,
                "is": "gradient all-reduce (NCCL, fp32 sum) on the comm stream: summed "
                      "duration of the buckets' all-reduces, and the tail by which the last "
                      "all-reduce ends after the last backward kernel (max over ranks)"}
    gms, gfl, gl = C.c_double(0), C.c_double(0), C.c_int64(0)
    _ttk.call("ttk_profile_enable", 0)
    _ttk.call("ttk_profile_read", C.byref(gms), C.byref(gfl), C.byref(gl))
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    step_ms = max_each_over_ranks([ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)])
    loss_dev = tr.last_loss()
    tokens_step = tokens_rank * world
    value = tokens_step / (ms / 1e3)

    # ---- e2e: public C ABI with host buffers (upload ids, read loss back).
    # tt_trainer_step_submit / _result: each step's ids go host -> device and
    # its loss device -> host inside the timed region; the host submits step
    # i + 1 before collecting step i, as a training loop would, so the device
    # never waits for the host between steps.
    ke = max(1, args.e2e_steps)
    # warm path: both submission slots (their pinned staging is allocated on
    # first use)
    for i in range(2):
        tr.step_submit(pin_idx[i].numpy(), pin_tgt[i].numpy(), B, T, n_micro, 3e-4)
    for i in range(2):
        tr.step_result()
    barrier()
    fe = [torch.cuda.Event(enable_timing=True) for _ in range(ke + 1)]
    f0, f1 = fe[0], fe[-1]
    loss_e2e = None
    c2 = clk.now()
    f0.record(stream)
    for i in range(ke):
        tr.step_submit(pin_idx[i % n_sets].numpy(), pin_tgt[i % n_sets].numpy(), B, T,
                       n_micro, 3e-4)
        fe[i + 1].record(stream)
        if i > 0:
            loss_e2e, _ = tr.step_result()
    loss_e2e, _ = tr.step_result()
    barrier()
    c3 = clk.now()
    ms_e2e = max_over_ranks(f0.elapsed_time(f1)) / ke
    step_ms_e2e = max_each_over_ranks([fe[i].elapsed_time(fe[i + 1]) for i in range(ke)])
    e2e = tokens_step / (ms_e2e / 1e3)

    # ---- optional: the same step replayed from a CUDA graph (one GPU). The
    # graph reads each step's ids from two fixed device buffers, filled by a
    # device copy before each launch (inside the timed region).
    graph = None
    if args.graph and world == 1:
        gi, gt = torch.empty_like(dev_idx[0]), torch.empty_like(dev_tgt[0])
        for i in range(2):  # an eager step, then the recording + first launch
            gi.copy_(dev_idx[i % n_sets])
            gt.copy_(dev_tgt[i % n_sets])
            tr.step_graph(gi.data_ptr(), gt.data_ptr(), B, T, n_micro, 3e-4)
        barrier()
        ge = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        c4 = clk.now()
        ge[0].record(stream)
        for i in range(args.steps):
            gi.copy_(dev_idx[i % n_sets])
            gt.copy_(dev_tgt[i % n_sets])
            tr.step_graph(gi.data_ptr(), gt.data_ptr(), B, T, n_micro, 3e-4)
            ge[i + 1].record(stream)
        barrier()
        c5 = clk.now()
        ms_g = ge[0].elapsed_time(ge[-1]) / args.steps
        graph = {"value": tokens_step / (ms_g / 1e3), "unit": "tokens/s", "ms_per_step": ms_g,
                 "step_ms": [round(ge[i].elapsed_time(ge[i + 1]), 3) for i in range(args.steps)],
                 "loss": tr.last_loss(), "clocks": clk.summary(c4, c5),
                 "is": "tt_trainer_step_graph: the step recorded once in a CUDA graph and "
                       "replayed (ids copied into fixed device buffers before each launch)"}
    clk.stop()
    status = _ttk.device_status()

    if rank == 0:
        hbm, bf16, bf16s, src = peaks()
        gemm_tf = gfl.value / (gms.value / 1e3) / 1e12 if gms.value > 0 else 0.0
        gemm_share = gms.value / (ms * args.steps) if ms > 0 else 0.0
        prec = "tf32x3" if _ttk.call("ttk_gemm_get_precision") == 1 else "bf16x3"
        # Useful FMAs cost 3 MMAs: bf16 ones at the bf16 rate, tf32 ones at half.
        ceil_div = 6.0 if prec == "tf32x3" else 3.0
        line = {
            "metric": "train tokens/sec", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "step_ms": [round(x, 2) for x in step_ms],
            "data": "synthetic (N(0,0.02) weights, uniform tokens)",
            "config": workload_config(w, world),
            "roofline": {
                "kernel": f"gemm_split3_kernel (tcgen05, {prec} split)", "bound": "tensor",
                "achieved": gemm_tf, "peak": bf16s, "unit": "TFLOP/s",
                "frac": gemm_tf / bf16s, "traffic": gemm_traffic(w["model"]),
                "peak_source": f"{src} bf16 sustained (kernel timed inside a long step)",
                "achieved_is": "algorithmic fp32 FLOP/s (2MNK per GEMM); each useful FMA "
                               f"costs 3 MMAs, so the {prec} ceiling is peak/{int(ceil_div)}",
                "ceiling_split3": bf16s / ceil_div,
                "frac_of_split3_ceiling": gemm_tf / (bf16s / ceil_div),
                "mma_rate": {"value": gemm_tf * ceil_div / (2.0 if prec == "tf32x3" else 1.0),
                             "unit": "TFLOP/s", "frac": gemm_tf * ceil_div / bf16s,
                             "is": f"{prec} MMA work the tensor pipe executes (3 MMAs per "
                                   "useful FMA), against the same bf16 peak"},
                "launches": gl.value, "share_of_step": gemm_share},
            "mfu_fp32_equiv": value * flops_per_token(w) / 1e12 / world,
            "gpu_launches": launches,
            "launches_before_timed": l0,
            "memory": memory,
            "allreduce": comm,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 2 * tokens_rank * 8,
                    "d2h_bytes_per_step": 4, "steps": ke,
                    "step_ms": [round(x, 2) for x in step_ms_e2e], "clocks": clk.summary(c2, c3)},
            "clocks": clk.summary(c0, c1),
            "loss": loss_dev, "loss_e2e": loss_e2e, "device_status": status,
            **({"graph": graph} if graph else {}),
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                r = reference_micro_step(w)
            except Exception as ex:  # reported, never fatal
                r = None
                line["cpu_baseline_error"] = str(ex)[:200]
            if r:
                line["cpu_baseline"] = {
                    "value": r["tokens_per_s"], "unit": "tokens/s",
                    "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())),
                    "kind": "reference", "cpu": cpu_model(), "sample": r["sample"]}
        print(json.dumps(line), flush=True)

    tr.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
