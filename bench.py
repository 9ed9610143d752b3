"""Benchmark of the B200 GGUF quantized-matmul path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (the metric's "Q4_K GEMV"): decode
of one Llama-3-8B-shaped layer, M=1 token, every projection Q4_K:
q 4096->4096, k/v 4096->1024, o 4096->4096, gate/up 4096->14336,
down 14336->4096 (218,103,808 weights = 122,683,392 bytes of GGUF blocks).
One step = the layer's 4 GEMV launches (q/k/v and gate/up each fused into one
grouped launch, as vLLM fuses QKV and gate_up). ``value`` is the whole-job
algorithmic HBM throughput (weight bytes + activation bytes read + output
bytes written, per step) in GB/s, timed with CUDA events on the launching
stream, weights resident in HBM. The weights rotate over 3 copies
(368 MB > 126 MB L2) so no step is served from L2.

Also reported: ``e2e`` (same metric through the public Python API with the
activations copied from pinned host memory and the outputs read back every
step), ``roofline`` for the dominant kernel, ``prefill`` (config 4 tensor-core
GEMM TFLOP/s), ``cpu_baseline`` (the reference's CPU arithmetic: gguf-py
dequantize + numpy fp32 matmul on a bounded sample) and sampled clocks.

Multi-GPU (torchrun, one process per GPU): the same layer split over the ranks
(TensorParallelLayerLinears: q/k/v and gate/up by output rows, o and down by
input columns, one NCCL all-reduce after each) -> strong scaling; value = one
layer's bytes per step / the max-over-ranks time, with the all-reduces' share of
the step reported in ``comm``. The config-4 prefill GEMM splits N over the ranks
with an NCCL all-gather of the outputs; the config-5 FFN splits its intermediate
dimension with one all-reduce.

``--impl reference`` times the reference's own CPU path for the same metric:
gguf.quants.dequantize (gguf-py, the reference's pinned dependency) followed
by a numpy fp32 matmul, on rank 0 only, over a bounded sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vllm-webgpu_b200"))

LAYER = [  # (name, N = out features, K = in features) -- Llama-3-8B layer
    ("q_proj", 4096, 4096), ("k_proj", 1024, 4096), ("v_proj", 1024, 4096), ("o_proj", 4096, 4096),
    ("gate_proj", 14336, 4096), ("up_proj", 14336, 4096), ("down_proj", 4096, 14336),
]
# one decode step = 4 launches: q/k/v and gate/up each fused into one grouped GEMV
GROUPS = [("qkv", (0, 1, 2), 4096), ("o", (3,), 4096), ("gate_up", (4, 5), 4096), ("down", (6,), 14336)]
Q4_K = 12
QK_BYTES = 144 / 256  # bytes per Q4_K weight
METRIC = "Q4_K GEMV HBM GB/s (% of peak); prefill dequant-GEMM TFLOP/s at 1/2/4/8 GPUs"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def layer_bytes(m: int = 1, act_bytes: int = 2, out_bytes: int = 4) -> int:
    """Algorithmic bytes of one layer decode: GGUF weight blocks + x read + y written."""
    total = 0
    for _, n, k in LAYER:
        total += n * k // 256 * 144 + m * k * act_bytes + m * n * out_bytes
    return total


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        rows = [r.split(",") for r in (self.out or "").strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def read_traffic(kernel_tag: str):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", f"{kernel_tag}.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_launch_full_layer_step:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


# ----------------------------------------------------------------------------
# CPU baseline: the reference's quantized matmul arithmetic on host cores
# ----------------------------------------------------------------------------

_CPU_WORK = None


def _cpu_worker_init(seed: int, max_rows: int) -> None:
    """Per-process slabs of the seven projections (valid Q4_K blocks, finite scales)."""
    global _CPU_WORK
    for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[v] = "1"  # one core per worker process
    import numpy as np
    try:
        from gguf import GGMLQuantizationType
        from gguf.quants import dequantize as deq
        qtype = GGMLQuantizationType.Q4_K
    except ImportError:  # the oracle port restates the same arithmetic
        sys.path.insert(0, ROOT)
        from oracle import gguf_oracle as O
        qtype = O.Q4_K

        def deq(raw, qt):
            return O.dequantize(raw, qt)
    rng = np.random.default_rng(seed)
    work = []
    for _, n, k in LAYER:
        rows = min(n, max_rows)
        raw = rng.integers(0, 256, size=(rows, k // 256 * 144), dtype=np.uint8)
        hdr = raw.reshape(rows, -1, 144)
        hdr[:, :, 0:2] = np.array([1e-3], np.float16).view(np.uint8)  # finite d / dmin
        hdr[:, :, 2:4] = np.array([1e-3], np.float16).view(np.uint8)
        work.append((raw, rng.standard_normal((1, k)).astype(np.float32), k))
    _CPU_WORK = (deq, qtype, work)


def _cpu_worker_step(rows: int) -> int:
    """Dequantize ``rows`` rows of each projection and multiply; returns the bytes."""
    deq, qtype, work = _CPU_WORK
    nbytes = 0
    for raw, x, k in work:
        r = min(rows, raw.shape[0])
        w = deq(raw[:r], qtype).reshape(r, k)
        _ = x @ w.T
        nbytes += r * raw.shape[1] + r * 4
    return nbytes


class CpuReference:
    """The reference's quantized-matmul arithmetic on the host cores: gguf-py's
    ``quants.dequantize`` (the reference loader's decoder, its pinned dependency)
    followed by a numpy fp32 matmul, over slabs of rows of the layer's seven Q4_K
    projections at M = 1. One step = ``rows`` rows of every projection, split over
    one worker process per host core (gguf-py's dequantize is single-threaded
    Python + numpy). Bytes per step are the GPU arm's algorithmic bytes (GGUF
    blocks + activations read + outputs written) for the rows processed."""

    def __init__(self, seed: int = 0, max_rows: int = 2048):
        import concurrent.futures as cf
        import multiprocessing as mp
        try:
            import gguf  # noqa: F401
            self.kind, self.how = "reference", "gguf-py 0.19 quants.dequantize + numpy fp32 matmul"
        except ImportError:
            self.kind, self.how = "port", "oracle numpy restatement of gguf dequantize + numpy fp32 matmul"
        self.procs = os.cpu_count() or 1
        self.max_rows = max_rows
        # spawned workers: the GPU arm's process has CUDA initialised, which fork must not copy
        self.pool = cf.ProcessPoolExecutor(self.procs, mp_context=mp.get_context("spawn"),
                                           initializer=_cpu_worker_init, initargs=(seed, max_rows))
        list(self.pool.map(_cpu_worker_step, [1] * self.procs))  # start every worker

    def step(self, rows: int) -> int:
        """One step over ``rows`` rows of each projection (spread over the workers); its bytes."""
        per = max(1, -(-rows // self.procs))
        parts = [per] * (rows // per) + ([rows % per] if rows % per else [])
        nbytes = sum(self.pool.map(_cpu_worker_step, parts))
        return nbytes + len(parts) * sum(k * 2 for _, _, k in LAYER)

    def run(self, steps: int, warmup: int, budget_s: float) -> dict:
        """Time ``steps`` steps after ``warmup``, each sized to about budget_s / (steps + warmup)."""
        t = time.perf_counter()
        self.step(8 * self.procs)
        per_row = (time.perf_counter() - t) / (8 * self.procs)
        target = max(0.002, min(5.0, budget_s / max(1, steps + warmup)))
        rows = int(max(1, min(self.max_rows * self.procs, target / max(per_row, 1e-9))))
        for _ in range(warmup):
            self.step(rows)
        times, nbytes = [], 0
        for _ in range(steps):
            t = time.perf_counter()
            nbytes = self.step(rows)
            times.append(time.perf_counter() - t)
        self.pool.shutdown()
        med = statistics.median(times)
        return {"value": nbytes / med / 1e9, "unit": "GB/s", "cores": self.procs, "kind": self.kind,
                "ms_per_step": med * 1e3, "rows": rows, "bytes_per_step": nbytes,
                "sample": (f"{self.how}; one step = {rows} rows of each of the 7 Llama-3-8B Q4_K projections, "
                           f"M=1 ({nbytes / 1e6:.2f} MB), split over {self.procs} worker processes; median of "
                           f"{steps} timed steps after {warmup} warm-up, {sum(times):.1f} s timed "
                           f"(os.cpu_count()={os.cpu_count()})")}


def cpu_reference_rate(budget_s: float, seed: int = 0) -> dict:
    """The CPU baseline for the GPU arm's line: about ``budget_s`` seconds of steps."""
    ref = CpuReference(seed)
    res = ref.run(steps=10, warmup=1, budget_s=budget_s)
    return {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    # bounded: the whole run ends within a few minutes whatever K is
    res = CpuReference().run(args.steps, args.warmup, budget_s=90.0)
    line = {
        "metric": METRIC, "value": round(res["value"], 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(res["ms_per_step"], 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u4 x fp32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "q4k_llama3_8b_layer_decode_m1", "m": 1, "qtype": "Q4_K",
                   "parallelism": "rank 0 only (CPU)", "rows_per_projection_per_step": res["rows"]},
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(res["value"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------

def run_ours(args, rank: int, world: int) -> None:
    import torch
    import torch.distributed as dist
    from vllm_webgpu_b200 import ops
    from vllm_webgpu_b200.quant.pack import random_weights

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    peaks, peak_src = load_peaks()
    m = 1
    copies = 3
    # weights: 3 copies of the layer (the same seeds on every rank), each split over the
    # ranks Megatron-style by TensorParallelLayerLinears: q/k/v and gate/up by output rows,
    # o and down by input columns with one NCCL all-reduce each. At world 1 it runs the
    # layer's four launches unsplit.
    from vllm_webgpu_b200.tp import TensorParallelLayerLinears
    NAMES = ("q", "k", "v", "o", "gate", "up", "down")
    tps, layers = [], []
    for c in range(copies):
        full = {p: random_weights(n, k, Q4_K, seed=10 * c + i, device=dev)
                for i, (p, (_, n, k)) in enumerate(zip(NAMES, LAYER))}
        tps.append(TensorParallelLayerLinears(full, rank=rank, world=world))
        layers.append([full[p] for p in NAMES] if world == 1 else None)
        del full
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    hid, inter = 4096, 14336
    xs = {"normed": torch.randn((m, hid), generator=g, device=dev).to(torch.bfloat16),
          "attn": torch.randn((m, hid), generator=g, device=dev).to(torch.bfloat16),
          "ffn": torch.randn((m, hid), generator=g, device=dev).to(torch.bfloat16),
          "act": torch.randn((m, inter), generator=g, device=dev).to(torch.bfloat16)}
    h0, h1 = rank * hid // world, (rank + 1) * hid // world
    i0, i1 = rank * inter // world, (rank + 1) * inter // world
    attn_local = xs["attn"][:, h0:h1].contiguous()
    act_local = xs["act"][:, i0:i1].contiguous()
    tp0 = tps[0]
    bufs = {p: torch.empty((m, tp0.w[p].n), dtype=torch.float32, device=dev) for p in ("q", "k", "v", "gate", "up")}
    bufs["o"] = torch.empty((m, hid), dtype=torch.float32, device=dev)
    bufs["down"] = torch.empty((m, hid), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(c: int, collective: bool = True) -> None:
        tps[c].collective = collective
        tps[c](xs["normed"], attn_local, xs["ffn"], act_local, bufs)

    # warm-up (also primes attributes / driver entry points / NCCL before capture)
    for i in range(max(3, args.warmup)):
        step(i % copies)
    torch.cuda.synchronize()

    # CUDA graphs of consecutive steps over the rotating weight copies (launch overhead
    # out of the device time): a 30-step graph replayed, plus one graph for the
    # remainder, so exactly --steps steps are timed
    def capture(nsteps: int, collective: bool = True):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for i in range(nsteps):
                step(i % copies, collective)
        for c in range(copies):
            tps[c].collective = True
        return gr
    chunk = 30
    big = capture(chunk)
    reps, rem = divmod(args.steps, chunk)
    small = capture(rem) if rem else None
    for _ in range(3):
        big.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_run(gbig=None, gsmall=None) -> float:
        if gbig is None:
            gbig, gsmall = big, small
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            gbig.replay()
        if gsmall is not None:
            gsmall.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    steps = args.steps
    # a timed region shorter than ~250 ms is repeated (same K steps each time) so the
    # clock sampler sees it under load; the median repeat is reported
    est = timed_run()
    repeats = int(max_over_ranks(max(1, min(200, int(250.0 / max(est, 1e-3)) + 1))))
    runs = []
    with ClockSampler(local) as clk:
        for _ in range(repeats):
            runs.append(timed_run())
    ms = max_over_ranks(statistics.median(runs))
    step_bytes = layer_bytes(m, act_bytes=2, out_bytes=4)
    # strong scaling: one layer's bytes per step whatever the rank count
    value = step_bytes * steps / (ms / 1e3) / 1e9
    comm = None
    if world > 1:
        # the same steps without the two all-reduces: what the collectives cost
        nb = capture(chunk, collective=False)
        ns = capture(rem, collective=False) if rem else None
        nb.replay()
        torch.cuda.synchronize()
        ms_nc = max_over_ranks(statistics.median([timed_run(nb, ns) for _ in range(max(1, repeats // 2))]))
        comm = {"step_us_without_allreduce": round(ms_nc / steps * 1e3, 2),
                "allreduce_share_of_step": round(max(0.0, 1.0 - ms_nc / ms), 4),
                "allreduces_per_step": 2, "allreduce_bytes": m * hid * 4,
                "collective": ("ggufmm_gemv_allreduce (the o / down GEMV and the all-reduce in one kernel, "
                               "NVLink peer memory, fp32)" if tp0.fused_allreduce else
                               "ggufmm_allreduce (one-shot, NVLink peer memory, fp32)" if tp0.peer_allreduce
                               else "NCCL all_reduce (fp32)")}
        del nb, ns

    # per-launch device time of each launch of the (local) step, each alone in a CUDA
    # graph of 30 launches over the rotating copies; bytes are this rank's share
    LOCAL_GROUPS = [("qkv", ("q", "k", "v"), "normed"), ("o", ("o",), "attn"), ("gate_up", ("gate", "up"), "ffn"),
                    ("down", ("down",), "act")]
    xin = {"normed": xs["normed"], "attn": attn_local, "ffn": xs["ffn"], "act": act_local}

    def launch(c: int, grp) -> None:
        _, ps, xn = grp
        if len(ps) == 1:
            ops.mul_mat(xin[xn], tps[c].w[ps[0]], out=bufs[ps[0]])
        else:
            ops.gemv_grouped(xin[xn], [tps[c].w[p] for p in ps], outs=[bufs[p] for p in ps])

    def group_bytes(ps, xn) -> int:
        ws = [tp0.w[p] for p in ps]
        return sum(w.nbytes + m * w.n * 4 for w in ws) + m * xin[xn].shape[1] * 2
    per, per_bytes = {}, {}
    for grp in LOCAL_GROUPS:
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gg):
            for r in range(30):
                launch(r % copies, grp)
        gg.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(5):
            gg.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        per[grp[0]] = e0.elapsed_time(e1) / 150
        per_bytes[grp[0]] = group_bytes(grp[1], grp[2])
        del gg
    kern_ms = sum(per.values())
    local_bytes = sum(per_bytes.values())
    achieved = local_bytes / (kern_ms / 1e3) / 1e9
    per_frac = {nm: round(per_bytes[nm] / (per[nm] / 1e3) / 1e9 / float(peaks["hbm_gbs"]), 4) for nm in per}

    # end to end through the public API, one CUDA-graph replay per step that copies the
    # step's activations in from pinned host memory (one packed copy), runs the layer's
    # projections (and, at N > 1, the all-reduces) and copies every output back (one
    # packed copy), then a host wait. N = 1: LlamaB200Model.layer_linears_graph (the
    # reference's per-layer projection calls); N > 1: TensorParallelLayerLinears.graph_step.
    if world == 1:
        from vllm_webgpu_b200.models.llama import PROJ, LlamaB200Model
        model = LlamaB200Model(None, device=dev)
        for c in range(copies):
            for i, (nm, _, _) in enumerate(LAYER):
                model.weights[f"model.layers.{c}.{PROJ[nm.split('_')[0]]}"] = layers[c][i]
        in_dims = (("normed", hid), ("attn_out", hid), ("ffn_normed", hid), ("ffn_act", inter))
        out_dims = [(nm.split("_")[0], n) for nm, n, _ in LAYER]
    else:
        in_dims = (("normed", hid), ("attn_out", h1 - h0), ("ffn_normed", hid), ("ffn_act", i1 - i0))
        out_dims = [(p, tp0.w[p].n) for p in ("q", "k", "v", "gate", "up")] + [("o", hid), ("down", hid)]
    kin = sum(kk for _, kk in in_dims)
    hin = torch.randn((m, kin)).to(torch.bfloat16).pin_memory()
    din = torch.empty((m, kin), dtype=torch.bfloat16, device=dev)
    d, off = {}, 0
    for nm, kk in in_dims:
        d[nm] = din[:, off:off + kk]
        off += kk
    nout = sum(n for _, n in out_dims)
    dout = torch.empty((nout * m,), dtype=torch.float32, device=dev)
    hout = torch.empty_like(dout, device="cpu").pin_memory()
    ebufs, off = {}, 0
    for nm, n in out_dims:
        ebufs[nm] = dout[off:off + m * n].view(m, n)
        off += m * n
    e2e_steps = max(30, min(2000, steps // 10))
    h2d = hin.numel() * 2
    d2h = dout.numel() * 4

    def run_graph(c: int, stage: bool) -> None:
        si, so = ([(din, hin)], [(hout, dout)]) if stage else ((), ())
        if world == 1:
            model.layer_linears_graph(c, d["normed"], d["attn_out"], d["ffn_normed"], d["ffn_act"], ebufs,
                                      stage_in=si, stage_out=so)
        else:
            tps[c].graph_step(d["normed"], d["attn_out"], d["ffn_normed"], d["ffn_act"], ebufs, stage_in=si,
                              stage_out=so)

    done = torch.cuda.Event()

    def host_wait() -> None:
        # spin on an event recorded after the step (a blocking stream sync adds the
        # thread's wake-up latency to every step)
        done.record(stream)
        while not done.query():
            pass

    def e2e_step(c: int) -> None:
        run_graph(c, True)
        host_wait()

    for i in range(5):
        e2e_step(i % copies)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i % copies)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = step_bytes * e2e_steps / (e2e_ms / 1e3) / 1e9

    # where an end-to-end step goes: each part alone with a host wait, host wall clock
    def host_us(fn, n=200) -> float:
        for _ in range(5):
            fn()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        return (time.perf_counter() - t0) / n * 1e6

    def only_h2d():
        din.copy_(hin, non_blocking=True)
        host_wait()

    def only_graph():
        run_graph(0, False)
        host_wait()

    def only_d2h():
        hout.copy_(dout, non_blocking=True)
        host_wait()
    e2e_parts = {"h2d_and_wait_us": round(host_us(only_h2d), 2), "graph_replay_and_wait_us": round(host_us(only_graph), 2),
                 "d2h_and_wait_us": round(host_us(only_d2h), 2), "step_us": round(e2e_ms / e2e_steps * 1e3, 2),
                 "device_step_us": round(ms / steps * 1e3, 2)}
    del ebufs

    # prefill (config 4): Q4_K / Q6_K GEMM, K=4096, N=14336, M in {512, 2048, 8192} on the
    # tensor cores, bf16 out; the headline key is Q4_K at M = 2048. At N > 1 the weight's
    # N dimension is split over the ranks (each computes [M, N/P]) and an NCCL
    # all-gather collects the [P, M, N/P] outputs on every rank; TFLOP/s is the whole
    # GEMM's 2 M N K over the max-over-ranks time, with the all-gather's share reported.
    pre = None
    prefill_sweep = None
    if not args.no_prefill:
        pn, pk = 14336, 4096
        r0, r1 = rank * pn // world, (rank + 1) * pn // world
        wts = {}
        for qt, sd in ((Q4_K, 4), (14, 77)):
            wfull = random_weights(pn, pk, qt, seed=sd, device=dev)
            wts[qt] = wfull if world == 1 else wfull.rows(r0, r1)
            del wfull
        prefill_sweep = {}
        for qt, qname in ((Q4_K, "q4_k"), (14, "q6_k")):
            for pm in (512, 2048, 8192):
                xp = torch.randn((pm, pk), device=dev).to(torch.bfloat16)
                yp = torch.empty((pm, r1 - r0), dtype=torch.bfloat16, device=dev)
                yg = torch.empty((world * pm, r1 - r0), dtype=torch.bfloat16, device=dev) if world > 1 else None

                pg = ops.PeerGather(pm, pn, torch.bfloat16, device=dev) if world > 1 else None

                def pstep(gather: bool = True) -> None:
                    if world > 1 and gather:
                        # the all-gather in the GEMM's epilogue (peer stores over NVLink) + a device barrier
                        ops.gemm_allgather(xp, wts[qt], pg)
                    else:
                        ops.gemm(xp, wts[qt], out=yp)

                def pstep_nccl() -> None:
                    ops.gemm(xp, wts[qt], out=yp)
                    dist.all_gather_into_tensor(yg, yp)
                for _ in range(3):
                    pstep()
                torch.cuda.synchronize()
                it = max(3, int(2e12 / (2.0 * pm * pn * pk)))  # ~10 ms of work at least

                def ptime(gather: bool, fn=None) -> float:
                    if world > 1:
                        dist.barrier()
                    torch.cuda.synchronize()
                    e0.record(stream)
                    for _ in range(it):
                        if fn is not None:
                            fn()
                        else:
                            pstep(gather)
                    e1.record(stream)
                    torch.cuda.synchronize()
                    return max_over_ranks(e0.elapsed_time(e1) / it)
                pms = ptime(True)
                tf = 2.0 * pm * pn * pk / (pms / 1e3) / 1e12
                rec = {"ms": round(pms, 4), "tflops": round(tf, 2),
                       "frac_of_bf16_peak": round(tf / world / peaks["bf16_tflops"], 4)}
                if world > 1:
                    pms_ng = ptime(False)
                    pstep_nccl()
                    pms_nccl = ptime(True, pstep_nccl)
                    rec["ms_epilogue_allgather"] = round(pms, 4)
                    rec["ms_gemm_then_nccl_allgather"] = round(pms_nccl, 4)
                    # the faster of the two gathers is the reported step (both are this
                    # library's paths: the GEMM whose epilogue stores into every GPU, or the
                    # GEMM followed by NCCL's all-gather)
                    best = min(pms, pms_nccl)
                    tf = 2.0 * pm * pn * pk / (best / 1e3) / 1e12
                    rec.update({"ms": round(best, 4), "tflops": round(tf, 2),
                                "frac_of_bf16_peak": round(tf / world / peaks["bf16_tflops"], 4),
                                "gather": "epilogue" if pms <= pms_nccl else "nccl",
                                "allgather_share": round(max(0.0, 1.0 - pms_ng / best), 4),
                                "ms_without_allgather": round(pms_ng, 4)})
                prefill_sweep[f"{qname}_m{pm}"] = rec
                del xp, yp, yg, pg
        p2 = prefill_sweep["q4_k_m2048"]
        pre = {"workload": "q4k_prefill_m2048_k4096_n14336", **p2,
               "path": ("dequant->fp16 + cast->fp16 workspace, persistent tcgen05 GEMM (3 kernels)"
                        + ("" if world == 1 else f"; N split over {world} ranks, all-gather "
                           + ("in the GEMM epilogue (peer stores over NVLink) + device barrier"
                              if p2.get("gather") == "epilogue" else "by NCCL after the GEMM")))}
        del wts

    # BASELINE configs 1 and 2 on the GPU: Q8_0 4096 x 4096 matvec with fp32 x, and the
    # Q4_0 14336 x 4096 GEMV at M in {1, 4, 8} with fp16 x; weight copies rotated past L2
    other = None
    if not args.no_configs and world == 1:
        other = {}
        for key, qt, n, k, ms_, xdt, ncopy in (("config1_q8_0_matvec_f32", 8, 4096, 4096, (1,), torch.float32, 8),
                                              ("config2_q4_0_gemv_f16", 2, 14336, 4096, (1, 4, 8), torch.float16, 5)):
            ws_ = [random_weights(n, k, qt, seed=500 + c, device=dev) for c in range(ncopy)]
            wb = ws_[0].nbytes
            other[key] = {"l2": f"{ncopy} rotating weight copies ({ncopy * wb / 1e6:.0f} MB > 126 MB L2)"}
            for mm in ms_:
                xo = torch.randn((mm, k), generator=g, device=dev).to(xdt)
                yo = torch.empty((mm, n), dtype=torch.float32, device=dev)
                gr = torch.cuda.CUDAGraph()
                for c in range(ncopy):
                    ops.gemv(xo, ws_[c], out=yo)
                torch.cuda.synchronize()
                with torch.cuda.graph(gr):
                    for r in range(10 * ncopy):
                        ops.gemv(xo, ws_[r % ncopy], out=yo)
                gr.replay()
                torch.cuda.synchronize()
                e0.record(stream)
                for _ in range(10):
                    gr.replay()
                e1.record(stream)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) / (100 * ncopy) * 1e3
                byts = wb + mm * k * xo.element_size() + mm * n * 4
                other[key][f"m{mm}"] = {"us": round(us, 2), "gbs": round(byts / us / 1e3, 1),
                                        "frac_of_hbm": round(byts / us / 1e3 / float(peaks["hbm_gbs"]), 4),
                                        "kernel": ["stream", "f16_tc", "int8_tc"][ops.gemv_kernel(mm, ws_[0], xdt)]}
            del ws_

    # batched decode of the same layer (config 3 at M = 16 and 64): above M = 8 q/k/v and
    # gate/up run as grouped fused-dequant tcgen05 GEMMs, o and down through ops.mul_mat
    # (split over the ranks with the all-reduces at N > 1), replayed from a CUDA graph
    # over the rotating weight copies
    batched = None
    if not args.no_batched:
        batched = {"workload": "q4k_llama3_8b_layer_decode", "path": "4 launch groups: ops.gemm_grouped (q/k/v, "
                   "gate/up) and ops.mul_mat (o, down); fused-dequant tcgen05 GEMM, K split where the "
                   "weights have few 128-row tiles" + ("" if world == 1 else f"; tp{world} with 2 all-reduces")}
        wbytes = sum(n * k // 256 * 144 for _, n, k in LAYER)
        for mb in (16, 64):
            xb = {nm: torch.randn((mb, kk), generator=g, device=dev).to(torch.bfloat16)
                  for nm, kk in (("normed", hid), ("attn", h1 - h0), ("ffn", hid), ("act", i1 - i0))}
            yb = {p: torch.empty((mb, tp0.w[p].n), dtype=torch.bfloat16, device=dev) for p in ("q", "k", "v", "gate", "up")}
            yb["o"] = torch.empty((mb, hid), dtype=torch.float32, device=dev)
            yb["down"] = torch.empty((mb, hid), dtype=torch.float32, device=dev)

            def bstep(c: int) -> None:
                tps[c](xb["normed"], xb["attn"], xb["ffn"], xb["act"], yb)

            for i in range(3):
                bstep(i % copies)
            torch.cuda.synchronize()
            bg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(bg):
                for c in range(copies):
                    bstep(c)
            bg.replay()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            reps_b = 20
            e0.record(stream)
            for _ in range(reps_b):
                bg.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            bms = max_over_ranks(e0.elapsed_time(e1) / (reps_b * copies))
            batched[f"m{mb}"] = {"us_per_step": round(bms * 1e3, 2), "weight_gbs": round(wbytes / (bms / 1e3) / 1e9, 2),
                                 "tflops": round(2.0 * mb * wbytes / 144 * 256 / (bms / 1e3) / 1e12, 2)}
            del bg

    # tensor-parallel SwiGLU FFN (config 5): Llama-3-70B shape, Q4_K, intermediate split over
    # the ranks, one NCCL all-reduce per step, M in {1, 32, 2048}
    tpf = None
    if not args.no_tp:
        from vllm_webgpu_b200.tp import TensorParallelSwiGLU
        hid, inter = 8192, 28672
        full = [random_weights(inter, hid, Q4_K, seed=901, device=dev), random_weights(inter, hid, Q4_K, seed=902, device=dev),
                random_weights(hid, inter, Q4_K, seed=903, device=dev)]
        ffn = TensorParallelSwiGLU(*full, rank=rank, world=world)
        del full
        wbytes = 3 * hid * inter // 256 * 144
        tpf = {"workload": "q4k_llama3_70b_ffn_tp", "tp": world, "weight_bytes_total": wbytes,
               "path": "fused gate/up/SwiGLU GEMV (M<=8) or GEMM with the SwiGLU epilogue, down projection, "
                       "all-reduce (one-shot peer-memory kernel up to 65536 values, NCCL above); "
                       "CUDA graph replay"}
        for mt in (1, 32, 2048):
            xt = torch.randn((mt, hid), generator=g, device=dev).to(torch.bfloat16)
            for _ in range(3):
                ffn(xt)
            torch.cuda.synchronize()
            # captured as a CUDA graph (the NCCL all-reduce included), replayed
            reps_f = 10 if mt <= 32 else 2
            fg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(fg):
                for _ in range(reps_f):
                    ffn(xt)
            fg.replay()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            it = 10
            e0.record(stream)
            for _ in range(it):
                fg.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            tms = max_over_ranks(e0.elapsed_time(e1) / (it * reps_f))
            rec = {"us_per_step": round(tms * 1e3, 2), "weight_gbs": round(wbytes / (tms / 1e3) / 1e9, 2)}
            if mt >= 2048:
                rec["tflops"] = round(6.0 * mt * hid * inter / (tms / 1e3) / 1e12, 2)
            tpf[f"m{mt}"] = rec
            del fg
        del ffn

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference_rate(args.cpu_seconds)

    if rank == 0:
        clocks = clk.summary()
        peak = float(peaks["hbm_gbs"])
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "timed_repeats": repeats,
            "warmup": args.warmup, "ms_per_step": round(ms / steps, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u4 x bf16 -> fp32", "data": "synthetic",
            "config": {"workload": "q4k_llama3_8b_layer_decode_m1", "m": 1, "qtype": "Q4_K",
                       "projections": {nm: [k, n] for nm, n, k in LAYER},
                       "weight_bytes_per_step": sum(n * k // 256 * 144 for _, n, k in LAYER),
                       "bytes_per_step": step_bytes, "l2": "3 rotating weight copies (368 MB > 126 MB L2)",
                       "graph": "CUDA graphs of 30 consecutive steps (+ one of the remainder), K steps per timed region, median of the repeated regions", "launches_per_step": [g[0] for g in GROUPS],
                       "parallelism": (f"tp{world}: q/k/v and gate/up split by output rows, o and down by input "
                                       f"columns, 2 all-reduces per step" if world > 1 else "tp1")},
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "kernel": "gemv_i8_kernel<Q4_K>", "achieved": round(achieved, 2),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": read_traffic("gemv_q4k_layer_m1"), "peak_source": peak_src,
                         "per_launch_us": {nm: round(v * 1e3, 2) for nm, v in per.items()},
                         "per_launch_frac": per_frac},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "breakdown": e2e_parts,
                    "path": ("LlamaB200Model.layer_linears_graph" if world == 1 else "TensorParallelLayerLinears.graph_step")
                    + " (one CUDA-graph replay per step holding the packed host-to-device copy of the "
                      "activations from pinned host memory, the projections and the packed device-to-host copy "
                      "of every output, the copies made by the ggufmm_stage_copy kernel over the bus"
                    + (", GGUFMM_STAGE_KERNEL=0: copy-engine memcpys" if os.environ.get("GGUFMM_STAGE_KERNEL") == "0" else "")
                    + "), and a host wait per step (spin on an event)"},
            "gpu_launches": len(GROUPS) * steps * repeats,
            "comm": comm,
            "clocks": clocks,
            "prefill": pre,
            "prefill_sweep": prefill_sweep,
            "configs_1_2": other,
            "decode_batched": batched,
            "tp_ffn": tpf,
            "cpu_baseline": cpu,
        }
        emit(line)


_JSON_OUT = None


def emit(line: dict) -> None:
    """The one JSON line, on the process's real stdout (libraries' banners -- NCCL's
    version line among them -- are sent to stderr while the bench runs)."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=15000)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-tp", action="store_true")
    ap.add_argument("--no-batched", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")  # the real stdout, for the JSON line only
    os.dup2(2, 1)                          # everything else printed on fd 1 goes to stderr
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        # NCCL prints its version banner on stdout at VERSION level; the driver reads one JSON line
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    try:
        run_ours(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
