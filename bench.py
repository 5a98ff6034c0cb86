"""Benchmark of the B200 depthwise Conv1D training path (FWD + dX + dK, FP32).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one FWD + dX + dK pass (dK deterministic two-pass, written, not
accumulated, so no zero-fill exists) over one batch of the primary workload,
B=16384 per GPU, H=128, L=48, K=48 (weak scaling: at N=8 the job is the
batch-sharded x[131072,128,48] configuration; for N>1 each step also sums
dK[128,48] over the ranks, through NVLink peer memory inside the backward
kernel, or with the NCCL all-reduce that is timed beside it).  Inputs are resident in HBM and each of
x, dy, y, dX is 402 MB, larger than the 126 MB L2, so no L2 flush is needed.

Printed (rank 0, one JSON line): ``value`` = whole-job effective GB/s of
FWD+dX+dK -- the reference's byte formula, (2*B*H*L + H*K)*4 per phase, three
phases -- over the device-timed step (CUDA events, max over ranks; the step's
backward is one fused kernel, which moves fewer bytes than the formula
credits, see ``step_moved_bytes``); ``aggregate_ms`` = the sum of the three
phases timed separately under the reference's protocol (each phase: 3 trials
of 50 untimed + 100 timed launches, mean of the trial means; outputs and the
dK workspace allocated before timing); ``roofline`` for the dominant kernel of
the step, its duration taken inside the timed steps (CUDA events between the
step's kernels, on the launching stream); ``cpu_baseline`` = the reference's PyTorch CPU path timed on this
host under the reference's protocol (1-GPU runs only); ``e2e`` = the same pass
through the host-buffer API (pinned host tensors, copies inside the timed
region); ``clocks`` sampled by NVML during the timed region (and per phase).
For N > 1, ``step_split`` gives the NCCL variant's ``compute_ms`` and
``allreduce_ms`` (max over ranks).

``--impl reference`` times the reference's own CPU implementation (its PyTorch
path F.pad + grouped conv1d with autograd, restated in oracle/) on this host's
cores under the reference's protocol (FWD, dX and dK timed separately, the
autograd graph built outside the timed region, summed), on a bounded sample of
the same workload, and prints the same metric; where the reference's own CUDA
kernels were built for sm_100a (oracle/_ref) it adds their times on this GPU.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "FWD+dX+dK aggregate ms & GB/s at B=16384,H=128,L=48,K=48 FP32; % roofline"
B_PER_GPU, H, L, K = 16384, 128, 48, 48
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "source": "fallback"}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    return dict(FALLBACK_PEAKS)


# ---------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01) -> None:
        self.idx, self.period = device_index, period_s
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception as exc:  # NVML missing: report no samples, never guess
            self._nv = None
            self.error = repr(exc)

    def _run(self) -> None:
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(int(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)))
                mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()
        return False

    def summary(self) -> dict:
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons - {"gpu_idle"})}


# ---------------------------------------------------------------------------
# Device-resident timing
# ---------------------------------------------------------------------------
def phase_bytes(B: int) -> int:
    return (2 * B * H * L + H * K) * 4


def time_loop(fn, iters: int, stream) -> float:
    """Mean ms of fn() over iters, CUDA events on `stream`, synchronised on both sides."""
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(iters):
        fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / iters


# The reference's GPU timing protocol (artifact/REPRODUCIBILITY.md:79-121,
# kernels/warp_tiled_ampere.py:1040-1084): 3 trials x (50 warm-up + 100 timed
# launches) per phase, phases timed separately.
PHASE_TRIALS, PHASE_WARMUP, PHASE_RUNS = 3, 50, 100
STEADY_S = 0.6  # interleaved warm-up before the phase trials (see run_ours)


def time_phase(fn, stream, device_index: int, pre=None, trials: int = PHASE_TRIALS, warmup: int = PHASE_WARMUP,
               runs: int = PHASE_RUNS) -> dict:
    """One phase under the reference protocol: per trial, `warmup` untimed launches
    then `runs` timed ones (CUDA events on the launching stream); the phase time
    is the mean of the trial means (the reference reports that; the median is
    kept beside it).  With `pre` (e.g. a zero-fill the reference
    keeps outside the timed region) every launch is bracketed by its own events,
    with `pre` before the start event."""
    trial_ms = []
    with ClockSampler(device_index) as clk:
        for _ in range(trials):
            for _ in range(warmup):
                if pre is not None:
                    pre()
                fn()
            if pre is None:
                trial_ms.append(time_loop(fn, runs, stream))
                continue
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(runs)]
            torch.cuda.synchronize()
            for a, b in ev:
                pre()
                a.record(stream)
                fn()
                b.record(stream)
            torch.cuda.synchronize()
            trial_ms.append(statistics.mean(a.elapsed_time(b) for a, b in ev))
    return {"ms": statistics.mean(trial_ms), "median_ms": statistics.median(trial_ms), "trials_ms": trial_ms,
            "clocks": clk.summary()}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_protocol(B: int, warmup: int = 5, runs: int = 30, seed: int = 42) -> dict:
    """The reference's PyTorch path on this host's CPU cores under the reference's
    own protocol (benchmark/benchmark_pytorch.py:22-24, 80-144): FWD timed around
    pad + conv; dX and dK timed around torch.autograd.grad only, each run's
    forward graph built outside the timed region; 5 warm-up + 30 timed runs per
    phase, perf_counter.  The path is restated in oracle/reference_torch.py (the
    reference module imports pycuda, which this host lacks)."""
    from oracle import reference_torch as ref

    torch.set_num_threads(os.cpu_count() or 1)
    x, k, dy = ref.make_inputs(B, H, L, K, seed=seed)
    xr = x.clone().requires_grad_(True)
    kr = k.clone().requires_grad_(True)

    def fwd():
        with torch.no_grad():
            t0 = time.perf_counter()
            ref.depthwise_same(x, k)
            return time.perf_counter() - t0

    def dx():
        y = ref.depthwise_same(xr, k)
        t0 = time.perf_counter()
        torch.autograd.grad(y, xr, dy)
        return time.perf_counter() - t0

    def dk():
        y = ref.depthwise_same(x, kr)
        t0 = time.perf_counter()
        torch.autograd.grad(y, kr, dy)
        return time.perf_counter() - t0

    phases = {}
    for name, fn in (("fwd", fwd), ("bwd_input", dx), ("bwd_weight", dk)):
        for _ in range(warmup):
            fn()
        ts = [1e3 * fn() for _ in range(runs)]
        phases[name] = {"median_ms": statistics.median(ts), "mean_ms": statistics.mean(ts)}
    agg = sum(p["mean_ms"] for p in phases.values())
    return {"B": B, "phase_ms": {n: p["mean_ms"] for n, p in phases.items()},
            "phase_median_ms": {n: p["median_ms"] for n, p in phases.items()},
            "aggregate_ms": agg, "GB/s": 3 * phase_bytes(B) / (agg / 1e3) / 1e9}


def cpu_baseline(B_sample: int = 1024) -> dict:
    """The reference's PyTorch CPU path on this host (reported baseline, not the target):
    the bounded sample of the primary shape, plus BASELINE's CPU configuration (B=64)."""
    main = cpu_protocol(B_sample)
    small = cpu_protocol(64)
    return {
        "value": main["GB/s"],
        "unit": "GB/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "cpu_model": cpu_model(),
        "aggregate_ms": main["aggregate_ms"],
        "phase_ms": main["phase_ms"],
        "phase_median_ms": main["phase_median_ms"],
        "config0_B64": {k_: small[k_] for k_ in ("phase_ms", "aggregate_ms", "GB/s")},
        "sample": (f"B={B_sample} of the primary shape (H=128,L=48,K=48), and B=64 (the CPU config); reference "
                   "PyTorch CPU path F.pad + conv1d(groups=H), FWD / dX / dK timed separately with the autograd "
                   "graph built outside the timed region, 5 warm-up + 30 timed runs per phase (the reference's "
                   "benchmark_pytorch.py protocol), mean per phase summed; restated in oracle/reference_torch.py"),
    }


def load_traffic() -> dict | None:
    p = ROOT / "profiles" / "dram_traffic_primary.json"
    if p.exists():
        return json.loads(p.read_text())
    return None


def apply_engine(ops, engine: str) -> None:
    """--engine: "frozen" keeps the frozen table; "ffma" / "tensor" force every path onto
    that engine where it applies (shapes it does not cover keep the FFMA kernels)."""
    if engine != "frozen":
        for p in ("fwd", "bwd_input", "bwd_weight"):
            ops.set_engine(p, engine)


def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    from pathtile_b200 import build, ops, runtime
    from pathtile_b200 import host as hostmod
    from pathtile_b200.host import HostPipeline

    build.build()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    apply_engine(ops, args.engine)
    dist = None
    if world > 1:
        import torch.distributed as dist
    B = args.batch
    g = torch.Generator(device=dev).manual_seed(42 + rank)
    x = torch.randn(B, H, L, device=dev, generator=g)
    k = torch.randn(H, K, device=dev, generator=torch.Generator(device=dev).manual_seed(42)) / (K ** 0.5)
    dy = torch.randn(B, H, L, device=dev, generator=g)
    y = torch.empty_like(x)
    gx = torch.empty_like(x)
    gk = torch.empty_like(k)
    stream = torch.cuda.current_stream(dev)

    fused = args.backward == "fused"
    # N > 1: dK summed over the ranks through the peers' exchange buffers (inside
    # the fused backward kernel where it applies), or by an NCCL all-reduce.
    exchange = None
    exchange_note = None
    if dist is not None and args.collective == "fused":
        from pathtile_b200.distributed import PeerExchange, PeerExchangeUnavailable, dx_dk_allreduce, peer_fused

        try:
            exchange = PeerExchange(H, K, dev)
        except PeerExchangeUnavailable as exc:  # every rank falls back alike
            exchange_note = f"peer exchange unavailable ({exc}); NCCL all_reduce used"

    def compute(nccl: bool = False, mid=None):
        ops.fwd(x, k, y)
        if mid is not None:  # between the FWD and the backward: splits the step per kernel
            mid.record(stream)
        if exchange is not None and not nccl:
            dx_dk_allreduce(dy, x, k, gk, exchange, gx=gx)
        elif fused:
            ops.dx_dk(dy, x, k, gk, gx=gx, mode="deterministic")
        else:
            ops.dx(dy, k, gx)
            ops.dk(dy, x, gk, mode="deterministic")

    def step(nccl: bool = False, mid=None):
        compute(nccl, mid)
        if dist is not None and (exchange is None or nccl):
            dist.all_reduce(gk)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    # Events between the kernels of each timed step give every kernel's device
    # time inside the timed region (the roofline figure below); for N > 1 with
    # NCCL they also split off the all-reduce.  They are recorded on the
    # launching stream and add no device work.
    marks = []
    in_step = []  # per step: (step start, after FWD, after the backward)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record(stream)
        for _ in range(args.steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record(stream)
            compute(mid=ev[3])
            ev[1].record(stream)
            if dist is not None and exchange is None:
                dist.all_reduce(gk)
            ev[2].record(stream)
            in_step.append((ev[0], ev[3], ev[1]))
            if dist is not None and exchange is None:
                marks.append(ev[:3])
        e_ev.record(stream)
        e_ev.synchronize()
        step_ms = s_ev.elapsed_time(e_ev) / args.steps
    step_fwd_ms = statistics.mean(a.elapsed_time(m) for a, m, _ in in_step)
    step_bwd_ms = statistics.mean(m.elapsed_time(b) for _, m, b in in_step)
    split = None
    if dist is not None:
        if exchange is not None:
            # The same step with the NCCL all-reduce after the backward, for comparison.
            for _ in range(args.warmup):
                step(nccl=True)
            torch.cuda.synchronize()
            dist.barrier()
            for _ in range(args.steps):
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                ev[0].record(stream)
                compute(nccl=True)
                ev[1].record(stream)
                dist.all_reduce(gk)
                ev[2].record(stream)
                marks.append(ev)
            torch.cuda.synchronize()
        nccl_step = statistics.mean(a.elapsed_time(c) for a, _, c in marks)
        comp = statistics.mean(a.elapsed_time(b) for a, b, _ in marks)
        red = statistics.mean(b.elapsed_time(c) for _, b, c in marks)
        t = torch.tensor([step_ms, comp, red, nccl_step, step_fwd_ms, step_bwd_ms], device=dev,
                         dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, comp, red, nccl_step, step_fwd_ms, step_bwd_ms = map(float, t.tolist())
        split = {"collective": ("dK summed inside the backward kernel through the peers' memory (NVLink)"
                                if exchange is not None and peer_fused(B, H, L, K) else
                                "peer-memory sum kernel after the backward" if exchange is not None else
                                exchange_note or "NCCL all_reduce after the backward"),
                 "nccl_variant": {"step_ms": nccl_step, "compute_ms": comp, "allreduce_ms": red}}

    # Per-phase times under the reference protocol, each phase timed separately.
    # Outputs exist already; the dK workspace is allocated by a call outside the
    # timed trials.  First the phases run interleaved for STEADY_S seconds, as
    # the reference warms all paths up before timing (kernels/warp_tiled_ampere.py:
    # 1040-1046): a B200 that goes from idle to full load dips its SM clock under
    # the power cap for a fraction of a second while the power ramps (measured:
    # 1575-1850 MHz for ~0.5 s, then 1965 MHz), which otherwise lands in the first
    # phase's first trials.
    ops.dk(dy, x, gk, mode="deterministic")
    torch.cuda.synchronize()
    t_end = time.perf_counter() + STEADY_S
    while time.perf_counter() < t_end:
        ops.fwd(x, k, y)
        ops.dx(dy, k, gx)
        ops.dk(dy, x, gk, mode="deterministic")
        if fused:
            ops.dx_dk(dy, x, k, gk, gx=gx, mode="deterministic")
        torch.cuda.synchronize()
    phases = {
        "fwd": time_phase(lambda: ops.fwd(x, k, y), stream, local_rank),
        "bwd_input": time_phase(lambda: ops.dx(dy, k, gx), stream, local_rank),
        "bwd_weight": time_phase(lambda: ops.dk(dy, x, gk, mode="deterministic"), stream, local_rank),
    }
    if fused:
        phases["bwd_fused"] = time_phase(lambda: ops.dx_dk(dy, x, k, gk, gx=gx, mode="deterministic"), stream,
                                         local_rank)
    phase_ms = {p: v["ms"] for p, v in phases.items()}
    if dist is not None:
        t = torch.tensor(list(phase_ms.values()), device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        phase_ms = dict(zip(phase_ms, map(float, t.tolist())))

    if args.no_e2e:
        err = ops.device_error()
        if exchange is not None:
            exchange.close()
        if rank == 0:
            print(json.dumps({"profile_run": True, "B": B, "ms_per_step": step_ms, "phase_ms": phase_ms,
                              "device_error_word": err}), flush=True)
        return None
    # End to end through the host-buffer API: pinned host inputs in, host outputs back.
    # The host buffers are allocated (and the copies driven) from the CPUs local to
    # this rank's GPU, then the process's own CPU set comes back for the CPU baseline.
    numa = contextlib.ExitStack()
    host_cpus = [] if args.no_numa_bind else numa.enter_context(hostmod.near_device(dev))
    pin = dict(device="cpu", pin_memory=True)
    x_h = torch.empty(B, H, L, **pin)
    dy_h = torch.empty(B, H, L, **pin)
    k_h = torch.empty(H, K, **pin)
    x_h.copy_(x)
    dy_h.copy_(dy)
    k_h.copy_(k)
    y_h = torch.empty(B, H, L, **pin)
    gx_h = torch.empty(B, H, L, **pin)
    gk_h = torch.empty(H, K, **pin)
    pipe = HostPipeline(H, L, K, chunk_b=args.e2e_chunk, device=local_rank)

    def e2e_step():
        pipe.run(x_h, k_h, dy_h, y_h, gx_h, gk_h)
        if dist is not None:
            dist.all_reduce(pipe.gk)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e2e_iters = max(3, min(args.e2e_steps, args.steps))
    e2e_ms = time_loop(e2e_step, e2e_iters, stream)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d, d2h = pipe.bytes_per_call(B)
    err = ops.device_error()
    numa.close()
    if exchange is not None:
        exchange.close()

    if rank != 0:
        return None
    peaks = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    pb = phase_bytes(B)
    total_bytes = 3 * pb * world
    fused_on = fused and ops.fused_backward(B, H, L, K)
    step_kernels = ("fwd", "bwd_fused") if fused_on else ("fwd", "bwd_input", "bwd_weight")
    # Algorithmic bytes of a launch: FWD / dX / dK move two activations + k; the
    # fused backward reads dy and x, writes dx, reads k and writes dK.
    kernel_bytes = {p: pb for p in ("fwd", "bwd_input", "bwd_weight")}
    kernel_bytes["bwd_fused"] = (3 * B * H * L + 2 * H * K) * 4
    step_moved = kernel_bytes["fwd"] + (kernel_bytes["bwd_fused"] if fused_on else 2 * pb)
    # The dominant kernel's duration inside the timed steps (events between the
    # step's two kernels); with dX then dK the backward is two launches, and the
    # separately timed phases stand in.
    if fused_on:
        in_step_ms = {"fwd": step_fwd_ms, "bwd_fused": step_bwd_ms}
        dominant = max(step_kernels, key=in_step_ms.get)
        dominant_ms, measured_in = in_step_ms[dominant], f"the {args.steps} timed steps (CUDA events between the step's kernels)"
    else:
        dominant = max(step_kernels, key=phase_ms.get)
        dominant_ms, measured_in = phase_ms[dominant], "its phase loop (reference protocol)"
    achieved = kernel_bytes[dominant] / (dominant_ms / 1e3) / 1e9
    sm_mhz = clocks.summary()["sm_mhz"] or 1965.0
    fma_peak = runtime.fp32_fma_peak_tflops(torch.cuda.get_device_properties(dev).multi_processor_count,
                                            float(sm_mhz))
    roof_ms = runtime.roofline_ms(B, H, L, K, hbm, fma_peak)
    traffic = load_traffic()
    engines = {p: ops.config(p, B, H, L, K)["engine"] for p in ("fwd", "bwd_input", "bwd_weight")}
    kernel_names = {
        "fwd": ("tc_conv_kernel<FWD> (tcgen05, 3xTF32, A in TMEM)" if engines["fwd"] == "tensor"
                else "conv_rows_kernel<48,48,FWD,TMA3D>"),
        "bwd_input": ("tc_conv_kernel<DX> (tcgen05, 3xTF32, A in TMEM)" if engines["bwd_input"] == "tensor"
                      else "conv_rows_kernel<48,48,DX,TMA3D>"),
        "bwd_weight": ("tc_dk_kernel (tcgen05) + tc_dk_reduce_kernel" if engines["bwd_weight"] == "tensor"
                       else "dk_rows_kernel<48,48,TMA3D> + dk_reduce_kernel"),
        "bwd_fused": "tc_bwd_kernel<48> (dX on tcgen05 3xTF32, dK on FFMA, one pass over dy and x)",
    }
    result = {
        "metric": METRIC,
        "value": total_bytes / (step_ms / 1e3) / 1e9,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: x, dy ~ N(0,1), k ~ N(0,1)/sqrt(K), seeded, generated on device",
        "config": {
            "workload": "primary: B=16384 per GPU, H=128, L=48, K=48 (N=8: batch-sharded x[131072,128,48])",
            "B_per_gpu": B, "global_batch": B * world, "H": H, "L": L, "K": K,
            "parallelism": f"dp{world}" + ((" + dK summed over NVLink peer memory" if exchange is not None
                                             else " + NCCL all_reduce(dK)") if world > 1 else ""),
            "dk_mode": "deterministic",
            "backward": ("fused dX+dK kernel (ops.dx_dk)" if fused_on else "dX then dK"),
            "engines": engines,
            "l2": "inputs larger than L2 (402,653,184 B per activation tensor vs 126 MB L2)",
        },
        "value_kind": ("effective: the reference's byte formula (3 phases of (2*B*H*L + H*K)*4 B) over the "
                       "measured step; the step itself moves step_moved_bytes"),
        "step_moved_bytes": step_moved * world,
        "aggregate_ms": sum(phase_ms[p] for p in ("fwd", "bwd_input", "bwd_weight")),
        "aggregate_protocol": (f"each phase separately, after {STEADY_S} s of the phases interleaved: "
                               f"{PHASE_TRIALS} trials x ({PHASE_WARMUP} untimed + {PHASE_RUNS} timed launches), "
                               "mean of the trial means (CUDA events), as the reference reports"),
        "phases": {p: {"ms": ms, "GB/s": kernel_bytes[p] / (ms / 1e3) / 1e9,
                       **({"frac_of_roofline": roof_ms / ms} if p != "bwd_fused" else
                          {"frac_of_hbm": kernel_bytes[p] / (ms / 1e3) / 1e9 / hbm}),
                       "median_ms": phases[p]["median_ms"], "trials_ms": phases[p]["trials_ms"],
                       "sm_mhz": phases[p]["clocks"]["sm_mhz"], "clock_reasons": phases[p]["clocks"]["reasons"]}
                   for p, ms in phase_ms.items()},
        "aggregate_frac_of_roofline": 3 * roof_ms / sum(phase_ms[p] for p in ("fwd", "bwd_input", "bwd_weight")),
        "roofline": {
            "bound": "hbm",
            "kernel": kernel_names[dominant],
            "achieved": achieved,
            "peak": hbm,
            "unit": "GB/s",
            "frac": achieved / hbm,
            "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)" if peaks["source"] == "measured" else "fallback",
            "algorithmic_bytes_per_launch": kernel_bytes[dominant],
            "kernel_ms": dominant_ms,
            "measured_in": measured_in,
            "in_step_ms": {"fwd": step_fwd_ms, "backward": step_bwd_ms},
            "traffic": (traffic or {}).get(dominant),
            "fp32_fma_peak_tflops_at_sampled_clock": fma_peak,
        },
        "e2e": {
            "value": total_bytes / (e2e_ms / 1e3) / 1e9,
            "unit": "GB/s",
            "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "pathtile_b200.host.HostPipeline.run (pinned host tensors)",
            "host_cpus": len(host_cpus) if host_cpus else None,
        },
        "gpu_launches": args.steps * (1 + (ops.dx_dk_launches(B, H, L, K) if fused else 3)),
        **({"step_split": split} if split else {}),
        "clocks": clocks.summary(),
        "device_error_word": err,
    }
    if not args.no_cpu_baseline and world == 1:  # the CPU baseline belongs to the 1-GPU line
        result["cpu_baseline"] = cpu_baseline(args.cpu_sample_b)
    return result


def reference_gpu_kernels() -> dict | None:
    """The reference's own warp-tiled CUDA kernels (its CUDA_TEMPLATE with the
    default launch constants, compiled for sm_100a into oracle/_ref by
    oracle/build_oracle.py) on this GPU at the primary shape, each phase under
    the reference protocol with the atomic dK's zero-fill outside the timed
    region -- the GPU-to-GPU comparison point.  None where not built or no GPU."""
    import ctypes

    lib_path = ROOT / "oracle" / "_ref" / "libref_warptile.so"
    if not lib_path.exists() or not torch.cuda.is_available():
        return None
    lib = ctypes.CDLL(str(lib_path))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(42)
    x = torch.randn(B_PER_GPU, H, L, device=dev, generator=g)
    k = torch.randn(H, K, device=dev, generator=g) / (K ** 0.5)
    dy = torch.randn(B_PER_GPU, H, L, device=dev, generator=g)
    y, gx, gk = torch.empty_like(x), torch.empty_like(x), torch.zeros_like(k)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    B = B_PER_GPU

    def launch(fn, *a):
        if fn(*a) != 0:
            raise RuntimeError("reference kernel launch failed")

    # The same interleaved steady-state warm-up as the native arm's phases.
    t_end = time.perf_counter() + STEADY_S
    while time.perf_counter() < t_end:
        launch(lib.ref_fwd, p(x), p(k), p(y), B, H, L, K, sp)
        launch(lib.ref_dx, p(dy), p(k), p(gx), B, H, L, K, sp)
        gk.zero_()
        launch(lib.ref_dk, p(dy), p(x), p(gk), B, H, L, K, sp)
        torch.cuda.synchronize()

    phases = {
        "fwd": time_phase(lambda: launch(lib.ref_fwd, p(x), p(k), p(y), B, H, L, K, sp), stream, 0),
        "bwd_input": time_phase(lambda: launch(lib.ref_dx, p(dy), p(k), p(gx), B, H, L, K, sp), stream, 0),
        "bwd_weight": time_phase(lambda: launch(lib.ref_dk, p(dy), p(x), p(gk), B, H, L, K, sp), stream, 0,
                                 pre=gk.zero_),
    }
    agg = sum(v["ms"] for v in phases.values())
    return {
        "kernels": "dwconv1d_warptile_fwd / _bwd_input / _bwd_weight (kernels/warp_tiled_ampere.py:372-619), "
                   "WARPS_PER_BLOCK=16, BWDK_BTILE=64, BWDK_BLOCK=128, compiled for sm_100a",
        "config": {"B": B, "H": H, "L": L, "K": K},
        "phase_ms": {n: v["ms"] for n, v in phases.items()},
        "aggregate_ms": agg,
        "GB/s": 3 * phase_bytes(B) / (agg / 1e3) / 1e9,
        "protocol": f"{PHASE_TRIALS} trials x ({PHASE_WARMUP} + {PHASE_RUNS}) launches per phase, CUDA events",
    }


def run_reference(args, rank: int) -> dict | None:
    """The reference's CPU path on this host, same metric and unit: each step
    times FWD, dX and dK separately under the reference's protocol (the autograd
    graph built outside the timed region) on a bounded sample and sums them."""
    if rank != 0:
        return None
    from oracle import reference_torch as ref

    torch.set_num_threads(os.cpu_count() or 1)
    Bs = args.ref_sample_b
    x, k, dy = ref.make_inputs(Bs, H, L, K, seed=42)
    xr = x.clone().requires_grad_(True)
    kr = k.clone().requires_grad_(True)

    def step() -> dict[str, float]:
        out = {}
        with torch.no_grad():
            t0 = time.perf_counter()
            ref.depthwise_same(x, k)
            out["fwd"] = time.perf_counter() - t0
        yx = ref.depthwise_same(xr, k)
        t0 = time.perf_counter()
        torch.autograd.grad(yx, xr, dy)
        out["bwd_input"] = time.perf_counter() - t0
        yk = ref.depthwise_same(x, kr)
        t0 = time.perf_counter()
        torch.autograd.grad(yk, kr, dy)
        out["bwd_weight"] = time.perf_counter() - t0
        return out

    for _ in range(args.warmup):
        step()
    runs = [step() for _ in range(args.steps)]
    phase_ms = {n: 1e3 * statistics.mean(r[n] for r in runs) for n in ("fwd", "bwd_input", "bwd_weight")}
    ms = sum(phase_ms.values())
    val = 3 * phase_bytes(Bs) / (ms / 1e3) / 1e9
    sample = (f"B={Bs} of the primary shape (H=128,L=48,K=48) per step; FWD, dX and dK timed separately with "
              "the autograd graph built outside the timed region (the reference's benchmark_pytorch.py "
              "protocol) and summed; reference PyTorch CPU path restated in oracle/reference_torch.py")
    small = cpu_protocol(64)
    res = {
        "metric": METRIC, "impl": "reference", "value": val, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: x, dy ~ N(0,1), k ~ N(0,1)/sqrt(K), seeded",
        "config": {"workload": "primary: B=16384 per GPU, H=128, L=48, K=48 (bounded CPU sample per step)",
                   "B_sample": Bs, "H": H, "L": L, "K": K, "parallelism": "cpu"},
        "aggregate_ms": ms,
        "phase_ms": phase_ms,
        "cpu_baseline": {"value": val, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "cpu_model": cpu_model(), "phase_ms": phase_ms, "sample": sample,
                         "config0_B64": {k_: small[k_] for k_ in ("phase_ms", "aggregate_ms", "GB/s")}},
        "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_ref_gpu:
        try:
            ref_gpu = reference_gpu_kernels()
        except Exception as exc:  # the CPU line stands on its own
            ref_gpu = {"error": repr(exc)}
        if ref_gpu is not None:
            res["reference_gpu_kernels"] = ref_gpu
    return res


def run_s4_train(args) -> dict:
    """S4ConvD training step (the reference's model and training configuration,
    kernels/warp_tiled_ampere.py:1122-1215 and :1432-1560: batch 16384, L = 48,
    H = 128, 4 blocks, SGD, RMSLE) on synthetic windows, device-timed.  The same
    model on PyTorch's grouped conv1d (cuDNN; the reference's "pytorch" backend,
    TF32 off as in its configure_torch) is timed beside it."""
    import torch.nn.functional as F

    from pathtile_b200 import build, ops, s4conv

    build.build()
    apply_engine(ops, args.engine)
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    B = args.batch
    x, target = s4conv.synthetic_batch(B, device=dev, seed=0)

    def cudnn_conv(xx, kk):
        K_ = int(kk.shape[1])
        left = K_ // 2
        return F.conv1d(F.pad(xx, (left, K_ - 1 - left)), kk.unsqueeze(1), groups=int(xx.shape[1]))

    out = {}
    for name, conv in (("pathtile_b200", None), ("pytorch_cudnn", cudnn_conv)):
        torch.manual_seed(0)
        model = s4conv.Model().to(dev)
        if conv is not None:
            for blk in model.blocks:
                blk.kernel_layer.conv = conv
        opt = s4conv.make_optimizer(model)
        for _ in range(args.warmup):
            s4conv.train_step(model, opt, x, target)
        ms = time_loop(lambda: s4conv.train_step(model, opt, x, target), args.steps, torch.cuda.current_stream(dev))
        out[name] = ms
        del model, opt
        torch.cuda.empty_cache()
    return {
        "metric": "S4ConvD training step (B=16384, L=48, H=128, 4 blocks, SGD, RMSLE), device-timed",
        "workload": "s4-train",
        "value": out["pathtile_b200"],
        "unit": "ms/step",
        "higher_is_better": False,
        "pytorch_cudnn_ms": out["pytorch_cudnn"],
        "speedup_vs_pytorch_cudnn": out["pytorch_cudnn"] / out["pathtile_b200"],
        "steps": args.steps,
        "warmup": args.warmup,
        "batch": B,
        "dtype": "f32",
        "data": "synthetic windows (the reference's ASHRAE data is not shipped): x ~ N(0,1), target ~ 3|N(0,1)|",
        "note": "each block's depthwise conv is the primary shape (B, 128, 48, K=48); skip term folded into the centre tap",
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-chunk", type=int, default=1024)
    ap.add_argument("--cpu-sample-b", type=int, default=1024, help="batch of the bounded CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-sample-b", type=int, default=1024)
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="--impl reference: skip timing the reference's CUDA kernels on the GPU")
    ap.add_argument("--batch", type=int, default=B_PER_GPU,
                    help="batch per GPU (default: the primary workload; smaller only for profiling)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer measurement (profiling)")
    ap.add_argument("--no-numa-bind", action="store_true",
                    help="e2e: leave host buffers where the OS puts them (default: near the GPU)")
    ap.add_argument("--backward", choices=("fused", "separate"), default="fused",
                    help="backward of the step: ops.dx_dk (one fused kernel where it applies) or dX then dK")
    ap.add_argument("--engine", choices=("frozen", "ffma", "tensor"), default="frozen",
                    help="kernels to run: the frozen per-shape table (default), or force one engine")
    ap.add_argument("--collective", choices=("fused", "nccl"), default="fused",
                    help="N > 1: sum dK through the peers' memory inside the backward (default) or NCCL all_reduce")
    ap.add_argument("--workload", choices=("primary", "s4-train"), default="primary",
                    help="s4-train: time the S4ConvD training step instead (single GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.workload == "s4-train":
        if rank == 0:
            print(json.dumps(run_s4_train(args)), flush=True)
        return

    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        res = run_ours(args, rank, world, local_rank)
        if res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
