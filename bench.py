#!/usr/bin/env python
"""Benchmark of the sm_100a attention forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (fp16 q, k, v of layout [B*H, N, 64], non-causal, scale 1/8):
  b1h8n8192     B=1  H=8  N=8192   N(0,1)            the headline configuration (default)
  b16h16n4096   B=16 H=16 N=4096   N(0,1)            throughput shape
  b1h32n32768   B=1  H=32 N=32768  q,k ~ N(0,3^2)    long sequence, peaky softmax
  b128h16n512   B=128 H=16 N=512   uniform[-1,1]     short sequence, HBM side of the ridge

Method (as benchs/benchmark_forward.py:218-325 of the reference): 4 rotating input buffers
seeded 0..3 (q, k, v drawn in that order from one generator per buffer), a 256 MB L2 flush
write before every step (outside the timed interval), CUDA events on the launching stream
around each forward call, TFLOPS = 4*B*H*N^2*D / t. W warm-up steps, then exactly K timed
steps bracketed by barrier + synchronize; the time is the max over ranks.

Multi-GPU (torchrun, one rank per GPU): every rank owns a contiguous block of batch*head rows
(mini_flash_attention.sharding); no collective runs on the data path. For the headline
workload each rank owns its own B=1, H=8 slice (weak scaling: the global batch grows with N);
for the others the global B*H is split over the ranks (strong scaling).

Besides `value` (whole-job TFLOPS over all ranks; `tflops_per_gpu` = value / n_gpus) the line
carries, for the default forward:
  kernel_only     CUDA events around the C-ABI call mfa_fwd_f16 (no torch allocation or
                  binding), same buffers, flush and steps: the kernels alone;
  kernel_us       per-kernel device durations of three flushed calls from a CUPTI trace;
  memory          device memory a call takes beyond its inputs: the torch allocator's peak
                  (the reference benchmark's figure: the output) and the split plan's scratch
                  from the library's own pool;
  strong          the strong splits of B128 H16 N512 (2048 batch*head rows contiguous over
                  the ranks), B16 H16 N4096 (256 rows) and B1 H32 N32768 (its 32 heads), in
                  that order, timed in the same process after the headline, max over ranks
                  (mean and median per call; B128 H16 N512 also as algorithmic HBM GB/s);
  reference_kernel (one GPU) a GPU baseline leg: the reference's own CuTe kernel (compiled from
                  its sources into oracle/_ref) on the same buffers, flush and events, timed
                  after everything else, like cpu_baseline;
  modes           (one GPU, headline) causal, bf16, D=128 and the backward pass at B1 H8 N8192;
  cudnn_sdpa      (one GPU) context: cuDNN's fused attention (torch SDPA, cuDNN backend) on
                  the same buffers, flush and events;
  e2e.copy_gbs    host<->device bytes of one rank's step / that rank's e2e time per step.
--no-extras leaves all of these out (for profiler runs).

--impl reference times the reference's CPU path (the naive torch attention of
benchs/benchmark_forward.py:98-115) on this host's cores, one head of the workload per step,
on rank 0 only; --impl reference --ref-kernel cute times the reference's own CuTe kernel
(built from its sources into oracle/_ref) on the GPU instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "mini-flash-attention_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "fwd TFLOPS/GPU (4·BH·N²·D/t), % dense-fp16 peak; ms at B1 H8 N8192"
UNIT = "TFLOPS"
PUBLISHED_TFLOPS = 9.510  # ms, RTX A4000, CuTe kernel at B1 H8 N8192 (reference README.md:97)
PUBLISHED_TFLOPS = 4 * 8 * 8192 ** 2 * 64 / (PUBLISHED_TFLOPS * 1e-3) / 1e12
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}
L2_FLUSH_MB = 256
INPUT_BUFFERS = 4
E2E_CHUNKS = 4  # pieces of decreasing size (forward_pinned): measured best

WORKLOADS = {
    "b1h8n8192": dict(B=1, H=8, N=8192, dist="normal", qk_scale=1.0, scaling="weak"),
    "b16h16n4096": dict(B=16, H=16, N=4096, dist="normal", qk_scale=1.0, scaling="strong"),
    "b1h32n32768": dict(B=1, H=32, N=32768, dist="normal", qk_scale=3.0, scaling="strong"),
    "b128h16n512": dict(B=128, H=16, N=512, dist="uniform", qk_scale=1.0, scaling="strong"),
    # not a reference configuration: one head, so that 2 or more GPUs split its query rows
    # (sharding.q_shard, forward_rows) with the whole k and v on every GPU
    "b1h1n65536": dict(B=1, H=1, N=65536, dist="normal", qk_scale=1.0, scaling="strong"),
}
D = 64


def attention_flops(bh: int, n: int, d: int = D, causal: bool = False) -> float:
    """4 * BH * (attended query-key pairs) * D, pairs = N^2, or N(N+1)/2 with the causal mask
    (benchs/benchmark_forward.py:315-325)."""
    pairs = n * (n + 1) / 2 if causal else n * n
    return 4.0 * bh * pairs * d


def attention_bytes(bh: int, n: int, d: int = D) -> float:
    return 4.0 * bh * n * d * 2  # read q, k, v once, write o once (fp16)


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(kernel: str, workload: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    path = ROOT / "profiles" / f"{kernel}_{workload}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------- clocks during timing
REASON_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU every millisecond (NVML, else
    nvidia-smi) while the timed region runs."""

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.device_index = device_index
        self.period = period_s
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._proc = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = self.device_index
            if visible:
                ids = [x for x in visible.split(",") if x.strip()]
                if idx < len(ids) and ids[idx].strip().isdigit():
                    idx = int(ids[idx])
            h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._nvml = (pynvml, h)
            self._thread = threading.Thread(target=self._run_nvml, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001
            self._nvml = None
        return self

    def _run_nvml(self):
        pynvml, h = self._nvml
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                reasons = int(get_reasons(h))
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def stop(self) -> dict:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        busy = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        mhz = statistics.median(s[0] for s in busy)
        seen = 0
        for _, r in busy:
            seen |= r
        reasons = [name for bit, name in REASON_BITS.items() if seen & bit and bit != 0x1]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(busy)}


# ---------------------------------------------------------------- inputs
def make_inputs(wl: dict, bh: int, seed: int, device, d: int = D, dtype=torch.float16,
                with_grad: bool = False) -> tuple:
    """One buffer: q, k, v drawn in that order from one generator (benchmark_forward.py:222-227),
    then the output gradient dO when with_grad."""
    shape = (bh, wl["N"], d)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if wl["dist"] == "uniform":
        q, k, v = (torch.rand(shape, device=device, generator=g, dtype=torch.float32) * 2 - 1
                   for _ in range(3))
    else:
        q, k, v = (torch.randn(shape, device=device, generator=g, dtype=torch.float32)
                   for _ in range(3))
        q, k = q * wl["qk_scale"], k * wl["qk_scale"]
    out = [q.to(dtype).contiguous(), k.to(dtype).contiguous(), v.to(dtype).contiguous()]
    if with_grad:
        out.append(torch.randn(shape, device=device, generator=g, dtype=torch.float32)
                   .to(dtype).contiguous())
    return tuple(out)


# ---------------------------------------------------------------- CPU baseline
CPU_SAMPLE_ROWS = 4096  # query rows of one head timed on the host when N is long


def cpu_sample(wl: dict, causal: bool = False):
    """(q, k, v, flops, text): one head of the workload for the host-core timing; for N above
    16384 without the mask only its first CPU_SAMPLE_ROWS query rows (against all N keys), so
    that the fp32 score matrix stays within a few GB."""
    q, k, v = make_inputs(wl, 1, 0, "cpu")
    n = wl["N"]
    if causal or n <= 16384:
        return q, k, v, attention_flops(1, n, causal=causal), f"[1,{n},64]"
    rows = CPU_SAMPLE_ROWS
    return (q[:, :rows].contiguous(), k, v, 4.0 * rows * n * D,
            f"query rows 0-{rows - 1} of [1,{n},64] against all {n} keys")


def cpu_baseline(wl: dict, budget_s: float = 10.0, causal: bool = False) -> dict:
    """The reference's naive torch attention on the host cores, one head of the workload."""
    from oracle.torch_naive import torch_naive_attention

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v, flops, what = cpu_sample(wl, causal)
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        torch_naive_attention(q, k, v, causal=causal)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= 50:
            break
    t = statistics.median(times)
    return {"value": flops / t / 1e12, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"1 of {wl['B'] * wl['H']} heads ({what}), naive fp32 torch "
                      f"attention (benchs/benchmark_forward.py:98-115), median of {len(times)} "
                      f"runs in {sum(times):.1f} s"}


def launches_per_call(fn, *args) -> tuple[int | None, list[str]]:
    """This library's kernels launched by one call of fn, counted from a CUDA activity trace
    (torch.profiler over CUPTI) of one untimed call."""
    try:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn(*args)
            torch.cuda.synchronize()
        names = [e.name for e in prof.events()
                 if e.device_type == torch.autograd.DeviceType.CUDA and "mfa_" in e.name]
        return len(names), sorted(set(names))
    except Exception as exc:  # profiler unavailable: report no count rather than a guess
        return None, [f"launch count unavailable: {type(exc).__name__}: {exc}"]


def kernel_durations(fn, inputs, flush, calls: int = 3) -> dict:
    """Median device duration (us) per kernel of this library over `calls` flushed calls, from
    a CUDA activity trace (torch.profiler over CUPTI)."""
    try:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(calls):
                flush.fill_(1.0)
                fn(*inputs[i % len(inputs)])
            torch.cuda.synchronize()
        per: dict[str, list[float]] = {}
        for e in prof.events():
            if e.device_type == torch.autograd.DeviceType.CUDA and "mfa_" in e.name:
                per.setdefault(e.name, []).append(e.device_time)
        return {name: round(statistics.median(v), 2) for name, v in sorted(per.items())}
    except Exception as exc:  # profiler unavailable
        return {"unavailable": f"{type(exc).__name__}: {exc}"}


def time_calls(fn, inputs, flush, stream, steps: int, warmup: int) -> list[float]:
    """CUDA-event milliseconds of `steps` calls of fn, a 256 MB L2 flush before each (outside
    the events), after `warmup` untimed calls."""
    for i in range(warmup):
        flush.fill_(1.0)
        fn(*inputs[i % len(inputs)])
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    torch.cuda.synchronize()
    for i in range(steps):
        flush.fill_(1.0)
        starts[i].record(stream)
        fn(*inputs[i % len(inputs)])
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in zip(starts, ends)]


# strong splits measured after the headline: (workload, warm-up calls, timed calls)
# lightest first: the B1 H32 N32768 leg holds the GPU at its power cap for ~80 ms, and a leg
# timed right after it starts at the lowered clock (B128 H16 N512 measured ~10% slower there)
STRONG = (("b128h16n512", 5, 30), ("b16h16n4096", 5, 10), ("b1h32n32768", 3, 5))


def extra_memory(fwd, inputs, flush, bh: int, n: int, d: int, causal: bool) -> dict:
    """Device memory a forward call takes beyond its inputs, as the reference's benchmark counts
    it (benchs/benchmark_forward.py:262-289: the torch allocator's peak over the calls above the
    memory held before them, i.e. the output tensor), and the split plan's partial-result
    scratch, which the library takes from its own stream-ordered pool, outside torch's count
    (mfa_fwd_workspace_bytes)."""
    from mini_flash_attention import capi

    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    for i in range(3):
        flush.fill_(1.0)
        out = fwd(*inputs[i % len(inputs)])
        del out
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    ws = capi.fwd_workspace_bytes(1, bh, n, d, causal)
    q = inputs[0][0]
    return {"allocator_peak_bytes": int(peak),
            "output_bytes": q.numel() * q.element_size(),
            "workspace_bytes": int(ws),
            "total_extra_bytes": int(peak + ws),
            "method": "torch.cuda.max_memory_allocated() - memory_allocated() over 3 flushed "
                      "calls (the reference benchmark's figure) + the workspace from the "
                      "library's pool (mfa_fwd_workspace_bytes)"}


def strong_splits(rank: int, world: int, dev, flush, stream) -> dict:
    """B16 H16 N4096, B1 H32 N32768 and B128 H16 N512 with their global batch*head rows split
    contiguously over the ranks (no collective on the data path); whole-job TFLOPS from the max
    over ranks."""
    import mini_flash_attention as mfa
    from mini_flash_attention.sharding import bh_shard

    out = {}
    for name, warmup, steps in STRONG:
        wl = WORKLOADS[name]
        global_bh = wl["B"] * wl["H"]
        sh = bh_shard(global_bh, rank, world)
        inputs = [make_inputs(wl, sh.rows, 100 + 2 * rank + i, dev) for i in range(2)]
        ms = time_calls(lambda q, k, v: mfa.forward(q, k, v), inputs, flush, stream, steps,
                        warmup)
        barrier(world)
        step_ms = max_over_ranks(sum(ms) / steps, world)
        median_ms = max_over_ranks(statistics.median(ms), world)
        job = attention_flops(global_bh, wl["N"])
        out[name] = {"ms_per_step": round(step_ms, 4), "median_ms": round(median_ms, 4),
                     "value": round(job / (step_ms / 1e3) / 1e12, 3), "unit": UNIT,
                     # q, k, v read once and out written once, whole job
                     "hbm_gbs": round(attention_bytes(global_bh, wl["N"]) / (step_ms / 1e3) / 1e9,
                                      1),
                     "bh_per_gpu": sh.rows, "global_bh": global_bh, "steps": steps,
                     "warmup": warmup,
                     "split": f"{global_bh} batch*head rows contiguous over {world} GPU(s)"}
        del inputs
    return out


def mode_legs(dev, flush, stream, steps: int = 20, warmup: int = 3) -> dict:
    """The headline shape (B1 H8 N8192) in the library's other modes, same flush and events:
    causal fp16 (flops over the N(N+1)/2 attended pairs), bf16, D = 128, and the backward pass
    (mfa.backward from forward_lse's output; flops 2.5x the forward's, the usual convention)."""
    import mini_flash_attention as mfa

    wl = WORKLOADS["b1h8n8192"]
    bh, n = wl["B"] * wl["H"], wl["N"]
    out = {}
    for name, d, dtype, causal in (("causal", D, torch.float16, True),
                                   ("bf16", D, torch.bfloat16, False),
                                   ("d128", 128, torch.float16, False)):
        inputs = [make_inputs(wl, bh, 200 + i, dev, d=d, dtype=dtype) for i in range(2)]
        ms = time_calls(lambda q, k, v, c=causal: mfa.forward(q, k, v, causal=c), inputs, flush,
                        stream, steps, warmup)
        t = sum(ms) / steps
        out[name] = {"ms_per_step": round(t, 4), "unit": UNIT,
                     "value": round(attention_flops(bh, n, d, causal) / (t / 1e3) / 1e12, 3)}
        del inputs
    prepared = []
    for i in range(2):
        q, k, v, do = make_inputs(wl, bh, 210 + i, dev, with_grad=True)
        o, lse = mfa.forward_lse(q, k, v)
        prepared.append((q, k, v, o, lse, do))
    ms = time_calls(lambda q, k, v, o, lse, do: mfa.backward(q, k, v, o, lse, do), prepared,
                    flush, stream, steps, warmup)
    t = sum(ms) / steps
    out["backward"] = {"ms_per_step": round(t, 4), "unit": UNIT,
                       "value": round(2.5 * attention_flops(bh, n) / (t / 1e3) / 1e12, 3)}
    return out


def reference_kernel_leg(wl: dict, inputs, flush, stream, steps: int, warmup: int) -> dict:
    """GPU baseline leg: the reference's CuTe kernel (src/mini_flash_attention/flash_attn_cuda.cu:
    190-420, built from its sources into oracle/_ref) on the same buffers, flush and events."""
    try:
        from oracle import ref

        if not ref.available():
            return {"value": None, "reason": f"{ref.LIB_PATH.name} not built"}
        ms = time_calls(lambda q, k, v: ref.reference_forward(q, k, v, kernel="cute"), inputs,
                        flush, stream, steps, warmup)
    except Exception as exc:  # noqa: BLE001  (a baseline must not break the bench line)
        return {"value": None, "reason": f"{type(exc).__name__}: {exc}"}
    bh, n = inputs[0][0].shape[0], inputs[0][0].shape[1]
    t = sum(ms) / steps
    return {"value": round(attention_flops(bh, n) / (t / 1e3) / 1e12, 3), "unit": UNIT,
            "ms_per_step": round(t, 4), "median_ms": round(statistics.median(ms), 4),
            "steps": steps, "warmup": warmup,
            "kernel": "FlashAttnCuteKernel, reference sources compiled for sm_100a; its binding's "
                      "zeros_like output inside the timed call (flash_attn.cpp:86)"}


def cudnn_leg(inputs, flush, stream, steps: int, warmup: int, causal: bool) -> dict:
    """Context leg: NVIDIA's fused attention from cuDNN (torch scaled_dot_product_attention with
    the cuDNN backend) on the same buffers, viewed [1, B*H, N, D], same flush and events. A
    library kernel, not on this library's path: it shows where the forward stands against the
    vendor's own B200 kernel on the same box."""
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel

        def run(q, k, v):
            return torch.nn.functional.scaled_dot_product_attention(
                q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), is_causal=causal)

        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            ms = time_calls(run, inputs, flush, stream, steps, warmup)
    except Exception as exc:  # noqa: BLE001  (a context leg must not break the bench line)
        return {"value": None, "reason": f"{type(exc).__name__}: {str(exc)[:160]}"}
    bh, n, d = inputs[0][0].shape
    t = sum(ms) / steps
    return {"value": round(attention_flops(bh, n, d, causal) / (t / 1e3) / 1e12, 3),
            "unit": UNIT, "ms_per_step": round(t, 4), "steps": steps, "warmup": warmup,
            "kernel": "cuDNN fused attention via torch SDPA (SDPBackend.CUDNN_ATTENTION), "
                      f"cuDNN {torch.backends.cudnn.version()}"}


# ---------------------------------------------------------------- arms
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args, wl) -> dict | None:
    import mini_flash_attention as mfa
    from mini_flash_attention.sharding import bh_shard, q_shard, shard_mode

    rank, world, local = init_dist()
    dev = torch.device("cuda", local)
    global_bh = wl["B"] * wl["H"] * (world if wl["scaling"] == "weak" else 1)
    n = wl["N"]
    d = args.head_dim
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    train = args.mode == "fwd_bwd"
    q_range = None
    if shard_mode(global_bh, world) == "rows":
        bh = bh_shard(global_bh, rank, world).rows
    else:
        # fewer batch*head rows than GPUs: every rank holds the whole q, k, v and computes a
        # range of query rows of every head
        if train:
            raise SystemExit("query-row sharding (B*H < GPUs) is forward-only")
        bh = global_bh
        qs = q_shard(n, rank, world, causal=args.causal)
        q_range = (qs.begin, qs.end)
    # query-row sharding: every rank holds the same whole inputs
    seed0 = (rank if q_range is None else 0) * INPUT_BUFFERS
    inputs = [make_inputs(wl, bh, seed0 + i, dev, d, dtype, with_grad=train)
              for i in range(INPUT_BUFFERS)]
    flush = torch.empty(L2_FLUSH_MB * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    causal = args.causal

    if train:
        # one training step of the attention op: forward with its log-sum-exp, then backward
        def fwd(q, k, v, do):
            out, lse = mfa.forward_lse(q, k, v, causal=causal)
            return mfa.backward(q, k, v, out, lse, do, causal=causal)
    elif q_range is None:
        def fwd(q, k, v):
            return mfa.forward(q, k, v, causal=causal)
    else:
        rows_out = torch.empty_like(inputs[0][0])

        def fwd(q, k, v):
            return mfa.forward_rows(q, k, v, q_range[0], q_range[1], out=rows_out,
                                    causal=causal)

    stream = torch.cuda.current_stream(dev)

    with torch.inference_mode():
        for i in range(args.warmup):
            flush.fill_(1.0)
            fwd(*inputs[i % INPUT_BUFFERS])
        torch.cuda.synchronize(dev)
        if args.no_launch_count:
            per_call, kernel_names = None, ["launch count skipped (--no-launch-count)"]
        else:
            per_call, kernel_names = launches_per_call(fwd, *inputs[0])

        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        sampler = ClockSampler(local).start()
        barrier(world)
        torch.cuda.synchronize(dev)
        wall0 = time.perf_counter()
        for i in range(args.steps):
            flush.fill_(1.0)  # L2 flush, outside the event interval
            starts[i].record(stream)
            fwd(*inputs[i % INPUT_BUFFERS])
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        wall = time.perf_counter() - wall0
        clocks = sampler.stop()
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        total_ms = max_over_ranks(sum(step_ms), world)

        # ---- end to end: pinned host q, k, v -> device -> forward -> pinned host output,
        # through the public host-buffer API (copies of batch*head slices overlap kernels)
        e2e_steps = max(args.steps, 3)
        e2e_ms = e2e_ms_rank = None
        if not train and q_range is None:
            host_in = [x.cpu().pin_memory() for x in inputs[0]]
            host_out = torch.empty(inputs[0][0].shape, dtype=dtype).pin_memory()
            chunks = min(bh, E2E_CHUNKS)
            # untimed warm-up: the first ~10 calls on freshly pinned buffers run ~20% slower
            for _ in range(max(args.warmup, 10)):
                mfa.forward_pinned(*host_in, causal=causal, out=host_out, chunks=chunks,
                                   device=dev)
            torch.cuda.synchronize(dev)
            barrier(world)
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                mfa.forward_pinned(*host_in, causal=causal, out=host_out, chunks=chunks,
                                   device=dev)
            e2e_ms_rank = (time.perf_counter() - t0) * 1e3
            e2e_ms = max_over_ranks(e2e_ms_rank, world)
            barrier(world)

        # ---- extras (outside every timed region above; every rank takes the same collective
        # steps): kernels alone through the C ABI, per-kernel durations, strong splits
        extras = {}
        default_fwd = (not train and q_range is None and d == D and dtype == torch.float16)
        if default_fwd and not args.no_extras:
            from mini_flash_attention import capi

            scale = D ** -0.5
            sid = stream.cuda_stream
            outs = [torch.empty_like(x[0]) for x in inputs]
            slot = {"i": 0}

            def capi_fwd(q, k, v):
                o = outs[slot["i"] % INPUT_BUFFERS]
                slot["i"] += 1
                capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), bh, n, D,
                         scale, causal=causal, stream=sid)

            ms_k = time_calls(capi_fwd, inputs, flush, stream, args.steps, args.warmup)
            k_ms = max_over_ranks(sum(ms_k) / args.steps, world)
            extras["kernel_only"] = {
                "value": round(attention_flops(global_bh, n, d, causal) / (k_ms / 1e3) / 1e12, 3),
                "unit": UNIT, "ms_per_step": round(k_ms, 4),
                "timing": "CUDA events around the C-ABI call mfa_fwd_f16, same buffers, flush "
                          "and step count as value, max over ranks"}
            extras["kernel_us"] = kernel_durations(fwd, inputs, flush)
            extras["memory"] = extra_memory(fwd, inputs, flush, bh, n, d, causal)
            if not causal:
                extras["strong"] = strong_splits(rank, world, dev, flush, stream)
            if world == 1:
                extras["reference_kernel"] = reference_kernel_leg(
                    wl, inputs, flush, stream, max(3, min(args.steps, 20)), 3)
                extras["cudnn_sdpa"] = cudnn_leg(inputs, flush, stream, args.steps, 3, causal)
                if not causal and args.workload == "b1h8n8192":
                    extras["modes"] = mode_legs(dev, flush, stream)

    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return None

    # a training step counts the forward (2 products) and the backward (5 products)
    flop_mult = 3.5 if train else 1.0
    flops_rank_step = flop_mult * attention_flops(bh, n, d, causal=causal)
    if q_range is not None:  # this rank's query rows (with the mask: keys up to each row)
        a, b = q_range
        flops_rank_step = (4.0 * bh * d * (b * (b + 1) / 2 - a * (a + 1) / 2) if causal
                           else flops_rank_step * (b - a) / n)
    job_flops_step = flop_mult * attention_flops(global_bh, n, d, causal=causal)
    value = job_flops_step * args.steps / (total_ms / 1e3) / 1e12
    kernel_ms = total_ms / args.steps
    achieved = flops_rank_step / (kernel_ms / 1e3) / 1e12
    peaks, peak_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    default_mode = not train and d == D and dtype == torch.float16 and not causal
    traffic = load_traffic("mfa_fwd", args.workload) if default_mode and q_range is None else None
    e2e_value = None if e2e_ms is None else job_flops_step * e2e_steps / (e2e_ms / 1e3) / 1e12
    bytes_in = 3 * global_bh * n * d * 2
    bytes_out = global_bh * n * d * 2
    line = {
        "metric": METRIC if not train else
        "training-step TFLOPS/GPU (3.5·4·BH·N²·D/t: forward with log-sum-exp + backward)",
        "value": round(value, 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(kernel_ms, 4),
        "higher_is_better": True,
        "scaling": wl["scaling"],
        "vs_baseline": round(value / PUBLISHED_TFLOPS, 2) if default_mode else None,
        "dtype": args.dtype,
        "data": "synthetic (seeded, shapes and distributions of the workload; no dataset)",
        "config": {
            "workload": args.workload,
            "B": wl["B"] * (world if wl["scaling"] == "weak" else 1), "H": wl["H"], "N": n,
            "D": d, "bh_per_gpu": bh, "causal": causal, "mode": args.mode,
            "parallelism": (f"batch*head sharded over {world} GPU(s), no collective"
                            if q_range is None else
                            f"query rows of every head sharded over {world} GPU(s) (whole k, v "
                            "on each), no collective"),
            "l2": f"{L2_FLUSH_MB} MB write before every step, outside the timed interval",
            "input_buffers": INPUT_BUFFERS,
            "timing": "CUDA events around each forward() call on its stream, max over ranks",
        },
        "value_scope": "whole job: TFLOPS summed over all n_gpus ranks (per GPU: "
                       "tflops_per_gpu); the metric's per-GPU figure is value / n_gpus",
        "tflops_per_gpu": round(value / world, 3),
        "pct_dense_fp16_peak": round(100.0 * achieved / peak, 2),
        "roofline": {
            "bound": "tensor",
            "achieved": round(achieved, 3),
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic,
            "algorithmic_bytes": attention_bytes(bh, n, d),
            # the memory side of the same call: q, k, v read once and out written once
            "hbm": {"achieved_gbs": round(attention_bytes(bh, n, d) / (kernel_ms / 1e3) / 1e9, 1),
                    "peak_gbs": float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])),
                    "frac": round(attention_bytes(bh, n, d) / (kernel_ms / 1e3) / 1e9
                                  / float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])), 4)},
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json bf16_tflops burst)"
            if peak_src == "measured" else "fallback 1.59 PFLOP/s",
            "kernel": "mfa_fwd_kernel<2,3> (+ mfa_merge_kernel when the key dimension is split); "
                      "achieved = flops / CUDA-event time of the whole forward call",
        },
        "e2e": ({
            "value": round(e2e_value, 3), "unit": UNIT,
            "h2d_bytes_per_step": bytes_in, "d2h_bytes_per_step": bytes_out,
            "copy_gbs_per_rank": round(4 * bh * n * d * 2 / (e2e_ms_rank / e2e_steps / 1e3) / 1e9,
                                       2),
            "copy_gbs_note": "one rank's host<->device bytes per step (q, k, v in, out back) / "
                             "that rank's e2e time per step: the e2e limiter is this copy rate",
            "path": "mini_flash_attention.forward_pinned: pinned host q,k,v -> H2D / forward / "
                    "D2H of batch*head slices pipelined on 3 streams -> pinned host out",
            "timing": "host wall clock around the synchronous calls, max over ranks",
        } if e2e_value is not None else {"value": None, "reason": (
            "no host-buffer training API" if train else
            "forward_pinned has no query-row range")}),
        **extras,
        "gpu_launches": None if per_call is None else per_call * args.steps,
        "gpu_kernels": kernel_names,
        "clocks": clocks,
        "wall_s_timed_region": round(wall, 4),
    }
    if world == 1 and not args.no_cpu_baseline and not train and d == D:
        line["cpu_baseline"] = cpu_baseline(wl, causal=causal)
    return line


def run_reference(args, wl) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    if args.ref_kernel == "cute":
        return run_reference_cute(args, wl)
    from oracle.torch_naive import torch_naive_attention

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v, flops, what = cpu_sample(wl)
    for _ in range(args.warmup):
        torch_naive_attention(q, k, v)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        torch_naive_attention(q, k, v)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = flops * args.steps / total / 1e12
    sample = (f"1 of {wl['B'] * wl['H']} heads ({what}) per step, naive fp32 torch "
              f"attention (benchs/benchmark_forward.py:98-115) on {threads} host threads")
    return {
        "metric": METRIC, "value": round(value, 5), "unit": UNIT, "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": wl["scaling"], "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic (seeded)", "impl": "reference",
        "config": {"workload": args.workload, "B": wl["B"], "H": wl["H"], "N": wl["N"], "D": D,
                   "sample": "one head per step"},
        "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_reference_cute(args, wl) -> dict:
    """The reference's own CuTe kernel (oracle/_ref, built from its sources) on this GPU."""
    from oracle import ref

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    bh, n = wl["B"] * wl["H"], wl["N"]
    inputs = [make_inputs(wl, bh, i, dev) for i in range(INPUT_BUFFERS)]
    flush = torch.empty(L2_FLUSH_MB * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        flush.fill_(1.0)
        ref.reference_forward(*inputs[i % INPUT_BUFFERS])
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(1.0)
        starts[i].record(stream)
        ref.reference_forward(*inputs[i % INPUT_BUFFERS])
        ends[i].record(stream)
    torch.cuda.synchronize()
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total = sum(ms)
    value = attention_flops(bh, n) * args.steps / (total / 1e3) / 1e12
    return {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps, 4),
            "median_ms": round(statistics.median(ms), 4), "higher_is_better": True,
            "scaling": wl["scaling"], "vs_baseline": round(value / PUBLISHED_TFLOPS, 2),
            "dtype": "fp16", "data": "synthetic (seeded)", "impl": "reference",
            "ref_kernel": "FlashAttnCuteKernel (src/mini_flash_attention/flash_attn_cuda.cu), "
                          "built for sm_100a from the reference sources, zeros_like output "
                          "inside the timed call as in the reference binding",
            "config": {"workload": args.workload, "B": wl["B"], "H": wl["H"], "N": n, "D": D}}


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="b1h8n8192")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-kernel", choices=["cpu", "cute"], default="cpu")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--dtype", choices=["fp16", "bf16"], default="fp16")
    ap.add_argument("--head-dim", type=int, choices=[32, 64, 128], default=D)
    ap.add_argument("--mode", choices=["fwd", "fwd_bwd"], default="fwd",
                    help="fwd: forward() (default); fwd_bwd: forward_lse + backward (D=64)")
    ap.add_argument("--causal", action="store_true",
                    help="mask key > query (flops counted over the N(N+1)/2 attended pairs)")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="skip the CUPTI trace that counts launches (for runs under ncu)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip kernel_only, kernel_us, strong and reference_kernel")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.mode == "fwd_bwd" and args.head_dim != 64:
        ap.error("--mode fwd_bwd needs --head-dim 64 (the backward pass is D = 64)")
    wl = WORKLOADS[args.workload]
    line = run_reference(args, wl) if args.impl == "reference" else run_ours(args, wl)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
