"""MSDA forward+backward benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config decoder]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --impl reference ...   # the reference's CPU implementation
    python bench.py --op grid_sample|roi_align   # the sibling gathers (1 GPU)

A step is one forward + backward of the multi-scale deformable attention op
over one batch of the configured operating point (default: the
Deformable-DETR decoder preset, B=4 Q=300 M=8 D=32 L=4 K=4, bf16). With N
ranks every rank runs the op on its own batch slice (msda_triton_b200.sharding:
weak scaling, B items per rank, for the per-GPU presets; strong scaling, the
global B split N ways, for `scale`/`scale_d64`); the op path has no
collective and NCCL only carries the timing reduction.

Reported (one JSON line on rank 0):
  value      queries/s over all ranks (B*Q*N / device time), inputs resident
             in HBM; device time = CUDA-event time of one CUDA-graph replay
             per step (forward then backward launches), L2 flushed before
             every step, max over ranks.
  in_graph_us  the step's device time between event nodes at the first and
             last node of its CUDA graph (without the graph launch latency).
  e2e        the same metric through the public op with pinned HOST buffers:
             every step copies its inputs host->device and the output and the
             three gradients device->host inside the timed region (the next
             step's uploads overlap this step's downloads on a copy stream);
             `copy_only_ms_per_step` times the same copies with no operator,
             `frac_of_copy_only` = copy-only time / e2e time. Each rank's
             host threads (and pinned buffers) sit on its GPU's NUMA node.
  roofline   the backward call (the dominant launch sequence): algorithmic
             bytes / its CUDA-event time against the measured HBM copy
             bandwidth; `step` gives the same for forward + backward.
  kernels_us per-kernel device times (CUPTI) of a few extra steps after the
             timed region; `gpu_launches` counts the msda kernels found there.
  cpu_baseline  the reference's CPU implementation (grid_sample forward +
             autograd backward, restated in oracle/msda_oracle.py) on the
             host cores, rank 0 at N=1.
  workloads  (decoder line, N=1) the encoder (bf16) and Mask2Former (fp16)
             operating points timed the same way, with their step rooflines.
  gpu_bar    (N=1) the reference's own Triton kernels (baseline/_ref, the
             unmodified package) and this build, both through their public op
             and torch.autograd, one CUDA graph per step, at the reference's
             B200 default accumulation (native) and with fp32_grad_accum.

With --op grid_sample / roi_align the line covers the sibling gathers on
their own workloads (GATHER_WORKLOADS), next to the operators they replace
(torch's grid_sample, torchvision's roi_align) timed the same way on the
same GPU; the headline benchmark is the default (--op msda).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "msda-triton_b200"))

from msda_triton_b200 import multi_scale_deformable_attention, presets, sharding  # noqa: E402
from msda_triton_b200 import ops as msda_ops  # noqa: E402

L2_FLUSH_BYTES = 512 << 20  # > 126 MB L2
L2_DRAIN_BYTES = 256 << 20
FALLBACK_HBM_GBS = 6650.0
METRIC = "MSDA fwd+bwd µs, queries/s & % HBM roofline, bf16 decoder/encoder, 1–8 B200"
NOMINAL_HBM_GBS = 8000.0


# ---------------------------------------------------------------------------
# Algorithmic byte model (labs/solutions/lab06.py:121-129 for the forward,
# extended to the backward): every gathered corner row counts, every
# grad_value contribution counts once at the op's element size, grad_value is
# written once. The same numerator serves every accumulator algorithm, so a
# slower algorithm shows up as a lower fraction, never as more "work".
# ---------------------------------------------------------------------------
def algorithmic_bytes(B, S, Q, M, D, L, K, e):
    ns = B * Q * M * L * K
    fwd = ns * 4 * D * e + ns * 3 * e + B * Q * M * D * e
    bwd = (ns * 4 * D * e + ns * 4 * D * e + ns * 6 * e + B * Q * M * D * e
           + B * S * M * D * e)
    return fwd, bwd


# ---------------------------------------------------------------------------
# Clock sampling (NVML reads only; no setting is changed)
# ---------------------------------------------------------------------------
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples: list[tuple[int, int, int]] = []
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self.error = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            uuid = None
            try:
                props = torch.cuda.get_device_properties(device_index)
                uuid = "GPU-" + str(props.uuid)
            except Exception:  # noqa: BLE001
                pass
            self._h = (pynvml.nvmlDeviceGetHandleByUUID(uuid) if uuid
                       else pynvml.nvmlDeviceGetHandleByIndex(device_index))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # noqa: BLE001
            self._nvml = None
            self.error = f"nvml unavailable: {exc}"
            self.max_mhz = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter_ns(), sm, reasons))
            except Exception as exc:  # noqa: BLE001
                self.error = str(exc)
                return
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
        if self._nvml is not None:
            self.samples.append((time.perf_counter_ns(),
                                 self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM),
                                 self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)))

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0, "note": self.error}
        mask = 0
        for _, _, r in self.samples:
            mask |= r
        reasons = sorted(name for bit, name in _REASONS.items() if mask & bit and name != "gpu_idle")
        return {"sm_mhz": statistics.median(s for _, s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
class _StdoutToStderr:
    """Send file descriptor 1 to stderr for a while (NCCL prints its version
    banner on stdout during communicator setup; stdout carries only the
    JSON line)."""

    def __enter__(self):
        import ctypes

        self._libc = ctypes.CDLL(None)
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        self._libc.fflush(None)
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch with torchrun for N>1")
    if world == 1:
        return sharding.init_ranks("nccl", timeout_s=120)
    with _StdoutToStderr():
        ranks = sharding.init_ranks("nccl", timeout_s=120)
        sharding.barrier(world)  # the communicator exists after the first collective
    return ranks


def bind_to_gpu_numa_node(device_index):
    """Run this rank's host threads on the CPUs of its GPU's NUMA node (when
    the host has more than one node), so pinned host buffers allocated
    afterwards are local to the GPU's PCIe root. Returns {"node", "cpus"} or
    None. Changes only this process's CPU affinity."""
    try:
        import pynvml

        pynvml.nvmlInit()
        uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
        bus = pynvml.nvmlDeviceGetPciInfo(h).busId
        bus = bus.decode() if isinstance(bus, bytes) else bus
        dom, rest = bus.lower().split(":", 1)
        node_file = Path(f"/sys/bus/pci/devices/{int(dom, 16):04x}:{rest}/numa_node")
        node = int(node_file.read_text())
        nodes = [p for p in Path("/sys/devices/system/node").glob("node[0-9]*")]
        if node < 0 or len(nodes) < 2:
            return None
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return {"node": node, "cpus": len(cpus)}
    except Exception:  # noqa: BLE001 - no NVML / sysfs: leave the affinity alone
        return None


max_over_ranks = sharding.max_over_ranks
barrier = sharding.barrier


# ---------------------------------------------------------------------------
# Legs
# ---------------------------------------------------------------------------
def device_leg(x, steps, warmup, fp32_acc, algo_flags=0, use_graph=True):
    """Forward and backward launches (one CUDA-graph replay per step, or
    direct launches with use_graph=False), L2 flushed before every step, each
    step bracketed by CUDA events. Returns (graph, step function, per-step
    events, in_graph) where in_graph(n) -> mean ms between the first and the
    last node of a second graph of the same step (None without graphs),
    measured after the timed region: event nodes cost time inside a graph,
    so the timed graph carries only the one that splits forward from
    backward."""
    args = (x["value"], x["spatial_shapes"], x["level_start_index"], x["sampling_locations"],
            x["attention_weights"])
    g = x["grad_output"].reshape(x["value"].shape[0], -1, x["value"].shape[2], x["value"].shape[3])
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    drain = torch.ones(L2_DRAIN_BYTES // 4, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up outside capture (allocator, lazy loading)
        for _ in range(2):
            msda_ops._forward(*args)
            msda_ops._backward(*args, g, fp32_acc, algo_flags)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]

    def flush_l2():
        # Write 512 MiB (evicts everything of ours from L2), then read 256 MiB
        # so the flush's own dirty lines are written back before the timed
        # region instead of inside it.
        flush.fill_(1)
        drain.sum()

    in_graph = None
    if use_graph:
        # One graph per step (forward then backward), as a training step
        # captured whole would run; an event recorded inside the graph
        # (external: a real event-record node) splits forward from backward.
        mid = torch.cuda.Event(enable_timing=True, external=True)
        gs = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gs):
            msda_ops._forward(*args)
            mid.record()
            msda_ops._backward(*args, g, fp32_acc, algo_flags)
        first = torch.cuda.Event(enable_timing=True, external=True)
        last = torch.cuda.Event(enable_timing=True, external=True)
        gi = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gi):
            first.record()
            msda_ops._forward(*args)
            msda_ops._backward(*args, g, fp32_acc, algo_flags)
            last.record()

        def one(e):
            flush_l2()
            e[0].record()
            gs.replay()
            e[2].record()
            # The in-graph event is overwritten by the next replay: read the
            # split now (outside the timed region of the next step).
            e[2].synchronize()
            e[1] = (e[0].elapsed_time(mid), mid.elapsed_time(e[2]))

        def in_graph(n):
            out = []
            for _ in range(n):
                flush_l2()
                gi.replay()
                last.synchronize()
                out.append(first.elapsed_time(last))
            return statistics.fmean(out)
    else:
        gs = None

        def one(e):
            flush_l2()
            e[0].record()
            msda_ops._forward(*args)
            e[1].record()
            msda_ops._backward(*args, g, fp32_acc, algo_flags)
            e[2].record()

    tmp = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(warmup):
        one(tmp)
    return gs, one, evs, in_graph


def split_ms(e):
    """(forward ms, backward ms) of one timed step."""
    if isinstance(e[1], tuple):
        return e[1][:2]
    return e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])


def workload_leg(name, dtype, steps, warmup):
    """Forward + backward of another operating point on this GPU (default
    accumulator policy), timed like the headline device leg: mean forward /
    backward / step times and the step's algorithmic-byte roofline."""
    preset = presets.get(name)
    x = presets.make_inputs(preset, dtype=dtype, device="cuda")
    fp32_acc = msda_ops._use_fp32_grad_accum(x["value"])
    gs, one, evs, in_graph = device_leg(x, steps, warmup, fp32_acc)
    for e in evs:
        one(e)
    f = statistics.fmean(split_ms(e)[0] for e in evs)
    b = statistics.fmean(split_ms(e)[1] for e in evs)
    inner = in_graph(steps)
    B, S, M, D = x["value"].shape
    Q = x["sampling_locations"].shape[1]
    fwd_b, bwd_b = algorithmic_bytes(B, S, Q, M, D, preset.L, preset.K, x["value"].element_size())
    peak, _ = load_peaks()
    del gs, x
    return {"dtype": str(dtype).replace("torch.", ""), "B": B, "Q": Q, "S": S,
            "fwd_us": f * 1e3, "bwd_us": b * 1e3, "fwd_bwd_us": (f + b) * 1e3,
            "in_graph_us": inner * 1e3, "queries_per_s": B * Q / ((f + b) / 1e3),
            "roofline": {"bound": "hbm", "unit": "GB/s", "peak": peak,
                         "fwd_frac": fwd_b / (f / 1e3) / 1e9 / peak,
                         "bwd_frac": bwd_b / (b / 1e3) / 1e9 / peak,
                         "step_frac": (fwd_b + bwd_b) / ((f + b) / 1e3) / 1e9 / peak,
                         "algorithmic_bytes": fwd_b + bwd_b}}


def kernel_breakdown(one, steps=5):
    """Per-kernel device times (CUPTI, through torch.profiler) of a few extra
    steps after the timed region: {kernel: (mean us, launches per step)}."""
    from torch.profiler import ProfilerActivity, profile

    tmp = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            one(tmp)
        torch.cuda.synchronize()
    agg = {}
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA or not ev.name.startswith("void msda::"):
            continue
        name = ev.name[len("void msda::"):].split("<")[0]
        agg.setdefault(name, []).append(ev.device_time)
    return {k: (statistics.fmean(v), len(v) / steps) for k, v in agg.items()}


def backward_algorithm(kernels, deterministic=False):
    if "msda_absmax_kernel" in kernels:
        kind = "counted" if "msda_count_kernel" in kernels else "scatter"
        return f"deterministic {kind} (64-bit fixed-point rows)"
    if deterministic and "msda_count_kernel" in kernels:
        return "deterministic counted (exact integer-valued fp32 rows; 64-bit rows past 32 hits)"
    if "msda_count_kernel" in kernels:
        return "counted (fp32 rows for multi-hit pixels)"
    if "msda_cast_kernel" in kernels:
        return "scatter into fp32 workspace + cast"
    return "scatter (native packed reductions)"


def e2e_leg(x, steps, warmup, fp32_acc, deterministic=False):
    """Public op with pinned host buffers. Every step copies its inputs
    host->device, runs forward + backward through
    multi_scale_deformable_attention, and copies the output and the three
    gradients device->host. The steps are pipelined the way a data loader
    would run them: the inputs of step i+1 go up on an upload stream and the
    results of step i go down on a download stream while the compute stream
    runs the next step (PCIe is full duplex), with two device input buffers;
    each result tensor is recorded on the download stream, so the allocator
    keeps it until its copy is done. Returns
    run(n, compute=True) -> None, which runs n such steps (compute=False:
    the same copies with no operator in between, the host link's own rate),
    and the bytes copied per step each way."""
    keys = ("value", "sampling_locations", "attention_weights", "grad_output")
    host = {k: x[k].cpu().pin_memory() for k in keys}
    shapes, starts = x["spatial_shapes"], x["level_start_index"]
    B, S, M, D = x["value"].shape
    Q = x["sampling_locations"].shape[1]
    out_h = torch.empty(B, Q, M * D, dtype=x["value"].dtype).pin_memory()
    gv_h = torch.empty_like(host["value"]).pin_memory()
    gl_h = torch.empty_like(host["sampling_locations"]).pin_memory()
    ga_h = torch.empty_like(host["attention_weights"]).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in (out_h, gv_h, gl_h, ga_h))
    compute = torch.cuda.current_stream()
    s_in = torch.cuda.Stream()
    s_out = torch.cuda.Stream()
    bufs = [{k: torch.empty_like(x[k]) for k in keys} for _ in range(2)]
    # Result-shaped device tensors for the copy-only leg.
    idle = (torch.zeros(B, Q, M * D, dtype=x["value"].dtype, device="cuda"), torch.zeros_like(x["value"]),
            torch.zeros_like(x["sampling_locations"]), torch.zeros_like(x["attention_weights"]))

    def run(n, compute_op=True):
        up = [torch.cuda.Event() for _ in range(2)]    # inputs of a buffer are on the device
        used = [torch.cuda.Event() for _ in range(2)]  # a buffer's step has finished with it
        used[0].record(compute)
        used[1].record(compute)

        def upload(i):
            s_in.wait_event(used[i % 2])
            with torch.cuda.stream(s_in):
                for k in keys:
                    bufs[i % 2][k].copy_(host[k], non_blocking=True)
            up[i % 2].record(s_in)

        upload(0)
        for i in range(n):
            compute.wait_event(up[i % 2])
            b = bufs[i % 2]
            if compute_op:
                v = b["value"].detach().requires_grad_(True)
                l = b["sampling_locations"].detach().requires_grad_(True)
                a = b["attention_weights"].detach().requires_grad_(True)
                out = multi_scale_deformable_attention(v, shapes, starts, l, a, fp32_grad_accum=fp32_acc,
                                                       deterministic=deterministic)
                out.backward(b["grad_output"])
                results = (out.detach(), v.grad, l.grad, a.grad)
            else:
                results = idle
            used[i % 2].record(compute)
            if i + 1 < n:
                upload(i + 1)  # into the other buffer, once step i-1 is done with it
            s_out.wait_event(used[i % 2])
            with torch.cuda.stream(s_out):
                for dst, src in zip((out_h, gv_h, gl_h, ga_h), results):
                    dst.copy_(src, non_blocking=True)
                    src.record_stream(s_out)
        compute.wait_stream(s_out)  # the last results are on the host when the caller's events fire

    run(warmup)
    torch.cuda.synchronize()
    return run, h2d, d2h


# ---------------------------------------------------------------------------
# GPU bar: the reference's own Triton kernels on the same GPU
# ---------------------------------------------------------------------------
REF_INSTALL = REPO / "baseline" / "_ref"


def reference_package():
    """The reference package (src/msda_triton) installed unmodified into
    baseline/_ref by baseline/install_reference.sh: (module, None), or
    (None, why it is unavailable)."""
    if not (REF_INSTALL / "msda_triton" / "kernels.py").is_file():
        return None, "baseline/_ref/msda_triton not installed (baseline/install_reference.sh)"
    if str(REF_INSTALL) not in sys.path:
        sys.path.insert(0, str(REF_INSTALL))
    try:
        import msda_triton  # noqa: PLC0415
    except Exception as exc:  # noqa: BLE001
        return None, f"import msda_triton failed: {exc}"
    if getattr(msda_triton.ops, "triton", None) is None:
        return None, "the reference's Triton path is unavailable (triton did not import)"
    return msda_triton, None


def public_op_leg(op, x, steps, warmup, **kwargs):
    """Forward + autograd backward through a public operator
    ``op(value, spatial_shapes, level_start_index, sampling_locations,
    attention_weights, **kwargs)``, captured as one CUDA graph per step and
    timed like the device leg (L2 flushed before every step, CUDA events).
    A second graph of the same step with event nodes at its first and last
    node, replayed after the timed ones, gives the step's device time without
    the graph launch latency. Returns mean (fwd ms, bwd ms, in-graph fwd+bwd
    ms)."""
    shapes, starts = x["spatial_shapes"], x["level_start_index"]
    v = x["value"].detach().clone().requires_grad_(True)
    l = x["sampling_locations"].detach().clone().requires_grad_(True)
    a = x["attention_weights"].detach().clone().requires_grad_(True)
    g = x["grad_output"]

    def body():
        out = op(v, shapes, starts, l, a, **kwargs)
        return out, torch.autograd.grad(out, (v, l, a), g)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # autotune, JIT and allocator warm-up outside capture
        for _ in range(3):
            body()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    ev = {k: torch.cuda.Event(enable_timing=True, external=True) for k in ("first", "mid", "last")}
    graph = torch.cuda.CUDAGraph()  # timed: one event node splits forward from backward
    with torch.cuda.graph(graph):
        out = op(v, shapes, starts, l, a, **kwargs)
        ev["mid"].record()
        grads = torch.autograd.grad(out, (v, l, a), g)
    inner_graph = torch.cuda.CUDAGraph()  # untimed copy with event nodes at its ends
    with torch.cuda.graph(inner_graph):
        ev["first"].record()
        out2 = op(v, shapes, starts, l, a, **kwargs)
        grads2 = torch.autograd.grad(out2, (v, l, a), g)
        ev["last"].record()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    drain = torch.ones(L2_DRAIN_BYTES // 4, dtype=torch.float32, device="cuda")
    fwd, bwd, inner = [], [], []
    for i in range(warmup + steps):
        flush.fill_(1)
        drain.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        if i >= warmup:
            fwd.append(e0.elapsed_time(ev["mid"]))
            bwd.append(ev["mid"].elapsed_time(e1))
    for i in range(steps):
        flush.fill_(1)
        drain.sum()
        inner_graph.replay()
        ev["last"].synchronize()
        inner.append(ev["first"].elapsed_time(ev["last"]))
    del graph, inner_graph, out, grads, out2, grads2
    return statistics.fmean(fwd), statistics.fmean(bwd), statistics.fmean(inner)


def gpu_bar(presets_dtypes, steps, warmup):
    """The reference's Triton kernels (baseline/_ref, through its public
    multi_scale_deformable_attention) and this build's public operator, timed
    the same way on the same GPU, at both accumulator settings: the
    reference's B200 default (native bf16 atomics, ops.py:21-33) and
    fp32_grad_accum=True (fp32 scratch + downcast). Keyed by workload."""
    ref, why = reference_package()
    if ref is None:
        return {"unavailable": why}
    from msda_triton_b200 import multi_scale_deformable_attention as ours  # noqa: PLC0415

    res = {"reference": "msda_triton (baseline/_ref, unmodified) Triton kernels, triton "
                        + __import__("triton").__version__,
           "method": "public op forward + torch.autograd.grad, one CUDA graph per step, L2 flushed, "
                     "CUDA events; in_graph_us excludes the graph launch latency"}
    for preset, dtype in presets_dtypes:
        x = presets.make_inputs(preset, dtype=dtype, device="cuda")
        row = {}
        for acc_name, acc in (("native", False), ("fp32", True)):
            for impl, op in (("triton", ref.multi_scale_deformable_attention), ("b200", ours)):
                f, b, inner = public_op_leg(op, x, steps, warmup, fp32_grad_accum=acc)
                row[f"{impl}_{acc_name}"] = {"fwd_us": f * 1e3, "bwd_us": b * 1e3,
                                             "fwd_bwd_us": (f + b) * 1e3, "in_graph_us": inner * 1e3}
            row[f"speedup_{acc_name}"] = (row[f"triton_{acc_name}"]["fwd_bwd_us"]
                                          / row[f"b200_{acc_name}"]["fwd_bwd_us"])
        res[preset.name] = row
        del x
    return res


CPU_SAMPLE_MAX_BATCH = 4  # the CPU legs time at most 4 batch items per step


def cpu_sample_batch(preset):
    return min(preset.B, CPU_SAMPLE_MAX_BATCH)


def cpu_reference_time(preset, dtype, steps, seed=0, min_seconds=0.0):
    """The reference's CPU implementation (grid_sample forward + autograd
    backward, oracle/msda_oracle.py) on all host cores, over
    cpu_sample_batch(preset) batch items: (seconds per step, threads, steps
    run). Runs at least `steps` steps and at least `min_seconds`."""
    sys.path.insert(0, str(REPO))
    from oracle import msda_oracle as orc

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = presets.make_inputs(preset, dtype=dtype, device="cpu", seed=seed,
                            batch=cpu_sample_batch(preset))

    def step():
        v = x["value"].clone().requires_grad_(True)
        l = x["sampling_locations"].clone().requires_grad_(True)
        a = x["attention_weights"].clone().requires_grad_(True)
        out = orc.msda_grid_sample(v, x["spatial_shapes"], l, a)
        out.backward(x["grad_output"])

    step()  # warm-up
    t0 = time.perf_counter()
    n = 0
    while n < steps or (min_seconds and time.perf_counter() - t0 < min_seconds):
        step()
        n += 1
    return (time.perf_counter() - t0) / n, threads, n


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
# Sibling gathers (--op grid_sample / roi_align): their own workloads, timed
# like the MSDA device leg (L2 flushed before every step, CUDA events around
# forward + backward through the public op), next to the operators they
# replace (torch's grid_sample, torchvision's roi_align) on the same GPU.
# ---------------------------------------------------------------------------
GATHER_WORKLOADS = {
    # A feature-map warp: N=8, C=128, 128x128 -> 128x128, bf16, an affine grid
    # (rotation, zoom, shift) with small jitter, so neighbouring outputs share
    # input pixels.
    "grid_sample": dict(N=8, C=128, H=128, W=128, Ho=128, Wo=128, dtype=torch.bfloat16),
    # Mask R-CNN box head on the stride-4 level of an 800x1216 image pair:
    # N=2, C=256, 200x304, 1024 boxes of 32-400 px, 7x7 bins, sampling_ratio 2,
    # aligned; fp32 (torchvision's kernel takes boxes in the input's dtype and
    # runs fp32 under autocast).
    "roi_align": dict(N=2, C=256, H=200, W=304, K=1024, P=7, sr=2, scale=0.25, dtype=torch.float32),
}


def _gather_inputs(op):
    w = GATHER_WORKLOADS[op]
    g = torch.Generator().manual_seed(0)
    dt = w["dtype"]
    x = torch.randn(w["N"], w["C"], w["H"], w["W"], generator=g).to("cuda", dt)
    if op == "grid_sample":
        ang = torch.rand(w["N"], generator=g) * 0.35 - 0.175
        zoom = 0.8 + 0.3 * torch.rand(w["N"], generator=g)
        theta = torch.zeros(w["N"], 2, 3)
        theta[:, 0, 0] = zoom * torch.cos(ang)
        theta[:, 0, 1] = -zoom * torch.sin(ang)
        theta[:, 1, 0] = zoom * torch.sin(ang)
        theta[:, 1, 1] = zoom * torch.cos(ang)
        theta[:, :, 2] = 0.1 * torch.randn(w["N"], 2, generator=g)
        grid = torch.nn.functional.affine_grid(theta, (w["N"], w["C"], w["Ho"], w["Wo"]), align_corners=False)
        grid = grid + 0.01 * torch.randn(grid.shape, generator=g)
        gout = torch.randn(w["N"], w["C"], w["Ho"], w["Wo"], generator=g).to("cuda", dt)
        return w, x, grid.to("cuda", dt), gout
    K = w["K"]
    img = torch.tensor([w["W"], w["H"]]) / w["scale"]
    wh = 32 + 368 * torch.rand(K, 2, generator=g)
    xy = torch.rand(K, 2, generator=g) * (img - wh).clamp(min=1)
    boxes = torch.cat([torch.randint(0, w["N"], (K, 1), generator=g).float(), xy, xy + wh], 1)
    gout = torch.randn(K, w["C"], w["P"], w["P"], generator=g).to("cuda", dt)
    return w, x, boxes.to("cuda"), gout


def _gather_call(op, impl, x, coords, w):
    if op == "grid_sample":
        if impl == "b200":
            from msda_triton_b200 import grid_sample
            return grid_sample(x, coords, align_corners=False)
        return torch.nn.functional.grid_sample(x, coords, mode="bilinear", padding_mode="zeros",
                                               align_corners=False)
    if impl == "b200":
        from msda_triton_b200 import roi_align
        return roi_align(x, coords, w["P"], w["scale"], w["sr"], True)
    import torchvision
    return torchvision.ops.roi_align(x, coords, w["P"], w["scale"], w["sr"], True)


def _gather_time(op, impl, x, coords, gout, w, steps, warmup):
    """Mean (forward ms, backward ms) per step; L2 flushed before each step."""
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    drain = torch.ones(L2_DRAIN_BYTES // 4, dtype=torch.float32, device="cuda")
    xl = x.clone().requires_grad_(True)
    cl = coords.clone().requires_grad_(op == "grid_sample")
    fwd, bwd = [], []
    for i in range(warmup + steps):
        flush.fill_(1)
        drain.sum()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record()
        out = _gather_call(op, impl, xl, cl, w)
        e[1].record()
        out.backward(gout)
        e[2].record()
        torch.cuda.synchronize()
        xl.grad = None
        cl.grad = None
        if i >= warmup:
            fwd.append(e[0].elapsed_time(e[1]))
            bwd.append(e[1].elapsed_time(e[2]))
    return statistics.fmean(fwd), statistics.fmean(bwd)


def gather_algorithmic_bytes(op, w):
    """Per step, counted like the MSDA model: every corner row gathered or
    reduced, parameters, outputs and gradients once, the input gradient
    zero-filled once."""
    e, C = w["dtype"].itemsize, w["C"]
    inp = w["N"] * w["H"] * w["W"] * C * e
    if op == "grid_sample":
        P = w["N"] * w["Ho"] * w["Wo"]
        fwd = P * (4 * C * e + 2 * e + C * e)
        bwd = P * (4 * C * e + 4 * C * e + C * e + 2 * e + 2 * e) + inp
        return fwd, bwd, P
    bins = w["K"] * w["P"] * w["P"]
    samples = bins * w["sr"] * w["sr"]
    fwd = samples * 4 * C * e + bins * C * e + w["K"] * 20
    bwd = samples * 4 * C * e + bins * C * e + w["K"] * 20 + inp
    return fwd, bwd, w["K"]


def run_gather_bench(args):
    op = args.op
    w, x, coords, gout = _gather_inputs(op)
    with ClockSampler(torch.cuda.current_device()) as clk:
        f_ms, b_ms = _gather_time(op, "b200", x, coords, gout, w, args.steps, args.warmup)
    rf_ms, rb_ms = _gather_time(op, "torch", x, coords, gout, w, args.steps, args.warmup)
    fwd_b, bwd_b, units = gather_algorithmic_bytes(op, w)
    peak, peak_kind = load_peaks()
    ms = f_ms + b_ms
    unit = "output pixels/s" if op == "grid_sample" else "rois/s"
    achieved = (fwd_b + bwd_b) / (ms / 1e3) / 1e9
    line = {
        "metric": f"{op} fwd+bwd {unit}", "value": units / (ms / 1e3), "unit": unit, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": str(w["dtype"]).replace("torch.", ""), "data": "synthetic",
        "config": {"workload": op, **{k: v for k, v in w.items() if k != "dtype"},
                   "l2": "flushed before every step"},
        "fwd_us": f_ms * 1e3, "bwd_us": b_ms * 1e3,
        "replaced_operator": {"impl": "torch.nn.functional.grid_sample" if op == "grid_sample"
                              else "torchvision.ops.roi_align", "fwd_us": rf_ms * 1e3, "bwd_us": rb_ms * 1e3,
                              "value": units / ((rf_ms + rb_ms) / 1e3)},
        "roofline": {"kernel": "forward + backward calls, CUDA-event time", "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes": fwd_b + bwd_b, "traffic": None},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_arm(args, preset, dtype):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    steps = max(1, args.steps)
    # Bound the CPU run to a few minutes whatever --steps asks for.
    per_step, threads, _ = cpu_reference_time(preset, dtype, 1)
    steps = max(1, min(steps, int(120.0 / max(per_step, 1e-3))))
    for _ in range(min(args.warmup, 2)):
        cpu_reference_time(preset, dtype, 1)
    sec, threads, steps = cpu_reference_time(preset, dtype, steps)
    nb = cpu_sample_batch(preset)
    qps = nb * preset.num_queries / sec
    sample = (f"{steps} fwd+bwd steps of {nb} batch item(s) of the {preset.name} workload "
              f"({dtype}) on {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": preset.scaling, "vs_baseline": None,
        "dtype": str(dtype).replace("torch.", ""), "data": "synthetic",
        "config": config_dict(preset, dtype, args.gpus),
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_dict(preset, dtype, n):
    gb = sharding.global_batch(preset, n)
    return {"workload": f"{preset.name} preset: {preset.note}", "batch_per_gpu": gb // n,
            "global_batch": gb, "queries": preset.num_queries, "heads": preset.M,
            "head_dim": preset.D, "levels": preset.L, "points": preset.K,
            "spatial_shapes": [list(s) for s in preset.shapes], "S": preset.S,
            "dtype": str(dtype).replace("torch.", ""), "parallelism": f"batch-sharded x{n}",
            "l2": "flushed before every timed step (512 MiB write, then 256 MiB read to drain dirty lines)"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="decoder", choices=sorted(presets.PRESETS))
    ap.add_argument("--dtype", default=None, choices=["bf16", "fp16", "fp32"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--op", default="msda", choices=["msda", "grid_sample", "roi_align"],
                    help="msda (default): the headline benchmark; grid_sample / roi_align: the "
                         "sibling gathers on their own workloads, next to torch / torchvision (1 GPU)")
    ap.add_argument("--fp32-grad-accum", default="auto", choices=["auto", "on", "off"])
    ap.add_argument("--bwd-algo", default="auto", choices=["auto", "scatter", "counted"],
                    help="force the grad_value algorithm of the device leg (default: automatic)")
    ap.add_argument("--deterministic", action="store_true",
                    help="bitwise-reproducible grad_value (64-bit fixed-point accumulation)")
    ap.add_argument("--no-graph", action="store_true",
                    help="time direct launches instead of CUDA-graph replays")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernel-breakdown", action="store_true",
                    help="skip the CUPTI per-kernel pass (use under ncu)")
    ap.add_argument("--no-gpu-bar", action="store_true",
                    help="skip timing the reference's Triton kernels (baseline/_ref) on this GPU")
    ap.add_argument("--no-workloads", action="store_true",
                    help="skip the encoder / m2f device legs of the default line")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    if args.op != "msda":
        if args.gpus != 1 or args.impl != "b200":
            ap.error("--op grid_sample / roi_align run on one GPU, b200 arm only")
        torch.cuda.set_device(0)
        return run_gather_bench(args)
    preset = presets.get(args.config)
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32,
             None: preset.dtype}[args.dtype]
    if args.impl == "reference":
        return run_reference_arm(args, preset, dtype)

    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    host_numa = bind_to_gpu_numa_node(local)
    b0, nb = sharding.rank_batch(preset, world, rank)
    x = presets.make_inputs(preset, dtype=dtype, device="cuda", batch=nb, batch_offset=b0)
    fp32_acc = {"auto": msda_ops._use_fp32_grad_accum(x["value"]), "on": True,
                "off": False}[args.fp32_grad_accum]

    lib = msda_ops._lib
    algo_flags = {"auto": 0, "scatter": lib.MSDA_BWD_FORCE_SCATTER,
                  "counted": lib.MSDA_BWD_FORCE_COUNTED}[args.bwd_algo]
    if args.deterministic:
        algo_flags |= lib.MSDA_BWD_DETERMINISTIC

    # ---- device leg -------------------------------------------------------
    gs, one, evs, in_graph = device_leg(x, args.steps, args.warmup, fp32_acc, algo_flags,
                                        use_graph=not args.no_graph)
    barrier(world)
    with ClockSampler(torch.cuda.current_device()) as clk:
        for e in evs:
            one(e)
        barrier(world)
    fwd_ms = [split_ms(e)[0] for e in evs]
    bwd_ms = [split_ms(e)[1] for e in evs]
    dev_total_ms = max_over_ranks(sum(f + b for f, b in zip(fwd_ms, bwd_ms)), world)
    # Device time of the same step between its graph's first and last node
    # (a second graph with those two event nodes, after the timed region).
    in_graph_us = (max_over_ranks(in_graph(min(args.steps, 50)), world) * 1e3
                   if in_graph is not None else None)
    fwd_mean = max_over_ranks(statistics.fmean(fwd_ms), world)
    bwd_mean = max_over_ranks(statistics.fmean(bwd_ms), world)

    B, S, M, D = x["value"].shape
    Q = x["sampling_locations"].shape[1]
    L, K = preset.L, preset.K
    queries_per_step = sharding.global_batch(preset, world) * Q
    value = queries_per_step * args.steps / (dev_total_ms / 1e3)

    # ---- e2e leg ----------------------------------------------------------
    e2e = None
    if not args.no_e2e:
        run_e2e, h2d, d2h = e2e_leg(x, args.steps, args.warmup, fp32_acc, args.deterministic)
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        run_e2e(args.steps)
        t1.record()
        barrier(world)
        e2e_ms = max_over_ranks(t0.elapsed_time(t1), world)
        # The same copies with no operator between them: the host link's rate.
        run_e2e(args.warmup, compute_op=False)
        barrier(world)
        t0.record()
        run_e2e(args.steps, compute_op=False)
        t1.record()
        barrier(world)
        copy_ms = max_over_ranks(t0.elapsed_time(t1), world)
        e2e = {"value": queries_per_step * args.steps / (e2e_ms / 1e3), "unit": "queries/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": e2e_ms / args.steps,
               "copy_only_ms_per_step": copy_ms / args.steps,
               "frac_of_copy_only": copy_ms / e2e_ms,
               "host_link_gbs_per_rank": (h2d + d2h) / (copy_ms / args.steps / 1e3) / 1e9,
               "host_numa": host_numa}

    # ---- per-kernel breakdown (CUPTI, untimed extra steps) -------------------
    if args.no_kernel_breakdown:
        kernels = {}
        launches_per_step = None
    else:
        kernels = kernel_breakdown(one)
        launches_per_step = sum(n for _, n in kernels.values())
    del gs

    # ---- roofline: the backward call (dominant), and the whole step ----------
    e = x["value"].element_size()
    fwd_b, bwd_b = algorithmic_bytes(B, S, Q, M, D, L, K, e)
    peak, peak_kind = load_peaks()
    achieved = bwd_b / (bwd_mean / 1e3) / 1e9
    step_achieved = (fwd_b + bwd_b) / ((fwd_mean + bwd_mean) / 1e3) / 1e9
    algo = backward_algorithm(kernels, args.deterministic) if kernels else "automatic (not inspected)"
    roofline = {"kernel": "msda_backward call (" + " + ".join(
                    k for k in kernels if k != "msda_fwd_kernel") + "), CUDA-event time",
                "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "frac_of_nominal_8TBs": achieved / NOMINAL_HBM_GBS,
                "traffic": None, "algorithmic_bytes": bwd_b,
                "fwd": {"achieved": fwd_b / (fwd_mean / 1e3) / 1e9, "algorithmic_bytes": fwd_b,
                        "us": fwd_mean * 1e3, "frac": fwd_b / (fwd_mean / 1e3) / 1e9 / peak},
                "step": {"achieved": step_achieved, "algorithmic_bytes": fwd_b + bwd_b,
                         "frac": step_achieved / peak,
                         "frac_of_nominal_8TBs": step_achieved / NOMINAL_HBM_GBS}}

    # ---- CPU baseline (rank 0, N=1) ----------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, threads, n = cpu_reference_time(preset, dtype, 3, min_seconds=10.0)
        nb = cpu_sample_batch(preset)
        cpu = {"value": nb * preset.num_queries / sec, "unit": "queries/s", "cores": threads,
               "kind": "port", "sample": f"{n} fwd+bwd steps of {nb} batch item(s) of the "
                                         f"{preset.name} workload, grid_sample oracle in "
                                         f"{str(dtype).replace('torch.', '')}"}

    # ---- other operating points and the reference's Triton kernels (N=1) ----
    workloads = None
    bar = None
    if world == 1 and not args.no_workloads and args.config == "decoder":
        workloads = {"encoder": workload_leg("encoder", torch.bfloat16, min(args.steps, 20), 3),
                     "m2f": workload_leg("m2f", torch.float16, min(args.steps, 20), 3)}
    if world == 1 and not args.no_gpu_bar:
        pd = [(preset, dtype)]
        if args.config == "decoder" and dtype == torch.bfloat16:
            pd += [(presets.get("encoder"), torch.bfloat16), (presets.get("m2f"), torch.float16)]
        bar = gpu_bar(pd, min(args.steps, 20), 3)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_total_ms / args.steps,
            "higher_is_better": True, "scaling": preset.scaling, "vs_baseline": None,
            "dtype": str(dtype).replace("torch.", ""), "data": "synthetic",
            "config": config_dict(preset, dtype, world),
            "fwd_us": fwd_mean * 1e3, "bwd_us": bwd_mean * 1e3,
            "fwd_bwd_us": (fwd_mean + bwd_mean) * 1e3,
            "fp32_grad_accum": fp32_acc, "deterministic": args.deterministic, "bwd_algo": algo,
            "in_graph_us": in_graph_us,
            "kernels_us": {k: round(t, 2) for k, (t, _) in kernels.items()},
            "kernels_us_note": "CUPTI spans; a kernel launched with programmatic dependent launch "
                               "starts before its predecessor ends, so its span includes that wait "
                               "and the spans can sum to more than the step",
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "workloads": workloads, "gpu_bar": bar,
            "gpu_launches": (None if launches_per_step is None
                             else int(round(launches_per_step * args.steps))),
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
