"""Benchmark of the W4A8 quantized linear (the headline workload) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload w4a8|w4a4|c1|mmdit|wan|ltx|sweep]
                    [--mode dp|tp|tp_fused]

One step = one pass of the hot path over one synthetic batch: activation rotation (ConvRot g256) + per-token
int8 quantization, then the packed-int4 x int8 tcgen05 GEMM with the per-group affine epilogue, bf16 out.
Workload: M=4096 tokens, K=3072, N=12288, awq-layout weights with group 128.

Timing: W warm-up steps, then K steps each bracketed by CUDA events on the launching stream; L2 is flushed
(256 MiB memset, outside the events) before every step so every step reads its inputs from HBM.  The K step
times are summed; the whole timed loop is bracketed by a barrier + synchronize; the max over ranks is taken.
N > 1 runs N data-parallel replicas (sampler batches, one process per GPU, no collective in the step:
"scaling": "weak"); ``--mode tp`` instead shards the linear's N column-parallel over the ranks (each rank rotates
and quantizes the full activation, runs its N/P columns, and an NCCL all-gather assembles the [M, N] bf16 output:
"scaling": "strong"); ``--mode tp_fused`` writes each rank's columns into every rank's output from inside the GEMM
(peer TMA stores into symmetric memory) instead of running an all-gather.

``--workload mmdit`` times one denoise step of a Qwen-Image-like 60-block dual-stream MMDiT with every linear on
the W4A8 affine path (4096 image + 256 text tokens, hidden 3072, MLP 12288; random init; graph-replayed), as
data-parallel replicas across ranks: value = steps/s over all ranks, ms_per_step = the step latency.
``--workload wan`` does the same for a Wan-2.2-5B-like 30-block video DiT (27,280 tokens, hidden 3072, FFN 14336)
whose linears follow the mixed plan: a seeded 35 % ConvRot W4A4 (Hadamard g64), the rest W8A8 int8_tensorwise.
``--workload ltx`` times one step of an LTX-like 48-block video DiT (hidden 4096, 32,768 tokens, every linear W4A8)
on one GPU, or tensor-parallel over the N ranks (head-parallel attention, column-parallel projections and MLP with
the gather inside the GEMM): value = the step latency in ms, "scaling": "strong".
``--workload sweep`` prints one line per case of the GEMM M sweep, the activation kernel at large M and the W4A4
rotation-group / SwiGLU cases.

``--impl reference`` times the reference's CPU path (dequantize-and-matmul, oracle port) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (M, K, N, rot, description)
    "w4a8": (4096, 3072, 12288, 256, "W4A8 linear, affine int4 g128 weights (bf16 scale/zero), ConvRot g256, "
                                     "per-token int8 acts, bf16 out"),
    "w4a4": (4096, 3072, 12288, 256, "ConvRot W4A4 linear, per-row int4 weights, per-token int4 acts, bf16 out"),
    "c1": (4096, 3072, 3072, 0, "W4A8 linear at K=N=3072, affine int4 g128, no rotation, per-token int8 acts"),
}


def _peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    def __init__(self, index: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self._nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()

    def summary(self) -> dict:
        if self._nv is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        nv = self._nv
        names = {
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        seen = set()
        for _, r in self.samples:
            for k, bit in names.items():
                if r & bit:
                    seen.add(k)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(self.samples)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() and args.impl == "ours" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allreduce_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bind_to_gpu_numa_node(index: int):
    """Pin this process's host threads to the CPUs of GPU `index`'s NUMA node, so that pinned host buffers allocated
    and first touched afterwards live on the node whose PCIe root the GPU hangs off.  Returns the node, or None when
    the topology cannot be read (the buffers then stay wherever the OS puts them)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        bus = pynvml.nvmlDeviceGetPciInfo(pynvml.nvmlDeviceGetHandleByIndex(index)).busId
        bus = (bus.decode() if isinstance(bus, bytes) else bus).lower()
        dom, rest = bus.split(":", 1)
        path = f"/sys/bus/pci/devices/{dom[-4:]}:{rest}/numa_node"
        node = int(open(path).read().strip())
        if node < 0:
            return None
        cpus = set()
        for part in open(f"/sys/devices/system/node/node{node}/cpulist").read().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        os.sched_setaffinity(0, cpus)
        return node
    except Exception:  # noqa: BLE001 - reported as unknown
        return None


def copy_gbs(dst: torch.Tensor, src: torch.Tensor, stream, reps: int = 5) -> float:
    """Achieved bandwidth of one host<->device copy of `src` into `dst` (median of reps, CUDA events)."""
    ts = []
    for _ in range(reps + 1):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dst.copy_(src, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return src.numel() * src.element_size() / (statistics.median(ts[1:]) / 1e3) / 1e9


def gemm_kernel_name(workload: str, m: int, n: int) -> str:
    """The GEMM kernel form the library's shape rule picks for this linear (cq_gemm_variant CQ_GEMM_AUTO)."""
    pair = m >= 1024 and ((m + 255) // 256) * ((n + 255) // 256) >= 74
    epi = "rowcol" if workload == "w4a4" else "affine"
    return f"gemm_pair_kernel<{epi}> (CTA pair, tcgen05 cta_group::2)" if pair else f"gemm_kernel<{epi}> (one SM)"


def make_problem(workload: str, seed: int, dev):
    from oracle import ref  # synthetic inputs only (seeded: N(0,1) activations with 1% outlier channels x20, N(0,0.02) weights)
    from comfy_quant_bench_b200 import ops
    m, k, n, rot, _ = WORKLOADS[workload]
    x_bits = ref.synth_activations(m, k, seed=seed)
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16).to(dev)
    w = torch.from_numpy(ref.synth_weight(n, k, seed=seed + 1)).to(dev)
    bias = torch.from_numpy(ref.synth_bias(n, seed=seed + 2).view(np.int16)).view(torch.bfloat16).to(dev)
    if workload in ("w4a8", "c1"):
        qw, s, z = ops.quantize_affine_w4_weight(w, group_size=128, convrot_groupsize=rot)
        weights = (qw, s, z)
    else:
        qw, sw = ops.quantize_convrot_w4a4_weight(w, convrot_groupsize=rot)
        weights = (qw, sw)
    del w
    return x, x_bits, weights, bias


def cpu_baseline(workload: str, rows: int, steps: int, warmup: int = 1) -> dict:
    """The reference's CPU path (oracle port, torch on all host threads), timed per linear call.

    Each timed call quantizes the activations of ``rows`` tokens, dequantizes the whole packed weight (the
    reference's eager path does this on every call) and runs the fp32 ``F.linear``.  With rows = M (the default)
    that is the real call.  With rows < M the weight dequantization, whose cost does not depend on the tokens, is
    charged once and the per-token part is scaled to M tokens: call_ms = dequant_ms + (quant_ms + linear_ms) * M / rows.
    """
    from oracle import cpu_path, ref
    m, k, n, rot, _ = WORKLOADS[workload]
    rows = max(1, min(rows, m))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = torch.from_numpy(ref.synth_activations(rows, k, seed=0).view(np.int16)).view(torch.bfloat16)
    w = ref.synth_weight(n, k, seed=1)
    qr, sr, zr = ref.weight_quant_affine(w, rot, 128)
    qw = torch.from_numpy(ref.pack_int4(qr))
    s = torch.from_numpy(sr)
    z = torch.from_numpy(zr)
    bias = torch.from_numpy(ref.bf16_bits_to_f32(ref.synth_bias(n, seed=2)))
    for _ in range(max(1, warmup)):
        cpu_path.w4a8_affine_call(x, rot, qw, s, z, bias)
    parts: list = []
    for _ in range(steps):
        cpu_path.w4a8_affine_call(x, rot, qw, s, z, bias, timings=parts)
    quant_ms, dequant_ms, linear_ms = (1e3 * sum(p[i] for p in parts) / steps for i in range(3))
    call_ms = dequant_ms + (quant_ms + linear_ms) * m / rows
    tops = 2.0 * m * n * k / (call_ms / 1e3) / 1e12
    how = ("the real call" if rows == m else
           f"{rows} of {m} tokens per timed call; call_ms = dequant_ms + (quant_ms + linear_ms) * {m}/{rows}")
    return {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port", "call_ms": call_ms,
            "split_ms": {"activation_quant": quant_ms, "weight_dequant": dequant_ms, "linear_fp32": linear_ms,
                         "tokens": rows},
            "sample": f"W4A8 linear M={m} N={n} K={k} on the CPU (torch, {threads} threads): per-token int8 "
                      f"activation quant (rotation as x @ H), whole-weight affine dequant, fp32 F.linear + bias; "
                      f"{how}; mean of {steps} calls after {max(1, warmup)} warm-up: {call_ms:.1f} ms per call"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    m, k, n, rot, desc = WORKLOADS["w4a8"]
    rows = min(args.cpu_rows, m)
    cb = cpu_baseline("w4a8", rows, max(1, args.steps), args.warmup)
    line = {
        "metric": "W4A8 linear INT8-TOPS", "value": cb["value"], "unit": "TOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["call_ms"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "w4a8_linear", "desc": desc, "M": m, "K": k, "N": n, "convrot_groupsize": rot,
                   "group_size": 128, "cpu_rows_per_step": rows},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    from comfy_quant_bench_b200 import ops, _lib
    dev = torch.device("cuda", local)
    m, k, n, rot, desc = WORKLOADS[args.workload]
    # data-parallel replicas draw their own inputs; a column-parallel layer shares one weight and one activation
    x, x_bits, weights, bias = make_problem(args.workload, seed=0 if args.mode in ("tp", "tp_fused") else rank,
                                            dev=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    # stage buffers for the kernel-level timing (same kernels the fused call enqueues)
    mp = (m + 15) // 16 * 16
    if args.mode in ("tp", "tp_fused"):
        return run_tp(args, world, rank, local, x, weights, bias)
    if args.workload in ("w4a8", "c1"):
        qw, s, z = weights
        zt = ops.prepare_affine_zeros(z, 128)   # once per weight, as the layout class does at load

        def stage1():
            return ops.rotquant(x, rot, _lib.CQ_ACT_INT8_ROW, m_pad=mp, group_sums=True, kperm=True)

        def stage2(a):
            q, sx, gs = a
            return ops.gemm_affine(q[:m], sx[:m], gs, qw, s, z, bias, a_kperm=True, zeros_prepared=zt)

        def public(xin):
            return ops.w4a8_affine_linear(xin, qw, s, z, bias, group_size=128, convrot_groupsize=rot,
                                          zeros_prepared=zt)
    else:
        qw, sw = weights

        def stage1():
            return ops.rotquant(x, rot, _lib.CQ_ACT_INT4_ROW, m_pad=mp, int4_as_int8=True, kperm=True)

        def stage2(a):
            q, sx, _ = a
            return ops.gemm_rowcol(q[:m], sx[:m], qw, sw, bias, a_kperm=True)

        def public(xin):
            return ops.convrot_w4a4_linear(xin, qw, sw, bias, convrot_groupsize=rot)

    def one_step(ev):
        # a ~0.5 ms spin on the device (outside the events) lets the host enqueue both stages before the GPU reaches
        # them, so the stage events time the kernels rather than host launch latency
        torch.cuda._sleep(1_000_000)
        ev[0].record(stream)
        a = stage1()
        ev[1].record(stream)
        stage2(a)
        ev[2].record(stream)

    for _ in range(args.warmup):
        flush.zero_()
        one_step([torch.cuda.Event(enable_timing=True) for _ in range(3)])
    torch.cuda.synchronize()
    _lib.take_device_status()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            one_step(evs[i])
        torch.cuda.synchronize()
    barrier(world)
    st = _lib.take_device_status()
    if st != (0, 0):
        raise RuntimeError(f"device status {st}")
    t_quant = [e[0].elapsed_time(e[1]) for e in evs]
    t_gemm = [e[1].elapsed_time(e[2]) for e in evs]
    per_step = [a + b for a, b in zip(t_quant, t_gemm)]
    total_ms = allreduce_max(sum(per_step), world)
    ms_per_step = total_ms / args.steps
    ops_per_step = 2.0 * m * n * k
    value = ops_per_step * args.steps * world / (total_ms / 1e3) / 1e12

    # the same step through the fused call (one C-ABI call: activation kernel, then the GEMM launched as its
    # programmatic dependent, whose prologue overlaps the activation kernel's tail), device-timed the same way
    ev_f = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(min(args.steps, 50))]
    for e0, e1 in ev_f:
        flush.zero_()
        torch.cuda._sleep(1_000_000)
        e0.record(stream)
        public(x)
        e1.record(stream)
    torch.cuda.synchronize()
    fused_call_ms = allreduce_max(statistics.mean(a.elapsed_time(b) for a, b in ev_f), world)

    # e2e through the public API with host buffers, as a pipeline: every step copies its x from pinned host memory
    # (copy stream), runs the op (compute stream; L2 flushed first), and copies its output back to pinned host memory
    # (a second copy stream).  Double buffers let step i's output copy overlap step i+1's input copy and op (the copy
    # engines run both directions at once); every step's copies are inside the timed region.
    numa_node = bind_to_gpu_numa_node(local)
    x_host = x.cpu().pin_memory()
    y_hosts = [torch.empty(m, n, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    for yh in y_hosts:
        yh.zero_()   # first touch on the GPU's node
    h2d_gbs = copy_gbs(torch.empty_like(x), x_host, stream)
    d2h_gbs = copy_gbs(y_hosts[0], torch.empty(m, n, dtype=torch.bfloat16, device=dev), stream)
    x_devs = [torch.empty_like(x) for _ in range(2)]
    s_in, s_c, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e2e_steps = max(3, min(args.steps, 50))

    def pipeline(nsteps):
        ev_in = [torch.cuda.Event() for _ in range(nsteps)]
        ev_c = [torch.cuda.Event() for _ in range(nsteps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(s_in)
        s_c.wait_event(t0)
        s_out.wait_event(t0)
        for i in range(nsteps):
            b = i % 2
            if i >= 2:
                s_in.wait_event(ev_c[i - 2])            # step i-2's op has read this input buffer
            with torch.cuda.stream(s_in):
                x_devs[b].copy_(x_host, non_blocking=True)
                ev_in[i].record(s_in)
            s_c.wait_event(ev_in[i])
            with torch.cuda.stream(s_c):
                flush.zero_()
                y = public(x_devs[b])
                ev_c[i].record(s_c)
            s_out.wait_event(ev_c[i])
            with torch.cuda.stream(s_out):
                y_hosts[b].copy_(y, non_blocking=True)   # y_hosts[b]'s previous copy is earlier on this stream
                y.record_stream(s_out)
        s_out.wait_event(ev_c[-1])
        t1.record(s_out)
        return t0, t1

    pipeline(2)
    torch.cuda.synchronize()
    barrier(world)
    t0, t1 = pipeline(e2e_steps)
    torch.cuda.synchronize()
    e2e_ms = allreduce_max(t0.elapsed_time(t1), world) / e2e_steps
    e2e_val = ops_per_step * world / (e2e_ms / 1e3) / 1e12

    # library int8 GEMM on the same shape, for context (cuBLASLt through torch._int_mm)
    lib_int8 = None
    try:
        a8 = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev)
        b8 = torch.randint(-127, 128, (k, n), dtype=torch.int8, device=dev)
        for _ in range(3):
            torch._int_mm(a8, b8)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ts = []
        for _ in range(10):
            flush.zero_()
            torch.cuda._sleep(1_000_000)
            e0.record(stream)
            torch._int_mm(a8, b8)
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        lib_int8 = {"kernel": "torch._int_mm (cuBLASLt int8, no dequant epilogue)", "ms": statistics.median(ts),
                    "tops": ops_per_step / (statistics.median(ts) / 1e3) / 1e12}
    except Exception as exc:  # noqa: BLE001
        lib_int8 = {"unavailable": str(exc).splitlines()[0][:200]}

    # The multi-GPU designs, measured beside the replicas of the headline line: the fused column-parallel linear
    # (strong scaling of the same linear over the ranks, gather inside the GEMM) at N > 1, the 60-block MMDiT step
    # as data-parallel replicas at every N, and 8 blocks of the LTX step split over the ranks (strong scaling,
    # row-parallel projections) at every N.  Every rank takes part; rank 0 reports.
    subrecords = {}
    if args.workload == "w4a8" and args.mode == "dp" and not args.no_subrecords:
        if world > 1:
            import copy
            a2 = copy.copy(args)
            a2.mode, a2.steps, a2.warmup = "tp_fused", min(args.steps, 20), max(3, min(args.warmup, 5))
            xs, _, ws, bs = make_problem("w4a8", seed=0, dev=dev)
            tl = run_tp(a2, world, rank, local, xs, ws, bs, emit=False)
            subrecords["tp_fused"] = {k: tl.get(k) for k in ("value", "unit", "ms_per_step", "per_gpu_tops",
                                                             "gather_check", "nvlink_gbs_per_rank", "scaling")}
            subrecords["tp_fused"]["parallelism"] = f"tp{world}"
            del xs, ws, bs
            torch.cuda.empty_cache()
        subrecords["mmdit_step"] = mmdit_dp_subrecord(world, rank, local)
        subrecords["ltx_step"] = ltx_tp_subrecord(world, rank, local)

    if rank != 0:
        return
    peaks = _peaks()
    gemm_ms = statistics.mean(t_gemm)
    quant_ms = statistics.mean(t_quant)
    int8_peak = 2.0 * peaks["bf16_tflops"]
    achieved = ops_per_step / (gemm_ms / 1e3) / 1e12
    traffic = None
    tf = os.path.join(ROOT, "profiles", f"gemm_{args.workload}_traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    act_bytes = m * k * 2 + m * k * 1 + m * 4 + (k // 128) * mp * 4
    line = {
        "metric": "W4A4 linear INT8-TOPS" if args.workload == "w4a4" else "W4A8 linear INT8-TOPS",
        "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"{args.workload}_linear", "desc": desc, "M": m, "K": k, "N": n,
                   "convrot_groupsize": rot, "group_size": None if args.workload == "w4a4" else 128,
                   "parallelism": f"dp{world}", "l2": "flushed before every step (256 MiB memset outside the events)",
                   "inputs": "x ~ N(0,1) bf16 with 1% outlier channels x20, W ~ N(0,0.02), bias ~ N(0,0.01), seeded"},
        "breakdown_ms": {"rotquant": quant_ms, "gemm": gemm_ms, "fused_call_overlapped": fused_call_ms,
                         "note": "value times the two kernels as separate calls (isolated); fused_call_overlapped is "
                                 "the public call, whose GEMM prologue overlaps the activation kernel's tail"},
        "step_ms_spread": {"median": statistics.median(per_step), "min": min(per_step), "max": max(per_step),
                           "of": "rank 0's device-timed steps (activation kernel + GEMM)"},
        "roofline": {"bound": "tensor", "kernel": gemm_kernel_name(args.workload, m, n),
                     "achieved": achieved, "peak": int8_peak, "unit": "TOPS", "frac": achieved / int8_peak,
                     "peak_source": f"2 x {peaks['source']} dense bf16 ({peaks['bf16_tflops']} TFLOP/s; B200 int8 "
                                    "dense rate is twice bf16)",
                     "frac_vs_library_int8": (achieved / lib_int8["tops"]) if "tops" in lib_int8 else None,
                     "traffic": traffic,
                     "traffic_source": (f"profiles/gemm_{args.workload}_traffic.json: dram__bytes_read.sum + "
                                        "dram__bytes_write.sum of one ncu capture of this kernel, not of this run")
                                       if traffic is not None else None,
                     "algorithmic": f"2*M*N*K = {ops_per_step:.4g} int-ops per launch"},
        "rotquant_roofline": {"bound": "hbm", "achieved": act_bytes / (quant_ms / 1e3) / 1e9,
                              "peak": peaks["hbm_gbs"], "unit": "GB/s",
                              "frac": act_bytes / (quant_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                              "algorithmic_bytes": act_bytes},
        "library_int8_gemm": lib_int8,
        "e2e": {"value": e2e_val, "unit": "TOPS", "ms_per_step": e2e_ms, "h2d_bytes_per_step": m * k * 2,
                "d2h_bytes_per_step": m * n * 2, "h2d_gbs": h2d_gbs, "d2h_gbs": d2h_gbs,
                "copy_bound_ms": max(m * k * 2 / h2d_gbs, m * n * 2 / d2h_gbs) / 1e6,
                "pinned_host_numa_node": numa_node,
                "path": ("ops.w4a8_affine_linear (C ABI cq_linear_w4a8_affine)" if args.workload != "w4a4" else
                         "ops.convrot_w4a4_linear (C ABI cq_linear_convrot_w4a4)") +
                        " with pinned host buffers; each step's input copy, op (after an L2 flush) and output copy run "
                        "as a three-stream pipeline over the steps"},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    line.update(subrecords)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline("w4a8" if args.workload == "w4a4" else args.workload, args.cpu_rows,
                                            args.cpu_steps)
    print(json.dumps(line), flush=True)


def run_tp(args, world, rank, local, x, weights, bias, emit=True):
    """Column-parallel linear: rotquant on every rank, the local N/P GEMM, NCCL all-gather of the bf16 output.
    Returns the JSON line (printed by rank 0 when ``emit``)."""
    import torch.distributed as dist
    from comfy_quant_bench_b200 import ops, _lib, dist as cqdist
    dev = torch.device("cuda", local)
    m, k, n, rot, desc = WORKLOADS[args.workload]
    if args.workload == "w4a4":
        raise SystemExit("--mode tp is built for the W4A8 affine workloads")
    qw, s, z, b = cqdist.shard_affine(*weights, bias, rank, world)
    zt = ops.prepare_affine_zeros(z, 128)
    nl = qw.shape[0]
    fused = cqdist.FusedColumnParallelW4A8(*weights, bias, rank, world, max_tokens=m, convrot_groupsize=rot) \
        if args.mode == "tp_fused" else None
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    mp = (m + 15) // 16 * 16
    gbuf = torch.empty(world * m, nl, dtype=torch.bfloat16, device=dev)

    align = torch.zeros(1, device=dev)

    def one_step(ev):
        torch.cuda._sleep(1_000_000)
        if world > 1:
            # line the ranks up on the device (outside the events), so that a rank whose host enqueued late does
            # not count as gather or barrier time on the others
            dist.all_reduce(align)
        ev[0].record(stream)
        if fused is not None:   # the GEMM writes every rank's output; the barriers are the only synchronization
            out = fused(x)
            ev[1].record(stream)
            ev[2].record(stream)
            return out
        q, sx, gs = ops.rotquant(x, rot, _lib.CQ_ACT_INT8_ROW, m_pad=mp, group_sums=True, kperm=True)
        y = ops.gemm_affine(q[:m], sx[:m], gs, qw, s, z, b, a_kperm=True, zeros_prepared=zt)
        ev[1].record(stream)
        if world > 1:
            dist.all_gather_into_tensor(gbuf, y)
            out = gbuf.view(world, m, nl).permute(1, 0, 2).reshape(m, world * nl)
        else:
            out = y
        ev[2].record(stream)
        return out

    for _ in range(args.warmup):
        flush.zero_()
        one_step([torch.cuda.Event(enable_timing=True) for _ in range(3)])
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            out = one_step(evs[i])
        torch.cuda.synchronize()
    barrier(world)
    if _lib.take_device_status() != (0, 0):
        raise RuntimeError("device status set")
    gather_check = None
    if fused is not None:
        # the assembled [M, N] output on this rank against this rank's own full single-GPU linear
        full = ops.w4a8_affine_linear(x, *weights, bias, 128, rot, zeros_prepared=ops.prepare_affine_zeros(weights[2], 128))
        same = torch.equal(out, full)
        bad = allreduce_max(0.0 if same else 1.0, world)
        gather_check = "bit-identical to the single-GPU linear on every rank" if bad == 0.0 else "MISMATCH"
    compute_ms = allreduce_max(sum(e[0].elapsed_time(e[1]) for e in evs), world)
    gather_ms = allreduce_max(sum(e[1].elapsed_time(e[2]) for e in evs), world)
    total_ms = allreduce_max(sum(e[0].elapsed_time(e[2]) for e in evs), world)
    ops_step = 2.0 * m * n * k
    gathered = m * n * 2
    line = {
        "metric": "W4A8 linear INT8-TOPS", "value": ops_step * args.steps / (total_ms / 1e3) / 1e12, "unit": "TOPS",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"{args.workload}_linear_column_parallel" + ("_fused_gather" if fused else ""),
                   "desc": desc, "M": m, "K": k, "N": n,
                   "N_per_rank": nl, "convrot_groupsize": rot, "group_size": 128, "parallelism": f"tp{world}",
                   "l2": "flushed before every step (256 MiB memset outside the events)"},
        "breakdown_ms": ({"rotquant_plus_gemm_with_peer_stores_and_barriers": compute_ms / args.steps} if fused else
                         {"rotquant_plus_local_gemm": compute_ms / args.steps,
                          "all_gather_plus_relayout": gather_ms / args.steps}),
        "per_gpu_tops": ops_step / world / (compute_ms / args.steps / 1e3) / 1e12,
        "all_gather": ({"bytes": gathered, "fused": "peer TMA stores inside the GEMM"} if fused else
                       {"bytes": gathered,
                        "algbw_gbs": gathered / (gather_ms / args.steps / 1e3) / 1e9 if world > 1 else None,
                        "busbw_gbs": gathered * (world - 1) / world / (gather_ms / args.steps / 1e3) / 1e9 if world > 1 else None}),
        "gpu_launches": 2 * args.steps, "clocks": clk.summary(),
    }
    if gather_check is not None:
        line["gather_check"] = gather_check
    if fused is not None and world > 1:
        # every rank sends its [M, N/P] block to the P - 1 other ranks over NVLink
        sent = m * nl * 2 * (world - 1)
        line["nvlink_gbs_per_rank"] = sent / (total_ms / args.steps / 1e3) / 1e9
    if rank == 0 and emit:
        print(json.dumps(line), flush=True)
    return line


def mmdit_dp_subrecord(world, rank, local, steps: int = 5, warmup: int = 3) -> dict:
    """The 60-block MMDiT step (fused glue, every linear W4A8) as data-parallel replicas, one CUDA graph per rank:
    step latency = max over ranks of the mean replay time; throughput = ranks / step latency."""
    from comfy_quant_bench_b200 import mmdit as mm
    dev = torch.device("cuda", local)
    model = mm.MMDiT(mm.MMDiTConfig(), device=dev, seed=0)
    img, txt, temb = model.inputs(seed=1 + rank)
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        model.step(img, txt, temb)
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        model.step(img, txt, temb)
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        model.step(img, txt, temb)
    graph.replay()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    for e0, e1 in evs:
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    step_ms = allreduce_max(sum(a.elapsed_time(b) for a, b in evs), world) / steps
    del graph, model
    torch.cuda.empty_cache()
    return {"workload": "mmdit_step (60 blocks, hidden 3072, 4096 + 256 tokens, every linear W4A8, fused glue)",
            "parallelism": f"dp{world}", "step_ms": step_ms, "steps_per_s": world / (step_ms / 1e3),
            "timing": f"{steps} graph replays per rank after {warmup} warm-up steps, max over ranks"}


def ltx_tp_subrecord(world, rank, local, blocks: int = 8, steps: int = 3, warmup: int = 2) -> dict:
    """An LTX-like video DiT step (hidden 4096, 32,768 tokens, every linear W4A8), ``blocks`` of its 48 blocks, split
    over the ranks (strong scaling): one GPU runs it whole; at N > 1 attention is head-parallel, the MLP-up
    column-parallel, the output projections and MLP-down row-parallel with NCCL all-reduces.  Eager; step latency =
    max over ranks of the mean device-timed step."""
    from comfy_quant_bench_b200 import ltx
    dev = torch.device("cuda", local)
    cfg = ltx.LTXConfig(blocks=blocks)
    model = ltx.LTXDiT(cfg, device=dev, seed=0, rank=rank, world=world)
    x, ctx = model.inputs(seed=1)
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        model.step(x, ctx)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    for e0, e1 in evs:
        e0.record(stream)
        model.step(x, ctx)
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    step_ms = allreduce_max(sum(a.elapsed_time(b) for a, b in evs), world) / steps
    del model
    torch.cuda.empty_cache()
    return {"workload": f"ltx_step ({blocks} of 48 blocks, hidden 4096, 32768 tokens, every linear W4A8)",
            "parallelism": f"tp{world}" if world > 1 else "1 GPU", "step_ms": step_ms, "ms_per_block": step_ms / blocks,
            "scaling": "strong",
            "sharding": "head-parallel attention, column-parallel MLP-up, row-parallel output projections and "
                        "MLP-down (NCCL all-reduces)" if world > 1 else None,
            "timing": f"{steps} eager steps per rank after {warmup} warm-up steps, max over ranks"}


def run_mmdit(args, world, rank, local):
    """One MMDiT denoise step per replica per iteration, graph-replayed; data-parallel over ranks."""
    from comfy_quant_bench_b200 import mmdit as mm
    dev = torch.device("cuda", local)
    cfg = mm.MMDiTConfig(blocks=args.mmdit_blocks, quantize_modulation=not args.mmdit_bf16_modulation)
    model = mm.MMDiT(cfg, device=dev, seed=0)
    img, txt, temb = model.inputs(seed=1 + rank)
    launches = model.launches_per_step()
    linears = ("every linear W4A8 affine g128, ConvRot g256 (modulation included)" if cfg.quantize_modulation else
               "every linear but the adaLN modulation W4A8 affine g128, ConvRot g256; modulation bf16 (torch), as "
               "the reference's quantization profiles leave it")
    config = {"workload": "mmdit_step", "blocks": cfg.blocks, "hidden": cfg.hidden, "heads": cfg.heads,
              "mlp": cfg.mlp, "img_tokens": cfg.img_tokens, "txt_tokens": cfg.txt_tokens, "batch": 1,
              "linears": linears,
              "glue": "layer norm + modulation fused into the QKV / MLP-up activation kernels, q/k RMSNorm + rotary "
                      "+ attention layout in one kernel" if cfg.fused_glue else "torch ops"}
    _run_dit(args, world, rank, local, model, (img, txt, temb), lambda o: o[0], "MMDiT denoise steps/s", config,
             launches)


def run_wan(args, world, rank, local):
    """One Wan-like video DiT denoise step (mixed W4A4 / W8A8 plan) per replica per iteration, graph-replayed."""
    from comfy_quant_bench_b200 import wan
    dev = torch.device("cuda", local)
    cfg = wan.WanConfig(blocks=args.wan_blocks)
    model = wan.WanDiT(cfg, device=dev, seed=0)
    x, ctx = model.inputs(seed=1 + rank)
    plan = model.plan()
    config = {"workload": "wan_step", "blocks": cfg.blocks, "hidden": cfg.hidden, "heads": cfg.heads, "ffn": cfg.ffn,
              "tokens": cfg.tokens, "grid": [cfg.frames, cfg.height, cfg.width], "ctx_tokens": cfg.ctx_tokens,
              "batch": 1,
              "linears": f"{plan['w4a4']} ConvRot W4A4 (Hadamard g{cfg.w4a4_rot}, per-row int4 weights, per-token "
                         f"int4 acts) + {plan['w8a8']} W8A8 int8_tensorwise (per-token int8 acts), seeded choice",
              "glue": ("modulated layer norms in the QKV / MLP-up activation kernels, q/k RMSNorm + rotary in one "
                       "kernel, GELU and the residual updates in the GEMM epilogues; affine layer norm and attention "
                       "torch" if cfg.fused_glue else "torch ops")}
    def block_check():
        errs = model.block_errors(x, ctx)
        return {"max_block_rel_l2": max(errs), "mean_block_rel_l2": sum(errs) / len(errs),
                "note": "teacher-forced: every block run by both paths on the kernel path's input to that block. "
                        "The step-level rel_l2 grows over the 30 blocks because per-token int4 requantization turns "
                        "a one-rounding difference in a linear's input into a code flip of 1/7 of the token scale"}

    _run_dit(args, world, rank, local, model, (x, ctx), lambda o: o, "Wan DiT denoise steps/s", config,
             model.launches_per_step(), block_check)


def run_ltx(args, world, rank, local):
    """One LTX-like video DiT step (48 blocks, hidden 4096, 32,768 tokens, every linear W4A8), tensor-parallel over
    the ranks: head-parallel attention and column-parallel MLP-up, row-parallel output projections and MLP-down
    with NCCL all-reduces (``--ltx-gather``: every linear column-parallel with the gather inside the GEMM).  Eager;
    device-timed, max over ranks."""
    from comfy_quant_bench_b200 import ltx, _lib, mmdit as mm
    dev = torch.device("cuda", local)
    cfg = ltx.LTXConfig(blocks=args.ltx_blocks)
    model = ltx.LTXDiT(cfg, device=dev, seed=0, rank=rank, world=world, row_parallel=not args.ltx_gather)
    x, ctx = model.inputs(seed=1)              # the same activation on every rank (one step, split by columns)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        out = model.step(x, ctx)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for e0, e1 in evs:
            e0.record(stream)
            out = model.step(x, ctx)
            e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    total_ms = allreduce_max(sum(a.elapsed_time(b) for a, b in evs), world)
    step_ms = total_ms / args.steps
    # e2e: the step's input from pinned host memory, the step, its output back to the host (rank 0's copy)
    hx, hc = x.cpu().pin_memory(), ctx.cpu().pin_memory()
    y_host = torch.empty_like(out, device="cpu").pin_memory()
    ee = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(2)]
    barrier(world)
    for e0, e1 in ee:
        e0.record(stream)
        x.copy_(hx, non_blocking=True)
        ctx.copy_(hc, non_blocking=True)
        out = model.step(x, ctx)
        y_host.copy_(out, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = allreduce_max(sum(a.elapsed_time(b) for a, b in ee), world) / len(ee)
    st = _lib.take_device_status()
    if st != (0, 0):
        raise RuntimeError(f"device status {st}")
    lin_ops = model.linear_int_ops()
    peaks = _peaks()
    line = {
        "metric": "LTX DiT step latency", "value": step_ms, "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 linears, bf16 glue",
        "data": "synthetic (random-init weights N(0,0.02), inputs N(0,1))",
        "config": {"workload": "ltx_step", "blocks": cfg.blocks, "hidden": cfg.hidden, "heads": cfg.heads,
                   "ffn": cfg.ffn, "tokens": cfg.tokens, "grid": [cfg.frames, cfg.height, cfg.width],
                   "ctx_tokens": cfg.ctx_tokens, "batch": 1,
                   "linears": "every linear W4A8 affine g128, ConvRot g256",
                   "parallelism": f"tp{world}" if world > 1 else "1 GPU",
                   "sharding": ("head-parallel attention (QKV / cross Q, KV rows by head) and column-parallel MLP-up "
                                "(GELU in its epilogue), all rank-local; row-parallel output projections and MLP-down "
                                "(per-token maxima all-reduced (MAX) before quantization, bf16 partial products "
                                "all-reduced (SUM) over NCCL)" if model.row_parallel else
                                "head-parallel attention (heads_to_rows peer gather); column-parallel out projections "
                                "and MLP (gather inside the GEMM)") if world > 1 else None,
                   "l2": "weights larger than L2", "graph": "none (eager)"},
        "step_latency_ms": step_ms,
        "linear_int_ops_per_step": lin_ops, "attention_flops_per_step": model.attention_flops(),
        "roofline": {"bound": "tensor", "kernel": "step-level: linear int-ops over all ranks / step time",
                     "achieved": lin_ops / (step_ms / 1e3) / 1e12, "peak": 2.0 * peaks["bf16_tflops"] * world,
                     "unit": "TOPS", "frac": lin_ops / (step_ms / 1e3) / 1e12 / (2.0 * peaks["bf16_tflops"] * world),
                     "traffic": None},
        "e2e": {"value": e2e_ms, "unit": "ms", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": (x.numel() + ctx.numel()) * 2, "d2h_bytes_per_step": out.numel() * 2,
                "path": "LTXDiT.step with pinned-host input/output copies"},
        "gpu_launches": (2 * len(model.linears()) + cfg.blocks) * args.steps,   # linears + the qkv glue per block
        "clocks": clk.summary(),
    }
    if world > 1 and not args.no_reference_check:
        # rank 0 runs the same step on one GPU (the full weights, same seed) and compares
        if rank == 0:
            single = ltx.LTXDiT(cfg, device=dev, seed=0)
            ref = single.step(x, ctx)
            line["tp_check"] = {"rel_l2_vs_one_gpu": mm.rel_l2(out, ref), "bit_identical": bool(torch.equal(out, ref))}
            del single, ref
        barrier(world)
    if rank == 0:
        print(json.dumps(line), flush=True)


def _run_dit(args, world, rank, local, model, inputs, main_out, metric, config, launches_per_step, extra_check=None):
    """Time model.step(*inputs) replayed from one CUDA graph (max over ranks), its end-to-end form with pinned host
    copies, and a reference check of rank 0's output against the fp32-linear reference step."""
    from comfy_quant_bench_b200 import _lib, mmdit as mm
    stream = torch.cuda.current_stream(torch.device("cuda", local))
    for _ in range(args.warmup):
        model.step(*inputs)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(stream.device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        model.step(*inputs)
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = main_out(model.step(*inputs))
    graph.replay()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for e0, e1 in evs:
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    total_ms = allreduce_max(sum(a.elapsed_time(b) for a, b in evs), world)
    step_ms = total_ms / args.steps
    # e2e: the step's inputs from pinned host memory into the graph's input buffers, the step, its main output back
    hosts = [t.cpu().pin_memory() for t in inputs]
    y_host = torch.empty_like(out, device="cpu").pin_memory()
    ee = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(max(3, min(args.steps, 10)))]
    barrier(world)
    for e0, e1 in ee:
        e0.record(stream)
        for t, hst in zip(inputs, hosts):
            t.copy_(hst, non_blocking=True)
        graph.replay()
        y_host.copy_(out, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = allreduce_max(sum(a.elapsed_time(b) for a, b in ee), world) / len(ee)
    st = _lib.take_device_status()
    if st != (0, 0):
        raise RuntimeError(f"device status {st}")
    lin_ops = model.linear_int_ops()
    peaks = _peaks()
    config = dict(config, parallelism=f"dp{world}", l2="weights (%.1f GB) larger than L2" % (model.weight_bytes() / 1e9),
                  graph="one CUDA graph per step")
    line = {
        "metric": metric, "value": world * args.steps / (total_ms / 1e3), "unit": "steps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/int4 linears, bf16 glue",
        "data": "synthetic (random-init weights N(0,0.02), inputs N(0,1))",
        "config": config,
        "step_latency_ms": step_ms,
        "linear_int_ops_per_step": lin_ops, "attention_flops_per_step": model.attention_flops(),
        "roofline": {"bound": "tensor", "kernel": "step-level: linear int-ops / step time (the GEMM kernels alone are "
                                                  "measured by the linear workloads)",
                     "achieved": lin_ops / (step_ms / 1e3) / 1e12, "peak": 2.0 * peaks["bf16_tflops"], "unit": "TOPS",
                     "frac": lin_ops / (step_ms / 1e3) / 1e12 / (2.0 * peaks["bf16_tflops"]), "traffic": None},
        "e2e": {"value": world / (e2e_ms / 1e3), "unit": "steps/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in inputs),
                "d2h_bytes_per_step": out.numel() * out.element_size(),
                "path": "graph-replayed step with pinned-host input/output copies"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and not args.no_reference_check:
        ref = main_out(model.step(*inputs, reference=True))
        line["reference_check"] = {"rel_l2": mm.rel_l2(out, ref),
                                   "against": "the same step with every linear as a torch fp32 product of the "
                                              "dequantized weight and the dequantized activation codes"}
        if extra_check is not None:
            line["reference_check"].update(extra_check())
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline("w4a8", args.cpu_rows, args.cpu_steps)
        line["cpu_baseline"] = {"value": cb["value"] * 1e12 / lin_ops, "unit": "steps/s", "cores": cb["cores"],
                                "kind": cb["kind"],
                                "sample": cb["sample"] + "; steps/s = that CPU rate over the step's linear int-ops "
                                                         "(attention and glue not counted)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph


def run_sweep(args, world, rank, local):
    """One JSON line per case: the W4A8 GEMM sweep over M, the activation kernel at large M, and the W4A4
    (ConvRot 256/64/16, SwiGLU prologue) linears.  Device-timed with CUDA events after a device-side lead; L2 is
    flushed before every timed call; each line is the median of the calls."""
    from comfy_quant_bench_b200 import ops, _lib
    dev = torch.device("cuda", local)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    peaks = _peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]

    spread = {}                           # the last timed case's fastest and slowest call, added to its line

    def timed(fn, reps):
        for _ in range(2):
            fn()
        ts = []
        for _ in range(reps):
            flush.zero_()
            torch.cuda._sleep(1_000_000)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        spread.update(ms_min=min(ts), ms_max=max(ts))
        return statistics.median(ts)

    def emit(d):
        if rank == 0:
            print(json.dumps({**d, **spread}), flush=True)

    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    # --- W4A8 affine GEMM sweep (activation kernel + GEMM per call), M x (N, K) ---
    for n, k in ((12288, 4096), (4096, 4096), (16384, 4096), (4096, 16384)):
        w = torch.randn(n, k, generator=gen, device=dev) * 0.02
        qw, sc, z = ops.quantize_affine_w4_weight(w, 128, 256)
        zt = ops.prepare_affine_zeros(z, 128)
        del w
        for m in (256, 512, 1024, 2048, 4096, 8192, 16384, 32768, 65536):
            x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
            ms = timed(lambda: ops.w4a8_affine_linear(x, qw, sc, z, None, 128, 256, zeros_prepared=zt), args.steps)
            emit({"case": "w4a8_affine_linear", "M": m, "N": n, "K": k, "ms": ms,
                  "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12, "frac_of_int8_peak": 2.0 * m * n * k / (ms / 1e3) / 1e12 / int8_peak})
            del x
        torch.cuda.empty_cache()
    # --- a few tokens (adaLN modulation: M=1, N=6*3072, K=3072): the one-warp-per-row product, bound by reading
    #     the packed weights, scales and zeros once ---
    n, k = 6 * 3072, 3072
    w = torch.randn(n, k, generator=gen, device=dev) * 0.02
    qw, sc, z = ops.quantize_affine_w4_weight(w, 128, 256)
    zt = ops.prepare_affine_zeros(z, 128)
    del w
    for m in (1, 8):
        x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
        ms = timed(lambda: ops.w4a8_affine_linear(x, qw, sc, z, None, 128, 256, zeros_prepared=zt), args.steps)
        byts = n * k // 2 + 2 * (k // 128) * n * 2
        emit({"case": "w4a8_affine_linear_few_tokens", "M": m, "N": n, "K": k, "ms": ms,
              "weight_gbs": byts / (ms / 1e3) / 1e9, "frac_of_hbm": byts / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
              "note": "activation kernel + product; weight bytes = packed codes + bf16 scales and zeros"})
    # --- activation rotation + int8 quantization at large M (HBM-bound) ---
    for m in (4096, 32768, 65536):
        k = 3072
        x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
        ms = timed(lambda: ops.rotquant(x, 256, _lib.CQ_ACT_INT8_ROW, group_sums=True, kperm=True), args.steps)
        byts = m * k * 2 + m * k + m * 4 + m * 2 * 64 * ((k // 128 + 31) // 32)
        emit({"case": "rotquant_int8_convrot256", "M": m, "K": k, "ms": ms, "gbs": byts / (ms / 1e3) / 1e9,
              "frac_of_hbm": byts / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]})
        # the reference's packed-int4 quantizer (quantize_int4_rowwise_convrot64): codes [M, K/2] + scales [M]
        ms = timed(lambda: ops.quantize_int4_rowwise_convrot64(x, 256), args.steps)
        byts = m * k * 2 + m * k // 2 + m * 4
        emit({"case": "rotquant_int4_packed_convrot256", "M": m, "K": k, "ms": ms, "gbs": byts / (ms / 1e3) / 1e9,
              "frac_of_hbm": byts / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]})
        del x
    # the fused SwiGLU quantizer (swiglu_quantize_int4_rowwise_convrot64) on h [M, 2 * 12288]
    for m in (4096, 32768):
        k = 12288
        h = torch.randn(m, 2 * k, generator=gen, device=dev).to(torch.bfloat16)
        ms = timed(lambda: ops.swiglu_quantize_int4_rowwise_convrot64(h), args.steps)
        byts = m * 2 * k * 2 + m * k // 2 + m * 4
        emit({"case": "swiglu_rotquant_int4_packed_convrot256", "M": m, "K": k, "ms": ms,
              "gbs": byts / (ms / 1e3) / 1e9, "frac_of_hbm": byts / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]})
        del h
    # --- W4A4 ConvRot linears (M=4096, K=3072, N=12288): rotation groups and the SwiGLU prologue ---
    m, k, n = 4096, 3072, 12288
    w = torch.randn(n, k, generator=gen, device=dev) * 0.02
    x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
    for rot in (256, 64, 16):
        qw, sw = ops.quantize_convrot_w4a4_weight(w, rot)
        ms = timed(lambda: ops.convrot_w4a4_linear(x, qw, sw, None, convrot_groupsize=rot), args.steps)
        emit({"case": "convrot_w4a4_linear", "M": m, "N": n, "K": k, "rot": rot, "ms": ms,
              "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12})
    # SwiGLU epilogue variant: the N=12288 up projection with silu(y[:, :6144]) * y[:, 6144:] formed in the epilogue
    qw, sw = ops.quantize_convrot_w4a4_weight(w, 256)
    qg, sg, _ = ops.prepare_swiglu_output_weight(qw, sw)
    ms = timed(lambda: ops.convrot_w4a4_linear_swiglu(x, qg, sg, None, convrot_groupsize=256), args.steps)
    emit({"case": "convrot_w4a4_linear_swiglu_epilogue", "M": m, "N": n, "K": k, "rot": 256, "out_cols": n // 2,
          "ms": ms, "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12})
    def unfused():
        y = ops.convrot_w4a4_linear(x, qw, sw, None, convrot_groupsize=256)
        return torch.nn.functional.silu(y[:, :n // 2]) * y[:, n // 2:]

    ms = timed(unfused, args.steps)
    emit({"case": "convrot_w4a4_linear_then_torch_swiglu", "M": m, "N": n, "K": k, "rot": 256, "out_cols": n // 2,
          "ms": ms, "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12})
    kd, nd = 6144, 3072   # down projection after SwiGLU: h [M, 2*6144] -> silu(g)*u -> [M, 6144] @ W^T
    wd = torch.randn(nd, kd, generator=gen, device=dev) * 0.02
    qd, sd = ops.quantize_convrot_w4a4_weight(wd, 256)
    h = torch.randn(m, 2 * kd, generator=gen, device=dev).to(torch.bfloat16)
    ms = timed(lambda: ops.convrot_w4a4_linear(h, qd, sd, None, convrot_groupsize=256, input_act="swiglu"), args.steps)
    emit({"case": "convrot_w4a4_linear_swiglu_prologue", "M": m, "N": nd, "K": kd, "rot": 256, "ms": ms,
          "tops": 2.0 * m * nd * kd / (ms / 1e3) / 1e12})
    # --- per-group scales on both sides (the reference GEMM's policy 4): the node's forward at T, and the GEMM
    #     alone at the reference bench's 4096^3 ---
    for m, n, k in ((4096, 12288, 3072), (4096, 4096, 4096)):
        w = torch.randn(n, k, generator=gen, device=dev) * 0.02
        qg, sg = ops.quantize_int4_groupwise_weight(w, 128, 256)
        x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
        ms = timed(lambda: ops.w4a4_groupwise_linear(x, qg, sg), args.steps)
        emit({"case": "w4a4_groupwise_linear_policy4", "M": m, "N": n, "K": k, "ms": ms,
              "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12, "frac_of_int8_peak": 2.0 * m * n * k / (ms / 1e3) / 1e12 / int8_peak,
              "note": "per-group activation quantizer + g128 x g128 GEMM (policy 4)"})
        qa, sa = ops.quant(x, 128)
        ms = timed(lambda: ops.gemm(qa, qg, sa, sg, pol=4), args.steps)
        emit({"case": "gemm_policy4", "M": m, "N": n, "K": k, "ms": ms,
              "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12, "frac_of_int8_peak": 2.0 * m * n * k / (ms / 1e3) / 1e12 / int8_peak})
        del w, x
    # --- integer weight ratios (policies 5 / 7 / 17) at the reference bench's 4096^3: int4 codes, ratios in [1, 255] ---
    m = n = k = 4096
    a4 = torch.randint(-7, 8, (m, k), generator=gen, device=dev, dtype=torch.int8)
    b4 = torch.randint(-7, 8, (n, k), generator=gen, device=dev, dtype=torch.int8)
    ap = ((a4[:, 0::2].to(torch.int16) & 0xF) | ((a4[:, 1::2].to(torch.int16) & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    bp = ((b4[:, 0::2].to(torch.int16) & 0xF) | ((b4[:, 1::2].to(torch.int16) & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    sa_r = torch.rand(m, generator=gen, device=dev) * 0.01 + 0.005
    sb_r = (torch.rand(n, generator=gen, device=dev) * 0.01 + 0.005) / 255
    for pol in (5, 7, 17):
        grp = 64 if pol % 10 == 5 else 128
        cw = torch.randint(1, 256, (k // grp, n), generator=gen, device=dev, dtype=torch.int32)
        if pol >= 10:
            cw = cw.to(torch.uint8)
        ms = timed(lambda: ops.gemm(ap, bp, sa_r, sb_r, None, cw, None, pol=pol), args.steps)
        emit({"case": f"gemm_policy{pol}", "M": m, "N": n, "K": k, "ms": ms,
              "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12, "frac_of_int8_peak": 2.0 * m * n * k / (ms / 1e3) / 1e12 / int8_peak,
              "note": "includes the activations' int4 unpack (the reference interface takes packed codes)"})
    del a4, b4, ap, bp
    # --- output operations in the affine epilogue (a DiT block's MLP-up with GELU, output projections with the
    #     gated residual), against the plain linear followed by the torch op ---
    for m, n, k, op in ((4096, 12288, 3072, "gelu"), (4096, 3072, 3072, "gated"), (4096, 3072, 12288, "gated")):
        w = torch.randn(n, k, generator=gen, device=dev) * 0.02
        qw, sc, z = ops.quantize_affine_w4_weight(w, 128, 256)
        zt = ops.prepare_affine_zeros(z, 128)
        x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
        res = torch.randn(m, n, generator=gen, device=dev).to(torch.bfloat16)
        gate = torch.randn(n, generator=gen, device=dev).to(torch.bfloat16)
        kw = {"residual": res, "gate": gate} if op == "gated" else {}
        ms = timed(lambda: ops.w4a8_affine_linear_op(x, qw, sc, zt, None, out_op=op, convrot_groupsize=256, **kw),
                   args.steps)

        def then_torch():
            y = ops.w4a8_affine_linear(x, qw, sc, z, None, 128, 256, zeros_prepared=zt)
            return torch.nn.functional.gelu(y, approximate="tanh") if op == "gelu" else torch.addcmul(res, gate, y)

        ms_t = timed(then_torch, args.steps)
        emit({"case": f"w4a8_affine_linear_epilogue_{op}", "M": m, "N": n, "K": k, "ms": ms,
              "ms_linear_then_torch_op": ms_t})
        del w, x, res
    # --- row-parallel activation stage (LTX MLP-down slice on one of 8 ranks: K = 16384 / 8), both phases ---
    m, k = 32768, 2048
    x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
    amax = ops.rotquant_absmax(x, 256)
    ms1 = timed(lambda: ops.rotquant_absmax(x, 256), args.steps)
    ms2 = timed(lambda: ops.rotquant_scaled(x, 256, amax, group_sums=True, kperm=True), args.steps)
    ms0 = timed(lambda: ops.rotquant(x, 256, _lib.CQ_ACT_INT8_ROW, group_sums=True, kperm=True), args.steps)
    emit({"case": "rotquant_row_parallel_phases", "M": m, "K": k, "ms_absmax": ms1, "ms_scaled": ms2,
          "ms_single_pass": ms0, "note": "the all-reduce MAX of the [2, M] maxima runs between the two phases"})
    del x
    if _lib.take_device_status() != (0, 0):
        raise RuntimeError("device status set")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["mmdit", "wan", "ltx", "sweep"], default="w4a8")
    ap.add_argument("--mode", choices=["dp", "tp", "tp_fused"], default="dp")
    ap.add_argument("--mmdit-blocks", type=int, default=60)
    ap.add_argument("--mmdit-bf16-modulation", action="store_true",
                    help="keep the adaLN modulation linears in bf16 (the reference's profiles exclude them)")
    ap.add_argument("--wan-blocks", type=int, default=30)
    ap.add_argument("--ltx-blocks", type=int, default=48)
    ap.add_argument("--ltx-gather", action="store_true",
                    help="LTX at N>1: every linear column-parallel with the gather inside the GEMM, instead of "
                         "row-parallel output projections and MLP-down with all-reduces")
    ap.add_argument("--no-reference-check", action="store_true")
    ap.add_argument("--cpu-rows", type=int, default=4096,
                    help="tokens per timed CPU call (default: the workload's M, the real call)")
    ap.add_argument("--cpu-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="skip the fused column-parallel and MMDiT-step measurements beside the headline line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "mmdit":
            run_mmdit(args, world, rank, local)
        elif args.workload == "wan":
            run_wan(args, world, rank, local)
        elif args.workload == "ltx":
            run_ltx(args, world, rank, local)
        elif args.workload == "sweep":
            run_sweep(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
