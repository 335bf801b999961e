"""Benchmark of the tensorcrate CUDA backend's hot path on B200.

Default workload ("config 2", the headline benchmark's configuration): one step is the
nine broadcast and reduction calls the reference's config names, on f32
x[64,512,1024] ~ N(0,1) and bias[1,1,1024] ~ N(0,1):
    x + bias, x * bias, x > bias          (Kernels::strided_binary)
    sum, mean, var over axis 2           (Kernels::reduce_axes)
    max, min over axes (0, 2)            (Kernels::reduce_axes)
    argmax over axis 1                   (Kernels::arg_reduce)
metric: HBM GB/s = algorithmic bytes of the nine calls / step time.

Under torchrun each rank holds its own [64,512,1024] slab of a
[64*P,512,1024] tensor (weak scaling): the per-slab results are final
locally and are all-gathered; max/min over (0,2) reduce across the sharded
axis, so their [512] partials are all-reduced (NCCL).

Other workloads (--workload): c1 (f32 1024^3 GEMM + matvec), c3 (f16 layout
copies), c4 (MLP training step), c5 (bf16 GEMM, --size), trait (the other
Kernels<T> methods, each timed alone).  --impl reference times the reference's
Host path restated in C++ (oracle/) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def traffic(workload: str, kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, or
    None if that kernel was not captured."""
    try:
        return json.loads((ROOT / "profiles" / "traffic.json").read_text())[workload].get(kernel)
    except Exception:
        return None


def peaks() -> tuple[dict, str]:
    try:
        return json.loads(PEAKS_FILE.read_text()), "measured"
    except Exception:
        return dict(FALLBACK), "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    """SM clock and clock-event reasons sampled through NVML every ~2 ms
    while the timed region runs (the same counters nvidia-smi reports)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, torch_device: int):
        self.dev, self.samples, self.max_mhz, self.error = torch_device, [], None, None
        self._stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            props = torch.cuda.get_device_properties(self.dev)
            try:
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                self.h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = nv.nvmlDeviceGetHandleByIndex(self.dev)
            self.nv = nv
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception as e:  # no NVML: report it
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _run(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM), int(get_reasons(self.h))))
            except Exception as e:
                self.error = str(e)
                return
            time.sleep(0.002)

    def __exit__(self, *exc):
        self._stop.set()
        if getattr(self, "thread", None):
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "error": self.error}
        mhz = [m for m, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# config 2 on the GPU
# ---------------------------------------------------------------------------
SHAPE2 = [64, 512, 1024]
MB = 1e6


def c2_ops_bytes():
    n = int(np.prod(SHAPE2)) * 4
    rows = SHAPE2[0] * SHAPE2[1]
    return {
        "add": 2 * n + 4096, "mul": 2 * n + 4096, "greater": 2 * n + 4096,
        "sum": n + rows * 4, "mean": n + rows * 4, "var": n + rows * 4,
        "max": n + 512 * 4, "min": n + 512 * 4,
        "argmax": n + SHAPE2[0] * SHAPE2[2] * 4,
    }


def run_c2(args, torch, world, rank, comm):
    from tensorcrate_b200 import _native as N
    from tensorcrate_b200 import cuda

    lib = N.lib()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    shape = SHAPE2
    n = int(np.prod(shape))
    rng = np.random.default_rng(1 + rank)
    x_host = rng.standard_normal(n, dtype=np.float32)
    bias_host = np.random.default_rng(2).standard_normal(1024, dtype=np.float32)
    x = cuda.CudaStorage.store(x_host, "f32")
    bias = cuda.CudaStorage.store(bias_host, "f32")
    rows = shape[0] * shape[1]
    outs = {k: cuda.CudaStorage("f32", n) for k in ("add", "mul", "greater")}
    # The reductions' results sit side by side in one block of 4-byte
    # elements, so that one all-gather carries all of them when P > 1.
    fields = [("sum", "f32", rows), ("mean", "f32", rows), ("var", "f32", rows),
              ("argmax", "u32", shape[0] * shape[2]), ("max", "f32", 512), ("min", "f32", 512)]
    pack_len = sum(c for _, _, c in fields)
    pack = cuda.CudaStorage("u32", pack_len)
    at = {}
    offset = 0
    for k, dt, count in fields:
        outs[k] = cuda.CudaStorage(dt, count, ptr=pack.ptr + 4 * offset)
        at[k] = offset
        offset += count

    sz = N.sizes
    xs, xst = sz(shape), sz(cuda.contiguous_strides(shape))
    bst = sz([0, 0, 1])
    ax2, ax02 = N.u32s([2]), N.u32s([0, 2])
    argp = C.cast(C.c_void_p(outs["argmax"].ptr), C.POINTER(C.c_uint32))

    def calls_on(x):
        """The nine calls of a step on the input at `x`."""
        return [
            ("add", lib.tc_strided_binary, (0, N.PAIR_ARITHMETIC, N.ADD, 3, xs, x.ptr, n, 0, xst, bias.ptr, 1024, 0, bst,
                                            outs["add"].ptr, sp)),
            ("mul", lib.tc_strided_binary, (0, N.PAIR_ARITHMETIC, N.MUL, 3, xs, x.ptr, n, 0, xst, bias.ptr, 1024, 0, bst,
                                            outs["mul"].ptr, sp)),
            ("greater", lib.tc_strided_binary, (0, N.PAIR_COMPARE, N.GREATER, 3, xs, x.ptr, n, 0, xst, bias.ptr, 1024, 0,
                                                bst, outs["greater"].ptr, sp)),
            ("sum", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 1, ax2, N.AXIS_FOLD, N.SUM, 0, outs["sum"].ptr, sp)),
            ("mean", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 1, ax2, N.AXIS_MEAN, 0, 0, outs["mean"].ptr, sp)),
            ("var", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 1, ax2, N.AXIS_VARIANCE, 0, 1024, outs["var"].ptr,
                                         sp)),
            ("max", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 2, ax02, N.AXIS_FOLD, N.RMAX, 0, outs["max"].ptr, sp)),
            ("min", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 2, ax02, N.AXIS_FOLD, N.RMIN, 0, outs["min"].ptr, sp)),
            ("argmax", lib.tc_arg_reduce, (0, 3, xs, x.ptr, n, 0, xst, 1, N.RMAX, argp, sp)),
        ]

    calls = calls_on(x)

    # Collectives for P > 1: one all-gather of every rank's block of results
    # (the slab results are then final, rank after rank); the [512] extremes
    # fold the sharded leading axis, so each is finished by reducing the P
    # gathered partials ([P, 512] with a stride of one block), exactly.
    gathered = cuda.CudaStorage("u32", pack_len * world) if world > 1 else None
    finals = {k: cuda.CudaStorage("f32", 512) for k in ("max", "min")} if world > 1 else {}
    g_shape, g_strides = sz([world, 512]), sz([pack_len, 1])

    def collectives():
        if world == 1:
            return
        N.check("allgather", lib.tc_allgather(comm, N.U32, pack.ptr, gathered.ptr, pack_len, sp))
        for k, op in (("max", N.RMAX), ("min", N.RMIN)):
            N.check("fold", lib.tc_reduce_axes(0, 2, g_shape, gathered.ptr, pack_len * world, at[k], g_strides, 1,
                                               N.u32s([0]), N.AXIS_FOLD, op, 0, finals[k].ptr, sp))

    events = {name: [] for name, _, _ in calls}

    def step(record=False, on=None):
        for name, fn, a in (on or calls):
            if record:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                st = fn(*a)
                e1.record(stream)
                events[name].append((e0, e1))
            else:
                st = fn(*a)
            if st:
                N.check(name, st)
        collectives()

    bytes_per_op = c2_ops_bytes()
    step_bytes = sum(bytes_per_op.values())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # device-timed region
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(torch.cuda.current_device()) as clocks:
        barrier(torch, world)
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        barrier(torch, world)
    ms = t0.elapsed_time(t1)
    ms = max_over_ranks(torch, world, ms)
    # Per-operation times, from events around each call, in a pass of their
    # own (events between the calls would sit inside the timed region).
    for _ in range(min(args.steps, 50)):
        step(record=True)
    torch.cuda.synchronize()
    per_op_ms = {k: statistics.mean(a.elapsed_time(b) for a, b in v) for k, v in events.items()}

    # e2e: through the public API with host buffers (pinned), copies inside.
    pinned_x = torch.from_numpy(x_host).pin_memory()
    pinned_b = torch.from_numpy(bias_host).pin_memory()
    out_host = {k: torch.empty(o.nbytes, dtype=torch.uint8).pin_memory() for k, o in outs.items()
                if k not in ("add", "mul", "greater")}
    h2d = pinned_x.numel() * 4 + pinned_b.numel() * 4
    d2h = sum(v.numel() for v in out_host.values())

    def e2e_step():
        N.check("h2d", lib.tc_memcpy_h2d(x.ptr, pinned_x.data_ptr(), pinned_x.numel() * 4, sp))
        N.check("h2d", lib.tc_memcpy_h2d(bias.ptr, pinned_b.data_ptr(), pinned_b.numel() * 4, sp))
        step()
        for k, h in out_host.items():
            N.check("d2h", lib.tc_memcpy_d2h(h.data_ptr(), outs[k].ptr, h.numel(), sp))

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(torch, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps = max(3, args.steps // 4)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    serial_ms = max_over_ranks(torch, world, e0.elapsed_time(e1) / e2e_steps)

    # The same steps as a streaming caller runs them: two device copies of
    # the input, step k+1's upload on a copy stream while step k's kernels
    # run (each upload waits for the step that last read its buffer; each
    # step waits for its own upload).  Every step still uploads its input
    # and reads its results back inside the timed region.
    x2 = cuda.CudaStorage("f32", n)
    bufs, on = [x, x2], [calls, calls_on(x2)]
    copy_stream = torch.cuda.Stream()
    csp = C.c_void_p(copy_stream.cuda_stream)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]

    def upload(k):
        b = k % 2
        if k >= 2:
            copy_stream.wait_event(consumed[b])
        N.check("h2d", lib.tc_memcpy_h2d(bufs[b].ptr, pinned_x.data_ptr(), pinned_x.numel() * 4, csp))
        copied[b].record(copy_stream)

    def pipelined(steps):
        copy_stream.wait_stream(stream)
        upload(0)
        for k in range(steps):
            if k + 1 < steps:
                upload(k + 1)
            stream.wait_event(copied[k % 2])
            N.check("h2d", lib.tc_memcpy_h2d(bias.ptr, pinned_b.data_ptr(), pinned_b.numel() * 4, sp))
            step(on=on[k % 2])
            consumed[k % 2].record(stream)
            for kk, h in out_host.items():
                N.check("d2h", lib.tc_memcpy_d2h(h.data_ptr(), outs[kk].ptr, h.numel(), sp))

    pipelined(2)
    torch.cuda.synchronize()
    barrier(torch, world)
    e0.record(stream)
    pipelined(e2e_steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, world, e0.elapsed_time(e1) / e2e_steps)

    ms_per_step = ms / args.steps
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9
    # Dominant kernel: the largest share of the step.
    dom = max(per_op_ms, key=lambda k: per_op_ms[k])
    pk, pk_kind = peaks()
    achieved = bytes_per_op[dom] / (per_op_ms[dom] * 1e-3) / 1e9
    ops = {k: {"ms": round(v, 5), "gbs": round(bytes_per_op[k] / (v * 1e-3) / 1e9, 1),
               "frac": round(bytes_per_op[k] / (v * 1e-3) / 1e9 / pk["hbm_gbs"], 3)} for k, v in per_op_ms.items()}
    line = {
        "metric": "config-2 broadcast + axis-reduction HBM throughput (GB/s)",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "config2: f32 x[64,512,1024] with bias[1,1,1024]: add, mul, greater; sum/mean/var ax2; "
                               "max/min ax(0,2); argmax ax1",
                   "per_rank_shape": SHAPE2, "global_shape": [64 * world, 512, 1024],
                   "parallelism": f"leading-axis shards x{world}" + (" (one NCCL all-gather of every result, "
                                                                     "then max/min folded over ranks)" if world > 1
                                                                     else ""),
                   "l2": "no flush: every call reads the 134.2 MB input, larger than the 126 MB L2",
                   "algorithmic_bytes_per_step": step_bytes},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                     "peak_source": pk_kind, "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 3),
                     "traffic": traffic("c2", dom), "algorithmic_bytes": bytes_per_op[dom]},
        "ops": ops,
        "e2e": {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "pipelined": "each step's input upload overlaps the previous step's kernels (two device buffers, "
                             "a copy stream)",
                "serial_ms_per_step": round(serial_ms, 4)},
        "gpu_launches": (len(calls) + (2 if world > 1 else 0)) * args.steps,
        "clocks": clocks.summary(),
    }
    return line


# ---------------------------------------------------------------------------
# CPU: the reference's Host path (oracle restatement) on a bounded sample
# ---------------------------------------------------------------------------
def cpu_c2(sample_rows: int = 16, reps: int = 1):
    import oracle as O

    shape = [sample_rows, 512, 1024]
    n = int(np.prod(shape))
    x = np.random.default_rng(1).standard_normal(n, dtype=np.float32)
    bias = np.random.default_rng(2).standard_normal(1024, dtype=np.float32)
    st = [512 * 1024, 1024, 1]
    t = time.perf_counter()
    for _ in range(reps):
        O.strided_binary("f32", 0, 0, shape, x, 0, st, bias, 0, [0, 0, 1])
        O.strided_binary("f32", 0, 2, shape, x, 0, st, bias, 0, [0, 0, 1])
        O.strided_binary("f32", 1, 5, shape, x, 0, st, bias, 0, [0, 0, 1])
        O.reduce_axes("f32", shape, x, 0, st, [2], 0, 0, 0)
        O.reduce_axes("f32", shape, x, 0, st, [2], 1, 0, 0)
        O.reduce_axes("f32", shape, x, 0, st, [2], 2, 0, 1024)
        O.reduce_axes("f32", shape, x, 0, st, [0, 2], 0, 2, 0)
        O.reduce_axes("f32", shape, x, 0, st, [0, 2], 0, 1, 0)
        O.arg_reduce("f32", shape, x, 0, st, 1, 2)
    dt = (time.perf_counter() - t) / reps
    scale = sample_rows / SHAPE2[0]
    step_bytes = sum(c2_ops_bytes().values()) * scale
    return {"value": round(step_bytes / dt / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"all nine calls on a [{sample_rows},512,1024] slab ({scale:.3g} of config 2), x{reps}, "
                      "single-threaded as the Host runs strided kernels",
            "seconds": round(dt * reps, 2)}


def timed(torch, world, fn, steps, warmup, stream, per_call=None):
    """Run fn warmup times, then time `steps` calls with CUDA events on
    `stream` (max over ranks).  Returns (ms per step, clocks summary)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(torch.cuda.current_device()) as clocks:
        barrier(torch, world)
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(steps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize()
        barrier(torch, world)
    return max_over_ranks(torch, world, t0.elapsed_time(t1)) / steps, clocks.summary()


def run_gemm(args, torch, world, rank, comm, dtype="bf16", size=8192):
    """Config 5 (bf16, M=N=K=size) or config 1 (f32 1024^3): C = A.B through
    tc_matmul, inputs resident.  metric TFLOP/s."""
    from tensorcrate_b200 import _native as N
    from tensorcrate_b200 import cuda
    lib = N.lib()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    m = k = n = size
    rng = np.random.default_rng(0)
    a_host = cuda.f32_to_bits(rng.uniform(-1, 1, m * k).astype(np.float32), dtype)
    b = cuda.CudaStorage.store(cuda.f32_to_bits(rng.uniform(-1, 1, k * n).astype(np.float32), dtype), dtype)
    code = N.DTYPES[dtype]
    panels = world > 1 and dtype != "f32"
    peer = None
    if panels:
        # Row panels: rank r computes rows [r*m/P, (r+1)*m/P) of C with B
        # replicated; the GEMM epilogue stores each tile into every rank's C.
        if m % world:
            raise SystemExit(f"M={m} does not split over {world} ranks")
        rows = m // world
        a = cuda.CudaStorage.store(a_host[rank * rows * k:(rank + 1) * rows * k], dtype)
        from tensorcrate_b200.sharding import PeerBuffer
        peer = PeerBuffer(comm, m * n * 2)

        def step():
            N.check("matmul_allgather", lib.tc_matmul_allgather(comm, code, rows, k, n, a.ptr, b.ptr, peer.handle, sp))
    else:
        a = cuda.CudaStorage.store(a_host, dtype)
        c = cuda.CudaStorage(dtype, m * n)

        def step():
            N.check("matmul", lib.tc_matmul(code, 0, m, k, n, a.ptr, b.ptr, c.ptr, 0, sp))

    ms, clocks = timed(torch, world, step, args.steps, args.warmup, stream)
    if peer is not None:
        peer.close()
    matvec = None
    if dtype == "f32" and size == 1024:
        # Config 1's matvec: y = M.x over 64 different [1024 x 1024] f32
        # matrices in turn (268 MB, more than L2), so every call reads HBM.
        mats = [cuda.CudaStorage.store(rng.uniform(-1, 1, m * k).astype(np.float32), "f32") for _ in range(64)]
        xv = cuda.CudaStorage.store(rng.uniform(-1, 1, k).astype(np.float32), "f32")
        yv = cuda.CudaStorage("f32", m)
        # The 64 launches are captured in one CUDA graph, so the time is the
        # device's and not the host's launch rate through ctypes.
        graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.graph(graph, stream=cap):
            csp = C.c_void_p(cap.cuda_stream)
            for M in mats:
                N.check("matvec", lib.tc_matvec(N.F32, m, k, M.ptr, xv.ptr, yv.ptr, 0, csp))
        ms_mv, _ = timed(torch, world, graph.replay, 8, 3, stream)
        ms_mv /= len(mats)
        mv_bytes = m * k * 4 + k * 4 + m * 4
        mv_gbs = mv_bytes / (ms_mv * 1e-3) / 1e9
        matvec = {"us": round(ms_mv * 1e3, 2), "gbs": round(mv_gbs, 1), "frac": round(mv_gbs / peaks()[0]["hbm_gbs"], 3),
                  "bytes": mv_bytes, "l2": "64 matrices in turn, 268 MB"}
    flops = 2.0 * m * n * k
    pk, pk_kind = peaks()
    # Whole-job TFLOP/s: replicas each do the whole product; panels share one.
    total = flops / (ms * 1e-3) / 1e12 * (1 if panels else world)
    per_gpu = total / world
    # f32 runs as three TF32 tensor-core passes (hi.hi + hi.lo + lo.hi): the
    # roofline counts those passes' flops against half the bf16 rate, the
    # tensor cores' TF32 throughput.
    passes = 3 if dtype == "f32" else 1
    peak = pk["bf16_tflops"] / (2 if dtype == "f32" else 1)
    workload = f"config{'5' if dtype != 'f32' else '1'}: C = A.B, M=N=K={size}, f32 accumulate"
    parallelism = (f"row panels x{world}, all-gather fused into the GEMM epilogue (NVLink peer stores)" if panels
                   else (f"replicas x{world}" if world > 1 else "single GPU"))
    line = {"metric": f"{dtype} GEMM TFLOP/s", "value": round(total, 1), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong" if panels else "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic uniform[-1,1], seeded",
            "config": {"workload": workload, "parallelism": parallelism,
                       "l2": "inputs resident; the working set exceeds L2 at 8192 and above"},
            "roofline": {"bound": "tensor", "kernel": "gemm_tc" if dtype != "f32" else "gemm_tc<tf32> x3 passes",
                         "achieved": round(per_gpu * passes, 1), "peak": round(peak, 1),
                         "peak_source": pk_kind if dtype != "f32" else f"{pk_kind} bf16 / 2 (TF32 rate)",
                         "unit": "TFLOP/s", "frac": round(per_gpu * passes / peak, 3), "traffic": None},
            # f32: two operand splits, the TF32 product, the split-K finish; bf16: the product
            "gpu_launches": (4 if dtype == "f32" else 1) * args.steps, "clocks": clocks}
    if matvec is not None:
        line["config"]["matvec"] = matvec
    return line


def run_c3(args, torch, world, rank, comm):
    """Config 3: f16 [8,16,128,64,32] permuted (0,3,1,4,2) and made
    contiguous; then sliced [:, 8:, :, :32, :], split in 4 along axis 1 and
    concatenated back (one assemble).  metric GB/s of the two copies."""
    from tensorcrate_b200 import cuda
    from tensorcrate_b200 import _native as N
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    shape = [8, 16, 128, 64, 32]
    n = int(np.prod(shape))
    x = cuda.CudaStorage.store(np.random.default_rng(3).standard_normal(n).astype(np.float16).view(np.uint16), "f16")
    t = cuda.Tensor(x, shape)
    perm = [0, 3, 1, 4, 2]
    pv = t.view().permute(perm)
    p_shape = pv.shape
    out_p = cuda.CudaStorage("f16", n)
    lib = N.lib()
    sl = cuda.TensorView(out_p, p_shape, cuda.contiguous_strides(p_shape)).slice(1, 8, p_shape[1]).slice(3, 0, 32)
    pieces = sl.chunk(1, 4)
    cat_shape = list(sl.shape)
    to = cuda.contiguous_strides(cat_shape)
    regions, at = [], 0
    for v in pieces:
        regions.append(cuda.Cuda._region((v.storage, v.shape, v.offset, v.strides, at * to[1], to)))
        at += v.shape[1]
    m = int(np.prod(cat_shape))
    out_c = cuda.CudaStorage("f16", m)
    arr = (N.Region * len(regions))(*regions)
    ps, pst = N.sizes(p_shape), N.sizes(pv.strides)

    def step():
        N.check("copy", lib.tc_strided_copy(2, 5, ps, x.ptr, n, 0, pst, out_p.ptr, C.c_void_p(sp)))
        N.check("assemble", lib.tc_assemble(2, out_c.ptr, m, arr, len(regions), C.c_void_p(sp)))

    ms, clocks = timed(torch, world, step, args.steps, args.warmup, stream)
    byts = 2 * n * 2 + 2 * m * 2
    gbs = byts / (ms * 1e-3) / 1e9
    pk, pk_kind = peaks()

    # Interpretation B: the slice's indices on the original axes,
    # x[:, 8:, :, :32, :] = [8, 8, 128, 32, 32], split in 4 along axis 1 and
    # concatenated back (one assemble of four regions).
    slb = t.view().slice(1, 8, shape[1]).slice(3, 0, 32)
    cat_b = list(slb.shape)
    to_b = cuda.contiguous_strides(cat_b)
    regions_b, at = [], 0
    for v in slb.chunk(1, 4):
        regions_b.append(cuda.Cuda._region((v.storage, v.shape, v.offset, v.strides, at * to_b[1], to_b)))
        at += v.shape[1]
    m_b = int(np.prod(cat_b))
    out_b = cuda.CudaStorage("f16", m_b)
    arr_b = (N.Region * len(regions_b))(*regions_b)

    def step_b():
        N.check("assemble", lib.tc_assemble(2, out_b.ptr, m_b, arr_b, len(regions_b), C.c_void_p(sp)))

    ms_b, _ = timed(torch, world, step_b, args.steps, args.warmup, stream)
    gbs_b = 2 * m_b * 2 / (ms_b * 1e-3) / 1e9
    return {"metric": "config-3 layout copy HBM throughput (GB/s)", "value": round(world * gbs, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1), seeded",
            "config": {"workload": "config3: permute(0,3,1,4,2)+contiguous, slice->split(4)->concat "
                                   "(interpretation A: slice of the permuted tensor)",
                       "algorithmic_bytes_per_step": byts,
                       "l2": "no flush: the permute moves 134 MB, more than the 126 MB L2",
                       "interpretation_b": {"workload": "x[:, 8:, :, :32, :] on the original axes -> [8,8,128,32,32], "
                                                        "split(4) along axis 1 -> concat",
                                            "ms": round(ms_b, 4), "gbs": round(gbs_b, 1),
                                            "frac": round(gbs_b / pk["hbm_gbs"], 3),
                                            "l2": "33.6 MB of traffic per step: L2-resident between steps"}},
            "roofline": {"bound": "hbm", "kernel": "strided copy + assemble", "achieved": round(gbs, 1),
                         "peak": pk["hbm_gbs"], "peak_source": pk_kind, "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 3), "traffic": None},
            "gpu_launches": 2 * args.steps, "clocks": clocks}


def run_trait(args, torch, world, rank, comm):
    """The Kernels<T> methods beyond the configs' hot path, each on an
    input larger than L2, timed alone: scan, sort, analytic
    unary and its dual, power, correlation, pad, flip, moments, a
    distribution function, and fused programs (plain, with row statistics,
    summed).  metric: algorithmic bytes of the HBM-bound calls / their time;
    "ops" gives each call against its own bound."""
    from tensorcrate_b200 import cuda
    from tensorcrate_b200 import _native as N
    lib = N.lib()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    pk, pk_kind = peaks()
    hbm = pk["hbm_gbs"]
    rng = np.random.default_rng(7)
    n = 64 << 20
    x = cuda.CudaStorage.store(rng.standard_normal(n, dtype=np.float32), "f32")
    y = cuda.CudaStorage.store(rng.uniform(0.5, 2.0, n).astype(np.float32), "f32")
    o1, o2 = cuda.CudaStorage("f32", n), cuda.CudaStorage("f32", n)
    ops, hbm_bytes, hbm_ms = {}, 0, 0.0

    def measure(name, fn, byts, flops=None, bound="hbm", peak=None, steps=None):
        nonlocal hbm_bytes, hbm_ms
        ms, _ = timed(torch, world, fn, steps or args.steps, args.warmup, stream)
        entry = {"ms": round(ms, 4), "bound": bound}
        if byts:
            gbs = byts / (ms * 1e-3) / 1e9
            entry.update(gbs=round(gbs, 1), bytes=byts)
            if bound == "hbm":
                entry["frac"] = round(gbs / hbm, 3)
                hbm_bytes += byts
                hbm_ms += ms
        if flops:
            tf = flops / (ms * 1e-3) / 1e12
            entry["tflops"] = round(tf, 2)
            if peak:
                entry["frac"] = round(tf / peak, 3)
        ops[name] = entry

    f32 = N.F32
    measure("prefix_sum", lambda: N.check("scan", lib.tc_prefix_sum(f32, x.ptr, o1.ptr, n, sp)), 2 * 4 * n)
    ns = 32 << 20
    measure("sort", lambda: N.check("sort", lib.tc_sort(f32, N.ASCENDING, x.ptr, o1.ptr, ns, sp)), 2 * 4 * ns)
    measure("unary_exp", lambda: N.check("unary", lib.tc_unary(f32, N.EXP, x.ptr, o1.ptr, n, sp)), 2 * 4 * n)
    measure("unary_dual_tanh",
            lambda: N.check("dual", lib.tc_unary_dual(f32, N.TANH, x.ptr, y.ptr, o1.ptr, o2.ptr, n, sp)), 4 * 4 * n)
    measure("power", lambda: N.check("pow", lib.tc_power(f32, y.ptr, x.ptr, o1.ptr, n, sp)), 3 * 4 * n)
    r = c = 8192
    w = cuda.CudaStorage.store(rng.uniform(-1, 1, 25).astype(np.float32), "f32")
    out_rc = (r - 4) * (c - 4)
    # FP32 pipe without FMA: one multiply and one add per tap, 128 lanes per SM
    fp32_peak = 148 * 128 * 1.965e9 / 1e12
    measure("correlate_5x5", lambda: N.check("corr", lib.tc_correlate(f32, r, c, 5, 5, 0, x.ptr, w.ptr, o1.ptr, sp)),
            4 * (r * c + out_rc), flops=2 * 25 * out_rc, bound="fp32 (mul + add per tap)", peak=fp32_peak)
    # the input gradient of that correlation: the 8188x8188 adjoint against
    # the 5x5 window back to 8192x8192 (each adjoint element meets each tap once)
    measure("correlate_input_gradient_5x5",
            lambda: N.check("cig", lib.tc_correlate_input_gradient(f32, r - 4, c - 4, 5, 5, 0, x.ptr, w.ptr, o1.ptr,
                                                                   sp)),
            4 * (out_rc + r * c), flops=2 * 25 * out_rc, bound="fp32 (mul + add per tap)", peak=fp32_peak)
    measure("pad_16", lambda: N.check("pad", lib.tc_pad(f32, r, c, 16, 16, x.ptr, o1.ptr, sp)),
            4 * (r * c + (r + 32) * (c + 32)))
    measure("flip", lambda: N.check("flip", lib.tc_flip(f32, r, c, x.ptr, o1.ptr, sp)), 2 * 4 * r * c)
    scalar = cuda.CudaStorage("f32", 1)
    measure("sgd", lambda: N.check("sgd", lib.tc_sgd(f32, n, o1.ptr, y.ptr, 1e-3, sp)), 3 * 4 * n)
    measure("dot", lambda: N.check("dot", lib.tc_dot(f32, x.ptr, y.ptr, n, scalar.ptr, sp)), 2 * 4 * n)
    measure("vector_sum", lambda: N.check("sum", lib.tc_vector_reduce(f32, N.SUM, x.ptr, n, scalar.ptr, sp)), 4 * n)
    mom = cuda.CudaStorage("f32", 2)
    measure("moments", lambda: N.check("moments", lib.tc_moments(f32, x.ptr, n, mom.ptr, sp)), 4 * n)
    rows, cols = 16384, 4096
    means, devs = cuda.CudaStorage("f32", rows), cuda.CudaStorage("f32", rows)
    measure("axis_moments_rows",
            lambda: N.check("axis", lib.tc_axis_moments(f32, rows, cols, N.ROWS, x.ptr, means.ptr, devs.ptr, sp)),
            4 * rows * cols)
    nd = 16 << 20
    measure("normal_cdf", lambda: N.check("dist", lib.tc_distribution(f32, N.NORMAL, N.CDF, x.ptr, nd, 0.0, 1.0,
                                                                      o1.ptr, sp)),
            2 * 4 * nd, bound="fp64 (Cody erfc per element)")

    def ins(code, dst=0, a=0, b=0, op=0, slot=0, value=0.0):
        i = N.Instr()
        i.code, i.dst, i.a, i.b, i.op, i.slot, i.value = code, dst, a, b, op, slot, value
        return i

    def place(ptr):
        p = N.Place()
        p.data, p.dtype, p.lead, p.offset, p.col_step = ptr, f32, 1, 0, 1
        p.dims[0], p.steps[0] = rows, cols
        return p

    prog = [ins(N.I_LOAD, 0, slot=0), ins(N.I_LOAD, 1, slot=1), ins(N.I_BINARY, 2, 0, 1, op=2),
            ins(N.I_CONST, 3, value=1.0), ins(N.I_BINARY, 4, 2, 3, op=0), ins(N.I_STORE, a=4, slot=0)]
    code = (N.Instr * len(prog))(*prog)
    pl2 = (N.Place * 2)(place(x.ptr), place(y.ptr))
    outs = (C.c_void_p * 1)(o1.ptr)
    dts = (C.c_int * 1)(f32)
    measure("fused_xy_plus_1", lambda: N.check("fused", lib.tc_fused(f32, rows, cols, code, len(prog), pl2, 2, outs,
                                                                      dts, 1, sp)), 3 * 4 * rows * cols)
    sums = cuda.CudaStorage("f32", rows)
    measure("fused_sum_rows", lambda: N.check("fsum", lib.tc_fused_sum(f32, rows, cols, code, len(prog), pl2, 2,
                                                                        N.ROWS, sums.ptr, sp)), 2 * 4 * rows * cols)
    ln = [ins(N.I_LOAD, 0, slot=0), ins(N.I_LOAD, 1, slot=1), ins(N.I_LOAD, 2, slot=2), ins(N.I_CONST, 3, value=1.0 / cols),
          ins(N.I_BINARY, 4, 2, 3, op=2), ins(N.I_UNARY, 5, 4, op=N.SQRT), ins(N.I_BINARY, 6, 0, 1, op=1),
          ins(N.I_BINARY, 7, 6, 5, op=3), ins(N.I_STORE, a=7, slot=0)]
    ln_code = (N.Instr * len(ln))(*ln)
    pl3 = (N.Place * 3)(place(x.ptr), N.Place(), N.Place())
    st = (N.RowStatistic * 2)(N.RowStatistic(0, 1, N.ROW_MEAN), N.RowStatistic(0, 2, N.ROW_DEVIATIONS))
    measure("layer_norm_with_statistics",
            lambda: N.check("stats", lib.tc_fused_with_statistics(f32, rows, cols, ln_code, len(ln), pl3, 3, st, 2,
                                                                  outs, dts, 1, sp)), 2 * 4 * rows * cols)
    gbs = hbm_bytes / (hbm_ms * 1e-3) / 1e9
    return {"metric": "trait-method kernels HBM throughput (GB/s)", "value": round(gbs, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(hbm_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1) / uniform, seeded",
            "config": {"workload": "each trait-method kernel alone: 64M-element vectors (sort: 32M, distribution: 16M), "
                                   "8192x8192 matrices, 16384x4096 programs",
                       "l2": "no flush: every input is 256 MB or more, above the 126 MB L2 (sort: 128 MB)",
                       "value": "algorithmic bytes of the HBM-bound calls / the sum of their times"},
            "roofline": {"bound": "hbm", "kernel": "all HBM-bound trait-method calls", "achieved": round(gbs, 1), "peak": hbm,
                         "peak_source": pk_kind, "unit": "GB/s", "frac": round(gbs / hbm, 3), "traffic": None},
            # our kernels per call (sort: the key maps; CUB's radix passes are not counted)
            "ops": ops, "gpu_launches": args.steps * sum(LAUNCHES_PER_CALL.get(k, 1) for k in ops)}


LAUNCHES_PER_CALL = {"prefix_sum": 3, "sort": 2, "moments": 4, "axis_moments_rows": 1, "dot": 2, "vector_sum": 2}


def run_c4(args, torch, world, rank, comm):
    """Config 4: one training step of the 1024-4096-4096-1024 ReLU MLP in
    bf16 (tape + Adam(1e-3, 0.9, 0.999, 1e-8), as the reference runs it),
    global batch 2048 split across the ranks (strong scaling), gradients
    summed with NCCL.  metric: steps/s."""
    from tensorcrate_b200 import _native as N
    from tensorcrate_b200 import cuda
    from tensorcrate_b200.mlp import Mlp, xavier
    dtype = "bf16"
    dims = [1024, 4096, 4096, 1024]
    gbatch = args.batch
    if gbatch % world:
        raise SystemExit("global batch must divide by the number of GPUs")
    batch = gbatch // world
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(6)
    ws = [xavier(dims[l + 1], dims[l], rng) for l in range(3)]
    bs = [np.zeros(dims[l + 1], np.float32) for l in range(3)]
    m = Mlp(dtype, dims, batch, gbatch)
    m.load(ws, bs)
    xr = np.random.default_rng(4 + rank).standard_normal((dims[0], batch)).astype(np.float32)
    yr = np.random.default_rng(5 + rank).standard_normal((dims[-1], batch)).astype(np.float32)
    x = cuda.CudaStorage.store(cuda.f32_to_bits(xr, dtype), dtype)
    y = cuda.CudaStorage.store(cuda.f32_to_bits(yr, dtype), dtype)
    loss = cuda.CudaStorage(dtype, 1)

    def step():
        m.step(x, y, comm=comm, stream=stream)

    ms, clocks = timed(torch, world, step, args.steps, args.warmup, stream)
    gemm_flops = 3 * 2 * gbatch * sum(dims[l] * dims[l + 1] for l in range(3))  # fwd + dW + dX
    pk, pk_kind = peaks()
    tflops = gemm_flops / (ms * 1e-3) / 1e12
    # e2e: inputs and targets uploaded from pinned host memory each step, the
    # loss read back.
    px = torch.from_numpy(cuda.f32_to_bits(xr, dtype).view(np.int16)).pin_memory()
    py = torch.from_numpy(cuda.f32_to_bits(yr, dtype).view(np.int16)).pin_memory()
    pl = torch.empty(1, dtype=torch.int16).pin_memory()
    lib = N.lib()
    sp = C.c_void_p(stream.cuda_stream)

    def e2e_step():
        N.check("h2d", lib.tc_memcpy_h2d(x.ptr, px.data_ptr(), px.numel() * 2, sp))
        N.check("h2d", lib.tc_memcpy_h2d(y.ptr, py.data_ptr(), py.numel() * 2, sp))
        m.step(x, y, comm=comm, loss=loss, stream=stream)
        N.check("d2h", lib.tc_memcpy_d2h(pl.data_ptr(), loss.ptr, 2, sp))

    serial_ms, _ = timed(torch, world, e2e_step, max(3, args.steps // 2), 2, stream)

    # As a streaming caller runs it: two device copies of the inputs and
    # targets, step k+1's uploads on a copy stream while step k trains (each
    # upload waits for the step that last read its buffers; each step waits
    # for its own uploads).  Every step still uploads its batch and reads its
    # loss back inside the timed region.
    x2, y2 = cuda.CudaStorage(dtype, x.len), cuda.CudaStorage(dtype, y.len)
    bufs = [(x, y), (x2, y2)]
    copy_stream = torch.cuda.Stream()
    csp = C.c_void_p(copy_stream.cuda_stream)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]

    def upload(k):
        b = k % 2
        if k >= 2:
            copy_stream.wait_event(consumed[b])
        N.check("h2d", lib.tc_memcpy_h2d(bufs[b][0].ptr, px.data_ptr(), px.numel() * 2, csp))
        N.check("h2d", lib.tc_memcpy_h2d(bufs[b][1].ptr, py.data_ptr(), py.numel() * 2, csp))
        copied[b].record(copy_stream)

    def pipelined(steps):
        copy_stream.wait_stream(stream)
        upload(0)
        for k in range(steps):
            if k + 1 < steps:
                upload(k + 1)
            stream.wait_event(copied[k % 2])
            m.step(bufs[k % 2][0], bufs[k % 2][1], comm=comm, loss=loss, stream=stream)
            consumed[k % 2].record(stream)
            N.check("d2h", lib.tc_memcpy_d2h(pl.data_ptr(), loss.ptr, 2, sp))

    e2e_steps = max(3, args.steps // 2)
    pipelined(2)
    torch.cuda.synchronize()
    barrier(torch, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipelined(e2e_steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, world, e0.elapsed_time(e1) / e2e_steps)
    return {"metric": "config-4 MLP training steps/s", "value": round(1000.0 / ms, 2), "unit": "steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic N(0,1) inputs/targets, Xavier-uniform weights, seeded",
            "config": {"workload": "config4: MLP 1024-4096-4096-1024 ReLU, MSE, Adam(1e-3,0.9,0.999,1e-8), bf16",
                       "global_batch": gbatch, "per_rank_batch": batch,
                       "parallelism": f"dp{world}" + (" (NCCL all-reduce of gradients)" if world > 1 else ""),
                       "gemm_flops_per_step": gemm_flops},
            "roofline": {"bound": "tensor", "kernel": "whole step (GEMM share)", "achieved": round(tflops, 1),
                         "peak": pk["bf16_tflops_sustained"], "peak_source": pk_kind + " sustained",
                         "unit": "TFLOP/s", "frac": round(tflops / pk["bf16_tflops_sustained"], 3), "traffic": None},
            "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "steps/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": (px.numel() + py.numel()) * 2, "d2h_bytes_per_step": 2,
                    "pipelined": "each step's uploads overlap the previous step (two device buffers, a copy stream)",
                    "serial_ms_per_step": round(serial_ms, 4)},
            # per step: 3 forward products + 1 split-K finish, the loss pass, per layer the bias
            # adjoints (matvec, vecmat + finish, an add below the top) and 2 products (+1 finish
            # for the split input-gradient product of layer 1), Adam: 24 (ncu launch list)
            "gpu_launches": 24 * args.steps, "clocks": clocks}


def barrier(torch, world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(torch, world, v: float) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def init_comm(torch, world, rank):
    """NCCL communicator of the library, bootstrapped over torch.distributed."""
    from tensorcrate_b200.sharding import nccl_comm
    return nccl_comm(torch, world, rank)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5", "trait"])
    ap.add_argument("--batch", type=int, default=2048, help="config 4's global batch")
    ap.add_argument("--size", type=int, default=8192, help="config 5's M=N=K")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_env()

    if args.impl == "reference":
        if rank != 0:
            return
        base = cpu_c2(sample_rows=64, reps=max(3, min(16, args.steps)))
        line = {"metric": "config-2 broadcast + axis-reduction HBM throughput (GB/s)", "value": base["value"],
                "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic N(0,1), seeded", "impl": "reference",
                "config": {"workload": "config2 (reference Host path restated in C++, oracle/)"},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    from tensorcrate_b200 import _native as N
    N.call("tc_set_device", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    comm = init_comm(torch, world, rank)
    if args.workload == "c5":
        line = run_gemm(args, torch, world, rank, comm, "bf16", args.size)
    elif args.workload == "c1":
        line = run_gemm(args, torch, world, rank, comm, "f32", 1024)
    elif args.workload == "c3":
        line = run_c3(args, torch, world, rank, comm)
    elif args.workload == "c4":
        line = run_c4(args, torch, world, rank, comm)
    elif args.workload == "trait":
        line = run_trait(args, torch, world, rank, comm)
    else:
        line = run_c2(args, torch, world, rank, comm)
    if rank == 0 and not args.no_cpu_baseline and args.workload == "c2":
        line["cpu_baseline"] = cpu_c2(sample_rows=64, reps=12)
    if comm is not None:
        N.call("tc_comm_destroy", comm)
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
