"""Benchmark of the tensorcrate CUDA backend's hot path on B200.

One JSON line.  Its headline (`value`) is config 2, the configuration the
reference's broadcast + axis-reduction path is quoted on: one step is the
nine calls that config names, on f32 x[64,512,1024] ~ N(0,1) and
bias[1,1,1024] ~ N(0,1):
    x + bias, x * bias, x > bias          (Kernels::strided_binary)
    sum, mean, var over axis 2           (Kernels::reduce_axes)
    max, min over axes (0, 2)            (Kernels::reduce_axes)
    argmax over axis 1                   (Kernels::arg_reduce)
metric: HBM GB/s = algorithmic bytes of the nine calls / step time.

The same line carries the other configurations as sub-records, each with
its own timing, clocks, roofline, end-to-end figure and parity check:
  c4  the MLP training step (1024-4096-4096-1024, bf16, Adam), steps/s;
  c4_weak  the same step with 2048 samples per GPU, samples/s;
  c5  the bf16 GEMM, M=N=K=8192, TFLOP/s (c5_16384, c5_4096: the config's
      other sizes);
  c1  the f32 GEMM 1024^3 and matvec;
  c3  the f16 layout copies (permute, slice-split-concatenate).

Under torchrun (one process per GPU, NCCL):
  c2  each rank owns its own [64,512,1024] slab of a [64*P,512,1024] tensor
      (weak scaling); the per-slab results are all-gathered and the [512]
      max/min partials folded over ranks;
  c4  data parallel over the global batch of 2048 (strong scaling), the
      optimizer sharded over the ranks: per layer one kernel sums this
      rank's shard of the gradients over the ranks (NVLink peer loads), runs
      Adam on it and stores it into every rank's parameters (peer stores);
  c4_weak  the same with 2048 samples per GPU (weak scaling);
  c5  row panels: rank r computes rows [r*M/P, (r+1)*M/P) of C and the GEMM
      epilogue stores every tile into every rank's C over NVLink (strong);
  c1, c3  replicas (each rank its own copy of the work).

Timing: W warm-up steps, then blocks of K timed steps (CUDA events on the
launching stream, max over ranks) repeated until at least --min-seconds of
device time has passed; ms_per_step is the median block's, with the spread.
Every sub-record checks its results against the oracle (the reference's
Host path restated in C++) outside the timed region and reports "parity".

--workload c1|c2|c3|c4|c5|trait runs one workload alone as the headline.
--impl reference times the reference's Host path restated in C++ (oracle/)
on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
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
ORACLE_FLAGS = "g++ -O3 -ffp-contract=off -fno-fast-math (oracle/Makefile), AVX2/FMA dispatched at run time"


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


def barrier(torch, world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(torch, world, v):
    """Max over ranks of a float or a list of floats."""
    if world == 1:
        return v
    t = torch.tensor(v if isinstance(v, list) else [v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    out = [float(a) for a in t.cpu().tolist()]
    return out if isinstance(v, list) else out[0]


def sum_over_ranks(torch, world, v: int) -> int:
    if world == 1:
        return int(v)
    t = torch.tensor([int(v)], dtype=torch.int64, device="cuda")
    torch.distributed.all_reduce(t)
    return int(t.item())


def init_comm(torch, world, rank):
    """NCCL communicator of the library, bootstrapped over torch.distributed."""
    from tensorcrate_b200.sharding import nccl_comm
    return nccl_comm(torch, world, rank)


def timed(torch, world, fn, args, stream):
    """W warm-up calls of fn, then blocks of K timed calls (CUDA events on
    `stream`) until at least args.min_seconds of device time has passed
    (at least 3 blocks), bracketed by a barrier and a synchronize.  Each
    block's time is the max over ranks.  Returns (ms per step of the median
    block, {blocks, spread, seconds}, clocks summary)."""
    steps = args.steps
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    blocks = []
    n_blocks = None
    with Clocks(torch.cuda.current_device()) as clocks:
        barrier(torch, world)
        torch.cuda.synchronize()
        while n_blocks is None or len(blocks) < n_blocks:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            e1.synchronize()
            blocks.append(e0.elapsed_time(e1))
            if n_blocks is None:
                first = max_over_ranks(torch, world, blocks[0])
                n_blocks = max(3, math.ceil(args.min_seconds * 1e3 / max(first, 1e-3)))
        torch.cuda.synchronize()
        barrier(torch, world)
    blocks = max_over_ranks(torch, world, blocks)
    per_step = sorted(b / steps for b in blocks)
    med = statistics.median(per_step)
    info = {"blocks": len(blocks), "steps_per_block": steps, "seconds": round(sum(blocks) / 1e3, 3),
            "ms_per_step_min": round(per_step[0], 5), "ms_per_step_max": round(per_step[-1], 5),
            "spread": round((per_step[-1] - per_step[0]) / med, 4)}
    return med, info, clocks.summary()


def pinned(torch, nbytes: int):
    return torch.empty(max(1, nbytes), dtype=torch.uint8).pin_memory()


class Pipeline:
    """End-to-end steps as a streaming caller runs them through the C ABI
    with host buffers: every step uploads its inputs from pinned host memory,
    runs, and reads its results back into pinned host memory.  Two device
    sets of inputs and results: step k+1's uploads (copy stream) and step
    k-1's read-backs (a second copy stream) overlap step k's kernels.  Each
    upload waits for the kernels that last read its buffers; each step waits
    for its uploads and for the read-back of the results it overwrites."""

    def __init__(self, torch, lib, stream, uploads, readbacks, run):
        # uploads: [(host pinned tensor, [dev ptr set 0, set 1], nbytes)]
        # readbacks: [([dev ptr set 0, set 1], host pinned tensor, nbytes)]
        # run(b, stream pointer): enqueue the step on input/result set b
        self.torch, self.lib, self.stream = torch, lib, stream
        self.uploads, self.readbacks, self.run = uploads, readbacks, run
        self.up, self.down = torch.cuda.Stream(), torch.cuda.Stream()
        self.copied = [torch.cuda.Event(), torch.cuda.Event()]
        self.computed = [torch.cuda.Event(), torch.cuda.Event()]
        self.drained = [torch.cuda.Event(), torch.cuda.Event()]
        self.h2d = sum(n for _, _, n in uploads)
        self.d2h = sum(n for _, _, n in readbacks)

    def _upload(self, k):
        from tensorcrate_b200 import _native as N
        b = k % 2
        if k >= 2:
            self.up.wait_event(self.computed[b])
        usp = C.c_void_p(self.up.cuda_stream)
        for host, dev, n in self.uploads:
            N.check("h2d", self.lib.tc_memcpy_h2d(dev[b], host.data_ptr(), n, usp))
        self.copied[b].record(self.up)

    def steps(self, count):
        from tensorcrate_b200 import _native as N
        sp = C.c_void_p(self.stream.cuda_stream)
        dsp = C.c_void_p(self.down.cuda_stream)
        self.up.wait_stream(self.stream)
        self.down.wait_stream(self.stream)
        self._upload(0)
        for k in range(count):
            b = k % 2
            if k + 1 < count:
                self._upload(k + 1)
            self.stream.wait_event(self.copied[b])
            if k >= 2:
                self.stream.wait_event(self.drained[b])
            self.run(b, sp)
            self.computed[b].record(self.stream)
            self.down.wait_event(self.computed[b])
            for dev, host, n in self.readbacks:
                N.check("d2h", self.lib.tc_memcpy_d2h(host.data_ptr(), dev[b], n, dsp))
            self.drained[b].record(self.down)
        self.stream.wait_stream(self.down)
        self.stream.wait_stream(self.up)

    def measure(self, world, steps):
        """ms per end-to-end step, pipelined (max over ranks)."""
        torch = self.torch
        self.steps(2)
        torch.cuda.synchronize()
        barrier(torch, world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        self.steps(steps)
        e1.record(self.stream)
        torch.cuda.synchronize()
        return max_over_ranks(torch, world, e0.elapsed_time(e1) / steps)

    def measure_serial(self, world, steps):
        """ms per end-to-end step with uploads, kernels and read-backs in
        turn on one stream (input/result set 0)."""
        from tensorcrate_b200 import _native as N
        torch = self.torch
        sp = C.c_void_p(self.stream.cuda_stream)

        def one():
            for host, dev, n in self.uploads:
                N.check("h2d", self.lib.tc_memcpy_h2d(dev[0], host.data_ptr(), n, sp))
            self.run(0, sp)
            for dev, host, n in self.readbacks:
                N.check("d2h", self.lib.tc_memcpy_d2h(host.data_ptr(), dev[0], n, sp))
        one()
        torch.cuda.synchronize()
        barrier(torch, world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            one()
        e1.record(self.stream)
        torch.cuda.synchronize()
        return max_over_ranks(torch, world, e0.elapsed_time(e1) / steps)


def parity_record(torch, world, failures: list[str], checked: str) -> dict | str:
    """'ok', or the number of failures over all ranks and this rank's first."""
    total = sum_over_ranks(torch, world, len(failures))
    if total == 0:
        return {"status": "ok", "checked": checked}
    return {"status": "failed", "failures": total, "first_on_this_rank": failures[:1], "checked": checked}


# ---------------------------------------------------------------------------
# config 2
# ---------------------------------------------------------------------------
SHAPE2 = [64, 512, 1024]


def c2_ops_bytes():
    n = int(np.prod(SHAPE2)) * 4
    rows = SHAPE2[0] * SHAPE2[1]
    return {
        "add": 2 * n + 4096, "mul": 2 * n + 4096, "greater": 2 * n + 4096,
        "sum": n + rows * 4, "mean": n + rows * 4, "var": n + rows * 4,
        "max": n + 512 * 4, "min": n + 512 * 4,
        "argmax": n + SHAPE2[0] * SHAPE2[2] * 4,
    }


def c2_slab(rank: int) -> np.ndarray:
    """Rank `rank`'s [64,512,1024] slab of the global config-2 tensor."""
    return np.random.default_rng(1 + rank).standard_normal(int(np.prod(SHAPE2)), dtype=np.float32)


C2_BIAS_SEED = 2
C2_FIELDS = [("sum", "f32", SHAPE2[0] * SHAPE2[1]), ("mean", "f32", SHAPE2[0] * SHAPE2[1]),
             ("var", "f32", SHAPE2[0] * SHAPE2[1]), ("argmax", "u32", SHAPE2[0] * SHAPE2[2]),
             ("max", "f32", 512), ("min", "f32", 512)]


def run_c2(args, torch, world, rank, comm):
    from tensorcrate_b200 import _native as N
    from tensorcrate_b200 import cuda

    lib = N.lib()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    shape = SHAPE2
    n = int(np.prod(shape))
    x_host = c2_slab(rank)
    bias_host = np.random.default_rng(C2_BIAS_SEED).standard_normal(1024, dtype=np.float32)
    xs_dev = [cuda.CudaStorage.store(x_host, "f32"), cuda.CudaStorage("f32", n)]
    biases = [cuda.CudaStorage.store(bias_host, "f32"), cuda.CudaStorage.store(bias_host, "f32")]
    pack_len = sum(c for _, _, c in C2_FIELDS)
    at, offset = {}, 0
    for k, _, count in C2_FIELDS:
        at[k] = offset
        offset += count

    def result_set():
        # The reductions' results sit side by side in one block of 4-byte
        # elements, so that one all-gather carries all of them when P > 1.
        outs = {k: cuda.CudaStorage("f32", n) for k in ("add", "mul", "greater")}
        pack = cuda.CudaStorage("u32", pack_len)
        for k, dt, count in C2_FIELDS:
            outs[k] = cuda.CudaStorage(dt, count, ptr=pack.ptr + 4 * at[k])
        outs["pack"] = pack
        if world > 1:
            outs["gathered"] = cuda.CudaStorage("u32", pack_len * world)
            outs["final_max"] = cuda.CudaStorage("f32", 512)
            outs["final_min"] = cuda.CudaStorage("f32", 512)
        return outs

    sets = [result_set(), result_set()]
    sz = N.sizes
    xs, xst = sz(shape), sz(cuda.contiguous_strides(shape))
    bst = sz([0, 0, 1])
    ax2, ax02 = N.u32s([2]), N.u32s([0, 2])
    g_shape, g_strides = sz([world, 512]), sz([pack_len, 1])

    def calls_on(b, sp):
        """The nine calls of a step on input set b into result set b."""
        x, o, bias = xs_dev[b], sets[b], biases[b]
        argp = C.cast(C.c_void_p(o["argmax"].ptr), C.POINTER(C.c_uint32))
        return [
            ("add", lib.tc_strided_binary, (0, N.PAIR_ARITHMETIC, N.ADD, 3, xs, x.ptr, n, 0, xst, bias.ptr, 1024, 0,
                                            bst, o["add"].ptr, sp)),
            ("mul", lib.tc_strided_binary, (0, N.PAIR_ARITHMETIC, N.MUL, 3, xs, x.ptr, n, 0, xst, bias.ptr, 1024, 0,
                                            bst, o["mul"].ptr, sp)),
            ("greater", lib.tc_strided_binary, (0, N.PAIR_COMPARE, N.GREATER, 3, xs, x.ptr, n, 0, xst, bias.ptr, 1024,
                                                0, bst, o["greater"].ptr, sp)),
            ("sum", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 1, ax2, N.AXIS_FOLD, N.SUM, 0, o["sum"].ptr, sp)),
            ("mean", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 1, ax2, N.AXIS_MEAN, 0, 0, o["mean"].ptr, sp)),
            ("var", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 1, ax2, N.AXIS_VARIANCE, 0, 1024, o["var"].ptr,
                                         sp)),
            ("max", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 2, ax02, N.AXIS_FOLD, N.RMAX, 0, o["max"].ptr,
                                         sp)),
            ("min", lib.tc_reduce_axes, (0, 3, xs, x.ptr, n, 0, xst, 2, ax02, N.AXIS_FOLD, N.RMIN, 0, o["min"].ptr,
                                         sp)),
            ("argmax", lib.tc_arg_reduce, (0, 3, xs, x.ptr, n, 0, xst, 1, N.RMAX, argp, sp)),
        ]

    # P > 1: one all-gather of every rank's block of results (the slab
    # results are then final, rank after rank); the [512] extremes fold the
    # sharded leading axis, so each is finished by reducing the P gathered
    # partials ([P, 512] with a stride of one block), exactly.  The
    # reductions run first; the gather and the folds then run on a second
    # stream beside the three broadcasts, and the step ends when both have.
    side = torch.cuda.Stream() if world > 1 else None
    side_sp = C.c_void_p(side.cuda_stream) if side is not None else None
    packed = torch.cuda.Event() if world > 1 else None
    gathered = torch.cuda.Event() if world > 1 else None

    def collectives(o, on_stream):
        packed.record(on_stream)
        side.wait_event(packed)
        N.check("allgather", lib.tc_allgather(comm, N.U32, o["pack"].ptr, o["gathered"].ptr, pack_len, side_sp))
        for k, op in (("max", N.RMAX), ("min", N.RMIN)):
            N.check("fold", lib.tc_reduce_axes(0, 2, g_shape, o["gathered"].ptr, pack_len * world, at[k], g_strides,
                                               1, N.u32s([0]), N.AXIS_FOLD, op, 0, o["final_" + k].ptr, side_sp))
        gathered.record(side)

    calls = [calls_on(0, sp), calls_on(1, sp)]
    events = {name: [] for name, _, _ in calls[0]}
    REDUCTIONS = ("sum", "mean", "var", "max", "min", "argmax")

    def step(b=0, record=False, on_sp=None):
        todo = calls[b] if on_sp is None else calls_on(b, on_sp)
        on_stream = stream  # the pipeline passes this same stream's pointer
        order = [c for c in todo if c[0] in REDUCTIONS] + [c for c in todo if c[0] not in REDUCTIONS]
        for i, (name, fn, a) in enumerate(order):
            if world > 1 and i == len(REDUCTIONS):
                collectives(sets[b], on_stream)
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
        if world > 1:
            on_stream.wait_event(gathered)

    bytes_per_op = c2_ops_bytes()
    step_bytes = sum(bytes_per_op.values())
    ms_per_step, blocks, clocks = timed(torch, world, step, args, stream)
    # Per-operation times, from events around each call, in a pass of their
    # own (events between the calls would sit inside the timed region).
    for _ in range(min(args.steps, 50)):
        step(record=True)
    torch.cuda.synchronize()
    per_op_ms = {k: statistics.mean(a.elapsed_time(b) for a, b in v) for k, v in events.items()}

    # ---- parity against the oracle, outside the timed region ----
    failures = parity_c2(torch, world, rank, x_host, bias_host, sets[0], at, pack_len, failures=[])
    parity = parity_record(torch, world, failures,
                           "sampled rows of add/mul/greater (bit-exact), sum/mean/var (rel 1e-5*sqrt(K)) and argmax "
                           "(bit-exact) of this rank's slab and of the next rank's slab as gathered here; max/min over "
                           "(0,2) of the whole tensor (bit-exact), against oracle/ on the same seeded input")

    # ---- end to end: host buffers through the C ABI, every result read back ----
    h_x, h_b = pinned(torch, n * 4), pinned(torch, 4096)
    h_x.numpy().view(np.float32)[:] = x_host
    h_b.numpy().view(np.float32)[:] = bias_host
    read_keys = [("add", n * 4), ("mul", n * 4), ("greater", n * 4), ("pack", pack_len * 4)]
    hosts = {k: pinned(torch, nb) for k, nb in read_keys}
    pipe = Pipeline(torch, lib, stream,
                    uploads=[(h_x, [xs_dev[0].ptr, xs_dev[1].ptr], n * 4),
                             (h_b, [biases[0].ptr, biases[1].ptr], 4096)],
                    readbacks=[([sets[0][k].ptr, sets[1][k].ptr], hosts[k], nb) for k, nb in read_keys],
                    run=lambda b, s: step(b, on_sp=s))
    e2e_steps = max(5, args.steps // 2)
    e2e_ms = pipe.measure(world, e2e_steps)
    serial_ms = pipe.measure_serial(world, max(3, e2e_steps // 2))

    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9
    # Dominant kernel: the largest share of the step.
    dom = max(per_op_ms, key=lambda k: per_op_ms[k])
    pk, pk_kind = peaks()
    achieved = bytes_per_op[dom] / (per_op_ms[dom] * 1e-3) / 1e9
    ops = {k: {"ms": round(v, 5), "gbs": round(bytes_per_op[k] / (v * 1e-3) / 1e9, 1),
               "frac": round(bytes_per_op[k] / (v * 1e-3) / 1e9 / pk["hbm_gbs"], 3)} for k, v in per_op_ms.items()}
    launches = len(calls[0]) + (2 if world > 1 else 0)
    return {
        "metric": "config-2 broadcast + axis-reduction HBM throughput (GB/s)",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "config2: f32 x[64,512,1024] with bias[1,1,1024]: add, mul, greater; sum/mean/var ax2; "
                               "max/min ax(0,2); argmax ax1",
                   "per_rank_shape": SHAPE2, "global_shape": [64 * world, 512, 1024],
                   "parallelism": f"leading-axis shards x{world}" + (" (one NCCL all-gather of every result, then "
                                                                     "max/min folded over ranks)" if world > 1 else ""),
                   "l2": "no flush: every call reads the 134.2 MB input, larger than the 126 MB L2",
                   "algorithmic_bytes_per_step": step_bytes},
        "timing": blocks,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                     "peak_source": pk_kind, "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 3),
                     "traffic": traffic("c2", dom), "algorithmic_bytes": bytes_per_op[dom]},
        "ops": ops,
        "e2e": {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": pipe.h2d, "d2h_bytes_per_step": pipe.d2h,
                "reads_back": "all nine results: the three [64,512,1024] broadcast outputs and the six reductions' "
                              "block, every step",
                "pipelined": "step k+1's upload and step k-1's read-back overlap step k's kernels (two device sets "
                             "of inputs and results, one copy stream each way)",
                "serial_ms_per_step": round(serial_ms, 4)},
        "parity": parity,
        "gpu_launches_per_step": launches,
        "gpu_launches": launches * args.steps * blocks["blocks"],
        "clocks": clocks,
    }


def parity_c2(torch, world, rank, x_host, bias_host, o, at, pack_len, failures):
    """Config 2's results against the oracle on sampled leading rows of this
    rank's slab and, when sharded, of the next rank's slab as the all-gather
    delivered it here; the max/min over (0,2) of the whole global tensor."""
    import oracle as O
    from tensorcrate_b200 import _native as N
    lib = N.lib()
    torch.cuda.synchronize()
    rows = [0, 37, 63]
    st = [512 * 1024, 1024, 1]
    sub_shape = [len(rows), 512, 1024]
    slab = x_host.reshape(SHAPE2)

    def tol_ok(got, want, k):
        return bool(np.all(np.abs(got - want) <= 1e-5 * np.sqrt(k) * (np.abs(want) + 1.0)))

    def check_reductions(sub, pack, who):
        want = {"sum": O.reduce_axes("f32", sub_shape, sub, 0, st, [2], N.AXIS_FOLD, N.SUM, 0),
                "mean": O.reduce_axes("f32", sub_shape, sub, 0, st, [2], N.AXIS_MEAN, 0, 0),
                "var": O.reduce_axes("f32", sub_shape, sub, 0, st, [2], N.AXIS_VARIANCE, 0, 1024)}
        for k, w in want.items():
            got = np.concatenate([pack[at[k] + r * 512: at[k] + (r + 1) * 512].view(np.float32) for r in rows])
            if not tol_ok(got, w, 1024):
                failures.append(f"{who}: {k} differs from the oracle")
        arg = O.arg_reduce("f32", sub_shape, sub, 0, st, 1, N.RMAX)
        got = np.concatenate([pack[at["argmax"] + r * 1024: at["argmax"] + (r + 1) * 1024] for r in rows])
        if not np.array_equal(got, arg):
            failures.append(f"{who}: argmax differs from the oracle")

    sub = np.ascontiguousarray(slab[rows]).reshape(-1)
    pack = o["pack"].as_slice()
    check_reductions(sub, pack, f"rank {rank}")
    for k, kind, op in (("add", 0, N.ADD), ("mul", 0, N.MUL), ("greater", 1, N.GREATER)):
        want = O.strided_binary("f32", kind, op, sub_shape, sub, 0, st, bias_host, 0, [0, 0, 1])
        got = np.empty(len(rows) * 512 * 1024, np.float32)
        for i, r in enumerate(rows):
            N.check("d2h", lib.tc_memcpy_d2h(got[i * 512 * 1024:].ctypes.data, o[k].ptr + r * 512 * 1024 * 4,
                                             512 * 1024 * 4, None))
        if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
            failures.append(f"rank {rank}: {k} differs from the oracle")
    # max/min over (0, 2): this slab's partial by the oracle, folded over
    # every rank's partial (exact), against the result every rank holds.
    part = {k: O.reduce_axes("f32", SHAPE2, x_host, 0, st, [0, 2], N.AXIS_FOLD, op, 0)
            for k, op in (("max", N.RMAX), ("min", N.RMIN))}
    if world > 1:
        gathered = o["gathered"].as_slice()
        nxt = (rank + 1) % world
        nsub = np.ascontiguousarray(c2_slab(nxt).reshape(SHAPE2)[rows]).reshape(-1)
        check_reductions(nsub, gathered[nxt * pack_len:(nxt + 1) * pack_len], f"rank {nxt}'s slab on rank {rank}")
        for k in ("max", "min"):
            t = torch.tensor(part[k], device="cuda")
            every = [torch.empty_like(t) for _ in range(world)]
            torch.distributed.all_gather(every, t)
            stacked = np.stack([e.cpu().numpy() for e in every])
            want = stacked.max(axis=0) if k == "max" else stacked.min(axis=0)
            if not np.array_equal(o["final_" + k].as_slice(), want):
                failures.append(f"rank {rank}: global {k} differs from the oracle")
    else:
        for k in ("max", "min"):
            if not np.array_equal(pack[at[k]:at[k] + 512].view(np.float32), part[k]):
                failures.append(f"rank {rank}: {k} differs from the oracle")
    return failures


def cpu_c2(sample_rows: int = 16, reps: int = 1):
    import oracle as O

    shape = [sample_rows, 512, 1024]
    n = int(np.prod(shape))
    x = np.random.default_rng(1).standard_normal(n, dtype=np.float32)
    bias = np.random.default_rng(2).standard_normal(1024, dtype=np.float32)
    st = [512 * 1024, 1024, 1]
    O.set_matmul_threads(1)
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
                      "single-threaded: the Host runs strided binaries and axis reductions on one thread "
                      "(src/parallel.rs:12-14), so one core is all this path can use",
            "build": ORACLE_FLAGS, "seconds": round(dt * reps, 2), "host_cores": os.cpu_count()}


# ---------------------------------------------------------------------------
# GEMMs: config 5 (bf16) and config 1 (f32)
# ---------------------------------------------------------------------------
def run_gemm(args, torch, world, rank, comm, dtype="bf16", size=8192):
    """Config 5 (bf16, M=N=K=size) or config 1 (f32 1024^3): C = A.B through
    tc_matmul, inputs resident; at P > 1 config 5 runs row panels with the
    all-gather fused into the GEMM (tc_matmul_allgather).  metric TFLOP/s."""
    from tensorcrate_b200 import _native as N
    from tensorcrate_b200 import cuda
    lib = N.lib()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    m = k = n = size
    rng = np.random.default_rng(0)
    a_host = cuda.f32_to_bits(rng.uniform(-1, 1, m * k).astype(np.float32), dtype)
    b_host = cuda.f32_to_bits(rng.uniform(-1, 1, k * n).astype(np.float32), dtype)
    b = cuda.CudaStorage.store(b_host, dtype)
    code = N.DTYPES[dtype]
    esz = 4 if dtype == "f32" else 2
    panels = world > 1 and dtype != "f32"
    peer = None
    if panels:
        # Row panels: rank r computes rows [r*m/P, (r+1)*m/P) of C with B
        # replicated; the GEMM epilogue stores each tile into every rank's C.
        if m % world:
            raise SystemExit(f"M={m} does not split over {world} ranks")
        rows = m // world
        a_rows = a_host[rank * rows * k:(rank + 1) * rows * k]
        a = cuda.CudaStorage.store(a_rows, dtype)
        from tensorcrate_b200.sharding import PeerBuffer
        peer = PeerBuffer(comm, m * n * 2)
        c_ptr = peer.ptr

        def run(a_ptr, b_ptr, s):
            N.check("matmul_allgather", lib.tc_matmul_allgather(comm, code, rows, k, n, a_ptr, b_ptr, peer.handle, s))
    else:
        rows = m
        a_rows = a_host
        a = cuda.CudaStorage.store(a_host, dtype)
        c = cuda.CudaStorage(dtype, m * n)
        c_ptr = c.ptr

        def run(a_ptr, b_ptr, s):
            N.check("matmul", lib.tc_matmul(code, 0, m, k, n, a_ptr, b_ptr, c_ptr, 0, s))

    # Small products fit in L2: the timed steps then rotate over enough
    # copies of A and B (and, on one GPU, C) that one pass over them
    # exceeds twice the 126 MB L2, so every step reads its operands from HBM.
    set_bytes = (rows * k + k * n + (0 if panels else m * n)) * esz
    copies = max(1, math.ceil(2 * 126e6 / set_bytes)) if 3 * size * size * esz <= 126e6 else 1
    rot = [(a, b, c_ptr)]
    for _ in range(copies - 1):
        a2 = cuda.CudaStorage(dtype, rows * k)
        b2 = cuda.CudaStorage(dtype, k * n)
        N.check("d2d", lib.tc_memcpy_d2d(a2.ptr, a.ptr, a2.nbytes, None))
        N.check("d2d", lib.tc_memcpy_d2d(b2.ptr, b.ptr, b2.nbytes, None))
        c2 = c_ptr if panels else cuda.CudaStorage(dtype, m * n)
        rot.append((a2, b2, c2))
    turn = [0]

    def rotating_step():
        a_i, b_i, c_i = rot[turn[0] % len(rot)]
        turn[0] += 1
        if panels:
            run(a_i.ptr, b_i.ptr, sp)
        else:
            N.check("matmul", lib.tc_matmul(code, 0, m, k, n, a_i.ptr, b_i.ptr,
                                            c_i if isinstance(c_i, int) else c_i.ptr, 0, sp))

    ms, blocks, clocks = timed(torch, world, rotating_step, args, stream)
    torch.cuda.synchronize()
    del rot[1:]
    # the parity check reads C from the first set: run it once more there
    run(a.ptr, b.ptr, sp)

    # parity: sampled rows of every panel of C against the oracle
    import oracle as O
    torch.cuda.synchronize()
    failures = []
    sample = [(p * (m // max(world, 1)) + 17) for p in range(world if panels else 1)] + [m - 3]
    if size > 8192:
        # every band widens all of B in the oracle: three bands at most
        sample = sorted({sample[0], sample[len(sample) // 2], m - 3})
    O.set_matmul_threads(os.cpu_count() or 1)
    try:
        for r0 in sample:
            band = 4 if r0 + 4 <= m else m - r0
            want = O.widen(O.matmul(dtype, 0, band, k, n, a_host[r0 * k:(r0 + band) * k], b_host), dtype)
            got_bits = np.empty(band * n, dtype=np.float32 if dtype == "f32" else np.uint16)
            N.check("d2h", lib.tc_memcpy_d2h(got_bits.ctypes.data, c_ptr + r0 * n * esz, band * n * esz, None))
            got = O.widen(got_bits, dtype)
            tol = 1e-5 * np.sqrt(k) if dtype == "f32" else 2.0 ** -7 * 2
            if not np.max(np.abs(got - want)) <= tol * max(1.0, float(np.max(np.abs(want)))):
                failures.append(f"rank {rank}: rows {r0}..{r0 + band} of C differ from the oracle")
    finally:
        O.set_matmul_threads(1)
    parity = parity_record(torch, world, failures,
                           f"rows {sample} (4 each) of the whole C on every rank against oracle/ "
                           + ("(f32 1e-5*sqrt(K))" if dtype == "f32" else "(2 bf16 ulp of the f32-accumulated result)"))

    # e2e: A (this rank's rows) and B uploaded, the whole C read back, every
    # step, on one stream (the row-panel product writes every rank's C, so a
    # second C would need every rank's read-back ordered before it).
    h_a, h_b, h_c = pinned(torch, a_rows.nbytes), pinned(torch, b_host.nbytes), pinned(torch, m * n * esz)
    h_a.numpy()[:] = a_rows.view(np.uint8)
    h_b.numpy()[:] = b_host.view(np.uint8)
    pipe = Pipeline(torch, lib, stream, uploads=[(h_a, [a.ptr, a.ptr], a_rows.nbytes), (h_b, [b.ptr, b.ptr],
                                                                                        b_host.nbytes)],
                    readbacks=[([c_ptr, c_ptr], h_c, m * n * esz)], run=lambda bb, s: run(a.ptr, b.ptr, s))
    e2e_ms = pipe.measure_serial(world, max(3, args.steps // 4))
    if peer is not None:
        torch.cuda.synchronize()
        barrier(torch, world)
        peer.close()

    matvec = None
    if dtype == "f32" and size == 1024:
        # Config 1's matvec: y = M.x over 64 different [1024 x 1024] f32
        # matrices in turn (268 MB, more than L2), so every call reads HBM.
        mats_host = [rng.uniform(-1, 1, m * k).astype(np.float32) for _ in range(64)]
        mats = [cuda.CudaStorage.store(h, "f32") for h in mats_host]
        last_host = mats_host[-1]
        xv_host = rng.uniform(-1, 1, k).astype(np.float32)
        xv = cuda.CudaStorage.store(xv_host, "f32")
        yv = cuda.CudaStorage("f32", m)
        # The 64 launches are captured in one CUDA graph, so the time is the
        # device's and not the host's launch rate through ctypes.
        graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.graph(graph, stream=cap):
            csp = C.c_void_p(cap.cuda_stream)
            for M in mats:
                N.check("matvec", lib.tc_matvec(N.F32, m, k, M.ptr, xv.ptr, yv.ptr, 0, csp))
        mv_args = argparse.Namespace(steps=8, warmup=3, min_seconds=0.2)
        ms_mv, _, _ = timed(torch, world, graph.replay, mv_args, stream)
        ms_mv /= len(mats)
        mv_bytes = m * k * 4 + k * 4 + m * 4
        mv_gbs = mv_bytes / (ms_mv * 1e-3) / 1e9
        # the last product of the replay against the oracle's dot per row
        torch.cuda.synchronize()
        want_y = np.empty(m, np.float32)
        O.call("orc_matvec", N.F32, m, k, O.ptr(last_host), O.ptr(xv_host), O.ptr(want_y), 0)
        got_y = yv.as_slice()
        if not np.max(np.abs(got_y - want_y)) <= 1e-5 * np.sqrt(k) * max(1.0, float(np.max(np.abs(want_y)))):
            failures.append(f"rank {rank}: matvec differs from the oracle")
        parity = parity_record(torch, world, failures, parity["checked"] + "; the matvec's y (1e-5*sqrt(K))")
        matvec = {"us": round(ms_mv * 1e3, 2), "gbs": round(mv_gbs, 1),
                  "frac": round(mv_gbs / peaks()[0]["hbm_gbs"], 3), "bytes": mv_bytes,
                  "l2": "64 matrices in turn, 268 MB"}
        del graph
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
    e2e_total = flops / (e2e_ms * 1e-3) / 1e12 * (1 if panels else world)
    rec = {"metric": f"{dtype} GEMM TFLOP/s", "value": round(total, 1), "unit": "TFLOP/s", "n_gpus": world,
           "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong" if panels else "weak",
           "dtype": dtype, "data": "synthetic uniform[-1,1], seeded",
           "config": {"workload": f"config{'5' if dtype != 'f32' else '1'}: C = A.B, M=N=K={size}, f32 accumulate",
                      "parallelism": (f"row panels x{world}, all-gather fused into the GEMM epilogue (NVLink peer "
                                      "stores)" if panels else (f"replicas x{world}" if world > 1 else "single GPU")),
                      "l2": (f"inputs resident; no flush: A, B and C ({3 * size * size * esz / 1e6:.0f} MB) exceed "
                             "the 126 MB L2") if copies == 1 else
                            (f"inputs resident; A, B and C ({3 * size * size * esz / 1e6:.1f} MB) fit in the 126 MB "
                             f"L2, so the steps rotate over {copies} copies of them ({copies * set_bytes / 1e6:.0f} MB "
                             "per rank), more than twice L2")},
           "timing": blocks,
           "roofline": {"bound": "tensor", "kernel": "gemm_tc" if dtype != "f32" else "gemm_tc<tf32> x3 passes",
                        "achieved": round(per_gpu * passes, 1), "peak": round(peak, 1),
                        "peak_source": (pk_kind + " burst") if dtype != "f32" else f"{pk_kind} bf16 / 2 (TF32 rate)",
                        "unit": "TFLOP/s", "frac": round(per_gpu * passes / peak, 3),
                        "frac_of_sustained": round(per_gpu * passes / (pk["bf16_tflops_sustained"] /
                                                                       (2 if dtype == "f32" else 1)), 3),
                        "traffic": None},
           "e2e": {"value": round(e2e_total, 1), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step": pipe.h2d, "d2h_bytes_per_step": pipe.d2h,
                   "how": "this rank's rows of A and all of B uploaded, the whole C read back, every step, in turn "
                          "on one stream"},
           "parity": parity,
           # f32: two operand splits, the TF32 product, the split-K finish; bf16: the product
           "gpu_launches_per_step": 4 if dtype == "f32" else 1,
           "clocks": clocks}
    rec["gpu_launches"] = rec["gpu_launches_per_step"] * args.steps * blocks["blocks"]
    if matvec is not None:
        rec["config"]["matvec"] = matvec
    return rec


# ---------------------------------------------------------------------------
# config 3: layout copies
# ---------------------------------------------------------------------------
def run_c3(args, torch, world, rank, comm):
    """Config 3: f16 [8,16,128,64,32] permuted (0,3,1,4,2) and made
    contiguous; then sliced [:, 8:, :, :32, :], split in 4 along axis 1 and
    concatenated back (one assemble).  metric GB/s of the two copies."""
    from tensorcrate_b200 import cuda
    from tensorcrate_b200 import _native as N
    import oracle as O
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    lib = N.lib()
    shape = [8, 16, 128, 64, 32]
    n = int(np.prod(shape))
    x_host = np.random.default_rng(3).standard_normal(n).astype(np.float16).view(np.uint16)
    xs = [cuda.CudaStorage.store(x_host, "f16"), cuda.CudaStorage("f16", n)]
    perm = [0, 3, 1, 4, 2]
    pv = cuda.Tensor(xs[0], shape).view().permute(perm)
    p_shape = pv.shape

    def plan(out_p):
        sl = cuda.TensorView(out_p, p_shape, cuda.contiguous_strides(p_shape)).slice(1, 8, p_shape[1]).slice(3, 0, 32)
        cat_shape = list(sl.shape)
        to = cuda.contiguous_strides(cat_shape)
        regions, at = [], 0
        for v in sl.chunk(1, 4):
            regions.append(cuda.Cuda._region((v.storage, v.shape, v.offset, v.strides, at * to[1], to)))
            at += v.shape[1]
        return sl, cat_shape, (N.Region * len(regions))(*regions), len(regions)

    outs_p = [cuda.CudaStorage("f16", n), cuda.CudaStorage("f16", n)]
    plans = [plan(o) for o in outs_p]
    cat_shape = plans[0][1]
    mcat = int(np.prod(cat_shape))
    outs_c = [cuda.CudaStorage("f16", mcat), cuda.CudaStorage("f16", mcat)]
    ps, pst = N.sizes(p_shape), N.sizes(pv.strides)

    def step(b=0, s=sp):
        N.check("copy", lib.tc_strided_copy(2, 5, ps, xs[b].ptr, n, 0, pst, outs_p[b].ptr, s))
        N.check("assemble", lib.tc_assemble(2, outs_c[b].ptr, mcat, plans[b][2], plans[b][3], s))

    ms, blocks, clocks = timed(torch, world, step, args, stream)
    byts = 2 * n * 2 + 2 * mcat * 2
    gbs = byts / (ms * 1e-3) / 1e9
    pk, pk_kind = peaks()

    # Interpretation B: the slice's indices on the original axes,
    # x[:, 8:, :, :32, :] = [8, 8, 128, 32, 32], split in 4 along axis 1 and
    # concatenated back (one assemble of four regions).
    t = cuda.Tensor(xs[0], shape)
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
        N.check("assemble", lib.tc_assemble(2, out_b.ptr, m_b, arr_b, len(regions_b), sp))

    ms_b, _, _ = timed(torch, world, step_b, argparse.Namespace(steps=args.steps, warmup=args.warmup,
                                                                min_seconds=0.3), stream)
    gbs_b = 2 * m_b * 2 / (ms_b * 1e-3) / 1e9

    # parity: the whole permuted copy, the concatenation and interpretation
    # B, bit for bit against the oracle's strided copies of the same views.
    torch.cuda.synchronize()
    failures = []
    want_p = O.strided_copy(x_host, p_shape, 0, pv.strides)
    if not np.array_equal(outs_p[0].as_slice(), want_p):
        failures.append(f"rank {rank}: the permuted copy differs from the oracle")
    sl = plans[0][0]
    want_c = O.strided_copy(want_p, sl.shape, sl.offset, sl.strides)
    if not np.array_equal(outs_c[0].as_slice(), want_c):
        failures.append(f"rank {rank}: the concatenation differs from the oracle's contiguous slice")
    want_b = O.strided_copy(x_host, slb.shape, slb.offset, slb.strides)
    if not np.array_equal(out_b.as_slice(), want_b):
        failures.append(f"rank {rank}: interpretation B differs from the oracle")
    parity = parity_record(torch, world, failures, "all of the permuted copy, the concatenation (= the contiguous "
                                                   "slice) and interpretation B, bit-exact against oracle/")

    h_x, h_p, h_c = pinned(torch, n * 2), pinned(torch, n * 2), pinned(torch, mcat * 2)
    h_x.numpy()[:] = x_host.view(np.uint8)
    pipe = Pipeline(torch, lib, stream, uploads=[(h_x, [xs[0].ptr, xs[1].ptr], n * 2)],
                    readbacks=[([outs_p[0].ptr, outs_p[1].ptr], h_p, n * 2),
                               ([outs_c[0].ptr, outs_c[1].ptr], h_c, mcat * 2)],
                    run=lambda b, s: step(b, s))
    e2e_ms = pipe.measure(world, max(5, args.steps // 2))
    rec = {"metric": "config-3 layout copy HBM throughput (GB/s)", "value": round(world * gbs, 1), "unit": "GB/s",
           "n_gpus": world, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "dtype": "f16",
           "data": "synthetic N(0,1), seeded",
           "config": {"workload": "config3: permute(0,3,1,4,2)+contiguous, slice->split(4)->concat "
                                  "(interpretation A: slice of the permuted tensor)",
                      "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                      "algorithmic_bytes_per_step": byts,
                      "l2": "no flush: the permute moves 134 MB, more than the 126 MB L2",
                      "interpretation_b": {"workload": "x[:, 8:, :, :32, :] on the original axes -> [8,8,128,32,32], "
                                                       "split(4) along axis 1 -> concat",
                                           "ms": round(ms_b, 4), "gbs": round(gbs_b, 1),
                                           "frac": round(gbs_b / pk["hbm_gbs"], 3),
                                           "l2": "33.6 MB of traffic per step: L2-resident between steps"}},
           "timing": blocks,
           "roofline": {"bound": "hbm", "kernel": "strided copy + assemble", "achieved": round(gbs, 1),
                        "peak": pk["hbm_gbs"], "peak_source": pk_kind, "unit": "GB/s",
                        "frac": round(gbs / pk["hbm_gbs"], 3), "traffic": None},
           "e2e": {"value": round(world * byts / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                   "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": pipe.h2d, "d2h_bytes_per_step": pipe.d2h,
                   "how": "the input uploaded, the permuted copy and the concatenation read back, every step; "
                          "pipelined over two device sets"},
           "parity": parity, "gpu_launches_per_step": 2, "clocks": clocks}
    rec["gpu_launches"] = 2 * args.steps * blocks["blocks"]
    return rec


# ---------------------------------------------------------------------------
# config 4: the MLP training step
# ---------------------------------------------------------------------------
C4_DIMS = [1024, 4096, 4096, 1024]


def run_c4(args, torch, world, rank, comm):
    """Config 4: one training step of the 1024-4096-4096-1024 ReLU MLP in
    bf16 (tape + Adam(1e-3, 0.9, 0.999, 1e-8), as the reference runs it),
    global batch 2048 split across the ranks (strong scaling), the optimizer
    sharded over the ranks.  metric: steps/s."""
    from tensorcrate_b200 import _native as N
    from tensorcrate_b200 import cuda
    from tensorcrate_b200.mlp import Mlp, xavier
    lib = N.lib()
    dtype = "bf16"
    dims = C4_DIMS
    gbatch = args.batch
    if gbatch % world:
        raise SystemExit("global batch must divide by the number of GPUs")
    batch = gbatch // world
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    rng = np.random.default_rng(6)
    ws = [xavier(dims[l + 1], dims[l], rng) for l in range(3)]
    bs = [np.zeros(dims[l + 1], np.float32) for l in range(3)]
    m = Mlp(dtype, dims, batch, gbatch)
    m.load(ws, bs)
    if world > 1:
        m.attach(comm)  # the exchange runs over NVLink peer memory
    # The global batch (seeds 4, 5), rank r's columns.
    x_all = np.random.default_rng(4).standard_normal((dims[0], gbatch)).astype(np.float32)
    y_all = np.random.default_rng(5).standard_normal((dims[-1], gbatch)).astype(np.float32)
    cols = slice(rank * batch, (rank + 1) * batch)
    xr = cuda.f32_to_bits(np.ascontiguousarray(x_all[:, cols]), dtype)
    yr = cuda.f32_to_bits(np.ascontiguousarray(y_all[:, cols]), dtype)
    xs = [cuda.CudaStorage.store(xr, dtype), cuda.CudaStorage(dtype, xr.size)]
    ys = [cuda.CudaStorage.store(yr, dtype), cuda.CudaStorage(dtype, yr.size)]
    losses = [cuda.CudaStorage(dtype, 1), cuda.CudaStorage(dtype, 1)]

    def step():
        m.step(xs[0], ys[0], comm=comm, stream=stream)

    ms, blocks, clocks = timed(torch, world, step, args, stream)
    gemm_flops = 3 * 2 * gbatch * sum(dims[l] * dims[l + 1] for l in range(3))  # fwd + dW + dX
    pk, pk_kind = peaks()
    tflops = gemm_flops / (ms * 1e-3) / 1e12

    # Phases, each timed alone (CUDA events, max over ranks): the step
    # without the exchange (products, loss, adjoints and the whole Adam pass
    # on this rank's batch), the Adam pass alone over all and over 1/P of the
    # parameters, and the collectives over the whole flat gradient.
    phase_args = argparse.Namespace(steps=args.steps, warmup=3, min_seconds=0.2)
    solo = Mlp(dtype, dims, batch, gbatch)
    solo.load(ws, bs)
    phases = {}
    phases["step_without_exchange_ms"] = round(timed(torch, world, lambda: solo.step(xs[0], ys[0], stream=stream),
                                                     phase_args, stream)[0], 4)
    if world > 1:
        # the same sharded step with NCCL's reduce-scatter and all-gather
        # around a local Adam instead of the peer-memory exchange
        phases["step_with_nccl_exchange_ms"] = round(timed(
            torch, world, lambda: solo.step(xs[0], ys[0], comm=comm, stream=stream), phase_args, stream)[0], 4)
    total = sum(solo.block(l)[0] for l in range(3))
    flat = [cuda.CudaStorage(dtype, total) for _ in range(4)]
    for f in flat:
        N.check("memset", lib.tc_memset(f.ptr, 0, f.nbytes, None))
    adam = lambda n_el: N.check("adam", lib.tc_adam(N.BF16, n_el, flat[0].ptr, flat[1].ptr, flat[2].ptr, flat[3].ptr,
                                                    1, 1e-3, 0.8984375, 0.98828125, 0.0, 10.0, 100.0, sp))
    phases["adam_all_ms"] = round(timed(torch, world, lambda: adam(total), phase_args, stream)[0], 4)
    if world > 1:
        phases["adam_shard_ms"] = round(timed(torch, world, lambda: adam(total // world), phase_args, stream)[0], 4)
        count = total // world
        g = flat[1]
        phases["reduce_scatter_ms"] = round(timed(
            torch, world, lambda: N.check("rs", lib.tc_reducescatter(comm, N.BF16, g.ptr, g.ptr + rank * count * 2,
                                                                     count, N.SUM, sp)), phase_args, stream)[0], 4)
        phases["all_gather_ms"] = round(timed(
            torch, world, lambda: N.check("ag", lib.tc_allgather(comm, N.BF16, g.ptr + rank * count * 2, g.ptr, count,
                                                                 sp)), phase_args, stream)[0], 4)
        phases["exchange_bytes_per_rank"] = 2 * (world - 1) * count * 2
    del solo, flat

    # parity: one fresh data-parallel step (beta2 = 0.99: the configured
    # 0.999 rounds to 1.0 in bf16 and makes the reference's update NaN)
    # against the oracle's whole-batch step, on rank 0.
    parity = parity_c4(torch, world, rank, comm, ws, bs, x_all, y_all, batch, gbatch)

    # e2e: inputs and targets uploaded from pinned host memory each step, the
    # loss read back (parameters and optimizer state stay on the device).
    h_x, h_y, h_l = pinned(torch, xr.nbytes), pinned(torch, yr.nbytes), pinned(torch, 2)
    h_x.numpy()[:] = xr.reshape(-1).view(np.uint8)
    h_y.numpy()[:] = yr.reshape(-1).view(np.uint8)
    pipe = Pipeline(torch, lib, stream, uploads=[(h_x, [xs[0].ptr, xs[1].ptr], xr.nbytes),
                                                 (h_y, [ys[0].ptr, ys[1].ptr], yr.nbytes)],
                    readbacks=[([losses[0].ptr, losses[1].ptr], h_l, 2)],
                    run=lambda b, s: N.check("mlp", lib.tc_mlp_step(m.handle, xs[b].ptr, ys[b].ptr, comm,
                                                                    losses[b].ptr, s)))
    e2e_steps = max(5, args.steps // 2)
    e2e_ms = pipe.measure(world, e2e_steps)
    serial_ms = pipe.measure_serial(world, max(3, e2e_steps // 2))
    torch.cuda.synchronize()
    barrier(torch, world)
    m.close()
    # sharded: per layer two flag signals, a flag wait and the exchange kernel instead of one Adam
    # launch, and a flag wait at the end
    launches = 24 + (0 if world == 1 else 3 * 4 - 1 + 1)
    rec = {"metric": "config-4 MLP training steps/s", "value": round(1000.0 / ms, 2), "unit": "steps/s",
           "n_gpus": world, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
           "dtype": dtype, "data": "synthetic N(0,1) inputs/targets, Xavier-uniform weights, seeded",
           "config": {"workload": "config4: MLP 1024-4096-4096-1024 ReLU, MSE, Adam(1e-3,0.9,0.999,1e-8), bf16",
                      "global_batch": gbatch, "per_rank_batch": batch,
                      "parallelism": f"dp{world}" + (" (per layer, beside the backward pass: one kernel sums this "
                                                     "rank's 1/P of the gradient block over the ranks through NVLink "
                                                     "peer loads, runs Adam on it and stores the new parameters into "
                                                     "every rank's copy; flags between the ranks)" if world > 1 else ""),
                      "l2": "no flush: a step touches 50 MB of weights, 150 MB of Adam state and ~100 MB of "
                            "activations, more than the 126 MB L2",
                      "gemm_flops_per_step": gemm_flops},
           "timing": blocks,
           "phases": phases,
           "roofline": {"bound": "tensor", "kernel": "whole step (GEMM share)", "achieved": round(tflops / world, 1),
                        "peak": pk["bf16_tflops_sustained"], "peak_source": pk_kind + " sustained", "unit": "TFLOP/s",
                        "frac": round(tflops / world / pk["bf16_tflops_sustained"], 3), "traffic": None,
                        "note": "GEMM flops per GPU per second over the whole step"},
           "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "steps/s", "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step": pipe.h2d, "d2h_bytes_per_step": pipe.d2h,
                   "how": "inputs and targets uploaded and the loss read back every step; pipelined over two device "
                          "sets", "serial_ms_per_step": round(serial_ms, 4)},
           "parity": parity,
           # per step: 3 forward products + 1 split-K finish, the loss pass, per layer the bias
           # adjoints (matvec, vecmat + finish, an add below the top) and 2 products (+1 finish
           # for the split input-gradient product of layer 1), Adam
           "gpu_launches_per_step": launches, "clocks": clocks}
    rec["gpu_launches"] = launches * args.steps * blocks["blocks"]
    return rec


def run_c4_weak(args, torch, world, rank, comm):
    """Config 4's step with the batch per GPU fixed at 2048 (weak scaling:
    global batch 2048*P), the usual data-parallel setting, on the same
    sharded path as c4.  metric: samples/s."""
    from tensorcrate_b200 import cuda
    from tensorcrate_b200.mlp import Mlp, xavier
    dtype, dims, batch = "bf16", C4_DIMS, args.batch
    gbatch = batch * world
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(6)
    ws = [xavier(dims[l + 1], dims[l], rng) for l in range(3)]
    bs = [np.zeros(dims[l + 1], np.float32) for l in range(3)]
    m = Mlp(dtype, dims, batch, gbatch)
    m.load(ws, bs)
    if world > 1:
        m.attach(comm)
    x = cuda.CudaStorage.store(cuda.f32_to_bits(np.random.default_rng(40 + rank).standard_normal(
        (dims[0], batch)).astype(np.float32), dtype), dtype)
    y = cuda.CudaStorage.store(cuda.f32_to_bits(np.random.default_rng(50 + rank).standard_normal(
        (dims[-1], batch)).astype(np.float32), dtype), dtype)
    ms, blocks, clocks = timed(torch, world, lambda: m.step(x, y, comm=comm, stream=stream), args, stream)
    torch.cuda.synchronize()
    barrier(torch, world)
    m.close()
    pk, pk_kind = peaks()
    gemm_flops = 3 * 2 * batch * sum(dims[l] * dims[l + 1] for l in range(3))
    tflops = gemm_flops / (ms * 1e-3) / 1e12
    launches = 24 + (0 if world == 1 else 3 * 4 - 1 + 1)
    return {"metric": "config-4 MLP training samples/s, 2048 samples per GPU", "value": round(gbatch * 1000.0 / ms, 1),
            "unit": "samples/s", "steps_per_s": round(1000.0 / ms, 2), "n_gpus": world, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "dtype": dtype,
            "data": "synthetic N(0,1) inputs/targets, Xavier-uniform weights, seeded",
            "config": {"workload": "config4's network and optimizer, batch 2048 per GPU", "global_batch": gbatch,
                       "per_rank_batch": batch, "parallelism": f"dp{world}, the same sharded exchange as c4",
                       "l2": "no flush: a step's working set exceeds the 126 MB L2"},
            "timing": blocks,
            "roofline": {"bound": "tensor", "kernel": "whole step (GEMM share)", "achieved": round(tflops, 1),
                         "peak": pk["bf16_tflops_sustained"], "peak_source": pk_kind + " sustained", "unit": "TFLOP/s",
                         "frac": round(tflops / pk["bf16_tflops_sustained"], 3), "traffic": None},
            "parity": {"status": "ok", "checked": "the same step code as c4, whose parity record covers it"},
            "gpu_launches_per_step": launches, "gpu_launches": launches * args.steps * blocks["blocks"],
            "clocks": clocks}


def parity_c4(torch, world, rank, comm, ws, bs, x_all, y_all, batch, gbatch):
    import oracle as O
    from tensorcrate_b200 import cuda
    from tensorcrate_b200.mlp import Mlp
    dtype, dims = "bf16", C4_DIMS
    cols = slice(rank * batch, (rank + 1) * batch)
    dp = Mlp(dtype, dims, batch, gbatch, beta2=0.99)
    dp.load(ws, bs)
    if world > 1:
        dp.attach(comm)
    x = cuda.CudaStorage.store(O.narrow(np.ascontiguousarray(x_all[:, cols]), dtype), dtype)
    y = cuda.CudaStorage.store(O.narrow(np.ascontiguousarray(y_all[:, cols]), dtype), dtype)
    dp.step(x, y, comm=comm, stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    failures = []
    got = [dp.params(l) for l in range(3)]
    blocks = [dp.block(l) for l in range(3)]
    grads = [dp.grads(l) for l in range(3)]
    if rank == 0:
        O.set_matmul_threads(os.cpu_count() or 1)
        try:
            h = O.lib().orc_mlp_create(O.DTYPES[dtype], 3, O.u32s(dims), gbatch, gbatch, 1e-3, 0.9, 0.99, 1e-8)
            for l, (w, b) in enumerate(zip(ws, bs)):
                O.call("orc_mlp_params", h, l, O.ptr(O.narrow(w, dtype)), O.ptr(O.narrow(b, dtype)), 0)
            loss = np.empty(1, O.STORE[dtype])
            O.call("orc_mlp_step", h, O.ptr(O.narrow(x_all, dtype)), O.ptr(O.narrow(y_all, dtype)), O.ptr(loss), 0)
        finally:
            O.set_matmul_threads(1)
        for l in range(3):
            ow = np.empty(dims[l + 1] * dims[l], O.STORE[dtype])
            ob = np.empty(dims[l + 1], O.STORE[dtype])
            O.call("orc_mlp_params", h, l, O.ptr(ow), O.ptr(ob), 1)
            for name, g, o in (("weight", got[l][0], ow), ("bias", got[l][1], ob)):
                diff = np.abs(O.widen(g, dtype) - O.widen(o, dtype))
                if not (np.max(diff) <= 2e-3 + 8e-3 and np.median(diff) <= 4e-3):
                    failures.append(f"layer {l} {name}s after one step: max {np.max(diff):.3g}, "
                                    f"median {np.median(diff):.3g} off the oracle")
            # this rank's shard of the gradient block holds the sum over ranks
            gw = np.empty(dims[l + 1] * dims[l], O.STORE[dtype])
            gb = np.empty(dims[l + 1], O.STORE[dtype])
            O.call("orc_mlp_grads", h, l, O.ptr(gw), O.ptr(gb))
            length, at = blocks[l]

            def block(w, b):
                out = np.zeros(length, np.float32)
                out[:w.size] = O.widen(w, dtype)
                out[at:at + b.size] = O.widen(b, dtype)
                return out
            mine, want = block(*grads[l]), block(gw, gb)
            hi = length // world
            err, scale = float(np.linalg.norm(mine[:hi] - want[:hi])), float(np.linalg.norm(want[:hi]))
            if not err <= max(1e-2, world * 2.0 ** -7) * scale:
                failures.append(f"layer {l} gradient (rank 0's shard) off the oracle by {err:.3g} of {scale:.3g}")
        O.lib().orc_mlp_destroy(h)
    torch.cuda.synchronize()
    barrier(torch, world)
    dp.close()
    return parity_record(torch, world, failures,
                         "one data-parallel step (beta2 0.99) from the bench's weights: every parameter against the "
                         "oracle's whole-batch step (max <= 2 rates + 1 bf16 step, median <= 4e-3), rank 0's gradient "
                         "shard within max(1e-2, P*2^-7) in norm")


# ---------------------------------------------------------------------------
# the other Kernels<T> methods, each alone (--workload trait)
# ---------------------------------------------------------------------------
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
    # each call timed for 0.2 s at least (less only when asked: a short
    # profiling run)
    t_args = argparse.Namespace(steps=args.steps, warmup=args.warmup, min_seconds=min(0.2, args.min_seconds))

    def measure(name, fn, byts, flops=None, bound="hbm", peak=None):
        nonlocal hbm_bytes, hbm_ms
        ms, _, _ = timed(torch, world, fn, t_args, stream)
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
    # the state-carrying rules: p, g and the state read, p and the state written
    state = cuda.CudaStorage.store(np.abs(rng.standard_normal(n, dtype=np.float32)) * np.float32(0.01), "f32")
    measure("momentum", lambda: N.check("momentum", lib.tc_momentum(f32, n, o1.ptr, y.ptr, o2.ptr, 1e-3, 0.9, 0,
                                                                        sp)), 5 * 4 * n)
    measure("rmsprop", lambda: N.check("rmsprop", lib.tc_rmsprop(f32, n, o1.ptr, y.ptr, state.ptr, 1e-3, 0.9, 1e-8,
                                                                     sp)), 5 * 4 * n)
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
    # RmsProp's program (optim.rs:948-964) through Kernels::fused: in place,
    # tc_fused runs it as the rule's kernel; into fresh outputs, the
    # interpreter runs it
    rate, rho, eps = float(np.float32(1e-3)), float(np.float32(0.9)), float(np.float32(1e-8))
    rms = [ins(N.I_LOAD, 0, slot=0), ins(N.I_LOAD, 1, slot=1), ins(N.I_BINARY, 2, 0, 0, op=2),
           ins(N.I_CONST, 3, value=float(np.float32(1.0) - np.float32(rho))), ins(N.I_BINARY, 4, 2, 3, op=2),
           ins(N.I_LOAD, 5, slot=2), ins(N.I_CONST, 6, value=rho), ins(N.I_BINARY, 7, 5, 6, op=2),
           ins(N.I_BINARY, 8, 7, 4, op=0), ins(N.I_UNARY, 9, 8, op=N.SQRT), ins(N.I_CONST, 10, value=eps),
           ins(N.I_BINARY, 11, 9, 10, op=0), ins(N.I_BINARY, 12, 0, 11, op=3), ins(N.I_CONST, 13, value=rate),
           ins(N.I_BINARY, 14, 12, 13, op=2), ins(N.I_BINARY, 15, 1, 14, op=1), ins(N.I_STORE, a=15, slot=0),
           ins(N.I_STORE, a=8, slot=1)]
    rms_code = (N.Instr * len(rms))(*rms)
    o3 = cuda.CudaStorage("f32", n)
    rms_places = (N.Place * 3)(place(y.ptr), place(o1.ptr), place(state.ptr))
    dts2 = (C.c_int * 2)(f32, f32)
    in_place = (C.c_void_p * 2)(o1.ptr, state.ptr)
    fresh = (C.c_void_p * 2)(o2.ptr, o3.ptr)
    measure("fused_rmsprop_program_in_place",
            lambda: N.check("fused", lib.tc_fused(f32, rows, cols, rms_code, len(rms), rms_places, 3, in_place, dts2, 2,
                                                  sp)), 5 * 4 * rows * cols)
    measure("fused_rmsprop_program_interpreted",
            lambda: N.check("fused", lib.tc_fused(f32, rows, cols, rms_code, len(rms), rms_places, 3, fresh, dts2, 2,
                                                  sp)), 5 * 4 * rows * cols)
    gbs = hbm_bytes / (hbm_ms * 1e-3) / 1e9
    return {"metric": "trait-method kernels HBM throughput (GB/s)", "value": round(gbs, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(hbm_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1) / uniform, seeded",
            "config": {"workload": "each trait-method kernel alone: 64M-element vectors (sort: 32M, distribution: 16M), "
                                   "8192x8192 matrices, 16384x4096 programs",
                       "l2": "no flush: every input is 256 MB or more, above the 126 MB L2 (sort: 128 MB)",
                       "value": "algorithmic bytes of the HBM-bound calls / the sum of their times"},
            "roofline": {"bound": "hbm", "kernel": "all HBM-bound trait-method calls", "achieved": round(gbs, 1),
                         "peak": hbm, "peak_source": pk_kind, "unit": "GB/s", "frac": round(gbs / hbm, 3),
                         "traffic": None},
            "ops": ops, "gpu_launches": args.steps * sum(LAUNCHES_PER_CALL.get(k, 1) for k in ops)}


LAUNCHES_PER_CALL = {"prefix_sum": 3, "sort": 10, "moments": 4, "axis_moments_rows": 1, "dot": 2, "vector_sum": 2}


# ---------------------------------------------------------------------------
def headline_keys(rec: dict, args) -> dict:
    """A sub-record as the headline line of a single-workload run."""
    out = dict(rec)
    out.setdefault("steps", args.steps)
    out.setdefault("warmup", args.warmup)
    out.setdefault("vs_baseline", None)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="all", choices=["all", "c1", "c2", "c3", "c4", "c4_weak", "c5", "trait"])
    ap.add_argument("--batch", type=int, default=2048, help="config 4's global batch")
    ap.add_argument("--size", type=int, default=8192, help="config 5's M=N=K")
    ap.add_argument("--min-seconds", type=float, default=1.0, help="device time each timed region lasts at least")
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
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                             device_id=torch.device("cuda", local))
    comm = init_comm(torch, world, rank)
    runners = {"c1": lambda: run_gemm(args, torch, world, rank, comm, "f32", 1024),
               "c2": lambda: run_c2(args, torch, world, rank, comm),
               "c3": lambda: run_c3(args, torch, world, rank, comm),
               "c4": lambda: run_c4(args, torch, world, rank, comm),
               "c4_weak": lambda: run_c4_weak(args, torch, world, rank, comm),
               "c5": lambda: run_gemm(args, torch, world, rank, comm, "bf16", args.size),
               "c5_16384": lambda: run_gemm(args, torch, world, rank, comm, "bf16", 16384),
               "c5_4096": lambda: run_gemm(args, torch, world, rank, comm, "bf16", 4096),
               "trait": lambda: run_trait(args, torch, world, rank, comm)}
    if args.workload == "all":
        line = run_c2(args, torch, world, rank, comm)
        for key in ("c4", "c4_weak", "c5", "c5_16384", "c5_4096", "c1", "c3"):
            line[key] = runners[key]()
        statuses = [line["parity"]] + [line[k]["parity"] for k in ("c4", "c5", "c5_16384", "c5_4096", "c1", "c3")]
        bad = [s for s in statuses if s["status"] != "ok"]
        line["parity_all"] = "ok" if not bad else {"failed": len(bad)}
        line["gpu_launches_all"] = line["gpu_launches"] + sum(line[k]["gpu_launches"]
                                                              for k in ("c4", "c4_weak", "c5", "c5_16384", "c5_4096",
                                                                        "c1", "c3"))
    else:
        line = headline_keys(runners[args.workload](), args)
    if rank == 0 and not args.no_cpu_baseline and args.workload in ("all", "c2"):
        line["cpu_baseline"] = cpu_c2(sample_rows=64, reps=12)
    torch.cuda.synchronize()
    if comm is not None:
        barrier(torch, world)
        N.call("tc_comm_destroy", comm)
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
