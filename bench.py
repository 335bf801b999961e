"""Benchmark of the tensorcrate CUDA backend's hot path on B200.

Default workload ("config 2"): one step is the
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
copies), c5 (bf16 GEMM, --size).  --impl reference times the reference's
Host path restated in C++ (oracle/) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> tuple[dict, str]:
    try:
        return json.loads(PEAKS_FILE.read_text()), "measured"
    except Exception:
        return dict(FALLBACK), "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.lines = device, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


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
    outs.update({k: cuda.CudaStorage("f32", rows) for k in ("sum", "mean", "var")})
    outs.update({k: cuda.CudaStorage("f32", 512) for k in ("max", "min")})
    outs["argmax"] = cuda.CudaStorage("u32", shape[0] * shape[2])

    sz = N.sizes
    xs, xst = sz(shape), sz(cuda.contiguous_strides(shape))
    bst = sz([0, 0, 1])
    ax2, ax02 = N.u32s([2]), N.u32s([0, 2])
    argp = C.cast(C.c_void_p(outs["argmax"].ptr), C.POINTER(C.c_uint32))
    calls = [
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

    # Collectives for P > 1: gather the per-slab results, all-reduce the
    # [512] extremes across the sharded leading axis.
    gathered = {}
    if world > 1:
        for k in ("sum", "mean", "var", "argmax"):
            gathered[k] = cuda.CudaStorage(outs[k].dtype, outs[k].len * world)

    def collectives():
        if world == 1:
            return
        for k in ("sum", "mean", "var", "argmax"):
            N.check("allgather", lib.tc_allgather(comm, N.DTYPES[outs[k].dtype], outs[k].ptr, gathered[k].ptr,
                                                  outs[k].len, sp))
        N.check("allreduce", lib.tc_allreduce(comm, N.F32, outs["max"].ptr, 512, N.RMAX, sp))
        N.check("allreduce", lib.tc_allreduce(comm, N.F32, outs["min"].ptr, 512, N.RMIN, sp))

    events = {name: [] for name, _, _ in calls}

    def step(record=False):
        for name, fn, a in calls:
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
            step(record=True)
        t1.record(stream)
        torch.cuda.synchronize()
        barrier(torch, world)
    ms = t0.elapsed_time(t1)
    ms = max_over_ranks(torch, world, ms)
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
                   "parallelism": f"leading-axis shards x{world}" + (" (NCCL all-gather + all-reduce)" if world > 1 else ""),
                   "l2": "no flush: every call reads the 134.2 MB input, larger than the 126 MB L2",
                   "algorithmic_bytes_per_step": step_bytes},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                     "peak_source": pk_kind, "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 3),
                     "traffic": None},
        "ops": ops,
        "e2e": {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": len(calls) * args.steps,
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
            "sample": f"all nine calls on a [{sample_rows},512,1024] slab ({scale:.3g} of config 2), x{reps}",
            "seconds": round(dt * reps, 2)}


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
    from tensorcrate_b200 import _native as N
    if world == 1:
        return None
    uid = (C.c_uint8 * 128)()
    if rank == 0:
        N.call("tc_comm_unique_id", uid)
    t = torch.tensor(list(uid), dtype=torch.uint8, device="cuda")
    torch.distributed.broadcast(t, 0)
    uid = (C.c_uint8 * 128)(*t.cpu().tolist())
    comm = C.c_void_p()
    N.call("tc_comm_init", rank, world, uid, C.byref(comm))
    return comm


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c2"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_env()

    if args.impl == "reference":
        if rank != 0:
            return
        reps = max(1, args.steps // 25)
        base = cpu_c2(sample_rows=16, reps=reps)
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
    line = run_c2(args, torch, world, rank, comm)
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_c2(sample_rows=16, reps=1)
    if comm is not None:
        N.call("tc_comm_destroy", comm)
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
