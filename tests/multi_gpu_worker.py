"""One rank of the multi-GPU parity checks, run by test_multi_gpu.py under
torch.distributed.run (one process per GPU, NCCL).  Each check computes a
sharded result through the library's collectives and compares it with the
same result computed whole on this rank's GPU:

- tc_matmul_allgather (row panels, all-gather fused into the GEMM epilogue
  over NVLink peer stores) against tc_matmul of the whole product: the same
  bits, on two calls in a row;
- config 2's reductions over a leading-axis shard, finished by all-gather
  (sum/mean over axis 2, argmax over axis 1) or all-reduce (max/min over
  axes 0 and 2), against the whole tensor: the same bits (the integral
  filler makes every sum exact in any order);
- one data-parallel training step (global batch split over the ranks,
  gradients all-reduced) against the whole batch on one GPU, f32.

Rank 0 prints one JSON line {"failures": [...]}; the exit status is 1 when
any check failed on any rank."""
from __future__ import annotations

import ctypes as C
import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import torch  # noqa: E402

from tensorcrate_b200 import _native as N  # noqa: E402
from tensorcrate_b200 import cuda  # noqa: E402
from tensorcrate_b200.mlp import Mlp, xavier  # noqa: E402
from tensorcrate_b200.sharding import PeerBuffer, nccl_comm, shard  # noqa: E402
from util import integral  # noqa: E402


def check_matmul_allgather(comm, world, rank, sp, failures):
    lib = N.lib()
    for rows, inner, cols in ((256, 512, 640), (200, 96, 136)):
        b = cuda.CudaStorage.store(
            cuda.f32_to_bits(np.random.default_rng(3).uniform(-1, 1, inner * cols).astype(np.float32), "bf16"), "bf16")
        c = PeerBuffer(comm, world * rows * cols * 2)
        try:
            for call, seed in enumerate((5, 6)):
                a_full = cuda.f32_to_bits(
                    np.random.default_rng(seed).uniform(-1, 1, world * rows * inner).astype(np.float32), "bf16")
                panel = cuda.CudaStorage.store(a_full[rank * rows * inner:(rank + 1) * rows * inner], "bf16")
                N.check("matmul_allgather", lib.tc_matmul_allgather(comm, N.BF16, rows, inner, cols, panel.ptr, b.ptr,
                                                                    c.handle, sp))
                torch.cuda.synchronize()
                got = np.empty(world * rows * cols, np.uint16)
                N.call("tc_memcpy_d2h", got.ctypes.data_as(C.c_void_p), C.c_void_p(c.ptr), got.nbytes, None)
                whole_a = cuda.CudaStorage.store(a_full, "bf16")
                want = cuda.CudaStorage("bf16", world * rows * cols)
                N.check("matmul", lib.tc_matmul(N.BF16, 0, world * rows, inner, cols, whole_a.ptr, b.ptr, want.ptr, 0,
                                                sp))
                torch.cuda.synchronize()
                if not np.array_equal(got, want.as_slice()):
                    bad = int(np.count_nonzero(got != want.as_slice()))
                    failures.append(f"rank {rank}: matmul_allgather {rows}x{inner}x{cols} call {call}: "
                                    f"{bad} elements differ from the whole product")
                torch.distributed.barrier()
        finally:
            c.close()


def check_reduction_shards(comm, world, rank, sp, failures):
    lib = N.lib()
    per = [4, 64, 256]
    total = per[0] * world
    whole = integral(total * per[1] * per[2]).reshape(total, per[1], per[2])
    start, count = shard(total, world, rank)
    mine = np.ascontiguousarray(whole[start:start + count])
    sz = N.sizes

    def run(x_host):
        shape = list(x_host.shape)
        n = x_host.size
        x = cuda.CudaStorage.store(x_host.ravel(), "f32")
        xs, xst = sz(shape), sz(cuda.contiguous_strides(shape))
        out = {k: cuda.CudaStorage("f32", shape[0] * shape[1]) for k in ("sum", "mean")}
        out.update({k: cuda.CudaStorage("f32", shape[1]) for k in ("max", "min")})
        out["argmax"] = cuda.CudaStorage("u32", shape[0] * shape[2])
        N.check("sum", lib.tc_reduce_axes(0, 3, xs, x.ptr, n, 0, xst, 1, N.u32s([2]), N.AXIS_FOLD, N.SUM, 0,
                                          out["sum"].ptr, sp))
        N.check("mean", lib.tc_reduce_axes(0, 3, xs, x.ptr, n, 0, xst, 1, N.u32s([2]), N.AXIS_MEAN, 0, 0,
                                           out["mean"].ptr, sp))
        for k, op in (("max", N.RMAX), ("min", N.RMIN)):
            N.check(k, lib.tc_reduce_axes(0, 3, xs, x.ptr, n, 0, xst, 2, N.u32s([0, 2]), N.AXIS_FOLD, op, 0,
                                          out[k].ptr, sp))
        argp = C.cast(C.c_void_p(out["argmax"].ptr), C.POINTER(C.c_uint32))
        N.check("argmax", lib.tc_arg_reduce(0, 3, xs, x.ptr, n, 0, xst, 1, N.RMAX, argp, sp))
        return x, out

    _, local = run(mine)
    gathered = {}
    for k in ("sum", "mean", "argmax"):
        gathered[k] = cuda.CudaStorage(local[k].dtype, local[k].len * world)
        N.check("allgather", lib.tc_allgather(comm, N.DTYPES[local[k].dtype], local[k].ptr, gathered[k].ptr,
                                              local[k].len, sp))
    for k, op in (("max", N.RMAX), ("min", N.RMIN)):
        N.check("allreduce", lib.tc_allreduce(comm, N.F32, local[k].ptr, local[k].len, op, sp))
    torch.cuda.synchronize()
    _, ref = run(whole)
    torch.cuda.synchronize()
    for k in ("sum", "mean", "argmax"):
        if not np.array_equal(gathered[k].as_slice(), ref[k].as_slice()):
            failures.append(f"rank {rank}: sharded {k} differs from the whole tensor's")
    for k in ("max", "min"):
        if not np.array_equal(local[k].as_slice(), ref[k].as_slice()):
            failures.append(f"rank {rank}: sharded {k} differs from the whole tensor's")


def check_data_parallel_step(comm, world, rank, sp, failures):
    for peers in (False, True):
        _data_parallel_f32(comm, world, rank, sp, failures, peers)


def _data_parallel_f32(comm, world, rank, sp, failures, peers):
    dims, gbatch = [64, 128, 64], 32
    batch = gbatch // world
    rng = np.random.default_rng(9)
    weights = [xavier(dims[l + 1], dims[l], rng) for l in range(len(dims) - 1)]
    biases = [np.zeros(dims[l + 1], np.float32) for l in range(len(dims) - 1)]
    x = rng.standard_normal((dims[0], gbatch)).astype(np.float32)
    y = rng.standard_normal((dims[-1], gbatch)).astype(np.float32)
    cols = slice(rank * batch, (rank + 1) * batch)
    dp = Mlp("f32", dims, batch, gbatch, rate=1e-3, beta2=0.99, eps=1e-4)
    one = Mlp("f32", dims, gbatch, gbatch, rate=1e-3, beta2=0.99, eps=1e-4)
    dp.load(weights, biases)
    one.load(weights, biases)
    if peers:
        dp.attach(comm)
    how = "peer" if peers else "nccl"
    xd = cuda.CudaStorage.store(np.ascontiguousarray(x[:, cols]).ravel(), "f32")
    yd = cuda.CudaStorage.store(np.ascontiguousarray(y[:, cols]).ravel(), "f32")
    xw = cuda.CudaStorage.store(x.ravel(), "f32")
    yw = cuda.CudaStorage.store(y.ravel(), "f32")
    for _ in range(2):
        dp.step(xd, yd, comm=comm, stream=torch.cuda.current_stream())
        one.step(xw, yw, stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    for l in range(len(dims) - 1):
        for name, got, want in zip(("weight", "bias"), dp.params(l), one.params(l)):
            # The gradient sums reorder over ranks: f32 rounding, then Adam.
            err = float(np.max(np.abs(got - want)))
            if not err <= 2e-5:
                failures.append(f"rank {rank}: data-parallel ({how}) layer {l} {name} differs by {err:.3g}")
    torch.cuda.synchronize()
    dp.close()


def check_data_parallel_bf16(comm, world, rank, sp, failures):
    for peers in (False, True):
        _data_parallel_bf16(comm, world, rank, sp, failures, peers)


def _data_parallel_bf16(comm, world, rank, sp, failures, peers):
    """bf16, the config's type: each rank's partial gradient is rounded to
    bf16 by its own products, and NCCL adds the partials in bf16 with a
    rounding per hop, so the data-parallel gradient is not the whole batch's
    bit for bit.  Bound the difference on this rank's shard of every layer
    block (the shard the sharded optimizer updates), then check the updated
    parameters: the same bits on every rank, and within Adam's first-step
    bounds of the whole-batch step."""
    dims, gbatch = [256, 512, 256], 64
    batch = gbatch // world
    rng = np.random.default_rng(11)
    weights = [xavier(dims[l + 1], dims[l], rng) for l in range(len(dims) - 1)]
    biases = [rng.uniform(-0.05, 0.05, dims[l + 1]).astype(np.float32) for l in range(len(dims) - 1)]
    x = rng.standard_normal((dims[0], gbatch)).astype(np.float32)
    y = rng.standard_normal((dims[-1], gbatch)).astype(np.float32)
    cols = slice(rank * batch, (rank + 1) * batch)
    dp = Mlp("bf16", dims, batch, gbatch, beta2=0.99)
    one = Mlp("bf16", dims, gbatch, gbatch, beta2=0.99)
    dp.load(weights, biases)
    one.load(weights, biases)
    if peers:
        dp.attach(comm)
    how = "peer" if peers else "nccl"
    bits = lambda a: cuda.CudaStorage.store(cuda.f32_to_bits(np.ascontiguousarray(a).ravel(), "bf16"), "bf16")
    dp.step(bits(x[:, cols]), bits(y[:, cols]), comm=comm, stream=torch.cuda.current_stream())
    one.step(bits(x), bits(y), stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    widen = lambda a: cuda.bits_to_f32(a, "bf16")
    for l in range(len(dims) - 1):
        length, at = dp.block(l)

        def block(w, b):
            out = np.zeros(length, np.float32)
            out[:w.size] = widen(w)
            out[at:at + b.size] = widen(b)
            return out
        got, want = block(*dp.grads(l)), block(*one.grads(l))
        lo, hi = rank * length // world, (rank + 1) * length // world
        err, scale = float(np.linalg.norm(got[lo:hi] - want[lo:hi])), float(np.linalg.norm(want[lo:hi]))
        if not err <= world * 2.0 ** -7 * scale:
            failures.append(f"rank {rank}: bf16 data-parallel ({how}) layer {l} gradient shard off by {err:.3g} "
                            f"(norm {scale:.3g})")
        for name, p, q in zip(("weight", "bias"), dp.params(l), one.params(l)):
            mine = torch.tensor(p.view(np.int16).astype(np.int64).sum(), device="cuda")
            lowest, highest = mine.clone(), mine.clone()
            torch.distributed.all_reduce(lowest, op=torch.distributed.ReduceOp.MIN)
            torch.distributed.all_reduce(highest, op=torch.distributed.ReduceOp.MAX)
            if int(lowest.item()) != int(highest.item()):
                failures.append(f"rank {rank}: bf16 data-parallel ({how}) layer {l} {name}s differ between ranks")
            diff = np.abs(widen(p) - widen(q))
            if not (np.max(diff) <= 2e-3 + 8e-3 and np.median(diff) <= 4e-3):
                failures.append(f"rank {rank}: bf16 data-parallel ({how}) layer {l} {name} off the whole-batch step by "
                                f"max {np.max(diff):.3g}, median {np.median(diff):.3g}")
    torch.cuda.synchronize()
    dp.close()


def check_peer_wait_gives_up(comm, world, rank, sp, failures):
    """A rank that stops stepping, between steps and with nothing of its own
    in flight, while the others step: their waits for its flags run out
    (the limit shortened to 50 ms), record the fault and return, and the
    context stays usable.  No GPU faults; the step's results are not used."""
    import time
    dims, batch = [64, 128, 64], 16
    rng = np.random.default_rng(13)
    m = Mlp("f32", dims, batch, batch * world, beta2=0.99, eps=1e-4)
    m.load([xavier(dims[l + 1], dims[l], rng) for l in range(2)], [np.zeros(dims[l + 1], np.float32) for l in range(2)])
    m.attach(comm)
    x = cuda.CudaStorage.store(rng.standard_normal(dims[0] * batch).astype(np.float32), "f32")
    y = cuda.CudaStorage.store(rng.standard_normal(dims[-1] * batch).astype(np.float32), "f32")
    torch.cuda.synchronize()
    torch.distributed.barrier()
    if rank == 0:
        N.call("tc_set_peer_wait_limit", 50_000_000)
        try:
            m.step(x, y, comm=comm, stream=torch.cuda.current_stream())
            torch.cuda.synchronize()  # the step's kernels returned
            fault = C.c_int(0)
            st = N.lib().tc_device_status(C.byref(fault))
            if st != N.ETIMEOUT or fault.value != 1:
                failures.append(f"rank 0: a wait for a silent rank did not report (status {st}, fault {fault.value})")
        finally:
            N.call("tc_set_peer_wait_limit", 0)
            N.call("tc_device_status_reset")
        a = cuda.CudaStorage.store(np.eye(4, dtype=np.float32).ravel(), "f32")
        if not np.array_equal(cuda.Cuda.matmul(a, a, 4, 4, 4).as_slice(), np.eye(4, dtype=np.float32).ravel()):
            failures.append("rank 0: the context is not usable after the wait gave up")
    else:
        time.sleep(1.0)  # on the host, nothing in flight on this GPU
    torch.cuda.synchronize()
    torch.distributed.barrier()
    m.close()


def main() -> int:
    world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    N.call("tc_set_device", local)
    torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                         device_id=torch.device("cuda", local))
    comm = nccl_comm(torch, world, rank)
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    failures: list[str] = []
    for check in (check_matmul_allgather, check_reduction_shards, check_data_parallel_step, check_data_parallel_bf16,
                  check_peer_wait_gives_up):
        try:
            check(comm, world, rank, sp, failures)
        except Exception as e:  # a failed call is a failed check; every rank still reaches the end
            failures.append(f"rank {rank}: {check.__name__}: {e}")
        torch.cuda.synchronize()
        torch.distributed.barrier()
    flags = torch.tensor([len(failures)], dtype=torch.int32, device="cuda")
    torch.distributed.all_reduce(flags)
    everyone = [None] * world
    torch.distributed.all_gather_object(everyone, failures)
    N.call("tc_comm_destroy", comm)
    torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps({"world": world, "failures": [f for fs in everyone for f in fs]}), flush=True)
    return 1 if int(flags.item()) else 0


if __name__ == "__main__":
    sys.exit(main())
