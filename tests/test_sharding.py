"""The sharded paths' host logic on CPU ranks (torch.distributed, gloo,
world size 2): shards of the leading axis reduced by the oracle and finished
by the collective tensorcrate_b200.sharding names equal the unsharded
oracle result; data-parallel gradients summed over ranks equal the
whole-batch gradient."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tensorcrate_b200.sharding import batch_split, finishing_collective, shard


def test_shards_cover_the_axis_in_order():
    for extent in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            pieces = [shard(extent, world, r) for r in range(world)]
            assert sum(c for _, c in pieces) == extent
            assert all(pieces[r][0] + pieces[r][1] == pieces[r + 1][0] for r in range(world - 1))
    assert finishing_collective([0, 2]) == "allreduce" and finishing_collective([2]) == "allgather"
    with pytest.raises(ValueError):
        batch_split(2048, 3)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reduce_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shape = [6, 5, 40]
        full = (np.random.default_rng(0).standard_normal(int(np.prod(shape)))).astype(np.float32).reshape(shape)
        start, count = shard(shape[0], world, rank)
        mine = np.ascontiguousarray(full[start:start + count])
        sh = list(mine.shape)
        st = [sh[1] * sh[2], sh[2], 1]
        out = {}
        for name, axes, kind, op in [("sum2", [2], 0, 0), ("max02", [0, 2], 0, 2), ("min02", [0, 2], 0, 1)]:
            local = torch.from_numpy(O.reduce_axes("f32", sh, mine.reshape(-1), 0, st, axes, kind, op, 0).copy())
            if finishing_collective(axes) == "allgather":
                parts = [torch.zeros_like(local) for _ in range(world)]
                dist.all_gather(parts, local)
                out[name] = torch.cat(parts).numpy()
            else:
                dist.all_reduce(local, op=dist.ReduceOp.MAX if op == 2 else dist.ReduceOp.MIN)
                out[name] = local.numpy()
        arg = torch.from_numpy(O.arg_reduce("f32", sh, mine.reshape(-1), 0, st, 1, 2).astype(np.int64))
        parts = [torch.zeros_like(arg) for _ in range(world)]
        dist.all_gather(parts, arg)
        out["argmax1"] = torch.cat(parts).numpy()
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def test_leading_axis_shards_finish_like_the_whole():
    import oracle as O
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_reduce_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shape = [6, 5, 40]
    full = (np.random.default_rng(0).standard_normal(int(np.prod(shape)))).astype(np.float32)
    st = [200, 40, 1]
    assert np.array_equal(got["sum2"], O.reduce_axes("f32", shape, full, 0, st, [2], 0, 0, 0))
    assert np.array_equal(got["max02"], O.reduce_axes("f32", shape, full, 0, st, [0, 2], 0, 2, 0))
    assert np.array_equal(got["min02"], O.reduce_axes("f32", shape, full, 0, st, [0, 2], 0, 1, 0))
    assert np.array_equal(got["argmax1"], O.arg_reduce("f32", shape, full, 0, st, 1, 2))


def _dp_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dims, gbatch = [16, 32, 8], 24
        batch = batch_split(gbatch, world)
        rng = np.random.default_rng(1)
        ws = [rng.uniform(-0.3, 0.3, (dims[l + 1], dims[l])).astype(np.float32) for l in range(2)]
        bs = [rng.uniform(-0.1, 0.1, dims[l + 1]).astype(np.float32) for l in range(2)]
        x = rng.standard_normal((dims[0], gbatch)).astype(np.float32)
        y = rng.standard_normal((dims[-1], gbatch)).astype(np.float32)
        start, _ = shard(gbatch, world, rank)
        xs = np.ascontiguousarray(x[:, start:start + batch])
        ys = np.ascontiguousarray(y[:, start:start + batch])
        h = O.lib().orc_mlp_create(0, 2, O.u32s(dims), batch, gbatch, 1e-3, 0.9, 0.999, 1e-8)
        for l in range(2):
            O.call("orc_mlp_params", h, l, O.ptr(ws[l]), O.ptr(bs[l]), 0)
        O.call("orc_mlp_step", h, O.ptr(xs), O.ptr(ys), None, 1)
        grads = []
        for l in range(2):
            gw = np.empty(dims[l + 1] * dims[l], np.float32)
            gb = np.empty(dims[l + 1], np.float32)
            O.call("orc_mlp_grads", h, l, O.ptr(gw), O.ptr(gb))
            for g in (gw, gb):
                t = torch.from_numpy(g)
                dist.all_reduce(t)
                grads.append(t.numpy().copy())
        O.lib().orc_mlp_destroy(h)
        if rank == 0:
            q.put((grads, ws, bs, x, y))
    finally:
        dist.destroy_process_group()


def test_data_parallel_gradients_sum_to_the_whole_batch():
    import oracle as O
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    grads, ws, bs, x, y = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    dims = [16, 32, 8]
    h = O.lib().orc_mlp_create(0, 2, O.u32s(dims), 24, 24, 1e-3, 0.9, 0.999, 1e-8)
    for l in range(2):
        O.call("orc_mlp_params", h, l, O.ptr(ws[l]), O.ptr(bs[l]), 0)
    O.call("orc_mlp_step", h, O.ptr(x), O.ptr(y), None, 1)
    k = 0
    for l in range(2):
        gw = np.empty(dims[l + 1] * dims[l], np.float32)
        gb = np.empty(dims[l + 1], np.float32)
        O.call("orc_mlp_grads", h, l, O.ptr(gw), O.ptr(gb))
        for want in (gw, gb):
            got = grads[k]
            k += 1
            assert np.max(np.abs(got - want)) <= 1e-5 * max(1e-3, np.max(np.abs(want)))
    O.lib().orc_mlp_destroy(h)
