"""Tensor-parallel linear layers on 2 GPUs (one process each, NCCL): column-parallel (N split, token
all-gather) and row-parallel (K split, reduce-scatter) against the same layer on one GPU.
Needs two B200s; skipped otherwise (the round-end GPU run has one). NVLS is off (NCCL_NVLS_ENABLE=0)."""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, errq):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from conftest import load_package
        from oracle import oracle as O

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        we = load_package()
        par = we.parallel
        g = we.Graph(rank)
        st = torch.cuda.Stream(device=dev)
        torch.cuda.set_stream(st)
        g.set_stream(st.cuda_stream)
        tp = par.TensorParallel()

        def mm(x, shard, m):
            w = torch.from_numpy(shard.weight).to(dev)
            cs = None if shard.chan_scale is None else torch.from_numpy(shard.chan_scale).to(dev)
            gs = None if shard.group_scale is None else torch.from_numpy(shard.group_scale.view(np.int16)).to(dev)
            b = None if shard.bias is None else torch.from_numpy(shard.bias).to(dev)
            y = torch.empty(m, shard.n, dtype=torch.float32, device=dev)
            we.kernels.matmul(g, x, w, y, m, shard.n, shard.k, shard.scale, x_dtype="bf16", w_dtype=shard.dtype,
                              chan_scale=cs, group_scale=gs, bias=b)
            return y

        t, k, n = 1024, 3072, 1536
        rng = np.random.default_rng(0)
        xh = O.bf16_round(rng.standard_normal(t * k).astype(np.float32)).reshape(t, k)
        wf = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
        q, s = O.quant_fp8_channel(wf, n, k)
        bias = rng.standard_normal(n).astype(np.float32)
        x = torch.from_numpy(xh).to(dev).to(torch.bfloat16)
        full = mm(x, par.Shard(q, "fp8", n, k, chan_scale=s), t) + torch.from_numpy(bias).to(dev)

        tb, te = par.split_range(t, world, rank)
        nb, ne = par.split_range(n, world, rank)
        y = tp.column_linear(mm, x[tb:te].contiguous(), par.shard_column(q, "fp8", n, k, world, rank, chan_scale=s,
                                                                           bias=bias))
        err = (y - full[:, nb:ne]).abs().max().item() / full.abs().max().item()
        assert err < 1e-5, ("column", err)
        kb, ke = par.split_range(k, world, rank, 16)
        y = tp.row_linear(mm, x[:, kb:ke].contiguous(), par.shard_row(q, "fp8", n, k, world, rank, chan_scale=s),
                          bias=torch.from_numpy(bias).to(dev))
        err = (y - full[tb:te]).abs().max().item() / full.abs().max().item()
        assert err < 1e-5, ("row", err)
        assert g.device_error() == 0
        g.destroy()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # noqa: BLE001
        errq.put(f"rank {rank}: {type(exc).__name__}: {exc}")
        raise


def test_tensor_parallel_linear_on_two_gpus():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp = torch.multiprocessing.get_context("spawn")
    errq = mp.SimpleQueue()
    world, port = 2, _free_port()
    procs = [mp.Process(target=_rank_main, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive and not errors and all(p.exitcode == 0 for p in procs), errors
