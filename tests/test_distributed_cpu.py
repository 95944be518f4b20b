"""Host logic of the multi-GPU path on CPU ranks: world_size 2 over gloo, 127.0.0.1.

The tensor-parallel choreography (web-engine_b200/parallel.py) runs with the float64 oracle as the
per-rank matmul, so the sharding of fp8 (per-channel scales) and int4 group-64 weights, the token
all-gather, the reduce-scatter and the single bias add are checked against the unsharded layer. The
collectives go through GlooComm, a test adapter with the interface of the library's communicator
(comm.Comm: all_gather / reduce_scatter on buffers) over torch.distributed's gloo backend; on GPUs the
same code runs on the library's NCCL communicator (tests/test_gpu_multi.py).
"""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, errq):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from conftest import load_package
        from oracle import oracle as O

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        we = load_package()
        par = we.parallel

        class GlooComm:
            """comm.Comm's collective interface on host numpy buffers (uint8 views), over gloo."""

            def __init__(self):
                self.rank, self.world = dist.get_rank(), dist.get_world_size()

            def all_gather(self, src, dst, nbytes):
                out = torch.from_numpy(dst.view(np.uint8)[:self.world * nbytes])
                dist.all_gather_into_tensor(out, torch.from_numpy(src.view(np.uint8)[:nbytes].copy()))

            def reduce_scatter(self, src, dst, count, dtype="f32"):
                assert dtype == "f32"
                parts = list(torch.from_numpy(src.view(np.float32)[:self.world * count].copy()).chunk(self.world))
                out = torch.empty(count, dtype=torch.float32)
                dist.reduce_scatter(out, parts)
                dst.view(np.float32)[:count] = out.numpy()

        tp = par.TensorParallel(GlooComm(), lambda nbytes: np.zeros(nbytes, np.uint8))

        def mm(x, shard, m):
            fmt = {"fp8": O.FP8, "int4": O.INT4G64, "bf16": O.BF16}[shard.dtype]
            y = O.matmul(x.view(np.float32)[:m * shard.k], fmt, shard.weight, m, shard.n, shard.k, scale=shard.scale,
                         chan_scale=shard.chan_scale, gscale=shard.group_scale)
            y = y.reshape(m, shard.n)
            if shard.bias is not None:
                y = y + shard.bias
            return np.ascontiguousarray(y, np.float32).view(np.uint8).ravel()

        def add_bias(y, bias, rows, n):
            return (y.view(np.float32)[:rows * n].reshape(rows, n) + bias).astype(np.float32).view(np.uint8).ravel()

        t, k, n = 8, 256, 96
        rng = np.random.default_rng(0)  # same data on every rank
        x = O.bf16_round(rng.standard_normal(t * k).astype(np.float32)).reshape(t, k)
        wf = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
        q, s = O.quant_fp8_channel(wf, n, k)
        p4, g4 = O.quant_int4_g64(wf, n, k)
        bias = rng.standard_normal(n).astype(np.float32)
        full8 = O.matmul(x.ravel(), O.FP8, q, t, n, k, chan_scale=s).reshape(t, n)
        full4 = O.matmul(x.ravel(), O.INT4G64, p4, t, n, k, gscale=g4).reshape(t, n)

        # column-parallel: token shard in, this rank's output channels out
        tb, te = par.split_range(t, world, rank)
        sh = par.shard_column(q, "fp8", n, k, world, rank, chan_scale=s, bias=bias)
        xl = np.ascontiguousarray(x[tb:te], np.float32).view(np.uint8).ravel()
        y = tp.column_linear(mm, xl, te - tb, k * 4, sh).view(np.float32).reshape(t, -1)
        nb, ne = par.split_range(n, world, rank)
        assert y.shape == (t, ne - nb)
        np.testing.assert_allclose(y, (full8 + bias)[:, nb:ne], rtol=1e-6, atol=1e-5)

        # row-parallel: K slice of activations and weights, reduce-scattered over tokens, bias added once
        for dtype, w, scales, gsc, full in (("fp8", q, s, None, full8), ("int4", p4, None, g4, full4)):
            sh = par.shard_row(w, dtype, n, k, world, rank, chan_scale=scales, group_scale=gsc)
            kb, ke = par.split_range(k, world, rank, 64 if dtype == "int4" else 16)
            assert sh.k == ke - kb
            xc = np.ascontiguousarray(x[:, kb:ke], np.float32).view(np.uint8).ravel()
            y = tp.row_linear(mm, xc, t, sh, bias=bias, add_bias=add_bias).view(np.float32).reshape(-1, n)
            np.testing.assert_allclose(y, (full + bias)[tb:te], rtol=1e-5, atol=1e-5)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # noqa: BLE001
        errq.put(f"rank {rank}: {type(exc).__name__}: {exc}")
        raise


def test_tensor_parallel_host_logic_on_two_gloo_ranks():
    torch = pytest.importorskip("torch")
    mp = torch.multiprocessing.get_context("spawn")
    errq = mp.SimpleQueue()
    world, port = 2, _free_port()
    procs = [mp.Process(target=_rank_main, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive and not errors and all(p.exitcode == 0 for p in procs), errors


def test_split_range_partitions():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import load_package

    par = load_package().parallel
    for total, world, align in [(12288, 8, 1), (3072, 8, 64), (24, 8, 1), (100, 3, 1), (3072, 3, 64)]:
        parts = [par.split_range(total, world, r, align) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        assert all((e - b) % align == 0 for b, e in parts)
    with pytest.raises(ValueError):
        par.split_range(100, 2, 0, 64)


def _rdv_main(rank, world, port, out):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import load_package

    we = load_package()
    out.put((rank, we.comm.rendezvous(rank, world, "127.0.0.1", port, payload=b"id-" + bytes(range(125)) if rank == 0
                                      else None, timeout_s=30)))


def test_rendezvous_carries_the_unique_id_to_every_rank():
    """comm.rendezvous (plain TCP, no GPU): rank 0's 128-byte payload reaches the other ranks."""
    import multiprocessing

    mp = multiprocessing.get_context("spawn")
    out = mp.SimpleQueue()
    world, port = 3, _free_port()
    procs = [mp.Process(target=_rdv_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    got = {}
    while not out.empty():
        r, v = out.get()
        got[r] = v
    assert all(p.exitcode == 0 for p in procs)
    assert set(got) == {0, 1, 2} and all(v == b"id-" + bytes(range(125)) for v in got.values())


def test_parallel_and_sequence_import_no_torch():
    """The multi-GPU product modules run on the library's communicator: importing them pulls in no torch."""
    code = ("import sys; sys.modules['torch'] = None; sys.path.insert(0, %r); sys.path.insert(0, %r); "
            "from conftest import load_package; we = load_package(); import web_engine_b200.parallel, "
            "web_engine_b200.sequence, web_engine_b200.comm; print('ok')") % (ROOT, os.path.join(ROOT, "tests"))
    import subprocess

    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr
