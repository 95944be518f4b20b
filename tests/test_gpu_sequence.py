"""Sequence parallelism of one image's step on 2, 4 or 8 GPUs (one process each): every rank runs the blocks on
its share of the rows, attention exchanges heads all-to-all, through peer memory or NCCL (we_all_to_all), both on the
library's communicator (comm.Comm); the velocity must equal the one-GPU step's. Peer memory in two forms: "fused",
the kernels that produce q, k and v store them straight into the attending ranks' regions (the q/k/v GEMM's epilogue
for v, we_qknorm_rope_peers for q and k) and a flag barrier follows; "copy", one exchange kernel copies them after
their producers (we_peer_exchange). 80 tokens (8 text + 72 image), so rank 0's shard holds text and image rows and the others
image rows only. The peer case also checks the exchange itself bit for bit: scattering each rank's q rows and
gathering them back through an identity "attention" returns them unchanged, and every rank receives exactly its
heads of every rank's rows. Skipped when fewer GPUs are visible. NVLS is off (NCCL_NVLS_ENABLE=0)."""
import os
import sys

import numpy as np
import pytest

from test_gpu_multi import gpu_count, run_ranks

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank_main(rank, world, port, errq, mode):
    peer = mode != "nccl"
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        from conftest import load_package
        from util import bf16, bf16_round, make_step, randn

        we = load_package()
        g = we.Graph(rank)
        uid = we.comm.rendezvous(rank, world, "127.0.0.1", port)
        comm = we.comm.Comm(g, rank, world, uid, timeout_ms=60000)
        T = we.transformer
        heads, kvh = (4, 2) if world == 2 else (world, world)  # GQA where the heads split over the ranks
        bc = we.blocks.BlockConfig(hidden=heads * 128, mlp=heads * 512, heads=heads, kv_heads=kvh, head_dim=128,
                                   mlp_act="gelu", attn_gate=False)
        scfg = T.StepConfig(block=bc, double=1, single=2, ctx_dim=256)
        h, w, text = 16, 18, 8
        _, wts = make_step(we, g, scfg, 1200, per_channel=True)  # same seeds on every rank: the same model
        lat, ctx = bf16_round(randn(16 * h * w, 1201)), bf16_round(randn(text * 256, 1202))
        inp = T.StepInputs(g.buffer(bf16(lat)), h, w, 0.37, g.buffer(bf16(ctx)), text)
        v1, _ = T.transformer(g, wts, scfg, inp, dtype="bf16")
        one = g.read(v1, 16 * h * w * 4, np.float32).copy()
        sp = we.sequence.SequenceParallel(comm, peer=peer, fused=mode == "fused")
        v2, _ = T.transformer(g, wts, scfg, inp, dtype="bf16", sp=sp)
        got = g.read(v2, 16 * h * w * 4, np.float32).copy()
        err = float(np.max(np.abs(got - one)) / np.max(np.abs(one)))
        assert err < 1e-6, ("sequence-parallel step differs from the one-GPU step", err)
        if peer:  # the same shard's blocks replayed from a CUDA graph: bit for bit the eager sequence-parallel step
            sgr = T.StepGraph(g, wts, scfg, h, w, text, dtype="bf16", sp=sp)
            v3, _ = T.transformer(g, wts, scfg, inp, dtype="bf16", sp=sp, captured=sgr)
            v3, _ = T.transformer(g, wts, scfg, inp, dtype="bf16", sp=sp, captured=sgr)  # a second replay
            assert np.array_equal(g.read(v3, 16 * h * w * 4, np.float32), got), "captured SP step differs"
            sgr.destroy()
        if peer:  # the exchange alone, bit for bit
            t, heads, kvh, hb = 40, 2 * world, world, 256
            rows = [np.random.default_rng(70 + r).integers(0, 65536, t * heads * 128, dtype=np.uint16)
                    for r in range(world)]
            kv = [np.random.default_rng(80 + r).integers(0, 65536, t * kvh * 128, dtype=np.uint16)
                  for r in range(world)]
            qb, kb = g.buffer(rows[rank]), g.buffer(kv[rank])
            seen = {}

            def identity(qh, kh, vh, oh):  # copies the received q block into the output
                seen["q"] = g.read(qh, world * t * heads // world * hb, np.uint16).copy()
                seen["k"] = g.read(kh, world * t * kvh // world * hb, np.uint16).copy()
                g.copy(qh, 0, oh, 0, world * t * heads // world * hb)

            o = sp.exchange_heads(g, qb, kb, kb, t, heads, kvh, hb, identity)
            back = g.read(o, t * heads * hb, np.uint16)
            assert np.array_equal(back, rows[rank]), "scatter + gather did not return the rows"
            hl, kl = heads // world, kvh // world
            want_q = np.concatenate([x.reshape(t, heads, 128)[:, rank * hl:(rank + 1) * hl] for x in rows]).ravel()
            want_k = np.concatenate([x.reshape(t, kvh, 128)[:, rank * kl:(rank + 1) * kl] for x in kv]).ravel()
            assert np.array_equal(seen["q"], want_q) and np.array_equal(seen["k"], want_k)
        assert g.device_error() == 0
        sp.destroy()
        comm.barrier()
        comm.destroy()
        g.destroy()
    except BaseException as exc:  # noqa: BLE001
        errq.put(f"rank {rank}: {type(exc).__name__}: {exc}")
        raise


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["fused", "copy", "nccl"])
def test_sequence_parallel_step(mode, world):
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    run_ranks(_rank_main, world, mode)
