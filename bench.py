#!/usr/bin/env python
"""Benchmark of the hot path: the dequant-GEMM of BASELINE config 2 (M=4608 tokens, K=3072,
N=12288; bf16 activations, fp8 e4m3 weights with per-output-channel scales) on B200.

One step = one linear layer forward through the public operator API (ops.linear -> activation
split + tcgen05 GEMM) on one batch of synthetic inputs that are already resident in HBM. L2 is
flushed between timed steps (256 MB write, then read back so no dirty lines remain), outside the
timed events. Multi-GPU: one process per
GPU (torchrun), each rank runs its own batch (data-parallel images, no data-path collective:
weak scaling); time = max over ranks of the summed per-step CUDA-event time.

Also reported on the same line: the GEMM kernel alone (roofline), the one-term fp8 mode and the
int4 group-64 variant, an end-to-end number with host buffers (pinned H2D of x, D2H of y inside
the timed region), SM clocks sampled during the timed region, and (rank 0, N=1) the CPU oracle on a
bounded sample. ``--impl reference`` times the reference's CPU path instead: the reference is
TypeScript (no Node here), so its arm is the C restatement of its float64 matmul reference
(oracle/), run on all host threads.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
M, K, N = 4608, 3072, 12288
FLOPS = 2.0 * M * N * K
METRIC = "dequant-GEMM TFLOPS (config 2: M=4608 K=3072 N=12288, bf16 x fp8 e4m3 per-channel)"


def load_package():
    pkg_dir = os.path.join(ROOT, "web-engine_b200")
    spec = importlib.util.spec_from_file_location("web_engine_b200", os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["web_engine_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks() -> dict:
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "fallback": True}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons of one GPU every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self) -> dict:
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": float(rows[0][2]), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()) if rows else None,
                "reasons": sorted(reasons)}


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _oracle_sample(O, np, rows: int, threads: int):
    """One timed float64 oracle matmul over `rows` rows of config 2 (the reference tests' CPU matmul)."""
    rng = np.random.default_rng(0)
    w = rng.integers(0, 256, N * K, dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0
    cs = np.full(N, 0.002, np.float32)
    x = O.bf16_round(rng.standard_normal(rows * K, dtype=np.float32))
    t0 = time.perf_counter()
    O.matmul(x, O.FP8, w, rows, N, K, chan_scale=cs, threads=threads)
    return time.perf_counter() - t0


def _calibrate_rows(O, np, threads: int, target_s: float) -> int:
    """Rows of config 2 whose oracle matmul takes about target_s on `threads` threads (untimed calibration)."""
    rows, dt = 2, 0.0
    while rows < M:
        dt = _oracle_sample(O, np, rows, threads)
        if dt > target_s / 2:
            break
        rows = min(M, max(rows * 2, int(rows * target_s / max(dt, 1e-3))))
    return rows


def cpu_baseline(threads: int | None, target_s: float = 12.0) -> dict:
    """The oracle's float64 matmul (the reference tests' CPU reference) on a bounded row sample of config 2, on all
    host threads (OpenMP) and on one thread (the reference runs in one JS thread)."""
    sys.path.insert(0, ROOT)
    import numpy as np

    from oracle import oracle as O  # the CPU baseline leg: the checker timed as the reference's CPU path

    nthreads = threads or os.cpu_count() or 1
    rows = _calibrate_rows(O, np, nthreads, target_s)
    dt = _oracle_sample(O, np, rows, nthreads)
    rows1 = max(2, rows // nthreads)
    dt1 = _oracle_sample(O, np, rows1, 1)
    return {"value": 2.0 * rows * N * K / dt / 1e12, "unit": "TFLOPS", "cores": nthreads, "kind": "port",
            "sample": f"{rows} of {M} rows of config 2 (float64 oracle, OpenMP {nthreads} threads), {dt:.1f} s",
            "single_thread": {"value": 2.0 * rows1 * N * K / dt1 / 1e12, "unit": "TFLOPS", "cores": 1,
                              "sample": f"{rows1} rows, {dt1:.2f} s"},
            "cpu_model": _cpu_model(), "nproc": os.cpu_count()}


def run_reference(args, rank: int) -> None:
    """The reference arm: every step is one real float64 oracle matmul over a fixed sample of config 2's rows (sized
    once, untimed, so that warm-up + steps take about a minute), timed step by step; ms_per_step is that measured
    time, value the sample's FLOPs over it."""
    if rank != 0:
        return
    sys.path.insert(0, ROOT)
    import numpy as np

    from oracle import oracle as O  # the reference arm: the reference's CPU path as restated in oracle/

    threads = os.cpu_count() or 1
    per_step_s = max(0.5, 60.0 / max(1, args.steps + args.warmup))
    rows = _calibrate_rows(O, np, threads, per_step_s)
    times = []
    for i in range(args.warmup + args.steps):
        dt = _oracle_sample(O, np, rows, threads)
        if i >= args.warmup:
            times.append(dt)
    times.sort()
    med = times[len(times) // 2]
    value = 2.0 * rows * N * K / med / 1e12
    rows1 = max(2, rows // threads)
    dt1 = _oracle_sample(O, np, rows1, 1)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": med * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": config_dict(args),
            "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": "port",
                             "sample": f"each step: {rows} of {M} rows of config 2 (float64 oracle, OpenMP "
                                       f"{threads} threads), median of {args.steps} timed steps",
                             "single_thread": {"value": 2.0 * rows1 * N * K / dt1 / 1e12, "unit": "TFLOPS",
                                               "cores": 1, "sample": f"{rows1} rows, {dt1:.2f} s"},
                             "cpu_model": _cpu_model(), "nproc": os.cpu_count()},
            "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "rows_per_step": rows, "step_s": times,
            "note": "the reference path is TypeScript/WGSL (no Node or WebGPU on this box); this arm is the C "
                    "restatement of its float64 CPU matmul reference (tests/gpu/matmul.test.ts:26-35); a step is "
                    "that matmul over rows_per_step rows of config 2, so ms_per_step is the measured time of the "
                    "sample, not an extrapolation to all 4608 rows"}
    print(json.dumps(line), flush=True)


def random_linear(we, g, torch, dev, gen, n: int, k: int):
    """fp8 e4m3 weights ~N(0, 0.02) with per-output-channel absmax scales (config 1's weight recipe)."""
    w32 = torch.randn(n, k, generator=gen, device=dev) * 0.02
    q = torch.empty(n, k, dtype=torch.uint8, device=dev)
    s = torch.empty(n, dtype=torch.float32, device=dev)
    we.kernels.quantize_fp8(g, w32, n, k, q, s, per_channel=True, w_dtype="f32")
    return we.Linear(q, "fp8", 1.0, n, k, chan_scale=s)


def random_block(we, g, torch, dev, gen, bc):
    """One block's random weights: fp8 linears, norm weights ~N(0, 0.5), modulation table ~N(0, 0.3)."""
    hid, hd = bc.hidden, bc.head_dim
    lin = {"wq": (bc.heads * hd, hid), "wk": (bc.kv_heads * hd, hid), "wv": (bc.kv_heads * hd, hid),
           "wo": (hid, hid), "mlp_up": (bc.mlp, hid), "mlp_down": (hid, bc.mlp)}
    if bc.attn_gate:
        lin["gate"] = (hid, hid)
    if bc.mlp_act == "swiglu":
        lin["mlp_gate"] = (bc.mlp, hid)
    w = {name: random_linear(we, g, torch, dev, gen, n, k) for name, (n, k) in lin.items()}
    for name, d, std in (("norm1", hid, 0.5), ("norm2", hid, 0.5), ("norm_q", hd, 0.5), ("norm_k", hd, 0.5),
                         ("table", 6 * hid, 0.3)):
        w[name] = torch.randn(d, generator=gen, device=dev) * std
    return we.blocks.fuse_qkv(g, we.blocks.BlockWeights(**w))


def random_model(we, g, torch, dev, gen, scfg):
    """Config 4's model: `double` two-stream and `single` one-stream blocks plus the edge linears."""
    bc, hid, ch = scfg.block, scfg.block.hidden, scfg.channels
    edge = {name: random_linear(we, g, torch, dev, gen, n, k) for name, (n, k) in
            (("first", (hid, 4 * ch)), ("tmlp0", (hid, scfg.time_dim)), ("tmlp2", (hid, hid)),
             ("tproj", (6 * hid, hid)), ("txt_in", (hid, scfg.ctx_dim)), ("last_linear", (4 * ch, hid)))}
    double = [(random_block(we, g, torch, dev, gen, bc), random_block(we, g, torch, dev, gen, bc))
              for _ in range(scfg.double)]
    single = [random_block(we, g, torch, dev, gen, bc) for _ in range(scfg.single)]
    vec = {name: torch.randn(hid, generator=gen, device=dev) * 0.3 for name in ("last_norm", "last_scale", "last_shift")}
    return we.transformer.TransformerWeights(double=double, single=single, **edge, **vec)


def bench_model(we, g, torch, dev, gen, timed, interleaved, steps: int, bf16_peak: float, world: int = 1,
                gpu: int = 0, step_ms=None) -> dict:
    """Config 3 (one single-stream block, 4608 tokens) and config 4 (one denoising step of the 19 + 38 block
    model at 1024x1024: 512 text + 4096 image tokens), bf16 path, weights resident, inputs ~N(0, 1)."""
    T = we.transformer
    scfg = T.StepConfig()
    bc, text_tokens, side = scfg.block, 512, 128
    rows, cols = T.patch_grid(side, side)
    tokens = text_tokens + rows * cols
    out = {}
    # config 3: one block
    bw = random_block(we, g, torch, dev, gen, bc)
    xb = torch.randn(tokens, bc.hidden, generator=gen, device=dev)
    tvec = torch.randn(6 * bc.hidden, generator=gen, device=dev) * 0.3
    cos_h, sin_h, pairs = we.kernels.rope_tables(we.kernels.positions(text_tokens, rows, cols), scfg.axes, scfg.theta)
    rope = we.Rope(torch.from_numpy(cos_h).to(dev), torch.from_numpy(sin_h).to(dev), pairs, tokens)

    def step_block():
        mark = g.mark()
        we.blocks.block(g, bw, bc, xb, tvec, rope, dtype="bf16")
        g.release(mark)

    l0 = g.stats["launches"]
    with ClockSampler(gpu) as blk_clocks:
        blk_ms = timed(step_block, steps, 3) / steps
    blk_launches = (g.stats["launches"] - l0) // (steps + 3)
    bf = we.blocks.block_flops(bc, tokens)
    out["block_config3"] = {"ms": blk_ms, "tflops": bf["total"] / (blk_ms * 1e-3) / 1e12,
                            "frac_bf16_peak": bf["total"] / (blk_ms * 1e-3) / 1e12 / bf16_peak,
                            "flop": bf["total"], "launches_per_block": blk_launches, "clocks": blk_clocks.summary(),
                            "note": "one single-stream block, 4608 tokens, hidden 3072, 24x128 heads, 4x GELU MLP, "
                                    "fp8 per-channel linears, bf16 activations, f32 residual"}
    del bw, xb
    # config 4: one whole denoising step
    model = random_model(we, g, torch, dev, gen, scfg)
    lat = torch.randn(scfg.channels, side, side, generator=gen, device=dev).to(torch.bfloat16)
    ctx = torch.randn(text_tokens, scfg.ctx_dim, generator=gen, device=dev).to(torch.bfloat16)
    vel = torch.empty(scfg.channels, side, side, dtype=torch.float32, device=dev)
    inp = T.StepInputs(lat, side, side, 0.7, ctx, text_tokens)

    def step_model():
        T.transformer(g, model, scfg, inp, dtype="bf16", velocity=vel)

    ksteps = max(3, steps // 4)
    l0 = g.stats["launches"]
    with ClockSampler(gpu) as st_clocks:
        st_ms = timed(step_model, ksteps, 3) / ksteps
    st_launches = (g.stats["launches"] - l0) // (ksteps + 3)
    sf = T.step_flops(scfg, text_tokens, rows * cols)
    assert torch.isfinite(vel).all().item(), "non-finite velocity"
    # end to end: latent + context from pinned host memory, velocity back to pinned host memory
    lat_h, ctx_h = lat.cpu().pin_memory(), ctx.cpu().pin_memory()
    vel_h = torch.empty(scfg.channels, side, side, dtype=torch.float32).pin_memory()
    lat_d, ctx_d = torch.empty_like(lat), torch.empty_like(ctx)
    inp_e = T.StepInputs(lat_d, side, side, 0.7, ctx_d, text_tokens)

    def step_e2e():
        lat_d.copy_(lat_h, non_blocking=True)
        ctx_d.copy_(ctx_h, non_blocking=True)
        T.transformer(g, model, scfg, inp_e, dtype="bf16", velocity=vel)
        g.read_into(vel, vel_h.data_ptr(), vel.numel() * 4)

    # the same step with its 57 blocks replayed from a CUDA graph (one launch from the host instead of ~1000)
    sgr = T.StepGraph(g, model, scfg, side, side, text_tokens, dtype="bf16")

    def step_graph():
        T.transformer(g, model, scfg, inp, dtype="bf16", velocity=vel, captured=sgr)

    def step_graph_e2e():
        lat_d.copy_(lat_h, non_blocking=True)
        ctx_d.copy_(ctx_h, non_blocking=True)
        T.transformer(g, model, scfg, inp_e, dtype="bf16", velocity=vel, captured=sgr)
        g.read_into(vel, vel_h.data_ptr(), vel.numel() * 4)

    # the four ways of running the step take turns, so that the power cap's clock drift falls on all of them
    with ClockSampler(gpu) as e2e_clocks:
        med = interleaved({"eager": step_model, "eager_e2e": step_e2e, "graph": step_graph,
                           "graph_e2e": step_graph_e2e}, ksteps, 2)
    e2e_ms, gr_ms, gr_e2e_ms = med["eager_e2e"], med["graph"], med["graph_e2e"]
    issue = {}
    for name, fn in (("eager", step_model), ("graph", step_graph)):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fn()
        issue[name] = (time.perf_counter() - t0) * 1e3
        torch.cuda.synchronize()
    sgr.destroy()
    out["step_config4"] = {"ms": st_ms, "tflops": sf["total"] / (st_ms * 1e-3) / 1e12,
                           "frac_bf16_peak": sf["total"] / (st_ms * 1e-3) / 1e12 / bf16_peak, "flop": sf["total"],
                           "launches_per_step": st_launches, "e2e_ms": e2e_ms, "clocks": st_clocks.summary(),
                           "graph_ms": gr_ms, "graph_e2e_ms": gr_e2e_ms, "host_issue_ms": issue,
                           "interleaved_median_ms": med, "e2e_clocks": e2e_clocks.summary(),
                           "e2e_h2d_bytes": lat.numel() * 2 + ctx.numel() * 2, "e2e_d2h_bytes": vel.numel() * 4,
                           "note": "19 double + 38 single blocks of config 3 shape, 512 text + 4096 image tokens "
                                   "(1024x1024), random fp8 per-channel weights resident (8.6 GB), bf16 latent/context"}
    # config 4's one image split over all ranks: sequence parallelism (rows sharded, heads exchanged by all-to-all)
    if world > 1:
        # the library's NCCL communicator (C ABI); its unique id travels over the bench's own process group
        import torch.distributed as dist

        uid = [we.comm.unique_id() if dist.get_rank() == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = we.comm.Comm(g, dist.get_rank(), world, uid[0], timeout_ms=120000)
        sp = we.sequence.SequenceParallel(comm)  # the peer-memory exchange kernel
        sp_nccl = we.sequence.SequenceParallel(comm, peer=False)

        def step_sp():
            T.transformer(g, model, scfg, inp, dtype="bf16", velocity=vel, sp=sp)

        def step_sp_nccl():
            T.transformer(g, model, scfg, inp, dtype="bf16", velocity=vel, sp=sp_nccl)

        sp_steps = max(6, steps // 2)
        with ClockSampler(gpu) as sp_clocks:
            sp_ms = timed(step_sp, sp_steps, 3) / sp_steps
        per = sorted(step_ms or [sp_ms])
        l0 = g.stats["launches"]
        step_sp()
        sp_launches = g.stats["launches"] - l0
        nccl_ms = timed(step_sp_nccl, sp_steps, 2) / sp_steps
        sgr_sp = T.StepGraph(g, model, scfg, side, side, text_tokens, dtype="bf16", sp=sp)

        def step_sp_graph():
            T.transformer(g, model, scfg, inp, dtype="bf16", velocity=vel, sp=sp, captured=sgr_sp)

        sp_graph_ms = timed(step_sp_graph, sp_steps, 2) / sp_steps
        sgr_sp.destroy()
        # the same with the q/k/v scatter fused into its producers' stores (no copy kernel after them)
        sp_fused = we.sequence.SequenceParallel(comm, fused=True)
        sgr_fu = T.StepGraph(g, model, scfg, side, side, text_tokens, dtype="bf16", sp=sp_fused)

        def step_fused_graph():
            T.transformer(g, model, scfg, inp, dtype="bf16", velocity=vel, sp=sp_fused, captured=sgr_fu)

        sp_fused_graph_ms = timed(step_fused_graph, sp_steps, 2) / sp_steps
        sgr_fu.destroy()
        sp_fused.destroy()
        sp.destroy()
        sp_nccl.destroy()
        # the same image split by tensor parallelism: every block's linears sharded over the ranks (N / K splits),
        # activations all-gathered and partial sums reduce-scattered on the same communicator
        tp_model = we.parallel.shard_model(g, model, scfg, world, dist.get_rank())
        tpg = we.parallel.TPGroup(comm)

        def step_tp():
            T.transformer(g, tp_model, scfg, inp, dtype="bf16", velocity=vel, tp=tpg)

        with ClockSampler(gpu) as tp_clocks:
            tp_ms = timed(step_tp, sp_steps, 2) / sp_steps
        del tp_model
        comm.destroy()
        out["step_config4_sequence_parallel"] = {
            "ms": sp_ms, "median_ms_this_rank": per[len(per) // 2], "steps": sp_steps, "n_gpus": world,
            "one_gpu_ms": st_ms, "tflops": sf["total"] / (sp_ms * 1e-3) / 1e12, "launches_per_step": sp_launches,
            "graph_ms": sp_graph_ms, "graph_ms_fused_exchange": sp_fused_graph_ms, "nccl_all_to_all_ms": nccl_ms,
            "clocks": sp_clocks.summary(),
            "tensor_parallel_ms": tp_ms, "tensor_parallel_clocks": tp_clocks.summary(),
            "note": "one 1024x1024 image's step over all GPUs: every rank runs the blocks on 4608 / n_gpus rows; "
                    "q/k/v go to the ranks attending their heads and o comes back through the peer-memory exchange "
                    "kernel (IPC-mapped HBM of every GPU, one kernel per exchange with a flag barrier); graph_ms: this "
                    "rank's blocks replayed from a CUDA graph; graph_ms_fused_exchange: the same with q/k/v stored "
                    "into the attending ranks' memory by the kernels that produce them (the q/k/v GEMM's epilogue "
                    "for v, q/k norm + RoPE for q and k) and a flag barrier instead of the copy; "
                    "nccl_all_to_all_ms: the same step with NCCL "
                    "all-to-all (we_all_to_all); tensor_parallel_ms: the same image by tensor parallelism (eager): "
                    "q/k/v and MLP up split over the ranks' heads and columns, wo and MLP down over K, the split "
                    "activations all-gathered and the f32 partial sums reduce-scattered (NCCL through the C ABI)"}

    # config 5's batch: 8 images per step in total, split data-parallel across the ranks (no collective); each
    # rank runs its share as one token stream (every linear one GEMM over all its images' rows)
    per = max(1, 8 // world)
    lats = [torch.randn(scfg.channels, side, side, generator=gen, device=dev).to(torch.bfloat16) for _ in range(per)]
    ctxs = [torch.randn(text_tokens, scfg.ctx_dim, generator=gen, device=dev).to(torch.bfloat16) for _ in range(per)]
    vels = [torch.empty(scfg.channels, side, side, dtype=torch.float32, device=dev) for _ in range(per)]
    binp = [T.StepInputs(l_, side, side, 0.7, c_, text_tokens) for l_, c_ in zip(lats, ctxs)]

    def step_batch():
        T.transformer(g, model, scfg, binp, dtype="bf16", velocity=vels)

    # config 5 as specified: 4-step turbo sampling (sigmas(4)) of the batch from seeded noise, the f32 latents
    # updated by the device Euler step; weights resident, and (one GPU) streamed from pinned host memory per block
    noise = [torch.randn(scfg.channels, side, side, generator=gen, device=dev) for _ in range(per)]
    ctx_b = list(ctxs)

    def sample4(streamed=None):
        def run():
            mark = g.mark()
            T.sample(g, model, scfg, noise, ctx_b, side, side, text_tokens, steps=4, dtype="bf16", streamed=streamed)
            g.release(mark)
        return run

    fns = {"step": step_batch, "sample4_resident": sample4()}
    streamed = None
    if world == 1:
        streamed = T.StreamedBlocks(g, model, slots=3)
        fns["sample4_streamed"] = sample4(streamed)
    with ClockSampler(gpu) as b_clocks:
        med = interleaved(fns, 2, 1)
    b_ms = med["step"]
    out["batch8_config5"] = {"ms_per_step": b_ms, "images_per_s": world * per / (b_ms * 1e-3),
                             "images_per_rank": per, "tflops": world * per * sf["total"] / (b_ms * 1e-3) / 1e12,
                             "clocks": b_clocks.summary(),
                             "scaling": "strong: 8 images per step in total, 8 / n_gpus per rank",
                             "note": "one denoising step of config 4's model on a batch of 1024x1024 images, "
                                     "data-parallel over images, weights resident; median of runs taking turns with "
                                     "the sampling runs below"}
    s4 = {"sample_ms": med["sample4_resident"], "steps": 4, "images_per_rank": per,
          "images_per_s": world * per / (med["sample4_resident"] * 1e-3),
          "note": "config 5: 4 Euler steps (sigmas(4), mu 1.15) of 8 images in total at 1024x1024, 8 / n_gpus per "
                  "rank as one token stream, text rows cached after the first step; runs take turns with the step "
                  "above (median of 2), clocks in batch8_config5"}
    if streamed is not None:
        s4["streamed_sample_ms"] = med["sample4_streamed"]
        s4["overlap_efficiency"] = med["sample4_resident"] / med["sample4_streamed"]
        s4["streamed_host_bytes_per_step"] = streamed.host_bytes
        s4["streamed_h2d_gbs"] = streamed.host_bytes * 4 / (med["sample4_streamed"] * 1e-3) / 1e9
        s4["streamed_note"] = ("every block's fp8 linears (8.6 GB per step) copied from pinned host memory into 3 "
                               "device slots on a side stream, one layer ahead of the block that uses it")
        streamed.close()
    out["sample4_batch8_config5"] = s4
    del model, lats, ctxs, vels
    torch.cuda.empty_cache()
    return out


def numa_local_cpus(torch, local: int) -> dict:
    """Bind this process to the CPUs of its GPU's NUMA node (sysfs local_cpulist of the GPU's PCI function), so that
    the pinned host buffers it allocates afterwards (first touch) sit in that node's memory and its DMA does not
    cross sockets. Returns what was done, for the bench line."""
    try:
        p = torch.cuda.get_device_properties(local)
        dev = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        base = f"/sys/bus/pci/devices/{dev}"
        node = int(open(f"{base}/numa_node").read().strip())
        cpus = set()
        for part in open(f"{base}/local_cpulist").read().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return {"numa_node": node, "bound": False, "why": "no allowed CPU on the GPU's node", "pci": dev}
        os.sched_setaffinity(0, cpus)
        return {"numa_node": node, "bound": True, "cpus": len(cpus), "pci": dev}
    except Exception as exc:  # noqa: BLE001 - a host without the sysfs entries keeps its affinity
        return {"bound": False, "why": f"{type(exc).__name__}: {exc}"[:120]}


def config_dict(args) -> dict:
    return {"workload": "config 2: dequant-GEMM M=4608 K=3072 N=12288, bf16 activations ~N(0,1), fp8 e4m3 weights "
                        "~N(0,0.02) with per-output-channel absmax scales, exact two-term e4m3 activation split",
            "m": M, "k": K, "n": N, "parallelism": f"dp{args.gpus}", "l2": "flushed between steps (256 MB write, then read back), outside the timed events"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-variants", action="store_true")
    ap.add_argument("--no-model", action="store_true", help="skip the config 3 block and config 4 step variants")
    ap.add_argument("--profile-block", action="store_true",
                    help="run config 3's block (bf16 path) three times, untimed, for an ncu launch list")
    ap.add_argument("--profile-case", action="store_true",
                    help="run each hot-path kernel of config 2 twice, untimed, for an ncu capture")
    ap.add_argument("--profile-rank", type=int, default=0,
                    help="run one sequence-parallel rank's block kernels at this many ranks' shapes (config 4: 4608 / "
                         "N rows, 24 / N heads over 4608 tokens) three times, untimed, on one GPU, for an ncu launch "
                         "list (the peer exchange needs every rank and is left out)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    # Several ranks on one host share its memory and PCIe root complexes: each binds to its GPU's NUMA node before
    # it allocates pinned buffers (one rank keeps every core, for the CPU baseline).
    torch.cuda.set_device(local)
    numa = numa_local_cpus(torch, local) if world > 1 else {"bound": False, "why": "one rank"}
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    we = load_package()
    g = we.Graph(local)
    dev = torch.device("cuda", local)
    # one stream for torch's plumbing (flush, copies, events) and the library's kernels
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    g.set_stream(stream.cuda_stream)

    # ---- synthetic inputs, resident in HBM (seeded per rank: each rank is its own image batch) ----
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    x = torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16)
    w32 = torch.randn(N, K, generator=gen, device=dev) * 0.02
    wq = torch.empty(N, K, dtype=torch.uint8, device=dev)
    ws = torch.empty(N, dtype=torch.float32, device=dev)
    we.kernels.quantize_fp8(g, w32, N, K, wq, ws, per_channel=True, w_dtype="f32")
    w4 = torch.empty(N, K // 2, dtype=torch.uint8, device=dev)
    w4s = torch.empty(N, K // 64, dtype=torch.int16, device=dev)
    we.kernels.quantize_int4(g, w32, N, K, w4, w4s, w_dtype="f32")
    del w32
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    flush_sum = torch.empty((), dtype=torch.float32, device=dev)

    def flush_l2():
        """Write 256 MB (> the 126 MB L2), then read it back so the evicted lines are clean: the timed
        step starts from a cold L2 without the flush's dirty lines draining to HBM underneath it."""
        flush.zero_()
        torch.amax(flush.view(torch.float32), dim=0, out=flush_sum)
    lin = we.Linear(wq, "fp8", 1.0, N, K, chan_scale=ws)
    lin4 = we.Linear(w4, "int4", 1.0, N, K, group_scale=w4s)
    hi = torch.empty(M, K, dtype=torch.uint8, device=dev)
    lo = torch.empty(M, K, dtype=torch.uint8, device=dev)
    rs = torch.empty(M, dtype=torch.float32, device=dev)
    yk = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()

    gate_cycles = int(0.25 * 1.965e9)  # about 130-250 ms of GPU sleep, whatever the clock

    def gate():
        """A fixed GPU sleep queued before a timed call, outside its events: the host enqueues the whole call while
        the GPU still sleeps, so the events time the device work, not the host (a descheduled Python thread on a
        shared host otherwise shows up as GPU idle time inside the timed region)."""
        torch.cuda._sleep(gate_cycles)

    def max_over_ranks(value: float) -> float:
        """The largest value over the ranks (the bench's own process group; timings are max over ranks)."""
        if world == 1:
            return float(value)
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    wall_ms = [0.0]
    step_ms: list = []  # per-step event times of the last timed() call, this rank

    def timed(step, steps, warmup, sampler=None):
        """Sum of per-step CUDA-event times (ms) with an L2 flush before each step, outside the events."""
        for _ in range(warmup):
            flush_l2()
            step()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        gate()
        for a, b in ev:
            flush_l2()
            a.record(stream)
            step()
            b.record(stream)
        torch.cuda.synchronize()
        wall_ms[0] = (time.perf_counter() - t0) * 1e3
        step_ms[:] = [a.elapsed_time(b) for a, b in ev]
        total = sum(step_ms)
        return max_over_ranks(total)

    def interleaved(fns: dict, rounds: int, warmup: int) -> dict:
        """Median CUDA-event ms per step of each function, the functions taking turns (one step each per round,
        an L2 flush before every step) so that clock and power drift over the run falls on all of them alike;
        max over ranks."""
        for _ in range(warmup):
            for fn in fns.values():
                flush_l2()
                fn()
        ev = {name: [] for name in fns}
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for _ in range(rounds):
            for name, fn in fns.items():
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                gate()
                flush_l2()
                a.record(stream)
                fn()
                b.record(stream)
                ev[name].append((a, b))
        torch.cuda.synchronize()
        out = {}
        for name, pairs in ev.items():
            t = sorted(a.elapsed_time(b) for a, b in pairs)
            out[name] = max_over_ranks(t[len(t) // 2])
        return out

    if args.profile_block:
        T = we.transformer
        bc = T.FLUX_BLOCK
        bw = random_block(we, g, torch, dev, gen, bc)
        rows, cols = T.patch_grid(128, 128)
        tokens = 512 + rows * cols
        xb = torch.randn(tokens, bc.hidden, generator=gen, device=dev)
        tvec = torch.randn(6 * bc.hidden, generator=gen, device=dev) * 0.3
        cos_h, sin_h, pairs = we.kernels.rope_tables(we.kernels.positions(512, rows, cols), (16, 56, 56), 1e4)
        rope = we.Rope(torch.from_numpy(cos_h).to(dev), torch.from_numpy(sin_h).to(dev), pairs, tokens)
        for _ in range(3):
            mark = g.mark()
            we.blocks.block(g, bw, bc, xb, tvec, rope, dtype="bf16")
            g.release(mark)
        torch.cuda.synchronize()
        assert g.device_error() == 0
        g.destroy()
        print("profile block done", flush=True)
        return

    if args.profile_rank:
        nr = args.profile_rank
        T = we.transformer
        bc = T.FLUX_BLOCK
        mr, hl = 4608 // nr, bc.heads // nr
        bw = random_block(we, g, torch, dev, gen, bc)
        xr = torch.randn(mr, bc.hidden, generator=gen, device=dev)
        ar = torch.randn(mr, bc.hidden, generator=gen, device=dev) * 0.1
        x1 = torch.empty_like(xr)
        hi_r = torch.empty(mr, bc.mlp, dtype=torch.uint8, device=dev)
        lo_r, rs_r = torch.empty_like(hi_r), torch.empty(mr, device=dev)
        qkv = [torch.empty(mr, bc.hidden, dtype=torch.bfloat16, device=dev) for _ in range(3)]
        cos_h, sin_h, pairs = we.kernels.rope_tables(we.kernels.positions(512, 64, 64), (16, 56, 56), 1e4)
        cs_r = torch.from_numpy(cos_h[:mr * pairs]).to(dev)
        sn_r = torch.from_numpy(sin_h[:mr * pairs]).to(dev)
        qa, ka, va = (torch.randn(4608, hl, 128, generator=gen, device=dev).to(torch.bfloat16) for _ in range(3))
        oa = torch.empty_like(qa)
        o_r = torch.empty(mr, bc.hidden, dtype=torch.bfloat16, device=dev)
        a_r = torch.empty(mr, bc.hidden, device=dev)
        u_r = torch.empty(mr, bc.mlp, dtype=torch.bfloat16, device=dev)
        dn_r = torch.empty(mr, bc.hidden, device=dev)
        gate_v = torch.randn(bc.hidden, device=dev) * 0.1
        for _ in range(3):
            we.kernels.add_norm_split(g, xr, ar, x1, bw.norm1, mr, bc.hidden, hi_r, lo_r, rs_r)
            we.kernels.gemm_fp8(g, hi_r, lo_r, rs_r, bw.wqkv.buffer, None, mr, bw.wqkv.n, bc.hidden,
                                chan_scale=bw.wqkv.chan_scale, y_dtype="bf16",
                                parts=[(qkv[0], bc.hidden), (qkv[1], bc.hidden), (qkv[2], bc.hidden)])
            for t_ in qkv[:2]:
                we.kernels.qknorm_rope(g, t_, bw.norm_q, cs_r, sn_r, mr, bc.heads, pairs, t_, x_dtype="bf16",
                                       out_dtype="bf16")
            we.kernels.attention(g, qa, ka, va, 4608, hl, hl, 128, oa, dtype="bf16", out_dtype="bf16")
            we.kernels.quantize_act(g, o_r, mr, bc.hidden, hi_r, lo_r, rs_r, terms=2)
            we.kernels.gemm_fp8(g, hi_r, lo_r, rs_r, bw.wo.buffer, a_r, mr, bc.hidden, bc.hidden,
                                chan_scale=bw.wo.chan_scale, y_dtype="f32", gate=gate_v)
            we.kernels.add_norm_split(g, xr, a_r, x1, bw.norm2, mr, bc.hidden, hi_r, lo_r, rs_r)
            we.kernels.gemm_fp8(g, hi_r, lo_r, rs_r, bw.mlp_up.buffer, u_r, mr, bc.mlp, bc.hidden,
                                chan_scale=bw.mlp_up.chan_scale, y_dtype="bf16", act="gelu_tanh")
            we.kernels.quantize_act(g, u_r, mr, bc.mlp, hi_r, lo_r, rs_r, terms=2)
            we.kernels.gemm_fp8(g, hi_r, lo_r, rs_r, bw.mlp_down.buffer, dn_r, mr, bc.hidden, bc.mlp,
                                chan_scale=bw.mlp_down.chan_scale, y_dtype="f32", gate=gate_v)
        torch.cuda.synchronize()
        assert g.device_error() == 0
        g.destroy()
        print(f"profile rank done ({nr} ranks: {mr} rows, {hl} heads)", flush=True)
        return

    if args.profile_case:
        # the activation split, the two-term and one-term GEMMs, the int4 decode + kind::f16 GEMM,
        # RMSNorm and q/k norm + RoPE at block size: two launches each, no timing
        wn = torch.randn(K, device=dev) * 0.1
        qn = torch.randn(128, device=dev) * 0.1
        pos = we.kernels.positions(512, 64, 64)
        cos_h, sin_h, pairs = we.kernels.rope_tables(pos, (16, 56, 56), 1e4)
        cs_d, sn_d = torch.from_numpy(cos_h).to(dev), torch.from_numpy(sin_h).to(dev)
        xn = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
        for _ in range(2):
            we.kernels.quantize_act(g, x, M, K, hi, lo, rs, terms=2)
            we.kernels.gemm_fp8(g, hi, lo, rs, wq, yk, M, N, K, chan_scale=ws, y_dtype="bf16")
            we.kernels.gemm_fp8(g, hi, None, rs, wq, yk, M, N, K, chan_scale=ws, y_dtype="bf16")
            mark = g.mark()
            we.linear(g, x, lin4, M, x_dtype="bf16", y_dtype="bf16")
            we.linear(g, x[:256], lin4, 256, x_dtype="bf16", y_dtype="bf16")  # one token tile: unpacked in the GEMM
            g.release(mark)
            we.kernels.rmsnorm(g, x, wn, M, K, xn, x_dtype="bf16", out_dtype="bf16")
            we.kernels.qknorm_rope(g, x, qn, cs_d, sn_d, M, K // 128, pairs, xn, x_dtype="bf16", out_dtype="bf16")
            we.kernels.rope_apply(g, x, cs_d, sn_d, M, K // 128, pairs, xn, x_dtype="bf16", out_dtype="bf16")
        torch.cuda.synchronize()
        assert g.device_error() == 0
        g.destroy()
        print("profile case done", flush=True)
        return

    def step_linear():
        mark = g.mark()
        we.linear(g, x, lin, M, x_dtype="bf16", y_dtype="bf16")
        g.release(mark)

    # ---- headline: the linear layer (activation split + tcgen05 GEMM), inputs resident ----
    launches0 = g.stats["launches"]
    with ClockSampler(local) as clocks:
        total_ms = timed(step_linear, args.steps, args.warmup)
    launches = (g.stats["launches"] - launches0) // (args.steps + args.warmup) * args.steps
    wall_headline_ms = wall_ms[0]
    assert g.device_error() == 0, "device error word set"
    ms = total_ms / args.steps
    value = world * FLOPS / (ms * 1e-3) / 1e12

    # ---- the GEMM kernel alone (roofline) and the activation split alone ----
    we.kernels.quantize_act(g, x, M, K, hi, lo, rs, terms=2)
    gemm_ms = timed(lambda: we.kernels.gemm_fp8(g, hi, lo, rs, wq, yk, M, N, K, chan_scale=ws, y_dtype="bf16"),
                    args.steps, 2) / args.steps
    split_ms = timed(lambda: we.kernels.quantize_act(g, x, M, K, hi, lo, rs, terms=2), args.steps, 2) / args.steps
    peaks = measured_peaks()
    bf16_peak = float(peaks.get("bf16_tflops", 1590.0))
    gemm_tflops = FLOPS / (gemm_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": gemm_tflops, "peak": bf16_peak, "unit": "TFLOP/s",
                "frac": gemm_tflops / bf16_peak,
                # dram__bytes_read.sum + dram__bytes_write.sum of this kernel, one ncu --set full capture of
                # `python bench.py --profile-case` (cold caches): 88.5 MB + 84.6 MB per launch
                "traffic": 173.1e6, "traffic_unit": "bytes per launch",
                "algorithmic_bytes_per_launch": N * K + 2 * M * K + 4 * M + 2 * M * N,
                "kernel": "gemm_tc2_kernel<256, 2, kind::f8f6f4> (cta_group::2 pairs)",
                "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst; two e4m3 MMAs per K step = bf16 rate)"
                if "fallback" not in peaks else "fallback 1.59 PFLOP/s",
                "algorithmic_flop_per_launch": FLOPS, "split_ms": split_ms, "gemm_ms": gemm_ms}

    variants = {}
    if not args.no_variants:
        fast_ms = timed(lambda: we.kernels.gemm_fp8(g, hi, None, rs, wq, yk, M, N, K, chan_scale=ws,
                                                    y_dtype="bf16"), args.steps, 2) / args.steps
        variants["fp8_one_term_gemm"] = {"tflops": FLOPS / (fast_ms * 1e-3) / 1e12, "ms": fast_ms,
                                         "note": "one e4m3 activation term (fp8 tensor-peak mode, ~3% rms act error)"}

        def step_int4():
            mark = g.mark()
            we.linear(g, x, lin4, M, x_dtype="bf16", y_dtype="bf16")
            g.release(mark)

        i4_ms = timed(step_int4, args.steps, 2) / args.steps
        variants["int4_g64_linear"] = {"tflops": FLOPS / (i4_ms * 1e-3) / 1e12, "ms": i4_ms,
                                       "note": "int4 group-64 at config 2's size: decode to bf16 in HBM + tcgen05 "
                                               "kind::f16 (the library's choice at 18 token tiles)"}
        os.environ["WE_TC_I4"] = "1"  # the in-kernel unpack at the same size, for comparison
        i4k_ms = timed(step_int4, args.steps, 2) / args.steps
        del os.environ["WE_TC_I4"]
        variants["int4_g64_linear"]["in_kernel_unpack_ms"] = i4k_ms
        # one token tile (M = 256): the library unpacks W inside the GEMM (converter warps -> shared memory)
        x256 = x[:256]

        def step_int4_256():
            mark = g.mark()
            we.linear(g, x256, lin4, 256, x_dtype="bf16", y_dtype="bf16")
            g.release(mark)

        i4s_ms = timed(step_int4_256, args.steps, 2) / args.steps
        os.environ["WE_TC_I4"] = "0"
        i4s_dec_ms = timed(step_int4_256, args.steps, 2) / args.steps
        del os.environ["WE_TC_I4"]
        variants["int4_g64_linear_m256"] = {"ms": i4s_ms, "tflops": 2.0 * 256 * N * K / (i4s_ms * 1e-3) / 1e12,
                                            "decode_first_ms": i4s_dec_ms,
                                            "note": "M=256 (one token tile): W unpacked inside the GEMM, the "
                                                    "library's choice here; decode_first_ms: decoding W to bf16 in "
                                                    "HBM first"}

    # ---- the bandwidth kernels around the GEMM at block size (config 3: 4608 tokens, hidden 3072, 24 heads) ----
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    wn = torch.randn(K, device=dev) * 0.1
    sc_v, sh_v = torch.randn(K, device=dev) * 0.3, torch.randn(K, device=dev) * 0.3
    qn = torch.randn(128, device=dev) * 0.1
    cos_h, sin_h, pairs = we.kernels.rope_tables(we.kernels.positions(512, 64, 64), (16, 56, 56), 1e4)
    cs_d, sn_d = torch.from_numpy(cos_h).to(dev), torch.from_numpy(sin_h).to(dev)
    # 8 launches per timed step over 8 distinct input / output sets (226 MB of inputs, more than the 126 MB L2):
    # every launch reads HBM, and the per-launch time is the step's over 8, without the events' own overhead
    NB = 8
    xs8 = [torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16) for _ in range(NB)]
    xn8 = [torch.empty(M, K, dtype=torch.bfloat16, device=dev) for _ in range(NB)]
    hi8 = [torch.empty(M, K, dtype=torch.uint8, device=dev) for _ in range(NB)]
    lo8 = [torch.empty(M, K, dtype=torch.uint8, device=dev) for _ in range(NB)]
    rs8 = [torch.empty(M, dtype=torch.float32, device=dev) for _ in range(NB)]
    xf8 = [torch.randn(M, K, generator=gen, device=dev) for _ in range(NB)]  # f32 residual stream, update, sum
    rf8 = [torch.randn(M, K, generator=gen, device=dev) for _ in range(NB)]
    xo8 = [torch.empty(M, K, device=dev) for _ in range(NB)]
    act_bytes = M * K * 2
    bw = {}
    for name, fn, nbytes in [
        ("rmsnorm_mod_bf16", lambda i: we.kernels.rmsnorm(g, xs8[i], wn, M, K, xn8[i], sc_v, sh_v, x_dtype="bf16",
                                                          out_dtype="bf16"), 2 * act_bytes + 3 * K * 4),
        ("qknorm_rope_bf16", lambda i: we.kernels.qknorm_rope(g, xs8[i], qn, cs_d, sn_d, M, K // 128, pairs, xn8[i],
                                                              x_dtype="bf16", out_dtype="bf16"),
         2 * act_bytes + 2 * M * pairs * 4 + 128 * 4),
        ("rope_bf16", lambda i: we.kernels.rope_apply(g, xs8[i], cs_d, sn_d, M, K // 128, pairs, xn8[i],
                                                      x_dtype="bf16", out_dtype="bf16"), 2 * act_bytes + 2 * M * pairs * 4),
        ("act_split_2term", lambda i: we.kernels.quantize_act(g, xs8[i], M, K, hi8[i], lo8[i], rs8[i], terms=2),
         act_bytes + 2 * M * K + M * 4),
        # a block's first norm: the f32 residual stream -> RMSNorm + modulation -> bf16 -> two e4m3 planes
        ("norm_split_f32", lambda i: we.kernels.norm_split(g, xf8[i], wn, M, K, hi8[i], lo8[i], rs8[i], scale=sc_v,
                                                           shift=sh_v, x_dtype="f32"), 2 * act_bytes + 2 * M * K + M * 4),
        # the residual form: x + r written back (f32), then the same norm + split
        ("add_norm_split", lambda i: we.kernels.add_norm_split(g, xf8[i], rf8[i], xo8[i], wn, M, K, hi8[i], lo8[i],
                                                               rs8[i], scale=sc_v, shift=sh_v),
         6 * act_bytes + 2 * M * K + M * 4),
    ]:
        t_ms = timed(lambda: [fn(i) for i in range(NB)], args.steps, 2) / args.steps / NB
        bw[name] = {"ms": t_ms, "gbs": nbytes / (t_ms * 1e-3) / 1e9, "frac_hbm": nbytes / (t_ms * 1e-3) / 1e9 / hbm,
                    "bytes": nbytes, "launches_per_step": NB}
    del xs8, xn8, hi8, lo8, rs8, xf8, rf8, xo8
    roofline["bandwidth_kernels"] = bw

    # ---- config 3's attention (4608 tokens, 24 heads x 128, bf16): tcgen05 flash attention ----
    if not args.no_variants:
        heads = K // 128
        qa = torch.randn(M, heads, 128, generator=gen, device=dev).to(torch.bfloat16)
        ka = torch.randn(M, heads, 128, generator=gen, device=dev).to(torch.bfloat16)
        va = torch.randn(M, heads, 128, generator=gen, device=dev).to(torch.bfloat16)
        oa = torch.empty(M, heads, 128, dtype=torch.bfloat16, device=dev)

        def step_attn():
            we.kernels.attention(g, qa, ka, va, M, heads, heads, 128, oa, dtype="bf16", out_dtype="bf16")

        at_ms = timed(step_attn, args.steps, 2) / args.steps
        at_flops = 4.0 * M * M * heads * 128
        variants["flash_attention_config3"] = {"tflops": at_flops / (at_ms * 1e-3) / 1e12, "ms": at_ms,
                                               "frac_bf16_peak": at_flops / (at_ms * 1e-3) / 1e12 / bf16_peak,
                                               "note": "4 T^2 H D FLOP, T=4608, 24 heads x 128"}
        del qa, ka, va, oa

    # ---- config 3 (one block) and config 4 (one whole denoising step) on the bf16 fused path ----
    if not args.no_variants and not args.no_model:
        variants.update(bench_model(we, g, torch, dev, gen, timed, interleaved, args.steps, bf16_peak, world, local,
                                     step_ms))

    # ---- fp8 dense peak of this GPU, measured like the bf16 one (cuBLAS through torch, 8192^3) ----
    if not args.no_variants:
        try:
            a8 = torch.randn(8192, 8192, device=dev).to(torch.float8_e4m3fn)
            b8 = torch.randn(8192, 8192, device=dev).to(torch.float8_e4m3fn)
            one = torch.ones((), device=dev)
            best = 1e9
            for _ in range(12):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                torch._scaled_mm(a8, b8.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
                e1.record(stream)
                torch.cuda.synchronize()
                best = min(best, e0.elapsed_time(e1))
            fp8_peak = 2 * 8192 ** 3 / (best * 1e-3) / 1e12
            variants["fp8_peak_cublas_tflops"] = fp8_peak
            variants["fp8_one_term_gemm"]["frac_fp8_peak"] = variants["fp8_one_term_gemm"]["tflops"] / fp8_peak
            roofline["frac_of_fp8_peak"] = gemm_tflops / fp8_peak
            del a8, b8
        except Exception as exc:  # noqa: BLE001
            variants["fp8_peak_cublas_tflops"] = f"unmeasured: {exc}"

    # ---- config 5's serving shape: a batch of 8 images (M = 8 x 4608) through 4 linears whose fp8 weights are
    #      streamed from pinned host memory into 2 device slots, overlapped with the GEMMs ----
    if not args.no_variants:
        mb, nl = 8 * M, 4
        xs = torch.randn(mb, K, generator=gen, device=dev).to(torch.bfloat16)
        host_w = [torch.empty(N, K, dtype=torch.uint8).pin_memory() for _ in range(nl)]
        for l in range(nl):
            host_w[l].copy_(wq)  # same bytes as the resident layer; each layer is its own host range
        ysb = torch.empty(mb, N, dtype=torch.bfloat16, device=dev)
        with we.Streamer(g, host_w, slots=2, pinned=True) as streamer:
            def step_stream():
                for l in range(nl):
                    wd = streamer.acquire(l)
                    we.kernels.matmul(g, xs, wd, ysb, mb, N, K, 1.0, x_dtype="bf16", w_dtype="fp8", y_dtype="bf16",
                                      chan_scale=ws)
                    streamer.release(l)

            def step_resident():
                for _ in range(nl):
                    we.kernels.matmul(g, xs, wq, ysb, mb, N, K, 1.0, x_dtype="bf16", w_dtype="fp8", y_dtype="bf16",
                                      chan_scale=ws)

            med = interleaved({"streamed": step_stream, "resident": step_resident}, max(3, args.steps // 4), 2)
            st_ms, rs_ms = med["streamed"], med["resident"]
            variants["streamed_weights_batch8"] = {
                "tflops": nl * 2.0 * mb * N * K / (st_ms * 1e-3) / 1e12, "ms": st_ms,
                "resident_ms": rs_ms, "overlap_efficiency": rs_ms / st_ms,
                "h2d_weight_bytes_per_step": nl * N * K,
                "note": "4 fp8 linears (M=36864, N=12288, K=3072) per step, weights copied host->HBM each step "
                        "through 2 slots on a side stream; streamed and resident steps take turns (medians)"}
        del xs, ysb, host_w

    # ---- end to end through the public API with host buffers: we_linear_host takes x from pinned host memory and
    #      returns y in pinned host memory, its row chunks' copies overlapping the GEMMs ----
    xh = x.cpu().pin_memory()
    yh = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()

    def step_e2e():
        we.linear_host(g, xh, lin, M, yh, x_dtype="bf16", y_dtype="bf16")

    e2e_rows = max(128, ((M + 11) // 12 + 127) // 128 * 128)  # the library's default chunk: about M / 12 rows
    l0 = g.stats["launches"]
    e2e_ms = timed(step_e2e, args.steps, 2) / args.steps
    e2e_launches = (g.stats["launches"] - l0) // (args.steps + 2)
    e2e = {"value": world * FLOPS / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS", "h2d_bytes_per_step": M * K * 2,
           "d2h_bytes_per_step": M * N * 2, "ms_per_step": e2e_ms,
           "call": f"we_linear_host ({(M + e2e_rows - 1) // e2e_rows} row chunks)",
           "gpu_launches_per_step": e2e_launches}
    # the same without the overlap: one upload, the linear, one read-back, in stream order
    xd = torch.empty_like(x)

    def step_serial():
        xd.copy_(xh, non_blocking=True)  # pinned host -> HBM on the library's stream
        mark = g.mark()
        y = we.linear(g, xd, lin, M, x_dtype="bf16", y_dtype="bf16")
        g.read_into(y, yh.data_ptr(), M * N * 2)  # HBM -> pinned host, then wait for the stream
        g.release(mark)

    serial_ms = timed(step_serial, max(3, args.steps // 2), 2) / max(3, args.steps // 2)
    e2e["serial_ms_per_step"] = serial_ms
    e2e["pcie_gbs_estimate"] = (M * K * 2 + M * N * 2) / (serial_ms - ms) / 1e6 if serial_ms > ms else None
    # host traffic of the end-to-end step: per rank, and for all ranks together (the slowest rank's time)
    e2e["host_gbs_per_rank"] = (M * K * 2 + M * N * 2) / (e2e_ms * 1e-3) / 1e9
    e2e["host_gbs_all_ranks"] = world * e2e["host_gbs_per_rank"]
    e2e["numa"] = numa

    line = None
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "fp8 e4m3 x2 (bf16 activations split exactly) -> f32 accumulate",
                "data": "synthetic (seeded torch.randn on device; weights quantised by we_quantize_fp8)",
                "config": config_dict(args), "roofline": roofline, "e2e": e2e, "gpu_launches": launches,
                "clocks": clocks.summary(), "variants": variants,
                "host_wall_ms_timed_region": wall_headline_ms}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(None, target_s=8.0)
    g.destroy()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
