#!/usr/bin/env python
"""Benchmark of the Q4 matmul hot path (BASELINE metric: Q4 matmul HBM GB/s,
% of peak).

Workload (BASELINE config 1's decode shape, one GPU): M = 1 row of fp16
activations against K = N = 4096 Q4_0 matrices. One step is one decode GEMV
through each of 64 distinct matrices (64 x 9.44 MB = 604 MB, more than the
126 MB L2, so weights stream from HBM), captured once as a CUDA graph with
programmatic dependent launch between the GEMVs, as a decode step chains its
projections. With --gpus N (torchrun) every rank runs its own replica
(replicas only: the path has no exchange step at this config); the step time
is the max over ranks and `value` sums all ranks' bytes.

Extra keys: `roofline` (the GEMV kernel against the measured HBM copy
bandwidth), `e2e` (the same GB/s through the C ABI with pinned host buffers,
copies inside the timed region: the step's matmuls recorded once with
wg_graph_begin / wg_graph_end and replayed by wg_graph_launch; `per_call`
beside it makes one C call per matmul), `cpu_baseline` (the CPU oracle's restatement
of the reference's shader arithmetic on the host cores), `clocks`, `sweep`
(config 1's other row counts, informational) and `decode` (BASELINE's
"decode tokens/s": greedy generation of the random-init decoders of configs
2, 3 and 4 on one GPU; with --gpus N, config 4 tensor-parallel over the N
GPUs).

`--impl reference` times the reference's algorithm on the CPU instead (the
reference's own path is WebGL2 shaders, unavailable on this host; the oracle
restates them), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M_ROWS, N_OUT, K_IN = 1, 4096, 4096
MATRICES = 64
SWEEP_M = [1, 4, 16, 64, 256, 1024]
MIN_TP_PREFIX = 32  # tokens a tensor-parallel run's sequences keep in common with one GPU's (median)
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def q4_bytes(N: int, K: int) -> int:
    return N * K * 18 // 32


def algorithmic_bytes(M: int, N: int, K: int, xsz: int = 2, ysz: int = 2) -> int:
    """Weights (18 bytes per 32) + activations + outputs, one matmul."""
    return q4_bytes(N, K) + M * K * xsz + M * N * ysz


def peaks() -> tuple[float, float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic(name: str) -> float | None:
    """DRAM bytes per launch from a committed ncu summary (profiles/), or None."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    m = re.search(r"^traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text(), re.M)
    return float(m.group(1)) if m else None


# ---------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.t0 = self.t1 = 0.0

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(", ") for r in out.strip().splitlines() if r.strip()]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                continue
            for nm, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(nm)
        busy = [s for s in sm if s > 0]
        return {"sm_mhz": statistics.median(busy) if busy else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU side


def cpu_baseline(seconds: float = 10.0) -> dict:
    """The oracle's shader emulation (the reference's arithmetic) of the
    same GEMV on all host cores, repeated for about `seconds`."""
    import oracle as O

    blocks = O.config_q4_0_blocks(N_OUT, K_IN, 0)
    host = O.HostQuantMatrix(N_OUT, K_IN)
    O.c_pack_q4_0(host, 0, blocks, N_OUT)
    x = O.config_activations(M_ROWS, K_IN, 0)
    threads = os.cpu_count() or 1
    O.c_split_emulate(host, x, threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        O.c_split_emulate(host, x, threads)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    gbs = n * algorithmic_bytes(M_ROWS, N_OUT, K_IN, 4, 4) / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} x the M=1 4096x4096 Q4_0 GEMV in the oracle's shader emulation "
                      f"(fp16 activations, fp32 block sums, fp16 K-slice partials), "
                      f"{dt:.1f} s, OpenMP over row groups"}


def run_reference(args) -> None:
    """The reference arm: the oracle's restatement of the reference's shader
    arithmetic on all host threads (rank 0 only). Each step repeats the full
    M=1 4096x4096 GEMV `reps` times, so that the timed region lasts at least
    ~10 s (a short region times a cold CPU); only when the requested steps
    would exceed ~90 s is a step cut to a row slice of one GEMV."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O

    threads = os.cpu_count() or 1
    blocks = O.config_q4_0_blocks(N_OUT, K_IN, 0)
    full = O.HostQuantMatrix(N_OUT, K_IN)
    O.c_pack_q4_0(full, 0, blocks, N_OUT)
    x = O.config_activations(M_ROWS, K_IN, 0)
    # warm the threads and caches (~1 s), then time one full GEMV
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 1.0:
        O.c_split_emulate(full, x, threads)
        n += 1
    t_full = (time.perf_counter() - t0) / n
    steps = max(1, args.steps)
    per_step = min(max(10.0 / steps, t_full), 90.0 / (steps + args.warmup))
    if per_step >= t_full:
        reps, rows = max(1, round(per_step / t_full)), N_OUT
        sub = full
    else:
        reps = 1
        rows = max(64, int(N_OUT * per_step / t_full) // 64 * 64)
        sub = O.HostQuantMatrix(rows, K_IN)
        O.c_pack_q4_0(sub, 0, blocks[: rows * (K_IN // 32) * 18], rows)

    def step():
        for _ in range(reps):
            O.c_split_emulate(sub, x, threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    per = reps * algorithmic_bytes(M_ROWS, rows, K_IN, 4, 4)
    gbs = steps * per / dt / 1e9
    what = f"{reps} x the M=1 4096x4096 Q4_0 GEMV" if rows == N_OUT else f"rows 0..{rows} of the M=1 4096x4096 Q4_0 GEMV"
    sample = (f"each step: {what} ({per} bytes) in the oracle's shader emulation, {threads} threads; "
              f"timed region {dt:.1f} s; the reference's WebGL2 path (headless Chromium + SwiftShader) "
              "is unavailable on this box")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config1 decode GEMV: M=1 row x K=N=4096 Q4_0 (CPU, repeated per step)",
                   "M": M_ROWS, "N": N_OUT, "K": K_IN, "rows_per_step": rows, "gemvs_per_step": reps},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "Q4 matmul HBM GB/s (decode GEMV, BASELINE config 1 shape)"


# ---------------------------------------------------------------- GPU side


def main() -> None:
    global MATRICES
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decoder generation runs")
    ap.add_argument("--matrices", type=int, default=MATRICES,
                    help="distinct matrices per step (default 64 = 604 MB; >= 14 exceeds L2)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    MATRICES = args.matrices

    import torch
    import torch.distributed as dist

    import webgllm_b200 as wg

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from webgllm_b200 import synthetic

    ctx = wg.context(local)
    distinct = [synthetic.q4_0_blocks(N_OUT, K_IN, s) for s in range(4)]
    mats = []
    for r in range(MATRICES):
        m = wg.newQuantMatrix(N_OUT, K_IN, ctx=ctx)
        wg.packQ4_0(m, 0, distinct[r % 4], N_OUT)
        mats.append(m)
    x = torch.from_numpy(synthetic.activations(M_ROWS, K_IN, 0)).to("cuda", torch.float16)
    ys = torch.empty((MATRICES, M_ROWS, N_OUT), device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()

    stream = torch.cuda.Stream()

    def step():
        for r in range(MATRICES):
            wg.matmul(x, mats[r], out=ys[r])

    with torch.cuda.stream(stream):
        step()  # first launches configure the kernels outside capture
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()

        # self-check of the timed path: a few outputs against the matrix's
        # own rows (matrixRow) in fp64 (the oracle parity lives in tests/)
        rows = [0, 1, 777, 2048, 4095]
        xr = x.double().cpu().numpy()[0]
        y_ref = {n: float(np.dot(wg.matrixRow(mats[0], n).astype(np.float64), xr)) for n in rows}
        y_got = ys[0, 0].float().cpu().numpy()
        scale = max(abs(v) for v in y_ref.values())
        assert all(abs(y_got[n] - y_ref[n]) <= 2e-3 * scale for n in rows), "timed path self-check failed"

        clocks = ClockSampler(local)
        clocks.start()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        clock = clocks.stop()
    ms_step = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    per_launch = algorithmic_bytes(M_ROWS, N_OUT, K_IN)
    value = world * MATRICES * per_launch / (ms_step / 1e3) / 1e9
    hbm, bf16, src = peaks()
    achieved = per_launch / (ms_step / MATRICES / 1e3) / 1e9
    traffic = profile_traffic("q4_gemv_config1_m1.txt")

    # ---- e2e: the same step through the C ABI with pinned host buffers
    e2e = None if args.no_e2e else run_e2e(args, ctx, mats, x, ys, per_launch, world, barrier, max_over_ranks)

    # ---- config 1 sweep (informational; each M on 8 rotating matrices)
    sweep = []
    if not args.no_sweep:
        sweep = run_sweep(mats, stream, hbm, bf16)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline()

    decode = None if args.no_decode else run_decode(world, rank, barrier, max_over_ranks, hbm)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = make_line(args, world, value, ms_step, per_launch, achieved, hbm, src, traffic, e2e, clock, cpu, sweep)
    line["decode"] = decode
    print(json.dumps(line), flush=True)
    # Tensor-parallel parity: the partitioned model sums its row-parallel
    # partials in another order than one GPU, and these random-init models
    # move their logits by ~1e-3 under any change of accumulation order, so
    # a near tie can go the other way after some hundred tokens; a wrong
    # shard or exchange breaks every sequence within its first tokens. So a
    # run fails when half its sequences or more part from one GPU's output
    # before token MIN_TP_PREFIX.
    bad = [d for d in decode or []
           if d.get("common_prefix_with_tp1") is not None
           and statistics.median(d["common_prefix_with_tp1"]) < MIN_TP_PREFIX]
    if bad:
        print(f"TENSOR-PARALLEL PARITY FAILED: {len(bad)} run(s) part from one GPU's greedy tokens early "
              f"(common prefixes {bad[0]['common_prefix_with_tp1']})", file=sys.stderr, flush=True)
        sys.exit(1)


def run_decode(world, rank, barrier, max_over_ranks, hbm):
    """Greedy generation (webgllm_b200.runner): configs 2 and 3 on one GPU
    and config 4 (batch 8) on all ranks, tensor-parallel when world > 1 (once
    with the push all-reduce, once with NCCL's).
    Times are the max over ranks; `frac_hbm` is the bytes one decode step
    must read per GPU over the step time, against the measured copy
    bandwidth."""
    from webgllm_b200 import runner

    runs = [("2", None), ("3", None), ("4", None)] if world == 1 else [("4", True), ("4", False)]
    out = []
    group = None
    if world > 1:
        # the library's own NCCL group; torch.distributed only carries its id
        import torch

        import webgllm_b200 as wg
        from webgllm_b200.comm import TensorGroup

        group = TensorGroup.from_torch(wg.context(torch.cuda.current_device()))
    for k, push in runs:
        cfg, batch, prompt, gen = runner.WORKLOADS[k]
        r = runner.measure(cfg, batch, prompt, gen, tp=group, barrier=barrier, push=bool(push))
        step_ms = max_over_ranks(r["decode_ms_per_step"])
        prefill_ms = max_over_ranks(r["prefill_ms"])
        steps = gen - 1
        total_s = (prefill_ms + step_ms * steps) / 1e3
        out.append({
            "config": int(k), "model": r["model"], "batch": batch, "prompt_tokens": prompt,
            "generated_tokens": gen, "tensor_parallel": world if k == "4" else 1,
            "exchange": None if push is None else ("push all-reduce (GEMV epilogue, NVLink P2P)" if push else "NCCL all-reduce (through the library, wg_tp_allreduce)"),
            "decode_tok_s": round(batch / (step_ms / 1e3), 1), "decode_ms_per_step": round(step_ms, 4),
            "prefill_ms": round(prefill_ms, 3), "prefill_tok_s": round(batch * prompt / (prefill_ms / 1e3), 1),
            "e2e_tok_s": round(batch * gen / total_s, 1),
            "step_bytes_per_gpu": int(r["step_bytes"]),
            "frac_hbm": round(r["step_bytes"] / (step_ms / 1e3) / 1e9 / hbm, 4),
            "first_tokens": r["tokens_head"][0],
            "tokens_sha256": r["tokens_sha256"],
        })
        out[-1]["_tokens"] = r["tokens"]
    if world > 1:
        # Parity of the partitioned model: rank 0 also generates config 4 on
        # its GPU alone (the unsharded model from the same seeds) and every
        # tensor-parallel run's whole output (batch x generated tokens) must
        # equal it.
        barrier()
        if rank == 0:
            cfg, batch, prompt, gen = runner.WORKLOADS["4"]
            r1 = runner.measure(cfg, batch, prompt, gen, tp=None)
            for o in out:
                got, want = o["_tokens"], r1["tokens"]
                o["tokens_match_tp1"] = bool(torch.equal(got, want))
                o["tp1_tokens_sha256"] = r1["tokens_sha256"]
                o["common_prefix_with_tp1"] = common_prefix(got, want)
        barrier()
    plain_tokens = next(o["_tokens"] for o in out if o["config"] == 4)
    for o in out:
        o.pop("_tokens", None)
    # config 4's speculative workload (draft k = 4), split like plain decoding
    # when world > 1: once with the independent 1.1B draft (random weights
    # rarely agree with the target: the acceptance rate comes with the rate)
    # and once with a draft that has the target's weights (nearly every
    # proposal kept: the machinery's upper bound). The emitted tokens are
    # compared with plain greedy decoding's: the verify batch's GEMM sums in
    # another order than the decode GEMV, so a near tie may go the other way
    # (common_prefix_with_plain_greedy says where, per sequence).
    cfg, batch, prompt, gen = runner.WORKLOADS["4"]
    plain = next(o for o in out if o["config"] == 4)
    for same in (False, True):
        r = runner.measure_speculative(cfg, batch, prompt, gen, k=4, tp=group, same_draft=same, barrier=barrier)
        ms_round = max_over_ranks(r["decode_ms_per_round"])
        out.append({
            "config": 4, "model": r["model"], "speculative": True, "draft": r["draft"], "k": r["k"],
            "tensor_parallel": world, "batch": batch, "prompt_tokens": prompt, "generated_tokens": gen,
            "decode_tok_s": round(r["decode_tok_s"] * r["decode_ms_per_round"] / ms_round, 1),
            "ms_per_round": round(ms_round, 4), "acceptance": round(r["acceptance"], 4),
            "prefill_ms": round(max_over_ranks(r["prefill_ms"]), 3),
            "tokens_match_plain_greedy": r["tokens_sha256"] == plain["tokens_sha256"],
            "common_prefix_with_plain_greedy": common_prefix(r["tokens"], plain_tokens),
        })
    if group is not None:
        group.close()
    return out


def common_prefix(a, b) -> list:
    """Per sequence, how many leading tokens of a and b agree."""
    out = []
    for x, y in zip(a.tolist(), b.tolist()):
        n = 0
        while n < min(len(x), len(y)) and x[n] == y[n]:
            n += 1
        out.append(n)
    return out


def run_e2e(args, ctx, mats, x, ys, per_launch, world, barrier, max_over_ranks):
    import ctypes

    from webgllm_b200 import _lib

    L = _lib.lib()
    hx = ctx.host_alloc(M_ROWS * K_IN * 2)
    hy = ctx.host_alloc(MATRICES * M_ROWS * N_OUT * 2)
    dx = ctx.alloc(M_ROWS * K_IN * 2)
    dy = ctx.alloc(MATRICES * M_ROWS * N_OUT * 2)
    np.ctypeslib.as_array((ctypes.c_uint16 * (M_ROWS * K_IN)).from_address(hx))[:] = \
        x.cpu().numpy().view(np.uint16).reshape(-1)
    ctx.set_stream(None)
    c_ctx = ctypes.c_void_p(ctx.handle)
    c_mats = [ctypes.c_void_p(m.handle) for m in mats]
    c_dx, c_hx = ctypes.c_void_p(dx), ctypes.c_void_p(hx)
    c_ys = [ctypes.c_void_p(dy + r * M_ROWS * N_OUT * 2) for r in range(MATRICES)]
    c_dy, c_hy = ctypes.c_void_p(dy), ctypes.c_void_p(hy)
    bi, bo = M_ROWS * K_IN * 2, MATRICES * M_ROWS * N_OUT * 2

    def matmuls():
        st = 0
        for r in range(MATRICES):
            st |= L.wg_q4_matmul(c_ctx, c_mats[r], c_dx, 1, M_ROWS, c_ys[r], 1)
        return st

    def check(st):
        if st:
            raise RuntimeError(L.wg_last_error(c_ctx).decode())

    def step_calls():  # one C call per matmul
        check(L.wg_upload(c_ctx, c_dx, c_hx, bi) | matmuls() | L.wg_read(c_ctx, c_hy, c_dy, bo))

    # the step's matmuls recorded once through the C ABI (wg_graph_*), as a
    # host repeating a decode step would, and replayed with one call
    graph = ctypes.c_void_p()
    step_calls()  # first calls outside the recording
    check(L.wg_graph_begin(c_ctx))
    check(matmuls())
    check(L.wg_graph_end(c_ctx, ctypes.byref(graph)))

    def step_graph():
        check(L.wg_upload(c_ctx, c_dx, c_hx, bi) | L.wg_graph_launch(c_ctx, graph) | L.wg_read(c_ctx, c_hy, c_dy, bo))

    e2e_steps = max(10, min(args.steps, 300))
    timed = {}
    for name, fn in (("calls", step_calls), ("graph", step_graph)):
        for _ in range(max(args.warmup, 3)):
            fn()
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            fn()
        timed[name] = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
        y_e2e = np.ctypeslib.as_array((ctypes.c_uint16 * N_OUT).from_address(hy)).view(np.float16)
        assert np.array_equal(y_e2e, ys[0, 0].cpu().numpy()), f"e2e output ({name}) differs from the bench graph's"
    check(L.wg_graph_free(c_ctx, graph))
    ctx.free(dx), ctx.free(dy), ctx.host_free(hx), ctx.host_free(hy)
    gbs = {k: world * MATRICES * per_launch / t / 1e9 for k, t in timed.items()}
    return {"value": round(gbs["graph"], 2), "unit": "GB/s", "h2d_bytes_per_step": bi,
            "d2h_bytes_per_step": bo,
            "how": f"wg_upload + the step's {MATRICES} wg_q4_matmul recorded once (wg_graph_begin/end) and "
                   "replayed by wg_graph_launch + wg_read through the C ABI (ctypes), pinned host buffers, "
                   "wall clock, max over ranks",
            "per_call": {"value": round(gbs["calls"], 2), "unit": "GB/s",
                         "how": f"wg_upload + {MATRICES} x wg_q4_matmul + wg_read, one C call per matmul"}}


def run_sweep(mats, stream, hbm, bf16):
    """Config 1's row counts on 8 rotating matrices (informational), each
    row count's chain of launches captured as a CUDA graph as the main step
    is (eager launches one by one would time the host's launch rate at small
    M); a row whose capture fails is timed eagerly and says so."""
    import torch

    import webgllm_b200 as wg
    from webgllm_b200 import synthetic

    sweep = []
    nm = min(8, len(mats))
    with torch.cuda.stream(stream):
        for M in SWEEP_M:
            xm = torch.from_numpy(synthetic.activations(M, K_IN, 1)).to("cuda", torch.float16)
            ym = torch.empty((M, N_OUT), device="cuda", dtype=torch.float16)
            reps = 8 if M <= 64 else 2

            def chain():
                for r in range(nm):
                    wg.matmul(xm, mats[r], out=ym)

            chain()  # first launches size the scratch and configure the kernels
            stream.synchronize()
            graph, timing = None, "cuda graph"
            try:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    chain()
                graph.replay()
                stream.synchronize()
            except Exception as e:  # noqa: BLE001 - informational rows fall back to eager timing
                graph, timing = None, f"eager ({type(e).__name__})"
                torch.cuda.synchronize()
            run = graph.replay if graph is not None else chain
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(reps):
                run()
            s1.record(stream)
            stream.synchronize()
            del graph
            t = s0.elapsed_time(s1) / 1e3 / (reps * nm)
            b = algorithmic_bytes(M, N_OUT, K_IN)
            f = 2.0 * M * N_OUT * K_IN
            sweep.append({"M": M, "us": round(t * 1e6, 2), "GB/s": round(b / t / 1e9, 1),
                          "TFLOP/s": round(f / t / 1e12, 2),
                          "frac_hbm": round(b / t / 1e9 / hbm, 3),
                          "frac_bf16": round(f / t / 1e12 / bf16, 3), "timing": timing})
    return sweep


def make_line(args, world, value, ms_step, per_launch, achieved, hbm, src, traffic, e2e, clock, cpu, sweep):
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": f"config1 decode GEMV: M=1 fp16 row x K=N=4096 Q4_0, {MATRICES} distinct "
                               "matrices per step, CUDA graph with programmatic dependent launch",
                   "M": M_ROWS, "N": N_OUT, "K": K_IN, "matrices_per_step": MATRICES,
                   "bytes_per_matmul": per_launch,
                   "l2": f"inputs larger than L2 ({MATRICES} x 9.44 MB of weights per step)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic,
                     "peak_source": src, "kernel": "q4 decode GEMV (gemv_kernel<1,false>)"},
        "e2e": e2e,
        "gpu_launches": MATRICES * args.steps,
        "clocks": clock,
        "cpu_baseline": cpu,
        "sweep": sweep,
    }


if __name__ == "__main__":
    main()
