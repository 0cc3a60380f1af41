"""Small, self-contained runs of single kernels for profiling (ncu) and
timing: `python -m webgllm_b200.profile_cases <case> [reps]`.

Each case builds its inputs, runs the kernel `reps` times (default 5) on
torch's current stream and prints the mean device time per launch (CUDA
events), so that the same command serves a plain timing run and an ncu
capture (`-k regex:<kernel> -s <warm-up launches> -c <n>`). Inputs are
larger than L2 where the kernel streams weights.
"""
from __future__ import annotations

import ctypes
import sys

import torch

from . import _lib
from .model import CONFIGS, DecoderModel, quantize_q4_0
from .q4 import context, newQuantMatrix, packQ4_0

P = ctypes.c_void_p


def _q4(N: int, K: int, seed: int = 0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    m = newQuantMatrix(N, K)
    packQ4_0(m, 0, quantize_q4_0(torch.randn((N, K), generator=g, device="cuda") * 0.02), N)
    return m


def _time(fn, reps: int) -> float:
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps


def gemv(M: int, N: int, K: int, reps: int):
    """The decode GEMV (tile-column or wide, by the library's choice) over
    `copies` distinct matrices (rotating, > L2)."""
    c = context()
    copies = max(2, (256 << 20) // (N * K * 18 // 32) + 1)
    mats = [_q4(N, K, i) for i in range(copies)]
    x = torch.randn((M, K), device="cuda").half()
    y = torch.empty((M, N), device="cuda")
    L = _lib.lib()
    c.use_torch_stream()
    i = [0]

    def run():
        m = mats[i[0] % copies]
        i[0] += 1
        _lib.check(L.wg_q4_matmul(P(c.handle), P(m.handle), P(x.data_ptr()), _lib.WG_F16, M, P(y.data_ptr()),
                                  _lib.WG_F32), c.handle)

    run()
    us = _time(run, reps)
    print(f"gemv M={M} N={N} K={K}: {us:.2f} us/launch, {N * K * 18 / 32 / us / 1e3:.1f} GB/s (weights)")


def trace_gemv_chain(M: int, N: int, K: int, reps: int, launches: int = 16):
    """Per-CTA timeline (wg_trace) of a chain of `launches` decode GEMVs over
    distinct matrices (> L2), captured as one CUDA graph with programmatic
    dependent launch, as bench.py times them. Per launch after the first
    two, medians over launches of: the period (last CTA exit to last CTA
    exit), the gap from the previous launch's last exit to this one's first
    dependency release, and per CTA (median) entry -> weight copies issued,
    copies issued -> release, release -> x staged, the multiplies, the tail
    (reduction, stores, exit); plus the spread of the CTAs' releases."""
    import numpy as np

    c = context()
    mats = [_q4(N, K, i) for i in range(launches)]
    x = torch.randn((M, K), device="cuda").half()
    ys = torch.empty((launches, M, N), device="cuda", dtype=torch.float16)
    L = _lib.lib()

    def chain():
        c.use_torch_stream()
        for i in range(launches):
            _lib.check(L.wg_q4_matmul(P(c.handle), P(mats[i].handle), P(x.data_ptr()), _lib.WG_F16, M,
                                      P(ys[i].data_ptr()), _lib.WG_F16), c.handle)

    s = torch.cuda.Stream()
    buf = torch.zeros(8 * 4096 * launches, dtype=torch.int64, device="cuda")
    with torch.cuda.stream(s):
        chain()
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            chain()
        for _ in range(3):
            g.replay()
        us = _time(g.replay, reps) / launches  # untraced
        gt = torch.cuda.CUDAGraph()  # the traced copy: the record buffer is a kernel argument
        _lib.check(L.wg_trace(P(c.handle), P(buf.data_ptr()), buf.numel() * 8), c.handle)
        with torch.cuda.graph(gt, stream=s):
            chain()
        for _ in range(3):
            gt.replay()
        s.synchronize()
        _lib.check(L.wg_trace(P(c.handle), P(buf.data_ptr()), buf.numel() * 8), c.handle)  # restart the records
        gt.replay()
        torch.cuda.synchronize()
    n = ctypes.c_size_t()
    _lib.check(L.wg_trace_count(P(c.handle), ctypes.byref(n)), c.handle)
    _lib.check(L.wg_trace(P(c.handle), None, 0), c.handle)
    rec = buf[: n.value * 8].view(-1, 8).cpu().numpy().astype(np.float64)
    launch = rec[:, 7].astype(np.int64) >> 32
    ids = sorted(set(launch.tolist()))
    cols = {k: [] for k in ("period", "gap", "entry->copies", "copies->release", "x", "mul", "tail",
                            "release spread")}
    prev_exit = None
    for j, li in enumerate(ids):
        r = rec[launch == li] / 1e3  # us
        if prev_exit is not None and j >= 2:
            cols["period"].append(r[:, 5].max() - prev_exit)
            cols["gap"].append(r[:, 2].min() - prev_exit)
            cols["entry->copies"].append(np.median(r[:, 1] - r[:, 0]))
            cols["copies->release"].append(np.median(r[:, 2] - r[:, 1]))
            cols["x"].append(np.median(r[:, 3] - r[:, 2]))
            cols["mul"].append(np.median(r[:, 4] - r[:, 3]))
            cols["tail"].append(np.median(r[:, 5] - r[:, 4]))
            cols["release spread"].append(r[:, 2].max() - r[:, 2].min())
        prev_exit = r[:, 5].max()
    print(f"gemv chain M={M} N={N} K={K}: {us:.2f} us/launch (graph of {launches}), {len(ids)} traced launches, "
          f"{len(rec) // max(1, len(ids))} CTAs each")
    print("  " + ", ".join(f"{k} {np.median(v):.2f}" for k, v in cols.items()) + " (us, medians)")


def gemm(M: int, N: int, K: int, reps: int):
    """The prefill GEMM over `copies` distinct matrices (rotating, > L2 when
    the weights dominate the bytes)."""
    c = context()
    copies = max(1, min(8, (256 << 20) // (N * K * 18 // 32) + 1)) if M <= 256 else 1
    mats = [_q4(N, K, i) for i in range(copies)]
    x = torch.randn((M, K), device="cuda").half()
    y = torch.empty((M, N), device="cuda", dtype=torch.float16)
    L = _lib.lib()
    c.use_torch_stream()
    i = [0]

    def run():
        m = mats[i[0] % copies]
        i[0] += 1
        _lib.check(L.wg_q4_matmul(P(c.handle), P(m.handle), P(x.data_ptr()), _lib.WG_F16, M, P(y.data_ptr()),
                                  _lib.WG_F16), c.handle)

    run()
    us = _time(run, reps)
    print(f"gemm M={M} N={N} K={K}: {us:.2f} us/launch, {2 * M * N * K / us / 1e6:.1f} TFLOP/s")


def attention(batch: int, H: int, Hkv: int, Dh: int, ctx_len: int, reps: int):
    c = context()
    cache = 2048
    kc = torch.randn((batch, Hkv, cache, Dh), device="cuda").half()
    vc = torch.randn_like(kc)
    q = (torch.randn((batch, H, Dh), device="cuda") / Dh ** 0.5).half()
    o = torch.empty_like(q)
    pos = torch.full((batch,), ctx_len - 1, dtype=torch.int32, device="cuda")
    L = _lib.lib()
    c.use_torch_stream()

    def run():
        _lib.check(L.wg_attention(P(c.handle), P(q.data_ptr()), batch, batch, H, Hkv, Dh, P(kc.data_ptr()),
                                  P(vc.data_ptr()), cache, P(pos.data_ptr()), P(o.data_ptr())), c.handle)

    run()
    us = _time(run, reps)
    kv = batch * Hkv * ctx_len * Dh * 2 * 2
    print(f"attention batch={batch} H={H} Hkv={Hkv} Dh={Dh} ctx={ctx_len}: {us:.2f} us, {kv / us / 1e3:.1f} GB/s KV")


def prefill_attention(batch: int, rps: int, H: int, Hkv: int, Dh: int, reps: int):
    """Causal attention of `batch` prompts of `rps` rows each (the flash
    kernel for rps >= 16); reports tensor FLOP/s of the causal work."""
    c = context()
    cache = rps + 64
    kc = torch.randn((batch, Hkv, cache, Dh), device="cuda").half()
    vc = torch.randn_like(kc)
    q = (torch.randn((batch * rps, H, Dh), device="cuda") / Dh ** 0.5).half()
    o = torch.empty_like(q)
    pos = torch.zeros((batch,), dtype=torch.int32, device="cuda")
    L = _lib.lib()
    c.use_torch_stream()

    def run():
        _lib.check(L.wg_attention(P(c.handle), P(q.data_ptr()), batch * rps, batch, H, Hkv, Dh, P(kc.data_ptr()),
                                  P(vc.data_ptr()), cache, P(pos.data_ptr()), P(o.data_ptr())), c.handle)

    run()
    us = _time(run, reps)
    flops = 4.0 * batch * H * Dh * rps * (rps + 1) / 2  # QK^T and PV over the causal triangle
    print(f"prefill attention batch={batch} rows={rps} H={H} Hkv={Hkv} Dh={Dh}: {us:.2f} us, "
          f"{flops / us / 1e6:.1f} TFLOP/s")


def head(rows: int, D: int, V: int, reps: int):
    c = context()
    W = (torch.randn((V, D), device="cuda") * 0.02).half()
    x = torch.randn((rows, D), device="cuda")
    w = torch.ones(D, device="cuda")
    logits = torch.empty((rows, V), device="cuda")
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    L = _lib.lib()
    c.use_torch_stream()

    def run():
        _lib.check(L.wg_head_rmsnorm(P(c.handle), P(x.data_ptr()), None, P(w.data_ptr()), ctypes.c_float(1e-5), rows,
                                     1, D, P(W.data_ptr()), V, 0, P(logits.data_ptr()), P(ids.data_ptr()), None),
                   c.handle)

    run()
    us = _time(run, reps)
    print(f"head rows={rows} D={D} V={V}: {us:.2f} us, {V * D * 2 / us / 1e3:.1f} GB/s")


def decode(config: str, batch: int, reps: int):
    """Eager decode steps (every launch visible to a profiler)."""
    cfg = CONFIGS[config]
    m = DecoderModel(cfg, seed=0, max_ctx=1024, max_rows=batch * 512, batch=batch)
    m.prefill(torch.randint(0, cfg.vocab, (batch, 512), device="cuda", dtype=torch.int32))
    m.decode_step()
    us = _time(m.decode_step, reps)
    print(f"decode config {config} batch {batch}: {us:.1f} us/step (eager)")


def trace_decode(config: str, batch: int, reps: int):
    """Per-CTA timeline of one decode step (CUDA graph) from wg_trace: for
    each of a layer's five traced launches (the q|k|v GEMV, attention, the
    o, gate|up and down GEMVs) the mean span from the dependency release to
    the last CTA's exit and its phases per CTA (GEMVs: release -> x staged,
    the multiplies, the tail; attention: release -> queries made, the K / V
    tiles, the merge of the key slices), the gap before it, and the CTAs
    released more than 5 us after the first (a second wave: CTAs that found
    no room until others finished)."""
    import numpy as np

    cfg = CONFIGS[config]
    m = DecoderModel(cfg, seed=0, max_ctx=1024, max_rows=batch * 512, batch=batch)
    m.prefill(torch.randint(0, cfg.vocab, (batch, 512), device="cuda", dtype=torch.int32))
    m.decode_step()
    torch.cuda.synchronize()
    c, L = m.ctx, _lib.lib()
    buf = torch.zeros(8 * 256 * 4 * cfg.layers * 2, dtype=torch.int64, device="cuda")
    _lib.check(L.wg_trace(P(c.handle), P(buf.data_ptr()), buf.numel() * 8), c.handle)
    m.capture_decode()
    for _ in range(3):
        m.graph.replay()
    us = _time(m.graph.replay, reps)
    _lib.check(L.wg_trace(P(c.handle), P(buf.data_ptr()), buf.numel() * 8), c.handle)  # restart the records
    m.graph.replay()
    torch.cuda.synchronize()
    n = ctypes.c_size_t()
    _lib.check(L.wg_trace_count(P(c.handle), ctypes.byref(n)), c.handle)
    _lib.check(L.wg_trace(P(c.handle), None, 0), c.handle)
    rec = buf[: n.value * 8].view(-1, 8).cpu().numpy().astype(np.float64)
    launch = rec[:, 7].astype(np.int64) >> 32
    ids = sorted(set(launch.tolist()))
    names = ["q|k|v", "attention", "o", "gate|up", "down"]
    acc = {k: {f: [] for f in ("span", "x", "mul", "tail", "gap", "late", "ctas")} for k in names}
    prev_exit = None
    for i, li in enumerate(ids):
        r = rec[launch == li] / 1e3  # us
        a = acc[names[i % len(names)]]
        a["span"].append(r[:, 5].max() - r[:, 2].min())
        a["x"].append(np.median(r[:, 3] - r[:, 2]))
        a["mul"].append(np.median(r[:, 4] - r[:, 3]))
        a["tail"].append(np.median(r[:, 5] - r[:, 4]))
        a["late"].append(int((r[:, 2] > r[:, 2].min() + 5).sum()))
        a["ctas"].append(len(r))
        if prev_exit is not None:
            a["gap"].append(r[:, 2].min() - prev_exit)
        prev_exit = r[:, 5].max()
    print(f"decode config {config} batch {batch}: {us:.1f} us/step (CUDA graph), {len(ids)} traced launches")
    for k in names:
        a = acc[k]
        print(f"  {k:8s} ctas {np.mean(a['ctas']):5.0f}  release->exit {np.mean(a['span']):6.2f} us  per CTA: x "
              f"{np.mean(a['x']):5.2f}, multiplies {np.mean(a['mul']):5.2f}, tail {np.mean(a['tail']):4.2f}  "
              f"gap before {np.mean(a['gap']) if a['gap'] else float('nan'):5.2f}  late CTAs {sum(a['late'])}")


def exchange(reps: int):
    """Cost of one push all-reduce of config 4's decode (batch 8) at the
    tensor-parallel degree of the launch (`python -m torch.distributed.run
    --nproc-per-node N ... -m webgllm_b200.profile_cases exchange_config4_b8`):
    the row-parallel GEMV shard pushing its partials + `wg_comm_reduce_norm`,
    against the same shard GEMV + a local norm, each as a graph of 32
    iterations replayed `reps` times; max over ranks."""
    import os

    import torch.distributed as dist

    from .comm import TensorGroup

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    c = context(rank)
    group = TensorGroup.from_torch(c)
    comm = group.push_comm()
    L = _lib.lib()
    D, M = 4096, 8
    for name, (N, K) in {"o": (D, D // world), "down": (D, 14336 // world)}.items():
        m = _q4(N, K, rank)
        x = torch.randn((M, K), device="cuda").half()
        r0 = torch.randn((M, D), device="cuda")
        r1 = torch.empty_like(r0)
        w = torch.ones(D, device="cuda")
        xo = torch.empty((M, D), dtype=torch.float16, device="cuda")
        y = torch.empty((M, D), device="cuda")
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        times = {}
        for mode in ("push", "local"):
            with torch.cuda.stream(s):
                c.use_torch_stream()

                def it():
                    if mode == "push":
                        comm.push(m, M, x=x)
                        comm.reduce_norm(r0, w, 1e-5, r1, xo, M, D)
                    else:
                        _lib.check(L.wg_q4_matmul(P(c.handle), P(m.handle), P(x.data_ptr()), _lib.WG_F16, M,
                                                  P(y.data_ptr()), _lib.WG_F32), c.handle)
                        _lib.check(L.wg_rmsnorm(P(c.handle), P(r0.data_ptr()), P(y.data_ptr()), P(w.data_ptr()),
                                                ctypes.c_float(1e-5), M, D, P(xo.data_ptr()), _lib.WG_F16),
                                   c.handle)

                it()
                s.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for _ in range(32):
                        it()
                g.replay()
                s.synchronize()
                dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                for _ in range(reps):
                    g.replay()
                e1.record(s)
                s.synchronize()
                t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (32 * reps)], device="cuda", dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                times[mode] = t.item()
                del g
        if rank == 0:
            print(f"TP{world} {name} shard {N}x{K}, M={M}: push GEMV + reduce_norm {times['push']:.2f} us, "
                  f"GEMV + local norm {times['local']:.2f} us, exchange {times['push'] - times['local']:.2f} us",
                  flush=True)
    comm.close()
    group.close()
    dist.destroy_process_group()


CASES = {
    "gemv_config1_m1": lambda r: gemv(1, 4096, 4096, r),
    "gemv_wide_m8": lambda r: gemv(8, 28672, 4096, r),
    "gemv_m1_28672x4096": lambda r: gemv(1, 28672, 4096, r),
    "trace_gemv_chain_m1": lambda r: trace_gemv_chain(1, 4096, 4096, r),
    "trace_gemv_chain_m1_2048": lambda r: trace_gemv_chain(1, 2048, 2048, r),
    # the GEMM's stamps: entry, copies issued, release, first x, last multiply, exit
    "trace_gemm_chain_m64": lambda r: trace_gemv_chain(64, 4096, 4096, r),
    "trace_gemm_chain_m256": lambda r: trace_gemv_chain(256, 4096, 4096, r),
    "gemm_m64": lambda r: gemm(64, 4096, 4096, r),
    "gemm_m256": lambda r: gemm(256, 4096, 4096, r),
    "gemm_m1024": lambda r: gemm(1024, 4096, 4096, r),
    "gemm_m4096_down": lambda r: gemm(4096, 4096, 14336, r),
    "attention_config4_b8": lambda r: attention(8, 32, 8, 128, 640, r),
    "attention_prefill_config4_b8": lambda r: prefill_attention(8, 512, 32, 8, 128, r),
    "attention_config2": lambda r: attention(1, 32, 4, 64, 256, r),
    "head_config2": lambda r: head(1, 2048, 32000, r),
    "head_config4_b8": lambda r: head(8, 4096, 128256, r),
    "decode_config4_b8": lambda r: decode("4", 8, r),
    "decode_config2": lambda r: decode("2", 1, r),
    "exchange_config4_b8": lambda r: exchange(r),
    "trace_decode_config4_b8": lambda r: trace_decode("4", 8, r),
    "trace_decode_config2": lambda r: trace_decode("2", 1, r),
}


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if not argv or argv[0] not in CASES:
        print("cases:", " ".join(CASES))
        return 2
    reps = int(argv[1]) if len(argv) > 1 else 5
    CASES[argv[0]](reps)
    return 0


if __name__ == "__main__":
    sys.exit(main())
