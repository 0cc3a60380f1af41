"""Tensor parallelism on 2 GPUs (NCCL): a random-init decoder split across
two ranks (webgllm_b200.tp) decodes the same greedy tokens as the unsharded
model on one GPU, with logits (the two vocabulary shards side by side)
within 2% of their scale, through prefill (GEMM), eager decode and CUDA-graph
replays that contain the NCCL all-reduces. Needs >= 2 GPUs; skipped
otherwise."""
import os
import random

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 CUDA GPUs", allow_module_level=True)

import datetime  # noqa: E402

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _cfg():
    from webgllm_b200.model import DecoderConfig

    return DecoderConfig("tiny-tp", 3, 512, 8, 4, 64, 1024, 1000, 1e-5, 1e4)


def _run(model, prompts, steps):
    toks, logits = [], []
    model.prefill(prompts)
    toks.append(model.next_id.clone())
    logits.append(model.logits.clone())
    model.decode_step()
    toks.append(model.next_id.clone())
    logits.append(model.logits.clone())
    model.capture_decode()
    for _ in range(steps):
        model.graph.replay()
        toks.append(model.next_id.clone())
        logits.append(model.logits.clone())
    torch.cuda.synchronize()
    return toks, logits


def _worker(rank, world, port, q, push):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from webgllm_b200.model import DecoderModel

        cfg = _cfg()
        m = DecoderModel(cfg, seed=7, max_ctx=128, max_rows=64, batch=2, tp=(rank, world, None), push=push)
        prompts = torch.randint(0, cfg.vocab, (2, 24), generator=torch.Generator().manual_seed(3)).cuda()
        toks, logits = _run(m, prompts, 4)
        m.ctx.sync()  # surfaces a timed-out exchange
        # both vocabulary shards, side by side
        full = []
        for lg in logits:
            parts = [torch.zeros_like(lg) for _ in range(world)]
            dist.all_gather(parts, lg)
            full.append(torch.cat(parts, dim=1))
        m.graph = None
        m.close()
        if rank == 0:
            single = DecoderModel(cfg, seed=7, max_ctx=128, max_rows=64, batch=2)
            stoks, slog = _run(single, prompts, 4)
            errs = [((a - b).abs().max() / b.abs().max()).item() for a, b in zip(full, slog)]
            same = [torch.equal(a, b) for a, b in zip(toks, stoks)]
            q.put((max(errs), same))
    finally:
        dist.destroy_process_group()


def _push_worker(rank, world, port, q):
    """Three exchanges of a pushing matmul against NCCL's sum of the same
    local products."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import webgllm_b200 as wg
        from webgllm_b200.comm import PushComm
        from webgllm_b200.model import quantize_q4_0

        ctx = wg.context(rank)
        ctx.use_torch_stream()
        comm = PushComm(ctx, rank, world)
        errs = []
        for it, (M, N, K) in enumerate([(1, 512, 256), (8, 4096, 1024), (3, 1024, 14336 // 2)]):
            g = torch.Generator(device="cuda")
            g.manual_seed(100 * it + rank)
            m = wg.newQuantMatrix(N, K)
            wg.packQ4_0(m, 0, quantize_q4_0(torch.randn((N, K), generator=g, device="cuda") * 0.02), N)
            x = torch.randn((M, K), generator=g, device="cuda").half()
            ref = wg.matmul(x, m, out_dtype=torch.float32)
            dist.all_reduce(ref)
            out = torch.full((M, N), float("nan"), device="cuda")
            ctx.use_torch_stream()
            comm.push(m, M, x=x)
            comm.reduce(out, M, N)
            ctx.sync()  # a missing push would surface here as WG_TIMEOUT
            errs.append(((out - ref).abs().max() / ref.abs().max()).item())
        # the exchange fused with the residual add and the next RMS norm
        M, N, K = 8, 4096, 512
        m = wg.newQuantMatrix(N, K)
        g = torch.Generator(device="cuda")
        g.manual_seed(7 + rank)
        wg.packQ4_0(m, 0, quantize_q4_0(torch.randn((N, K), generator=g, device="cuda") * 0.02), N)
        x = torch.randn((M, K), generator=g, device="cuda").half()
        resid = torch.randn((M, N), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
        w = torch.rand(N, device="cuda", generator=torch.Generator(device="cuda").manual_seed(2)) + 0.5
        part = wg.matmul(x, m, out_dtype=torch.float32)
        dist.all_reduce(part)
        v = resid + part
        want = (v * torch.rsqrt((v * v).mean(-1, keepdim=True) + 1e-5) * w).half()
        new_resid = torch.empty_like(resid)
        xh = torch.empty((M, N), dtype=torch.float16, device="cuda")
        ctx.use_torch_stream()
        comm.push(m, M, x=x)
        comm.reduce_norm(resid, w, 1e-5, new_resid, xh, M, N)
        ctx.sync()
        errs.append(((new_resid - v).abs().max() / v.abs().max()).item())
        xerr = ((xh.float() - want.float()).abs().max() / want.float().abs().max()).item()  # fp16 rounding
        comm.close()
        q.put((rank, max(errs), xerr))
    finally:
        dist.destroy_process_group()


def _spawn(target, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + random.Random().randrange(0, 2000)
    procs = [ctx.Process(target=target, args=(r, 2, port, q, *extra)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return q


def test_push_all_reduce_matches_nccl():
    q = _spawn(_push_worker)
    for _ in range(2):
        rank, err, xerr = q.get(timeout=10)
        assert err < 1e-6, (rank, err)
        assert xerr < 2e-3, (rank, xerr)


@pytest.mark.parametrize("push", [True, False])
def test_tp2_decodes_like_one_gpu(push):
    """push: the row-parallel sums go through the fused push all-reduce
    (decode) and NCCL (prefill); otherwise NCCL everywhere."""
    q = _spawn(_worker, (push,))
    err, same = q.get(timeout=10)
    assert err < 2e-2, err
    assert all(same), same
