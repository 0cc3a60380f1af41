"""Tensor-parallel partition (webgllm_b200.tp) on the host: the plan's
divisibility rules, Q4_0 byte shards against slices of the dequantised
matrix, the packed greedy keys' order, and a world-size-2 gloo run of a
torch fp32 tensor-parallel forward (column / row splits, all-reduce after o
and down, vocabulary-parallel head with an int64 MAX pick) against the
unsharded forward. No GPU: the placement of every cut and collective is what
is checked; the GPU kernels are checked by the -m gpu tests."""
import math
import os
import random
import struct

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from webgllm_b200 import tp as TP  # noqa: E402
from webgllm_b200.model import CONFIG2, CONFIG3, CONFIG4, DecoderConfig, dequantize_q4_0, quantize_q4_0  # noqa: E402


def test_plan_divisibility():
    for n in (1, 2, 4, 8):
        s = TP.plan(CONFIG4, n - 1, n)
        assert s.heads * n == 32 and s.kv_heads * n == 8 and s.ffn * n == 14336 and s.vocab * n == 128256
        assert s.vocab_offset == (n - 1) * s.vocab
    with pytest.raises(ValueError):
        TP.plan(CONFIG2, 0, 8)  # 4 KV heads over 8 GPUs
    TP.plan(CONFIG2, 1, 4)
    with pytest.raises(ValueError):
        TP.plan(CONFIG3, 0, 2)  # conv layers are not split
    with pytest.raises(ValueError):
        TP.plan(CONFIG4, 2, 2)


def test_q4_shards_are_slices_of_the_matrix():
    g = torch.Generator().manual_seed(1)
    N, K = 24, 256
    blocks = quantize_q4_0(torch.randn((N, K), generator=g) * 0.02)
    full = dequantize_q4_0(blocks, N, K)
    rows = torch.tensor([3, 0, 17, 23, 8])
    assert torch.equal(dequantize_q4_0(TP.q4_rows(blocks, N, K, rows), 5, K), full[rows])
    assert torch.equal(dequantize_q4_0(TP.q4_cols(blocks, N, K, 64, 192), N, 128), full[:, 64:192])
    with pytest.raises(ValueError):
        TP.q4_cols(blocks, N, K, 16, 64)


def test_qkv_and_gate_up_rows_cover_the_matrix_once():
    cfg = CONFIG4
    n = 4
    qkv = torch.cat([TP.qkv_rows(cfg, TP.plan(cfg, r, n)) for r in range(n)])
    assert sorted(qkv.tolist()) == list(range((cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim))
    gu = torch.cat([TP.gate_up_rows(cfg, TP.plan(cfg, r, n)) for r in range(n)])
    assert sorted(gu.tolist()) == list(range(2 * cfg.ffn))


def test_argmax_key_orders_by_value_then_lower_index():
    rnd = random.Random(3)
    vals = [0.0, -0.0, 1.5, -1.5, 3.4e38, -3.4e38, float("inf"), -float("inf"), 1e-40, -1e-40]
    vals += [rnd.uniform(-100, 100) for _ in range(40)]
    pairs = [(struct.unpack("<f", struct.pack("<f", v))[0], rnd.randrange(0, 200000)) for v in vals]
    pairs += [(1.5, 7), (1.5, 3)]
    for a in pairs:
        for b in pairs:
            ka, kb = TP.argmax_key(*a), TP.argmax_key(*b)
            if a[0] != b[0]:
                assert (ka > kb) == (a[0] > b[0]), (a, b)
            elif a[1] != b[1]:
                assert (ka > kb) == (a[1] < b[1]), (a, b)
            assert TP.key_index(ka) == a[1]


# ---------------------------------------------------------------- gloo world 2

TINY = DecoderConfig("tiny-tp", 2, 128, 4, 2, 32, 256, 96, 1e-5, 1e4)


def _weights(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    D, H, Hkv, Dh, I, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
    W = {"embed": torch.randn((V, D), generator=g) * 0.5, "head": torch.randn((V, D), generator=g) * 0.05,
         "layers": []}
    for _ in range(cfg.layers):
        W["layers"].append({
            "qkv": quantize_q4_0(torch.randn(((H + 2 * Hkv) * Dh, D), generator=g) * 0.05),
            "o": quantize_q4_0(torch.randn((D, H * Dh), generator=g) * 0.05),
            "gu": quantize_q4_0(torch.randn((2 * I, D), generator=g) * 0.05),
            "down": quantize_q4_0(torch.randn((D, I), generator=g) * 0.05),
        })
    return W


def _norm(x, eps):
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)


def _rope(t, pos, theta):
    Dh = t.shape[-1]
    half = Dh // 2
    j = torch.arange(half, dtype=torch.float32)
    ang = pos[:, None].float() * torch.pow(torch.tensor(theta), -2.0 * j / Dh)[None, :]
    cs, sn = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    a, b = t[..., :half], t[..., half:]
    return torch.cat([a * cs - b * sn, b * cs + a * sn], dim=-1)


def _forward(cfg, W, ids, s, reduce_sum, reduce_max):
    """Prefill of `ids` on shard s (s None: the whole model); returns the
    last row's logits of this shard and the picked token."""
    D, H, Hkv, Dh, I, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
    Hl, Hkvl, Il = (s.heads, s.kv_heads, s.ffn) if s else (H, Hkv, I)
    T = ids.numel()
    x = W["embed"][ids]
    pos = torch.arange(T)
    for Lw in W["layers"]:
        wq = Lw["qkv"] if s is None else TP.q4_rows(Lw["qkv"], (H + 2 * Hkv) * Dh, D, TP.qkv_rows(cfg, s))
        wq = dequantize_q4_0(wq, (Hl + 2 * Hkvl) * Dh, D)
        qkv = _norm(x, cfg.eps) @ wq.t()
        q = _rope(qkv[:, :Hl * Dh].reshape(T, Hl, Dh), pos, cfg.theta)
        k = _rope(qkv[:, Hl * Dh:(Hl + Hkvl) * Dh].reshape(T, Hkvl, Dh), pos, cfg.theta)
        v = qkv[:, (Hl + Hkvl) * Dh:].reshape(T, Hkvl, Dh)
        G = Hl // Hkvl
        att = torch.zeros((T, Hl, Dh))
        mask = torch.tril(torch.ones(T, T, dtype=torch.bool))
        for h in range(Hl):
            sc = (q[:, h] @ k[:, h // G].t()) / math.sqrt(Dh)
            sc = sc.masked_fill(~mask, -float("inf"))
            att[:, h] = torch.softmax(sc, dim=1) @ v[:, h // G]
        wo = Lw["o"] if s is None else TP.q4_cols(Lw["o"], D, H * Dh, *TP.o_cols(cfg, s))
        o = att.reshape(T, Hl * Dh) @ dequantize_q4_0(wo, D, Hl * Dh).t()
        x = x + reduce_sum(o)
        wg = Lw["gu"] if s is None else TP.q4_rows(Lw["gu"], 2 * I, D, TP.gate_up_rows(cfg, s))
        gu = _norm(x, cfg.eps) @ dequantize_q4_0(wg, 2 * Il, D).t()
        act = torch.nn.functional.silu(gu[:, :Il]) * gu[:, Il:]
        wd = Lw["down"] if s is None else TP.q4_cols(Lw["down"], D, I, *TP.down_cols(cfg, s))
        x = x + reduce_sum(act @ dequantize_q4_0(wd, D, Il).t())
    head = W["head"] if s is None else W["head"][s.vocab_offset:s.vocab_offset + s.vocab]
    logits = _norm(x[-1:], cfg.eps) @ head.t()
    i = int(logits[0].argmax())
    off = s.vocab_offset if s else 0
    key = reduce_max(torch.tensor([TP.argmax_key(float(logits[0, i]), off + i)], dtype=torch.int64))
    return logits[0], TP.key_index(int(key[0]))


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = TINY
        W = _weights(cfg, 11)
        ids = torch.randint(0, cfg.vocab, (9,), generator=torch.Generator().manual_seed(2))

        def rsum(t):
            t = t.clone()
            dist.all_reduce(t)
            return t

        def rmax(t):
            t = t.clone()
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t

        s = TP.plan(cfg, rank, world)
        logits, tok = _forward(cfg, W, ids, s, rsum, rmax)
        parts = [torch.zeros_like(logits) for _ in range(world)]
        dist.all_gather(parts, logits)
        full_logits, full_tok = _forward(cfg, W, ids, None, lambda t: t, lambda t: t)
        got = torch.cat(parts)
        q.put((rank, (got - full_logits).abs().max().item() / full_logits.abs().max().item(), tok, full_tok,
               int(full_logits.argmax())))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_forward_matches_unsharded_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + random.Random().randrange(0, 2000)
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = sorted(q.get(timeout=10) for _ in range(2))
    for rank, err, tok, full_tok, full_argmax in results:
        assert err < 1e-5, (rank, err)
        assert tok == full_tok == full_argmax, (rank, tok, full_tok)
