"""Greedy generation throughput of the random-init decoders (BASELINE
configs 2-4): prompt prefill, then decode steps replayed from a CUDA graph.

Used by bench.py; a run is `measure(cfg, batch, prompt_len, gen_len, tp)`:
every rank of a tensor-parallel group calls it with the same arguments.
"""
from __future__ import annotations

import hashlib

import torch

from .model import CONFIGS, DecoderModel

# BASELINE workloads: (config, batch, prompt tokens, generated tokens)
WORKLOADS = {
    "2": (CONFIGS["2"], 1, 128, 128),
    "3": (CONFIGS["3"], 1, 512, 256),
    "4": (CONFIGS["4"], 8, 512, 256),
}


def step_bytes(m: DecoderModel, ctx_len: float) -> float:
    """HBM bytes one decode step must read on this rank: every Q4 matrix
    (18 bytes per 32 weights), the head shard (fp16), the embedding rows, and
    the K / V cache of `ctx_len` positions per sequence."""
    cfg = m.cfg
    q4 = 0
    for lay in m.layers:
        for k in ("qkv", "o", "in", "out", "gu", "down"):
            if k in lay:
                q4 += lay[k].N * lay[k].K * 18 // 32
    head = m.V * cfg.hidden * 2
    n_attn = sum(t == "attn" for t in cfg.layer_types)
    kv = n_attn * m.batch * m.Hkv * ctx_len * cfg.head_dim * 2 * 2
    return q4 + head + m.batch * cfg.hidden * 2 + kv


def measure(cfg, batch: int, prompt_len: int, gen_len: int, tp=None, seed: int = 0, barrier=None,
            push: bool = True) -> dict:
    """Prefill `batch` random prompts of `prompt_len` tokens and generate
    `gen_len` tokens each (the first from the prefill, the rest from graph
    replays). Device-timed with CUDA events; `barrier` (if given) runs before
    and after the timed region."""
    m = DecoderModel(cfg, seed=seed, max_ctx=prompt_len + gen_len + 8, max_rows=batch * prompt_len, batch=batch,
                     tp=tp, push=push)
    g = torch.Generator().manual_seed(seed + 1)
    prompts = torch.randint(0, cfg.vocab, (batch, prompt_len), generator=g).to("cuda", torch.int32)
    out = torch.zeros((batch, gen_len), dtype=torch.int32, device="cuda")
    # warm-up: every kernel configured, graph captured
    m.prefill(prompts)
    m.decode_step()
    m.capture_decode()
    m.graph.replay()
    torch.cuda.synchronize()
    m.reset()
    if barrier:
        barrier()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record(s)
    m.prefill(prompts)
    out[:, 0].copy_(m.next_id)
    ev[1].record(s)
    for i in range(1, gen_len):
        m.graph.replay()
        out[:, i].copy_(m.next_id)
    ev[2].record(s)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    prefill_ms = ev[0].elapsed_time(ev[1])
    decode_ms = ev[1].elapsed_time(ev[2])
    steps = gen_len - 1
    res = {
        "model": cfg.name, "batch": batch, "prompt": prompt_len, "generated": gen_len,
        "tp": m.world, "prefill_ms": prefill_ms, "decode_ms_per_step": decode_ms / max(steps, 1),
        "decode_tok_s": batch * steps / (decode_ms / 1e3) if steps else None,
        "prefill_tok_s": batch * prompt_len / (prefill_ms / 1e3),
        "e2e_tok_s": batch * gen_len / ((prefill_ms + decode_ms) / 1e3),
        "step_bytes": step_bytes(m, prompt_len + gen_len / 2),
        "tokens_head": out[:, :8].tolist(),
        "tokens": out.cpu(),
        "tokens_sha256": hashlib.sha256(out.cpu().numpy().astype("<i4").tobytes()).hexdigest(),
    }
    m.graph = None
    m.close()
    del m
    torch.cuda.empty_cache()
    return res


def measure_speculative(cfg, batch: int, prompt_len: int, gen_len: int, k: int = 4, seed: int = 0, tp=None,
                        same_draft: bool = False, barrier=None) -> dict:
    """Config 4's speculative workload: a random-init draft of config 2's
    layout (the target's vocabulary) proposes k tokens a round and the
    target verifies them. With independent random weights the draft almost
    never agrees with the target, so a round yields about one token per
    sequence: the acceptance rate is reported with the throughput.
    same_draft: the draft is a copy of the target (same config and seed), so
    every proposal is accepted: the machinery's upper bound.
    tp: the target is split across the group (its verify rows go through
    the row-parallel GEMM and NCCL sums, the picks through one MAX
    all-reduce); the 1.1B draft runs whole on every rank (its 4 KV heads do
    not split 8 ways, and it is small), the same-weights draft split like
    the target."""
    from .speculative import SpeculativeDecoder, draft_config

    ctx_len = prompt_len + gen_len + 2 * (k + 1) + 8
    t = DecoderModel(cfg, seed=seed, max_ctx=ctx_len, max_rows=batch * prompt_len, batch=batch, tp=tp)
    if same_draft:
        d = DecoderModel(cfg, seed=seed, max_ctx=ctx_len, max_rows=batch * prompt_len, batch=batch, tp=tp)
    else:
        d = DecoderModel(draft_config(cfg), seed=seed + 100, max_ctx=ctx_len, max_rows=batch * prompt_len,
                         batch=batch)
    spec = SpeculativeDecoder(t, d, k=k, max_new=gen_len)
    g = torch.Generator().manual_seed(seed + 1)
    prompts = torch.randint(0, cfg.vocab, (batch, prompt_len), generator=g).to("cuda", torch.int32)
    spec.prefill(prompts)
    spec.step()
    spec.capture()
    t.reset()
    d.reset()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    s = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record(s)
    spec.prefill(prompts)
    ev[1].record(s)
    rounds = 0
    # rounds until every sequence has gen_len tokens (checked every 16 rounds)
    while True:
        for _ in range(16):
            spec.graph.replay()
        rounds += 16
        if int(spec.out_len.min().item()) >= gen_len or rounds >= 4 * gen_len:
            break
    ev[2].record(s)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    prefill_ms = ev[0].elapsed_time(ev[1])
    decode_ms = ev[1].elapsed_time(ev[2])
    produced = int(spec.out_len.sum().item()) - batch  # after the prefill's token
    out = spec.out[:, :gen_len].cpu()
    res = {
        "model": cfg.name, "draft": d.cfg.name + (" (the target's weights)" if same_draft else ""), "k": k,
        "batch": batch, "rounds": rounds, "tp": t.world,
        "decode_ms_per_round": decode_ms / rounds, "decode_tok_s": produced / (decode_ms / 1e3),
        "acceptance": float(spec.accepted.sum().item()) / (rounds * batch * k),
        "prefill_ms": prefill_ms, "tokens": out,
        "tokens_sha256": hashlib.sha256(out.numpy().astype("<i4").tobytes()).hexdigest(),
    }
    spec.graph = None
    t.close()
    d.close()
    del spec, t, d
    torch.cuda.empty_cache()
    return res

