"""Plain PyTorch fp32 references of the decoder-layer kernels and of a whole
decoder forward, for the GPU parity tests (test infrastructure only).

Each function restates the op the library's kernel computes (the semantics
in include/webgllm_decoder.h, which follow the reference engine's passes:
packages/webgllm/src/gpu/kernels.ts RMS / headPrep / scores / attend /
REDUCE_SWIGLU / shortConv, src/engine.ts head and argmax). Rounding points
match the kernels' (fp16 where the kernel stores fp16) so that differences
are accumulation order only.
"""
from __future__ import annotations

import math

import torch


def rmsnorm(x, add, w, eps):
    """Returns (new x, normed) in fp32; the kernel rounds `normed` to its
    output dtype."""
    if add is not None:
        x = x + add
    inv = torch.rsqrt((x * x).mean(dim=-1, keepdim=True) + eps)
    return x, x * inv * w


def rope_kv(qkv, H, Hkv, Dh, pos0, theta, q_norm=None, k_norm=None, eps=1e-5):
    """qkv fp32 [rows][(H + 2 Hkv) Dh] -> (q fp16 [rows][H][Dh] scaled by
    1/sqrt(Dh), k fp16 [rows][Hkv][Dh], v fp16 [rows][Hkv][Dh])."""
    rows = qkv.shape[0]
    q = qkv[:, : H * Dh].reshape(rows, H, Dh)
    k = qkv[:, H * Dh:(H + Hkv) * Dh].reshape(rows, Hkv, Dh)
    v = qkv[:, (H + Hkv) * Dh:].reshape(rows, Hkv, Dh)

    def norm(t, w):
        if w is None:
            return t
        return t * torch.rsqrt((t * t).mean(dim=-1, keepdim=True) + eps) * w

    q, k = norm(q, q_norm), norm(k, k_norm)
    half = Dh // 2
    j = torch.arange(half, device=qkv.device, dtype=torch.float32)
    freq = torch.pow(torch.tensor(theta, dtype=torch.float32, device=qkv.device), -2.0 * j / Dh)
    pos = (pos0 + torch.arange(rows, device=qkv.device, dtype=torch.float32))[:, None]
    ang = pos * freq[None, :]
    cs, sn = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]

    def rot(t):
        a, b = t[..., :half], t[..., half:]
        return torch.cat([a * cs - b * sn, b * cs + a * sn], dim=-1)

    return (rot(q) / math.sqrt(Dh)).half(), rot(k).half(), v.half()


def attention(q, k_cache, v_cache, pos0, H, Hkv):
    """q fp16 [rows][H][Dh] (scaled); caches fp16 [Hkv][cache_len][Dh];
    row r attends keys 0..pos0+r. Returns fp32 [rows][H][Dh]. Query head h
    reads KV head h // (H / Hkv) (grouped-query attention)."""
    rows, _, Dh = q.shape
    G = H // Hkv
    L = pos0 + rows
    keys = torch.arange(L, device=q.device)
    masked = keys[None, :] > (pos0 + torch.arange(rows, device=q.device))[:, None]  # [rows][L]
    kk = k_cache[:, :L].float()  # [Hkv][L][Dh]
    vv = v_cache[:, :L].float()
    qh = q.float().permute(1, 0, 2).reshape(Hkv, G * rows, Dh)  # entry g * rows + r of KV head j: head j * G + g
    s = (qh @ kk.transpose(1, 2)).masked_fill(masked.repeat(G, 1)[None], float("-inf"))
    o = torch.softmax(s, dim=2) @ vv  # [Hkv][G * rows][Dh]
    return o.reshape(H, rows, Dh).permute(1, 0, 2).contiguous()


def swiglu(gu, I):
    g, u = gu[:, :I], gu[:, I:]
    return g * torch.sigmoid(g) * u


def short_conv(bcx, D, W, weight, state):
    """bcx fp32 [rows][3D]; weight [D][W]; state fp16 [W-1][D] (oldest
    first). Returns (out fp32 [rows][D], new state fp16)."""
    B, C, x = bcx[:, :D], bcx[:, D:2 * D], bcx[:, 2 * D:]
    y = B * x
    hist = torch.cat([state.float(), y], dim=0)  # [W-1 + rows][D]
    rows = bcx.shape[0]
    out = torch.zeros((rows, D), dtype=torch.float32, device=bcx.device)
    for t in range(rows):
        win = hist[t:t + W]  # y_{t-(W-1)} .. y_t
        out[t] = C[t] * (win * weight.t()).sum(dim=0)
    new_state = hist[-(W - 1):].half() if W > 1 else state
    return out, new_state


def dequant_linear(lin):
    from webgllm_b200.model import dequantize_q4_0

    return dequantize_q4_0(lin.blocks, lin.N, lin.K)


def reference_weights(model):
    """The model's linears dequantised to fp32 (its Linears must keep their
    Q4_0 blocks) and its fp16 head as fp32: shared by the references of
    several sequences."""
    return {"layers": [{k: dequant_linear(v) for k, v in L.items() if hasattr(v, "blocks")} for L in model.layers],
            "head": model.head.float()}


class ReferenceDecoder:
    """The same forward as webgllm_b200.model.DecoderModel for one sequence,
    in torch fp32, from the model's own weights (`weights` from
    reference_weights(model), or made here)."""

    # Matmuls of this many rows or more run on the library's tensor-core
    # GEMM, whose weights are rounded to fp16 ((q - z) * d, as the reference's
    # f16 prompt route rounds them): the restatement rounds them too.
    GEMM_ROWS = 17

    def __init__(self, model, weights=None):
        self.m = model
        cfg = model.cfg
        weights = weights or reference_weights(model)
        self.W = weights["layers"]
        self.head = weights["head"]
        n_attn = sum(t == "attn" for t in cfg.layer_types)
        n_conv = sum(t == "conv" for t in cfg.layer_types)
        self.k = [torch.zeros((cfg.kv_heads, model.max_ctx, cfg.head_dim), dtype=torch.float16, device="cuda")
                  for _ in range(n_attn)]
        self.v = [torch.zeros_like(t) for t in self.k]
        self.state = [torch.zeros((cfg.conv_width - 1, cfg.hidden), dtype=torch.float16, device="cuda")
                      for _ in range(n_conv)]
        self.pos = 0

    def forward(self, ids):
        m, cfg = self.m, self.m.cfg
        H, Hkv, Dh, I = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn
        rows = ids.numel()
        x = m.embed[ids.long()].float()
        add = None
        for li, L in enumerate(m.layers):
            W = self.W[li]
            if rows >= self.GEMM_ROWS:
                W = {k: v.half().float() for k, v in W.items()}
            x, h = rmsnorm(x, add, L["norm1"], cfg.eps)
            h = h.half().float()
            if L["type"] == "attn":
                s = L["slot"]
                qkv = h @ W["qkv"].t()
                q, k, v = rope_kv(qkv, H, Hkv, Dh, self.pos, cfg.theta, L.get("q_norm"), L.get("k_norm"), cfg.eps)
                self.k[s][:, self.pos:self.pos + rows] = k.transpose(0, 1)
                self.v[s][:, self.pos:self.pos + rows] = v.transpose(0, 1)
                att = attention(q, self.k[s], self.v[s], self.pos, H, Hkv).half().float().reshape(rows, H * Dh)
                o = att @ W["o"].t()
            else:
                s = L["slot"]
                bcx = h @ W["in"].t()
                cv, self.state[s] = short_conv(bcx, cfg.hidden, cfg.conv_width, L["conv_w"], self.state[s])
                o = cv.half().float() @ W["out"].t()
            x, h = rmsnorm(x, o, L["norm2"], cfg.eps)
            gu = h.half().float() @ W["gu"].t()
            act = swiglu(gu, I).half().float()
            o = act @ W["down"].t()
            add = o
        x, h = rmsnorm(x[-1:], add[-1:], m.final_norm, cfg.eps)
        logits = h.half().float() @ self.head.t()
        self.pos += rows
        return logits[0]


def greedy_or_near_tie(plain, prompts, got, want, tol=1e-2):
    """Checks tokens `got` [batch][n] against plain greedy decoding's `want`
    (from `plain`, a DecoderModel with the target's weights): equal, or
    parting only where plain decoding's own pick was a near tie. At each
    sequence's first difference, plain decoding (which read the same tokens
    until there) must rank its pick above `got`'s token by no more than
    tol * max |logit| — a margin that another accumulation order can
    overturn. Returns the first difference per sequence (None: none)."""
    n = want.shape[1]
    firsts = []
    for b in range(want.shape[0]):
        d = (got[b, :n] != want[b]).nonzero()
        firsts.append(int(d[0]) if d.numel() else None)
    if all(f is None for f in firsts):
        return firsts
    # plain decoding again (deterministic), keeping each step's logits
    plain.reset()
    plain.prefill(prompts)
    logits = [plain.logits.clone()]
    for _ in range(1, max(f for f in firsts if f is not None) + 1):
        plain.decode_step()
        logits.append(plain.logits.clone())
    for b, f in enumerate(firsts):
        if f is None:
            continue
        lg = logits[f][b]
        w, g = int(want[b, f]), int(got[b, f])
        assert int(lg.argmax()) == w, "plain decoding is not deterministic"
        margin = (lg[w] - lg[g]).item() / lg.abs().max().item()
        assert margin <= tol, f"sequence {b}: token {f} is {g}, plain greedy {w} by a margin of {margin:.3e}"
    return firsts
