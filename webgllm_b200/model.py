"""Random-init decoders of BASELINE configs 2-4 on the B200 kernels.

The reference's engine runs a layer loop of matmul and non-matmul passes
(src/engine.ts:8875-9304 forwardBatch; per layer normInput -> attend |
convolve -> add + norm -> gate|up -> REDUCE_SWIGLU -> down -> add). This module
runs the same structure on the library's kernels: every linear is a Q4_0
matrix through wg_q4_matmul (decode GEMV or tcgen05 GEMM), the rest through
include/webgllm_decoder.h. Weights are random (BASELINE: "random init"),
quantised to Q4_0 by the llama.cpp rule on the device.

A decode step is captured once as a CUDA graph and replayed: the token ids
(argmax) and the positions live on the device, so no host round trip is
needed between tokens. `batch` independent sequences decode together (one
row each), and with `tp` (a webgllm_b200.comm.TensorGroup) the model is split
across the GPUs of a node (webgllm_b200.tp): per layer two row-parallel sums
(the push exchange for decode rows, NCCL's all-reduce through the library
for prompt rows) and one MAX all-reduce for the greedy pick.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import torch

from . import _lib
from . import tp as TP
from .q4 import QuantMatrix, context, newQuantMatrix, packQ4_0
from ._lib import WG_F16, WG_F32, WG_PRO_RMSNORM, WG_PRO_SWIGLU

P = ctypes.c_void_p


@dataclass
class DecoderConfig:
    name: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-5
    theta: float = 1e4
    layer_types: list = field(default_factory=list)  # "attn" | "conv"
    conv_width: int = 3
    qk_norm: bool = False

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = ["attn"] * self.layers
        assert len(self.layer_types) == self.layers


# Decode batches of up to this many sequences run RoPE + KV append inside the
# attention launch (WG_FUSED_ROPE_MAX_ROWS overrides: tuning).
_FUSED_ROPE_MAX_ROWS = int(os.environ.get("WG_FUSED_ROPE_MAX_ROWS", "8"))

# Llama-style 1.1B.
CONFIG2 = DecoderConfig("llama-1.1b", 22, 2048, 32, 4, 64, 5632, 32000, 1e-5, 1e4)
# hybrid conv/attention (LFM2-style): 10 gated short-conv
# layers (kernel 3) and 6 GQA attention layers, placed as in LFM2-350M.
_HYBRID = ["conv", "conv", "attn", "conv", "conv", "attn", "conv", "conv", "attn", "conv", "attn", "conv",
           "attn", "conv", "attn", "conv"]
CONFIG3 = DecoderConfig("hybrid-350m", 16, 1536, 24, 8, 64, 4608, 65536, 1e-5, 1e6, _HYBRID, 3, True)
# BASELINE config 4's target model (Llama-3-8B shape).
CONFIG4 = DecoderConfig("llama3-8b-shape", 32, 4096, 32, 8, 128, 14336, 128256, 1e-5, 5e5)
CONFIGS = {"2": CONFIG2, "3": CONFIG3, "4": CONFIG4}


def quantize_q4_0(w: torch.Tensor) -> torch.Tensor:
    """Float rows [N][K] (device) -> llama.cpp Q4_0 blocks, uint8 [N*K/32*18]
    on the device. Per 32 weights, with max the element of largest magnitude:
    d = max / -8, q = min(15, floor(w / d + 8.5)), d stored as fp16 (round to
    nearest even); byte j holds q[j] low and q[j+16] high."""
    N, K = w.shape
    b = w.float().reshape(N, K // 32, 32)
    idx = b.abs().argmax(dim=2, keepdim=True)
    mx = torch.gather(b, 2, idx)
    d = mx / -8.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp(torch.floor(b * inv + 8.5), 0, 15).to(torch.uint8)
    out = torch.empty((N, K // 32, 18), dtype=torch.uint8, device=w.device)
    out[:, :, 0:2] = d.to(torch.float16).view(torch.uint8).reshape(N, K // 32, 2)
    out[:, :, 2:] = q[:, :, :16] | (q[:, :, 16:] << 4)
    return out.reshape(-1)


def dequantize_q4_0(blocks: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """GGUF Q4_0 blocks -> float32 [N][K], d * (q - 8)."""
    b = blocks.reshape(N, K // 32, 18)
    d = b[:, :, 0:2].contiguous().view(torch.float16).float()
    q = b[:, :, 2:]
    w = torch.cat([(q & 15), (q >> 4)], dim=2).float() - 8.0
    return (w * d).reshape(N, K)


class Linear:
    """A Q4_0 matrix on the device (and its GGUF bytes, for references)."""

    def __init__(self, ctx, blocks: torch.Tensor, N: int, K: int, keep_blocks=False, perm=None):
        self.N, self.K = N, K
        self.m: QuantMatrix = newQuantMatrix(N, K, ctx=ctx)
        ctx.use_torch_stream()
        packQ4_0(self.m, 0, blocks, N, perm)
        torch.cuda.synchronize()
        self.blocks = blocks if keep_blocks else None


def swiglu_pairs_perm(I: int):
    """Row order of a gate|up matrix [2I] for the SwiGLU-pairs epilogue
    (WG_EPI_SWIGLU_PAIRS): destination row 16t + i is gate row 8t + i for
    i < 8 and up row I + 8t + i - 8 otherwise."""
    import numpy as np

    d = np.arange(2 * I)
    t, r = d // 16, d % 16
    return np.where(r < 8, 8 * t + r, I + 8 * t + r - 8).astype(np.int32)


def random_q4(N: int, K: int, gen: torch.Generator, std: float = 0.02) -> torch.Tensor:
    """GGUF Q4_0 bytes of an N x K matrix drawn from N(0, std^2) (device)."""
    w = torch.randn((N, K), generator=gen, device="cuda") * std
    return quantize_q4_0(w)


class DecoderModel:
    """Weights, caches and the forward pass of one decoder on one GPU (or on
    this rank's GPU of a tensor-parallel group).

    tp: None, or this rank's webgllm_b200.comm.TensorGroup; every rank
    draws the same full random weights and keeps its shard (webgllm_b200.tp),
    so the model is the same for every world size."""

    def __init__(self, cfg: DecoderConfig, seed: int = 0, max_ctx: int = 1024, max_rows: int = 512,
                 keep_blocks: bool = False, device: int | None = None, fused: bool = True, batch: int = 1,
                 tp=None, push: bool = True):
        self.cfg = cfg
        self.fused = fused
        self.batch = batch
        self.ctx = context(device)
        self.max_ctx, self.max_rows = max_ctx, max_rows
        self.group = tp
        rank, world = (tp.rank, tp.world) if tp is not None else (0, 1)
        self.world = world
        sh = self.shard = TP.plan(cfg, rank, world) if world > 1 else None
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        D, H, Hkv, Dh, I, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
        self.H = sh.heads if sh else H
        self.Hkv = sh.kv_heads if sh else Hkv
        self.I = sh.ffn if sh else I
        self.V = sh.vocab if sh else V
        self.vocab_offset = sh.vocab_offset if sh else 0
        self.embed = (torch.randn((V, D), generator=g, device="cuda") * 0.02).half()
        head = (torch.randn((V, D), generator=g, device="cuda") * 0.02).half()
        self.head = head[self.vocab_offset:self.vocab_offset + self.V].contiguous()
        del head
        self.final_norm = torch.ones(D, device="cuda")
        self.layers = []
        n_attn = n_conv = 0
        kb = keep_blocks

        def lin(N, K, rows=None, cols=None, perm=None):
            blocks = random_q4(N, K, g)
            if rows is not None:
                blocks, N = TP.q4_rows(blocks, N, K, rows), rows.numel()
            if cols is not None:
                blocks, K = TP.q4_cols(blocks, N, K, *cols), cols[1] - cols[0]
            return Linear(self.ctx, blocks, N, K, kb, perm)

        for t in cfg.layer_types:
            L = {"type": t, "norm1": torch.ones(D, device="cuda"), "norm2": torch.ones(D, device="cuda")}
            if t == "attn":
                L["qkv"] = lin((H + 2 * Hkv) * Dh, D, rows=TP.qkv_rows(cfg, sh) if sh else None)
                L["o"] = lin(D, H * Dh, cols=TP.o_cols(cfg, sh) if sh else None)
                if cfg.qk_norm:
                    L["q_norm"] = torch.ones(Dh, device="cuda")
                    L["k_norm"] = torch.ones(Dh, device="cuda")
                L["slot"] = n_attn
                n_attn += 1
            else:
                L["in"] = lin(3 * D, D)
                L["conv_w"] = torch.randn((D, cfg.conv_width), generator=g, device="cuda") * 0.1
                L["out"] = lin(D, D)
                L["slot"] = n_conv
                n_conv += 1
            # gate|up packed interleaved by 8: SwiGLU runs in the matmul's epilogue
            L["gu"] = lin(2 * I, D, rows=TP.gate_up_rows(cfg, sh) if sh else None,
                          perm=swiglu_pairs_perm(sh.ffn if sh else I))
            L["down"] = lin(D, I, cols=TP.down_cols(cfg, sh) if sh else None)
            self.layers.append(L)
        B = batch
        self.k_cache = torch.zeros((max(n_attn, 1), B, self.Hkv, max_ctx, Dh), dtype=torch.float16, device="cuda")
        self.v_cache = torch.zeros_like(self.k_cache)
        self.conv_state = torch.zeros((max(n_conv, 1), B, cfg.conv_width - 1, D), dtype=torch.float16,
                                      device="cuda")
        # activations for up to max_rows rows
        R = max_rows
        Hl, Hkvl, Il = self.H, self.Hkv, self.I
        self.x = torch.zeros((R, D), device="cuda")                      # residual stream
        self.x2 = torch.zeros((R, D), device="cuda")                     # its other copy (fused path)
        self.h = torch.zeros((R, D), dtype=torch.float16, device="cuda")  # normed input of a matmul
        self.qkv = torch.zeros((R, (Hl + 2 * Hkvl) * Dh), device="cuda")
        self.q = torch.zeros((R, Hl * Dh), dtype=torch.float16, device="cuda")
        self.att = torch.zeros((R, Hl * Dh), dtype=torch.float16, device="cuda")
        self.bcx = torch.zeros((R, 3 * D), device="cuda")
        self.cv = torch.zeros((R, D), dtype=torch.float16, device="cuda")
        self.o = torch.zeros((R, D), device="cuda")
        self.gu = torch.zeros((R, 2 * Il), device="cuda")
        self.act = torch.zeros((R, Il), dtype=torch.float16, device="cuda")
        # the norm statistics a residual-epilogue matmul leaves for the next
        # norm: [D / 16][rows] sums of squares (decode batches of 2-8 rows)
        self.stats = torch.zeros((D // 16, 8), device="cuda")
        self.logits = torch.zeros((B, self.V), device="cuda")
        self.keys = torch.zeros(B, dtype=torch.int64, device="cuda")
        self.pos = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.ids = torch.zeros(R, dtype=torch.int32, device="cuda")
        self.next_id = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.graph = None
        # speculative verification: greedy picks after every row of each
        # sequence, [rows per sequence][batch] (None: the last row only)
        self.row_picks = None
        self.row_keys = None  # their packed keys under tensor parallelism, [rows per sequence][batch]
        # speculative decoding of conv models: the conv state after each draft
        # token ([conv layers][batch][slots][W-1][D]) and where this forward's
        # first row goes (None: not kept)
        self.conv_prefixes = None
        self.prefix_slot = None
        self._resid_mode, self._resid = False, None  # inside _forward_residual
        # row-parallel exchange: the push all-reduce for decode rows, NCCL
        # for the rest (and for everything when push is False)
        self.comm = None
        if world > 1 and push:
            self.comm = tp.push_comm()

    # -- low level ---------------------------------------------------------

    def _c(self, st):
        _lib.check(st, self.ctx.handle)

    def _mm(self, lin: Linear, x: torch.Tensor, y: torch.Tensor, rows: int):
        L = _lib.lib()
        xd = WG_F16 if x.dtype == torch.float16 else WG_F32
        yd = WG_F16 if y.dtype == torch.float16 else WG_F32
        self._c(L.wg_q4_matmul(P(self.ctx.handle), P(lin.m.handle), P(x.data_ptr()), xd, rows, P(y.data_ptr()), yd))

    def _all_reduce(self, t: torch.Tensor, op: str = "sum"):
        if self.world > 1:
            self.group.all_reduce(t, op)

    def reset(self):
        self.pos.zero_()
        self.k_cache.zero_()
        self.v_cache.zero_()
        self.conv_state.zero_()

    def _mm_norm(self, lin: Linear, resid, add, w, resid_out, y: torch.Tensor, rows: int):
        """y = rmsnorm(resid + add) * w . W^T in one launch (decode rows)."""
        pro = _lib.wg_prologue(WG_PRO_RMSNORM, resid.data_ptr(), add.data_ptr() if add is not None else None,
                               w.data_ptr(), self.cfg.eps, resid_out.data_ptr() if resid_out is not None else None)
        self._c(_lib.lib().wg_q4_matmul_fused(P(self.ctx.handle), P(lin.m.handle), ctypes.byref(pro), rows,
                                              P(y.data_ptr()), WG_F32))

    def _gate_up(self, lin: Linear, resid, add, w, resid_out, rows: int):
        """self.act = silu(gate) * up of rmsnorm(resid + add) * w: the norm in
        the matmul's prologue and SwiGLU in its epilogue (decode rows); more
        rows go through the gate|up product and a separate SwiGLU pass."""
        pro = _lib.wg_prologue(WG_PRO_RMSNORM, resid.data_ptr(), add.data_ptr() if add is not None else None,
                               w.data_ptr(), self.cfg.eps, resid_out.data_ptr() if resid_out is not None else None)
        L, c = _lib.lib(), P(self.ctx.handle)
        if rows <= 32:
            self._c(L.wg_q4_matmul_ex(c, P(lin.m.handle), ctypes.byref(pro), None, WG_F16, rows,
                                      P(self.act.data_ptr()), WG_F16, _lib.WG_EPI_SWIGLU_PAIRS))
            return
        self._c(L.wg_q4_matmul_fused(c, P(lin.m.handle), ctypes.byref(pro), rows, P(self.gu.data_ptr()), WG_F32))
        self._c(L.wg_swiglu_pairs(c, P(self.gu.data_ptr()), rows, self.I, P(self.act.data_ptr()), WG_F16))

    def _mm_swiglu(self, lin: Linear, gu, y: torch.Tensor, rows: int):
        pro = _lib.wg_prologue(WG_PRO_SWIGLU, gu.data_ptr(), None, None, 0.0, None)
        self._c(_lib.lib().wg_q4_matmul_fused(P(self.ctx.handle), P(lin.m.handle), ctypes.byref(pro), rows,
                                              P(y.data_ptr()), WG_F32))

    def forward(self, ids: torch.Tensor, rows: int):
        """Runs `rows` tokens (device int32 ids; batch sequences of rows /
        batch tokens each) at the current positions; leaves each sequence's
        last-row logits in self.logits and greedy next token in self.next_id,
        and advances the positions."""
        if rows % self.batch or rows > self.max_rows:
            raise ValueError(f"rows {rows} for batch {self.batch} (max rows {self.max_rows})")
        if self.fused:
            return self._forward_fused(ids, rows)
        return self._forward_passes(ids, rows)

    def _attend(self, lay, rows):
        self._rope_attend(lay, rows)
        self._mm_rowpar(lay["o"], rows, x=self.att)

    def _rope_attend(self, lay, rows):
        """RoPE + KV append + attention into self.att."""
        cfg, L, c = self.cfg, _lib.lib(), P(self.ctx.handle)
        H, Hkv, Dh = self.H, self.Hkv, cfg.head_dim
        s = lay["slot"]
        kc, vc = self.k_cache[s], self.v_cache[s]
        qn, kn = lay.get("q_norm"), lay.get("k_norm")
        # decode of up to 8 sequences: one launch (measured: configs 2 / 3
        # gain 3-5 %; config 4 at batch 8, with the tensor-core attention,
        # 3.07 -> 3.00 ms a step)
        if rows == self.batch and rows <= _FUSED_ROPE_MAX_ROWS and Dh % 64 == 0:
            self._c(L.wg_rope_attention(c, P(self.qkv.data_ptr()), rows, H, Hkv, Dh, P(self.pos.data_ptr()), cfg.theta,
                                        P(qn.data_ptr() if qn is not None else None),
                                        P(kn.data_ptr() if kn is not None else None), cfg.eps, P(kc.data_ptr()),
                                        P(vc.data_ptr()), self.max_ctx, P(self.att.data_ptr())))
            return
        self._c(L.wg_rope_kv(c, P(self.qkv.data_ptr()), rows, self.batch, H, Hkv, Dh, P(self.pos.data_ptr()),
                             cfg.theta, P(qn.data_ptr() if qn is not None else None),
                             P(kn.data_ptr() if kn is not None else None), cfg.eps, P(self.q.data_ptr()),
                             P(kc.data_ptr()), P(vc.data_ptr()), self.max_ctx))
        self._c(L.wg_attention(c, P(self.q.data_ptr()), rows, self.batch, H, Hkv, Dh, P(kc.data_ptr()),
                               P(vc.data_ptr()), self.max_ctx, P(self.pos.data_ptr()), P(self.att.data_ptr())))

    def _mm_rowpar(self, lin: Linear, rows: int, x=None, pro=None):
        """self.o[:rows] = the sum over ranks of this rank's partial x . W^T
        (x given, or made by the prologue `pro`)."""
        D = self.cfg.hidden
        if self.comm is not None and rows <= 8 and rows * D <= self.comm.slot:
            self.comm.push(lin.m, rows, x=x, pro=pro)
            self.comm.reduce(self.o, rows, D)
            return
        if pro is not None:
            self._c(_lib.lib().wg_q4_matmul_fused(P(self.ctx.handle), P(lin.m.handle), ctypes.byref(pro), rows,
                                                  P(self.o.data_ptr()), WG_F32))
        else:
            self._mm(lin, x, self.o, rows)
        self._all_reduce(self.o[:rows])

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    def _residual(self, lin: Linear, x: torch.Tensor, resid: torch.Tensor, rows: int):
        """resid += x . W^T in the matmul's epilogue, leaving the next norm's
        statistics in self.stats."""
        xd = WG_F16 if x.dtype == torch.float16 else WG_F32
        self._c(_lib.lib().wg_q4_matmul_residual(P(self.ctx.handle), P(lin.m.handle), None, P(x.data_ptr()), xd,
                                                 rows, P(resid.data_ptr()), P(self.stats.data_ptr())))

    def _stats_norm(self, resid, w):
        """The prologue x = rmsnorm(resid) * w whose statistics come from the
        last residual-epilogue matmul."""
        return _lib.wg_prologue(WG_PRO_RMSNORM, resid.data_ptr(), None, w.data_ptr(), self.cfg.eps, None,
                                self.stats.data_ptr())

    def _convolve(self, lay, rows):
        cfg, L, c = self.cfg, _lib.lib(), P(self.ctx.handle)
        s = lay["slot"]
        if self.prefix_slot is not None:
            # a draft batch: keep the state after each prefix (speculative accept)
            self._c(L.wg_short_conv_prefixes(c, P(self.bcx.data_ptr()), rows, self.batch, cfg.hidden,
                                             cfg.conv_width, P(lay["conv_w"].data_ptr()),
                                             P(self.conv_state[s].data_ptr()), P(self.cv.data_ptr()), WG_F16,
                                             P(self.conv_prefixes[s].data_ptr()), self.prefix_slot,
                                             self.conv_prefixes.shape[2]))
        else:
            self._c(L.wg_short_conv(c, P(self.bcx.data_ptr()), rows, self.batch, cfg.hidden, cfg.conv_width,
                                    P(lay["conv_w"].data_ptr()), P(self.conv_state[s].data_ptr()),
                                    P(self.cv.data_ptr()), WG_F16))
        if self._resid_mode:
            self._residual(lay["out"], self.cv, self._resid, rows)
        else:
            self._mm(lay["out"], self.cv, self.o, rows)

    @property
    def has_conv(self) -> bool:
        return any(t == "conv" for t in self.cfg.layer_types)

    def keep_prefixes(self, slots: int):
        """Buffers for the conv state after each of `slots` draft tokens
        (speculative decoding; nothing for attention-only models)."""
        if self.has_conv and (self.conv_prefixes is None or self.conv_prefixes.shape[2] != slots):
            n, B, W1, D = self.conv_state.shape
            self.conv_prefixes = torch.zeros((n, B, slots, W1, D), dtype=torch.float16, device="cuda")

    def restore_prefix(self, pos_before: torch.Tensor):
        """After speculative accept: each conv layer's state becomes the one
        after the kept prefix of the last draft batch (kept = self.pos -
        pos_before per sequence, on the device)."""
        if not self.has_conv:
            return
        cfg, L, c = self.cfg, _lib.lib(), P(self.ctx.handle)
        slots = self.conv_prefixes.shape[2]
        for lay in self.layers:
            if lay["type"] != "conv":
                continue
            s = lay["slot"]
            self._c(L.wg_conv_restore(c, P(self.conv_prefixes[s].data_ptr()), slots, self.batch, cfg.hidden,
                                      cfg.conv_width, P(pos_before.data_ptr()), P(self.pos.data_ptr()),
                                      P(self.conv_state[s].data_ptr())))

    def _head(self, cur, add, rows):
        """Final norm + head on each sequence's last row, greedy pick, and the
        position advance."""
        cfg, L, c = self.cfg, _lib.lib(), P(self.ctx.handle)
        B, rps = self.batch, rows // self.batch
        last = rps - 1
        sharded = self.world > 1

        def head(j, argmax, keys):
            self._c(L.wg_head_rmsnorm(c, P(cur[j].data_ptr()), P(add[j].data_ptr() if add is not None else None),
                                      P(self.final_norm.data_ptr()), cfg.eps, B, rps, cfg.hidden,
                                      P(self.head.data_ptr()), self.V, self.vocab_offset, P(self.logits.data_ptr()),
                                      P(argmax), P(keys)))

        if self.row_picks is not None:
            # speculative verification: a pick after every row of each
            # sequence (the last row's logits stay in self.logits); sharded,
            # every row's packed keys go through one MAX all-reduce
            if sharded:
                if self.row_keys is None or self.row_keys.shape[0] < rps:
                    self.row_keys = torch.zeros((rps, B), dtype=torch.int64, device="cuda")
                keys = self.row_keys[:rps]
                for j in range(rps):
                    head(j, None, keys[j].data_ptr())
                self._all_reduce(keys, "max")
                self._c(L.wg_pick_keys(c, P(keys.data_ptr()), rps * B, P(self.row_picks.data_ptr())))
            else:
                for j in range(rps):
                    head(j, self.row_picks[j].data_ptr(), None)
            self.next_id.copy_(self.row_picks[last])
        elif sharded:
            head(last, None, self.keys.data_ptr())
            self._all_reduce(self.keys, "max")
            self._c(L.wg_pick_keys(c, P(self.keys.data_ptr()), B, P(self.next_id.data_ptr())))
        else:
            head(last, self.next_id.data_ptr(), None)
        self._c(L.wg_add_i32(c, P(self.pos.data_ptr()), B, rps))

    def _forward_fused(self, ids: torch.Tensor, rows: int):
        """Each norm runs inside the matmul that consumes it, SwiGLU inside the
        gate|up projection's epilogue and the final norm inside the head: per
        layer the residual stream alternates between self.x and self.x2. Under
        tensor parallelism with the push exchange (decode rows), each
        row-parallel sum arrives together with the residual add and the next
        norm (wg_comm_reduce_norm), and the next matmul takes its fp16 x."""
        cfg, L, c = self.cfg, _lib.lib(), P(self.ctx.handle)
        D = cfg.hidden
        self.ctx.use_torch_stream()
        self._c(L.wg_embed(c, P(ids.data_ptr()), rows, P(self.embed.data_ptr()), cfg.vocab, D, P(self.x.data_ptr())))
        if self._use_residual_epilogue(rows):
            return self._forward_residual(rows)
        cur, other = self.x, self.x2
        fused_ex = self.comm is not None and rows <= 8 and rows * D <= self.comm.slot
        add = None
        normed = False  # self.h already holds the fp16 input of the next q|k|v (or in) projection
        n = len(self.layers)
        for li, lay in enumerate(self.layers):
            proj = self.qkv if lay["type"] == "attn" else self.bcx
            lin = lay["qkv"] if lay["type"] == "attn" else lay["in"]
            if normed:
                self._mm(lin, self.h, proj, rows)
            elif add is None:
                self._mm_norm(lin, cur, None, lay["norm1"], None, proj, rows)
            else:
                self._mm_norm(lin, cur, add, lay["norm1"], other, proj, rows)
                cur, other = other, cur
            if lay["type"] == "attn":
                self._rope_attend(lay, rows)
                if fused_ex:
                    self.comm.push(lay["o"].m, rows, x=self.att)
                    self.comm.reduce_norm(cur, lay["norm2"], cfg.eps, other, self.h, rows, D)
                    cur, other = other, cur
                    self._c(L.wg_q4_matmul_ex(c, P(lay["gu"].m.handle), None, P(self.h.data_ptr()), WG_F16, rows,
                                              P(self.act.data_ptr()), WG_F16, _lib.WG_EPI_SWIGLU_PAIRS))
                else:
                    self._mm_rowpar(lay["o"], rows, x=self.att)
                    self._gate_up(lay["gu"], cur, self.o, lay["norm2"], other, rows)
                    cur, other = other, cur
            else:
                self._convolve(lay, rows)
                self._gate_up(lay["gu"], cur, self.o, lay["norm2"], other, rows)
                cur, other = other, cur
            if fused_ex and li + 1 < n:
                self.comm.push(lay["down"].m, rows, x=self.act)
                self.comm.reduce_norm(cur, self.layers[li + 1]["norm1"], cfg.eps, other, self.h, rows, D)
                cur, other = other, cur
                normed, add = True, None
            else:
                self._mm_rowpar(lay["down"], rows, x=self.act)
                normed, add = False, self.o
        self._head(cur, add, rows)

    # Decode batches whose norm statistics would make every CTA of a fused
    # GEMV read more than this many bytes take the residual epilogue.
    _NORM_FUSE_BYTES = 64 << 10

    def _use_residual_epilogue(self, rows: int) -> bool:
        """On one GPU, a decode batch of 2-8 rows whose norms are too large
        to fuse from the residual alone (each CTA would read rows * D * 8
        bytes): each layer's residual add runs in the epilogue of the matmul
        that makes the addend, which leaves the next norm's statistics for
        the next matmul's prologue — no norm pass of its own."""
        mode = os.environ.get("WG_RESIDUAL_EPILOGUE", "1")  # 0 off, 1 by size, 2 every batch of 2-8 rows
        if mode == "0" or self.world != 1 or self.row_picks is not None or self.prefix_slot is not None:
            return False
        if not 2 <= rows <= 8 or self.cfg.hidden % 16:
            return False
        return mode == "2" or rows * self.cfg.hidden * 8 > self._NORM_FUSE_BYTES

    def _forward_residual(self, rows: int):
        """The fused forward with the residual add in the epilogues (see
        _use_residual_epilogue): per layer q|k|v (norm from the statistics)
        -> attention -> o (+= residual) -> gate|up (norm from the
        statistics, SwiGLU epilogue) -> down (+= residual); the first
        layer's norm reads the embedding rows."""
        cfg, L, c = self.cfg, _lib.lib(), P(self.ctx.handle)
        cur = self.x
        self._resid_mode, self._resid = True, cur
        try:
            for li, lay in enumerate(self.layers):
                proj = self.qkv if lay["type"] == "attn" else self.bcx
                lin = lay["qkv"] if lay["type"] == "attn" else lay["in"]
                if li == 0:
                    self._mm_norm(lin, cur, None, lay["norm1"], None, proj, rows)
                else:
                    pro = self._stats_norm(cur, lay["norm1"])
                    self._c(L.wg_q4_matmul_fused(c, P(lin.m.handle), ctypes.byref(pro), rows, P(proj.data_ptr()),
                                                 WG_F32))
                if lay["type"] == "attn":
                    self._rope_attend(lay, rows)
                    self._residual(lay["o"], self.att, cur, rows)
                else:
                    self._convolve(lay, rows)
                pro = self._stats_norm(cur, lay["norm2"])
                self._c(L.wg_q4_matmul_ex(c, P(lay["gu"].m.handle), ctypes.byref(pro), None, WG_F16, rows,
                                          P(self.act.data_ptr()), WG_F16, _lib.WG_EPI_SWIGLU_PAIRS))
                self._residual(lay["down"], self.act, cur, rows)
        finally:
            self._resid_mode, self._resid = False, None
        self._head(cur, None, rows)

    def _forward_passes(self, ids: torch.Tensor, rows: int):
        """One launch per engine pass (norm, matmul, SwiGLU, ... each on its
        own)."""
        cfg, L, c = self.cfg, _lib.lib(), P(self.ctx.handle)
        D = cfg.hidden
        self.ctx.use_torch_stream()
        self._c(L.wg_embed(c, P(ids.data_ptr()), rows, P(self.embed.data_ptr()), cfg.vocab, D, P(self.x.data_ptr())))
        add = None
        for lay in self.layers:
            self._c(L.wg_rmsnorm(c, P(self.x.data_ptr()), P(add), P(lay["norm1"].data_ptr()), cfg.eps, rows, D,
                                 P(self.h.data_ptr()), WG_F16))
            if lay["type"] == "attn":
                self._mm(lay["qkv"], self.h, self.qkv, rows)
                self._attend(lay, rows)
            else:
                self._mm(lay["in"], self.h, self.bcx, rows)
                self._convolve(lay, rows)
            self._c(L.wg_rmsnorm(c, P(self.x.data_ptr()), P(self.o.data_ptr()), P(lay["norm2"].data_ptr()), cfg.eps,
                                 rows, D, P(self.h.data_ptr()), WG_F16))
            self._mm(lay["gu"], self.h, self.gu, rows)
            self._c(L.wg_swiglu_pairs(c, P(self.gu.data_ptr()), rows, self.I, P(self.act.data_ptr()), WG_F16))
            self._mm(lay["down"], self.act, self.o, rows)
            self._all_reduce(self.o[:rows])
            add = self.o.data_ptr()
        self._head(self.x, self.o, rows)

    def prefill(self, prompts: torch.Tensor):
        """prompts: device ids [batch][T] (or [T] for batch 1)."""
        prompts = prompts.reshape(self.batch, -1)
        rows = prompts.numel()
        if rows > self.max_rows:
            raise ValueError(f"prompt rows {rows} > max_rows {self.max_rows}")
        self.ids[:rows].copy_(prompts.reshape(-1).to(torch.int32))
        self.forward(self.ids, rows)

    def decode_step(self):
        """One greedy token per sequence: input = the last picks (on the
        device)."""
        self.forward(self.next_id, self.batch)

    def capture_decode(self):
        """Records decode_step as a CUDA graph (after one eager step, so that
        every kernel is configured)."""
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):  # captures on a side stream of torch's
            self.decode_step()

    def generate(self, prompts: torch.Tensor, n_new: int, use_graph: bool = True) -> torch.Tensor:
        """Greedy continuation of `prompts` (device ids [batch][T]): returns
        [batch][n_new] ids."""
        out = torch.zeros((self.batch, n_new), dtype=torch.int32, device="cuda")
        self.prefill(prompts)
        if n_new == 0:
            return out
        out[:, 0].copy_(self.next_id)
        for i in range(1, n_new):
            if use_graph and self.graph is not None:
                self.graph.replay()
            else:
                self.decode_step()
            out[:, i].copy_(self.next_id)
        return out
