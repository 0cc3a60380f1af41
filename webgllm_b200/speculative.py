"""Greedy speculative decoding (a 1.1B draft with config
2's layout and the target's vocabulary proposes k = 4 tokens per step).

The reference drafts on the host and verifies with forwardDraft / accept
(packages/webgllm/src/engine.ts:8035,8063). Here one step stays on the GPU
and is captured as one CUDA graph: the draft decodes k + 1 tokens (its own
greedy picks, from the last kept token; the extra step puts d_k in its cache
for when every proposal is kept), the target reads the last kept token and
d_1..d_k as k + 1 rows per sequence and picks after every row, and
wg_spec_accept keeps the longest agreeing prefix plus the target's own next
token, rewinding both models' positions (the KV caches are indexed by
position, so nothing else is undone there); models with gated short-conv
layers (config 3's hybrid) keep their conv state after every draft token
(wg_short_conv_prefixes) and set it back to the kept prefix's
(wg_conv_restore). Every emitted token is the target's greedy pick for
its position as the verify batch computes it, whatever the draft proposes.
A verify batch of more than 16 rows (batch x (k + 1)) runs on the
tensor-core GEMM, whose accumulation order (and fp16 weights) differ from
the decode GEMV's: its logits differ from a plain decode step's at the level
that any change of accumulation order produces in these models (~1e-3
relative, from activations that land on the other side of an fp16
rounding), so a near tie can be picked otherwise than plain greedy decoding
picks it (WG_OPT_EXACT_ROWS routes the verify through the GEMV: fewer such
ties, a slower round).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .model import DecoderConfig, DecoderModel

P = ctypes.c_void_p


def draft_config(target: DecoderConfig) -> DecoderConfig:
    """Config 2's layout with the target's vocabulary."""
    return DecoderConfig("draft-1.1b", 22, 2048, 32, 4, 64, 5632, target.vocab, 1e-5, 1e4)


class SpeculativeDecoder:
    def __init__(self, target: DecoderModel, draft: DecoderModel, k: int = 4, max_new: int = 512):
        if target.batch != draft.batch or target.cfg.vocab != draft.cfg.vocab:
            raise ValueError("target and draft must share batch and vocabulary")
        if target.max_rows < target.batch * (k + 1):
            raise ValueError(f"the target needs max_rows >= {target.batch * (k + 1)}")
        self.t, self.d, self.k = target, draft, k
        B = target.batch
        self.drafts = torch.zeros((B, max(k, 1)), dtype=torch.int32, device="cuda")
        self.picks = torch.zeros((k + 1, B), dtype=torch.int32, device="cuda")
        self.ver = torch.zeros((B, k + 1), dtype=torch.int32, device="cuda")
        self.out = torch.zeros((B, max_new + k + 1), dtype=torch.int32, device="cuda")
        self.out_len = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.accepted = torch.zeros(B, dtype=torch.int32, device="cuda")
        # conv models roll their state back to the kept prefix (convPrefixes /
        # accept, src/gpu/kernels.ts:1504, src/engine.ts:8063): positions
        # before the round, and the state after each of the k + 1 draft tokens
        self.pos_t0 = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.pos_d0 = torch.zeros(B, dtype=torch.int32, device="cuda")
        target.keep_prefixes(k + 1)
        draft.keep_prefixes(k + 1)
        self.graph = None

    def prefill(self, prompts: torch.Tensor):
        """Both models read the prompts; the first emitted token is the
        target's pick."""
        self.t.prefill(prompts)
        self.d.prefill(prompts)
        self.out_len.zero_()
        self.accepted.zero_()
        self.out[:, 0].copy_(self.t.next_id)
        self.out_len.fill_(1)
        self.d.next_id.copy_(self.t.next_id)

    def step(self):
        """One draft-and-verify round (every sequence gains 1 .. k + 1 tokens)."""
        t, d, k = self.t, self.d, self.k
        self.ver[:, 0].copy_(t.next_id)
        if d.has_conv:
            self.pos_d0.copy_(d.pos)
        if t.has_conv:
            self.pos_t0.copy_(t.pos)
        for j in range(k + 1):
            d.prefix_slot = j if d.has_conv else None
            try:
                d.decode_step()
            finally:
                d.prefix_slot = None
            if j < k:
                self.drafts[:, j].copy_(d.next_id)
                self.ver[:, j + 1].copy_(d.next_id)
        t.row_picks = self.picks
        t.prefix_slot = 0 if t.has_conv else None
        try:
            t.forward(self.ver.reshape(-1), t.batch * (k + 1))
        finally:
            t.row_picks = None
            t.prefix_slot = None
        L = _lib.lib()
        t._c(L.wg_spec_accept(P(t.ctx.handle), P(self.drafts.data_ptr()), P(self.picks.data_ptr()), t.batch, k,
                              P(t.pos.data_ptr()), P(d.pos.data_ptr()), P(t.next_id.data_ptr()),
                              P(d.next_id.data_ptr()), P(self.out.data_ptr()), self.out.shape[1],
                              P(self.out_len.data_ptr()), P(self.accepted.data_ptr())))
        t.restore_prefix(self.pos_t0)
        d.restore_prefix(self.pos_d0)

    def capture(self):
        """Records step() as one CUDA graph (after one eager step)."""
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()

    def run_step(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.step()
