"""Parity of the BASELINE decoders at their real sizes (configs 2, 3 and 4).

Each case builds the random-init model of its config at full size on one GPU
(config 4 at batch 8, its BASELINE batch), prefills its prompts (the tcgen05
GEMM and the prompt attention), then decodes STEPS greedy tokens per sequence
with the decode step replayed from a CUDA graph (the GEMVs, decode attention,
conv state, head and pick). The torch fp32 forward of
tests/decoder_reference.py runs every sequence on its own from the model's
own dequantised weights (rounded to fp16 where the library's GEMM rounds
them), reading the library's tokens (teacher forcing), so that every step
compares the same inputs.

Stated criteria (north_star: "logits within tolerance plus identical greedy
tokens over a stated prefix for full models"):
- logits, at every one of the TOKENS generated tokens of every sequence:
  ||got - want|| / ||want|| <= LOGIT_REL_L2 and
  max |got - want| <= LOGIT_REL_MAX * max |want|. (The reference engine's
  own numeric gate for a model is a relative error of 1e-2,
  packages/webgllm/src/handler.ts:455, SELF_CHECK_MAX; these are tighter.
  The floor any fp16-activation implementation meets here: the same
  restatement with fp64 instead of fp32 accumulation moves these models'
  logits by 0.7e-3 (4 layers) to 1.2e-3 (16 layers) relative, as
  activations cross fp16 rounding boundaries; measured here: 1.8e-3
  (config 2), 2.1e-3 (config 3), 4.2e-3 (config 4).)
- tokens: the library's greedy token equals the fp32 forward's argmax at
  every one of those TOKENS steps, except where the two disagree inside the
  logit tolerance (the forward's top-2 margin below 2 * LOGIT_REL_MAX *
  max |want|, a near tie that any finite-precision path may resolve either
  way); at most NEAR_TIE_SHARE of a config's tokens (at least 2) may be such
  ties — what the ~1e-3 floor below predicts for these logit spreads.
"""
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import decoder_reference as R  # noqa: E402

STEPS = 32             # decode steps after the prefill's token
TOKENS = STEPS + 1     # generated tokens compared per sequence: the prefill's pick + STEPS
LOGIT_REL_L2 = 6e-3
LOGIT_REL_MAX = 6e-3
NEAR_TIE_SHARE = 0.03

# config: (batch, prompt tokens) — BASELINE's prompt lengths and batches
CASES = {"2": (1, 128), "3": (1, 512), "4": (8, 512)}


def rel(got, want):
    d = (got - want).float()
    return (d.norm() / want.norm()).item(), (d.abs().max() / want.abs().max()).item()


@pytest.mark.parametrize("config", ["2", "3", "4"])
def test_full_size_decoder_matches_fp32_forward(config):
    from webgllm_b200.model import CONFIGS, DecoderModel

    cfg = CONFIGS[config]
    batch, plen = CASES[config]
    m = DecoderModel(cfg, seed=0, max_ctx=plen + STEPS + 8, max_rows=batch * plen, keep_blocks=True, batch=batch)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab, (batch, plen), generator=g).to("cuda", torch.int32)

    # the library: prefill, one eager step (configures every kernel), then
    # the captured decode step
    got_tok = torch.zeros((batch, TOKENS), dtype=torch.int64)
    got_logits = []
    m.prefill(prompts)
    torch.cuda.synchronize()
    got_tok[:, 0] = m.next_id.cpu()
    got_logits.append(m.logits.clone())
    for step in range(1, TOKENS):
        if step == 1:
            m.decode_step()
        else:
            m.graph.replay()
        torch.cuda.synchronize()
        got_tok[:, step] = m.next_id.cpu()
        got_logits.append(m.logits.clone())
        if step == 1:
            m.capture_decode()
    m.graph = None
    assert m.pos.cpu().tolist() == [plen + STEPS] * batch

    # the fp32 forward of each sequence, reading the library's tokens
    W = R.reference_weights(m)
    worst_l2 = worst_max = 0.0
    ties = []
    for b in range(batch):
        ref = R.ReferenceDecoder(m, W)
        want = ref.forward(prompts[b])
        for step in range(TOKENS):
            got = got_logits[step][b]
            l2, mx = rel(got, want)
            worst_l2, worst_max = max(worst_l2, l2), max(worst_max, mx)
            assert l2 <= LOGIT_REL_L2 and mx <= LOGIT_REL_MAX, \
                f"config {config} sequence {b} step {step}: logits rel L2 {l2:.2e}, rel max {mx:.2e}"
            tok, want_tok = int(got_tok[b, step]), int(want.argmax().item())
            if tok != want_tok:
                margin = (want[want_tok] - want[tok]).item()
                bound = 2 * LOGIT_REL_MAX * want.abs().max().item()
                assert margin <= bound, \
                    f"config {config} sequence {b}: token {step} is {tok}, the fp32 forward's {want_tok} " \
                    f"by a margin of {margin:.3e} (> {bound:.3e})"
                ties.append((b, step, margin / want.abs().max().item()))
            if step < STEPS:
                want = ref.forward(torch.tensor([tok], device="cuda", dtype=torch.int32))
        del ref
    print(f"config {config}: worst logits rel L2 {worst_l2:.3e}, rel max {worst_max:.3e} over "
          f"{batch} x {TOKENS} tokens; near ties {ties}")
    assert len(ties) <= max(2, int(NEAR_TIE_SHARE * batch * TOKENS)), ties
    del W
    m.close()
    del m
    torch.cuda.empty_cache()
