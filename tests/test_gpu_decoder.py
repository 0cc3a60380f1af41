"""Parity of the decoder-layer kernels (include/webgllm_decoder.h) with plain
PyTorch fp32 references of the same ops (tests/decoder_reference.py), and of
a whole random-init decoder (webgllm_b200.model) with the reference forward.

Tolerances: fp16 outputs within 2e-3 relative to the output's scale
(fp16 rounding is 4.9e-4 relative; the rest is accumulation order);
integer outputs (embedding copies, argmax, positions) exact.
"""
import math

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import ctypes  # noqa: E402

import decoder_reference as R  # noqa: E402
import webgllm_b200 as wg  # noqa: E402
from webgllm_b200 import _lib  # noqa: E402
from webgllm_b200._lib import WG_F16, WG_F32  # noqa: E402

P = ctypes.c_void_p


def lib():
    return _lib.lib()


def ctx():
    c = wg.context()
    c.use_torch_stream()
    return c


def call(fn, *args):
    c = ctx()
    _lib.check(fn(P(c.handle), *args), c.handle)
    torch.cuda.synchronize()


def ptr(t):
    return P(t.data_ptr()) if t is not None else P(None)


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


# ------------------------------------------------------------------ kernels


def test_embed_copies_rows_exactly():
    V, D = 1000, 256
    g = gen(1)
    table = torch.randn((V, D), generator=g, device="cuda").half()
    ids = torch.tensor([5, 0, 999, 5, -3, 1000], dtype=torch.int32, device="cuda")
    out = torch.empty((ids.numel(), D), device="cuda")
    call(lib().wg_embed, ptr(ids), ids.numel(), ptr(table), V, D, ptr(out))
    want = table[ids.clamp(0, V - 1).long()].float()
    want[4] = table[0].float()  # out of range reads row 0
    want[5] = table[0].float()
    assert torch.equal(out, want)


@pytest.mark.parametrize("rows,D,with_add", [(1, 2048, True), (7, 1536, False), (64, 4096, True), (3, 100, True)])
def test_rmsnorm_fused_add(rows, D, with_add):
    g = gen(rows + D)
    x = torch.randn((rows, D), generator=g, device="cuda")
    add = torch.randn((rows, D), generator=g, device="cuda") if with_add else None
    w = torch.rand(D, generator=g, device="cuda") + 0.5
    x0 = x.clone()
    out = torch.empty((rows, D), dtype=torch.float16, device="cuda")
    call(lib().wg_rmsnorm, ptr(x), ptr(add), ptr(w), ctypes.c_float(1e-5), rows, D, ptr(out), WG_F16)
    xr, want = R.rmsnorm(x0, add, w, 1e-5)
    assert torch.allclose(x, xr, rtol=0, atol=1e-6 * xr.abs().max().item())
    assert rel(out, want) < 2e-3


@pytest.mark.parametrize("rows,H,Hkv,Dh,pos0,qk", [
    (1, 32, 4, 64, 0, False), (1, 32, 4, 64, 777, False), (5, 24, 8, 64, 100, True), (3, 32, 8, 128, 4000, False),
    (48, 8, 2, 64, 16, True),
])
def test_rope_kv_append(rows, H, Hkv, Dh, pos0, qk):
    g = gen(rows * 31 + H + Dh)
    cache_len = 4096 + 64
    qkv = torch.randn((rows, (H + 2 * Hkv) * Dh), generator=g, device="cuda")
    qn = torch.rand(Dh, generator=g, device="cuda") + 0.5 if qk else None
    kn = torch.rand(Dh, generator=g, device="cuda") + 0.5 if qk else None
    pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
    q = torch.empty((rows, H, Dh), dtype=torch.float16, device="cuda")
    kc = torch.zeros((Hkv, cache_len, Dh), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    call(lib().wg_rope_kv, ptr(qkv), rows, 1, H, Hkv, Dh, ptr(pos), ctypes.c_float(1e4 if Dh == 64 else 5e5),
         ptr(qn), ptr(kn), ctypes.c_float(1e-5), ptr(q), ptr(kc), ptr(vc), cache_len)
    wq, wk, wv = R.rope_kv(qkv, H, Hkv, Dh, pos0, 1e4 if Dh == 64 else 5e5, qn, kn, 1e-5)
    assert rel(q, wq) < 2e-3
    assert rel(kc[:, pos0:pos0 + rows].transpose(0, 1), wk) < 2e-3
    assert torch.equal(vc[:, pos0:pos0 + rows].transpose(0, 1), wv)
    # nothing else in the caches was written
    assert not kc[:, :pos0].any() and not kc[:, pos0 + rows:].any()


def test_rope_kv_position_past_cache_is_reported():
    H, Hkv, Dh, cache_len = 4, 2, 64, 16
    qkv = torch.randn((2, (H + 2 * Hkv) * Dh), device="cuda")
    pos = torch.tensor([15], dtype=torch.int32, device="cuda")  # row 1 lands at 16
    q = torch.empty((2, H, Dh), dtype=torch.float16, device="cuda")
    kc = torch.zeros((Hkv, cache_len, Dh), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    c = ctx()
    assert lib().wg_rope_kv(P(c.handle), ptr(qkv), 2, 1, H, Hkv, Dh, ptr(pos), ctypes.c_float(1e4), None, None,
                            ctypes.c_float(1e-5), ptr(q), ptr(kc), ptr(vc), cache_len) == 0
    with pytest.raises(wg.GpuError):
        c.sync()
    c.sync()  # the flag is cleared once reported
    assert kc[:, 15].any()


@pytest.mark.parametrize("rows,H,Hkv,Dh,pos0", [
    (1, 32, 4, 64, 0), (1, 32, 4, 64, 1023), (1, 24, 8, 64, 300), (1, 32, 8, 128, 2047), (4, 16, 2, 64, 517),
    (40, 8, 8, 64, 0), (1, 16, 1, 256, 130), (2, 6, 2, 32, 70),
    # prompts (>= 16 rows a sequence, Dh 64 / 128): the tensor-core flash kernel
    (64, 32, 8, 128, 0), (100, 32, 8, 128, 37), (200, 16, 2, 64, 500), (17, 8, 1, 64, 3), (130, 24, 8, 64, 1800),
])
def test_attention_causal_gqa(rows, H, Hkv, Dh, pos0):
    g = gen(rows * 7 + H * 3 + pos0)
    cache_len = 2048 + 16
    L = pos0 + rows
    kc = torch.zeros((Hkv, cache_len, Dh), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    kc[:, :L] = (torch.randn((Hkv, L, Dh), generator=g, device="cuda") * 2).half()
    vc[:, :L] = torch.randn((Hkv, L, Dh), generator=g, device="cuda").half()
    # a poisoned tail: keys past each row's position must not be read
    kc[:, L:L + 8] = 1e4
    vc[:, L:L + 8] = float("nan")
    q = (torch.randn((rows, H, Dh), generator=g, device="cuda") / math.sqrt(Dh)).half()
    pos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
    out = torch.empty((rows, H, Dh), dtype=torch.float16, device="cuda")
    call(lib().wg_attention, ptr(q), rows, 1, H, Hkv, Dh, ptr(kc), ptr(vc), cache_len, ptr(pos), ptr(out))
    want = R.attention(q, kc, vc, pos0, H, Hkv)
    assert torch.isfinite(out.float()).all()
    assert (out.float() - want).abs().max().item() < 2e-3 * max(1.0, want.abs().max().item())


@pytest.mark.parametrize("Dh,H,Hkv", [(128, 32, 8), (64, 32, 4)])
def test_flash_prefill_batched_sequences(Dh, H, Hkv):
    """Prompts of 3 sequences (70 rows each, at their own positions and
    caches) through the flash kernel: each equals the single-sequence
    reference."""
    B, rps, cache_len = 3, 70, 512
    g = gen(Dh + H)
    pos0 = [0, 130, 400]
    kc = torch.zeros((B, Hkv, cache_len, Dh), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    for b in range(B):
        L = pos0[b] + rps
        kc[b, :, :L] = (torch.randn((Hkv, L, Dh), generator=g, device="cuda") * 2).half()
        vc[b, :, :L] = torch.randn((Hkv, L, Dh), generator=g, device="cuda").half()
    q = (torch.randn((B * rps, H, Dh), generator=g, device="cuda") / math.sqrt(Dh)).half()
    pos = torch.tensor(pos0, dtype=torch.int32, device="cuda")
    out = torch.empty((B * rps, H, Dh), dtype=torch.float16, device="cuda")
    call(lib().wg_attention, ptr(q), B * rps, B, H, Hkv, Dh, ptr(kc), ptr(vc), cache_len, ptr(pos), ptr(out))
    for b in range(B):
        want = R.attention(q[b * rps:(b + 1) * rps], kc[b], vc[b], pos0[b], H, Hkv)
        got = out[b * rps:(b + 1) * rps].float()
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() < 2e-3 * max(1.0, want.abs().max().item()), b


def test_rope_and_attention_batched_sequences():
    """3 independent sequences of 2 rows each, at different positions, with
    their own caches: each equals the single-sequence computation."""
    B, rps, H, Hkv, Dh, cache_len = 3, 2, 8, 2, 64, 512
    rows = B * rps
    g = gen(31)
    pos0 = [5, 200, 0]
    qkv = torch.randn((rows, (H + 2 * Hkv) * Dh), generator=g, device="cuda")
    kc = (torch.randn((B, Hkv, cache_len, Dh), generator=g, device="cuda")).half()
    vc = torch.randn((B, Hkv, cache_len, Dh), generator=g, device="cuda").half()
    kc0, vc0 = kc.clone(), vc.clone()
    pos = torch.tensor(pos0, dtype=torch.int32, device="cuda")
    q = torch.empty((rows, H, Dh), dtype=torch.float16, device="cuda")
    out = torch.empty((rows, H, Dh), dtype=torch.float16, device="cuda")
    call(lib().wg_rope_kv, ptr(qkv), rows, B, H, Hkv, Dh, ptr(pos), ctypes.c_float(1e4), None, None,
         ctypes.c_float(1e-5), ptr(q), ptr(kc), ptr(vc), cache_len)
    call(lib().wg_attention, ptr(q), rows, B, H, Hkv, Dh, ptr(kc), ptr(vc), cache_len, ptr(pos), ptr(out))
    for b in range(B):
        sl = slice(b * rps, (b + 1) * rps)
        wq, wk, wv = R.rope_kv(qkv[sl], H, Hkv, Dh, pos0[b], 1e4)
        assert rel(q[sl], wq) < 2e-3
        ref_k, ref_v = kc0[b].clone(), vc0[b].clone()
        ref_k[:, pos0[b]:pos0[b] + rps] = wk.transpose(0, 1)
        ref_v[:, pos0[b]:pos0[b] + rps] = wv.transpose(0, 1)
        assert rel(kc[b], ref_k) < 2e-3 and torch.equal(vc[b], ref_v)
        want = R.attention(q[sl], kc[b], vc[b], pos0[b], H, Hkv)
        assert (out[sl].float() - want).abs().max().item() < 2e-3 * max(1.0, want.abs().max().item())


@pytest.mark.parametrize("B,H,Hkv,Dh,qk", [(1, 32, 4, 64, False), (3, 24, 8, 64, True), (8, 32, 8, 128, False),
                                         (2, 16, 1, 256, True)])
def test_rope_attention_equals_the_two_kernels(B, H, Hkv, Dh, qk):
    """The fused decode launch gives the same caches and outputs as wg_rope_kv
    followed by wg_attention."""
    g = gen(B * 100 + H + Dh)
    cache_len = 700
    pos0 = [int(v) for v in torch.randint(0, 650, (B,), generator=torch.Generator().manual_seed(B))]
    qkv = torch.randn((B, (H + 2 * Hkv) * Dh), generator=g, device="cuda")
    qn = torch.rand(Dh, generator=g, device="cuda") + 0.5 if qk else None
    kn = torch.rand(Dh, generator=g, device="cuda") + 0.5 if qk else None
    kc = torch.randn((B, Hkv, cache_len, Dh), generator=g, device="cuda").half()
    vc = torch.randn_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    pos = torch.tensor(pos0, dtype=torch.int32, device="cuda")
    q = torch.empty((B, H, Dh), dtype=torch.float16, device="cuda")
    out1 = torch.empty((B, H, Dh), dtype=torch.float16, device="cuda")
    out2 = torch.empty_like(out1)
    call(lib().wg_rope_kv, ptr(qkv), B, B, H, Hkv, Dh, ptr(pos), ctypes.c_float(1e4), ptr(qn), ptr(kn),
         ctypes.c_float(1e-5), ptr(q), ptr(kc), ptr(vc), cache_len)
    call(lib().wg_attention, ptr(q), B, B, H, Hkv, Dh, ptr(kc), ptr(vc), cache_len, ptr(pos), ptr(out1))
    call(lib().wg_rope_attention, ptr(qkv), B, H, Hkv, Dh, ptr(pos), ctypes.c_float(1e4), ptr(qn), ptr(kn),
         ctypes.c_float(1e-5), ptr(kc2), ptr(vc2), cache_len, ptr(out2))
    assert torch.equal(vc2, vc)
    # keys: the qk-norm's sum runs in another order (a warp, not the CTA)
    assert (kc2.float() - kc.float()).abs().max().item() <= 1e-3 * kc.float().abs().max().item()
    if not qk:
        assert torch.equal(kc2, kc)
    assert (out2.float() - out1.float()).abs().max().item() <= 2e-3 * max(1.0, out1.float().abs().max().item())


def test_short_conv_batched_states():
    B, rps, D, W = 2, 5, 256, 3
    g = gen(5)
    bcx = torch.randn((B * rps, 3 * D), generator=g, device="cuda")
    w = torch.randn((D, W), generator=g, device="cuda") * 0.3
    state = torch.randn((B, W - 1, D), generator=g, device="cuda").half()
    st0 = state.clone()
    out = torch.empty((B * rps, D), dtype=torch.float16, device="cuda")
    call(lib().wg_short_conv, ptr(bcx), B * rps, B, D, W, ptr(w), ptr(state), ptr(out), WG_F16)
    for b in range(B):
        want, want_state = R.short_conv(bcx[b * rps:(b + 1) * rps], D, W, w, st0[b])
        assert rel(out[b * rps:(b + 1) * rps], want) < 2e-3
        assert rel(state[b], want_state) < 1e-3


def test_head_rmsnorm_shards_rows_and_keys():
    """Two vocabulary shards of one head over 3 strided rows: the int64 MAX of
    the shards' keys picks the full head's argmax; pick_keys decodes it."""
    from webgllm_b200 import tp as TP

    rows, stride, D, V = 3, 4, 512, 3000
    g = gen(77)
    resid = torch.randn((rows * stride, D), generator=g, device="cuda")
    add = torch.randn((rows * stride, D), generator=g, device="cuda")
    w = torch.rand(D, generator=g, device="cuda") + 0.5
    W = (torch.randn((V, D), generator=g, device="cuda") * 0.05).half()
    _, h = R.rmsnorm(resid[stride - 1::stride], add[stride - 1::stride], w, 1e-5)
    full = h.half().float() @ W.float().t()
    keys = []
    for k0, k1 in [(0, 1700), (1700, 3000)]:
        lg = torch.empty((rows, k1 - k0), device="cuda")
        key = torch.empty(rows, dtype=torch.int64, device="cuda")
        ids = torch.empty(rows, dtype=torch.int32, device="cuda")
        Ws = W[k0:k1].contiguous()
        call(lib().wg_head_rmsnorm, ptr(resid[stride - 1]), ptr(add[stride - 1]), ptr(w), ctypes.c_float(1e-5), rows,
             stride, D, ptr(Ws), k1 - k0, k0, ptr(lg), ptr(ids), ptr(key))
        assert rel(lg, full[:, k0:k1]) < 2e-3
        assert torch.equal(ids.long(), lg.argmax(dim=1) + k0)  # global indices
        for r in range(rows):
            v = lg[r, ids[r] - k0].item()
            assert key[r].item() == TP.argmax_key(v, ids[r].item())
        keys.append(key)
    best = torch.maximum(keys[0], keys[1])
    picked = torch.empty(rows, dtype=torch.int32, device="cuda")
    call(lib().wg_pick_keys, ptr(best), rows, ptr(picked))
    got_full = torch.cat([full[:, :1700], full[:, 1700:]], dim=1)
    assert torch.equal(picked.long(), got_full.argmax(dim=1))


@pytest.mark.parametrize("rows,I,dt", [(1, 5632, WG_F16), (33, 4608, WG_F16), (2, 100, WG_F32)])
def test_swiglu(rows, I, dt):
    gu = torch.randn((rows, 2 * I), generator=gen(I), device="cuda") * 3
    out = torch.empty((rows, I), dtype=torch.float16 if dt == WG_F16 else torch.float32, device="cuda")
    call(lib().wg_swiglu, ptr(gu), rows, I, ptr(out), dt)
    assert rel(out, R.swiglu(gu, I)) < (2e-3 if dt == WG_F16 else 1e-5)


@pytest.mark.parametrize("rows,D,W", [(1, 1536, 3), (17, 1536, 3), (5, 300, 4), (2, 64, 1)])
def test_short_conv_and_state(rows, D, W):
    g = gen(rows + D + W)
    bcx = torch.randn((rows, 3 * D), generator=g, device="cuda")
    w = torch.randn((D, W), generator=g, device="cuda") * 0.3
    state = torch.randn((max(W - 1, 1), D), generator=g, device="cuda").half()
    st0 = state.clone()
    out = torch.empty((rows, D), dtype=torch.float16, device="cuda")
    call(lib().wg_short_conv, ptr(bcx), rows, 1, D, W, ptr(w), ptr(state), ptr(out), WG_F16)
    want, want_state = R.short_conv(bcx, D, W, w, st0[: W - 1] if W > 1 else st0[:0])
    assert rel(out, want) < 2e-3
    if W > 1:
        assert rel(state, want_state) < 1e-3
    # a second call continues from the state: same as one call over both
    bcx2 = torch.randn((3, 3 * D), generator=g, device="cuda")
    out2 = torch.empty((3, D), dtype=torch.float16, device="cuda")
    call(lib().wg_short_conv, ptr(bcx2), 3, 1, D, W, ptr(w), ptr(state), ptr(out2), WG_F16)
    both, _ = R.short_conv(torch.cat([bcx, bcx2]), D, W, w, st0[: W - 1] if W > 1 else st0[:0])
    assert rel(out2, both[rows:]) < 2e-3


@pytest.mark.parametrize("rows,D,V", [(1, 2048, 32000), (3, 1536, 65536), (8, 4096, 1000), (1, 64, 7)])
def test_head_and_argmax(rows, D, V):
    g = gen(rows + D + V)
    x = torch.randn((rows, D), generator=g, device="cuda").half()
    W = (torch.randn((V, D), generator=g, device="cuda") * 0.02).half()
    logits = torch.empty((rows, V), device="cuda")
    fused = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    call(lib().wg_head, ptr(x), rows, D, ptr(W), V, ptr(logits), ptr(fused))
    want = x.float() @ W.float().t()
    assert rel(logits, want) < 1e-4
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    call(lib().wg_argmax, ptr(logits), rows, V, ptr(ids))
    assert torch.equal(ids.long(), logits.argmax(dim=1))
    assert torch.equal(fused, ids)
    # again (the fused pick's counter must have been reset), without argmax
    fused.fill_(-1)
    call(lib().wg_head, ptr(x), rows, D, ptr(W), V, ptr(logits), ptr(fused))
    assert torch.equal(fused, ids)
    call(lib().wg_head, ptr(x), rows, D, ptr(W), V, ptr(logits), None)


def test_argmax_picks_the_lowest_index_on_ties():
    V = 50000
    logits = torch.zeros((2, V), device="cuda")
    logits[0, [7, 123, 40000]] = 5.0
    logits[1, :] = -1.0
    ids = torch.empty(2, dtype=torch.int32, device="cuda")
    call(lib().wg_argmax, ptr(logits), 2, V, ptr(ids))
    assert ids.tolist() == [7, 0]


@pytest.mark.parametrize("rows,D,V,with_add", [(1, 2048, 32000, True), (3, 1536, 5000, False)])
def test_head_rmsnorm_is_norm_then_head(rows, D, V, with_add):
    g = gen(rows * D + V)
    resid = torch.randn((rows, D), generator=g, device="cuda")
    add = torch.randn((rows, D), generator=g, device="cuda") if with_add else None
    w = torch.rand(D, generator=g, device="cuda") + 0.5
    W = (torch.randn((V, D), generator=g, device="cuda") * 0.02).half()
    r0 = resid.clone()
    logits = torch.empty((rows, V), device="cuda")
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    call(lib().wg_head_rmsnorm, ptr(resid), ptr(add), ptr(w), ctypes.c_float(1e-5), rows, 1, D, ptr(W), V, 0,
         ptr(logits), ptr(ids), None)
    assert torch.equal(resid, r0)  # not written
    _, h = R.rmsnorm(r0, add, w, 1e-5)
    want = h.half().float() @ W.float().t()
    assert rel(logits, want) < 2e-3
    assert torch.equal(ids.long(), logits.argmax(dim=1))


@pytest.mark.parametrize("D", [64, 128])  # the CUDA-core kernel; the TMA-ring tensor-core kernel (D % 128 == 0)
def test_head_fused_argmax_ties_pick_the_lowest_index(D):
    V = 5000
    x = torch.ones((1, D), dtype=torch.float16, device="cuda")
    W = torch.zeros((V, D), dtype=torch.float16, device="cuda")
    logits = torch.empty((1, V), device="cuda")
    ids = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    call(lib().wg_head, ptr(x), 1, D, ptr(W), V, ptr(logits), ptr(ids))
    assert ids.item() == 0  # all logits equal
    W[4000] = 0.5
    W[10] = 0.5
    call(lib().wg_head, ptr(x), 1, D, ptr(W), V, ptr(logits), ptr(ids))
    assert ids.item() == 10


def test_add_i32():
    c = torch.tensor([41], dtype=torch.int32, device="cuda")
    call(lib().wg_add_i32, ptr(c), 1, 1)
    call(lib().wg_add_i32, ptr(c), 1, -2)
    assert c.item() == 40
    v = torch.arange(100, dtype=torch.int32, device="cuda")
    call(lib().wg_add_i32, ptr(v), 100, 7)
    assert torch.equal(v, torch.arange(100, dtype=torch.int32, device="cuda") + 7)


def test_decoder_shape_errors():
    c = ctx()
    x = torch.zeros(16, device="cuda")
    assert lib().wg_attention(P(c.handle), ptr(x), 1, 1, 33, 4, 64, ptr(x), ptr(x), 8, ptr(x), ptr(x)) == \
        _lib.WG_INVALID_SHAPE
    assert lib().wg_attention(P(c.handle), ptr(x), 3, 2, 8, 4, 64, ptr(x), ptr(x), 8, ptr(x), ptr(x)) == \
        _lib.WG_INVALID_SHAPE  # rows not a multiple of batch
    assert lib().wg_head(P(c.handle), ptr(x), 9, 64, ptr(x), 10, ptr(x), None) == _lib.WG_INVALID_SHAPE
    assert lib().wg_rope_kv(P(c.handle), ptr(x), 1, 1, 4, 2, 48, ptr(x), ctypes.c_float(1e4), None, None,
                            ctypes.c_float(1e-5), ptr(x), ptr(x), ptr(x), 8) == _lib.WG_INVALID_SHAPE
    assert lib().wg_short_conv(P(c.handle), ptr(x), 1, 1, 4, 9, ptr(x), ptr(x), ptr(x), WG_F16) == \
        _lib.WG_INVALID_SHAPE


# ------------------------------------------------------------------ a whole decoder


def small_config(hybrid):
    from webgllm_b200.model import DecoderConfig

    if hybrid:
        return DecoderConfig("tiny-hybrid", 4, 256, 8, 2, 64, 512, 1000, 1e-5, 1e6, ["conv", "attn", "conv", "attn"], 3,
                             True)
    return DecoderConfig("tiny-llama", 3, 256, 8, 2, 64, 768, 1000, 1e-5, 1e4)


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("hybrid", [False, True])
def test_decoder_matches_reference_forward(hybrid, fused):
    """Prefill 40 tokens (the tcgen05 GEMM path) then 6 decode steps (the
    GEMV path, replayed from a CUDA graph) against the torch fp32 forward:
    logits within 2% of their scale, and the same greedy tokens wherever the
    reference's top-2 margin is clear."""
    from webgllm_b200.model import DecoderModel

    cfg = small_config(hybrid)
    torch.manual_seed(0)
    m = DecoderModel(cfg, seed=3, max_ctx=128, max_rows=64, keep_blocks=True, fused=fused)
    ref = R.ReferenceDecoder(m)
    prompt = torch.randint(0, cfg.vocab, (40,), generator=gen(9), device="cuda").to(torch.int32)
    m.prefill(prompt)
    torch.cuda.synchronize()
    want = ref.forward(prompt)
    scale = want.abs().max().item()
    assert (m.logits[0] - want).abs().max().item() < 2e-2 * scale
    tok = m.next_id.clone()
    m.decode_step()  # eager first step configures every kernel
    m.capture_decode()
    for step in range(6):
        want_next = ref.forward(tok)
        if step == 0:
            pass  # the eager step above already ran this token
        else:
            m.graph.replay()
        torch.cuda.synchronize()
        got = m.logits[0]
        s = want_next.abs().max().item()
        assert (got - want_next).abs().max().item() < 2e-2 * s, step
        top2 = torch.topk(want_next, 2).values
        if (top2[0] - top2[1]).item() > 4e-2 * s:
            assert m.next_id.item() == int(want_next.argmax().item()), step
        # both continue from the library's token
        tok = m.next_id.clone()
    assert m.pos.item() == 40 + 6


@pytest.mark.parametrize("hybrid", [False, True])
def test_decoder_batched_sequences_match_single_runs(hybrid):
    """Two sequences decoding together (per-sequence positions, caches and
    conv states) give each sequence's single-sequence reference logits."""
    from webgllm_b200.model import DecoderModel

    cfg = small_config(hybrid)
    m = DecoderModel(cfg, seed=5, max_ctx=128, max_rows=64, keep_blocks=True, batch=2)
    refs = [R.ReferenceDecoder(m), R.ReferenceDecoder(m)]
    prompts = torch.randint(0, cfg.vocab, (2, 20), generator=gen(4), device="cuda").to(torch.int32)
    m.prefill(prompts)
    torch.cuda.synchronize()
    for b in range(2):
        want = refs[b].forward(prompts[b])
        assert (m.logits[b] - want).abs().max().item() < 2e-2 * want.abs().max().item(), b
    toks = m.next_id.clone()
    m.decode_step()
    m.capture_decode()
    for step in range(4):
        if step:
            m.graph.replay()
        torch.cuda.synchronize()
        for b in range(2):
            want = refs[b].forward(toks[b:b + 1])
            assert (m.logits[b] - want).abs().max().item() < 2e-2 * want.abs().max().item(), (step, b)
        toks = m.next_id.clone()
    assert m.pos.tolist() == [20 + 4, 20 + 4]


# ------------------------------------------------------------------ fused matmul prologues


def _q4(N, K, seed):
    from webgllm_b200.model import dequantize_q4_0, quantize_q4_0

    w = torch.randn((N, K), generator=gen(seed), device="cuda") * 0.02
    blocks = quantize_q4_0(w)
    m = wg.newQuantMatrix(N, K)
    wg.packQ4_0(m, 0, blocks, N)
    torch.cuda.synchronize()
    return m, dequantize_q4_0(blocks, N, K)


def _fused(m, pro, rows, y):
    c = ctx()
    _lib.check(lib().wg_q4_matmul_fused(P(c.handle), P(m.handle), ctypes.byref(pro), rows, ptr(y), WG_F32), c.handle)
    torch.cuda.synchronize()


@pytest.mark.parametrize("rows", [1, 3, 8, 12, 40])
@pytest.mark.parametrize("N,K", [(3072, 2048), (2048, 5632), (512, 4096)])
def test_matmul_fused_rmsnorm(rows, N, K):
    """rmsnorm(a + b) * w feeds the matmul in the same launch (rows <= 8) or
    through the standalone prologue (more rows): y within rel 1e-3 of the
    fp32 product of the fp16-rounded normed input, resid_out == a + b."""
    m, Wd = _q4(N, K, N + K)
    g = gen(rows + K)
    a = torch.randn((rows, K), generator=g, device="cuda")
    b = torch.randn((rows, K), generator=g, device="cuda")
    w = torch.rand(K, generator=g, device="cuda") + 0.5
    out = torch.full((rows, K), float("nan"), device="cuda")
    y = torch.empty((rows, N), device="cuda")
    pro = _lib.wg_prologue(_lib.WG_PRO_RMSNORM, a.data_ptr(), b.data_ptr(), w.data_ptr(), 1e-5, out.data_ptr())
    _fused(m, pro, rows, y)
    assert torch.equal(out, a + b)
    _, h = R.rmsnorm(a, b, w, 1e-5)
    want = h.half().float() @ Wd.t()
    assert rel(y, want) < 1e-3
    # no addend, no residual output
    pro = _lib.wg_prologue(_lib.WG_PRO_RMSNORM, a.data_ptr(), None, w.data_ptr(), 1e-5, None)
    _fused(m, pro, rows, y)
    _, h = R.rmsnorm(a, None, w, 1e-5)
    assert rel(y, h.half().float() @ Wd.t()) < 1e-3


@pytest.mark.parametrize("rows", [2, 5, 8])
@pytest.mark.parametrize("N,K", [(4096, 4096), (4096, 14336), (2048, 5632), (1536, 4608)])
def test_matmul_residual_epilogue_and_stats_prologue(rows, N, K):
    """wg_q4_matmul_residual: resid += x . W^T in the GEMV's epilogue (in
    place) and stats [N/16][rows] = per-16-row sums of squares of the new
    residual (K = 14336: the K split over a cluster, whose columns are then
    summed whole by one CTA each); then a matmul whose RMSNORM prologue takes
    those stats normalises like one that reads the residual itself."""
    m, Wd = _q4(N, K, N + K + rows)
    g = gen(rows * 7 + K)
    x = torch.randn((rows, K), generator=g, device="cuda").half()
    resid = torch.randn((rows, N), generator=g, device="cuda")
    stats = torch.full((N // 16, rows), float("nan"), device="cuda")
    want = resid + x.float() @ Wd.t()
    c = ctx()
    _lib.check(lib().wg_q4_matmul_residual(P(c.handle), P(m.handle), None, ptr(x), WG_F16, rows, ptr(resid),
                                           ptr(stats)), c.handle)
    torch.cuda.synchronize()
    assert rel(resid, want) < 1e-4
    want_stats = (resid * resid).reshape(rows, N // 16, 16).sum(-1).t()
    assert torch.allclose(stats, want_stats, rtol=1e-5, atol=0)
    # the consumer: a [N -> 1024] matmul normalising resid from the stats
    m2, Wd2 = _q4(1024, N, 5)
    w = torch.rand(N, generator=g, device="cuda") + 0.5
    y_stats = torch.empty((rows, 1024), device="cuda")
    y_plain = torch.empty((rows, 1024), device="cuda")
    pro = _lib.wg_prologue(_lib.WG_PRO_RMSNORM, resid.data_ptr(), None, w.data_ptr(), 1e-5, None, stats.data_ptr())
    _fused(m2, pro, rows, y_stats)
    pro = _lib.wg_prologue(_lib.WG_PRO_RMSNORM, resid.data_ptr(), None, w.data_ptr(), 1e-5, None)
    _fused(m2, pro, rows, y_plain)
    _, h = R.rmsnorm(resid, None, w, 1e-5)
    ref = h.half().float() @ Wd2.t()
    assert rel(y_stats, ref) < 1e-3 and rel(y_stats, y_plain) < 1e-3
    # stats reject an addend or a residual output
    pro = _lib.wg_prologue(_lib.WG_PRO_RMSNORM, resid.data_ptr(), resid.data_ptr(), w.data_ptr(), 1e-5, None,
                           stats.data_ptr())
    assert lib().wg_q4_matmul_fused(P(c.handle), P(m2.handle), ctypes.byref(pro), rows, ptr(y_stats), WG_F32) == \
        _lib.WG_INVALID_ARGUMENT


@pytest.mark.parametrize("hybrid", [False, True])
def test_decoder_residual_epilogue_matches_the_fused_forward(hybrid, monkeypatch):
    """Batched decode steps with the residual add in the matmul epilogues
    (norms from the epilogue's statistics; WG_RESIDUAL_EPILOGUE=2 takes it at
    any size) give the same logits as the norm-pass forward, within the
    accumulation-order floor, and match the fp32 reference."""
    from webgllm_b200.model import DecoderModel

    cfg = small_config(hybrid)
    prompts = torch.randint(0, cfg.vocab, (4, 12), generator=gen(41), device="cuda").to(torch.int32)
    logits = {}
    for mode in ("0", "2"):
        monkeypatch.setenv("WG_RESIDUAL_EPILOGUE", mode)
        m = DecoderModel(cfg, seed=6, max_ctx=64, max_rows=64, keep_blocks=True, batch=4)
        m.prefill(prompts)
        steps = []
        for _ in range(3):
            m.decode_step()
            steps.append(m.logits.clone())
        m.decode_step()
        m.capture_decode()  # the residual forward also runs from a graph
        m.graph.replay()
        steps.append(m.logits.clone())
        torch.cuda.synchronize()
        logits[mode] = torch.stack(steps)
    d = (logits["2"] - logits["0"]).float()
    assert (d.norm() / logits["0"].norm()).item() < 5e-3


@pytest.mark.parametrize("rows", [1, 8, 33])
def test_matmul_fused_swiglu(rows):
    N, K = 2048, 5632
    m, Wd = _q4(N, K, 77)
    gu = torch.randn((rows, 2 * K), generator=gen(rows), device="cuda") * 2
    y = torch.empty((rows, N), device="cuda")
    pro = _lib.wg_prologue(_lib.WG_PRO_SWIGLU, gu.data_ptr(), None, None, 0.0, None)
    _fused(m, pro, rows, y)
    want = R.swiglu(gu, K).half().float() @ Wd.t()
    assert rel(y, want) < 1e-3


def test_matmul_fused_rejects_aliasing_and_bad_kind():
    m, _ = _q4(64, 256, 1)
    a = torch.zeros((1, 256), device="cuda")
    w = torch.ones(256, device="cuda")
    y = torch.empty((1, 64), device="cuda")
    c = ctx()
    pro = _lib.wg_prologue(_lib.WG_PRO_RMSNORM, a.data_ptr(), None, w.data_ptr(), 1e-5, a.data_ptr())
    assert lib().wg_q4_matmul_fused(P(c.handle), P(m.handle), ctypes.byref(pro), 1, ptr(y), WG_F32) == \
        _lib.WG_INVALID_ARGUMENT
    pro = _lib.wg_prologue(7, a.data_ptr(), None, w.data_ptr(), 1e-5, None)
    assert lib().wg_q4_matmul_fused(P(c.handle), P(m.handle), ctypes.byref(pro), 1, ptr(y), WG_F32) == \
        _lib.WG_INVALID_ARGUMENT


@pytest.mark.parametrize("rows,I,K", [(1, 2816, 2048), (3, 1024, 8192), (8, 14336 // 8, 4096), (20, 512, 1024)])
def test_matmul_swiglu_pairs_epilogue(rows, I, K):
    """gate|up packed interleaved by 8 (model.swiglu_pairs_perm): the
    epilogue's silu(gate) * up equals SwiGLU of the plain product, with and
    without the norm prologue; wg_swiglu_pairs does the same from a stored
    interleaved product."""
    from webgllm_b200.model import dequantize_q4_0, quantize_q4_0, swiglu_pairs_perm

    g = gen(rows + I + K)
    w = torch.randn((2 * I, K), generator=g, device="cuda") * 0.02
    blocks = quantize_q4_0(w)
    Wd = dequantize_q4_0(blocks, 2 * I, K)
    m = wg.newQuantMatrix(2 * I, K)
    perm = swiglu_pairs_perm(I)
    wg.packQ4_0(m, 0, blocks, 2 * I, perm)
    x = torch.randn((rows, K), generator=g, device="cuda").half()
    act = torch.empty((rows, I), dtype=torch.float16, device="cuda")
    c = ctx()
    _lib.check(lib().wg_q4_matmul_ex(P(c.handle), P(m.handle), None, ptr(x), WG_F16, rows, ptr(act), WG_F16,
                                     _lib.WG_EPI_SWIGLU_PAIRS), c.handle)
    torch.cuda.synchronize()
    want = R.swiglu(x.float() @ Wd.t(), I)
    assert rel(act, want) < 2e-3
    # with the norm prologue
    a = torch.randn((rows, K), generator=g, device="cuda")
    nw = torch.rand(K, generator=g, device="cuda") + 0.5
    pro = _lib.wg_prologue(_lib.WG_PRO_RMSNORM, a.data_ptr(), None, nw.data_ptr(), 1e-5, None)
    _lib.check(lib().wg_q4_matmul_ex(P(c.handle), P(m.handle), ctypes.byref(pro), None, WG_F16, rows, ptr(act),
                                     WG_F16, _lib.WG_EPI_SWIGLU_PAIRS), c.handle)
    torch.cuda.synchronize()
    _, h = R.rmsnorm(a, None, nw, 1e-5)
    assert rel(act, R.swiglu(h.half().float() @ Wd.t(), I)) < 2e-3
    # stored interleaved product, then the pairs pass
    gu = torch.empty((rows, 2 * I), device="cuda")
    _lib.check(lib().wg_q4_matmul(P(c.handle), P(m.handle), ptr(x), WG_F16, rows, ptr(gu), WG_F32), c.handle)
    act2 = torch.empty((rows, I), dtype=torch.float16, device="cuda")
    call(lib().wg_swiglu_pairs, ptr(gu), rows, I, ptr(act2), WG_F16)
    assert rel(act2, want) < 2e-3


@pytest.mark.parametrize("same_draft", [True, False])
def test_speculative_decoding_emits_the_target_greedy_tokens(same_draft):
    """Draft k = 4, verify, accept on the GPU (one CUDA graph per round): the
    emitted tokens equal the target's plain greedy continuation; a draft
    identical to the target has every proposal accepted."""
    from webgllm_b200.model import DecoderConfig, DecoderModel
    from webgllm_b200.speculative import SpeculativeDecoder

    cfg = DecoderConfig("tiny-target", 3, 256, 8, 2, 64, 512, 1000, 1e-5, 1e4)
    dcfg = cfg if same_draft else DecoderConfig("tiny-draft", 2, 128, 2, 1, 64, 256, 1000, 1e-5, 1e4)
    B, k, n_new = 2, 4, 24
    prompts = torch.randint(0, cfg.vocab, (B, 16), generator=gen(21), device="cuda").to(torch.int32)
    plain = DecoderModel(cfg, seed=11, max_ctx=128, max_rows=64, batch=B)
    want = plain.generate(prompts, n_new, use_graph=False)
    t = DecoderModel(cfg, seed=11, max_ctx=128, max_rows=64, batch=B)
    d = DecoderModel(dcfg, seed=11 if same_draft else 12, max_ctx=128, max_rows=64, batch=B)
    spec = SpeculativeDecoder(t, d, k=k, max_new=64)
    spec.prefill(prompts)
    spec.step()  # eager round configures every kernel
    spec.capture()
    rounds = 1
    while int(spec.out_len.min().item()) < n_new and rounds < 40:
        spec.run_step()
        rounds += 1
    torch.cuda.synchronize()
    got = spec.out[:, :n_new]
    assert torch.equal(got, want), (got, want)
    if same_draft:
        # every round keeps all k proposals and adds the target's own token
        assert spec.accepted.tolist() == [k * rounds] * B
        assert spec.out_len.tolist() == [1 + (k + 1) * rounds] * B


@pytest.mark.parametrize("draft_kind", ["independent", "perturbed", "same"])
def test_hybrid_speculative_decoding_rolls_back_the_conv_state(draft_kind):
    """The hybrid (gated short conv + attention) target and draft under
    speculative decoding: every draft step and the target's verify batch keep
    the conv state after each token (wg_short_conv_prefixes) and accept sets
    it back to the kept prefix's (wg_conv_restore; convPrefixes / accept,
    src/gpu/kernels.ts:1504, src/engine.ts:8063). The emitted tokens equal
    the target's plain greedy continuation whether the draft never agrees
    (rollback to one token every round), agrees sometimes (a copy of the
    target with its final norm perturbed: rollbacks to varying prefixes) or
    always (nothing to roll back)."""
    from webgllm_b200.model import DecoderConfig, DecoderModel
    from webgllm_b200.speculative import SpeculativeDecoder

    cfg = small_config(True)
    B, k, n_new = 2, 4, 28
    prompts = torch.randint(0, cfg.vocab, (B, 12), generator=gen(31), device="cuda").to(torch.int32)
    plain = DecoderModel(cfg, seed=13, max_ctx=128, max_rows=64, batch=B)
    want = plain.generate(prompts, n_new, use_graph=False)
    t = DecoderModel(cfg, seed=13, max_ctx=128, max_rows=64, batch=B)
    if draft_kind == "independent":
        dcfg = DecoderConfig("tiny-hybrid-draft", 2, 128, 2, 1, 64, 256, 1000, 1e-5, 1e6, ["conv", "attn"], 3, True)
        d = DecoderModel(dcfg, seed=14, max_ctx=128, max_rows=64, batch=B)
    else:
        d = DecoderModel(cfg, seed=13, max_ctx=128, max_rows=64, batch=B)
        if draft_kind == "perturbed":
            d.final_norm.mul_(1.0 + 2.0 * torch.rand(cfg.hidden, generator=gen(15), device="cuda"))
    spec = SpeculativeDecoder(t, d, k=k, max_new=96)
    spec.prefill(prompts)
    spec.step()
    spec.capture()
    rounds = 1
    while int(spec.out_len.min().item()) < n_new and rounds < 60:
        spec.run_step()
        rounds += 1
    torch.cuda.synchronize()
    assert torch.equal(spec.out[:, :n_new], want), (spec.out[:, :n_new], want)
    acc = spec.accepted.tolist()
    if draft_kind == "same":
        assert acc == [k * rounds] * B
    elif draft_kind == "perturbed":
        assert 0 < sum(acc) < k * rounds * B, (acc, rounds)  # partial prefixes were kept
