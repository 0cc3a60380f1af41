"""The oracle pinned against the reference's own known-answer tests.

Each test ports one test of webgllm's suite (paths inside packages/webgllm/),
with the same inputs and the same expected values, computed the way the
reference test computes them. No GPU needed.
"""
import math

import numpy as np
import pytest

import oracle as O


def _imul(a, b):
    return (a * b) & 0xFFFFFFFF


def _matmulnbits_data(N, K, seed=3):
    """src/repack.test.ts:18-27: random MatMulNBits data from the test's LCG."""
    s = seed

    def nxt():
        nonlocal s
        s = (_imul(s, 1103515245) + 12345) & 0xFFFFFFFF
        return s >> 16

    blocks = K // 32
    quant = np.array([nxt() & 255 for _ in range(N * blocks * 16)], dtype=np.uint8)
    scales = np.array([nxt() & 255 for _ in range(N * blocks * 2)], dtype=np.uint8)
    zp = np.array([nxt() & 255 for _ in range(N * math.ceil(blocks / 2))], dtype=np.uint8)
    return quant, scales, zp, blocks


# -- src/half.test.ts:5-30 ---------------------------------------------------


@pytest.mark.parametrize("v", [0, 1, -1, 0.5, 2, 65504, -65504, 6.103515625e-5,
                               5.960464477539063e-8, 0.333251953125])
def test_half_exact_values_round_trip(v):
    assert O.c_from_half(O.c_to_half(v)) == v


def test_half_rounds_to_nearest_even():
    assert O.c_from_half(O.c_to_half(1 + 2 ** -11)) == 1
    assert O.c_from_half(O.c_to_half(1 + 3 * 2 ** -12)) == 1 + 2 ** -10


def test_half_overflow_nan_signed_zero():
    assert O.c_from_half(O.c_to_half(1e6)) == math.inf
    assert O.c_from_half(O.c_to_half(-1e6)) == -math.inf
    assert math.isnan(O.c_from_half(O.c_to_half(math.nan)))
    z = O.c_from_half(O.c_to_half(-0.0))
    assert z == 0 and math.copysign(1, z) == -1


def test_half_table_values():
    for h in [0, 1, 0x3C00, 0x7BFF, 0x8001, 0xC000, 0x7C00, 0x0400]:
        want = np.array([h], dtype=np.uint16).view(np.float16).astype(np.float64)[0]
        assert O.c_from_half(h) == want
    assert [O.c_from_half(h) for h in (0x3C00, 0xC000, 0x3800)] == [1, -2, 0.5]


def test_bench_to_half_rounds_ties_up():
    # bench/q4-matmul.js:196-213 adds 0x1000 before the shift: a tie goes up,
    # where src/half.ts goes to even. Both agree off ties.
    assert O.c_to_half_bench(1 + 2 ** -11) == 0x3C01
    assert O.c_to_half(1 + 2 ** -11) == 0x3C00
    for v in (0.004, 0.0123, 0.024, 1.5, -3.25):
        assert O.c_to_half_bench(v) == O.c_to_half(v)


# -- src/repack-words.test.ts:5-27 (the Q4_0 case) ----------------------------


@pytest.mark.parametrize("offset", [0, 1, 2, 3])
def test_q4_0_word_copies_unaligned_row_offsets_permutations(offset):
    nbytes, stride = 16, 18
    raw = np.array([(i * 71 + 19) & 255 for i in range(offset + 4 * 2 * stride)], dtype=np.uint8)
    src = raw[offset:]
    perm = [3, 0, 2, 1]
    actual = O.HostQuantMatrix(12, 64)
    want = O.HostQuantMatrix(12, 64)
    target = want.quants.view(np.uint8)
    for i in range(4):
        for b in range(2):
            at = (((4 + i) >> 2) * 2 + b) * 4 + ((4 + i) & 3)
            frm = (perm[i] * 2 + b) * stride
            want.scales[at] = int(src[frm]) | (int(src[frm + 1]) << 8)
            target[at * nbytes:(at + 1) * nbytes] = src[frm + 2:frm + stride]
    O.c_pack_q4_0(actual, 4, np.ascontiguousarray(src), 4, perm)
    assert np.array_equal(actual.quants, want.quants)
    assert np.array_equal(actual.scales, want.scales)


def test_q4_0_shape_and_range_errors():
    # src/repack.ts:21-24 and :47-54, :69
    with pytest.raises(O.OracleError) as e:
        O.HostQuantMatrix(6, 64)
    assert e.value.code == 2
    with pytest.raises(O.OracleError) as e:
        O.HostQuantMatrix(8, 48)
    assert e.value.code == 2
    m = O.HostQuantMatrix(8, 64)
    with pytest.raises(O.OracleError) as e:
        O.c_pack_q4_0(m, 6, np.zeros(4 * 2 * 18, np.uint8), 4)
    assert e.value.code == 3
    with pytest.raises(O.OracleError) as e:
        O.c_pack_q4_0(m, 0, np.zeros(4 * 2 * 18 - 1, np.uint8), 4)
    assert e.value.code == 4


# -- src/repack.test.ts (MatMulNBits) -----------------------------------------


def test_quants_from_raw_matches_pack_matmulnbits():
    # src/repack.test.ts:60-67
    N, K = 12, 128
    quant, scales, zp, _ = _matmulnbits_data(N, K)
    m = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(m, 0, quant, scales, zp, N)
    assert np.array_equal(O.c_quants_from_raw(quant, N, K), m.quants)


@pytest.mark.parametrize("N,K", [(4, 32), (12, 2048), (64, 7680), (8, 64)])
def test_quants_from_raw_shapes_of_the_repacker_test(N, K):
    # src/q4-repacker.test.ts:5-14: the same shapes and data; the reference
    # checks its hand-assembled repacker against quantsFromRaw, here the
    # word-at-a-time quantsFromRaw is checked against packMatMulNBits' bytes.
    raw = np.array([_imul(i + 1, 2654435761) >> 24 for i in range(N * K // 2)], dtype=np.uint8)
    m = O.HostQuantMatrix(N, K)
    O.c_pack_matmulnbits(m, 0, raw, np.zeros(N * K // 16, np.uint8), None, N)
    assert np.array_equal(O.c_quants_from_raw(raw, N, K), m.quants)


def test_zero_points_unpack_low_nibble_first():
    # src/repack.test.ts:98-110
    m = O.HostQuantMatrix(4, 64, with_zeros=True)
    zp = np.array([0x21, 0x43, 0x65, 0x87], dtype=np.uint8)
    O.c_pack_matmulnbits(m, 0, np.zeros(4 * 2 * 16, np.uint8), np.zeros(4 * 2 * 2, np.uint8), zp, 4)
    for r in range(4):
        assert m.zeros[0 * 4 + r] == 2 * r + 1
        assert m.zeros[1 * 4 + r] == 2 * r + 2


def test_rows_land_at_row0():
    # src/repack.test.ts:81-96
    N, K = 8, 64
    a = _matmulnbits_data(4, K, 1)
    b = _matmulnbits_data(4, K, 2)
    m = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(m, 0, a[0], a[1], a[2], 4)
    O.c_pack_matmulnbits(m, 4, b[0], b[1], b[2], 4)
    whole = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(whole, 0, np.concatenate([a[0], b[0]]), np.concatenate([a[1], b[1]]),
                         np.concatenate([a[2], b[2]]), N)
    assert np.array_equal(m.scales, whole.scales)
    assert np.array_equal(m.zeros, whole.zeros)
    assert np.array_equal(m.quants, whole.quants)


def _dequantize_nbits_row(K, quant, scales, zp, n):
    """src/load-onnx.ts:471-501 (4-bit): the independent expected value."""
    blocks = K // 32
    zp_stride = math.ceil(blocks / 2)
    out = np.zeros(K, dtype=np.float32)
    for b in range(blocks):
        sp = (n * blocks + b) * 2
        scale = O.c_from_half(int(scales[sp]) | (int(scales[sp + 1]) << 8))
        zero = (int(zp[n * zp_stride + (b >> 1)]) >> ((b & 1) << 2)) & 15 if zp is not None else 8
        q = (n * blocks + b) * 16
        for j in range(16):
            byte = int(quant[q + j])
            out[b * 32 + 2 * j] = np.float32(scale * ((byte & 15) - zero))
            out[b * 32 + 2 * j + 1] = np.float32(scale * ((byte >> 4) - zero))
    return out


def test_matrix_row_reads_repacked_rows_as_the_loader_dequantizes():
    # src/repack.test.ts:146-170 (the 4-bit packed case)
    N, K = 8, 64
    blocks = K // 32
    seed = 7

    def rand():
        nonlocal seed
        v = float(seed) * 1103515245.0 + 12345.0  # a JS double, not Math.imul
        seed = int(v) % 2 ** 32
        return (seed >> 8) / 2 ** 24

    quant = np.array([int(rand() * 256) for _ in range(N * blocks * 16)], dtype=np.uint8)
    scales = np.zeros(N * blocks * 2, dtype=np.uint8)
    for i in range(N * blocks):
        h = O.c_to_half(0.01 + rand() * 0.1)
        scales[2 * i] = h & 255
        scales[2 * i + 1] = h >> 8
    zp = np.array([int(rand() * 256) for _ in range(N * math.ceil(blocks / 2))], dtype=np.uint8)
    packed = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(packed, 0, quant, scales, zp, N)
    for n in range(N):
        want = _dequantize_nbits_row(K, quant, scales, zp, n)
        assert np.array_equal(O.c_matrix_row(packed, n), want)


# -- src/lfm2-gguf.test.ts:11-20: the constant-block GGUF fixture -------------


def test_constant_q4_0_block_fixture_is_zero_weights():
    # Blocks of bytes (0, 60) = fp16 1.0 and nibble bytes 136 = 0x88 (q = 8).
    N, K = 96, 32
    blocks = np.tile(np.array([0, 60] + [136] * 16, dtype=np.uint8), N * K // 32)
    m = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(m, 0, blocks, N)
    assert np.all(m.scales == 0x3C00)
    assert np.all(m.quants == 0x88888888)
    for n in (0, 37, 95):
        assert np.array_equal(O.c_matrix_row(m, n), np.zeros(K, np.float32))


# -- the oracle's two restatements agree -------------------------------------


@pytest.mark.parametrize("N,K,M", [(4, 32, 1), (12, 96, 3), (64, 256, 5), (256, 2048, 2)])
def test_c_and_numpy_restatements_agree(N, K, M):
    blk = O.config_q4_0_blocks(N, K, N + K)
    m = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(m, 0, blk, N)
    q, s = O.np_pack_q4_0(N, K, blk)
    assert np.array_equal(q, m.quants) and np.array_equal(s, m.scales)
    W = O.np_dequant_gguf(blk, N, K)
    for n in range(0, N, max(1, N // 7)):
        assert np.array_equal(O.c_matrix_row(m, n), W[n].astype(np.float32))
    x = O.config_activations(M, K, 1)
    r = O.c_ref_f64(blk, x, N, K)
    assert np.allclose(r, O.np_ref_f64(blk, x, N, K), rtol=1e-12, atol=1e-12)
    for emul in (O.c_split_emulate(m, x), O.c_prefill_emulate(m, x)):
        l2, mx = O.rel_errors(emul, r)
        assert l2 <= O.TOL and mx <= O.TOL


def test_split_sizing_matches_engine():
    # src/engine.ts:5316-5327 at the config shapes: config 0 (2048x2048) is
    # 512 row groups -> 8 slices of 8 blocks; K = N = 4096 -> 4 x 32.
    assert O.split_slices(2048, 2048) == (8, 8)
    assert O.split_slices(4096, 4096) == (32, 4)
    # blocks / 4 below 1: one slice
    assert O.split_slices(4, 32) == (1, 1)
    # fractional split (6 blocks / 4 = 1.5): kbSlice ceil(6 / 1.5) = 4, 2 slices
    assert O.split_slices(4, 192) == (4, 2)
    # src/engine.ts:4957-4967: K 4096 -> min(4, round(4096 / 512)) = 4 slices
    assert O.quad_slices(4096, 4096) == (32, 4)
    # wide matrices (> 2048 row groups) take 1024-wide slices
    assert O.quad_slices(16384, 4096) == (32, 4)
    assert O.quad_slices(16384, 2048) == (32, 2)


def test_bench_generator_matches_reference_seeding():
    # bench/gpu-bench-worker.js:18-39: mulberry32(1234) drives the bench's
    # random Q4_0 blocks; scales fall in [0.004, 0.024] as fp16.
    rand = O.mulberry32(1234)
    vals = [rand() for _ in range(5)]
    assert all(0 <= v < 1 for v in vals) and len(set(vals)) == 5
    blk = O.bench_random_q4_0(4, 64, O.mulberry32(1234))
    d = blk.reshape(-1, 18)[:, :2].copy().view(np.uint16).reshape(-1)
    dv = O.np_from_half(d)
    assert np.all(dv >= 0.0039) and np.all(dv <= 0.0241)
