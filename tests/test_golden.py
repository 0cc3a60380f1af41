"""The committed golden fixtures (tests/golden/, written by make_golden.py).

* reference_vectors.json: the literals of webgllm's own known-answer tests
  (file:line in each entry), checked here against the oracle. These run on
  any host.
* config0_gemv.npz: BASELINE config 0's outputs from the oracle's two
  restatements, pinned by the digests of their seeded inputs. The CPU tests
  check that the oracle and the input generator still reproduce them; the
  GPU test checks the CUDA GEMV against them through the library.
"""
import hashlib
import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from webgllm_b200 import synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"
VEC = json.loads((GOLDEN / "reference_vectors.json").read_text())


def _imul(a, b):
    return (a * b) & 0xFFFFFFFF


def sha(a: np.ndarray) -> str:
    """As make_golden.py digests the seeded inputs."""
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_half_literals():
    for v in VEC["half_exact_round_trip"]["values"]:
        assert O.c_from_half(O.c_to_half(v)) == v
    for key in ("half_tie_to_even", "half_round_up"):
        assert O.c_from_half(O.c_to_half(VEC[key]["input"])) == VEC[key]["want"]
    for h in VEC["half_table_bits"]["bits"]:
        want = np.array([h], dtype=np.uint16).view(np.float16).astype(np.float64)[0]
        got = O.c_from_half(h)
        assert got == want or (math.isnan(got) and math.isnan(want))
    v = VEC["halves_to_floats"]
    assert [O.c_from_half(h) for h in v["bits"]] == v["want"]


def test_zero_point_literals():
    v = VEC["zero_points_low_nibble_first"]
    N, K = v["N"], v["K"]
    m = O.HostQuantMatrix(N, K, with_zeros=True)
    O.c_pack_matmulnbits(m, 0, np.zeros(N * K // 2, np.uint8), np.zeros(N * K // 16, np.uint8),
                         np.array(v["zp"], np.uint8), N)
    assert list(m.zeros[0:4]) == v["want_block0"]
    assert list(m.zeros[4:8]) == v["want_block1"]


def test_constant_block_literal_is_zero_weights():
    blk = np.array(VEC["constant_q4_0_block"]["block"], np.uint8)
    N, K = 8, 64
    m = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(m, 0, np.tile(blk, N * K // 32), N)
    assert np.all(m.scales == (int(blk[0]) | (int(blk[1]) << 8)))
    for n in range(N):
        assert not np.any(O.c_matrix_row(m, n))


def test_word_copy_literals():
    # src/repack-words.test.ts: the expectation built as that test builds it
    v = VEC["q4_0_word_copies"]
    stride, nbytes, perm, row0 = 18, 16, v["perm"], v["row0"]
    for off in v["offsets"]:
        raw = np.array([(i * v["mul"] + v["add"]) & 255 for i in range(off + 4 * 2 * stride)], np.uint8)
        src = np.ascontiguousarray(raw[off:])
        got = O.HostQuantMatrix(v["N"], v["K"])
        want = O.HostQuantMatrix(v["N"], v["K"])
        target = want.quants.view(np.uint8)
        for i in range(v["rows"]):
            for b in range(2):
                at = (((row0 + i) >> 2) * 2 + b) * 4 + ((row0 + i) & 3)
                frm = (perm[i] * 2 + b) * stride
                want.scales[at] = int(src[frm]) | (int(src[frm + 1]) << 8)
                target[at * nbytes:(at + 1) * nbytes] = src[frm + 2:frm + stride]
        O.c_pack_q4_0(got, row0, src, v["rows"], perm)
        assert np.array_equal(got.quants, want.quants) and np.array_equal(got.scales, want.scales)


@pytest.mark.parametrize("shape", VEC["q4_repacker_shapes"]["shapes"])
def test_repacker_shape_literals(shape):
    N, K = shape
    v = VEC["q4_repacker_shapes"]
    raw = np.array([_imul(i + 1, v["mul"]) >> v["shift"] for i in range(N * K // 2)], np.uint8)
    m = O.HostQuantMatrix(N, K)
    O.c_pack_matmulnbits(m, 0, raw, np.zeros(N * K // 16, np.uint8), None, N)
    assert np.array_equal(O.c_quants_from_raw(raw, N, K), m.quants)


def _config0():
    g = np.load(GOLDEN / "config0_gemv.npz")
    N, K, seed = int(g["N"]), int(g["K"]), int(g["seed"])
    blocks = synthetic.q4_0_blocks(N, K, seed)
    x = synthetic.activations(1, K, seed)
    assert sha(blocks) == str(g["blocks_sha256"]), "the seeded weight generator changed"
    assert sha(x) == str(g["x_sha256"]), "the seeded activation generator changed"
    return g, N, K, blocks, x


def test_config0_golden_outputs_reproduce():
    g, N, K, blocks, x = _config0()
    assert np.array_equal(O.c_ref_f64(blocks, x, N, K, threads=1), g["y_ref_f64"])
    host = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(host, 0, blocks, N)
    assert np.array_equal(O.c_split_emulate(host, x, 1), g["y_split_emulation"])
    l2, mx = O.rel_errors(g["y_split_emulation"], g["y_ref_f64"])
    assert l2 <= O.TOL and mx <= O.TOL


@pytest.mark.gpu
def test_config0_gpu_matches_golden_outputs():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import webgllm_b200 as wg

    g, N, K, blocks, x = _config0()
    m = wg.newQuantMatrix(N, K)
    wg.packQ4_0(m, 0, blocks, N)
    xd = torch.from_numpy(x).cuda()  # config 0: fp32 activations and outputs
    y = wg.matmul(xd, m, out_dtype=torch.float32)
    torch.cuda.synchronize()
    got = y.cpu().numpy().reshape(-1)
    for key in ("y_ref_f64", "y_split_emulation"):
        l2, mx = O.rel_errors(got, g[key].reshape(-1))
        assert l2 <= O.TOL and mx <= O.TOL, f"{key}: {l2:.2e} {mx:.2e}"
    m.free()
