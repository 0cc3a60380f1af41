"""Writes the golden fixtures of this directory. Run it where the reference
tree exists (it is read as text, never executed):

    python tests/golden/make_golden.py --reference <webgllm package dir>

Two files come out:

* ``reference_vectors.json`` -- the literal inputs and expected values of
  webgllm's own known-answer tests for the Q4 path, lifted from its test
  sources (each entry records file:line). webgllm is TypeScript and needs
  Node and a browser GPU stack, none of which this host has, so its tests
  cannot run here; their literals are the golden vectors. The extraction
  fails loudly if a test no longer holds the expected literal.
* ``config0_gemv.npz`` -- BASELINE config 0 (M = 1, N = K = 2048, seed 0):
  SHA-256 digests of the seeded Q4_0 bytes and activations, and the outputs
  of the oracle's two restatements of the reference arithmetic (the bench's
  fp64 ``reference()``, bench/gpu-bench-worker.js:41-55, and the split
  shader emulation). The reference cannot produce them here, so they pin the
  oracle over time and give the GPU tests a fixed target.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


class Source:
    def __init__(self, pkg: Path, rel: str):
        self.rel = rel
        self.lines = (pkg / rel).read_text().splitlines()

    def find(self, pattern: str) -> tuple[re.Match, str]:
        rx = re.compile(pattern)
        for i, line in enumerate(self.lines, 1):
            m = rx.search(line)
            if m:
                return m, f"{self.rel}:{i}"
        raise SystemExit(f"{self.rel}: no line matches {pattern!r}; the reference test changed")


def ints(text: str) -> list[int]:
    return [int(t, 0) for t in re.findall(r"0x[0-9a-fA-F]+|\d+", text)]


def js_number(tok: str) -> float:
    """A numeric literal or a `2 ** -11`-style power as the test writes it."""
    tok = tok.strip()
    if "**" in tok:
        b, e = tok.split("**")
        return float(b) ** float(e)
    return float(tok)


def reference_vectors(pkg: Path) -> dict:
    out = {}
    half = Source(pkg, "src/half.test.ts")
    m, at = half.find(r"for \(const v of \[([^\]]+)\]\)")
    out["half_exact_round_trip"] = {"at": at, "values": [js_number(t) for t in m.group(1).split(",")]}
    m, at = half.find(r"toHalf\(1 \+ 2 \*\* -11\)\), 1\)")
    out["half_tie_to_even"] = {"at": at, "input": 1 + 2 ** -11, "want": 1.0}
    m, at = half.find(r"toHalf\(1 \+ 3 \* 2 \*\* -12\)\), 1 \+ 2 \*\* -10\)")
    out["half_round_up"] = {"at": at, "input": 1 + 3 * 2 ** -12, "want": 1 + 2 ** -10}
    m, at = half.find(r"for \(const h of \[([^\]]+)\]\)")
    out["half_table_bits"] = {"at": at, "bits": ints(m.group(1))}
    m, at = half.find(r"new Uint16Array\(\[([^\]]+)\]\)")
    m2, _ = half.find(r"halvesToFloats\(bytes\)\]\, \[([^\]]+)\]")
    out["halves_to_floats"] = {"at": at, "bits": ints(m.group(1)),
                               "want": [js_number(t) for t in m2.group(1).split(",")]}

    rep = Source(pkg, "src/repack.test.ts")
    m, at = rep.find(r"const zp = Uint8Array\.of\(([^)]+)\)")
    out["zero_points_low_nibble_first"] = {
        "at": at, "N": 4, "K": 64, "zp": ints(m.group(1)),
        # zeros[0*4 + r] == 2r + 1 and zeros[1*4 + r] == 2r + 2 (the next lines)
        "want_block0": [2 * r + 1 for r in range(4)], "want_block1": [2 * r + 2 for r in range(4)]}
    rep.find(r"zeros\[0 \* 4 \+ r\], 2 \* r \+ 1")
    rep.find(r"zeros\[1 \* 4 \+ r\], 2 \* r \+ 2")
    m, at = rep.find(r"Math\.imul\(s, (\d+)\) \+ (\d+)\) >>> 0\) >>> 16")
    out["matmulnbits_lcg"] = {"at": at, "mul": int(m.group(1)), "add": int(m.group(2)), "shift": 16}

    words = Source(pkg, "src/repack-words.test.ts")
    m, at = words.find(r"raw\[i\] = \(i \* (\d+) \+ (\d+)\) & 255")
    m2, _ = words.find(r"perm = \[([^\]]+)\]")
    out["q4_0_word_copies"] = {"at": at, "mul": int(m.group(1)), "add": int(m.group(2)),
                               "perm": ints(m2.group(1)), "offsets": [0, 1, 2, 3],
                               "N": 12, "K": 64, "row0": 4, "rows": 4}

    rq = Source(pkg, "src/q4-repacker.test.ts")
    m, at = rq.find(r"for \(const \[N, K\] of \[(.+)\]\)")
    shapes = ints(m.group(1))
    m2, _ = rq.find(r"Math\.imul\(i \+ 1, (\d+)\) >>> 24")
    out["q4_repacker_shapes"] = {"at": at, "shapes": [shapes[i:i + 2] for i in range(0, len(shapes), 2)],
                                 "mul": int(m2.group(1)), "shift": 24}

    lf = Source(pkg, "src/lfm2-gguf.test.ts")
    m, at = lf.find(r"bytes\[i\]=(\d+);bytes\[i\+1\]=(\d+);bytes\.fill\((\d+),i\+2,i\+18\)")
    out["constant_q4_0_block"] = {"at": at, "block": [int(m.group(1)), int(m.group(2))] + [int(m.group(3))] * 16}
    return out


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def config0(path: Path) -> None:
    sys.path.insert(0, str(ROOT))
    import oracle as O
    from webgllm_b200 import synthetic

    N = K = 2048
    blocks = synthetic.q4_0_blocks(N, K, 0)
    x = synthetic.activations(1, K, 0)
    host = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(host, 0, blocks, N)
    y64 = O.c_ref_f64(blocks, x, N, K, threads=1)
    yem = O.c_split_emulate(host, x, 1)
    np.savez_compressed(path, N=N, K=K, seed=0, blocks_sha256=sha(blocks), x_sha256=sha(x),
                        y_ref_f64=y64.astype(np.float64), y_split_emulation=yem.astype(np.float32))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True,
                    help="the webgllm package directory (packages/webgllm of the reference tree)")
    args = ap.parse_args()
    vec = reference_vectors(args.reference)
    (HERE / "reference_vectors.json").write_text(json.dumps(vec, indent=1) + "\n")
    config0(HERE / "config0_gemv.npz")
    print("wrote", HERE / "reference_vectors.json", HERE / "config0_gemv.npz")


if __name__ == "__main__":
    main()
