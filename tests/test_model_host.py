"""Host-side pieces of the decoder runner (no GPU): the Q4_0 quantiser used
for random-init weights against the oracle's C quantiser (llama.cpp's
quantize_row_q4_0 rule), its dequantiser, and the BASELINE config presets."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")

from webgllm_b200 import model as M  # noqa: E402


@pytest.mark.parametrize("N,K,std", [(8, 256, 0.05), (4, 32, 1.0), (16, 4096, 0.02)])
def test_quantize_q4_0_matches_the_gguf_rule(N, K, std):
    g = torch.Generator().manual_seed(N * K)
    w = torch.randn((N, K), generator=g) * std
    w[0, :32] = 0.0  # an all-zero block: scale 0, codes 8
    got = M.quantize_q4_0(w).numpy()
    want = O.c_quantize_q4_0(w.numpy().astype(np.float32))
    assert np.array_equal(got, want)


def test_dequantize_is_the_oracle_matrix_row():
    N, K = 8, 128
    blocks = O.config_q4_0_blocks(N, K, 11)
    got = M.dequantize_q4_0(torch.from_numpy(blocks), N, K).numpy()
    host = O.HostQuantMatrix(N, K)
    O.c_pack_q4_0(host, 0, blocks, N)
    for n in range(N):
        assert np.array_equal(got[n], O.c_matrix_row(host, n)), n


def params(cfg):
    D, H, Hkv, Dh, I, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
    n = 2 * V * D
    for t in cfg.layer_types:
        n += (H + 2 * Hkv) * Dh * D + H * Dh * D if t == "attn" else 3 * D * D + D * D
        n += 3 * D * I
    return n


def test_config_presets():
    assert M.CONFIG2.layers == 22 and params(M.CONFIG2) / 1e9 == pytest.approx(1.1, abs=0.05)
    assert M.CONFIG3.layer_types.count("conv") == 10 and M.CONFIG3.layer_types.count("attn") == 6
    assert params(M.CONFIG4) / 1e9 == pytest.approx(8.0, abs=0.1)
