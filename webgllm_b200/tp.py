"""Tensor-parallel partition of a decoder across the GPUs of one node.

The reference runs one model on one device; BASELINE's 8B-shape config
splits its projections across 2/4/8 GPUs (Megatron-style):

* q|k|v rows and gate|up rows are split by output (column parallel): rank r
  keeps query heads [r H/n, (r+1) H/n), KV heads [r Hkv/n, (r+1) Hkv/n) and
  FFN rows [r I/n, (r+1) I/n) of both gate and up, so attention, the KV
  cache, SwiGLU and the norm prologues all run locally;
* o and down are split by input (row parallel): rank r keeps the K columns
  of its heads / FFN rows and produces a partial sum over them, summed
  across ranks by one all-reduce each;
* the LM head is split by vocabulary: each rank scores its shard and the
  greedy pick is an all-reduce MAX over packed (logit, index) int64 keys;
* embeddings, norms and the residual stream are replicated.

Every cut falls on a Q4_0 block boundary (K multiples of 32, whole rows),
so shards are taken from the quantised GGUF bytes themselves: the sharded
model is bit-for-bit the unsharded one, for any n.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

BLOCK = 32
BLOCK_BYTES = 18


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    heads: int      # query heads per rank
    kv_heads: int   # KV heads per rank
    ffn: int        # FFN rows (of gate and of up) per rank
    vocab: int      # LM-head rows per rank
    vocab_offset: int

    @property
    def q0(self) -> int:
        return self.rank * self.heads


def plan(cfg, rank: int, world: int) -> Shard:
    """The shard of `rank` among `world` GPUs; ValueError if cfg does not
    split evenly on block boundaries."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    H, Hkv, Dh, I, V = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
    if H % world or Hkv % world:
        raise ValueError(f"{H} query / {Hkv} KV heads do not split over {world} GPUs")
    if I % world or (I // world) % BLOCK:
        raise ValueError(f"FFN {I} does not split over {world} GPUs on {BLOCK}-column blocks")
    if ((H // world) * Dh) % BLOCK:
        raise ValueError("attention output columns per GPU are not whole Q4_0 blocks")
    if "conv" in cfg.layer_types and world > 1:
        raise ValueError("tensor parallelism covers attention decoders (the conv layers stay on one GPU)")
    v = V // world if V % world == 0 else V
    off = rank * v if V % world == 0 else 0
    return Shard(rank, world, H // world, Hkv // world, I // world, v, off)


def qkv_rows(cfg, s: Shard) -> torch.Tensor:
    """Rows of the full q|k|v matrix that rank s keeps (q heads, then k, then v)."""
    H, Hkv, Dh = cfg.heads, cfg.kv_heads, cfg.head_dim
    q = torch.arange(s.rank * s.heads * Dh, (s.rank + 1) * s.heads * Dh)
    k = H * Dh + torch.arange(s.rank * s.kv_heads * Dh, (s.rank + 1) * s.kv_heads * Dh)
    v = (H + Hkv) * Dh + torch.arange(s.rank * s.kv_heads * Dh, (s.rank + 1) * s.kv_heads * Dh)
    return torch.cat([q, k, v])


def gate_up_rows(cfg, s: Shard) -> torch.Tensor:
    """Rows of the full gate|up matrix that rank s keeps (its gate rows, then
    the same up rows: the local matrix is again gate | up)."""
    I = cfg.ffn
    g = torch.arange(s.rank * s.ffn, (s.rank + 1) * s.ffn)
    return torch.cat([g, I + g])


def o_cols(cfg, s: Shard) -> tuple[int, int]:
    """K columns of o that rank s keeps (its heads' outputs)."""
    w = s.heads * cfg.head_dim
    return s.rank * w, (s.rank + 1) * w


def down_cols(cfg, s: Shard) -> tuple[int, int]:
    return s.rank * s.ffn, (s.rank + 1) * s.ffn


def q4_rows(blocks: torch.Tensor, N: int, K: int, rows: torch.Tensor) -> torch.Tensor:
    """GGUF Q4_0 bytes of the listed rows of an N x K matrix."""
    b = blocks.reshape(N, (K // BLOCK) * BLOCK_BYTES)
    return b.index_select(0, rows.to(b.device)).reshape(-1).contiguous()


def q4_cols(blocks: torch.Tensor, N: int, K: int, k0: int, k1: int) -> torch.Tensor:
    """GGUF Q4_0 bytes of columns [k0, k1) (block-aligned) of an N x K matrix."""
    if k0 % BLOCK or k1 % BLOCK:
        raise ValueError("column cut inside a Q4_0 block")
    b = blocks.reshape(N, K // BLOCK, BLOCK_BYTES)
    return b[:, k0 // BLOCK:k1 // BLOCK].reshape(-1).contiguous()


# Packed greedy keys (include/webgllm_decoder.h wg_head_rmsnorm): the int64
# key of (logit v, index i) orders as (v, then lower i). Host mirror of the
# kernel's encoding, for the reference path in tests.
def argmax_key(value: float, index: int) -> int:
    import struct

    u = struct.unpack("<I", struct.pack("<f", 0.0 if value == 0 else value))[0]
    u = (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
    key = (u << 32) | (0xFFFFFFFF - index)
    key ^= 1 << 63
    return key - (1 << 64) if key >= 1 << 63 else key


def key_index(key: int) -> int:
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)
