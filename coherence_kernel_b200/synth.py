"""Seeded synthetic GGUF tensors and activations for the quantized path.

The reference's real GGUF blobs are not available, so every workload uses seeded synthetic inputs
with the shapes and value distributions its benchmark configurations state:

* Q8_0 (``block_q8_0``, 34 bytes / 32 weights: f16 ``d`` then 32 int8 codes; the layout read by
  form/form-stdlib/q8-0-msl.fk:53-72): codes uniform in [-127, 127], ``d = |N(0,1)| * 0.01``.
* Q4_K (``block_q4_K``, 144 bytes / 256 weights: f16 ``d`` @0, f16 ``dmin`` @2, ``scales[12]``
  @4, ``qs[128]`` @16; the layout read by form/form-stdlib/q4k-msl.fk:55-86): 4-bit codes uniform
  0..15, 6-bit scales and mins uniform 0..63 packed by the inverse of get_scale_min_k4
  (q4k-dequant.fk:19-31), ``d = |N(0,1)| * 0.002``, ``dmin = |N(0,1)| * 0.001``.
* activations ``N(0,1)`` rounded to bf16 (round to nearest even); router ``N(0, 0.02)`` fp32;
  router bias ``N(0, 0.01)`` fp32.

All generators draw from ``numpy.random.default_rng(seed)``.
"""
from __future__ import annotations

import numpy as np

Q8_0_BLOCK_BYTES = 34
Q8_0_BLOCK_WEIGHTS = 32
Q4K_BLOCK_BYTES = 144
Q4K_BLOCK_WEIGHTS = 256


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.size > (1 << 20):
        import torch
        return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    u = x.view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def q8_0_bytes(n_weights: int) -> int:
    assert n_weights % Q8_0_BLOCK_WEIGHTS == 0, "a Q8_0 tensor is a whole number of 32-weight blocks"
    return n_weights // Q8_0_BLOCK_WEIGHTS * Q8_0_BLOCK_BYTES


def q4k_bytes(n_weights: int) -> int:
    assert n_weights % Q4K_BLOCK_WEIGHTS == 0, "a Q4_K tensor is a whole number of 256-weight superblocks"
    return n_weights // Q4K_BLOCK_WEIGHTS * Q4K_BLOCK_BYTES


def make_q8_0(rng: np.random.Generator, n_weights: int) -> np.ndarray:
    """``n_weights`` Q8_0 weights (flat, row-major along K) as a uint8 array of blocks."""
    nb = n_weights // Q8_0_BLOCK_WEIGHTS
    out = np.empty((nb, Q8_0_BLOCK_BYTES), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(nb)) * 0.01).astype(np.float16)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def pack_q4k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of get_scale_min_k4 (q4k-dequant.fk:19-31): [nb, 8] 6-bit scales and mins ->
    [nb, 12] packed bytes."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    nb = sc.shape[0]
    s = np.zeros((nb, 12), dtype=np.uint8)
    s[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    return s


def make_q4k(rng: np.random.Generator, n_weights: int, chunk_blocks: int = 1 << 20) -> np.ndarray:
    """``n_weights`` Q4_K weights (flat) as a uint8 array of 144-byte superblocks."""
    nb = n_weights // Q4K_BLOCK_WEIGHTS
    assert nb * Q4K_BLOCK_WEIGHTS == n_weights
    out = np.empty((nb, Q4K_BLOCK_BYTES), dtype=np.uint8)
    for b0 in range(0, nb, chunk_blocks):
        b1 = min(nb, b0 + chunk_blocks)
        n = b1 - b0
        d = (np.abs(rng.standard_normal(n)) * 0.002).astype(np.float16)
        dmin = (np.abs(rng.standard_normal(n)) * 0.001).astype(np.float16)
        out[b0:b1, 0:2] = d.view(np.uint8).reshape(n, 2)
        out[b0:b1, 2:4] = dmin.view(np.uint8).reshape(n, 2)
        sc = rng.integers(0, 64, size=(n, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, size=(n, 8), dtype=np.uint8)
        out[b0:b1, 4:16] = pack_q4k_scales(sc, mn)
        # two uniform 4-bit codes per byte == one uniform byte
        out[b0:b1, 16:] = rng.integers(0, 1 << 32, size=n * 32, dtype=np.uint32).view(np.uint8).reshape(n, 128)
    return out.reshape(-1)


Q6K_BLOCK_BYTES = 210


def q6k_bytes(n_weights: int) -> int:
    assert n_weights % Q4K_BLOCK_WEIGHTS == 0, "a Q6_K tensor is a whole number of 256-weight superblocks"
    return n_weights // Q4K_BLOCK_WEIGHTS * Q6K_BLOCK_BYTES


def make_q6k(rng: np.random.Generator, n_weights: int, chunk_blocks: int = 1 << 20) -> np.ndarray:
    """``n_weights`` Q6_K weights (flat) as a uint8 array of 210-byte superblocks: ql[128] and
    qh[64] uniform (6-bit codes uniform over 0..63), 16 signed 8-bit scales uniform over -128..127,
    fp16 d = |N(0,1)| * 0.0005."""
    nb = n_weights // Q4K_BLOCK_WEIGHTS
    assert nb * Q4K_BLOCK_WEIGHTS == n_weights
    out = np.empty((nb, Q6K_BLOCK_BYTES), dtype=np.uint8)
    for b0 in range(0, nb, chunk_blocks):
        b1 = min(nb, b0 + chunk_blocks)
        n = b1 - b0
        out[b0:b1, 0:208] = rng.integers(0, 256, size=(n, 208), dtype=np.uint8)
        d = (np.abs(rng.standard_normal(n)) * 0.0005).astype(np.float16)
        out[b0:b1, 208:210] = d.view(np.uint8).reshape(n, 2)
    return out.reshape(-1)


def make_bf16(rng: np.random.Generator, shape) -> np.ndarray:
    """N(0,1) activations as bf16 bit patterns (uint16)."""
    return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))


def make_router(rng: np.random.Generator, n_experts: int, hidden: int) -> np.ndarray:
    return (rng.standard_normal((n_experts, hidden), dtype=np.float32) * np.float32(0.02)).astype(np.float32)


def make_bias(rng: np.random.Generator, n_experts: int) -> np.ndarray:
    return (rng.standard_normal(n_experts, dtype=np.float32) * np.float32(0.01)).astype(np.float32)


def f16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)
