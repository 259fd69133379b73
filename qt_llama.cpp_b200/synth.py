"""Seeded synthetic inputs for the MoE FFN layer, and the host-side GGUF block
quantisers used to build them.

There is no model checkpoint on the box, so every workload is synthetic:
router weights and expert weights N(0, 0.02), activations N(0, 1), all drawn
from seeded numpy PCG64 streams (and splitmix64 for permutations).  Expert weights are quantised with the same rules as the
reference's host quantisers, so the bytes handed to the GPU are the bytes a
GGUF file written by MRML would hold:

* Q4_0 (crates/mrml-tensor/src/quant.rs:372-389): d = max|v| / 8, stored as
  a truncating f16; q = clamp(round(v * (1/d)), -8, 7) + 8, low nibble holds
  element j, high nibble element j + 16.
* Q8_0 (quant.rs:193-228): d = max|v| / 127 (f16, truncating); the inverse
  uses the unrounded f32 scale; q = clamp(round(v * id), -128, 127).

`round` is C roundf (half away from zero), restated exactly below.
"""

from __future__ import annotations

import numpy as np

Q4_0 = 2
Q8_0 = 8
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}

_MASK = (1 << 64) - 1


def splitmix64(seed: int, n: int) -> np.ndarray:
    """n successive outputs of splitmix64 started at `seed` (uint64)."""
    with np.errstate(over="ignore"):
        state = np.uint64(seed & _MASK) + np.arange(1, n + 1, dtype=np.uint64) * np.uint64(
            0x9E3779B97F4A7C15
        )
        z = state
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def normal(seed: int, n: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    """n float32 samples of N(mean, std^2) from numpy's seeded PCG64 stream
    (deterministic for a given numpy release; the image pins numpy)."""
    z = np.random.Generator(np.random.PCG64(seed)).standard_normal(n, dtype=np.float32)
    if std != 1.0:
        z *= np.float32(std)
    if mean != 0.0:
        z += np.float32(mean)
    return z


def permutation(seed: int, n: int) -> np.ndarray:
    """A seeded permutation of range(n) (Fisher-Yates over splitmix64)."""
    bits = splitmix64(seed, n)
    p = np.arange(n, dtype=np.int64)
    for i in range(n - 1, 0, -1):
        j = int(bits[i] % np.uint64(i + 1))
        p[i], p[j] = p[j], p[i]
    return p


def f32_to_f16_trunc(v: np.ndarray) -> np.ndarray:
    """quant.rs:81-104: truncating f32 -> f16 bits, exponent underflow -> +0."""
    bits = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32)
    sign = ((bits >> 31) & 1).astype(np.uint16)
    exp = ((bits >> 23) & 0xFF).astype(np.int32)
    mant = bits & 0x7FFFFF
    exp16 = exp - 127 + 15
    out = (sign << 15) | (np.clip(exp16, 0, 31).astype(np.uint16) << 10) | (mant >> 13).astype(np.uint16)
    out = np.where(exp16 >= 31, (sign << 15) | 0x7C00, out)
    out = np.where(exp16 <= 0, 0, out)
    out = np.where(exp == 255, (sign << 15) | np.where(mant == 0, 0x7C00, 0x7E00), out)
    return out.astype(np.uint16)


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    """quant.rs:47-77 (IEEE half decode; numpy's float16 is exact for it)."""
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def roundf(v: np.ndarray) -> np.ndarray:
    """C roundf: nearest integer, halfway cases away from zero (exact)."""
    v = np.asarray(v, dtype=np.float32)
    t = np.trunc(v)
    frac = np.abs(v - t)  # exact in binary floating point
    return (t + np.where(frac >= np.float32(0.5), np.sign(v), np.float32(0))).astype(np.float32)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Rows of float32 (last axis a multiple of 32) -> Q8_0 bytes per row."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    nb = x.shape[-1] // 32
    blocks = x.reshape(-1, 32)
    amax = np.fmax.reduce(np.abs(blocks), axis=1)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    d = f32_to_f16_trunc(scale)
    with np.errstate(divide="ignore"):
        inv = np.where(scale != 0, np.float32(1.0) / scale, np.float32(0.0)).astype(np.float32)
    v = roundf(blocks * inv[:, None])
    v = np.nan_to_num(v, nan=0.0)
    q = np.clip(v, -128, 127).astype(np.int8)
    out = np.empty((blocks.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(*lead, nb * 34)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """Rows of float32 (last axis a multiple of 32) -> Q4_0 bytes per row."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    nb = x.shape[-1] // 32
    blocks = x.reshape(-1, 32)
    amax = np.fmax.reduce(np.abs(blocks), axis=1)
    scale = np.where(amax > 0, amax / np.float32(8.0), np.float32(0.0)).astype(np.float32)
    d = f32_to_f16_trunc(scale)
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, np.float32(1.0) / scale, np.float32(0.0)).astype(np.float32)
    v = np.nan_to_num(roundf(blocks * inv[:, None]), nan=0.0)
    q = (np.clip(v, -8, 7).astype(np.int32) + 8).astype(np.uint8)
    out = np.empty((blocks.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(*lead, nb * 18)


def quantize(x: np.ndarray, wtype: int) -> np.ndarray:
    if wtype == Q4_0:
        return quantize_q4_0(x)
    if wtype == Q8_0:
        return quantize_q8_0(x)
    raise ValueError(f"unsupported weight type {wtype}")


def expert_weights(seed: int, wtype: int, H: int, I: int, E: int, std: float = 0.02, quantize_fn=None):
    """GGUF-layout expert slabs: gate_up [E][2I][H/32 blocks], down [E][H][I/32 blocks].

    Generated and quantised one expert at a time to bound host memory.
    quantize_fn(rows, wtype) -> bytes may replace the numpy quantisers (for
    instance a compiled one with the same rules, for large layers)."""
    bb = BLOCK_BYTES[wtype]
    q = quantize if quantize_fn is None else quantize_fn
    gu = np.empty((E, 2 * I, H // 32 * bb), dtype=np.uint8)
    dn = np.empty((E, H, I // 32 * bb), dtype=np.uint8)
    for e in range(E):
        gu[e] = np.asarray(q(normal(seed * 1000003 + 2 * e + 1, 2 * I * H, std).reshape(2 * I, H), wtype)).reshape(
            2 * I, -1)
        dn[e] = np.asarray(q(normal(seed * 1000003 + 2 * e + 2, H * I, std).reshape(H, I), wtype)).reshape(H, -1)
    return gu, dn


def zipf_bias(seed: int, E: int, s: float = 1.1) -> np.ndarray:
    """Per-expert logit bias b_e = -s * ln(rank_e), rank a seeded permutation of
    1..E, so that softmax mass is proportional to rank^-s (skewed loads)."""
    rank = permutation(seed, E) + 1
    return (-s * np.log(rank.astype(np.float64))).astype(np.float32)


def expert_weights_device(seed: int, wtype: int, H: int, I: int, E: int, device, quantize_fn, std: float = 0.02):
    """Device-generated expert slabs for large configs: torch's seeded CUDA
    normal stream, quantised on the GPU by `quantize_fn(wtype, src, dst)` (the
    library's GGUF quantiser, byte-identical to the reference's).  Returns
    (gate_up, down) uint8 device tensors in the GGUF layout."""
    import torch

    bb = BLOCK_BYTES[wtype]
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    gu = torch.empty((E, 2 * I, H // 32 * bb), dtype=torch.uint8, device=device)
    dn = torch.empty((E, H, I // 32 * bb), dtype=torch.uint8, device=device)
    for e in range(E):
        src = torch.randn((2 * I, H), generator=gen, device=device, dtype=torch.float32).mul_(std)
        quantize_fn(wtype, src, gu[e])
        src = torch.randn((H, I), generator=gen, device=device, dtype=torch.float32).mul_(std)
        quantize_fn(wtype, src, dn[e])
    return gu, dn
