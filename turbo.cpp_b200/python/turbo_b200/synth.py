"""Seeded synthetic inputs in the GGUF block formats.

Weights are quantized the way a GGUF writer stores them, so that the same bytes
can be fed to the CUDA path and to the CPU reference:

* Q8_0 (34 B per 32 values): d = amax/127 stored as IEEE half (round to nearest
  even), id = 1/d computed from the fp32 d, q = round-half-away(w * id).  This is
  the reference's own quantizer (src/tensor/quant_math.hpp:68-90), vectorised.
* Q4_0 (18 B per 32 values): m = the value of largest magnitude (first one on
  ties), d = m / -8 stored as half, q = clamp(round-half-away(w / d) + 8, 0, 15);
  byte j holds value j in its low nibble and value j+16 in its high nibble
  (the layout read by src/tensor/quant_math.hpp:158-174).
"""
import numpy as np

Q8_0_BYTES = 34
Q4_0_BYTES = 18


def rng(seed):
    return np.random.default_rng(seed)


def normal(shape, std=1.0, seed=0):
    r = rng(seed)
    return (r.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def uniform(shape, lo, hi, seed=0):
    r = rng(seed)
    return r.uniform(lo, hi, size=shape).astype(np.float32)


def _round_half_away(v32):
    v = v32.astype(np.float64)
    return np.sign(v) * np.floor(np.abs(v) + 0.5)


def quantize_q8_0(w):
    """w: float32 [..., K] with K % 32 == 0 -> uint8 [..., K/32*34]."""
    w = np.ascontiguousarray(w, np.float32)
    lead = w.shape[:-1]
    K = w.shape[-1]
    assert K % 32 == 0
    b = w.reshape(-1, 32)
    amax = np.max(np.abs(b), axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    d16 = d.astype(np.float16)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = _round_half_away((b * idv[:, None]).astype(np.float32)).astype(np.int8)
    out = np.empty((b.shape[0], Q8_0_BYTES), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(*lead, K // 32 * Q8_0_BYTES)


def quantize_q4_0(w):
    """w: float32 [..., K] with K % 32 == 0 -> uint8 [..., K/32*18]."""
    w = np.ascontiguousarray(w, np.float32)
    lead = w.shape[:-1]
    K = w.shape[-1]
    assert K % 32 == 0
    b = w.reshape(-1, 32)
    idx = np.argmax(np.abs(b), axis=1)  # first index of the largest magnitude
    m = b[np.arange(b.shape[0]), idx]
    d = (m / np.float32(-8.0)).astype(np.float32)
    d16 = d.astype(np.float16)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = _round_half_away((b * idv[:, None]).astype(np.float32)) + 8
    q = np.clip(q, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], Q4_0_BYTES), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(*lead, K // 32 * Q4_0_BYTES)


def dequantize_q8_0(wq, K):
    """Exact fp32 values of Q8_0 rows (q * d, one rounding): [..., K]."""
    lead = wq.shape[:-1]
    b = np.ascontiguousarray(wq).reshape(-1, Q8_0_BYTES)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).astype(np.float32).reshape(*lead, K)


def dequantize_q4_0(wq, K):
    lead = wq.shape[:-1]
    b = np.ascontiguousarray(wq).reshape(-1, Q4_0_BYTES)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    lo = (b[:, 2:] & 0x0F).astype(np.int32) - 8
    hi = (b[:, 2:] >> 4).astype(np.int32) - 8
    q = np.concatenate([lo, hi], axis=1).astype(np.float32)
    return (q * d).astype(np.float32).reshape(*lead, K)
