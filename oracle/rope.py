"""RoPE shift oracle (numpy). Test infrastructure only; see oracle/__init__.py.

threadcut/kv.py:15-25:
    rotate_half(x) = cat(-x2, x1)
    shift_keys(keys, delta, inv_freq): angle = delta * inv_freq (fp32); emb = cat(angle, angle);
        k = keys.float(); return (k * emb.cos() + rotate_half(k) * emb.sin()).to(keys.dtype)
numpy float32 ufuncs round every product and sum separately (no contraction), which is how torch
evaluates that expression, so with the reference's cos/sin table the result is bit-exact.
"""
import numpy as np


def f32_to_bf16_bits(x):
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even; NaN -> canonical quiet NaN."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(np.isnan(x), 0x7FC0, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b):
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_to(x, dtype):
    """Round fp32 values to the storage dtype ('bf16', 'f16', 'f32') and return them as fp32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def rotate_half(x):
    h = x.shape[-1] // 2
    return np.concatenate((-x[..., h:], x[..., :h]), axis=-1)


def inv_freq_default(d, theta):
    """Default RoPE frequencies 1 / theta^(2i/d), i < d/2, in fp32 (the Qwen3 rotary init)."""
    return (1.0 / (np.float32(theta) ** (np.arange(0, d, 2, dtype=np.int64).astype(np.float32) / np.float32(d))))\
        .astype(np.float32)


def cos_sin_ref(delta, inv_freq):
    """(cos, sin) of the fp32 angle delta*inv_freq, numpy fp32 (within an ulp or so of torch's)."""
    angle = np.float32(delta) * np.asarray(inv_freq, dtype=np.float32)
    return np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)


def shift_keys_f32(keys, delta=None, inv_freq=None, cos_sin=None):
    """fp32 result of the shift BEFORE the cast to the cache dtype. keys [..., d] (fp32 values);
    either (delta, inv_freq) or an explicit cos_sin = (cos[d/2], sin[d/2]) table."""
    k = np.asarray(keys, dtype=np.float32)
    if cos_sin is None:
        cos_sin = cos_sin_ref(delta, inv_freq)
    c, s = (np.asarray(a, dtype=np.float32) for a in cos_sin)
    h = k.shape[-1] // 2
    x, y = k[..., :h], k[..., h:]
    lo = x * c + (-y) * s
    hi = y * c + x * s
    return np.concatenate((lo, hi), axis=-1).astype(np.float32)


def shift_keys_ref(keys, delta=None, inv_freq=None, dtype="bf16", cos_sin=None):
    """shift_keys with the final cast: returns fp32 values representable in `dtype`."""
    return round_to(shift_keys_f32(keys, delta, inv_freq, cos_sin), dtype)


def rope_at_positions(k, positions, inv_freq):
    """Rotate raw keys k [..., n, d] to absolute positions (one per row): the shift formula with
    delta = position, fp32 (used to build pre-rotated caches)."""
    k = np.asarray(k, dtype=np.float32)
    angle = np.asarray(positions, dtype=np.float32)[:, None] * np.asarray(inv_freq, dtype=np.float32)[None, :]
    c, s = np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)
    h = k.shape[-1] // 2
    x, y = k[..., :h], k[..., h:]
    return np.concatenate((x * c + (-y) * s, y * c + x * s), axis=-1).astype(np.float32)
