"""Shared test helpers: golden-vector access and tolerance constants."""
import hashlib
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")

# north_star tolerances
ATTN_ATOL = 2e-3          # bf16 attention output, max-abs vs the fp32 SDPA math on the same inputs
ORACLE_ATOL = 2e-5        # oracle (fp64) vs the reference's own fp32 SDPA on the CPU
MANTISSA = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}


def half_ulp(ref, dtype):
    """Half an ulp of `dtype` at |ref|: the error of the final cast of the result to the input
    dtype (threadcut/flash_decode.py:69 `.to(q.dtype)`), which no kernel can avoid."""
    a = np.abs(np.asarray(ref, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 1e-30)))
    if dtype == torch.float16:
        e = np.maximum(e, -14.0)
    return 0.5 * np.exp2(e - MANTISSA[dtype])


class AttnError(float):
    """The error compared with ATTN_ATOL (half-ulp adjusted) that also carries the raw max-abs
    difference; both appear wherever the value is printed (assertion messages, smoke)."""

    def __new__(cls, adjusted, raw):
        obj = super().__new__(cls, adjusted)
        obj.raw = raw
        return obj

    def __repr__(self):
        return f"{float(self):.3e} (raw max-abs {self.raw:.3e})"

    __str__ = __repr__


def attn_error(out, ref, dtype):
    """Max-abs error of a kernel output against the fp32/fp64 math with the unavoidable output
    rounding (half an ulp of the output dtype) taken off; it is compared with ATTN_ATOL. The raw
    max-abs difference rides along as `.raw` and is printed beside it."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if ref.size == 0:
        return AttnError(0.0, 0.0)
    diff = np.abs(out - ref)
    return AttnError(float(np.max(diff - half_ulp(ref, dtype))), float(np.max(diff)))

_gold = None
_meta = None


def gold():
    global _gold
    if _gold is None:
        _gold = dict(np.load(os.path.join(GOLDEN, "golden.npz")))
    return _gold


def meta():
    global _meta
    if _meta is None:
        with open(os.path.join(GOLDEN, "golden_meta.json")) as f:
            _meta = json.load(f)
    return _meta


def split_cases():
    with open(os.path.join(GOLDEN, "split_cases.json")) as f:
        return json.load(f)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def values(a):
    """Stored array -> fp32 values (uint16 arrays are bf16 bit patterns)."""
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return bf16_bits_to_f32(a)
    return a.astype(np.float32)


def storage_dtype(a):
    a = np.asarray(a)
    return {np.dtype(np.uint16): "bf16", np.dtype(np.float16): "f16", np.dtype(np.float32): "f32"}[a.dtype]


TORCH_DTYPE = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def sha(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return hashlib.sha256(t.view(torch.uint8).numpy().tobytes()).hexdigest()
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def ref_cos_sin(delta, inv_freq):
    """The reference's fp32 table for one shift (threadcut/kv.py:22-25), as numpy (cos, sin)."""
    angle = delta * inv_freq.float()
    emb = torch.cat((angle, angle))
    h = angle.numel()
    return emb.cos()[:h].numpy(), emb.sin()[:h].numpy()
