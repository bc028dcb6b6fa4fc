"""KV splice oracle (numpy). Test infrastructure only; see oracle/__init__.py.

GrowingLayer.splice (threadcut/kv.py:83-92): if c > 0, K rows [c0, c0+c) are shifted by -gap
(or cloned when gap == 0) and, with the V rows, written to [a, a+c) — the whole source is read
before anything is written; then n = a + c.
splice copy path (threadcut/kv.py:34-41): keep rows [0, a) and [c0, c0+c); shift the kept C part
of K by -gap when c and gap are both non-zero.
"""
import numpy as np

from .rope import shift_keys_ref


def growing_splice_ref(kbuf, vbuf, a, c0, c, inv_freq=None, dtype="bf16", cos_sin=None):
    """kbuf, vbuf [hkv, cap, d] (fp32 values). Returns new (kbuf, vbuf, n) — the full buffers after
    the in-place splice, rows beyond n untouched."""
    kb = np.array(kbuf, dtype=np.float32, copy=True)
    vb = np.array(vbuf, dtype=np.float32, copy=True)
    if c:
        gap = c0 - a
        k = kb[:, c0:c0 + c, :].copy()
        if gap:
            k = shift_keys_ref(k, -gap, inv_freq, dtype, cos_sin)
        v = vb[:, c0:c0 + c, :].copy()
        kb[:, a:a + c, :] = k
        vb[:, a:a + c, :] = v
    return kb, vb, a + c


def copy_splice_ref(keys, values, a, c0, c, inv_freq=None, dtype="bf16", cos_sin=None):
    """keys/values [hkv, n, d] -> new [hkv, a+c, d] tensors."""
    keys = np.asarray(keys, dtype=np.float32)
    values = np.asarray(values, dtype=np.float32)
    keep = np.concatenate((np.arange(0, a), np.arange(c0, c0 + c))).astype(np.int64)
    k = keys[:, keep, :].copy()
    v = values[:, keep, :].copy()
    if c and c0 - a:
        k[:, a:, :] = shift_keys_ref(k[:, a:, :], -(c0 - a), inv_freq, dtype, cos_sin)
    return k, v
