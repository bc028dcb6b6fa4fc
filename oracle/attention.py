"""Decode-attention oracle (numpy). Test infrastructure only; see oracle/__init__.py.

The reference's decode branch (threadcut/attention.py:35-42,47) folds the g = Hq/Hkv query heads
of each KV head into a g-row query and computes softmax(scale * q k^T) v over the unexpanded cache
(SDPA math on CPU; the Triton kernel of threadcut/flash_decode.py:21-69 computes the same thing in
fp32 by slices and merges them by log-sum-exp, flash_decode.py:68-69).
"""
import numpy as np


def decode_attention_ref(q, k, v, scale, dtype=np.float64, return_lse=False):
    """q [hkv, g, d]; k, v [hkv, n, d] (any float arrays; bf16 inputs passed as their fp32 values).
    Returns out [hkv, g, d] (and natural-log LSE [hkv, g]) computed in `dtype`. n == 0 gives zeros,
    as the reference's merge over zero slices does."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    hkv, g, d = q.shape
    if k.shape[1] == 0:
        out = np.zeros((hkv, g, d), dtype=dtype)
        return (out, np.full((hkv, g), -np.inf, dtype=dtype)) if return_lse else out
    s = np.matmul(q, np.swapaxes(k, 1, 2)) * dtype(scale)  # [hkv, g, n]
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    out = np.matmul(p, v) / l
    if return_lse:
        return out, (m + np.log(l))[..., 0]
    return out


def attention_decode_ref(query, key, value, scale=None, dtype=np.float64):
    """The plugin-level view (threadcut/attention.py:30-47) for one query token:
    query [b, Hq, 1, d], key/value [b, Hkv, n, d] -> out [b, 1, Hq, d]."""
    b, hq, q1, d = query.shape
    assert q1 == 1
    hkv = key.shape[1]
    g = hq // hkv
    scale = d ** -0.5 if scale is None else scale
    outs = [decode_attention_ref(np.asarray(query[i]).reshape(hkv, g, d), key[i], value[i], scale, dtype)
            for i in range(b)]
    return np.stack(outs).reshape(b, hq, 1, d).transpose(0, 2, 1, 3)


def merge_ref(o_parts, lse_parts):
    """Log-sum-exp merge of normalised partials: o_parts [P, rows, d], lse_parts [P, rows] ->
    (out [rows, d], lse [rows]); a part with lse = -inf contributes nothing."""
    o_parts = np.asarray(o_parts, dtype=np.float64)
    lse_parts = np.asarray(lse_parts, dtype=np.float64)
    m = lse_parts.max(axis=0)
    safe = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(lse_parts - safe)  # [P, rows]
    tot = w.sum(axis=0)
    out = np.einsum("pr,prd->rd", w, o_parts) / np.where(tot > 0, tot, 1.0)[:, None]
    lse = np.where(tot > 0, safe + np.log(np.where(tot > 0, tot, 1.0)), -np.inf)
    return out, lse
