"""The reference's own CPU path for the hot path, as the torch expressions it evaluates.
Test and baseline infrastructure only (see oracle/__init__.py): bench.py times these as the CPU
baseline and as its reference arm; nothing in threadcut_b200 imports them.

threadcut is pure Python over torch, so its CPU path is torch on CPU tensors:
  * decode (threadcut/attention.py:35-42,47 with no Triton or a CPU query): the g query heads of a
    KV head are folded into a g-row query and SDPA runs against the unexpanded cache;
  * shift_keys (threadcut/kv.py:20-25): fp32 angle delta*inv_freq, emb = cat(angle, angle),
    k*cos + rotate_half(k)*sin in fp32, cast back to the cache dtype;
  * GrowingLayer.splice (threadcut/kv.py:83-92): C's keys shifted by -gap and its values cloned,
    both written over [a, a + c) of the buffers.
The functions below evaluate the same expressions (same ops, same order, same dtypes), so a timing of
them is a timing of the reference's CPU path without needing its source at run time.
"""
import torch
import torch.nn.functional as F


def folded_decode(query, key, value, scale):
    """query [b, Hq, 1, d], key/value [b, Hkv, n, d] -> out [b, 1, Hq, d] (contiguous)."""
    b, hq, _, d = query.shape
    hkv = key.shape[1]
    g = hq // hkv
    out = F.scaled_dot_product_attention(query.reshape(b, hkv, g, d), key, value, scale=scale)
    return out.reshape(b, hq, 1, d).transpose(1, 2).contiguous()


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def shift_keys(keys, delta, inv_freq):
    """Post-RoPE keys moved by `delta` positions: fp32 math, result in keys.dtype."""
    angle = delta * inv_freq.float()
    emb = torch.cat((angle, angle), dim=-1)
    k = keys.float()
    return (k * emb.cos() + _rotate_half(k) * emb.sin()).to(keys.dtype)


def growing_splice(kbuf, vbuf, a, c0, c, inv_freq):
    """In place on buffers [b, hkv, cap, d]: rows [a, a + c) := C = rows [c0, c0 + c), keys shifted
    by -(c0 - a). Returns the new length a + c."""
    gap = c0 - a
    if c and gap:
        k = shift_keys(kbuf[..., c0:c0 + c, :], -gap, inv_freq)
        v = vbuf[..., c0:c0 + c, :].clone()
        kbuf[..., a:a + c, :] = k
        vbuf[..., a:a + c, :] = v
    return a + c
