"""GQA-aware attention plugin for transformers on B200 — drop-in for threadcut/attention.py.

Registered as attention implementation "threadcut" (threadcut/attention.py:22,50-51), selected by
`attn_implementation=attention.NAME`. Signature and result are the reference's
(attention.py:30-47): `attention(module, query[b,Hq,q,D], key[b,Hkv,n,D], value, attention_mask,
dropout=0.0, scaling=None, **kw) -> (out[b,q,Hq,D] contiguous, None)`.

Decode (one query token, no mask): the g = Hq/Hkv query heads of each KV head are folded into a
g-row query (query.reshape(hkv, g, d), attention.py:39) and run by the B200 split-KV kernel over
the unexpanded cache, b == 1 through decode_attention and b > 1 through decode_attention_batched
(the reference used folded SDPA there). When the cache is a GrowingLayer whose newest row is still
pending (fused append, set up by new_cache for this attention), that row is written by the same
launch (decode_attention_append) instead of a separate copy before attention (kv.py:71-72).
With a paged cache (kv.new_cache(..., paged=True)) the key is a stand-in: the one-token step decodes
over the pages (PagedKV.decode, fused append), a causal prefill chunk runs the tcgen05 kernel over
the pages (PagedKV.prefill), and other branches get a contiguous copy.
Decode on a non-CUDA tensor raises: there is no CPU path.
Prefill (q > 1 or a mask): a causal prefill over the cache (query p sees keys up to lk - lq + p;
b == 1, 4 query heads per KV head, head_dim 128, 16-bit) runs the tcgen05 kernel of
threadcut_b200.prefill over the unexpanded cache; anything else keeps the reference's torch SDPA
branch (attention.py:43-46), with SDPA's GQA mode instead of an explicit repeat_kv expansion.
"""
import weakref

import torch
import torch.nn.functional as F
from transformers import AttentionInterface
from transformers.masking_utils import AttentionMaskInterface, causal_mask_function, sdpa_mask

from .flash_decode import decode_attention, decode_attention_append, decode_attention_batched
from .kv import FUSED_ATTENTION, paged_pending, pending_append
from . import prefill as _prefill

NAME = FUSED_ATTENTION  # "threadcut", as threadcut/attention.py:22

__all__ = ["NAME", "attention", "attention_mask", "repeat_kv"]


def repeat_kv(x, n):
    """[b, h, s, d] -> [b, h*n, s, d], each KV head repeated n times (prefill only)."""
    if n == 1:
        return x
    b, h, s, d = x.shape
    return x.unsqueeze(2).expand(b, h, n, s, d).reshape(b, h * n, s, d)


_mask_seen = {}  # the last mask tensor found to be the causal-offset mask (weak reference) + version


def _is_causal_offset(mask, lq, lk):
    """True when `mask` means query p sees keys [0, lk - lq + p]: None with lq == lk (HF drops the
    mask of a plain causal prefill), or the boolean [1, 1, lq, lk] mask HF builds for a prefill over
    a cache. The comparison runs once per mask tensor (HF passes one mask to every layer)."""
    if mask is None:
        return lq == lk
    if mask.dtype != torch.bool or tuple(mask.shape) != (1, 1, lq, lk):
        return False
    hit = _mask_seen.get("last")
    if hit is not None and hit[0]() is mask and hit[1] == mask._version:
        return True
    ok = bool(torch.equal(mask[0, 0], _prefill.causal_offset_mask(lq, lk, mask.device)))
    if ok:
        _mask_seen["last"] = (weakref.ref(mask), mask._version)
    return ok


def attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    b, hq, q, d = query.shape
    hkv = key.shape[1]
    g = hq // hkv
    scaling = scaling if scaling is not None else d ** -0.5
    paged = paged_pending(key)
    if paged is not None:
        if q == 1 and attention_mask is None and b == 1 and paged._pending is not None:
            # paged cache, one-token step: attend over the pages, the step's row written by the launch
            out = paged.decode(query.reshape(hkv, g, d), scaling).reshape(1, hq, 1, d)
            return out.transpose(1, 2).contiguous(), None
        if paged.can_prefill(query) and _is_causal_offset(attention_mask, q, paged.get_seq_length()):
            # paged cache, prefill chunk (rows already in the pages): tcgen05 kernel over the pages
            return paged.prefill(query, scaling), None
        key, value = paged.materialize()
    layer = pending_append(key)
    if q == 1 and attention_mask is None and b == 1 and layer is not None:
        # the cache's newest row is still pending (GrowingLayer with fused append): write it and
        # attend over the whole cache in one launch
        k_new, v_new, stable = layer.take_pending()
        out = decode_attention_append(query.reshape(hkv, g, d), key[0], value[0], k_new, v_new, scaling,
                                      stable_rows=stable).reshape(1, hq, 1, d)
        return out.transpose(1, 2).contiguous(), None
    if layer is not None:
        layer._flush()
    if q == 1 and attention_mask is None:
        if b == 1:
            out = decode_attention(query.reshape(hkv, g, d), key[0], value[0], scaling).reshape(1, hq, 1, d)
        else:
            out = decode_attention_batched(query.reshape(b, hkv, g, d), key, value, scaling).reshape(b, hq, 1, d)
    elif _prefill.supported(query, key, value) and _is_causal_offset(attention_mask, q, key.shape[2]):
        # causal prefill over the cache (the engine's D chunk): tcgen05 kernel, K/V never expanded
        return _prefill.prefill_attention(query, key, value, scaling), None
    else:
        # the reference expands K/V with repeat_kv first (attention.py:43-46); SDPA's own GQA mode
        # computes the same attention without materialising the expansion (4x the cache per layer)
        is_causal = attention_mask is None and q > 1 and q == key.shape[2]
        out = F.scaled_dot_product_attention(query, key, value, attn_mask=attention_mask, scale=scaling,
                                             is_causal=is_causal, enable_gqa=g > 1)
    return out.transpose(1, 2).contiguous(), None


def attention_mask(batch_size, q_length, kv_length, q_offset=0, kv_offset=0, mask_function=causal_mask_function,
                   attention_mask=None, local_size=None, allow_is_causal_skip=True, **kwargs):
    """The mask builder registered with the attention (the reference registers sdpa_mask,
    threadcut/attention.py:50-51). It returns sdpa_mask's result, except for one case that sdpa_mask
    cannot tell apart from an export trace: a one-token step with no padding mask, the plain causal
    pattern and the query at or after every key. Every key is then visible, so the mask would be all
    True, and None is returned (sdpa_mask returns None there too, unless a CUDA graph is being
    captured). The decode branch then needs no mask. Without None, the capture of a decode step
    would reach the prefill mask check, which reads the mask back to the host."""
    if (q_length == 1 and attention_mask is None and local_size is None and allow_is_causal_skip
            and mask_function is causal_mask_function and isinstance(q_offset, int) and isinstance(kv_offset, int)
            and q_offset >= kv_offset + kv_length - 1):
        return None
    return sdpa_mask(batch_size=batch_size, q_length=q_length, kv_length=kv_length, q_offset=q_offset,
                     kv_offset=kv_offset, mask_function=mask_function, attention_mask=attention_mask,
                     local_size=local_size, allow_is_causal_skip=allow_is_causal_skip, **kwargs)


AttentionInterface.register(NAME, attention)
AttentionMaskInterface.register(NAME, attention_mask)
