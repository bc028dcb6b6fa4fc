"""GQA prefill attention on the B200 tensor cores (tcgen05) — the prefill branch of
threadcut/attention.py:43-46 without expanding K/V.

`prefill_attention(query, key, value, scale)`: query [1, hq, lq, d], key/value [1, hkv, lk, d] with
hq = 4*hkv and d = 128 (bf16 or fp16, CUDA). Query position p (of the lq newest tokens) attends to
keys [0, lk - lq + p], the causal mask of a prefill over a cache that ends with those tokens.
Returns [1, lq, hq, d] contiguous (the layout the attention plugin returns). `supported()` says
whether the kernel takes the inputs; the plugin keeps torch SDPA for everything else.
"""
import torch

from . import _lib
from ._lib import check, lib, require_cuda, stream_ptr, workspaces

__all__ = ["prefill_attention", "supported", "causal_offset_mask"]


def supported(query, key, value):
    return (query.is_cuda and key.is_cuda and value.is_cuda and query.dim() == 4 and key.dim() == 4
            and query.shape[0] == 1 and key.shape[0] == 1 and query.shape[-1] == 128
            and query.dtype in (torch.bfloat16, torch.float16) and key.dtype == query.dtype
            and value.dtype == query.dtype and key.shape[1] * 4 == query.shape[1]
            and value.shape == key.shape and 1 <= query.shape[2] <= key.shape[2])


def causal_offset_mask(lq, lk, device):
    """The boolean SDPA mask [lq, lk] the kernel implements: True where key j <= lk - lq + p."""
    p = torch.arange(lq, device=device)[:, None]
    j = torch.arange(lk, device=device)[None, :]
    return j <= (lk - lq) + p


def prefill_attention(query, key, value, scale, *, splits=None):
    what = "prefill_attention"
    require_cuda(query, key, value, what=what)
    if not supported(query, key, value):
        raise ValueError(f"{what}: needs query [1, 4*hkv, lq, 128], key/value [1, hkv, lk, 128] with lq <= lk, "
                         f"bf16/fp16; got {tuple(query.shape)}, {tuple(key.shape)}, {query.dtype}")
    _, hq, lq, d = query.shape
    hkv, lk = key.shape[1], key.shape[2]
    q, k, v = query[0], key[0], value[0]
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    out = torch.empty((1, lq, hq, d), dtype=query.dtype, device=query.device)
    L = lib()
    s = int(splits or 0)
    with torch.cuda.device(query.device):
        nb = L.tc_prefill_workspace_size(hq, hkv, lq, lk, s)
        ws = workspaces.get("prefill", query.device, nb) if nb else None
        st = L.tc_prefill_attention(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), hq, hkv, lq, lk, d, q.stride(0), q.stride(1),
            k.stride(0), k.stride(1), v.stride(0), v.stride(1), out.stride(1), out.stride(2), float(scale), s,
            _lib.DTYPE_CODE[query.dtype], ws.data_ptr() if ws is not None else None, nb, stream_ptr(query.device))
    check(what, st)
    return out
