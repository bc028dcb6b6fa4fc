"""Split-KV GQA decode attention on B200 — drop-in for threadcut/flash_decode.py.

`decode_attention(q, k, v, scale, split=256, block=16)` keeps the reference signature and result
(threadcut/flash_decode.py:57-69): q [hkv, g, d], k/v [hkv, n, d] with the last dim contiguous and
free head/token strides (a GrowingLayer view), returns [hkv, g, d] in q's dtype, softmax in fp32.
`split`/`block` were the Triton kernel's slice and tile sizes; here the KV partition is planned from
the SM count (pass `splits=` to force a number of slices). The kernel is csrc/decode_attn.cuh,
called through tc_decode_attention; there is no CPU or Triton path.

Extra entry points beside it (same math): `decode_attention_lse` (also returns the natural-log
LSE, the partial form for sequence-sharded decode), `decode_attention_batched` (b > 1 sequences
in one strided tensor, the b > 1 decode branch of threadcut/attention.py:41-42),
`decode_attention_ragged` (per-sequence caches and lengths) and `merge_partials` (LSE merge).
"""
import ctypes

import torch

from . import _lib
from ._lib import check, dtype_code, lib, require_cuda, stream_ptr, workspaces

__all__ = ["decode_attention", "decode_attention_append", "decode_attention_lse", "decode_attention_partial", "decode_attention_batched",
           "decode_attention_ragged", "merge_partials", "RaggedKV"]


def _last_contig(t):
    return t if t.stride(-1) == 1 else t.contiguous()


def _check_same_dtype(what, *ts):
    for t in ts[1:]:
        if t.dtype != ts[0].dtype:
            raise TypeError(f"threadcut_b200.{what}: dtype mismatch {ts[0].dtype} vs {t.dtype}")


def _decode_fast(q, k, v, scale, splits, stable_rows):
    """decode_attention through the compiled host binding (one crossing, checks in C++); None when
    it is unavailable or declines the inputs, so that the checked Python path below runs."""
    hb = _lib.host()
    if hb is None:
        return None
    dev = q.device
    if dev.type != "cuda":
        return None
    code = _lib.DTYPE_CODE.get(q.dtype)
    if code is None or q.dim() != 3:
        return None
    hkv, g, d = q.shape
    ws = workspaces.get(("decode", hkv), dev, _lib.decode_workspace_bound(1, hkv, g, d, code))
    return hb.decode(q, k, v, float(scale), int(splits or 0), int(stable_rows), ws)


def _decode(q, k, v, scale, splits, want_lse, partial=False, stable_rows=0):
    what = "decode_attention"
    dev = q.device
    if dev.type != "cuda" or k.device != dev or v.device != dev:
        require_cuda(q, k, v, what=what)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        _check_same_dtype(what, q, k, v)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError(f"{what}: expected q [hkv, g, d], k/v [hkv, n, d]; got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    hkv, g, d = q.shape
    n = k.shape[1]
    if k.shape[0] != hkv or k.shape[2] != d or v.shape != k.shape:
        raise ValueError(f"{what}: k/v shape {tuple(k.shape)}/{tuple(v.shape)} does not match q {tuple(q.shape)}")
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        q, k, v = _last_contig(q), _last_contig(k), _last_contig(v)
    code = _lib.DTYPE_CODE.get(q.dtype)
    if code is None:
        dtype_code(q, what)
    out = torch.empty((hkv, g, d), dtype=torch.float32 if partial else q.dtype, device=dev)
    lse = torch.empty((hkv, g), dtype=torch.float32, device=dev) if want_lse else None
    L = lib()
    s = int(splits or 0)
    stream = stream_ptr(dev)
    ws = workspaces.get(("decode", hkv), dev, _lib.decode_workspace_bound(1, hkv, g, d, code), stream)
    if stable_rows and not want_lse:
        args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), hkv, g, d, n, q.stride(0), q.stride(1),
                k.stride(0), k.stride(1), v.stride(0), v.stride(1), out.stride(0), out.stride(1), float(scale), s,
                code, int(stable_rows), ws.data_ptr(), ws.numel(), stream)
        fn = L.tc_decode_attention_stable
    elif stable_rows and partial:
        args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(), hkv, g, d, n, q.stride(0),
                q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1), out.stride(0), out.stride(1),
                float(scale), s, code, int(stable_rows), ws.data_ptr(), ws.numel(), stream)
        fn = L.tc_decode_attention_partial_stable
    else:
        args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr() if want_lse else None,
                hkv, g, d, n, q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
                out.stride(0), out.stride(1), float(scale), s, code, ws.data_ptr(), ws.numel(), stream)
        fn = L.tc_decode_attention_partial if partial else L.tc_decode_attention_lse
    if torch.cuda.current_device() == dev.index:
        st = fn(*args)
    else:
        with torch.cuda.device(dev):
            st = fn(*args)
    if st:
        check("tc_decode_attention", st)
    return (out, lse) if want_lse else out


def decode_attention(q, k, v, scale, split=256, block=16, *, splits=None, stable_rows=0):
    """q: [hkv, g, d]; k, v: [hkv, n, d] (last dim contiguous). Returns [hkv, g, d].

    `split` and `block` are accepted for call compatibility with the reference; the B200 kernel
    plans its own partition. `splits` (keyword only) forces the number of KV slices per head.
    `stable_rows` (keyword only) declares that rows [0, stable_rows) of k and v are written by no
    kernel still in flight on the GPU (e.g. n - 1 in a decode step whose append wrote only the last
    row); the kernel may then load them before the preceding decode launch has finished. The
    default 0 declares nothing."""
    if stable_rows < 0:
        raise ValueError("decode_attention: stable_rows must be >= 0")
    out = _decode_fast(q, k, v, scale, splits, stable_rows)
    if out is not None:
        return out
    return _decode(q, k, v, scale, splits, False, stable_rows=stable_rows)


def decode_attention_append(q, k, v, k_new, v_new, scale, *, splits=None, stable_rows=0):
    """GrowingLayer.update of one token fused with decode_attention: writes k_new / v_new [hkv, d]
    as the LAST row of the cache views k / v [hkv, n, d] and returns attention of q [hkv, g, d] over
    all n rows ([hkv, g, d]) — one launch instead of two copies and a decode. The last row of k/v
    is an output here: its previous contents are never read. stable_rows as for decode_attention."""
    what = "decode_attention_append"
    require_cuda(q, k, v, k_new, v_new, what=what)
    _check_same_dtype(what, q, k, v, k_new, v_new)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3 or k_new.dim() != 2 or v_new.dim() != 2:
        raise ValueError(f"{what}: expected q [hkv, g, d], k/v [hkv, n, d], k_new/v_new [hkv, d]")
    hkv, g, d = q.shape
    n = k.shape[1]
    if (k.shape[0] != hkv or k.shape[2] != d or v.shape != k.shape or tuple(k_new.shape) != (hkv, d)
            or tuple(v_new.shape) != (hkv, d) or n < 1):
        raise ValueError(f"{what}: shapes q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}, "
                         f"k_new {tuple(k_new.shape)}, v_new {tuple(v_new.shape)} do not fit")
    if k.stride(-1) != 1 or v.stride(-1) != 1:
        raise ValueError(f"{what}: the cache views must have a contiguous last dimension (they are written)")
    if stable_rows < 0:
        raise ValueError(f"{what}: stable_rows must be >= 0")
    q, k_new, v_new = _last_contig(q), _last_contig(k_new), _last_contig(v_new)
    code = dtype_code(q, what)
    dev = q.device
    out = torch.empty((hkv, g, d), dtype=q.dtype, device=dev)
    L = lib()
    s = int(splits or 0)
    stream = stream_ptr(dev)
    ws = workspaces.get(("decode", hkv), dev, _lib.decode_workspace_bound(1, hkv, g, d, code), stream)
    with torch.cuda.device(dev):
        st = L.tc_decode_attention_append(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), hkv, g, d,
            n, q.stride(0), q.stride(1), k_new.stride(0), v_new.stride(0), k.stride(0), k.stride(1), v.stride(0),
            v.stride(1), out.stride(0), out.stride(1), float(scale), s, code, int(stable_rows), ws.data_ptr(),
            ws.numel(), stream)
    check(what, st)
    return out


def decode_attention_append_rope(q, k, v, k_new, v_new, q_norm, k_norm, cos, sin, eps, scale, *, splits=None,
                                 stable_rows=0):
    """decode_attention_append with Qwen3's q/k norm and RoPE in the same launch: q [hkv, g, d] and
    k_new [hkv, d] are the raw projections; each d-vector gets RMSNorm (weights q_norm / k_norm [d],
    eps) and x*cos + rotate_half(x)*sin (cos/sin [d]) with the arithmetic of the separate
    tc_qk_norm_rope launch, and the rotated k_new is the row written to the cache. bf16/fp16, head
    dim 64/128/256, 16-byte aligned cache rows only (tc_decode_attention_append_rope)."""
    what = "decode_attention_append_rope"
    require_cuda(q, k, v, k_new, v_new, q_norm, k_norm, cos, sin, what=what)
    _check_same_dtype(what, q, k, v, k_new, v_new, q_norm, k_norm, cos, sin)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3 or k_new.dim() != 2 or v_new.dim() != 2:
        raise ValueError(f"{what}: expected q [hkv, g, d], k/v [hkv, n, d], k_new/v_new [hkv, d]")
    hkv, g, d = q.shape
    n = k.shape[1]
    if (k.shape[0] != hkv or k.shape[2] != d or v.shape != k.shape or tuple(k_new.shape) != (hkv, d)
            or tuple(v_new.shape) != (hkv, d) or n < 1):
        raise ValueError(f"{what}: shapes q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}, "
                         f"k_new {tuple(k_new.shape)}, v_new {tuple(v_new.shape)} do not fit")
    for name, t in (("q_norm", q_norm), ("k_norm", k_norm), ("cos", cos), ("sin", sin)):
        if t.numel() != d:
            raise ValueError(f"{what}: {name} must hold d = {d} values, got {tuple(t.shape)}")
    if k.stride(-1) != 1 or v.stride(-1) != 1:
        raise ValueError(f"{what}: the cache views must have a contiguous last dimension (they are written)")
    if stable_rows < 0:
        raise ValueError(f"{what}: stable_rows must be >= 0")
    q, k_new, v_new = _last_contig(q), _last_contig(k_new), _last_contig(v_new)
    q_norm, k_norm, cos, sin = (t.contiguous() for t in (q_norm, k_norm, cos, sin))
    code = dtype_code(q, what)
    dev = q.device
    out = torch.empty((hkv, g, d), dtype=q.dtype, device=dev)
    stream = stream_ptr(dev)
    ws = workspaces.get(("decode", hkv), dev, _lib.decode_workspace_bound(1, hkv, g, d, code), stream)
    with torch.cuda.device(dev):
        st = lib().tc_decode_attention_append_rope(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), hkv, g, d,
            n, q.stride(0), q.stride(1), k_new.stride(0), v_new.stride(0), k.stride(0), k.stride(1), v.stride(0),
            v.stride(1), out.stride(0), out.stride(1), q_norm.data_ptr(), k_norm.data_ptr(), cos.data_ptr(),
            sin.data_ptr(), float(eps), float(scale), int(splits or 0), code, int(stable_rows), ws.data_ptr(),
            ws.numel(), stream)
    check(what, st)
    return out


def decode_attention_lse(q, k, v, scale, *, splits=None):
    """Like decode_attention, plus the natural-log log-sum-exp of the scaled scores, fp32 [hkv, g]."""
    return _decode(q, k, v, scale, splits, True)


def decode_attention_partial(q, k, v, scale, *, splits=None, stable_rows=0):
    """Partial result of a KV slice for sequence-sharded decode: (o fp32 [hkv, g, d], natural-log
    lse fp32 [hkv, g]). Partials of disjoint token ranges merge exactly with merge_partials.
    `stable_rows` as for decode_attention."""
    if stable_rows < 0:
        raise ValueError("decode_attention_partial: stable_rows must be >= 0")
    hb = _lib.host()
    if hb is not None and hasattr(hb, "partial") and q.device.type == "cuda" and q.dim() == 3:
        code = _lib.DTYPE_CODE.get(q.dtype)
        if code is not None:
            hkv, g, d = q.shape
            ws = workspaces.get(("decode", hkv), q.device, _lib.decode_workspace_bound(1, hkv, g, d, code))
            res = hb.partial(q, k, v, float(scale), int(splits or 0), int(stable_rows), ws)
            if res is not None:
                return res
    return _decode(q, k, v, scale, splits, True, partial=True, stable_rows=stable_rows)


def decode_attention_batched(q, k, v, scale, lengths=None, *, splits=None):
    """q: [b, hkv, g, d]; k, v: [b, hkv, n, d]; lengths: optional int32 CUDA tensor [b] of valid
    lengths (<= n). Returns [b, hkv, g, d]."""
    what = "decode_attention_batched"
    require_cuda(q, k, v, what=what)
    _check_same_dtype(what, q, k, v)
    b, hkv, g, d = q.shape
    n = k.shape[2]
    if tuple(k.shape) != (b, hkv, n, d) or tuple(v.shape) != (b, hkv, n, d):
        raise ValueError(f"{what}: k/v shape {tuple(k.shape)} does not match q {tuple(q.shape)}")
    q, k, v = _last_contig(q), _last_contig(k), _last_contig(v)
    lens_ptr = None
    if lengths is not None:
        lengths = lengths.to(device=q.device, dtype=torch.int32).contiguous()
        if lengths.shape != (b,):
            raise ValueError(f"{what}: lengths must be [{b}]")
        lens_ptr = lengths.data_ptr()
    code = dtype_code(q, what)
    dev = q.device
    out = torch.empty((b, hkv, g, d), dtype=q.dtype, device=dev)
    L = lib()
    s = int(splits or 0)
    ws = workspaces.get(("decode", b * hkv), dev, L.tc_decode_attention_workspace_size(b, hkv, g, d, n, b * n, s, code))
    with torch.cuda.device(dev):
        st = L.tc_decode_attention_batched(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, hkv, g, d, n, lens_ptr,
            q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
            v.stride(0), v.stride(1), v.stride(2), out.stride(0), out.stride(1), out.stride(2),
            float(scale), s, code, ws.data_ptr(), ws.numel(), stream_ptr(dev))
    check("tc_decode_attention_batched", st)
    return out


class RaggedKV:
    """Device-side descriptor of per-sequence K/V caches for decode_attention_ragged.

    ks[i], vs[i]: [hkv, cap_i, d] tensors (cap_i >= lengths[i]) sharing dtype, token stride and the
    head stride of the K/V pair; lengths: python ints. Building it copies three small arrays to the
    device once; reuse it across steps while the caches stay in place."""

    def __init__(self, ks, vs, lengths):
        what = "RaggedKV"
        if not (len(ks) == len(vs) == len(lengths)) or not ks:
            raise ValueError(f"{what}: ks, vs, lengths must be non-empty and of equal length")
        require_cuda(*ks, *vs, what=what)
        _check_same_dtype(what, *ks, *vs)
        hkv, _, d = ks[0].shape
        sn = ks[0].stride(1)
        for k, v, n in zip(ks, vs, lengths):
            if k.dim() != 3 or k.shape[0] != hkv or k.shape[2] != d or v.shape != k.shape:
                raise ValueError(f"{what}: every cache must be [hkv={hkv}, cap, d={d}] with matching K/V")
            if k.stride(2) != 1 or v.stride(2) != 1 or k.stride(1) != sn or v.stride(1) != sn:
                raise ValueError(f"{what}: caches must share the token stride and have a contiguous last dim")
            if k.stride(0) != v.stride(0):
                raise ValueError(f"{what}: K and V of a sequence must share the head stride")
            if not 0 <= n <= k.shape[1]:
                raise ValueError(f"{what}: length {n} outside [0, {k.shape[1]}]")
            es = k.element_size()
            if k.data_ptr() % 16 or v.data_ptr() % 16 or (k.stride(0) * es) % 16 or (sn * es) % 16:
                raise ValueError(f"{what}: K/V bases must be 16-byte aligned and strides multiples of 16 bytes")
        dev = ks[0].device
        self.ks, self.vs = list(ks), list(vs)  # keep the storage alive
        self.tensormaps = None
        code = _lib.DTYPE_CODE[ks[0].dtype]
        if code != _lib.TC_F32 and d in (64, 128, 256):
            # tensor maps (one per K and V of every sequence) for the TMA kernel, encoded once here
            L = lib()
            bsz = len(ks)
            host = torch.empty(L.tc_ragged_tensormaps_size(bsz), dtype=torch.uint8)
            arr = ctypes.c_void_p * bsz
            i64 = ctypes.c_int64 * bsz
            st = L.tc_ragged_encode_tensormaps(
                host.data_ptr(), arr(*[k.data_ptr() for k in ks]), arr(*[v.data_ptr() for v in vs]),
                i64(*[k.shape[1] for k in ks]), i64(*[k.stride(0) for k in ks]), sn, bsz, hkv, d, code)
            check("tc_ragged_encode_tensormaps", st)
            self.tensormaps = host.to(dev)
        self.lengths_host = [int(n) for n in lengths]
        self.k_ptrs = torch.tensor([k.data_ptr() for k in ks], dtype=torch.int64).to(dev)
        self.v_ptrs = torch.tensor([v.data_ptr() for v in vs], dtype=torch.int64).to(dev)
        self.head_strides = torch.tensor([k.stride(0) for k in ks], dtype=torch.int64).to(dev)
        self.lengths = torch.tensor(self.lengths_host, dtype=torch.int32).to(dev)
        self.batch, self.hkv, self.d, self.token_stride = len(ks), hkv, d, sn
        self.max_n, self.total = max(self.lengths_host), sum(self.lengths_host)
        self.dtype, self.device = ks[0].dtype, dev


def decode_attention_ragged(q, kv: RaggedKV, scale, *, splits=None, out=None):
    """q: [b, hkv, g, d] (one query token per sequence). Returns [b, hkv, g, d]."""
    what = "decode_attention_ragged"
    require_cuda(q, what=what)
    if q.dtype != kv.dtype or q.device != kv.device:
        raise TypeError(f"{what}: q must match the caches' dtype/device")
    b, hkv, g, d = q.shape
    if b != kv.batch or hkv != kv.hkv or d != kv.d:
        raise ValueError(f"{what}: q {tuple(q.shape)} does not match the ragged caches")
    q = _last_contig(q)
    code = dtype_code(q, what)
    dev = q.device
    if out is None:
        out = torch.empty((b, hkv, g, d), dtype=q.dtype, device=dev)
    L = lib()
    s = int(splits or 0)
    ws = workspaces.get(("decode", b * hkv), dev, L.tc_decode_attention_workspace_size(b, hkv, g, d, kv.max_n, kv.total, s,
                                                                            code))
    with torch.cuda.device(dev):
        st = L.tc_decode_attention_ragged(
            q.data_ptr(), out.data_ptr(), kv.k_ptrs.data_ptr(), kv.v_ptrs.data_ptr(), kv.head_strides.data_ptr(),
            kv.lengths.data_ptr(), kv.tensormaps.data_ptr() if kv.tensormaps is not None else None,
            b, hkv, g, d, kv.max_n, kv.total, kv.token_stride,
            q.stride(0), q.stride(1), q.stride(2), out.stride(0), out.stride(1), out.stride(2),
            float(scale), s, code, ws.data_ptr(), ws.numel(), stream_ptr(dev))
    check("tc_decode_attention_ragged", st)
    return out


def merge_partials(o_parts, lse_parts, out_dtype):
    """LSE merge: o_parts fp32 [P, rows, d] (each normalised), lse_parts fp32 [P, rows] (natural
    log). Returns (out [rows, d] in out_dtype, lse fp32 [rows])."""
    what = "merge_partials"
    require_cuda(o_parts, lse_parts, what=what)
    o_parts = o_parts.float().contiguous()
    lse_parts = lse_parts.float().contiguous()
    p, rows, d = o_parts.shape
    if tuple(lse_parts.shape) != (p, rows):
        raise ValueError(f"{what}: lse_parts must be [{p}, {rows}]")
    out = torch.empty((rows, d), dtype=out_dtype, device=o_parts.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=o_parts.device)
    code = _lib.DTYPE_CODE[out_dtype]
    with torch.cuda.device(o_parts.device):
        st = lib().tc_merge_partials(o_parts.data_ptr(), lse_parts.data_ptr(), out.data_ptr(), lse.data_ptr(), p,
                                     rows, d, out.stride(0), code, stream_ptr(o_parts.device))
    check("tc_merge_partials", st)
    return out, lse

