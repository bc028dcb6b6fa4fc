"""ctypes binding of the C ABI in include/threadcut_b200.h (libthreadcut_b200.so, built in-tree).

There is no fallback: if the shared library is missing or fails to load, every call raises. The
only torch involvement here is turning tensors into (pointer, stride, stream) triples and keeping
per-(device, stream) workspaces alive.
"""
import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libthreadcut_b200.so")

TC_F32, TC_F16, TC_BF16 = 0, 1, 2
DTYPE_CODE = {torch.float32: TC_F32, torch.float16: TC_F16, torch.bfloat16: TC_BF16}

_vp, _i, _i64, _f, _sz, _u32 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                ctypes.c_size_t, ctypes.c_uint32)
_fp = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); mirrors include/threadcut_b200.h one to one
SIGNATURES = {
    "tc_status_string": (ctypes.c_char_p, [_i]),
    "tc_abi_version": (_i, []),
    "tc_device_errors": (_i, [_i]),
    "tc_set_pdl": (_i, [_i]),
    "tc_decode_attention_workspace_size": (_sz, [_i, _i, _i, _i, _i64, _i64, _i, _i]),
    "tc_decode_attention": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 8
                            + [_f, _i, _i, _vp, _sz, _vp]),
    "tc_decode_attention_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 8 + [_f, _i, _i, _vp]),
    "tc_decode_attention_stable": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 8
                                   + [_f, _i, _i, _i64, _vp, _sz, _vp]),
    "tc_decode_attention_append": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 10
                                   + [_f, _i, _i, _i64, _vp, _sz, _vp]),
    "tc_decode_attention_append_rope": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 10
                                        + [_vp, _vp, _vp, _vp, _f, _f, _i, _i, _i64, _vp, _sz, _vp]),
    "tc_decode_attention_partial": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 8
                                    + [_f, _i, _i, _vp, _sz, _vp]),
    "tc_decode_attention_partial_stable": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 8
                                           + [_f, _i, _i, _i64, _vp, _sz, _vp]),
    "tc_decode_attention_lse": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i64] + [_i64] * 8
                                + [_f, _i, _i, _vp, _sz, _vp]),
    "tc_decode_attention_batched": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _vp] + [_i64] * 12
                                    + [_f, _i, _i, _vp, _sz, _vp]),
    "tc_decode_attention_ragged": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _i64, _i64]
                                   + [_i64] * 6 + [_f, _i, _i, _vp, _sz, _vp]),
    "tc_ragged_tensormaps_size": (_sz, [_i]),
    "tc_prefill_splits": (_i, [_i, _i, _i]),
    "tc_prefill_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "tc_prefill_attention": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i] + [_i64] * 8
                             + [_f, _i, _i, _vp, _sz, _vp]),
    "tc_split_workspace_size": (_sz, [_i64]),
    "tc_split": (_i, [_vp, _i64, _vp, _i64, _i, _i, _vp, _vp, _sz, _vp]),
    "tc_ragged_encode_tensormaps": (_i, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_i64),
                                         ctypes.POINTER(_i64), _i64, _i, _i, _i, _i]),
    "tc_shift_keys": (_i, [_vp, _vp, _i64, _i64, _i] + [_i64] * 4 + [_fp, _i, _vp]),
    "tc_splice_workspace_size": (_sz, [_i, _i, _i64]),
    "tc_splice_inplace": (_i, [ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i, _i, _i, _i64, _i64, _i64, _i64,
                               _i64, _i64, _fp, _i, _vp, _sz, _u32, _vp]),
    "tc_splice_copy": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i64, _i64, _i64] + [_i64] * 4 + [_fp, _i, _vp]),
    "tc_merge_partials": (_i, [_vp, _vp, _vp, _vp, _i, _i64, _i, _i64, _i, _vp]),
    "tc_add_rmsnorm": (_i, [_vp, _vp, _vp, _vp, _i64, _i, _f, _i, _vp]),
    "tc_qk_norm_rope": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _vp]),
    "tc_silu_mul": (_i, [_vp, _vp, _i64, _i, _i, _vp]),
    "tc_gemv": (_i, [_vp, _vp, _vp, _i64, _i, _i, _vp]),
    "tc_gemv_swiglu": (_i, [_vp, _vp, _vp, _i64, _i, _i, _vp]),
    "tc_decode_attention_paged": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i64, _i64, _i64, _i64, _i64, _vp, _i64,
                                       _i64, _vp, _vp, _i64, _i64] + [_i64] * 4 + [_f, _i, _i, _i64, _vp, _sz, _vp]),
    "tc_prefill_attention_paged": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i64, _i64, _i64, _i64, _i64, _vp,
                                        _i64, _vp, _i64, _i64, _i64, _i64, _f, _i, _i, _vp, _sz, _vp]),
    "tc_paged_gather": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64,
                             _i, _vp]),
    "tc_paged_rotate_keys": (_i, [ctypes.POINTER(_vp), _i, _i, _i, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _fp,
                                  _i, _vp]),
    "tc_paged_write": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i64] + [_i64] * 4 + [_i64] * 5 + [_vp, _i, _vp]),
    "tc_peer_handle_bytes": (_sz, []),
    "tc_peer_alloc": (_i, [_sz, ctypes.POINTER(_vp), _vp]),
    "tc_peer_open": (_i, [_vp, ctypes.POINTER(_vp)]),
    "tc_peer_close": (_i, [_vp]),
    "tc_peer_free": (_i, [_vp]),
    "tc_allreduce_region_bytes": (_sz, [_i, _i64]),
    "tc_gemv_allreduce": (_i, [_vp, _vp, _i64, _i, ctypes.POINTER(_vp), _i, _i, _i, _vp]),
    "tc_gemv_allreduce_swiglu": (_i, [_vp, _vp, _i64, _i, ctypes.POINTER(_vp), _i, _i, _i, _vp]),
    "tc_allreduce_add_rmsnorm": (_i, [_vp, _vp, _vp, _i, _f, _vp, _i, _i, _vp]),
    "tc_gemv_allreduce_residual": (_i, [_vp, _vp, _i64, _i, ctypes.POINTER(_vp), _i, _i, _vp, _i, _vp]),
    "tc_gemv_allreduce_residual_swiglu": (_i, [_vp, _vp, _i64, _i, ctypes.POINTER(_vp), _i, _i, _vp, _i, _vp]),
    "tc_gemv_rmsnorm": (_i, [_vp, _vp, _vp, _f, _vp, _vp, _i64, _i, _i, _vp]),
    "tc_gemv_rmsnorm_swiglu": (_i, [_vp, _vp, _vp, _f, _vp, _vp, _i64, _i, _i, _vp]),
    "tc_gather_region_bytes": (_sz, [_i, _i64, _i]),
    "tc_peer_gather_merge": (_i, [_vp, _vp, _vp, _vp, _i64, _i, _i64, ctypes.POINTER(_vp), _i, _i, _i, _vp]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded C library. Raises RuntimeError when it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"threadcut_b200: {LIB_PATH} is missing; build it with "
                        "`python -m threadcut_b200.build` (there is no non-CUDA fallback)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype, fn.argtypes = res, args
                _lib = handle
    return _lib


HOST_PATH = os.path.join(_HERE, "_host", "threadcut_b200_host.so")
_host = None


def host():
    """The compiled host binding (csrc/host_binding.cpp) with its pointer to this package's loaded
    tc_decode_attention_stable, or None when it has not been built (the ctypes path is used then).
    It only moves the argument marshalling out of the interpreter; the kernels are the same."""
    global _host
    if _host is None:
        handle = lib()  # outside the lock below: lib() takes it itself
        with _lock:
            if _host is None:
                mod = False
                if os.path.exists(HOST_PATH):
                    import importlib.util
                    spec = importlib.util.spec_from_file_location("threadcut_b200_host", HOST_PATH)
                    mod = importlib.util.module_from_spec(spec)
                    spec.loader.exec_module(mod)
                    mod.init(ctypes.cast(handle.tc_decode_attention_stable, ctypes.c_void_p).value)
                    if hasattr(mod, "init_partial"):
                        mod.init_partial(ctypes.cast(handle.tc_decode_attention_partial_stable, ctypes.c_void_p).value)
                _host = mod
    return _host or None


class TCError(RuntimeError):
    def __init__(self, fn, status):
        msg = lib().tc_status_string(status).decode()
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def check(fn, status):
    if status != 0:
        raise TCError(fn, status)


def require_cuda(*tensors, what):
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(f"threadcut_b200.{what}: tensors must be on a CUDA device (B200 only, no CPU path); "
                               f"got {t.device}")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"threadcut_b200.{what}: all tensors must be on {dev}, got {t.device}")


def dtype_code(t, what):
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise TypeError(f"threadcut_b200.{what}: unsupported dtype {t.dtype}") from None


def stream_ptr(device):
    """Raw cudaStream_t of torch's current stream on `device` (what every launch goes to)."""
    return torch._C._cuda_getCurrentRawStream(device.index if device.index is not None
                                             else torch.cuda.current_device())


_MAX_N_FOR_BOUND = 1 << 31
_ws_bound_cache = {}


def decode_workspace_bound(batch, hkv, g, d, code):
    """Workspace bytes that suffice for every decode call of this geometry whatever n or splits is
    (the planner never uses more than 128 slices per head), cached per geometry."""
    key = (batch, hkv, g, d, code)
    nb = _ws_bound_cache.get(key)
    if nb is None:
        nb = lib().tc_decode_attention_workspace_size(batch, hkv, g, d, _MAX_N_FOR_BOUND, batch * _MAX_N_FOR_BOUND,
                                                      128, code)
        _ws_bound_cache[key] = nb
    return nb


def cos_sin_table(delta, inv_freq):
    """fp32 host table [cos(delta*inv_freq) ..., sin(delta*inv_freq) ...] as threadcut/kv.py:22-25
    builds it: the angle is delta * inv_freq in fp32, cos/sin of it in fp32 (torch, on the host)."""
    angle = delta * inv_freq.detach().to("cpu", torch.float32)
    emb = torch.cat((angle, angle))
    h = angle.numel()
    tab = torch.cat((emb.cos()[:h], emb.sin()[:h])).contiguous()
    return tab, ctypes.cast(tab.data_ptr(), _fp)


class _Workspaces:
    """Per (kind, device, stream) scratch buffers, zero-initialised, grown on demand. The kernels
    leave their ticket counters at zero, so a buffer is only zeroed when it is (re)allocated.
    Decode workspaces are keyed by ("decode", batch*hkv): the ticket prefix grows with batch*hkv,
    and a prefix that overlapped an earlier call's partials would not start at zero."""

    def __init__(self):
        self._bufs = {}
        self._epochs = {}
        self._lock = threading.Lock()

    def get(self, kind, device, nbytes, stream=None):
        key = (kind, device.index, stream_ptr(device) if stream is None else stream)
        buf = self._bufs.get(key)
        if buf is not None and buf.numel() >= nbytes:
            return buf
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
                self._epochs[key] = 0
            return buf

    def next_epoch(self, kind, device):
        key = (kind, device.index, stream_ptr(device))
        with self._lock:
            e = (self._epochs.get(key, 0) % 0xFFFFFFFF) + 1
            self._epochs[key] = e
            return e


workspaces = _Workspaces()


def device_errors(clear=True):
    """Device error bits of the current device (synchronises). 0 means no bounded wait gave up."""
    v = lib().tc_device_errors(1 if clear else 0)
    if v < 0:
        raise RuntimeError("threadcut_b200: reading the device error word failed")
    return v
