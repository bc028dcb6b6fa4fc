"""Splice bookkeeping (host, integer) — drop-in for threadcut/match.py.

    cached = A . B . C . (stale tail)        new = A . C . D

A is the longest common prefix, B the pruned span, C the longest run of `new` after A that also
occurs in the cache after A (at least `min_suffix` tokens), D what the model still has to run.
`Split(a, c0, c)` with gap = c0 - a is what the device splice consumes. Same rule and tie-breaking
as threadcut/match.py:33-48: at least one token of D is always left, and among candidate C starts
the first one with the longest match wins.
"""
from dataclasses import dataclass

import numpy as np

__all__ = ["Split", "lcp", "split", "split_device"]


@dataclass(frozen=True)
class Split:
    a: int   # len(A)
    c0: int  # C starts at cached[c0]; B = cached[a:c0]
    c: int   # len(C); D = new[a + c:]

    @property
    def gap(self):
        return self.c0 - self.a


def lcp(x, y):
    """Length of the longest common prefix of two token sequences."""
    m = min(len(x), len(y))
    if m == 0:
        return 0
    neq = np.asarray(x[:m]) != np.asarray(y[:m])
    first = int(np.argmax(neq))
    return first if neq[first] else m


def _window_starts(hay, needle):
    """Ascending offsets i with hay[i:i+len(needle)] == needle (numpy, vectorised per needle token)."""
    k = len(needle)
    if len(hay) < k:
        return np.empty(0, dtype=np.int64)
    span = len(hay) - k + 1
    ok = np.ones(span, dtype=bool)
    for t, tok in enumerate(needle):
        ok &= hay[t:t + span] == tok
        if not ok.any():
            break
    return np.flatnonzero(ok)


def split(cached, new, min_suffix=32, suffix=True):
    a = min(lcp(cached, new), len(new) - 1)  # keep >= 1 token of D so there are logits to return
    rest = list(new[a:])
    if not suffix or len(rest) <= min_suffix or len(cached) - (a + 1) < min_suffix:
        return Split(a, a, 0)
    hay = np.asarray(cached[a + 1:])
    starts = _window_starts(hay, np.asarray(rest[:min_suffix])) + (a + 1)
    best = Split(a, a, 0)
    for j in starts.tolist():
        c = min(lcp(cached[j:], rest), len(rest) - 1)
        if c > best.c:
            best = Split(a, j, c)
    return best


def split_device(cached, new, min_suffix=32, suffix=True, device=None):
    """split() computed on the GPU (tc_split): same rule and tie-breaking, integer-exact. `cached`
    and `new` are token-id sequences (lists, numpy arrays or int tensors; ids must fit int32);
    host sequences are copied to `device` (default: the current CUDA device). Returns a Split
    (reading it back synchronises the stream). `new` must be non-empty."""
    import torch

    from ._lib import check, lib, stream_ptr, workspaces

    if len(new) == 0:
        raise ValueError("split_device: `new` must hold at least one token")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise RuntimeError("split_device: needs a CUDA device (the host rule is split())")

    def as_dev(x):
        if isinstance(x, torch.Tensor) and x.dtype == torch.int32:
            return x.to(device=dev).contiguous()
        t = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x, dtype=np.int64))
        if t.numel() and (int(t.max()) > 2**31 - 1 or int(t.min()) < -2**31):
            raise ValueError("split_device: token ids must fit int32")
        return t.to(device=dev, dtype=torch.int32).contiguous()

    c, n = as_dev(cached), as_dev(new)
    L = lib()
    ws = workspaces.get(("split",), dev, L.tc_split_workspace_size(c.numel()))
    out = torch.empty(3, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        check("tc_split", L.tc_split(c.data_ptr() if c.numel() else None, c.numel(), n.data_ptr(), n.numel(),
                                     int(min_suffix), 1 if suffix else 0, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                     stream_ptr(dev)))
    a, c0, cl = out.tolist()
    return Split(int(a), int(c0), int(cl))

