"""Paged K/V cache: the layout threadcut names as its next step (README.md:141-144, "drop B by
freeing pages, rotate C in place with no move").

threadcut's splice (kv.py:28-41, 83-92) turns A.B.C into A.C by copying C's K and V rows down to
position a and re-rotating the keys by -(c0 - a) positions. Here every layer keeps its K and V in
pools of fixed-size pages, and a sequence is an ordered list of runs (page, first row, rows). The
splice then

  * cuts the run list at a, c0 and c0 + c and keeps A's and C's runs, in that order;
  * returns every page that no kept run touches to the free list (B and the stale tail);
  * re-rotates C's keys where they lie (tc_paged_rotate_keys, every layer in one launch).

No row of K or V moves, and V is not touched at all: the splice costs a read and a write of C's
keys instead of a read and a write of C's keys and values. Decode reads the pages through a tile
table (tc_decode_attention_paged); appends write into the free rows after the last run and then
into fresh pages (tc_paged_write, or fused into the decode launch for one token).

The logical order of the runs is always the reference cache's token order, and rows inside a page
are only ever written in that order, so the rows after the last run's end in its page hold no
live token and the next append may take them.
"""
import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import check, dtype_code, lib, require_cuda, stream_ptr, workspaces
from .match import Split

__all__ = ["PageTable", "PagedKV", "TILE_ROWS"]

TILE_ROWS = 32  # rows per tile-table entry (the decode kernel's tile height)


class PageTable:
    """Host bookkeeping of one paged sequence: free pages, the run list, slot allocation, splice and
    the decode tile table. No device work; PagedKV drives the kernels with what this returns."""

    def __init__(self, num_pages, page_rows):
        if page_rows < TILE_ROWS:
            raise ValueError(f"page_rows must be >= {TILE_ROWS}")
        self.num_pages = int(num_pages)
        self.page_rows = int(page_rows)
        self.free = list(range(self.num_pages - 1, -1, -1))  # stack: page 0 is taken first
        self.runs = []  # [page, first row, rows] in logical order
        self.n = 0
        self.version = 0  # bumped whenever the run list changes

    # ---------------------------------------------------------------- allocation
    def _take_page(self):
        if not self.free:
            raise MemoryError("PagedKV: no free page left in the pool")
        return self.free.pop()

    def reserve(self, t):
        """Slots (page, row) for t new tokens at the end of the sequence, in order: first the rows
        after the last run in its page, then fresh pages. Returns an int32 array [t, 2]."""
        t = int(t)
        out = np.empty((t, 2), dtype=np.int32)
        i = 0
        while i < t:
            if self.runs:
                last = self.runs[-1]
                room = self.page_rows - (last[1] + last[2])
            else:
                room = 0
            if room <= 0:
                self.runs.append([self._take_page(), 0, 0])
                continue
            take = min(room, t - i)
            r0 = last[1] + last[2]
            out[i:i + take, 0] = last[0]
            out[i:i + take, 1] = np.arange(r0, r0 + take, dtype=np.int32)
            last[2] += take
            i += take
        self.n += t
        self.version += 1
        return out

    # ---------------------------------------------------------------- splice
    def _cut(self, lo, hi):
        """Runs covering logical tokens [lo, hi), split at the ends."""
        out, pos = [], 0
        for page, r0, cnt in self.runs:
            a, b = max(lo, pos), min(hi, pos + cnt)
            if a < b:
                out.append([page, r0 + (a - pos), b - a])
            pos += cnt
            if pos >= hi:
                break
        return out

    def splice(self, s: Split):
        """Keep A = [0, a) and C = [c0, c0 + c) (threadcut/kv.py:28-33 semantics, everything after C
        dropped). Returns (C's runs in the new list, pages freed)."""
        a, c0, c = int(s.a), int(s.c0), int(s.c)
        if not (0 <= a <= c0 and c >= 0 and c0 + c <= self.n):
            raise ValueError(f"splice {s} outside a sequence of {self.n} tokens")
        runs_a = self._cut(0, a)
        runs_c = self._cut(c0, c0 + c)
        kept = {r[0] for r in runs_a} | {r[0] for r in runs_c}
        dropped = sorted({r[0] for r in self.runs} - kept)
        self.free.extend(reversed(dropped))
        self.runs = runs_a + runs_c
        self.n = a + c
        self.version += 1
        return runs_c, dropped

    def truncate(self, n):
        """Keep the first n tokens (a crop), freeing pages no longer used."""
        n = int(n)
        if n >= self.n:
            return []
        return self.splice(Split(n, n, 0))[1]

    # ---------------------------------------------------------------- tables
    @staticmethod
    def tiles_of(runs):
        """Tile table [n_tiles, 3] (page, first row, rows <= TILE_ROWS) covering `runs` in order."""
        rows = []
        for page, r0, cnt in runs:
            for off in range(0, cnt, TILE_ROWS):
                rows.append((page, r0 + off, min(TILE_ROWS, cnt - off)))
        return np.asarray(rows, dtype=np.int32).reshape(-1, 3)

    def tiles(self):
        return self.tiles_of(self.runs)

    def positions(self):
        """(page, row) of every logical token, int64 [n, 2] (for gathers and checks)."""
        out = np.empty((self.n, 2), dtype=np.int64)
        i = 0
        for page, r0, cnt in self.runs:
            out[i:i + cnt, 0] = page
            out[i:i + cnt, 1] = np.arange(r0, r0 + cnt)
            i += cnt
        return out


class PagedKV:
    """Paged K/V of `layers` attention layers of one sequence on one GPU.

    Pools: k[l], v[l] of shape [pages, hkv, page_rows, d] (16-bit dtypes for decode). A step is
    `reserve(t)` (once, for all layers) followed by `write(l, k, v)` per layer, or, for a one-token
    decode step, `decode(l, q, scale, k_new=..., v_new=...)` per layer, which writes the new row in
    the same launch that reads the cache."""

    def __init__(self, layers, hkv, d, *, max_tokens, page_rows=64, dtype=torch.bfloat16, device=None,
                 spare_pages=2):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise RuntimeError("PagedKV: needs a CUDA device")
        self.layers, self.hkv, self.d = int(layers), int(hkv), int(d)
        self.page_rows = int(page_rows)
        pages = -(-int(max_tokens) // self.page_rows) + int(spare_pages)
        self.table = PageTable(pages, self.page_rows)
        self.dtype, self.device = dtype, dev
        shape = (pages, self.hkv, self.page_rows, self.d)
        self.k = [torch.zeros(shape, dtype=dtype, device=dev) for _ in range(self.layers)]
        self.v = [torch.zeros(shape, dtype=dtype, device=dev) for _ in range(self.layers)]
        self._kptrs = (ctypes.c_void_p * self.layers)(*[t.data_ptr() for t in self.k])
        self._slots = None       # device int32 [t, 2] of the step reserved last
        self._tiles_dev = None   # device int32 [n_tiles, 3] of table version _tiles_ver
        self._tiles_n = 0
        self._tiles_ver = -1

    @property
    def n(self):
        return self.table.n

    def _strides(self):
        s = self.k[0].stride()
        return s[0], s[1], s[2]

    def _tiles(self):
        if self._tiles_ver != self.table.version:
            tab = self.table.tiles()
            self._tiles_n = tab.shape[0]
            self._tiles_dev = torch.from_numpy(tab).to(self.device) if tab.size else None
            self._tiles_ver = self.table.version
        return self._tiles_dev, self._tiles_n

    # ---------------------------------------------------------------- step
    def reserve(self, t):
        """Takes t slots at the end of the sequence for the next write/decode of every layer."""
        slots = self.table.reserve(t)
        self._slots = torch.from_numpy(slots).to(self.device)
        return self._slots

    def write(self, layer, k, v):
        """Writes the reserved step's rows of one layer: k, v [hkv, t, d] (or [1, hkv, t, d])."""
        if k.dim() == 4:
            k, v = k[0], v[0]
        require_cuda(k, v, what="PagedKV.write")
        t = k.shape[1]
        if self._slots is None or self._slots.shape[0] != t:
            raise ValueError("PagedKV.write: reserve(t) the step's slots first (same t)")
        if k.shape != (self.hkv, t, self.d) or v.shape != k.shape or k.dtype != self.dtype or v.dtype != self.dtype:
            raise ValueError(f"PagedKV.write: expected [{self.hkv}, t, {self.d}] {self.dtype}, got {tuple(k.shape)} {k.dtype}")
        if k.stride(-1) != 1 or v.stride(-1) != 1:
            k, v = k.contiguous(), v.contiguous()
        sp, sh, sr = self._strides()
        with torch.cuda.device(self.device):
            check("tc_paged_write", lib().tc_paged_write(
                k.data_ptr(), v.data_ptr(), self.k[layer].data_ptr(), self.v[layer].data_ptr(), self.hkv, self.d, t,
                k.stride(0), k.stride(1), v.stride(0), v.stride(1), self.page_rows, self.table.num_pages,
                sp, sh, sr, self._slots.data_ptr(), dtype_code(k, "PagedKV.write"), stream_ptr(self.device)))

    def decode(self, layer, q, scale, *, k_new=None, v_new=None, splits=None):
        """Decode attention of q [hkv, g, d] over the whole sequence (threadcut/flash_decode.py:57-69
        semantics). With k_new/v_new [hkv, d] the last reserved row (a one-token step) is written by
        the same launch (fused append)."""
        require_cuda(q, what="PagedKV.decode")
        hkv, g, d = q.shape
        if hkv != self.hkv or d != self.d or q.dtype != self.dtype:
            raise ValueError(f"PagedKV.decode: q {tuple(q.shape)} {q.dtype} does not match the cache")
        if (k_new is None) != (v_new is None):
            raise ValueError("PagedKV.decode: k_new and v_new go together")
        if k_new is not None:
            if self._slots is None or self._slots.shape[0] != 1:
                raise ValueError("PagedKV.decode: reserve(1) the step's slot before a fused append")
            if k_new.dim() == 3:
                k_new, v_new = k_new.reshape(hkv, d), v_new.reshape(hkv, d)
            if k_new.shape != (hkv, d) or v_new.shape != (hkv, d):
                raise ValueError("PagedKV.decode: k_new/v_new must be [hkv, d]")
            if k_new.stride(-1) != 1 or v_new.stride(-1) != 1:
                k_new, v_new = k_new.contiguous(), v_new.contiguous()
        if q.stride(-1) != 1:
            q = q.contiguous()
        tiles, nt = self._tiles()
        out = torch.empty((hkv, g, d), dtype=q.dtype, device=q.device)
        code = dtype_code(q, "PagedKV.decode")
        ws = workspaces.get(("decode", hkv), q.device, _lib.decode_workspace_bound(1, hkv, g, d, code))
        sp, sh, sr = self._strides()
        with torch.cuda.device(q.device):
            check("tc_decode_attention_paged", lib().tc_decode_attention_paged(
                q.data_ptr(), self.k[layer].data_ptr(), self.v[layer].data_ptr(), out.data_ptr(), hkv, g, d,
                self.page_rows, self.table.num_pages, sp, sh, sr, tiles.data_ptr() if tiles is not None else None,
                nt, self.table.n, k_new.data_ptr() if k_new is not None else None,
                v_new.data_ptr() if v_new is not None else None, k_new.stride(0) if k_new is not None else 0,
                v_new.stride(0) if v_new is not None else 0, q.stride(0), q.stride(1), out.stride(0), out.stride(1),
                float(scale), int(splits or 0), code, ws.data_ptr(), ws.numel(), stream_ptr(q.device)))
        return out

    # ---------------------------------------------------------------- splice
    def splice(self, s: Split, inv_freq):
        """A.B.C -> A.C on every layer (threadcut/kv.py:28-41, 83-92 semantics): B's pages return to
        the pool, C's keys are re-rotated by -(c0 - a) positions where they lie, nothing moves."""
        runs_c, _ = self.table.splice(s)
        gap = int(s.c0) - int(s.a)
        if gap == 0 or not runs_c:
            return  # the reference clones C onto itself: nothing to rotate
        tab = PageTable.tiles_of(runs_c)
        tiles = torch.from_numpy(tab).to(self.device)
        cs, cs_ptr = _lib.cos_sin_table(-gap, inv_freq)
        sp, sh, sr = self._strides()
        with torch.cuda.device(self.device):
            check("tc_paged_rotate_keys", lib().tc_paged_rotate_keys(
                self._kptrs, self.layers, self.hkv, self.d, self.page_rows, self.table.num_pages, sp, sh, sr,
                tiles.data_ptr(), tab.shape[0], cs_ptr, _lib.DTYPE_CODE[self.dtype], stream_ptr(self.device)))
        del cs  # the table is copied into the launch parameters

    def truncate(self, n):
        self.table.truncate(n)

    # ---------------------------------------------------------------- views
    def gather(self, layer):
        """Contiguous copies (K, V) [hkv, n, d] of one layer in logical order (torch indexing; for
        prefill chunks and checks, not the decode path)."""
        pos = torch.from_numpy(self.table.positions()).to(self.device)
        k = self.k[layer][pos[:, 0], :, pos[:, 1], :]  # [n, hkv, d]
        v = self.v[layer][pos[:, 0], :, pos[:, 1], :]
        return k.transpose(0, 1).contiguous(), v.transpose(0, 1).contiguous()
