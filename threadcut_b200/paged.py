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
    the decode tile table. No device work; PagedKV drives the kernels with what this returns.

    Runs are an int64 array [R, 3] (page, first row, rows) and the tile table an int32 array
    [T, 3] kept in step with them in a growable buffer: an append touches only the tail of the
    table (tiles from `dirty` on changed; a one-token append is O(1)), and a splice keeps the tiles
    of every run it does not cut and re-tiles only the runs cut at a, c0 and c0 + c."""

    def __init__(self, num_pages, page_rows):
        if page_rows < TILE_ROWS:
            raise ValueError(f"page_rows must be >= {TILE_ROWS}")
        self.num_pages = int(num_pages)
        self.page_rows = int(page_rows)
        self.free = list(range(self.num_pages - 1, -1, -1))  # stack: page 0 is taken first
        self._runs = np.zeros((0, 3), np.int64)
        self._tbuf = np.zeros((64, 3), np.int32)
        self._nt = 0
        self.n = 0
        self.version = 0  # bumped whenever the run list changes
        self.dirty = 0    # tiles [dirty, T) changed since the last mark_clean()

    @property
    def runs(self):
        return self._runs.tolist()

    def tiles(self):
        return self._tbuf[:self._nt]

    def mark_clean(self):
        self.dirty = self._nt

    def _set_tiles(self, keep, tail):
        """Tile table = the first `keep` tiles + `tail`."""
        need = keep + tail.shape[0]
        if need > self._tbuf.shape[0]:
            buf = np.zeros((max(need, 2 * self._tbuf.shape[0]), 3), np.int32)
            buf[:keep] = self._tbuf[:keep]
            self._tbuf = buf
        self._tbuf[keep:need] = tail
        self._nt = need
        self.dirty = min(self.dirty, keep)

    # ---------------------------------------------------------------- allocation
    def reserve(self, t):
        """Slots (page, row) for t new tokens at the end of the sequence, in order: first the rows
        after the last run in its page, then fresh pages. Returns an int32 array [t, 2]."""
        t = int(t)
        P = self.page_rows
        out = np.empty((t, 2), dtype=np.int32)
        if t == 0:
            return out
        runs = self._runs
        room = P - int(runs[-1, 1] + runs[-1, 2]) if runs.shape[0] else 0
        if t == 1 and room >= 1:
            # one-token step inside the last page: extend the last run and its last tile
            page, r = int(runs[-1, 0]), int(runs[-1, 1] + runs[-1, 2])
            out[0, 0], out[0, 1] = page, r
            runs[-1, 2] += 1
            last = self._tbuf[self._nt - 1]
            if int(last[2]) < TILE_ROWS and int(last[0]) == page and int(last[1] + last[2]) == r:
                last[2] += 1
                self.dirty = min(self.dirty, self._nt - 1)
            else:
                self._set_tiles(self._nt, np.asarray([[page, r, 1]], np.int32))
            self.n += 1
            self.version += 1
            return out
        first = min(room, t)
        n_new = -(-(t - first) // P)
        if n_new > len(self.free):
            raise MemoryError("PagedKV: no free page left in the pool")
        retile_run = runs.shape[0]  # runs from this index on are (re)tiled below
        keep = self._nt             # tiles before this index stay as they are
        if first > 0:
            page, r0 = int(runs[-1, 0]), int(runs[-1, 1] + runs[-1, 2])
            out[:first, 0] = page
            out[:first, 1] = np.arange(r0, r0 + first, dtype=np.int32)
            keep = self._nt - int(-(-runs[-1, 2] // TILE_ROWS))  # the last run's tiles are redone
            retile_run = runs.shape[0] - 1
            runs[-1, 2] += first
        if n_new:
            pages = [self.free.pop() for _ in range(n_new)]
            counts = np.full(n_new, P, np.int64)
            counts[-1] = (t - first) - P * (n_new - 1)
            new = np.stack([np.asarray(pages, np.int64), np.zeros(n_new, np.int64), counts], axis=1)
            out[first:, 0] = np.repeat(np.asarray(pages, np.int32), P)[:t - first]
            out[first:, 1] = np.tile(np.arange(P, dtype=np.int32), n_new)[:t - first]
            self._runs = np.concatenate((runs, new))
        self._set_tiles(keep, self.tiles_of(self._runs[retile_run:]))
        self.n += t
        self.version += 1
        return out

    # ---------------------------------------------------------------- splice
    def _index(self):
        cnt = self._runs[:, 2]
        end = np.cumsum(cnt)
        nt = (cnt + TILE_ROWS - 1) // TILE_ROWS
        tile0 = np.concatenate(([0], np.cumsum(nt)))
        return end, end - cnt, tile0

    def _span(self, lo, hi, end, start, tile0):
        """Runs covering logical tokens [lo, hi) cut at the ends, and their tiles: the tiles of runs
        kept whole are copied from the current table, cut runs are re-tiled."""
        if hi <= lo or self._runs.shape[0] == 0:
            return np.zeros((0, 3), np.int64), np.zeros((0, 3), np.int32)
        i0 = int(np.searchsorted(end, lo, side="right"))
        i1 = int(np.searchsorted(start, hi, side="left"))
        sel = self._runs[i0:i1].copy()
        cut_lo = lo - int(start[i0])
        cut_hi = int(end[i1 - 1]) - hi
        if cut_lo > 0:
            sel[0, 1] += cut_lo
            sel[0, 2] -= cut_lo
        if cut_hi > 0:
            sel[-1, 2] -= cut_hi
        k = sel.shape[0]
        a = 1 if cut_lo > 0 else 0                 # runs [a, b) of sel keep their old tiles
        b = k - 1 if (cut_hi > 0 and k - 1 >= a) else k
        parts = []
        if a:
            parts.append(self.tiles_of(sel[:1]))
        if b > a:
            parts.append(self._tbuf[tile0[i0 + a]:tile0[i0 + b]])
        if b < k:
            parts.append(self.tiles_of(sel[b:]))
        return sel, np.concatenate(parts) if parts else np.zeros((0, 3), np.int32)

    def _cut(self, lo, hi):
        """Runs covering logical tokens [lo, hi), split at the ends (int64 [k, 3])."""
        end, start, tile0 = self._index()
        return self._span(lo, hi, end, start, tile0)[0]

    def splice(self, s: Split):
        """Keep A = [0, a) and C = [c0, c0 + c) (threadcut/kv.py:28-33 semantics, everything after C
        dropped). Returns (C's runs in the new list as [k, 3] int64, pages freed)."""
        a, c0, c = int(s.a), int(s.c0), int(s.c)
        if not (0 <= a <= c0 and c >= 0 and c0 + c <= self.n):
            raise ValueError(f"splice {s} outside a sequence of {self.n} tokens")
        end, start, tile0 = self._index()
        runs_a, tiles_a = self._span(0, a, end, start, tile0)
        runs_c, tiles_c = self._span(c0, c0 + c, end, start, tile0)
        new = np.concatenate((runs_a, runs_c))
        old_used = np.zeros(self.num_pages, bool)
        old_used[self._runs[:, 0]] = True
        old_used[new[:, 0]] = False
        dropped = np.flatnonzero(old_used).tolist()
        self.free.extend(reversed(dropped))
        self._runs = new
        self._set_tiles(0, np.concatenate((tiles_a, tiles_c)))
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
        """Tile table [n_tiles, 3] int32 (page, first row, rows <= TILE_ROWS) covering `runs`."""
        runs = np.asarray(runs, np.int64).reshape(-1, 3)
        if runs.shape[0] == 0:
            return np.zeros((0, 3), np.int32)
        nt = (runs[:, 2] + TILE_ROWS - 1) // TILE_ROWS
        idx = np.repeat(np.arange(runs.shape[0]), nt)
        off = (np.arange(idx.shape[0]) - np.repeat(np.cumsum(nt) - nt, nt)) * TILE_ROWS
        sel = runs[idx]
        out = np.empty((idx.shape[0], 3), np.int32)
        out[:, 0] = sel[:, 0]
        out[:, 1] = sel[:, 1] + off
        out[:, 2] = np.minimum(TILE_ROWS, sel[:, 2] - off)
        return out

    def positions(self):
        """(page, row) of every logical token, int64 [n, 2] (for gathers and checks)."""
        runs = self._runs
        if runs.shape[0] == 0:
            return np.zeros((0, 2), np.int64)
        cnt = runs[:, 2]
        idx = np.repeat(np.arange(runs.shape[0]), cnt)
        k = np.arange(idx.shape[0]) - np.repeat(np.cumsum(cnt) - cnt, cnt)
        return np.stack((runs[idx, 0], runs[idx, 1] + k), axis=1)


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
        self._tiles_dev = None   # device int32 [capacity, 3]: the tile table, rows [0, n) valid
        self._tiles_ver = -1     # table version the device copy reflects
        self._ktab = None        # device int32 [T, 4]: tiles + logical start, for prefill
        self._ktab_starts = None
        self._ktab_ver = -1

    @property
    def n(self):
        return self.table.n

    @property
    def n_tiles(self):
        return self.table.tiles().shape[0]

    def _strides(self):
        s = next(t for t in self.k if t is not None).stride()  # compact() frees pools layer by layer
        return s[0], s[1], s[2]

    def _tiles(self):
        """Device tile table and its length, brought up to date by copying only the rows that
        changed since the last call (an append changes the tail; a splice everything)."""
        tab = self.table.tiles()
        nt = tab.shape[0]
        if self._tiles_ver != self.table.version:
            lo = self.table.dirty
            if self._tiles_dev is None or self._tiles_dev.shape[0] < nt:
                cap = max(nt, 2 * (self._tiles_dev.shape[0] if self._tiles_dev is not None else 0), 64)
                self._tiles_dev = torch.empty((cap, 3), dtype=torch.int32, device=self.device)
                lo = 0
            if lo < nt:
                self._tiles_dev[lo:nt].copy_(torch.from_numpy(np.ascontiguousarray(tab[lo:nt])))
            self.table.mark_clean()
            self._tiles_ver = self.table.version
        return (self._tiles_dev if nt else None), nt

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

    def decode(self, layer, q, scale, *, k_new=None, v_new=None, splits=None, stable_tiles=0):
        """Decode attention of q [hkv, g, d] over the whole sequence (threadcut/flash_decode.py:57-69
        semantics). With k_new/v_new [hkv, d] the last reserved row (a one-token step) is written by
        the same launch (fused append). stable_tiles: the leading tiles of the table (see
        `n_tiles`) whose rows no kernel still running writes, which the launch may load before the
        previous one ends (0: none; n_tiles - 1 in a layer-by-layer decode step with fused append,
        where each launch writes only the last row of its own layer)."""
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
                float(scale), int(splits or 0), code, int(stable_tiles), ws.data_ptr(), ws.numel(),
                stream_ptr(q.device)))
        return out

    def _prefill_table(self):
        """Device int32 [T, 4] = (page, first row, rows, logical position of the first row) of the
        current tile table, and the host copy of the logical starts."""
        if self._ktab_ver != self.table.version:
            tab = self.table.tiles()
            starts = (np.cumsum(tab[:, 2], dtype=np.int64) - tab[:, 2]).astype(np.int32)
            k4 = np.ascontiguousarray(np.concatenate((tab, starts[:, None]), axis=1))
            self._ktab = torch.from_numpy(k4).to(self.device)
            self._ktab_starts = starts
            self._ktab_ver = self.table.version
        return self._ktab, self._ktab_starts

    def prefill(self, layer, query, scale, *, splits=None):
        """Causal attention of a chunk's queries over the whole paged sequence, whose last lq tokens
        are the chunk (already written): query [1, 4*hkv, lq, 128] (bf16/fp16) -> [1, lq, hq, 128],
        as threadcut_b200.prefill.prefill_attention on the contiguous cache, with no copy of it."""
        require_cuda(query, what="PagedKV.prefill")
        _, hq, lq, d = query.shape
        n = self.table.n
        if (query.shape[0] != 1 or d != 128 or d != self.d or hq != 4 * self.hkv or query.dtype != self.dtype
                or query.dtype not in (torch.bfloat16, torch.float16) or not 1 <= lq <= n):
            raise ValueError(f"PagedKV.prefill: query {tuple(query.shape)} {query.dtype} does not fit the cache")
        ktab, starts = self._prefill_table()
        n_sub = ktab.shape[0]
        nqb = -(-lq // 64)
        kend = np.minimum(n, (n - lq) + 64 * (np.arange(nqb, dtype=np.int64) + 1))
        qbt = np.maximum(np.searchsorted(starts[::4], kend, side="left"), 1).astype(np.int32)
        qb_tiles = torch.from_numpy(qbt).to(self.device)
        q = query[0]
        if q.stride(-1) != 1:
            q = q.contiguous()
        out = torch.empty((1, lq, hq, d), dtype=query.dtype, device=query.device)
        L = lib()
        sp, sh, sr = self._strides()
        s = int(splits or 0)
        with torch.cuda.device(query.device):
            nb = L.tc_prefill_workspace_size(hq, self.hkv, lq, 128 * (-(-n_sub // 4)), s)
            ws = workspaces.get("prefill", query.device, nb) if nb else None
            st = L.tc_prefill_attention_paged(
                q.data_ptr(), self.k[layer].data_ptr(), self.v[layer].data_ptr(), out.data_ptr(), hq, self.hkv, lq, n,
                d, self.page_rows, self.table.num_pages, sp, sh, sr, ktab.data_ptr(), n_sub, qb_tiles.data_ptr(),
                q.stride(0), q.stride(1), out.stride(1), out.stride(2), float(scale), s, _lib.DTYPE_CODE[query.dtype],
                ws.data_ptr() if ws is not None else None, nb, stream_ptr(query.device))
        check("tc_prefill_attention_paged", st)
        return out

    # ---------------------------------------------------------------- splice
    def splice(self, s: Split, inv_freq):
        """A.B.C -> A.C on every layer (threadcut/kv.py:28-41, 83-92 semantics): B's pages return to
        the pool, C's keys are re-rotated by -(c0 - a) positions where they lie, nothing moves."""
        runs_c, _ = self.table.splice(s)
        gap = int(s.c0) - int(s.a)
        if gap == 0 or runs_c.shape[0] == 0:
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

    def compact(self):
        """Re-packs the sequence into pages in logical order (one copy of every layer's K and V into
        fresh pools), for when splices have left so many partly used pages that an append finds no
        free page. Peak memory: the old and the new pools."""
        new = PagedKV(self.layers, self.hkv, self.d, max_tokens=self.table.num_pages * self.page_rows,
                      page_rows=self.page_rows, dtype=self.dtype, device=self.device, spare_pages=0)
        n = self.n
        if n:
            new.reserve(n)
            for l in range(self.layers):
                k, v = self.gather(l)
                new.write(l, k, v)
                self.k[l] = self.v[l] = None  # free the old pools layer by layer
        self.__dict__.update(new.__dict__)

    # ---------------------------------------------------------------- views
    def gather(self, layer):
        """Contiguous copies (K, V) [hkv, n, d] of one layer in logical order (tc_paged_gather), for
        the attention paths that do not read pages and for compact()."""
        n = self.table.n
        k = torch.empty((self.hkv, n, self.d), dtype=self.dtype, device=self.device)
        v = torch.empty_like(k)
        if n == 0:
            return k, v
        ktab, _ = self._prefill_table()
        sp, sh, sr = self._strides()
        with torch.cuda.device(self.device):
            check("tc_paged_gather", lib().tc_paged_gather(
                self.k[layer].data_ptr(), self.v[layer].data_ptr(), k.data_ptr(), v.data_ptr(), self.hkv, self.d, n,
                k.stride(0), k.stride(1), self.page_rows, self.table.num_pages, sp, sh, sr, ktab.data_ptr(),
                ktab.shape[0], _lib.DTYPE_CODE[self.dtype], stream_ptr(self.device)))
        return k, v
