"""KV-cache surgery on B200 — drop-in for threadcut/kv.py.

A request that prunes span B turns the cache A.B.C into A.C. Keys are cached after RoPE and
rotations compose, so moving C left by gap = |B| positions only needs every key of C re-rotated by
-gap (threadcut/kv.py:1-7); values move unchanged.

* `shift_keys(keys, delta, inv_freq)` (kv.py:20-25): out-of-place re-rotation, kernel
  tc_shift_keys. Bit-identical to the reference's fp32 torch expression for the same cos/sin table.
* `GrowingLayer` (kv.py:44-92): the same preallocated, 1.25x-growing per-layer buffer
  [b, hkv, cap, d] with `keys`/`values` views; `splice` runs tc_splice_inplace (one launch, in
  place even when C's source and destination rows overlap).
* `splice(cache, s, inv_freq)` (kv.py:28-41): when every layer is a GrowingLayer with the same
  buffer geometry, ALL layers are spliced in ONE launch; otherwise the copy path (tc_splice_copy per
  layer, new tensors, as the reference's index_select path).
* `new_cache(config)` (kv.py:95-98); `use_paged_cache()` switches what it builds to the paged layout.
The cos/sin table is built on the host exactly as the reference builds it (fp32 angle
delta*inv_freq, torch cos/sin) and passed by value into the launch.
"""
import ctypes

import torch
from transformers import DynamicCache
from transformers.cache_utils import DynamicLayer

from ._lib import check, cos_sin_table, dtype_code, lib, require_cuda, stream_ptr, workspaces
from .match import Split

__all__ = ["rotate_half", "shift_keys", "splice", "GrowingLayer", "new_cache", "use_paged_cache"]

# attention implementation that consumes deferred appends (threadcut_b200.attention.NAME)
FUSED_ATTENTION = "threadcut"
# kbuf address -> GrowingLayer whose last appended row is not written yet (the fused decode writes it)
_PENDING = {}


def rotate_half(x):
    """(x1, x2) -> (-x2, x1) over the two halves of the last dim (torch; used by callers' RoPE)."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _rows_view(t):
    """View t [..., n, d] as [outer, n, d] without copying when the leading dims collapse."""
    if t.dim() == 2:
        return t.unsqueeze(0)
    return t.reshape(-1, t.shape[-2], t.shape[-1])


def shift_keys(keys, delta, inv_freq):
    """Move post-RoPE keys by `delta` positions (negative = left). Math in fp32, result in keys.dtype."""
    what = "shift_keys"
    require_cuda(keys, what=what)
    code = dtype_code(keys, what)
    d = keys.shape[-1]
    if inv_freq.numel() * 2 != d:
        raise ValueError(f"{what}: inv_freq has {inv_freq.numel()} entries, keys need {d // 2}")
    src = keys if keys.stride(-1) == 1 else keys.contiguous()
    src3 = _rows_view(src)
    out = torch.empty(keys.shape, dtype=keys.dtype, device=keys.device)
    out3 = out.view(src3.shape)
    tab, tab_ptr = cos_sin_table(int(delta), inv_freq)
    with torch.cuda.device(keys.device):
        st = lib().tc_shift_keys(src3.data_ptr(), out3.data_ptr(), src3.shape[0], src3.shape[1], d,
                                 src3.stride(0), src3.stride(1), out3.stride(0), out3.stride(1), tab_ptr, code,
                                 stream_ptr(keys.device))
    check("tc_shift_keys", st)
    del tab
    return out


def _splice_growing(layers, s: Split, inv_freq):
    """In-place A.B.C -> A.C over GrowingLayers that share buffer geometry: one kernel launch."""
    kb0 = layers[0].kbuf
    require_cuda(kb0, what="splice")
    b, hkv, cap, d = kb0.shape
    code = dtype_code(kb0, "splice")
    L = len(layers)
    # the batch dim folds into the head dim (b = 1 in the engine; b > 1 works when contiguous)
    kptrs = (ctypes.c_void_p * L)(*[ly.kbuf.data_ptr() for ly in layers])
    vptrs = (ctypes.c_void_p * L)(*[ly.vbuf.data_ptr() for ly in layers])
    if b != 1 and kb0.stride(0) != hkv * kb0.stride(1):
        raise ValueError("splice: batched GrowingLayer buffers must be contiguous over (b, hkv)")
    if s.a < 0 or s.c < 0 or s.c0 < s.a or s.c0 + s.c > cap:
        raise ValueError(f"splice: {s} does not fit a buffer of {cap} rows")
    tab, tab_ptr = cos_sin_table(-s.gap, inv_freq)
    dev = kb0.device
    lk = lib()
    ws = workspaces.get("splice", dev, lk.tc_splice_workspace_size(L, b * hkv, s.c))
    epoch = workspaces.next_epoch("splice", dev)
    with torch.cuda.device(dev):
        st = lk.tc_splice_inplace(kptrs, vptrs, L, b * hkv, d, cap, s.a, s.c0, s.c, kb0.stride(1), kb0.stride(2),
                                  tab_ptr, code, ws.data_ptr(), ws.numel(), epoch, stream_ptr(dev))
    check("tc_splice_inplace", st)
    del tab


def _same_geometry(layers):
    k0 = layers[0].kbuf
    for ly in layers:
        for t in (ly.kbuf, ly.vbuf):
            if (t is None or t.shape != k0.shape or t.stride() != k0.stride() or t.dtype != k0.dtype
                    or t.device != k0.device):
                return False
    return True


def splice(cache, s: Split, inv_freq):
    """Rewrite every layer of a DynamicCache from A.B.C.(tail) to A.C."""
    layers = cache.layers
    if layers and all(isinstance(layer, PagedLayer) for layer in layers):
        state = layers[0].state
        state.flush_all()
        if state.kv is not None:
            state.kv.splice(s, inv_freq)  # B's pages freed, C's keys re-rotated in place
        return
    if all(isinstance(layer, GrowingLayer) for layer in layers):
        live = [ly for ly in layers if ly.kbuf is not None]
        if s.c and s.gap and live:
            if _same_geometry(live):
                _splice_growing(live, s, inv_freq)
            else:
                for ly in live:
                    _splice_growing([ly], s, inv_freq)
        for ly in layers:
            ly.n = s.a + s.c
            if ly.kbuf is not None:
                ly._view()
        return
    for layer in layers:
        k, v = layer.keys, layer.values
        require_cuda(k, v, what="splice")
        bsz, hkv, _, d = k.shape
        nk = torch.empty((bsz, hkv, s.a + s.c, d), dtype=k.dtype, device=k.device)
        nv = torch.empty_like(nk)
        tab, tab_ptr = cos_sin_table(-s.gap, inv_freq)
        code = dtype_code(k, "splice")
        for i in range(bsz):
            ki, vi = k[i], v[i]
            if ki.stride(-1) != 1:
                ki = ki.contiguous()
            if vi.stride(-1) != 1 or vi.stride() != ki.stride():
                vi = vi.contiguous()
                ki = ki.contiguous()
            with torch.cuda.device(k.device):
                st = lib().tc_splice_copy(ki.data_ptr(), vi.data_ptr(), nk[i].data_ptr(), nv[i].data_ptr(), hkv, d,
                                          s.a, s.c0, s.c, ki.stride(0), ki.stride(1), nk.stride(1), nk.stride(2),
                                          tab_ptr, code, stream_ptr(k.device))
            check("tc_splice_copy", st)
        del tab
        layer.keys, layer.values = nk, nv


class GrowingLayer(DynamicLayer):
    """DynamicLayer backed by a preallocated buffer: appending a token writes in place instead of
    re-copying the whole cache with torch.cat. Grows by max(need, 1.25x, +2048 tokens), the same
    policy as threadcut/kv.py:53-63.

    Fused append (`fuse_append`, set by new_cache when the model's attention is threadcut_b200's):
    a one-token update on a CUDA cache does not write the row; it returns the views with the row
    pending, and the decode branch of threadcut_b200.attention writes it in the same launch that
    reads the cache (tc_decode_attention_append). Any other use of the cache (another update,
    crop, splice, a prefill or batched attention call) writes the pending row first. A model switched
    to another attention implementation after new_cache reads the cache itself: set fuse_append to
    False on its layers, or the step's row is not in the buffer when that attention reads it."""

    fuse_append = False

    def lazy_initialization(self, key_states, value_states, *args, **kwargs):
        super().lazy_initialization(key_states, value_states)
        self.n, self.kbuf, self.vbuf = 0, None, None
        self._pending = None   # (k [hkv, d], v [hkv, d]) of row n-1, not yet in the buffers
        self._plain_write = True  # the buffers were last written by a plain copy (not a fused decode)

    def _reserve(self, need, like):
        cap = 0 if self.kbuf is None else self.kbuf.shape[-2]
        if need <= cap:
            return
        grown = max(need, int(cap * 1.25), cap + 2048)
        kb = like.new_empty((*like.shape[:-2], grown, like.shape[-1]))
        vb = torch.empty_like(kb)
        if self.n:
            kb[..., :self.n, :] = self.kbuf[..., :self.n, :]
            vb[..., :self.n, :] = self.vbuf[..., :self.n, :]
        self.kbuf, self.vbuf = kb, vb
        self._plain_write = True

    def _view(self):
        self.keys, self.values = self.kbuf[..., :self.n, :], self.vbuf[..., :self.n, :]

    def _flush(self):
        """Write a pending appended row with plain copies (kv.py:71-72)."""
        pend = getattr(self, "_pending", None)
        if pend is not None:
            k, v = pend
            self._pending = None
            _PENDING.pop(self.kbuf.data_ptr(), None)
            self.kbuf[0, :, self.n - 1, :] = k
            self.vbuf[0, :, self.n - 1, :] = v
            self._plain_write = True

    def take_pending(self):
        """For the fused decode: (k_new, v_new, stable_rows) of the pending row, which the caller
        must write (tc_decode_attention_append). stable_rows is n-1 unless a plain copy wrote the
        buffers since the last fused decode (that copy may still be in flight), else 0."""
        k, v = self._pending
        self._pending = None
        _PENDING.pop(self.kbuf.data_ptr(), None)
        stable = 0 if self._plain_write else self.n - 1
        self._plain_write = False
        return k, v, stable

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self._flush()
        add = key_states.shape[-2]
        self._reserve(self.n + add, key_states)
        if (add == 1 and self.fuse_append and key_states.is_cuda and key_states.shape[0] == 1
                and key_states.dtype in (torch.bfloat16, torch.float16)):
            self._pending = (key_states[0, :, 0, :], value_states[0, :, 0, :])
            _PENDING[self.kbuf.data_ptr()] = self
        else:
            self.kbuf[..., self.n:self.n + add, :] = key_states
            self.vbuf[..., self.n:self.n + add, :] = value_states
            self._plain_write = True
        self.n += add
        self._view()
        return self.keys, self.values

    def crop(self, max_length):
        self._flush()
        self.n = min(self.n, max_length)
        self._view()

    def splice(self, s: Split, inv_freq):
        """In-place A.B.C -> A.C: only C is touched, O(|C|) bytes, one kernel launch."""
        self._flush()
        if s.c and s.gap:
            _splice_growing([self], s, inv_freq)
            self._plain_write = True
        self.n = s.a + s.c
        self._view()


def pending_append(key):
    """The GrowingLayer whose keys view `key` ([1, hkv, n, d]) has its last row pending, or None."""
    if not _PENDING or not key.is_cuda:
        return None
    layer = _PENDING.get(key.data_ptr())
    if layer is None or layer._pending is None or key.shape[-2] != layer.n or key.dim() != 4:
        return None
    return layer


def flush_pending(key):
    """Write the pending row behind `key`, if any (for readers other than the fused decode)."""
    layer = pending_append(key)
    if layer is not None:
        layer._flush()


_PAGED_PENDING = {}  # data_ptr of a step's key_states -> the PagedLayer whose row is pending


class _PagedState:
    """The PagedKV shared by the PagedLayers of one cache, created at the first update (when the
    head count, head size, dtype and device are known)."""

    def __init__(self, layers, max_tokens, page_rows, fuse):
        self.kv = None
        self.layers, self.max_tokens, self.page_rows, self.fuse = layers, max_tokens, page_rows, fuse
        self.members = []

    def ensure(self, key_states):
        if self.kv is None:
            from .paged import PagedKV
            _, hkv, _, d = key_states.shape
            pages = -(-self.max_tokens // self.page_rows)
            self.kv = PagedKV(self.layers, hkv, d, max_tokens=self.max_tokens, page_rows=self.page_rows,
                              dtype=key_states.dtype, device=key_states.device, spare_pages=max(64, pages // 4))
            self.fuse = (self.fuse and key_states.is_cuda and key_states.dtype in (torch.bfloat16, torch.float16)
                         and d in (64, 128, 256))

    def flush_all(self):
        for ly in self.members:
            ly._flush()


class PagedLayer(DynamicLayer):
    """Cache layer over a paged K/V store (threadcut_b200.paged.PagedKV, the layout threadcut's
    README.md:141-144 names as the next step); all layers of a cache share one PagedKV. Appends go
    into page slots (layer 0 reserves them for every layer of the step), a splice drops B's pages
    and re-rotates C's keys in place (kv.splice), and a one-token step with the threadcut attention
    leaves the new row pending: the plugin's decode branch writes it in the launch that attends over
    the pages. Prefill chunks (and any other reader) get a contiguous copy of the layer's K/V."""

    def __init__(self, state, index):
        super().__init__()
        self.state, self.index = state, index
        self._pending = None   # (k [hkv, d], v [hkv, d]) of a one-token step, not yet in the pages
        self._standin = None   # data_ptr of the key stand-in update() returned this step
        state.members.append(self)

    def lazy_initialization(self, key_states, value_states, *args, **kwargs):
        super().lazy_initialization(key_states, value_states)
        self.state.ensure(key_states)
        # `keys`/`values` carry the layout only ([1, hkv, 1, d] of the cache's dtype and device, not
        # its rows), for callers that size the cache from them (threadcut/engine.py:99-100); the
        # rows live in the pages (materialize() gives a contiguous copy)
        kv = self.state.kv
        self.keys = torch.zeros((1, kv.hkv, 1, kv.d), dtype=kv.dtype, device=kv.device)
        self.values = self.keys

    def get_seq_length(self):
        return self.state.kv.n if self.state.kv is not None else 0

    def _release(self):
        if self._standin is not None:
            _PAGED_PENDING.pop(self._standin, None)
            self._standin = None

    def _flush(self):
        pend = self._pending
        self._release()
        if pend is not None:
            self._pending = None
            self.state.kv.write(self.index, pend[0][:, None], pend[1][:, None])

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if key_states.shape[0] != 1:
            raise ValueError("PagedLayer: one sequence per cache (batch 1)")
        kv = self.state.kv
        t = key_states.shape[-2]
        if self.index == 0:
            self.state.flush_all()
            try:
                kv.reserve(t)
            except MemoryError:
                kv.compact()
                kv.reserve(t)
        if self.state.fuse:
            # stand-ins: the plugin's decode and prefill branches read the pages themselves
            if t == 1:
                self._pending = (key_states[0, :, 0, :], value_states[0, :, 0, :])
            else:
                kv.write(self.index, key_states[0], value_states[0])
            self._standin = key_states.data_ptr()
            _PAGED_PENDING[self._standin] = self
            return key_states, value_states
        kv.write(self.index, key_states[0], value_states[0])
        k, v = kv.gather(self.index)
        return k[None], v[None]

    def decode(self, q, scale):
        """The step's attention for the threadcut plugin: q [hkv, g, d] over the pages with the
        pending row written by the same launch."""
        k, v = self._pending
        self._pending = None
        self._release()
        kv = self.state.kv
        return kv.decode(self.index, q, scale, k_new=k, v_new=v, stable_tiles=kv.n_tiles - 1)

    def can_prefill(self, query):
        return (self._pending is None and query.shape[0] == 1 and query.shape[-1] == 128
                and query.shape[1] == 4 * self.state.kv.hkv and query.dtype == self.state.kv.dtype
                and query.dtype in (torch.bfloat16, torch.float16))

    def prefill(self, query, scale):
        """The chunk's causal attention for the threadcut plugin, straight over the pages."""
        self._release()
        return self.state.kv.prefill(self.index, query, scale)

    def materialize(self):
        """Writes the pending row and returns contiguous (K, V) [1, hkv, n, d] (other readers)."""
        self._flush()
        k, v = self.state.kv.gather(self.index)
        return k[None], v[None]

    def crop(self, max_length):
        self.state.flush_all()
        n = self.get_seq_length()
        if max_length < 0:
            max_length = n - abs(max_length)
        if self.state.kv is not None and n > max_length:
            self.state.kv.truncate(max_length)


def paged_pending(key):
    """The PagedLayer that returned `key` as this step's stand-in from update(), or None."""
    if not _PAGED_PENDING or not key.is_cuda:
        return None
    layer = _PAGED_PENDING.get(key.data_ptr())
    if layer is None or layer._standin != key.data_ptr():
        return None
    return layer


# Layout of the caches new_cache(config) builds when the caller does not say: the reference's
# engine calls new_cache(self.model.config) (threadcut/engine.py:53), so a process that wants the
# paged layout under that unchanged caller selects it here (use_paged_cache) instead.
_LAYOUT = {"paged": False, "max_tokens": 32768, "page_rows": 64}


def use_paged_cache(enabled=True, max_tokens=32768, page_rows=64):
    """Make new_cache(config) build paged caches (PagedLayers over one PagedKV of max_tokens rows in
    page_rows-row pages) from now on, or contiguous GrowingLayer caches again (enabled=False)."""
    if max_tokens < 1 or page_rows < 1:
        raise ValueError("use_paged_cache: max_tokens and page_rows must be positive")
    _LAYOUT.update(paged=bool(enabled), max_tokens=int(max_tokens), page_rows=int(page_rows))


def new_cache(config, paged=None, max_tokens=None, page_rows=None):
    """A DynamicCache of GrowingLayers (the reference's layout, threadcut/kv.py:44-98) or, with
    paged=True, of PagedLayers over one PagedKV sized for max_tokens (plus spare pages for the
    partly used pages splices leave; a full pool is re-packed by PagedKV.compact). Arguments left
    None take the process-wide choice of use_paged_cache (default: contiguous, 32768, 64)."""
    paged = _LAYOUT["paged"] if paged is None else paged
    max_tokens = _LAYOUT["max_tokens"] if max_tokens is None else max_tokens
    page_rows = _LAYOUT["page_rows"] if page_rows is None else page_rows
    cache = DynamicCache(config=config)
    fused = getattr(config, "_attn_implementation", None) == FUSED_ATTENTION
    if paged:
        state = _PagedState(len(cache.layers), int(max_tokens), int(page_rows), fused)
        cache.layers = [PagedLayer(state, i) for i in range(len(cache.layers))]
        return cache
    cache.layers = [GrowingLayer() for _ in cache.layers]
    if fused:
        for layer in cache.layers:
            layer.fuse_append = True  # the decode branch of threadcut_b200.attention writes the row
    return cache


def cache_bytes(cache):
    """Bytes of the live K and V of every layer (paged or contiguous)."""
    layers = cache.layers
    if layers and isinstance(layers[0], PagedLayer):
        kv = layers[0].state.kv
        return 0 if kv is None else 2 * kv.n * kv.hkv * kv.d * kv.k[0].element_size() * kv.layers
    n = cache.get_seq_length()
    layer = layers[0]
    return 2 * n * layer.keys[0, :, 0].numel() * layer.keys.element_size() * len(layers)
