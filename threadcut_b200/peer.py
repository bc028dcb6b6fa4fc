"""Device memory shared by the ranks of a process group over NVLink (CUDA IPC), and the sums of the
tensor-parallel step that run through it.

threadcut runs one GPU (threadcut/engine.py:21-104); the tensor-parallel step of config 5
(threadcut_b200/tp.py) needs two sums over the ranks per layer. `PeerRegion` gives every rank one
region of its own memory mapped into every other rank's address space: the library allocates it
(tc_peer_alloc), the ranks exchange the IPC handles through the process group (an all-gather of the
handle bytes), and each rank maps the others' (tc_peer_open). `AllReduce` keeps one such region
per decoder and runs the fused sum: the row-split projection writes its rows into every rank's
region (tc_gemv_allreduce), and the next kernel adds them up with the residual add and RMSNorm
(tc_allreduce_add_rmsnorm); or, in the residual form the tensor-parallel step uses, each CTA of the
projection waits for the other ranks' rows of its own block and adds them into the residual itself
(tc_gemv_allreduce_residual), and the next projection stages RMSNorm of the residual as its input
(tc_gemv_rmsnorm). No collective library runs on that path; all ranks must make the same sequence
of calls.
"""
import ctypes

import torch
import torch.distributed as dist

from ._lib import check, dtype_code, lib, require_cuda, stream_ptr

__all__ = ["PeerRegion", "AllReduce", "GatherMerge"]


class PeerRegion:
    """`nbytes` of zeroed device memory on every rank of `group`, each rank's region mapped into
    every other rank's process. `ptrs[p]` is rank p's region as seen from this process. Collective:
    every rank of the group constructs it at the same point (world=1: this process's region alone,
    not collective)."""

    def __init__(self, nbytes, device, group=None, world=None):
        self.device = torch.device(device)
        if world == 1:  # a region of this process only (no exchange, whatever group exists)
            self.world, self.rank = 1, 0
        else:
            self.world = dist.get_world_size(group) if dist.is_initialized() else 1
            self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        L = lib()
        hb = L.tc_peer_handle_bytes()
        handle = (ctypes.c_uint8 * hb)()
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check("tc_peer_alloc", L.tc_peer_alloc(int(nbytes), ctypes.byref(own), handle))
        self._own = own.value
        self.ptrs = [None] * self.world
        self.ptrs[self.rank] = self._own
        if self.world > 1:
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
            every = torch.empty(self.world * hb, dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = every.cpu().numpy().reshape(self.world, hb)
            for p in range(self.world):
                if p == self.rank:
                    continue
                buf = (ctypes.c_uint8 * hb).from_buffer_copy(every[p].tobytes())
                peer = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    check("tc_peer_open", L.tc_peer_open(buf, ctypes.byref(peer)))
                self.ptrs[p] = peer.value
        self._arr = (ctypes.c_void_p * self.world)(*self.ptrs)

    def close(self):
        """Unmaps the peers' regions and frees this rank's (after the device finished using them)."""
        if self._own is None:
            return
        L = lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p, ptr in enumerate(self.ptrs):
                if p != self.rank and ptr is not None:
                    L.tc_peer_close(ctypes.c_void_p(ptr))
            L.tc_peer_free(ctypes.c_void_p(self._own))
        self._own = None
        self.ptrs = [None] * self.world


class AllReduce:
    """The sums of the tensor-parallel step over the ranks of `group` (world=1: one process, no
    group), for vectors of `hidden` elements. Two forms:
      gemv(x, w) starts one (w's rows are split over the ranks' columns: each rank holds a partial
      product), add_rmsnorm(h, weight, out, eps) finishes it: h += sum, out = RMSNorm(h) * weight;
      gemv_residual(x, w, h) does both halves of the sum in the projection (h += sum), and
      gemv_norm(h, weight, w2, eps) is the next projection of RMSNorm(h) * weight (two launches
      where the first form and the next projection take three)."""

    def __init__(self, hidden, device, group=None, world=None):
        self.hidden = int(hidden)
        if world is None:
            world = dist.get_world_size(group) if dist.is_initialized() else 1
        nbytes = lib().tc_allreduce_region_bytes(world, self.hidden)
        if nbytes == 0:
            raise ValueError(f"AllReduce: {world} ranks x {hidden} elements is outside the supported range")
        self.region = PeerRegion(nbytes, device, group, world=world)

    def gemv(self, x, w, swiglu=False):
        """Starts the sum of x @ w^T over the ranks (w [hidden, k], x [k]); swiglu: x is gate|up
        [2k] and the product is of the SwiGLU activation computed from it (tc_gemv_allreduce_swiglu)."""
        require_cuda(x, w, what="gemv_allreduce")
        n, k = w.shape
        if n != self.hidden or x.numel() != (2 * k if swiglu else k) or not (x.is_contiguous() and w.is_contiguous()):
            raise ValueError("gemv_allreduce: w must be [hidden, k] and x [k] (gate|up [2k]), both contiguous")
        r = self.region
        fn = lib().tc_gemv_allreduce_swiglu if swiglu else lib().tc_gemv_allreduce
        check("tc_gemv_allreduce", fn(x.data_ptr(), w.data_ptr(), n, k, r._arr, r.world, r.rank,
                                      dtype_code(x, "gemv_allreduce"), stream_ptr(x.device)))

    def gemv_residual(self, x, w, h, swiglu=False):
        """h [hidden] += the sum over the ranks of x @ w^T, completed inside the projection
        (tc_gemv_allreduce_residual[_swiglu]); swiglu as for gemv. Every rank ends with the same h."""
        require_cuda(x, w, h, what="gemv_allreduce_residual")
        n, k = w.shape
        if (n != self.hidden or x.numel() != (2 * k if swiglu else k) or h.numel() != n
                or not (x.is_contiguous() and w.is_contiguous() and h.is_contiguous())
                or not (x.dtype == w.dtype == h.dtype)):
            raise ValueError("gemv_allreduce_residual: w [hidden, k], x [k] (gate|up [2k]), h [hidden], contiguous, "
                             "one dtype")
        r = self.region
        fn = lib().tc_gemv_allreduce_residual_swiglu if swiglu else lib().tc_gemv_allreduce_residual
        check("tc_gemv_allreduce_residual", fn(x.data_ptr(), w.data_ptr(), n, k, r._arr, r.world, r.rank, h.data_ptr(),
                                               dtype_code(x, "gemv_allreduce_residual"), stream_ptr(x.device)))

    def gemv_norm(self, h, weight, w, eps):
        """[1, n] = (RMSNorm(h) * weight) @ w^T for w [n, hidden], right after a gemv_residual that
        left h (tc_gemv_rmsnorm: the norm is the projection's input staging, its 1/rms from the sums
        of squares that gemv_residual recorded)."""
        require_cuda(h, weight, w, what="gemv_rmsnorm")
        n, k = w.shape
        if (k != self.hidden or h.numel() != k or weight.numel() != k
                or not (h.is_contiguous() and weight.is_contiguous() and w.is_contiguous())
                or not (h.dtype == weight.dtype == w.dtype)):
            raise ValueError("gemv_rmsnorm: h and weight [hidden], w [n, hidden], contiguous, one dtype")
        out = torch.empty((1, n), dtype=h.dtype, device=h.device)
        r = self.region
        check("tc_gemv_rmsnorm", lib().tc_gemv_rmsnorm(h.data_ptr(), weight.data_ptr(), r.ptrs[r.rank], float(eps),
                                                       w.data_ptr(), out.data_ptr(), n, k, dtype_code(h, "gemv_rmsnorm"),
                                                       stream_ptr(h.device)))
        return out

    def gemv_norm_swiglu(self, h, weight, w, eps):
        """The SwiGLU activation [1, n/2] of (RMSNorm(h) * weight) @ w^T for the MLP's gate/up
        projection with interleaved rows (w [n, hidden], row 2i gate_i, row 2i + 1 up_i), right
        after a gemv_residual (tc_gemv_rmsnorm_swiglu): the projection's epilogue computes
        silu(gate) * up once per element, so the down projection takes it as a plain input."""
        require_cuda(h, weight, w, what="gemv_rmsnorm_swiglu")
        n, k = w.shape
        if (k != self.hidden or n % 2 or h.numel() != k or weight.numel() != k
                or not (h.is_contiguous() and weight.is_contiguous() and w.is_contiguous())
                or not (h.dtype == weight.dtype == w.dtype)):
            raise ValueError("gemv_rmsnorm_swiglu: h and weight [hidden], w [n, hidden] (n even), contiguous, "
                             "one dtype")
        out = torch.empty((1, n // 2), dtype=h.dtype, device=h.device)
        r = self.region
        check("tc_gemv_rmsnorm_swiglu", lib().tc_gemv_rmsnorm_swiglu(
            h.data_ptr(), weight.data_ptr(), r.ptrs[r.rank], float(eps), w.data_ptr(), out.data_ptr(), n, k,
            dtype_code(h, "gemv_rmsnorm_swiglu"), stream_ptr(h.device)))
        return out

    def add_rmsnorm(self, h, weight, out, eps):
        require_cuda(h, weight, out, what="allreduce_add_rmsnorm")
        if h.numel() != self.hidden:
            raise ValueError("allreduce_add_rmsnorm: h must hold `hidden` elements")
        r = self.region
        check("tc_allreduce_add_rmsnorm", lib().tc_allreduce_add_rmsnorm(
            h.data_ptr(), weight.data_ptr(), out.data_ptr(), self.hidden, float(eps), r.ptrs[r.rank], r.world,
            dtype_code(h, "allreduce_add_rmsnorm"), stream_ptr(h.device)))

    def close(self):
        self.region.close()


class GatherMerge:
    """The combine of a sequence-sharded decode over the ranks of `group`, through peer memory:
    __call__(o, lse, out) pushes this rank's fp32 partials o [rows, d] and LSE [rows] into every
    other rank's region and writes the log-sum-exp merge of all ranks' partials (rank order, the
    arithmetic of flash_decode.merge_partials) into out [rows, d] — one launch in place of an
    all-gather and a merge (tc_peer_gather_merge). All ranks call it in the same order."""

    def __init__(self, rows, d, device, group=None):
        self.rows, self.d = int(rows), int(d)
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        nbytes = lib().tc_gather_region_bytes(world, self.rows, self.d)
        if nbytes == 0:
            raise ValueError(f"GatherMerge: {world} ranks x {rows} x {d} is outside the supported range")
        self.region = PeerRegion(nbytes, device, group)

    def __call__(self, o, lse, out, lse_out=None):
        require_cuda(o, lse, out, what="peer_gather_merge")
        if (o.dtype != torch.float32 or lse.dtype != torch.float32 or tuple(o.shape) != (self.rows, self.d)
                or lse.numel() != self.rows or not o.is_contiguous() or not lse.is_contiguous()
                or out.shape[-1] != self.d or out.stride(-1) != 1):
            raise ValueError("peer_gather_merge: o fp32 [rows, d], lse fp32 [rows] (contiguous), out [rows, d]")
        r = self.region
        check("tc_peer_gather_merge", lib().tc_peer_gather_merge(
            o.data_ptr(), lse.data_ptr(), out.data_ptr(), None if lse_out is None else lse_out.data_ptr(), self.rows,
            self.d, out.stride(-2), r._arr, r.world, r.rank, dtype_code(out, "peer_gather_merge"), stream_ptr(o.device)))
        return out

    def close(self):
        self.region.close()
