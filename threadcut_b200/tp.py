"""Tensor-parallel one-token decode of a Qwen3 model across GPUs (config 5 on N GPUs).

threadcut runs the whole model on one GPU through transformers (threadcut/engine.py:21-104, the
per-token call at engine.py:66-73); splitting the model over GPUs is new here. Rank r of `world`
holds, for every layer:

* KV heads head_shard(hkv, r, world) of the cache, the matching rows of k_proj / v_proj, the g
  query heads of each of them (q_proj rows) and the matching o_proj columns. Attention of a head
  needs nothing from other heads, so it runs locally (the fused append + decode kernel,
  decode_attention_append, over the rank's GrowingLayer);
* 1/world of the MLP's intermediate dimension (gate/up rows, down_proj columns);
* 1/world of the vocabulary (lm_head rows); norms and the embedding are replicated.

A layer ends in two sums over ranks of [hidden] partials (after o_proj and after down_proj). On
more than one rank they run through peer memory (threadcut_b200.peer.AllReduce): the row-split
projection writes its fp32 rows into every rank's region over NVLink, and the residual add + RMSNorm
kernel that follows sums them in rank order, so every rank holds the same bits; with
peer_sums=False, torch.distributed.all_reduce (NCCL) between the projection and the norm. The next token is the first index of the largest logit over
all ranks' vocabulary slices (torch's argmax rule), found from an all-gather of each rank's
(best logit, index). The arithmetic is HF's Qwen3 (modeling_qwen3: RMSNorm in fp32 cast back to
the weights' dtype, q/k RMSNorm per head, RoPE with cos/sin rounded to the model dtype, SwiGLU),
so at world == 1 the step is the HF forward with threadcut_b200's attention.

The small ops between the projections are fused into their neighbours: the residual add with the
next RMSNorm (csrc/layer_ops.cuh, or the sum over ranks on more than one rank), q/k norm + RoPE
with the attention launch, and SwiGLU with the input staging of down_proj; the q/k/v and the
gate/up projections are one GEMV each (their rows side by side). That is 7 launches per layer
instead of HF's ~50 kernels, and the whole step can be captured in a CUDA graph (`capture`): it
reads nothing back to the host.

The cache is the rank's heads only, kept as GrowingLayers: a splice (kv.splice) re-rotates and
moves only the local heads, with no exchange. There is no CPU path: the kernels need CUDA.
"""
import torch
import torch.distributed as dist

from . import kv as _kv
from ._lib import check, dtype_code, lib, require_cuda, stream_ptr
from .flash_decode import decode_attention_append, decode_attention_append_rope
from .sharded import head_shard

__all__ = ["TPDecoder", "accelerate"]


def _add_rmsnorm(h, delta, w, out, eps):
    """h [rows, H] += delta (None: no add), out = Qwen3RMSNorm(h) with weight w [H]; one launch
    (tc_add_rmsnorm). All contiguous, one dtype, on one GPU."""
    require_cuda(h, w, out, *(() if delta is None else (delta,)), what="add_rmsnorm")
    st = lib().tc_add_rmsnorm(h.data_ptr(), None if delta is None else delta.data_ptr(), w.data_ptr(),
                              out.data_ptr(), h.shape[0], h.shape[1], float(eps), dtype_code(h, "add_rmsnorm"),
                              stream_ptr(h.device))
    check("tc_add_rmsnorm", st)


def _qk_norm_rope(q, k, wq, wk, cos, sin, eps):
    """In place: q [hq, d], k [hk, d] := RoPE(RMSNorm per head) (q_norm/k_norm weights wq, wk [d],
    cos/sin [d] of the model dtype); one launch (tc_qk_norm_rope)."""
    require_cuda(q, k, wq, wk, cos, sin, what="qk_norm_rope")
    st = lib().tc_qk_norm_rope(q.data_ptr(), k.data_ptr(), wq.data_ptr(), wk.data_ptr(), cos.data_ptr(),
                               sin.data_ptr(), q.shape[0], k.shape[0], q.shape[1], float(eps),
                               dtype_code(q, "qk_norm_rope"), stream_ptr(q.device))
    check("tc_qk_norm_rope", st)


def _silu_mul(gu, out):
    """out [rows, I] = silu(gu[:, :I]) * gu[:, I:] (gate and up side by side); one launch."""
    require_cuda(gu, out, what="silu_mul")
    st = lib().tc_silu_mul(gu.data_ptr(), out.data_ptr(), gu.shape[0], out.shape[1], dtype_code(gu, "silu_mul"),
                           stream_ptr(gu.device))
    check("tc_silu_mul", st)


def _gemv(x, w):
    """x [1, K] @ w[N, K]^T -> [1, N] for the one-token projections: tc_gemv (HBM-bound, fp32
    accumulation) for contiguous 16-bit operands with K a multiple of 8 and 16-byte aligned; other
    operands take the GPU library matmul. CPU tensors raise."""
    require_cuda(x, w, what="gemv")
    n, k = w.shape
    if (x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype and x.is_contiguous() and w.is_contiguous()
            and k % 8 == 0 and k <= 24576 and x.numel() == k and (x.data_ptr() | w.data_ptr()) % 16 == 0):
        out = x.new_empty((1, n))
        check("tc_gemv", lib().tc_gemv(x.data_ptr(), w.data_ptr(), out.data_ptr(), n, k, dtype_code(x, "gemv"),
                                       stream_ptr(x.device)))
        return out
    return x @ w.t()


def _gemv_swiglu(gu, w):
    """silu(gate) * up from gu [1, 2I] (gate | up) times w[N, I]^T -> [1, N]: the SwiGLU activation
    computed while the GEMV stages its input (tc_gemv_swiglu, one launch)."""
    require_cuda(gu, w, what="gemv_swiglu")
    n, k = w.shape
    if not (gu.dtype == w.dtype and gu.dtype in (torch.bfloat16, torch.float16) and gu.is_contiguous()
            and w.is_contiguous() and k % 8 == 0 and k <= 24576 and gu.numel() == 2 * k
            and (gu.data_ptr() | w.data_ptr()) % 16 == 0):
        act = gu.new_empty((1, k))
        _silu_mul(gu, act)
        return _gemv(act, w)
    out = gu.new_empty((1, n))
    check("tc_gemv_swiglu", lib().tc_gemv_swiglu(gu.data_ptr(), w.data_ptr(), out.data_ptr(), n, k,
                                                 dtype_code(gu, "gemv_swiglu"), stream_ptr(gu.device)))
    return out


def _attend(layer, q, k, v, scale):
    """The rank's attention for one step: q [hr, g, d] over the layer's cache plus the step's row
    k, v [hr, d], which the same launch appends (GrowingLayer fused append, decode_attention_append)."""
    hr, d = k.shape
    layer.update(k.view(1, hr, 1, d), v.view(1, hr, 1, d))
    kp, vp, stable = layer.take_pending()
    return decode_attention_append(q, layer.keys[0], layer.values[0], kp, vp, scale, stable_rows=stable)


def _attend_rope(layer, q, k, v, wq, wk, cos, sin, eps, scale):
    """_attend with the step's q/k norm and RoPE in the same launch: q [hr, g, d] and k [hr, d] are
    the raw projections (decode_attention_append_rope); the cache receives the rotated k."""
    hr, d = k.shape
    layer.update(k.view(1, hr, 1, d), v.view(1, hr, 1, d))
    kp, vp, stable = layer.take_pending()
    return decode_attention_append_rope(q, layer.keys[0], layer.values[0], kp, vp, wq, wk, cos, sin, eps, scale,
                                        stable_rows=stable)


class _Shard:
    """One layer's weights on this rank."""

    def __init__(self, layer, h0, h1, g, d, i0, i1, dev, interleave_gu=False):
        at, mlp = layer.self_attn, layer.mlp

        def rows(w, lo, hi):
            return w.detach()[lo:hi].to(dev).contiguous()

        def cols(w, lo, hi):
            return w.detach()[:, lo:hi].to(dev).contiguous()

        # q, k and v rows of this rank side by side: one projection per step
        self.wqkv = torch.cat((rows(at.q_proj.weight, h0 * g * d, h1 * g * d), rows(at.k_proj.weight, h0 * d, h1 * d),
                               rows(at.v_proj.weight, h0 * d, h1 * d)))
        self.wo = cols(at.o_proj.weight, h0 * g * d, h1 * g * d)
        self.q_norm = at.q_norm.weight.detach().to(dev)
        self.k_norm = at.k_norm.weight.detach().to(dev)
        self.in_norm = layer.input_layernorm.weight.detach().to(dev)
        self.post_norm = layer.post_attention_layernorm.weight.detach().to(dev)
        gate, up = rows(mlp.gate_proj.weight, i0, i1), rows(mlp.up_proj.weight, i0, i1)
        # gate | up, or interleaved (row 2i gate_i, row 2i + 1 up_i) for the projection whose
        # epilogue computes the SwiGLU activation (tc_gemv_rmsnorm_swiglu)
        self.gu_interleaved = interleave_gu
        self.wgu = (torch.stack((gate, up), dim=1).reshape(2 * gate.shape[0], gate.shape[1]).contiguous()
                    if interleave_gu else torch.cat((gate, up)))
        del gate, up
        self.wd = cols(mlp.down_proj.weight, i0, i1)
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            if getattr(at, name).bias is not None:
                raise ValueError(f"TPDecoder: {name} with a bias is not supported (Qwen3 has none)")


class TPDecoder:
    """One-token decode of a Qwen3ForCausalLM over `world` ranks of `group` (this process is rank
    dist.get_rank(group); world 1 needs no process group).

    model: the full HF model (any device; only this rank's slices are copied to `device`).
    step(token, pos) -> next token id (int64 device tensor [1]); appends the token's K/V row.
    load(layer, k, v): fill layer's cache from full-head K/V [1 or -, hkv, n, d] (own heads kept).
    splice(s, inv_freq): kv.splice on the local heads.  crop(n): drop rows past n."""

    def __init__(self, model, device, group=None, world=None, rank=None, peer_sums=True):
        cfg = model.config
        kinds = set(getattr(cfg, "layer_types", None) or ["full_attention"])
        if getattr(cfg, "use_sliding_window", False) or kinds != {"full_attention"}:
            raise ValueError("TPDecoder: sliding-window attention layers are not supported")
        rope = (getattr(cfg, "rope_parameters", None) or {}).get("rope_type", "default")
        if rope in ("dynamic", "longrope"):
            raise ValueError(f"TPDecoder: RoPE type {rope!r} changes its frequencies with the length")
        self.group = group
        self.world = world if world is not None else (dist.get_world_size(group) if dist.is_initialized() else 1)
        self.rank = rank if rank is not None else (dist.get_rank(group) if dist.is_initialized() else 0)
        self.dev = torch.device(device)
        self.hq, self.hkv, self.d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        self.g = self.hq // self.hkv
        self.h0, self.h1 = head_shard(self.hkv, self.rank, self.world)
        inter = cfg.intermediate_size
        if inter % self.world or cfg.vocab_size % self.world:
            raise ValueError("TPDecoder: intermediate size and vocabulary must split evenly over the ranks")
        i0, i1 = inter * self.rank // self.world, inter * (self.rank + 1) // self.world
        self.v0 = cfg.vocab_size * self.rank // self.world
        v1 = cfg.vocab_size * (self.rank + 1) // self.world
        self.eps = cfg.rms_norm_eps
        base = model.model
        peer_capable = self.dev.type == "cuda" and base.embed_tokens.weight.dtype in (torch.bfloat16, torch.float16)
        self.layers_w = [_Shard(layer, self.h0, self.h1, self.g, self.d, i0, i1, self.dev,
                                interleave_gu=peer_sums and peer_capable) for layer in base.layers]
        self.embed = base.embed_tokens.weight.detach().to(self.dev)
        self.final_norm = base.norm.weight.detach().to(self.dev)
        self.lm_head = model.lm_head.weight.detach()[self.v0:v1].to(self.dev).contiguous()
        self.inv_freq = base.rotary_emb.inv_freq.detach().float().to(self.dev)
        self.attn_scaling = float(getattr(base.rotary_emb, "attention_scaling", 1.0))
        self.scale = model.model.layers[0].self_attn.scaling
        self.dtype = self.embed.dtype
        self.layers = [_kv.GrowingLayer() for _ in base.layers]
        for layer in self.layers:
            layer.fuse_append = True  # the decode launch writes each step's row
        # q/k norm + RoPE inside the attention launch (the tensor-core decode kernel's shapes)
        self.fuse_rope = (self.dev.type == "cuda" and self.dtype in (torch.bfloat16, torch.float16)
                          and self.d in (64, 128, 256))
        # the two sums per layer: the residual form of the peer-memory sums (the row-split
        # projection completes the sum into h, the next projection stages RMSNorm(h) as its input;
        # at world 1 the same two kernels with no peer) unless peer_sums is False, else a separate
        # GEMV, the collective library's all-reduce and the residual add + norm kernel
        self._ar = None
        self.use_peer_sums = False
        if peer_sums and self.dev.type == "cuda" and self.dtype in (torch.bfloat16, torch.float16):
            from .peer import AllReduce
            self._ar = AllReduce(cfg.hidden_size, self.dev, group, world=self.world)
            self.use_peer_sums = True

    # ------------------------------------------------------------------ cache
    def load(self, i, k, v):
        """Layer i's cache := the rank's heads of full-head K/V [b=1, hkv, n, d] (or [hkv, n, d])."""
        k = k.reshape(-1, *k.shape[-3:])[0] if k.dim() == 4 else k
        v = v.reshape(-1, *v.shape[-3:])[0] if v.dim() == 4 else v
        layer = self.layers[i]
        if layer.is_initialized:
            layer.crop(0)
        layer.update(k[None, self.h0:self.h1].to(self.dev), v[None, self.h0:self.h1].to(self.dev))

    def load_local(self, i, k, v):
        """Layer i's cache := K/V [1, h1 - h0, n, d] that already hold only this rank's heads."""
        layer = self.layers[i]
        if layer.is_initialized:
            layer.crop(0)
        layer.update(k, v)

    def get_seq_length(self):
        return self.layers[0].n if self.layers[0].is_initialized else 0

    def crop(self, n):
        for layer in self.layers:
            layer.crop(n)

    def splice(self, s, inv_freq):
        """A.B.C -> A.C on the local heads of every layer (threadcut/kv.py:28-41, one launch)."""
        _kv.splice(self, s, inv_freq)

    # ------------------------------------------------------------------ step
    def _all_reduce(self, x):
        if self.world > 1:
            dist.all_reduce(x, group=self.group)
        return x

    def _rope(self, pos):
        ang = float(pos) * self.inv_freq
        emb = torch.cat((ang, ang))
        return (emb.cos() * self.attn_scaling).to(self.dtype), (emb.sin() * self.attn_scaling).to(self.dtype)

    def _attention(self, w, layer, qkv, cos, sin):
        """The rank's attention of one layer from its q|k|v projection row (appends the K/V row):
        q/k norm + RoPE inside the attention launch, or as a launch of its own where the decode
        kernel cannot take it. Returns [1, local query heads * d]."""
        hr, d, g = self.h1 - self.h0, self.d, self.g
        nq = hr * g
        q, k, v = qkv[:nq * d].view(nq, d), qkv[nq * d:(nq + hr) * d].view(hr, d), qkv[(nq + hr) * d:].view(hr, d)
        if self.fuse_rope:
            o = _attend_rope(layer, q.view(hr, g, d), k, v, w.q_norm, w.k_norm, cos, sin, self.eps, self.scale)
        else:
            _qk_norm_rope(q, k, w.q_norm, w.k_norm, cos, sin, self.eps)
            o = _attend(layer, q.view(hr, g, d), k, v, self.scale)
        return o.reshape(1, nq * d)

    def _logits_part(self, token, pos):
        """This rank's vocabulary slice of the next-token logits, [1, v_local] (appends the token's
        K/V row). With the residual sums (peer_sums, the default on a GPU), per layer: the q/k/v
        projection with the input norm as its staging (the first layer: after its own norm
        launch), attention, o_proj completing the sum over ranks into the residual, the gate/up
        projection with the post-attention norm as its staging, down_proj of the SwiGLU activation
        completing its sum; the final norm is the staging of lm_head: 5 launches per layer. Every
        kernel launches with programmatic dependent launch: it starts while its predecessor
        finishes (the projections pulling their weights into shared memory) and waits for it before
        reading what it wrote."""
        if not self.use_peer_sums:
            return _gemv(self._final_hidden(token, pos), self.lm_head)
        ar, eps = self._ar, self.eps
        h = self.embed[token]  # [1, hidden], a fresh tensor (advanced indexing copies)
        x = torch.empty_like(h)
        cos, sin = self._rope(pos)
        _add_rmsnorm(h, None, self.layers_w[0].in_norm, x, eps)
        for i, (w, layer) in enumerate(zip(self.layers_w, self.layers)):
            qkv = _gemv(x, w.wqkv)[0] if i == 0 else ar.gemv_norm(h, w.in_norm, w.wqkv, eps)[0]
            ar.gemv_residual(self._attention(w, layer, qkv, cos, sin), w.wo, h)
            if w.gu_interleaved:  # the SwiGLU activation from the gate/up projection's epilogue
                ar.gemv_residual(ar.gemv_norm_swiglu(h, w.post_norm, w.wgu, eps)[0], w.wd, h)
            else:
                ar.gemv_residual(ar.gemv_norm(h, w.post_norm, w.wgu, eps), w.wd, h, swiglu=True)
        return ar.gemv_norm(h, self.final_norm, self.lm_head, eps)

    def _final_hidden(self, token, pos):
        """The step's arithmetic up to the final norm without the residual sums: [1, hidden]
        (appends the token's K/V row). Per layer: the q/k/v projection, attention, o_proj, sum over
        ranks (the collective library), residual add + post-attention norm (one launch), the gate/up
        projection, down_proj of the SwiGLU activation (computed by the projection's input staging),
        sum over ranks, and the residual add fused with the next layer's input norm (the final norm
        after the last layer)."""
        eps = self.eps
        h = self.embed[token]  # [1, hidden], a fresh tensor (advanced indexing copies)
        x = torch.empty_like(h)
        cos, sin = self._rope(pos)
        _add_rmsnorm(h, None, self.layers_w[0].in_norm, x, eps)
        nxt = [w.in_norm for w in self.layers_w[1:]] + [self.final_norm]
        for w, layer, norm_next in zip(self.layers_w, self.layers, nxt):
            o = self._attention(w, layer, _gemv(x, w.wqkv)[0], cos, sin)
            self._sum_add_norm(o, w.wo, h, w.post_norm, x)
            gu = _gemv(x, w.wgu)
            if w.gu_interleaved:  # [gate_0, up_0, gate_1, ...] -> [gate | up]
                gu = gu.view(-1, 2).t().reshape(1, -1)
            self._sum_add_norm(gu, w.wd, h, norm_next, x, swiglu=True)
        return x

    def _sum_add_norm(self, a, w, h, norm, x, swiglu=False):
        """h += sum over ranks of a @ w^T (w: this rank's columns of a row-split projection), then
        x = RMSNorm(h) * norm, with a collective all-reduce between tc_gemv and tc_add_rmsnorm.
        swiglu: a is gate|up and the projection's input is its SwiGLU activation, computed by the
        GEMV as it stages its input."""
        part = _gemv_swiglu(a, w) if swiglu else _gemv(a, w)
        _add_rmsnorm(h, self._all_reduce(part), norm, x, self.eps)

    def close(self):
        """Releases the peer-memory region of the sums (collective: every rank calls it, after the
        device finished every step that uses it)."""
        if self._ar is not None:
            if self.world > 1:
                dist.barrier(group=self.group)
            self._ar.close()
            self._ar = None
            self.use_peer_sums = False

    def step(self, token, pos):
        """Decode `token` (int64 device tensor [1]) at position `pos` (the cache length before the
        step); returns the greedy next token (int64 device tensor [1])."""
        logits = self._logits_part(token, pos)[0]  # this rank's vocabulary slice
        idx = logits.argmax()  # first index of the slice's maximum
        if self.world == 1:
            return idx.view(1)
        # no indexing by a 0-dim device tensor below: torch reads such an index back to the host,
        # which a CUDA graph capture cannot hold
        pair = torch.stack((logits.max().float(), (idx + self.v0).float()))  # ids < 2^24: exact in fp32
        pairs = pair.new_empty(self.world * 2)
        dist.all_gather_into_tensor(pairs, pair, group=self.group)
        pairs = pairs.view(self.world, 2)  # rank order: ranks hold increasing vocabulary slices
        first = (pairs[:, 0] == pairs[:, 0].max()).int().argmax()  # first rank holding the maximum
        return pairs[:, 1].index_select(0, first.view(1)).long()

    def capture(self, token, pos):
        """A CUDA graph of step(token, pos) (the all-reduces inside it) and its output tensor; the
        cache is cropped back to `pos` rows, so each replay decodes the same step. The capture is
        thread-local: the process group's watchdog thread polls events meanwhile, which a global
        capture would count as an illegal call. Every rank must capture at the same point.

        Before capturing, every layer's buffer gets room for row `pos` (a buffer that is exactly
        full would otherwise grow inside the capture: the new buffer would come from the graph's
        private pool and the copy of the old rows would only be recorded, leaving the replayed cache
        uninitialised and reading the freed old buffer), and one eager step runs on the capture
        stream, so that the decode workspace of that stream is allocated and zeroed outside the
        graph."""
        for layer in self.layers:
            if layer.is_initialized and layer.kbuf is not None:
                layer._flush()
                layer._reserve(pos + 1, layer.kbuf)
        torch.cuda.synchronize(self.dev)
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        try:
            with torch.cuda.stream(s):
                self.step(token, pos)  # eager warm-up on the capture stream
                self.crop(pos)
            torch.cuda.synchronize(self.dev)
            with torch.cuda.graph(graph, stream=s, capture_error_mode="thread_local"):
                out = self.step(token, pos)
        finally:
            self.crop(pos)
            torch.cuda.current_stream(self.dev).wait_stream(s)
            torch.cuda.synchronize(self.dev)
        return graph, out

    def step_logits(self, token, pos):
        """The next-token logits in the model dtype, [1, vocab] (as the HF model's lm_head returns
        them), of `token` at `pos`; appends the token's row like step."""
        part = self._logits_part(token, pos)
        if self.world == 1:
            return part
        parts = [torch.empty_like(part) for _ in range(self.world)]
        dist.all_gather(parts, part, group=self.group)
        return torch.cat(parts, dim=1)

    def logits(self, token, pos):
        """The full next-token logits (fp32 [vocab]) of `token` at `pos`, for checks: the step's
        arithmetic with the vocabulary slices all-gathered. Appends the token's row like step."""
        part = self._logits_part(token, pos)[0].float()
        if self.world == 1:
            return part
        parts = [torch.empty_like(part) for _ in range(self.world)]
        dist.all_gather(parts, part, group=self.group)
        return torch.cat(parts)


def _fusable(cache, dec):
    """True when `cache` is this package's contiguous cache of the model `dec` decodes: every layer a
    GrowingLayer holding rows, with the fused append on, in the model's dtype, on its device, with
    the local head count."""
    layers = getattr(cache, "layers", None)
    if not layers or len(layers) != len(dec.layers_w):
        return False
    for ly in layers:
        if not (isinstance(ly, _kv.GrowingLayer) and ly.fuse_append and ly.is_initialized
                and getattr(ly, "kbuf", None) is not None and ly.n > 0):
            return False
        kb = ly.kbuf
        if kb.dtype != dec.dtype or kb.device != dec.dev or kb.shape[0] != 1 or kb.shape[1] != dec.h1 - dec.h0:
            return False
    return True


def accelerate(model, device=None):
    """Route the one-token decode steps of a one-GPU Qwen3 model through the fused step of this
    module, behind the model's own call: after accelerate(model), model(input_ids=[[t]],
    past_key_values=cache, use_cache=True) over a cache of this package (kv.new_cache with the
    threadcut attention: GrowingLayers with the fused append, holding rows) returns HF's output type
    with `.logits` [1, 1, vocab] computed by TPDecoder at world 1 (7 launches per layer instead
    of transformers' ~50), appending the token's K/V row to the same cache. Every other call (a
    prefill chunk, another cache, extra arguments) goes to the model's own forward. The reference's
    engine (threadcut/engine.py:66-73, 88-95) makes exactly such calls, so it runs unchanged on the
    fused step. Returns the TPDecoder doing the work (it shares the model's weights where no copy is
    needed: the q|k|v and gate|up rows are concatenated copies). bf16/fp16 models only."""
    from transformers.modeling_outputs import CausalLMOutputWithPast
    dev = torch.device(device) if device is not None else next(model.parameters()).device
    dec = TPDecoder(model, dev, world=1, rank=0)
    if dec.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("accelerate: the fused step needs a bf16 or fp16 model")
    inner = model.forward

    def forward(*args, **kwargs):
        ids = kwargs.get("input_ids")
        cache = kwargs.get("past_key_values")
        extra = set(kwargs) - {"input_ids", "past_key_values", "use_cache", "logits_to_keep"}
        if (not args and not extra and ids is not None and ids.dim() == 2 and tuple(ids.shape) == (1, 1)
                and kwargs.get("use_cache", True) is not False and _fusable(cache, dec)):
            pos = cache.get_seq_length()
            dec.layers = cache.layers
            logits = dec.step_logits(ids.view(1), pos)
            return CausalLMOutputWithPast(logits=logits.view(1, 1, -1), past_key_values=cache)
        return inner(*args, **kwargs)

    model.forward = forward
    model._threadcut_fused_step = (dec, inner)
    return dec


def restore(model):
    """Undo accelerate(model)."""
    saved = getattr(model, "_threadcut_fused_step", None)
    if saved is not None:
        model.forward = saved[1]
        del model._threadcut_fused_step
        saved[0].close()
