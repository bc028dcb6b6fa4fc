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

A layer ends in two sums over ranks of [hidden] partials (after o_proj and after down_proj:
torch.distributed.all_reduce, NCCL). The next token is the first index of the largest logit over
all ranks' vocabulary slices (torch's argmax rule), found from an all-gather of each rank's
(best logit, index). The arithmetic is HF's Qwen3 (modeling_qwen3: RMSNorm in fp32 cast back to
the weights' dtype, q/k RMSNorm per head, RoPE with cos/sin rounded to the model dtype, SwiGLU),
so at world == 1 the step is the HF forward with threadcut_b200's attention.

The cache is the rank's heads only, kept as GrowingLayers: a splice (kv.splice) re-rotates and
moves only the local heads, with no exchange. There is no CPU path: the attention kernel needs CUDA.
"""
import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import kv as _kv
from .flash_decode import decode_attention_append
from .sharded import head_shard

__all__ = ["TPDecoder"]


def _rms(x, w, eps):
    """Qwen3RMSNorm.forward: fp32 mean of squares, rsqrt, cast back, times the weight."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _attend(layer, q, k, v, scale):
    """The rank's attention for one step: q [hr, g, d] over the layer's cache plus the step's row
    k, v [hr, d], which the same launch appends (GrowingLayer fused append, decode_attention_append)."""
    hr, d = k.shape
    layer.update(k.view(1, hr, 1, d), v.view(1, hr, 1, d))
    kp, vp, stable = layer.take_pending()
    return decode_attention_append(q, layer.keys[0], layer.values[0], kp, vp, scale, stable_rows=stable)


class _Shard:
    """One layer's weights on this rank."""

    def __init__(self, layer, h0, h1, g, d, i0, i1, dev):
        at, mlp = layer.self_attn, layer.mlp

        def rows(w, lo, hi):
            return w.detach()[lo:hi].to(dev).contiguous()

        def cols(w, lo, hi):
            return w.detach()[:, lo:hi].to(dev).contiguous()

        self.wq = rows(at.q_proj.weight, h0 * g * d, h1 * g * d)
        self.wk = rows(at.k_proj.weight, h0 * d, h1 * d)
        self.wv = rows(at.v_proj.weight, h0 * d, h1 * d)
        self.wo = cols(at.o_proj.weight, h0 * g * d, h1 * g * d)
        self.q_norm = at.q_norm.weight.detach().to(dev)
        self.k_norm = at.k_norm.weight.detach().to(dev)
        self.in_norm = layer.input_layernorm.weight.detach().to(dev)
        self.post_norm = layer.post_attention_layernorm.weight.detach().to(dev)
        self.wg = rows(mlp.gate_proj.weight, i0, i1)
        self.wu = rows(mlp.up_proj.weight, i0, i1)
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

    def __init__(self, model, device, group=None, world=None, rank=None):
        cfg = model.config
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
        self.layers_w = [_Shard(layer, self.h0, self.h1, self.g, self.d, i0, i1, self.dev) for layer in base.layers]
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

    def _final_hidden(self, token, pos):
        """The step's arithmetic up to the final norm: [1, hidden] (appends the token's K/V row)."""
        hr, d, g = self.h1 - self.h0, self.d, self.g
        h = self.embed[token]  # [1, hidden]
        ang = float(pos) * self.inv_freq
        emb = torch.cat((ang, ang))
        cos = (emb.cos() * self.attn_scaling).to(self.dtype)
        sin = (emb.sin() * self.attn_scaling).to(self.dtype)
        for w, layer in zip(self.layers_w, self.layers):
            x = _rms(h, w.in_norm, self.eps)
            q = _rms((x @ w.wq.t()).view(hr * g, d), w.q_norm, self.eps)
            k = _rms((x @ w.wk.t()).view(hr, d), w.k_norm, self.eps)
            v = (x @ w.wv.t()).view(hr, d)
            q = q * cos + _rotate_half(q) * sin
            k = k * cos + _rotate_half(k) * sin
            o = _attend(layer, q.view(hr, g, d), k, v, self.scale)
            h = h + self._all_reduce(o.reshape(1, hr * g * d) @ w.wo.t())
            x = _rms(h, w.post_norm, self.eps)
            h = h + self._all_reduce((F.silu(x @ w.wg.t()) * (x @ w.wu.t())) @ w.wd.t())
        return _rms(h, self.final_norm, self.eps)

    def step(self, token, pos):
        """Decode `token` (int64 device tensor [1]) at position `pos` (the cache length before the
        step); returns the greedy next token (int64 device tensor [1])."""
        logits = (self._final_hidden(token, pos) @ self.lm_head.t())[0]  # this rank's vocabulary slice
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
        capture would count as an illegal call. Every rank must capture at the same point."""
        torch.cuda.synchronize(self.dev)
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                out = self.step(token, pos)
        finally:
            self.crop(pos)
        return graph, out

    def logits(self, token, pos):
        """The full next-token logits (fp32 [vocab]) of `token` at `pos`, for checks: the step's
        arithmetic with the vocabulary slices all-gathered. Appends the token's row like step."""
        part = (self._final_hidden(token, pos) @ self.lm_head.t())[0].float()
        if self.world == 1:
            return part
        parts = [torch.empty_like(part) for _ in range(self.world)]
        dist.all_gather(parts, part, group=self.group)
        return torch.cat(parts)
