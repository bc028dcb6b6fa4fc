"""Host logic of the tensor-parallel decoder on CPU: weight slicing, the two sums per layer, the
vocabulary-sliced argmax, and the local-head cache, on one rank and on two `gloo` ranks.

The kernels need a GPU, so these tests replace the launches of the step (`tp._attend`: append +
attention; `_add_rmsnorm`, `_qk_norm_rope`, `_silu_mul`, `_gemv`, `_gemv_swiglu`) with torch restatements of HF's Qwen3
arithmetic on CPU; everything else is the product code. The expected logits
are the HF model's own fp32 forward over the whole prompt (modeling_qwen3 with eager attention).
The step also must not read any tensor value back to the host, so that it can be captured in a
CUDA graph on the GPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch.utils._python_dispatch import TorchDispatchMode
from transformers import AutoModelForCausalLM, Qwen3Config

from threadcut_b200 import tp


def _cpu_add_rmsnorm(h, delta, w, out, eps):
    if delta is not None:
        h += delta
    hf = h.float()
    out.copy_(w * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)).to(h.dtype))


def _cpu_qk_norm_rope(q, k, wq, wk, cos, sin, eps):
    for x, w in ((q, wq), (k, wk)):
        xf = x.float()
        y = w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
        h = y.shape[-1] // 2
        x.copy_(y * cos + torch.cat((-y[..., h:], y[..., :h]), -1) * sin)


def _cpu_silu_mul(gu, out):
    i = out.shape[1]
    out.copy_(torch.nn.functional.silu(gu[:, :i]) * gu[:, i:])


def _cpu_ops(target):
    """Put the CPU stand-ins in place of the GPU launches (attribute setter: monkeypatch or setattr)."""
    target(tp, "_attend", _cpu_attend)
    target(tp, "_add_rmsnorm", _cpu_add_rmsnorm)
    target(tp, "_qk_norm_rope", _cpu_qk_norm_rope)
    target(tp, "_silu_mul", _cpu_silu_mul)
    target(tp, "_gemv", lambda x, w: x @ w.t())
    target(tp, "_gemv_swiglu", _cpu_gemv_swiglu)


def _cpu_gemv_swiglu(gu, w):
    i = w.shape[1]
    return (torch.nn.functional.silu(gu[:, :i]) * gu[:, i:]) @ w.t()


def _cpu_attend(layer, q, k, v, scale):
    hr, d = k.shape
    layer.update(k.view(1, hr, 1, d), v.view(1, hr, 1, d))  # a CPU cache writes the row at once
    kk, vv = layer.keys[0].float(), layer.values[0].float()
    p = (torch.einsum("hgd,hnd->hgn", q.float(), kk) * scale).softmax(-1)
    return torch.einsum("hgn,hnd->hgd", p, vv).to(q.dtype)


class _NoHostRead(TorchDispatchMode):
    """Fails on any op that reads a tensor value back to the host (.item(), int(t), indexing by a
    0-dim tensor): a CUDA graph capture of the step could not hold it."""

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        if func is torch.ops.aten._local_scalar_dense.default:
            raise AssertionError("the decode step reads a tensor value back to the host")
        return func(*args, **(kwargs or {}))


def _model():
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=4096)
    return AutoModelForCausalLM.from_config(cfg, dtype=torch.float32, attn_implementation="eager").eval()


def _run(rank, world, n_ctx=20, interleave=False):
    model = _model()
    ids = torch.randint(0, 512, (1, n_ctx + 1), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model(input_ids=ids).logits[0, -1]  # logits after the last token, full context
        out = model(input_ids=ids[:, :n_ctx], use_cache=True)
        dec = tp.TPDecoder(model, "cpu", world=world, rank=rank, group=None)
        if interleave:  # the GPU layout of gate|up (row 2i gate_i, row 2i + 1 up_i)
            for w in dec.layers_w:
                gate, up = w.wgu.chunk(2)
                w.wgu = torch.stack((gate, up), dim=1).reshape(-1, gate.shape[1]).contiguous()
                w.gu_interleaved = True
        for i, layer in enumerate(out.past_key_values.layers):
            dec.load(i, layer.keys, layer.values)
        assert dec.get_seq_length() == n_ctx
        logits = dec.logits(ids[0, n_ctx:], n_ctx)
        assert dec.get_seq_length() == n_ctx + 1
        dec.crop(n_ctx)
        with _NoHostRead():
            tok = dec.step(ids[0, n_ctx:], n_ctx)
    return ref, logits, tok


def test_one_rank_equals_the_hf_forward(monkeypatch):
    _cpu_ops(monkeypatch.setattr)
    ref, logits, tok = _run(0, 1)
    torch.testing.assert_close(logits, ref, atol=1e-4, rtol=0)
    assert int(tok) == int(ref.argmax())


def test_interleaved_gate_up_rows_on_the_separate_sums_path(monkeypatch):
    """With the gate/up rows interleaved (as the GPU decoder stores them for the SwiGLU epilogue),
    the separate-sums step de-interleaves the projection's output and still equals the HF forward."""
    _cpu_ops(monkeypatch.setattr)
    ref, logits, tok = _run(0, 1, interleave=True)
    torch.testing.assert_close(logits, ref, atol=1e-4, rtol=0)
    assert int(tok) == int(ref.argmax())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, interleave=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _cpu_ops(setattr)
        ref, logits, tok = _run(rank, world, interleave=interleave)
        err = float((logits - ref).abs().max())
        q.put((rank, err, int(tok), int(ref.argmax())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,interleave", [(2, False), (2, True)])
def test_two_gloo_ranks_equal_the_hf_forward(world, interleave):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, interleave)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, err, tok, ref_tok in res:
        assert err < 1e-4, (rank, err)
        assert tok == ref_tok


def test_uneven_splits_are_rejected():
    model = _model()
    with pytest.raises(ValueError):
        tp.TPDecoder(model, "cpu", world=3, rank=0)  # 2 KV heads over 3 ranks


def test_unsupported_attention_kinds_are_rejected():
    model = _model()
    model.config.use_sliding_window = True
    with pytest.raises(ValueError):
        tp.TPDecoder(model, "cpu", world=1, rank=0)
    model.config.use_sliding_window = False
    model.config.rope_parameters = {"rope_type": "dynamic", "rope_theta": 1e6, "factor": 2.0}
    with pytest.raises(ValueError):
        tp.TPDecoder(model, "cpu", world=1, rank=0)
