"""End-to-end through the reference engine's calls and the transformers plugin on the GPU.

Mirrors the reference's engine tests (tests/test_core.py): T2 (splice == fresh compute), T3 (greedy
tokens == stock transformers SDPA generate) on the reference's tiny Qwen3 configuration, and
config 5: a random-init Qwen3-4B decoding one token over a 128k cache with a 32k span pruned, whose
next-token logits must have the same top-1 as the torch SDPA path on the same spliced cache. The
engine's calls (split, splice or new_cache, chunked prefill, greedy decode; threadcut/engine.py:
41-95) are made by tests/caller.py.
"""
import numpy as np
import pytest
import torch
from transformers import AutoModelForCausalLM, DynamicCache, Qwen3Config

import workloads
from caller import Session
from helpers import ref_cos_sin
from oracle.rope import shift_keys_ref
from threadcut_b200 import _lib
from threadcut_b200 import attention as tc_attention
from threadcut_b200.kv import new_cache, splice
from threadcut_b200.match import Split

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def tiny_engine(dtype):
    """The reference's tiny test model (tests/test_core.py:15-22); stop ids 510/511 stand in for a
    tokenizer's end-of-turn ids (threadcut/engine.py:36)."""
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=4096)
    model = AutoModelForCausalLM.from_config(cfg, dtype=dtype, attn_implementation=tc_attention.NAME).to(DEV)
    return Session(model, min_suffix=4, prefill_chunk=7)


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    _lib.device_errors(clear=True)
    yield
    assert _lib.device_errors(clear=True) == 0


def rand_ids(n, seed, vocab=500):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(10, vocab, (n,), generator=g).tolist()


def kv_alone(model, ids, start):
    """KV of `ids` at positions start.., computed with no other context visible."""
    cache = DynamicCache(config=model.config)
    x = torch.tensor([ids], device=model.device)
    pos = torch.arange(start, start + len(ids), device=model.device)[None]
    model(input_ids=x, position_ids=pos, past_key_values=cache, use_cache=True)
    return cache


def concat(*caches):
    out = caches[0]
    for c in caches[1:]:
        for lo, li in zip(out.layers, c.layers):
            lo.keys = torch.cat((lo.keys, li.keys), 2)
            lo.values = torch.cat((lo.values, li.values), 2)
    return out


@pytest.mark.parametrize("dtype,atol", [(torch.float32, 1e-4), (torch.bfloat16, 3e-2)])
def test_T2_splice_matches_fresh_compute(dtype, atol):
    engine = tiny_engine(dtype)
    m = engine.model
    A, B, C, D = rand_ids(9, 1), rand_ids(13, 2), rand_ids(11, 3), rand_ids(5, 4)
    with torch.no_grad():
        ref = concat(kv_alone(m, A, 0), kv_alone(m, C, len(A)))
        ref_logits = m(input_ids=torch.tensor([D], device=DEV), past_key_values=ref).logits[0, -1]
        engine.cache = concat(kv_alone(m, A, 0), kv_alone(m, B, len(A)), kv_alone(m, C, len(A) + len(B)))
        engine.ids = A + B + C
        logits, stats = engine.load(A + C + D)
    assert (stats["reused_prefix"], stats["reused_suffix"], stats["computed_tokens"]) == (9, 11, 5)
    assert torch.allclose(logits[0].float(), ref_logits.float(), atol=atol, rtol=0)


def test_growing_cache_inplace_splice_matches_copy_splice():
    """The engine's own GrowingLayer cache spliced in place (all layers, one launch) gives the same
    logits as the copy-path splice (threadcut/kv.py:34-41) of a plain DynamicCache holding the same
    A.B.C tensors."""
    engine = tiny_engine(torch.float32)
    m = engine.model
    A, B, C, D = rand_ids(20, 5), rand_ids(17, 6), rand_ids(40, 7), rand_ids(6, 8)
    with torch.no_grad():
        engine.generate(A + B + C, max_new_tokens=0)
        plain = DynamicCache(config=m.config)
        for lp, lg in zip(plain.layers, engine.cache.layers):
            lp.update(lg.keys.clone(), lg.values.clone())
        logits, stats = engine.load(A + C + D)
        splice(plain, Split(len(A), len(A) + len(B), len(C)), engine.inv_freq)
        ref_logits = engine.prefill(D, plain)
    assert (stats["reused_prefix"], stats["reused_suffix"], stats["computed_tokens"]) == (20, 40, 6)
    assert torch.allclose(logits.float(), ref_logits.float(), atol=1e-5, rtol=0)


def hf_generate(m, ids, n, stop):
    impl = m.config._attn_implementation
    m.set_attn_implementation("sdpa")
    try:
        return m.generate(torch.tensor([ids], device=m.device), max_new_tokens=n, do_sample=False,
                          eos_token_id=list(stop))[0, len(ids):].tolist()
    finally:
        m.set_attn_implementation(impl)


def test_T3_no_pruning_matches_hf_generate():
    engine = tiny_engine(torch.float32)
    m = engine.model
    p1 = rand_ids(20, 5)
    out1, _ = engine.generate(p1, max_new_tokens=12)
    ref1 = hf_generate(m, p1, 12, engine.stop_ids)
    assert out1 == [t for t in ref1 if t not in engine.stop_ids][:len(out1)]
    p2 = p1 + out1 + rand_ids(6, 6)
    out2, s2 = engine.generate(p2, max_new_tokens=12)
    assert s2["reused_tokens"] == len(p1) + len(out1) and s2["computed_tokens"] == 6
    ref2 = hf_generate(m, p2, 12, engine.stop_ids)
    assert out2 == [t for t in ref2 if t not in engine.stop_ids][:len(out2)]


def test_cfg5_full_model_128k_spliced_top1_matches_sdpa():
    torch.manual_seed(0)
    cfg = workloads.qwen3_4b_config()
    with torch.device(DEV):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation=tc_attention.NAME)
    model.eval()
    inv = model.model.rotary_emb.inv_freq
    ctx = workloads.CFG5_CTX
    lo, hi = workloads.CFG5_PRUNE
    s = Split(lo, hi, ctx - hi)
    cache = new_cache(cfg)
    gen = torch.Generator(device=DEV).manual_seed(0)
    for layer in cache.layers:
        k = torch.randn(1, 8, ctx, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
        v = torch.randn(1, 8, ctx, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
        layer.update(k, v)
        del k, v
    # a strided sample of C's source rows in two layers, to check the full-size shift (delta = -32768)
    rows = torch.arange(s.c0, s.c0 + s.c, 997, device=DEV)
    picked = (0, len(cache.layers) - 1)
    src = {i: cache.layers[i].keys[0][:, rows].float().cpu().numpy() for i in picked}
    splice(cache, s, inv)
    n = s.a + s.c
    assert cache.get_seq_length() == n == 98304
    cos_sin = ref_cos_sin(-s.gap, inv.detach().cpu())
    for i in picked:
        got = cache.layers[i].keys[0][:, rows - s.gap].float().cpu().numpy()
        assert np.array_equal(got, shift_keys_ref(src[i], dtype="bf16", cos_sin=cos_sin)), i
    x = torch.tensor([[1234]], device=DEV)
    with torch.no_grad():
        ours = model(input_ids=x, past_key_values=cache, use_cache=True).logits[0, -1].float()
        for layer in cache.layers:
            layer.crop(n)  # drop the token the first pass appended
        model.set_attn_implementation("sdpa")
        for layer in cache.layers:
            layer.fuse_append = False  # SDPA reads the cache itself: appends must be written, not deferred
        ref = model(input_ids=x, past_key_values=cache, use_cache=True).logits[0, -1].float()
    assert int(ours.argmax()) == int(ref.argmax())
    # bf16 logits through 36 layers differ by rounding noise; the distributions must still agree
    assert torch.corrcoef(torch.stack([ours, ref]))[0, 1].item() > 0.999


def small_bf16_engine(paged):
    """bf16, head_dim 128, 4 query heads per KV head: the paged decode and the tcgen05 prefill run."""
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=8192)
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation=tc_attention.NAME).to(DEV)
    return Session(model, min_suffix=4, prefill_chunk=64, max_ctx=4096, layout={"paged": paged, "max_tokens": 4096})


def test_paged_engine_matches_the_contiguous_engine():
    """The engine on a paged cache (splice = page drop + in-place key rotation, decode over pages with
    the fused append) against the same engine on the reference's contiguous layout: identical
    tokens while the pages hold the sequence in order, and after a splice turn the same reuse and
    last logits within the bf16 tolerance of T2."""
    from threadcut_b200.kv import PagedLayer
    eng_p, eng_c = small_bf16_engine(True), small_bf16_engine(False)
    p1 = rand_ids(150, 11)
    out_p, st_p = eng_p.generate(p1, max_new_tokens=20)
    out_c, st_c = eng_c.generate(p1, max_new_tokens=20)
    assert isinstance(eng_p.cache.layers[0], PagedLayer)
    assert out_p == out_c and st_p["kv_tokens"] == st_c["kv_tokens"] and st_p["kv_mb"] == st_c["kv_mb"]
    A, B, C, D = p1[:40], p1[40:97], p1[97:] + out_p, rand_ids(9, 12)
    with torch.no_grad():
        lp, sp = eng_p.load(A + C + D)
        lc, sc = eng_c.load(A + C + D)
    assert (sp["reused_prefix"], sp["reused_suffix"]) == (sc["reused_prefix"], sc["reused_suffix"]) == (40, len(C))
    assert eng_p.cache.get_seq_length() == len(A + C + D)
    assert torch.allclose(lp.float(), lc.float(), atol=3e-2, rtol=0)
    out_p2, _ = eng_p.generate(A + C + D + rand_ids(3, 13), max_new_tokens=8)
    assert len(out_p2) > 0


@pytest.mark.parametrize("kind", ["fp32_d16", "bf16_g2"])
def test_paged_engine_fallbacks_match_the_contiguous_engine(kind):
    """Paged caches the kernels cannot read directly: fp32 with head_dim 16 (no fused decode: rows are
    written and the attention sees a gathered copy) and bf16 with 2 query heads per KV head (decode
    over the pages, prefill on a gathered copy). Same tokens as the contiguous engine, two turns."""
    def make(paged):
        torch.manual_seed(0)
        if kind == "fp32_d16":
            cfg = Qwen3Config(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                              num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=4096)
            dtype = torch.float32
        else:
            cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                              num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=4096)
            dtype = torch.bfloat16
        model = AutoModelForCausalLM.from_config(cfg, dtype=dtype, attn_implementation=tc_attention.NAME).to(DEV)
        return Session(model, min_suffix=4, prefill_chunk=16, max_ctx=2048,
                       layout={"paged": paged, "max_tokens": 2048})
    eng_p, eng_c = make(True), make(False)
    p1 = rand_ids(60, 21)
    out_p, _ = eng_p.generate(p1, max_new_tokens=10)
    out_c, _ = eng_c.generate(p1, max_new_tokens=10)
    assert out_p == out_c
    p2 = p1[:20] + p1[35:] + out_p + rand_ids(5, 22)  # a pruned span: the splice path
    out_p2, sp = eng_p.generate(p2, max_new_tokens=10)
    out_c2, sc = eng_c.generate(p2, max_new_tokens=10)
    assert (sp["reused_prefix"], sp["reused_suffix"]) == (sc["reused_prefix"], sc["reused_suffix"])
    assert sp["reused_suffix"] > 0
    if kind == "fp32_d16":
        assert out_p2 == out_c2
    else:
        assert len(out_p2) > 0


def test_decode_step_replays_from_a_cuda_graph():
    """A one-token decode step through the plugin (fused append + decode kernel) can be captured in
    a CUDA graph: the registered mask builder keeps the capture free of host reads, and each replay
    gives the eager step's logits."""
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=8192)
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation=tc_attention.NAME)
    model = model.to(DEV).eval()
    cache = new_cache(model.config)
    ids = torch.randint(0, 512, (1, 300), device=DEV)
    x = torch.tensor([[7]], device=DEV)
    with torch.no_grad():
        model(input_ids=ids, past_key_values=cache, use_cache=True)
        n = cache.get_seq_length()
        eager = model(input_ids=x, past_key_values=cache, use_cache=True).logits.float()
        for layer in cache.layers:
            layer.crop(n)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = model(input_ids=x, past_key_values=cache, use_cache=True).logits
        for layer in cache.layers:
            layer.crop(n)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        replayed = out.float().clone()
        del graph
    assert int(replayed.argmax()) == int(eager.argmax())
    torch.testing.assert_close(replayed, eager, atol=2e-2, rtol=0)


def test_tensor_parallel_decoder_on_one_gpu_matches_the_hf_forward():
    """threadcut_b200.tp.TPDecoder at world 1: the HF forward's top-1 and logits, and a CUDA graph
    of its step replays the eager token (tests/tp_worker.py)."""
    from tp_worker import check
    res = check(torch.device(DEV))
    assert res["max_abs"] < 0.1, res


def test_accelerated_model_matches_the_plugin_forward_and_sdpa():
    """tp.accelerate(model): the engine's one-token calls (model(input_ids=[[t]],
    past_key_values=cache, use_cache=True)) run the fused step over the same cache. Teacher-forced
    over 6 steps after a 300-token prompt, each step's logits have the top-1 of the plugin forward
    (HF's Qwen3 layer with this attention) and of HF's SDPA forward on copies of the same cache, and
    correlate; the cache grows by one row per step as the reference's would; a prefill chunk still
    goes through the model's own forward; restore() undoes it."""
    from threadcut_b200 import tp
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=8192)
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation=tc_attention.NAME)
    model = model.to(DEV).eval()
    ids = torch.randint(0, 512, (1, 306), generator=torch.Generator().manual_seed(4)).to(DEV)
    with torch.no_grad():
        fast, plain = new_cache(model.config), new_cache(model.config)
        model(input_ids=ids[:, :300], past_key_values=fast, use_cache=True)
        model(input_ids=ids[:, :300], past_key_values=plain, use_cache=True)
        tp.accelerate(model)
        for i in range(300, 306):
            x = ids[:, i:i + 1]
            ref_cache = DynamicCache(config=model.config)
            for lr, lp in zip(ref_cache.layers, plain.layers):
                lr.update(lp.keys.clone(), lp.values.clone())
            got = model(input_ids=x, past_key_values=fast, use_cache=True).logits[0, -1].float()
            tp.restore(model)
            want = model(input_ids=x, past_key_values=plain, use_cache=True).logits[0, -1].float()
            model.set_attn_implementation("sdpa")
            sdpa = model(input_ids=x, past_key_values=ref_cache, use_cache=True).logits[0, -1].float()
            model.set_attn_implementation(tc_attention.NAME)
            tp.accelerate(model)
            assert fast.get_seq_length() == plain.get_seq_length() == i + 1
            assert int(got.argmax()) == int(want.argmax()) == int(sdpa.argmax()), i
            assert torch.corrcoef(torch.stack([got, want]))[0, 1].item() > 0.999
        chunk = model(input_ids=ids[:, :5], past_key_values=fast, use_cache=True)  # not one token: HF's forward
        assert chunk.logits.shape[1] == 5 and fast.get_seq_length() == 311
        tp.restore(model)
    assert not hasattr(model, "_threadcut_fused_step")
