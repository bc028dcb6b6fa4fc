"""Host-side logic and the C ABI boundary (CPU only: no kernel is launched here)."""
import ctypes
import os
import re

import pytest
import torch

from helpers import split_cases
from threadcut_b200 import _lib
from threadcut_b200.match import Split, lcp, split

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "threadcut_b200.h")


# ------------------------------------------------------------------ split (threadcut/match.py)
def test_split_rule_reference_cases():
    """The reference's own test_split_rule (tests/test_core.py:59-64)."""
    A, B, C, D = [1, 2, 3], [7, 7], [4, 5, 6, 8, 9], [10, 11]
    assert split(A + B + C, A + C + D, min_suffix=3) == Split(3, 5, 5)
    assert split(A + B + C, A + C + D, min_suffix=3, suffix=False) == Split(3, 3, 0)
    assert split(A + C, A + C + D, min_suffix=3) == Split(8, 8, 0)
    assert split(A + C, A + C, min_suffix=3).a == len(A + C) - 1


def test_split_matches_reference_golden_cases():
    cases = split_cases()
    assert len(cases) > 200
    for cs in cases:
        s = split(cs["cached"], cs["new"], min_suffix=cs["min_suffix"], suffix=cs["suffix"])
        assert [s.a, s.c0, s.c] == cs["expect"], cs


def test_lcp_and_gap():
    assert lcp([], [1]) == 0
    assert lcp([1, 2, 3], [1, 2, 4]) == 2
    assert lcp([1, 2], [1, 2, 3]) == 2
    assert Split(4, 9, 3).gap == 5


# ------------------------------------------------------------------ C ABI library
def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*|int|size_t)\s+(tc_\w+)\s*\(", text, re.M)))


def test_library_loads_and_exports_every_header_symbol():
    L = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 12, syms
    for name in syms:
        assert hasattr(L, name), f"{name} declared in include/threadcut_b200.h but not exported"
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_abi_version_and_status_strings():
    L = _lib.lib()
    assert L.tc_abi_version() == 1
    for code in range(6):
        assert L.tc_status_string(code)
    assert L.tc_status_string(0) == b"ok"


def test_argument_validation_without_a_gpu():
    """Entry points reject bad arguments before touching CUDA."""
    L = _lib.lib()
    # unsupported dtype
    assert L.tc_decode_attention(None, None, None, None, 8, 4, 128, 0, 0, 0, 0, 0, 0, 0, 0, 0,
                                 0.1, 0, 7, None, 0, None) == 3
    # K/V missing for a non-empty cache
    assert L.tc_decode_attention(None, None, None, None, 8, 4, 128, 16, 0, 0, 0, 0, 0, 0, 0, 0,
                                 0.1, 0, 2, None, 0, None) == 1
    # odd head_dim for the rope shift
    tab = (ctypes.c_float * 8)()
    assert L.tc_shift_keys(None, None, 1, 1, 7, 0, 0, 0, 0, tab, 2, None) == 1
    # missing cos/sin table
    assert L.tc_shift_keys(None, None, 1, 1, 8, 0, 0, 0, 0, None, 2, None) == 1
    # c0 < a is not a splice
    kp = (ctypes.c_void_p * 1)(None)
    assert L.tc_splice_inplace(kp, kp, 1, 8, 128, 100, 10, 5, 3, 0, 0, tab, 2, None, 0, 1, None) == 1
    # splice with gap 0 is a no-op that succeeds without launching anything
    assert L.tc_splice_inplace(kp, kp, 1, 8, 128, 100, 10, 10, 3, 0, 0, tab, 2, None, 0, 1, None) == 0
    # too many layers
    assert L.tc_splice_inplace(kp, kp, 129, 8, 128, 100, 1, 5, 3, 0, 0, tab, 2, None, 0, 1, None) == 1
    # C reaching past the buffer's capacity
    assert L.tc_splice_inplace(kp, kp, 1, 8, 128, 100, 1, 50, 51, 0, 0, tab, 2, None, 0, 1, None) == 1
    # merge with no parts
    assert L.tc_merge_partials(None, None, None, None, 0, 4, 128, 128, 2, None) == 1
    # empty shift is fine
    assert L.tc_shift_keys(None, None, 0, 5, 8, 0, 0, 0, 0, tab, 2, None) == 0


def test_paged_prefill_and_split_argument_validation_without_a_gpu():
    """The paged, paged-prefill, gather and device-split entry points reject bad arguments (and
    accept empty work) before touching CUDA."""
    L = _lib.lib()
    z = [0] * 4
    # paged decode: fp32 pools, pages shorter than a tile, a fused row without its value half
    assert L.tc_decode_attention_paged(None, None, None, None, 8, 4, 128, 64, 10, 0, 0, 0, None, 0, 0, None, None,
                                       0, 0, *z, 0.1, 0, 0, 0, None, 0, None) == 3
    assert L.tc_decode_attention_paged(None, None, None, None, 8, 4, 128, 16, 10, 0, 0, 0, None, 0, 0, None, None,
                                       0, 0, *z, 0.1, 0, 2, 0, None, 0, None) == 1
    kn = ctypes.c_void_p(16)
    assert L.tc_decode_attention_paged(kn, kn, kn, kn, 8, 4, 128, 64, 10, 0, 0, 0, kn, 1, 32, kn, None,
                                       0, 0, *z, 0.1, 0, 2, 0, None, 0, None) == 1
    # stable_tiles must not be negative
    assert L.tc_decode_attention_paged(kn, kn, kn, kn, 8, 4, 128, 64, 10, 0, 0, 0, kn, 1, 32, None, None,
                                       0, 0, *z, 0.1, 0, 2, -1, None, 0, None) == 1
    # paged prefill: head_dim 64, 2 query heads per KV head, no sub-tile table
    assert L.tc_prefill_attention_paged(kn, kn, kn, kn, 32, 8, 4, 100, 64, 64, 10, 0, 0, 0, kn, 4, kn, 0, 0, 0, 0,
                                        0.1, 0, 2, None, 0, None) == 1
    assert L.tc_prefill_attention_paged(kn, kn, kn, kn, 16, 8, 4, 100, 128, 64, 10, 0, 0, 0, kn, 4, kn, 0, 0, 0, 0,
                                        0.1, 0, 2, None, 0, None) == 1
    assert L.tc_prefill_attention_paged(kn, kn, kn, kn, 32, 8, 4, 100, 128, 64, 10, 0, 0, 0, None, 4, kn, 0, 0, 0, 0,
                                        0.1, 0, 2, None, 0, None) == 1
    # rotate / write / gather: no layers, no heads, bad dtype; empty work succeeds without a launch
    tab = (ctypes.c_float * 128)()
    kp = (ctypes.c_void_p * 1)(16)
    assert L.tc_paged_rotate_keys(kp, 0, 8, 128, 64, 10, 0, 0, 0, kn, 1, tab, 2, None) == 1
    assert L.tc_paged_rotate_keys(kp, 1, 8, 128, 64, 10, 0, 0, 0, None, 0, tab, 2, None) == 0
    assert L.tc_paged_write(kn, kn, kn, kn, 0, 128, 3, 0, 0, 0, 0, 64, 10, 0, 0, 0, kn, 2, None) == 1
    assert L.tc_paged_write(kn, kn, kn, kn, 8, 128, 0, 0, 0, 0, 0, 64, 10, 0, 0, 0, kn, 2, None) == 0
    assert L.tc_paged_gather(kn, kn, kn, kn, 8, 128, 10, 0, 0, 64, 10, 0, 0, 0, kn, 1, 7, None) == 3
    assert L.tc_paged_gather(kn, kn, kn, kn, 8, 128, 0, 0, 0, 64, 10, 0, 0, 0, kn, 1, 2, None) == 0
    # device split: an empty request, a missing workspace
    out = (ctypes.c_int64 * 3)()
    assert L.tc_split(kn, 10, kn, 0, 32, 1, out, kn, 1 << 20, None) == 1
    assert L.tc_split(kn, 10, kn, 5, 32, 1, out, None, 0, None) == 4
    assert L.tc_split_workspace_size(1000) >= 16 * 1000


def test_splice_workspace_bound():
    L = _lib.lib()
    assert L.tc_splice_workspace_size(36, 8, 4096) >= 16 + 4 * 36 * 8 * (4096 // 64)
    assert L.tc_splice_workspace_size(0, 8, 10) == 0


# ------------------------------------------------------------------ no CPU fallback
def test_decode_on_cpu_tensors_fails_loudly():
    from threadcut_b200.flash_decode import decode_attention
    q = torch.randn(8, 4, 128)
    k = torch.randn(8, 10, 128)
    with pytest.raises(RuntimeError, match="CUDA"):
        decode_attention(q, k, k, 0.1)


def test_shift_on_cpu_tensors_fails_loudly():
    from threadcut_b200.kv import shift_keys
    with pytest.raises(RuntimeError, match="CUDA"):
        shift_keys(torch.randn(1, 2, 5, 16), -3, torch.ones(8))


def test_plugin_decode_branch_on_cpu_fails_loudly():
    from threadcut_b200.attention import attention
    with pytest.raises(RuntimeError, match="CUDA"):
        attention(None, torch.randn(1, 8, 1, 16), torch.randn(1, 2, 5, 16), torch.randn(1, 2, 5, 16), None)


def test_missing_library_is_an_error(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="missing"):
        _lib.lib()


# ------------------------------------------------------------------ GrowingLayer bookkeeping
def test_growing_layer_growth_policy_and_views():
    from threadcut_b200.kv import GrowingLayer, new_cache
    ly = GrowingLayer()
    k = torch.randn(1, 2, 3, 16)
    ly.update(k, k + 1)
    assert ly.kbuf.shape[-2] == 2048 + 0 and ly.n == 3  # max(3, 0, 0 + 2048)
    assert torch.equal(ly.keys, k) and torch.equal(ly.values, k + 1)
    ly.update(torch.randn(1, 2, 2100, 16), torch.randn(1, 2, 2100, 16))
    assert ly.kbuf.shape[-2] == max(2103, int(2048 * 1.25), 2048 + 2048)
    assert torch.equal(ly.keys[..., :3, :], k)
    ly.crop(5)
    assert ly.get_seq_length() == 5
    ly.crop(100)
    assert ly.get_seq_length() == 5
    from transformers import Qwen3Config
    cache = new_cache(Qwen3Config(num_hidden_layers=3))
    assert len(cache.layers) == 3 and all(isinstance(x, GrowingLayer) for x in cache.layers)


def test_splice_c_zero_needs_no_device():
    """Split with c == 0 only truncates (kv.py:85-91): no kernel, works on any tensors."""
    from threadcut_b200.kv import GrowingLayer
    ly = GrowingLayer()
    k = torch.randn(1, 2, 10, 16)
    ly.update(k, k)
    ly.splice(Split(4, 4, 0), torch.ones(8))
    assert ly.get_seq_length() == 4 and torch.equal(ly.keys, k[..., :4, :])


def test_workspace_epochs_are_unique_and_nonzero():
    ws = _lib._Workspaces()

    class Dev:
        index = None
    seen = set()
    # next_epoch keys on the current stream; emulate with a CPU-only key by monkeypatching
    orig = _lib.stream_ptr
    try:
        _lib.stream_ptr = lambda d: 0
        for _ in range(5):
            e = ws.next_epoch("splice", Dev())
            assert e != 0 and e not in seen
            seen.add(e)
    finally:
        _lib.stream_ptr = orig


def test_host_binding_loads_without_a_gpu():
    """The compiled host binding of decode_attention loads, is wired to the library's
    tc_decode_attention_stable, and declines CPU tensors so the checked path raises as before."""
    hb = _lib.host()
    assert hb is not None, "threadcut_b200/_host/threadcut_b200_host.so is missing: run threadcut_b200.build"
    assert callable(hb.decode) and callable(hb.init)
    t = torch.zeros(8, 4, 128, dtype=torch.bfloat16)
    assert hb.decode(t, t, t, 0.1, 0, 0, torch.zeros(16, dtype=torch.uint8)) is None


def test_host_binding_first_use_in_a_fresh_process():
    """The first decode call of a process loads the library and the binding in one go (no lock
    taken twice): run it in a fresh interpreter with a deadline."""
    import subprocess
    import sys
    code = ("import torch; from threadcut_b200 import _lib; from threadcut_b200.flash_decode import _decode_fast; "
            "assert _lib.host() is not None; t = torch.zeros(2, 1, 64); "
            "assert _decode_fast(t, t, t, 0.1, None, 0) is None; print('ok')")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


def test_qwen3_4b_config_geometry_and_size():
    """The config-5 model: BASELINE geometry, and about 4.0B parameters (8 GB of bf16 weights with the
    tied embedding stored once), counted on the meta device without allocating them."""
    from transformers import AutoModelForCausalLM

    import workloads
    cfg = workloads.qwen3_4b_config()
    assert (cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads, cfg.num_key_value_heads,
            cfg.head_dim) == (2560, 36, 32, 8, 128)
    assert cfg.rope_parameters["rope_theta"] == 1.0e6 and cfg.max_position_embeddings >= 131072
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16)
    params = sum(p.numel() for p in model.parameters())
    assert 3.9e9 < params < 4.1e9, params


def _mask_cases():
    from transformers.masking_utils import causal_mask_function, sliding_window_causal_mask_function
    pad = torch.ones(1, 9, dtype=torch.bool)
    pad[0, 2] = False
    for q_len, kv_len, q_off in ((1, 9, 8), (1, 9, 5), (4, 9, 5), (9, 9, 0), (1, 1, 0)):
        yield dict(batch_size=1, q_length=q_len, kv_length=kv_len, q_offset=q_off, kv_offset=0)
        yield dict(batch_size=1, q_length=q_len, kv_length=kv_len, q_offset=q_off, kv_offset=0, attention_mask=pad[:, :kv_len])
        yield dict(batch_size=1, q_length=q_len, kv_length=kv_len, q_offset=q_off, kv_offset=0, allow_is_causal_skip=False)
        yield dict(batch_size=1, q_length=q_len, kv_length=kv_len, q_offset=q_off, kv_offset=0, local_size=4,
                   mask_function=sliding_window_causal_mask_function(4))
    yield dict(batch_size=2, q_length=1, kv_length=9, q_offset=8, kv_offset=0, mask_function=causal_mask_function)


@pytest.mark.parametrize("capturing", [False, True])
def test_plugin_mask_equals_sdpa_mask(capturing, monkeypatch):
    """The registered mask builder returns sdpa_mask's mask (reference attention.py:50-51). While a
    CUDA graph is being captured, sdpa_mask builds the all-True mask of a one-token step, and the
    plugin's builder returns None there instead; every other case is unchanged."""
    import transformers.masking_utils as mu
    from threadcut_b200 import attention as tc_attention
    if capturing:
        monkeypatch.setattr(mu, "is_tracing", lambda *a, **k: True)
    for kw in _mask_cases():
        ref = mu.sdpa_mask(**kw)
        ours = tc_attention.attention_mask(**kw)
        decode_skip = (kw["q_length"] == 1 and kw.get("attention_mask") is None and kw.get("local_size") is None
                       and kw.get("allow_is_causal_skip", True) and kw["q_offset"] >= kw["kv_length"] - 1)
        if capturing and decode_skip:
            assert ours is None and ref is not None and bool(ref.all()), kw
        elif ref is None:
            assert ours is None, kw
        else:
            assert ours is not None and torch.equal(ours, ref), kw


def test_layer_ops_on_cpu_tensors_fail_loudly():
    """The tensor-parallel step's launches refuse host tensors (no CPU path, no device call)."""
    from threadcut_b200 import tp
    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    w = torch.ones(64, dtype=torch.bfloat16)
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        tp._add_rmsnorm(x, None, w, torch.empty_like(x), 1e-6)
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        tp._qk_norm_rope(x, x, w, w, w, w, 1e-6)
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        tp._silu_mul(torch.zeros(1, 128, dtype=torch.bfloat16), x)


def test_layer_ops_argument_validation_without_a_gpu():
    L = _lib.lib()
    assert L.tc_add_rmsnorm(None, None, None, None, 0, 64, 1e-6, 2, None) == 0  # no rows: nothing to do
    assert L.tc_add_rmsnorm(None, None, None, None, 1, 64, 1e-6, 2, None) != 0
    assert L.tc_add_rmsnorm(None, None, None, None, 1, 0, 1e-6, 2, None) != 0
    assert L.tc_add_rmsnorm(None, None, None, None, 1, 64, 1e-6, 7, None) != 0
    assert L.tc_qk_norm_rope(None, None, None, None, None, None, 0, 0, 128, 1e-6, 2, None) == 0
    assert L.tc_qk_norm_rope(None, None, None, None, None, None, 1, 0, 127, 1e-6, 2, None) != 0
    assert L.tc_qk_norm_rope(None, None, None, None, None, None, 1, 0, 2048, 1e-6, 2, None) != 0
    assert L.tc_qk_norm_rope(None, None, None, None, None, None, 1, 1, 128, 1e-6, 2, None) != 0
    assert L.tc_silu_mul(None, None, 0, 64, 2, None) == 0
    assert L.tc_silu_mul(None, None, 1, 64, 2, None) != 0
    assert L.tc_silu_mul(None, None, 1, 0, 2, None) != 0


def test_gemv_argument_validation_without_a_gpu():
    L = _lib.lib()
    assert L.tc_gemv(None, None, None, 0, 64, 2, None) == 0  # no rows: nothing to do
    assert L.tc_gemv(None, None, None, 4, 64, 2, None) != 0  # null operands
    assert L.tc_gemv(16, 32, 64, 4, 60, 2, None) != 0  # k not a multiple of 8
    assert L.tc_gemv(16, 32, 64, 4, 64, 0, None) != 0  # fp32: not supported
    assert L.tc_gemv(8, 32, 64, 4, 64, 2, None) != 0   # x not 16-byte aligned (rejected before any access)
    assert L.tc_gemv(16, 32, 64, 4, 32768, 2, None) != 0  # x would not fit in shared memory


# ------------------------------------------------------------------ the reference's engine over this package
REFERENCE = os.environ.get("THREADCUT_REFERENCE", "/root/reference")


def test_reference_engine_runs_unchanged_over_this_package(monkeypatch):
    """threadcut/engine.py, loaded from the reference checkout as it is (no copy in this
    repository), with its package's attention / kv / match modules resolved to threadcut_b200's:
    its imports bind to this package, its cache calls build this package's caches (contiguous by
    default, paged after kv.use_paged_cache()), and a request runs through the plugin (the prefill
    chunk on the CPU through the reference's torch branch) until the first decode step reaches the
    CUDA kernels, which refuse CPU tensors: there is no CPU path. Skipped without the checkout
    (it is not shipped to GPU machines)."""
    import importlib.util
    import sys
    import types
    from transformers import AutoModelForCausalLM, Qwen3Config
    from threadcut_b200 import attention, kv, match
    src = os.path.join(REFERENCE, "threadcut", "engine.py")
    if not os.path.exists(src):
        pytest.skip("the reference checkout is not present")
    pkg = types.ModuleType("threadcut")
    pkg.__path__ = []
    pkg.attention, pkg.kv, pkg.match = attention, kv, match
    for name, mod in (("threadcut", pkg), ("threadcut.attention", attention), ("threadcut.kv", kv),
                      ("threadcut.match", match)):
        monkeypatch.setitem(sys.modules, name, mod)
    spec = importlib.util.spec_from_file_location("threadcut.engine", src)
    engine = importlib.util.module_from_spec(spec)
    monkeypatch.setitem(sys.modules, "threadcut.engine", engine)
    spec.loader.exec_module(engine)
    assert engine.attention is attention and engine.new_cache is kv.new_cache
    assert engine.splice is kv.splice and engine.split is match.split

    class Tok:  # the engine only asks the tokenizer for its stop ids (threadcut/engine.py:36)
        eos_token_id = 511

        def convert_tokens_to_ids(self, tok):
            return 510

    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=4096)
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.float32, attn_implementation=attention.NAME)
    eng = engine.Engine(None, device="cpu", model=model, tokenizer=Tok(), min_suffix=4, prefill_chunk=7)
    cache = engine.new_cache(model.config)
    assert all(isinstance(ly, kv.GrowingLayer) and ly.fuse_append for ly in cache.layers)
    try:
        kv.use_paged_cache(True, max_tokens=1024)
        assert all(isinstance(ly, kv.PagedLayer) for ly in engine.new_cache(model.config).layers)
    finally:
        kv.use_paged_cache(False)
    ids = torch.randint(10, 500, (20,), generator=torch.Generator().manual_seed(5)).tolist()
    logits, stats = eng.load(ids)  # fresh cache + chunked prefill: the reference's torch prefill branch
    assert logits.shape == (1, 512) and stats["computed_tokens"] == 20 and eng.cache.get_seq_length() == 20
    assert isinstance(eng.cache.layers[0], kv.GrowingLayer)
    with pytest.raises(RuntimeError, match="CUDA device"):
        eng.generate(ids + [7, 8], max_new_tokens=2)  # the decode step reaches the kernels


def test_peer_sum_argument_validation_without_a_gpu():
    """The peer-memory sums check their arguments before touching the device."""
    L = _lib.lib()
    assert L.tc_peer_handle_bytes() == 64
    # 2 KB of control (sequence, CTA count, the residual form's sums of squares), then 2 slots of words
    assert L.tc_allreduce_region_bytes(8, 2560) == 2048 + 2 * 8 * 2560 * 8
    assert L.tc_allreduce_region_bytes(9, 2560) == 0 and L.tc_allreduce_region_bytes(2, 0) == 0
    regs = (ctypes.c_void_p * 2)(256, 512)
    assert L.tc_gemv_allreduce(16, 16, 2560, 512, regs, 2, 0, 0, None) == 3        # fp32: dtype
    assert L.tc_gemv_allreduce(16, 16, 2560, 512, regs, 2, 2, 2, None) == 1        # rank outside world
    assert L.tc_gemv_allreduce(16, 16, 2560, 500, regs, 2, 0, 2, None) == 1        # k not a multiple of 8
    assert L.tc_gemv_allreduce(8, 16, 2560, 512, regs, 2, 0, 2, None) == 2         # x misaligned
    assert L.tc_gemv_allreduce(16, 16, 2560, 512, None, 2, 0, 2, None) == 1        # no regions
    assert L.tc_allreduce_add_rmsnorm(16, 16, 16, 9000, 1e-6, 256, 2, 2, None) == 1  # hidden too large
    assert L.tc_allreduce_add_rmsnorm(16, 16, 16, 2560, 1e-6, 100, 2, 2, None) == 1  # region misaligned
    assert L.tc_peer_open(None, None) == 1 and L.tc_peer_close(None) == 1 and L.tc_peer_free(None) == 1
    # residual form and the normalised-input projection
    assert L.tc_gemv_allreduce_residual(16, 16, 2560, 512, regs, 2, 0, None, 2, None) == 1    # no residual
    assert L.tc_gemv_allreduce_residual(16, 16, 2560, 512, regs, 2, 0, 32, 0, None) == 3      # fp32: dtype
    assert L.tc_gemv_allreduce_residual_swiglu(16, 16, 2560, 500, regs, 2, 0, 32, 2, None) == 1  # k % 8
    assert L.tc_gemv_rmsnorm(16, 16, 256, 1e-6, 16, 16, 64, 2560, 0, None) == 3               # fp32: dtype
    assert L.tc_gemv_rmsnorm(16, 16, 256, 1e-6, 16, 16, 64, 2561, 2, None) == 1               # k % 8
    assert L.tc_gemv_rmsnorm(16, 16, 256, -1.0, 16, 16, 64, 2560, 2, None) == 1               # eps < 0
    assert L.tc_gemv_rmsnorm(8, 16, 256, 1e-6, 16, 16, 64, 2560, 2, None) == 2                # h misaligned
    assert L.tc_gemv_rmsnorm(16, 16, None, 1e-6, 16, 16, 64, 2560, 2, None) == 1              # no region
    # the gate/up projection with the SwiGLU epilogue (interleaved rows: n even)
    assert L.tc_gemv_rmsnorm_swiglu(16, 16, 256, 1e-6, 16, 16, 64, 2560, 0, None) == 3        # fp32: dtype
    assert L.tc_gemv_rmsnorm_swiglu(16, 16, 256, 1e-6, 16, 16, 63, 2560, 2, None) == 1        # n odd
    assert L.tc_gemv_rmsnorm_swiglu(16, 16, 256, 1e-6, 16, 16, 64, 2561, 2, None) == 1        # k % 8
    assert L.tc_gemv_rmsnorm_swiglu(16, 16, 256, 1e-6, 24, 16, 64, 2560, 2, None) == 2        # w misaligned
    assert L.tc_gemv_rmsnorm_swiglu(16, 16, 256, 1e-6, 16, None, 64, 2560, 2, None) == 1      # no output
    assert L.tc_gemv_rmsnorm_swiglu(16, 16, 256, 1e-6, 16, 16, 0, 2560, 2, None) == 0         # nothing to do


def test_peer_gather_argument_validation_without_a_gpu():
    L = _lib.lib()
    # o [rows][d] then lse [rows] per source, padded to a multiple of 4 floats, two slots
    assert L.tc_gather_region_bytes(8, 1152, 128) == 256 + 2 * 8 * (1152 * 129) * 4
    assert L.tc_gather_region_bytes(2, 3, 128) == 256 + 2 * 2 * 388 * 4
    assert L.tc_gather_region_bytes(9, 3, 128) == 0 and L.tc_gather_region_bytes(2, 3, 6) == 0
    regs = (ctypes.c_void_p * 2)(256, 512)
    assert L.tc_peer_gather_merge(16, 16, 16, None, 3, 128, 128, regs, 2, 0, 7, None) == 3   # dtype
    assert L.tc_peer_gather_merge(16, 16, 16, None, 3, 128, 100, regs, 2, 0, 2, None) == 1   # out stride < d
    assert L.tc_peer_gather_merge(8, 16, 16, None, 3, 128, 128, regs, 2, 0, 2, None) == 2    # o misaligned
    assert L.tc_peer_gather_merge(16, 16, 16, None, 3, 128, 128, regs, 2, 5, 2, None) == 1   # rank
