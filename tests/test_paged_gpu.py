"""Paged K/V cache on the GPU (needs a B200) against the reference's contiguous cache model.

* after appends and splices the pools, read in run order, equal the reference cache bit for bit
  (keys re-rotated by the same fp32 expression as threadcut/kv.py:25, values untouched);
* paged decode is within the decode tolerance of the fp32 oracle on the gathered cache, and
  bit-identical to the contiguous kernel when the pages hold the sequence in order (same tiles,
  same split);
* the fused append (one-token step written by the decode launch) is bit-identical to writing the
  row first and decoding.
"""
import numpy as np
import pytest
import torch

from helpers import ATTN_ATOL, attn_error, ref_cos_sin
from oracle.attention import decode_attention_ref
from oracle.paged import ListCache, gather_ref
from oracle.rope import inv_freq_default
from threadcut_b200 import _lib
from threadcut_b200.flash_decode import decode_attention
from threadcut_b200.match import Split
from threadcut_b200.paged import PagedKV

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    _lib.device_errors(clear=True)
    yield
    assert _lib.device_errors(clear=True) == 0


def f32(t):
    return t.float().cpu().numpy()


def drive(seed, layers=2, hkv=8, d=128, dtype=torch.bfloat16, page_rows=64, ops=14, max_tokens=3000):
    """Random engine-like traffic on a PagedKV and on the reference's list model side by side."""
    rng = np.random.default_rng(seed)
    g = torch.Generator(device=DEV).manual_seed(seed)
    inv_freq = torch.as_tensor(inv_freq_default(d, 1e6), dtype=torch.float32)
    kv = PagedKV(layers, hkv, d, max_tokens=max_tokens, page_rows=page_rows, dtype=dtype, device=DEV)
    ref = ListCache(layers, hkv, d)
    for i in range(ops):
        if i % 3 != 2 or kv.n == 0:
            t = int(rng.choice([1, 1, 7, 40, 64, 130, 300]))
            if kv.n + t > max_tokens - 2 * page_rows:
                t = 1
            kv.reserve(t)
            for l in range(layers):
                k = torch.randn(hkv, t, d, generator=g, device=DEV).to(dtype)
                v = torch.randn(hkv, t, d, generator=g, device=DEV).to(dtype)
                kv.write(l, k, v)
                ref.append(l, f32(k), f32(v))
        else:
            n = kv.n
            a = int(rng.integers(0, n + 1))
            c0 = int(rng.integers(a, n + 1))
            c = int(rng.integers(0, n - c0 + 1))
            kv.splice(Split(a, c0, c), inv_freq)
            ref.splice(a, c0, c, dtype="bf16" if dtype == torch.bfloat16 else "f16",
                       cos_sin=ref_cos_sin(-(c0 - a), inv_freq))
    torch.cuda.synchronize()
    return kv, ref, g


@pytest.mark.parametrize("seed,page_rows,d", [(0, 64, 128), (1, 32, 128), (2, 96, 128), (3, 64, 64), (4, 128, 256)])
def test_pools_match_the_reference_cache_bit_for_bit(seed, page_rows, d):
    kv, ref, _ = drive(seed, d=d, page_rows=page_rows)
    for l in range(kv.layers):
        k = gather_ref(f32(kv.k[l]), kv.table.runs)
        v = gather_ref(f32(kv.v[l]), kv.table.runs)
        assert k.shape == ref.k[l].shape
        assert np.array_equal(k.view(np.uint32), ref.k[l].view(np.uint32)), (seed, l)
        assert np.array_equal(v.view(np.uint32), ref.v[l].view(np.uint32)), (seed, l)
        gk, gv = kv.gather(l)
        assert np.array_equal(f32(gk), k) and np.array_equal(f32(gv), v)


@pytest.mark.parametrize("seed,page_rows,d,dtype", [(5, 64, 128, torch.bfloat16), (6, 32, 128, torch.float16),
                                                    (7, 64, 64, torch.bfloat16), (8, 128, 256, torch.bfloat16)])
@pytest.mark.parametrize("splits", [None, 1, 7])
def test_paged_decode_matches_the_oracle(seed, page_rows, d, dtype, splits):
    kv, ref, g = drive(seed, d=d, dtype=dtype, page_rows=page_rows)
    q = torch.randn(kv.hkv, 4, d, generator=g, device=DEV).to(dtype)
    for l in range(kv.layers):
        out = kv.decode(l, q, 0.088, splits=splits)
        torch.cuda.synchronize()
        want = decode_attention_ref(f32(q), ref.k[l], ref.v[l], 0.088)
        assert attn_error(f32(out), want, dtype) <= ATTN_ATOL, (seed, l, splits)


@pytest.mark.parametrize("n", [1, 31, 32, 100, 4096, 16384])
def test_in_order_pages_are_bit_identical_to_the_contiguous_kernel(n):
    """One append of n rows fills pages 0, 1, 2, ... in order: the paged tiles are the contiguous
    kernel's tiles, so with the same per-head split (the planner's one wave of SM-count / heads
    slices per head, which the contiguous kernel runs when the split count is given) every partial
    sum is the same."""
    g = torch.Generator(device=DEV).manual_seed(n)
    kv = PagedKV(1, 8, 128, max_tokens=n, page_rows=64, device=DEV)
    k = torch.randn(8, n, 128, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(8, n, 128, generator=g, device=DEV).to(torch.bfloat16)
    kv.reserve(n)
    kv.write(0, k, v)
    q = torch.randn(8, 4, 128, generator=g, device=DEV).to(torch.bfloat16)
    got = kv.decode(0, q, 0.0883)
    per_head = torch.cuda.get_device_properties(DEV).multi_processor_count // 8
    want = decode_attention(q, k, v, 0.0883, splits=per_head)
    torch.cuda.synchronize()
    assert torch.equal(got, want), n


@pytest.mark.parametrize("seed,page_rows", [(9, 64), (10, 32)])
def test_fused_append_is_write_then_decode(seed, page_rows):
    kv_a, _, g = drive(seed, page_rows=page_rows)
    kv_b, _, _ = drive(seed, page_rows=page_rows)
    for step in range(5):
        q = torch.randn(kv_a.hkv, 4, 128, generator=g, device=DEV).to(torch.bfloat16)
        kn = torch.randn(kv_a.hkv, 128, generator=g, device=DEV).to(torch.bfloat16)
        vn = torch.randn(kv_a.hkv, 128, generator=g, device=DEV).to(torch.bfloat16)
        kv_a.reserve(1)
        kv_b.reserve(1)
        for l in range(kv_a.layers):
            kv_a.write(l, kn[:, None], vn[:, None])
            want = kv_a.decode(l, q, 0.09)
            got = kv_b.decode(l, q, 0.09, k_new=kn, v_new=vn)
            torch.cuda.synchronize()
            assert torch.equal(got, want), (step, l)
    for l in range(kv_a.layers):
        assert torch.equal(kv_a.k[l], kv_b.k[l]) and torch.equal(kv_a.v[l], kv_b.v[l])


def test_empty_and_rejected_cases():
    kv = PagedKV(1, 8, 128, max_tokens=256, device=DEV)
    q = torch.randn(8, 4, 128, device=DEV).to(torch.bfloat16)
    assert torch.count_nonzero(kv.decode(0, q, 0.1)) == 0
    with pytest.raises(ValueError):
        PagedKV(1, 8, 128, max_tokens=256, page_rows=16, device=DEV)
    with pytest.raises(ValueError):
        kv.write(0, torch.zeros(8, 3, 128, device=DEV, dtype=torch.bfloat16),
                 torch.zeros(8, 3, 128, device=DEV, dtype=torch.bfloat16))  # nothing reserved
    kv32 = PagedKV(1, 8, 128, max_tokens=256, dtype=torch.float32, device=DEV)
    kv32.reserve(4)
    kv32.write(0, torch.randn(8, 4, 128, device=DEV), torch.randn(8, 4, 128, device=DEV))
    with pytest.raises(_lib.TCError):
        kv32.decode(0, torch.randn(8, 4, 128, device=DEV), 0.1)  # decode over pages: 16-bit only


@pytest.mark.parametrize("seed,page_rows", [(11, 64), (12, 32)])
def test_stable_tiles_back_to_back_matches_plain(seed, page_rows):
    """Layer-by-layer one-token steps with the fused append, launched back to back with every tile
    but the last declared stable (loaded before the previous launch ends), give the same outputs
    and pools as the plain calls."""
    kv_a, _, g = drive(seed, layers=4, page_rows=page_rows)
    kv_b, _, _ = drive(seed, layers=4, page_rows=page_rows)
    for step in range(4):
        qs = [torch.randn(8, 4, 128, generator=g, device=DEV).to(torch.bfloat16) for _ in range(4)]
        kn = [torch.randn(8, 128, generator=g, device=DEV).to(torch.bfloat16) for _ in range(4)]
        vn = [torch.randn(8, 128, generator=g, device=DEV).to(torch.bfloat16) for _ in range(4)]
        kv_a.reserve(1)
        kv_b.reserve(1)
        want = [kv_a.decode(l, qs[l], 0.09, k_new=kn[l], v_new=vn[l]) for l in range(4)]
        got = [kv_b.decode(l, qs[l], 0.09, k_new=kn[l], v_new=vn[l], stable_tiles=kv_b.n_tiles - 1)
               for l in range(4)]
        torch.cuda.synchronize()
        for l in range(4):
            assert torch.equal(got[l], want[l]), (step, l)
    for l in range(4):
        assert torch.equal(kv_a.k[l], kv_b.k[l]) and torch.equal(kv_a.v[l], kv_b.v[l])


def test_compact_repacks_in_order_and_keeps_the_contents():
    kv, ref, g = drive(13, page_rows=64)
    before = [kv.gather(l) for l in range(kv.layers)]
    kv.compact()
    runs = kv.table.runs
    assert [r[0] for r in runs] == list(range(len(runs))) and all(r[1] == 0 for r in runs)
    for l in range(kv.layers):
        k, v = kv.gather(l)
        assert torch.equal(k, before[l][0]) and torch.equal(v, before[l][1])
    q = torch.randn(kv.hkv, 4, 128, generator=g, device=DEV).to(torch.bfloat16)
    out = kv.decode(0, q, 0.088)
    torch.cuda.synchronize()
    assert attn_error(f32(out), decode_attention_ref(f32(q), ref.k[0], ref.v[0], 0.088), torch.bfloat16) <= ATTN_ATOL


def prefill_reference(q, k, v, scale):
    """fp32 SDPA with the causal-over-cache mask on the gathered (contiguous) cache."""
    from threadcut_b200.prefill import causal_offset_mask
    hq, hkv = q.shape[1], k.shape[1]
    kk = k.float().repeat_interleave(hq // hkv, 1)
    vv = v.float().repeat_interleave(hq // hkv, 1)
    mask = causal_offset_mask(q.shape[2], k.shape[2], q.device)
    return torch.nn.functional.scaled_dot_product_attention(q.float(), kk, vv, attn_mask=mask,
                                                            scale=scale).transpose(1, 2)


@pytest.mark.parametrize("seed,page_rows,hkv,lq", [(14, 64, 8, 1), (15, 64, 8, 200), (16, 32, 2, 64), (17, 96, 8, 65),
                                                   (18, 128, 2, 300), (19, 64, 2, 7)])
@pytest.mark.parametrize("splits", [None, 1, 3])
def test_paged_prefill_matches_the_reference(seed, page_rows, hkv, lq, splits):
    """A prefill chunk appended after random appends and splices (ragged runs, runs starting inside
    pages) attends over the pages directly, within the prefill kernel's 1e-2 of fp32 SDPA on the
    gathered cache."""
    kv, _, g = drive(seed, layers=1, hkv=hkv, page_rows=page_rows)
    kv.reserve(lq)
    kv.write(0, torch.randn(hkv, lq, 128, generator=g, device=DEV).to(torch.bfloat16),
             torch.randn(hkv, lq, 128, generator=g, device=DEV).to(torch.bfloat16))
    q = torch.randn(1, 4 * hkv, lq, 128, generator=g, device=DEV).to(torch.bfloat16)
    out = kv.prefill(0, q, 0.0883, splits=splits)
    torch.cuda.synchronize()
    k, v = kv.gather(0)
    err = (out.float() - prefill_reference(q, k[None], v[None], 0.0883)).abs().max().item()
    assert out.shape == (1, lq, 4 * hkv, 128) and err <= 1e-2, (seed, lq, splits, err)


def test_paged_prefill_long_cache_and_fresh_sequence():
    """A 512-token chunk over a 20k-token spliced cache, and a first chunk (cache = the chunk)."""
    g = torch.Generator(device=DEV).manual_seed(20)
    inv_freq = torch.as_tensor(inv_freq_default(128, 1e6), dtype=torch.float32)
    kv = PagedKV(1, 8, 128, max_tokens=24000, device=DEV)
    kv.reserve(22000)
    kv.write(0, torch.randn(8, 22000, 128, generator=g, device=DEV).to(torch.bfloat16),
             torch.randn(8, 22000, 128, generator=g, device=DEV).to(torch.bfloat16))
    kv.splice(Split(3001, 5077, 16000), inv_freq)
    kv.reserve(512)
    kv.write(0, torch.randn(8, 512, 128, generator=g, device=DEV).to(torch.bfloat16),
             torch.randn(8, 512, 128, generator=g, device=DEV).to(torch.bfloat16))
    q = torch.randn(1, 32, 512, 128, generator=g, device=DEV).to(torch.bfloat16)
    out = kv.prefill(0, q, 0.0883)
    k, v = kv.gather(0)
    assert (out.float() - prefill_reference(q, k[None], v[None], 0.0883)).abs().max().item() <= 1e-2
    fresh = PagedKV(1, 8, 128, max_tokens=300, device=DEV)
    fresh.reserve(300)
    fresh.write(0, torch.randn(8, 300, 128, generator=g, device=DEV).to(torch.bfloat16),
                torch.randn(8, 300, 128, generator=g, device=DEV).to(torch.bfloat16))
    q = torch.randn(1, 32, 300, 128, generator=g, device=DEV).to(torch.bfloat16)
    out = fresh.prefill(0, q, 0.0883)
    k, v = fresh.gather(0)
    assert (out.float() - prefill_reference(q, k[None], v[None], 0.0883)).abs().max().item() <= 1e-2
