"""RoPE shift and KV splice on the GPU vs the oracle and the reference's golden outputs.

Bar: shifted keys bit-identical to the reference's fp32 expression when both use the same cos/sin
table (the host table is built with the reference's own torch ops), hence within 1 bf16 ulp of an
fp32 rotation; values moved exactly.
"""
import numpy as np
import pytest
import torch

import workloads
from helpers import TORCH_DTYPE, gold, meta, ref_cos_sin, sha, storage_dtype, values
from oracle.rope import shift_keys_ref
from oracle.splice import growing_splice_ref
from threadcut_b200 import _lib
from threadcut_b200.kv import GrowingLayer, new_cache, shift_keys, splice
from threadcut_b200.match import Split

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    _lib.device_errors(clear=True)
    yield
    assert _lib.device_errors(clear=True) == 0


def dev_tensor(a, dtype):
    return torch.as_tensor(np.asarray(a, dtype=np.float32)).to(DEV).to(dtype)


def exact(t, ref_values):
    """Bitwise equality of a device tensor with fp32 reference values of its dtype."""
    got = t.float().cpu().numpy()
    return np.array_equal(got.view(np.uint32), np.asarray(ref_values, dtype=np.float32).view(np.uint32))


@pytest.mark.parametrize("ci", range(7))
def test_shift_keys_golden_bit_exact(ci):
    G, M = gold(), meta()["cases"][f"shift{ci}"]
    dt = storage_dtype(G[f"shift{ci}_in"])
    keys = dev_tensor(values(G[f"shift{ci}_in"]), TORCH_DTYPE[dt])
    inv = workloads.inv_freq(M["d"], M["theta"])
    out = shift_keys(keys, M["delta"], inv)
    assert out.dtype == keys.dtype and out.shape == keys.shape
    assert exact(out, values(G[f"shift{ci}_out"]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_shift_keys_strided_view_matches_oracle(dtype):
    """A GrowingLayer-style view (head stride = cap*d) and the vector/scalar paths."""
    gen = torch.Generator(device=DEV).manual_seed(1)
    buf = torch.randn(1, 8, 500, 128, generator=gen, device=DEV).to(dtype)
    keys = buf[..., 100:433, :]
    inv = workloads.inv_freq()
    out = shift_keys(keys, -2048, inv)
    cs = ref_cos_sin(-2048, inv)
    name = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    assert exact(out, shift_keys_ref(keys.float().cpu().numpy(), dtype=name, cos_sin=cs))
    odd = torch.randn(2, 7, 130, generator=gen, device=DEV).to(dtype)[..., 1:129]  # unaligned rows
    out = shift_keys(odd, 77, inv)
    assert exact(out, shift_keys_ref(odd.float().cpu().numpy(), dtype=name, cos_sin=ref_cos_sin(77, inv)))


@pytest.mark.parametrize("d,theta", [(128, 1e6), (16, 1e4)])
def test_T1_shift_is_rotation_composition(d, theta):
    """The reference's T1 (tests/test_core.py:67-74): shifting a key rotated to 900 by -350 gives
    the key rotated to 550 (fp32, atol 1e-4)."""
    inv = workloads.inv_freq(d, theta)
    k = torch.randn(1, 2, 5, d)

    def rope_at(x, p):
        return workloads.rope_to_positions(x, torch.full((x.shape[-2],), p), inv)
    got = shift_keys(rope_at(k, 900).to(DEV), -350, inv).cpu()
    assert torch.allclose(got, rope_at(k, 550), atol=1e-4)


def test_cfg2_splice_then_decode_matches_reference():
    """Config 2: splice the pre-rotated 8192-token cache (Split(2048, 4096, 4096)) in place, then
    decode one query over the 6144 remaining tokens."""
    from threadcut_b200.flash_decode import decode_attention
    G, Mt = gold(), meta()
    kc, vc = workloads.cfg2_cache()
    assert [sha(kc), sha(vc)] == Mt["cfg2_sha_in"]
    ly = GrowingLayer()
    ly.update(kc[None].to(DEV), vc[None].to(DEV))
    ly.splice(Split(*workloads.CFG2_SPLIT), workloads.inv_freq())
    assert [sha(ly.keys[0]), sha(ly.values[0])] == Mt["cfg2_sha_spliced"]
    q = workloads.cfg2_query().to(DEV).reshape(8, 4, 128)
    out = decode_attention(q, ly.keys[0], ly.values[0], workloads.SCALE)
    assert np.abs(out.float().cpu().numpy().reshape(1, 1, 32, 128) - G["cfg2_out"]).max() <= 2e-3


@pytest.mark.parametrize("ci", range(9))
def test_growing_splice_golden(ci):
    G, M = gold(), meta()["cases"][f"grow{ci}"]
    dt = TORCH_DTYPE[M["dtype"]]
    inv = workloads.inv_freq(M["d"], M["theta"])
    ly = GrowingLayer()
    ly.update(dev_tensor(values(G[f"grow{ci}_k"]), dt), dev_tensor(values(G[f"grow{ci}_v"]), dt))
    ly.splice(Split(*M["split"]), inv)
    assert exact(ly.keys, values(G[f"grow{ci}_kout"]))
    assert exact(ly.values, values(G[f"grow{ci}_vout"]))


def test_copy_splice_golden():
    from transformers import DynamicCache, Qwen3Config
    G = gold()
    cache = DynamicCache(config=Qwen3Config(num_hidden_layers=1))
    cache.layers[0].update(torch.from_numpy(G["copy_k"]).to(DEV), torch.from_numpy(G["copy_v"]).to(DEV))
    splice(cache, Split(10, 17, 20), workloads.inv_freq(16, 1e4))
    assert exact(cache.layers[0].keys, G["copy_kout"]) and exact(cache.layers[0].values, G["copy_vout"])


SPLITS = [(0, 1, 4000), (10, 11, 3000), (5, 69, 2000), (100, 164, 1000), (3, 3000, 900), (0, 64, 64),
          (63, 127, 1800), (2048, 4096, 4096), (1, 4096, 4096), (700, 733, 2500)]


@pytest.mark.parametrize("a,c0,c", SPLITS)
def test_inplace_splice_overlap_sweep(a, c0, c):
    """Overlapping (gap < |C|, including gaps of 1 row, smaller than a unit, equal to a unit) and
    disjoint moves, bit-exact against the oracle, rows outside [a, a+c) untouched."""
    cap = c0 + c + 5
    gen = torch.Generator(device=DEV).manual_seed(a * 7 + c0)
    kb = torch.randn(1, 8, cap, 128, generator=gen, device=DEV).to(torch.bfloat16)
    vb = torch.randn(1, 8, cap, 128, generator=gen, device=DEV).to(torch.bfloat16)
    kref, vref, n = growing_splice_ref(kb[0].float().cpu().numpy(), vb[0].float().cpu().numpy(), a, c0, c,
                                       dtype="bf16", cos_sin=ref_cos_sin(-(c0 - a), workloads.inv_freq()))
    ly = GrowingLayer()
    ly.update(kb, vb)
    ly.splice(Split(a, c0, c), workloads.inv_freq())
    assert ly.get_seq_length() == n
    assert exact(ly.kbuf[0, :, :cap], kref) and exact(ly.vbuf[0, :, :cap], vref)


def test_all_layers_one_launch_equals_per_layer():
    """splice() over a 36-layer GrowingLayer cache (one launch) == splicing each layer alone."""
    from transformers import Qwen3Config
    cfg = Qwen3Config(num_hidden_layers=36, num_key_value_heads=8, head_dim=128)
    s = Split(300, 1000, 2500)
    inv = workloads.inv_freq()
    gen = torch.Generator(device=DEV).manual_seed(3)
    cache = new_cache(cfg)
    singles = []
    for layer in cache.layers:
        k = torch.randn(1, 8, 3600, 128, generator=gen, device=DEV).to(torch.bfloat16)
        v = torch.randn(1, 8, 3600, 128, generator=gen, device=DEV).to(torch.bfloat16)
        layer.update(k, v)
        one = GrowingLayer()
        one.update(k.clone(), v.clone())
        one.splice(s, inv)
        singles.append(one)
    splice(cache, s, inv)
    for layer, one in zip(cache.layers, singles):
        assert layer.get_seq_length() == s.a + s.c
        assert torch.equal(layer.keys, one.keys) and torch.equal(layer.values, one.values)
    # appending after a splice keeps working (reference test_growing_layer_splice_matches_copy_splice)
    cache.layers[0].update(torch.ones(1, 8, 3, 128, device=DEV, dtype=torch.bfloat16),
                           torch.ones(1, 8, 3, 128, device=DEV, dtype=torch.bfloat16))
    assert cache.layers[0].get_seq_length() == s.a + s.c + 3


def test_repeated_splices_reuse_the_workspace():
    """Tickets and flags are reset/epoch-stamped: many splices in a row stay exact."""
    gen = torch.Generator(device=DEV).manual_seed(4)
    kb = torch.randn(1, 8, 3000, 128, generator=gen, device=DEV).to(torch.bfloat16)
    vb = torch.randn(1, 8, 3000, 128, generator=gen, device=DEV).to(torch.bfloat16)
    kref, vref = kb[0].float().cpu().numpy(), vb[0].float().cpu().numpy()
    ly = GrowingLayer()
    ly.update(kb, vb)
    n = 3000
    inv = workloads.inv_freq()
    for i in range(12):
        a, gap = 50 + 13 * i, 7 + 29 * i
        c = n - a - gap
        kref, vref, n = growing_splice_ref(kref, vref, a, a + gap, c, dtype="bf16",
                                           cos_sin=ref_cos_sin(-gap, inv))
        ly.splice(Split(a, a + gap, c), inv)
    assert exact(ly.kbuf[0, :, :3000], kref) and exact(ly.vbuf[0, :, :3000], vref)


def test_splice_dtypes_and_head_dims():
    for dtype, name in ((torch.float16, "f16"), (torch.float32, "f32")):
        for d in (64, 128):
            gen = torch.Generator(device=DEV).manual_seed(d)
            inv = workloads.inv_freq(d, 1e4)
            kb = torch.randn(1, 4, 900, d, generator=gen, device=DEV).to(dtype)
            vb = torch.randn(1, 4, 900, d, generator=gen, device=DEV).to(dtype)
            kref, vref, n = growing_splice_ref(kb[0].float().cpu().numpy(), vb[0].float().cpu().numpy(), 20, 90,
                                               800, dtype=name, cos_sin=ref_cos_sin(-70, inv))
            ly = GrowingLayer()
            ly.update(kb, vb)
            ly.splice(Split(20, 90, 800), inv)
            assert exact(ly.kbuf[0, :, :900], kref) and exact(ly.vbuf[0, :, :900], vref)
