"""tcgen05 GQA prefill attention against the fp32 SDPA math with the causal-offset mask (needs a
B200). P enters the second MMA in 16 bits (as in flash attention), so the bar is 1e-2."""
import pytest
import torch
import torch.nn.functional as F

from threadcut_b200 import _lib
from threadcut_b200.prefill import causal_offset_mask, prefill_attention

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def reference(q, k, v, scale):
    hq, hkv = q.shape[1], k.shape[1]
    lq, lk = q.shape[2], k.shape[2]
    kk = k.float().repeat_interleave(hq // hkv, 1)
    vv = v.float().repeat_interleave(hq // hkv, 1)
    mask = causal_offset_mask(lq, lk, q.device)
    return F.scaled_dot_product_attention(q.float(), kk, vv, attn_mask=mask, scale=scale).transpose(1, 2)


@pytest.mark.parametrize("lq,lk", [(1, 1), (5, 5), (1, 300), (32, 32), (33, 100), (128, 128), (129, 700),
                                   (300, 1000), (512, 4096), (100, 5000)])
@pytest.mark.parametrize("hkv", [8, 2])
def test_prefill_matches_sdpa(lq, lk, hkv):
    g = torch.Generator(device=DEV).manual_seed(lq * 7 + lk + hkv)
    q = torch.randn(1, 4 * hkv, lq, 128, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(1, hkv, lk, 128, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(1, hkv, lk, 128, generator=g, device=DEV).to(torch.bfloat16)
    out = prefill_attention(q, k, v, 0.0883)
    torch.cuda.synchronize()
    ref = reference(q, k, v, 0.0883)
    err = (out.float() - ref).abs().max().item()
    assert out.shape == (1, lq, 4 * hkv, 128) and err <= 1e-2, (lq, lk, hkv, err)
    assert _lib.device_errors(clear=True) == 0


def test_prefill_fp16_strided_and_peaked():
    g = torch.Generator(device=DEV).manual_seed(3)
    # HF layout: query [1, hq, lq, d] as a transposed view of [1, lq, hq, d]
    q = torch.randn(1, 200, 32, 128, generator=g, device=DEV).to(torch.float16).transpose(1, 2)
    kb = torch.randn(1, 8, 1000, 128, generator=g, device=DEV).to(torch.float16)
    k, v = kb[:, :, :900], kb[:, :, 100:]  # cache views with a head stride larger than the length
    out = prefill_attention(q, k, v, 0.5)  # large scale: peaked softmax, exercises the O rescale
    ref = reference(q, k, v, 0.5)
    assert (out.float() - ref).abs().max().item() <= 1e-2
    assert _lib.device_errors(clear=True) == 0


def test_prefill_rejects_unsupported_shapes():
    q = torch.randn(1, 32, 4, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        prefill_attention(q, q[:, :8], q[:, :8], 0.1)


def test_plugin_prefill_branch_uses_the_kernel_for_causal_masks():
    """The plugin's prefill branch: the HF causal-over-cache mask and the plain causal case (no mask,
    lq == lk) take the tcgen05 kernel; any other mask keeps SDPA; both agree with the reference."""
    from threadcut_b200 import attention as plug
    g = torch.Generator(device=DEV).manual_seed(9)
    q = torch.randn(1, 32, 64, 128, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(1, 8, 640, 128, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(1, 8, 640, 128, generator=g, device=DEV).to(torch.bfloat16)
    mask = causal_offset_mask(64, 640, q.device)[None, None]
    assert plug._is_causal_offset(mask, 64, 640) and plug._is_causal_offset(mask, 64, 640)  # second: cached
    out, _ = plug.attention(None, q, k, v, mask, scaling=0.0883)
    assert torch.equal(out, prefill_attention(q, k, v, 0.0883))
    assert (out.float() - reference(q, k, v, 0.0883)).abs().max().item() <= 1e-2
    other = mask.clone()
    other[..., 0] = False  # not the causal-offset pattern: SDPA path
    assert not plug._is_causal_offset(other, 64, 640)
    out2, _ = plug.attention(None, q, k, v, other, scaling=0.0883)
    assert out2.shape == out.shape
    qc = q[:, :, :, :]
    kc, vc = k[:, :, :64], v[:, :, :64]
    out3, _ = plug.attention(None, qc, kc, vc, None, scaling=0.0883)  # plain causal, lq == lk
    assert (out3.float() - reference(qc, kc, vc, 0.0883)).abs().max().item() <= 1e-2


@pytest.mark.parametrize("lq,lk", [(32, 4096), (100, 5000), (512, 20000), (7, 300), (64, 164), (200, 1350)])
@pytest.mark.parametrize("splits", [1, 2, 3, 7, 16])
def test_prefill_kv_splits_merge(lq, lk, splits):
    """KV-split prefill: fp32 partials merged by log-sum-exp agree with the reference for every split
    count, including splits that get no visible key for some rows or no tile at all."""
    g = torch.Generator(device=DEV).manual_seed(lq + lk + splits)
    q = torch.randn(1, 32, lq, 128, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(1, 8, lk, 128, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(1, 8, lk, 128, generator=g, device=DEV).to(torch.bfloat16)
    out = prefill_attention(q, k, v, 0.0883, splits=splits)
    assert torch.isfinite(out).all()
    assert (out.float() - reference(q, k, v, 0.0883)).abs().max().item() <= 1e-2, (lq, lk, splits)
    assert _lib.device_errors(clear=True) == 0
