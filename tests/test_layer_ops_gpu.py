"""The tensor-parallel step's fused layer ops (csrc/layer_ops.cuh) against the torch ops of
transformers' Qwen3 layer they replace (modeling_qwen3: Qwen3RMSNorm, q_norm/k_norm +
apply_rotary_pos_emb, act_fn(gate) * up), on the same bf16 inputs.

The sum of squares is reduced in a different order than torch's mean, so an element may round to
the neighbouring bf16 value: the bar is two bf16 ulps, and nearly all elements bit-identical."""
import pytest
import torch
import torch.nn.functional as F
from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb

from threadcut_b200 import _lib, tp
from threadcut_b200 import flash_decode as fd

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    _lib.device_errors(clear=True)
    yield
    assert _lib.device_errors(clear=True) == 0


def close_bf16(got, want, min_equal=0.98, row_scale=False):
    """Within two bf16 ulps of each element (of the row's largest element when row_scale: RoPE's
    sum can cancel, and a one-ulp change of a term is then large next to the result), and at least
    `min_equal` of the elements bit-identical."""
    got, want = got.float(), want.float()
    mag = want.abs().amax(-1, keepdim=True) if row_scale else want.abs()
    tol = torch.clamp(mag, min=2 ** -120) * 2 ** -6
    assert bool(((got - want).abs() <= tol).all()), float((got - want).abs().max())
    assert float((got == want).float().mean()) >= min_equal


@pytest.mark.parametrize("hidden,rows", [(2560, 1), (256, 3), (100, 2)])
@pytest.mark.parametrize("add", [False, True])
def test_add_rmsnorm_matches_residual_add_and_qwen3_rmsnorm(hidden, rows, add):
    g = torch.Generator(device=DEV).manual_seed(hidden + rows)
    h = torch.randn(rows, hidden, generator=g, device=DEV).to(torch.bfloat16)
    delta = torch.randn(rows, hidden, generator=g, device=DEV).to(torch.bfloat16) if add else None
    norm = Qwen3RMSNorm(hidden, eps=1e-6).to(DEV).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(hidden, generator=g, device=DEV))
        want_h = h + delta if add else h.clone()
        want = norm(want_h)
    out = torch.empty_like(h)
    tp._add_rmsnorm(h, delta, norm.weight.detach(), out, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(h, want_h)  # the residual add rounds exactly as torch's
    close_bf16(out, want)


@pytest.mark.parametrize("nq,nk,pos", [(32, 8, 98304), (4, 1, 7), (8, 2, 0)])
def test_qk_norm_rope_matches_qwen3_attention_prologue(nq, nk, pos):
    d = 128
    g = torch.Generator(device=DEV).manual_seed(nq * 7 + pos)
    q = torch.randn(nq, d, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(nk, d, generator=g, device=DEV).to(torch.bfloat16)
    qn, kn = Qwen3RMSNorm(d, 1e-6).to(DEV).to(torch.bfloat16), Qwen3RMSNorm(d, 1e-6).to(DEV).to(torch.bfloat16)
    with torch.no_grad():
        qn.weight.copy_(1 + 0.1 * torch.randn(d, generator=g, device=DEV))
        kn.weight.copy_(1 + 0.1 * torch.randn(d, generator=g, device=DEV))
        inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device=DEV).float() / d))
        ang = pos * inv
        emb = torch.cat((ang, ang))
        cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
        wq, wk = apply_rotary_pos_emb(qn(q)[None, :, None], kn(k)[None, :, None], cos[None, None], sin[None, None])
    q2, k2 = q.clone(), k.clone()
    tp._qk_norm_rope(q2, k2, qn.weight.detach(), kn.weight.detach(), cos, sin, 1e-6)
    torch.cuda.synchronize()
    close_bf16(q2, wq[0, :, 0], row_scale=True)
    close_bf16(k2, wk[0, :, 0], row_scale=True)


@pytest.mark.parametrize("inter,rows", [(9728, 1), (1216, 1), (33, 3)])
def test_silu_mul_matches_qwen3_mlp_activation(inter, rows):
    g = torch.Generator(device=DEV).manual_seed(inter)
    gu = (3 * torch.randn(rows, 2 * inter, generator=g, device=DEV)).to(torch.bfloat16)
    want = F.silu(gu[:, :inter]) * gu[:, inter:]
    out = torch.empty(rows, inter, device=DEV, dtype=torch.bfloat16)
    tp._silu_mul(gu, out)
    torch.cuda.synchronize()
    close_bf16(out, want, min_equal=0.99)


@pytest.mark.parametrize("n,k,dtype", [(6144, 2560, torch.bfloat16), (2560, 4096, torch.bfloat16),
                                       (2560, 9728, torch.bfloat16), (19456, 2560, torch.bfloat16),
                                       (18992, 2560, torch.bfloat16), (7, 16, torch.bfloat16),
                                       (1000, 1216, torch.float16)])
def test_gemv_matches_the_library_projection(n, k, dtype):
    """tc_gemv against nn.Linear's matmul (cuBLAS) on the same 16-bit operands: both accumulate in
    fp32 and round once, in different orders, so results agree to a rounding step."""
    g = torch.Generator(device=DEV).manual_seed(n + k)
    x = torch.randn(1, k, generator=g, device=DEV).to(dtype)
    w = (torch.randn(n, k, generator=g, device=DEV) * k ** -0.5).to(dtype)
    got = tp._gemv(x, w)
    want = x @ w.t()
    exact = (x.float() @ w.float().t())
    torch.cuda.synchronize()
    assert got.shape == (1, n) and got.dtype == dtype
    torch.testing.assert_close(got.float(), want.float(), rtol=2 ** -6, atol=1e-3)
    torch.testing.assert_close(got.float(), exact, rtol=2 ** -7, atol=1e-3)
    assert float((got == want).float().mean()) >= 0.8


@pytest.mark.parametrize("n,k,dtype", [(2560, 9728, torch.bfloat16), (2560, 1216, torch.bfloat16),
                                       (300, 64, torch.float16)])
def test_gemv_swiglu_equals_silu_mul_then_gemv(n, k, dtype):
    """tc_gemv_swiglu computes the SwiGLU activation while staging its input: the same bits as
    tc_silu_mul followed by tc_gemv (same rounding of the activation, same accumulation order)."""
    g = torch.Generator(device=DEV).manual_seed(n * 7 + k)
    gu = (torch.randn(1, 2 * k, generator=g, device=DEV) * 2).to(dtype)
    w = (torch.randn(n, k, generator=g, device=DEV) * k ** -0.5).to(dtype)
    act = gu.new_empty((1, k))
    tp._silu_mul(gu, act)
    want = tp._gemv(act, w)
    got = tp._gemv_swiglu(gu, w)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    ref = (F.silu(gu[:, :k].float()).to(dtype).float() * gu[:, k:].float()).to(dtype).float() @ w.float().t()
    torch.testing.assert_close(got.float(), ref, rtol=2 ** -7, atol=1e-3)


@pytest.mark.parametrize("hkv,g,d,n,dtype", [(1, 4, 128, 98305, torch.bfloat16), (8, 4, 128, 2049, torch.bfloat16),
                                             (2, 4, 128, 40, torch.float16), (2, 8, 64, 777, torch.bfloat16),
                                             (1, 2, 256, 300, torch.float16)])
def test_attention_with_norm_rope_equals_separate_launches(hkv, g, d, n, dtype):
    """tc_decode_attention_append_rope (q/k norm + RoPE inside the attention launch) gives the bits
    of tc_qk_norm_rope followed by tc_decode_attention_append: the same output, the same rotated row
    n-1 in the cache, and every other cache row untouched; and the rotated q/k it uses are within
    the Qwen3 prologue's tolerance of the torch ops (checked above for the separate launch)."""
    gen = torch.Generator(device=DEV).manual_seed(hkv * 1000 + n)
    k = torch.randn(hkv, n, d, generator=gen, device=DEV).to(dtype)
    v = torch.randn(hkv, n, d, generator=gen, device=DEV).to(dtype)
    q = torch.randn(hkv, g, d, generator=gen, device=DEV).to(dtype)
    kn = torch.randn(hkv, d, generator=gen, device=DEV).to(dtype)
    vn = torch.randn(hkv, d, generator=gen, device=DEV).to(dtype)
    wq = (1 + 0.1 * torch.randn(d, generator=gen, device=DEV)).to(dtype)
    wk = (1 + 0.1 * torch.randn(d, generator=gen, device=DEV)).to(dtype)
    ang = (n - 1) * (1.0 / (1e6 ** (torch.arange(0, d, 2, device=DEV).float() / d)))
    emb = torch.cat((ang, ang))
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    scale = d ** -0.5
    # separate launches
    q1, k1 = q.clone(), kn.clone()
    tp._qk_norm_rope(q1.view(hkv * g, d), k1, wq, wk, cos, sin, 1e-6)
    ka, va = k.clone(), v.clone()
    want = fd.decode_attention_append(q1, ka, va, k1, vn, scale)
    # one launch
    kb, vb = k.clone(), v.clone()
    q0, kn0 = q.clone(), kn.clone()
    got = fd.decode_attention_append_rope(q, kb, vb, kn, vn, wq, wk, cos, sin, 1e-6, scale)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(kb, ka) and torch.equal(vb, va)
    assert torch.equal(kb[:, :n - 1], k[:, :n - 1]) and torch.equal(kb[:, n - 1], k1)
    assert torch.equal(q, q0) and torch.equal(kn, kn0)  # the raw projections are only read


def test_attention_with_norm_rope_rejects_what_it_cannot_fuse():
    q = torch.randn(1, 4, 128, device=DEV)
    k = torch.randn(1, 8, 128, device=DEV)
    row = torch.randn(1, 128, device=DEV)
    w = torch.ones(128, device=DEV)
    with pytest.raises(RuntimeError):  # fp32: the tensor-core kernel does not take it
        fd.decode_attention_append_rope(q, k, k.clone(), row, row, w, w, w, w, 1e-6, 0.1)
    qb, kb, rb, wb = (t.to(torch.bfloat16) for t in (q, k, row, w))
    with pytest.raises(ValueError):
        fd.decode_attention_append_rope(qb, kb, kb.clone(), rb, rb, wb[:64], wb, wb, wb, 1e-6, 0.1)


@pytest.mark.parametrize("hidden,k,n,swiglu", [(2560, 4096, 19456, False), (2560, 9728, 6144, True),
                                               (256, 512, 300, False), (2048, 64, 24, True)])
def test_residual_sum_and_norm_staging_equal_the_separate_launches(hidden, k, n, swiglu):
    """World 1 of the residual-form sums (peer.AllReduce.gemv_residual, then gemv_norm): h after the
    projection has exactly the bits of tc_gemv (or tc_gemv_swiglu) followed by tc_add_rmsnorm's
    residual add, and the next projection of RMSNorm(h) equals tc_add_rmsnorm + tc_gemv within one
    rounding step (its 1/rms adds the squares in another order), nearly all bit-identical. Several
    rounds in a row, so the recorded sums of squares are always the last residual sum's."""
    from threadcut_b200.peer import AllReduce
    dt = torch.bfloat16
    gen = torch.Generator(device=DEV).manual_seed(hidden + k + n)
    ar = AllReduce(hidden, DEV, world=1)
    try:
        h_a = torch.randn(1, hidden, generator=gen, device=DEV).to(dt)
        h_b = h_a.clone()
        nw = (1 + 0.1 * torch.randn(hidden, generator=gen, device=DEV)).to(dt)
        for rnd in range(3):
            x = (torch.randn(1, 2 * k if swiglu else k, generator=gen, device=DEV) * (1 + rnd)).to(dt)
            w = (torch.randn(hidden, k, generator=gen, device=DEV) * k ** -0.5).to(dt)
            w2 = (torch.randn(n, hidden, generator=gen, device=DEV) * hidden ** -0.5).to(dt)
            # separate launches
            part = tp._gemv_swiglu(x, w) if swiglu else tp._gemv(x, w)
            xn = torch.empty_like(h_a)
            tp._add_rmsnorm(h_a, part, nw, xn, 1e-6)
            want = tp._gemv(xn, w2)
            # residual form
            ar.gemv_residual(x[0], w, h_b, swiglu=swiglu)
            got = ar.gemv_norm(h_b, nw, w2, 1e-6)
            torch.cuda.synchronize()
            assert torch.equal(h_b, h_a), rnd
            diff = (got.float() - want.float()).abs()
            assert bool((diff <= 2 ** -6 * want.float().abs().clamp(min=1.0)).all()), (rnd, float(diff.max()))
            assert float((got == want).float().mean()) >= 0.9, rnd
    finally:
        torch.cuda.synchronize()
        ar.close()


@pytest.mark.parametrize("hidden,inter", [(2560, 9728), (2560, 1216), (256, 304), (2048, 8)])
def test_gate_up_with_swiglu_epilogue_equals_projection_then_silu_mul(hidden, inter):
    """peer.AllReduce.gemv_norm_swiglu (tc_gemv_rmsnorm_swiglu: the gate/up projection of RMSNorm(h)
    with interleaved rows, writing silu(gate) * up from its epilogue) against gemv_norm of the same
    rows as [gate | up] followed by tc_silu_mul: bit for bit, after a residual sum as in the step.
    The down projection of that activation (plain input) equals the SwiGLU-staging down projection
    bit for bit too. Three rounds in a row."""
    from threadcut_b200.peer import AllReduce
    dt = torch.bfloat16
    gen = torch.Generator(device=DEV).manual_seed(hidden + inter)
    ar = AllReduce(hidden, DEV, world=1)
    try:
        h = torch.randn(1, hidden, generator=gen, device=DEV).to(dt)
        nw = (1 + 0.1 * torch.randn(hidden, generator=gen, device=DEV)).to(dt)
        for rnd in range(3):
            o = (torch.randn(1, 512, generator=gen, device=DEV) * (1 + rnd)).to(dt)
            wo = (torch.randn(hidden, 512, generator=gen, device=DEV) * 512 ** -0.5).to(dt)
            gate = (torch.randn(inter, hidden, generator=gen, device=DEV) * hidden ** -0.5).to(dt)
            up = (torch.randn(inter, hidden, generator=gen, device=DEV) * hidden ** -0.5).to(dt)
            wd = (torch.randn(hidden, inter, generator=gen, device=DEV) * inter ** -0.5).to(dt)
            ar.gemv_residual(o[0], wo, h)
            gu = ar.gemv_norm(h, nw, torch.cat((gate, up)), 1e-6)
            want = torch.empty(1, inter, dtype=dt, device=DEV)
            tp._silu_mul(gu, want)
            inter_rows = torch.stack((gate, up), dim=1).reshape(2 * inter, hidden).contiguous()
            got = ar.gemv_norm_swiglu(h, nw, inter_rows, 1e-6)
            torch.cuda.synchronize()
            assert torch.equal(got, want), (rnd, float((got.float() - want.float()).abs().max()))
            h_a, h_b = h.clone(), h.clone()
            ar.gemv_residual(gu[0], wd, h_a, swiglu=True)
            ar.gemv_residual(got[0], wd, h_b)
            torch.cuda.synchronize()
            assert torch.equal(h_a, h_b), rnd
            h = h_b
    finally:
        torch.cuda.synchronize()
        ar.close()
