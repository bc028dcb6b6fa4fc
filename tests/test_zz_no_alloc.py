"""tc_decode_attention_noalloc: decode attention for callers that cannot allocate device memory.

Some callers cannot give the library a workspace: a plugin inside another runtime that owns all
device memory and forbids allocating while it executes, a loop that cannot afford cudaMalloc's
implicit synchronisation, or C code with no allocator at hand. For them the library keeps its
scratch in one fixed array of its own. These checks call that entry point through the C ABI and
compare it with tc_decode_attention (the workspace-taking entry point, reached through
threadcut_b200.flash_decode) and with the CPU oracle of the reference's decode math on two calls in
a row with different problem sizes, so a stale workspace state from the first call would show up
in the second.

This file is collected last on purpose; it needs no state from the other tests.
"""
import numpy as np
import pytest
import torch

from helpers import ATTN_ATOL, attn_error
from oracle.attention import decode_attention_ref
from threadcut_b200 import _lib
from threadcut_b200.flash_decode import decode_attention

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def call_noalloc(q, k, v, scale, splits=0):
    out = torch.empty_like(q)
    st = _lib.lib().tc_decode_attention_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), q.shape[0], q.shape[1], q.shape[2], k.shape[1],
        q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1), out.stride(0), out.stride(1),
        float(scale), splits, _lib.DTYPE_CODE[q.dtype], torch.cuda.current_stream().cuda_stream)
    return st, out


def make(n, cap, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(8, 4, 128, generator=g, device=DEV).to(torch.bfloat16)
    kb = torch.randn(8, cap, 128, generator=g, device=DEV).to(torch.bfloat16)  # GrowingLayer-style buffers
    vb = torch.randn(8, cap, 128, generator=g, device=DEV).to(torch.bfloat16)
    return q, kb[:, :n], vb[:, :n]


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    torch.cuda.set_device(DEV)
    scale = 128 ** -0.5
    for n, cap, seed in ((5000, 5100, 1), (1300, 2048, 2)):
        q, k, v = make(n, cap, seed)
        st, out = call_noalloc(q, k, v, scale)
        assert st == 0, _lib.lib().tc_status_string(st)
        ref = decode_attention(q, k, v, scale)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        err = attn_error(got, ref.float().cpu().numpy(), torch.bfloat16)
        assert err <= ATTN_ATOL, (n, err)
        math = decode_attention_ref(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), scale)
        err = attn_error(got, math, torch.bfloat16)
        assert err <= ATTN_ATOL, (n, err)
        assert np.isfinite(got).all()


def test_noalloc_rejects_problems_larger_than_its_array():
    """16 query heads of head_dim 256 over 8 KV heads, forced to 128 slices, needs 16 MiB of
    partials: more than the fixed 4 MiB, so the call must refuse before launching anything."""
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(8, 16, 256, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(8, 4096, 256, generator=g, device=DEV).to(torch.bfloat16)
    st, _ = call_noalloc(q, k, k, 0.0625, splits=128)
    assert st == 4  # TC_ERR_WORKSPACE
