"""Seeded synthetic inputs for the BASELINE configurations of threadcut's decode hot path.

There are no datasets or checkpoints on this path: every input is N(0,1) data from a seeded torch
CPU generator (deterministic for the pinned torch build), with the shapes of Qwen3-4B
(32 query / 8 KV heads, head_dim 128, 36 layers, RoPE theta 1e6). Used by bench.py, the tests,
__graft_entry__.smoke() and tests/golden/make_golden.py, so all of them see identical inputs.

  cfg1   single layer: q [1,32,1,128], K/V [1,8,1536,128]
  cfg2   8192-token cache, keys pre-rotated at positions 0..8191; Split(2048, 4096, 4096) then
         decode one query [32,128] over the 6144 remaining tokens
  cfg3   36 layers, n in {4096, 16384, 32768} (the bench's 16k headline is n = 16384)
  cfg4   64 ragged sequences, lengths ~ U[1024, 16384] (inclusive) from Generator().manual_seed(0)
  cfg5   Qwen3-4B random init, 128k context, span [49152, 81920) pruned, suffix shifted by -32768
"""
import torch

HQ, HKV, D, LAYERS, THETA = 32, 8, 128, 36, 1.0e6
G = HQ // HKV
SCALE = D ** -0.5

CFG2_N, CFG2_SPLIT = 8192, (2048, 4096, 4096)  # (a, c0, c)
CFG4_BATCH, CFG4_LO, CFG4_HI = 64, 1024, 16384
CFG5_CTX, CFG5_PRUNE = 131072, (49152, 81920)


def qwen3_4b_config(layers=LAYERS):
    """Qwen3-4B geometry (hidden 2560, 36 layers, 32/8 heads, head_dim 128, RoPE theta 1e6) for the
    random-init config-5 model; intermediate 9728, vocab 151936, tied embeddings and eps 1e-6 are the
    published values, and 262144 positions make 128k contexts legal."""
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=151936, hidden_size=2560, intermediate_size=9728, num_hidden_layers=layers,
                       num_attention_heads=HQ, num_key_value_heads=HKV, head_dim=D, rms_norm_eps=1e-6,
                       tie_word_embeddings=True, max_position_embeddings=262144,
                       rope_parameters={"rope_type": "default", "rope_theta": THETA})


def inv_freq(d=D, theta=THETA):
    """Default RoPE frequencies (transformers' rotary init): 1 / theta^(2i/d), fp32 [d/2]."""
    return 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))


def rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope_to_positions(k, positions, freqs):
    """Rotate raw keys k [..., n, d] (fp32) to absolute positions [n]: the reference's shift formula
    (threadcut/kv.py:22-25) with delta = position, in fp32."""
    angle = positions.float()[:, None] * freqs.float()[None, :]
    emb = torch.cat((angle, angle), dim=-1)
    return k * emb.cos() + rotate_half(k) * emb.sin()


def cfg1(seed=0, n=1536):
    """q [1,32,1,128], k/v [1,8,n,128] fp32 N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, HQ, 1, D, generator=g)
    k = torch.randn(1, HKV, n, D, generator=g)
    v = torch.randn(1, HKV, n, D, generator=g)
    return q, k, v


def cfg2_cache(seed=0, n=CFG2_N, dtype=torch.bfloat16):
    """K [8, n, 128] pre-rotated to positions 0..n-1 and V [8, n, 128], both cast to `dtype`."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(HKV, n, D, generator=g)
    v = torch.randn(HKV, n, D, generator=g)
    k = rope_to_positions(k, torch.arange(n), inv_freq())
    return k.to(dtype), v.to(dtype)


def cfg2_query(seed=1, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(HQ, D, generator=g).to(dtype)


def cfg4_lengths(seed=0, batch=CFG4_BATCH, lo=CFG4_LO, hi=CFG4_HI):
    return torch.randint(lo, hi + 1, (batch,), generator=torch.Generator().manual_seed(seed)).tolist()


def layer_kv(n, layers, device, dtype=torch.bfloat16, seed=0, cap=None, heads=HKV):
    """`layers` distinct K/V buffers [heads, cap, 128] (cap >= n, default n) of N(0,1) data drawn on
    the device (Philox, deterministic for a seed), as GrowingLayer-style views [heads, n, 128]."""
    cap = n if cap is None else cap
    g = torch.Generator(device=device).manual_seed(seed)
    ks, vs = [], []
    for _ in range(layers):
        kb = torch.randn(heads, cap, D, generator=g, device=device, dtype=torch.float32).to(dtype)
        vb = torch.randn(heads, cap, D, generator=g, device=device, dtype=torch.float32).to(dtype)
        ks.append(kb[:, :n])
        vs.append(vb[:, :n])
    return ks, vs
