"""Generate the golden vectors in tests/golden/ by running the REFERENCE implementation.

Run in the build container, where the reference is mounted (it is absent on the GPU box; the
committed .npz/.json are what travels):

    python tests/golden/make_golden.py --reference <reference checkout>

(or set THREADCUT_REFERENCE to the checkout instead of passing --reference).

It imports threadcut.attention / threadcut.kv / threadcut.match from the reference checkout and
records their outputs on the CPU (the decode branch there is the folded SDPA of
threadcut/attention.py:41-42, fp32 math). Inputs come from ../../workloads.py (seeded torch CPU
generators) or are stored in the fixture when small; large inputs are pinned by a SHA-256 of their
bytes so a drifting generator is detected instead of silently compared.
"""
import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
import workloads  # noqa: E402


def sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16
                          else t.contiguous().numpy().tobytes()).hexdigest()


def bits(t):
    """bf16 tensor -> uint16 numpy bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def store(t):
    """Compact exact storage: bf16 as uint16 bits, fp16 as float16, fp32 as float32."""
    if t.dtype == torch.bfloat16:
        return bits(t)
    return t.contiguous().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("THREADCUT_REFERENCE"),
                    help="path of the reference checkout (the directory holding threadcut/)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or THREADCUT_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    from threadcut import attention as ref_attn  # noqa: E402
    from threadcut import kv as ref_kv  # noqa: E402
    from threadcut import match as ref_match  # noqa: E402
    from transformers import DynamicCache, Qwen3Config  # noqa: E402

    torch.set_num_threads(8)
    out = {}
    meta = {"reference": "threadcut (reference checkout, no commit hash)", "torch": torch.__version__,
            "cases": {}}

    def ref_decode(q, k, v, scale):
        """reference plugin on CPU -> folded SDPA branch; q [1,Hq,1,d], k/v [1,Hkv,n,d] fp32."""
        o, _ = ref_attn.attention(None, q, k, v, None, scaling=scale)
        return o  # [1, 1, Hq, d]

    # 1) small decode cases, bf16-representable inputs stored as bf16 bits
    g = torch.Generator().manual_seed(1234)
    small = [(2, 2, 16, 1), (2, 2, 16, 7), (8, 4, 128, 1), (8, 4, 128, 33), (2, 4, 128, 300),
             (4, 8, 64, 100), (2, 16, 32, 65), (1, 1, 128, 5), (2, 4, 256, 70), (3, 3, 64, 257)]
    for ci, (hkv, gg, d, n) in enumerate(small):
        q = torch.randn(1, hkv * gg, 1, d, generator=g).to(torch.bfloat16)
        k = torch.randn(1, hkv, n, d, generator=g).to(torch.bfloat16)
        v = torch.randn(1, hkv, n, d, generator=g).to(torch.bfloat16)
        scale = d ** -0.5
        o = ref_decode(q.float(), k.float(), v.float(), scale)
        key = f"dec{ci}"
        out[f"{key}_q"], out[f"{key}_k"], out[f"{key}_v"] = bits(q), bits(k), bits(v)
        out[f"{key}_out"] = o.numpy()
        meta["cases"][key] = {"hkv": hkv, "g": gg, "d": d, "n": n, "scale": scale}

    # 2) config 1 (fp32 inputs from the seed) and its bf16-input variant; 3) the 16k single layer
    q, k, v = workloads.cfg1()
    meta["cfg1_sha"] = [sha(q), sha(k), sha(v)]
    out["cfg1_out_f32"] = ref_decode(q, k, v, workloads.SCALE).numpy()
    qb, kb, vb = (t.to(torch.bfloat16).float() for t in (q, k, v))
    out["cfg1_out_bf16in"] = ref_decode(qb, kb, vb, workloads.SCALE).numpy()
    q, k, v = workloads.cfg1(n=16384)
    meta["cfg16k_sha"] = [sha(q), sha(k), sha(v)]
    qb, kb, vb = (t.to(torch.bfloat16).float() for t in (q, k, v))
    out["cfg16k_out_bf16in"] = ref_decode(qb, kb, vb, workloads.SCALE).numpy()

    # 4) shift_keys: bf16 / fp16 / fp32 keys, several deltas; the reference's own cos/sin table
    inv128 = workloads.inv_freq(128, 1e6)
    inv16 = workloads.inv_freq(16, 1e4)
    gk = torch.Generator().manual_seed(99)
    shift_cases = [("bf16", torch.bfloat16, 128, inv128, (2, 64), -350),
                   ("bf16", torch.bfloat16, 128, inv128, (2, 64), -2048),
                   ("bf16", torch.bfloat16, 128, inv128, (3, 9), 7),
                   ("bf16", torch.bfloat16, 128, inv128, (1, 33), -32768),
                   ("f16", torch.float16, 128, inv128, (2, 17), -1),
                   ("f32", torch.float32, 16, inv16, (2, 5), -350),
                   ("f32", torch.float32, 128, inv128, (2, 40), 12345)]
    for ci, (name, dt, d, inv, (h, n), delta) in enumerate(shift_cases):
        keys = torch.randn(1, h, n, d, generator=gk).to(dt)
        res = ref_kv.shift_keys(keys, delta, inv)
        angle = delta * inv.float()
        emb = torch.cat((angle, angle))
        key = f"shift{ci}"
        out[f"{key}_in"], out[f"{key}_out"] = store(keys), store(res)
        out[f"{key}_cos"] = emb.cos()[: d // 2].numpy()
        out[f"{key}_sin"] = emb.sin()[: d // 2].numpy()
        meta["cases"][key] = {"dtype": name, "d": d, "delta": delta, "theta": 1e6 if d == 128 else 1e4}

    # 5) config 2: splice the pre-rotated 8192-token cache, then decode one query over 6144 tokens
    kc, vc = workloads.cfg2_cache()
    a, c0, c = workloads.CFG2_SPLIT
    meta["cfg2_sha_in"] = [sha(kc), sha(vc)]
    layer = ref_kv.GrowingLayer()
    layer.update(kc[None].clone(), vc[None].clone())
    layer.splice(ref_match.Split(a, c0, c), inv128)
    ks, vs = layer.keys[0], layer.values[0]
    meta["cfg2_sha_spliced"] = [sha(ks), sha(vs)]
    rows = torch.tensor([0, 1, a - 1, a, a + 1, a + 777, a + c - 1])
    out["cfg2_rows"] = rows.numpy()
    out["cfg2_k_rows"] = bits(ks[:, rows])
    qd = workloads.cfg2_query()
    meta["cfg2_sha_q"] = sha(qd)
    out["cfg2_out"] = ref_decode(qd.float().reshape(1, 32, 1, 128), ks.float()[None], vs.float()[None],
                                 workloads.SCALE).numpy()

    # 6) GrowingLayer in-place splice, small buffers (fp32 and bf16)
    gs = torch.Generator().manual_seed(7)
    grow_cases = [((2, 40, 16), torch.float32, inv16, (10, 17, 20)), ((2, 40, 16), torch.float32, inv16, (12, 12, 0)),
                  ((2, 40, 16), torch.float32, inv16, (3, 5, 30)), ((2, 40, 16), torch.float32, inv16, (0, 8, 32)),
                  ((2, 40, 16), torch.float32, inv16, (5, 30, 10)), ((2, 40, 16), torch.float32, inv16, (4, 4, 30)),
                  ((2, 300, 128), torch.bfloat16, inv128, (37, 100, 200)),
                  ((2, 300, 128), torch.bfloat16, inv128, (0, 1, 299)),
                  ((2, 300, 128), torch.bfloat16, inv128, (64, 200, 100))]
    for ci, ((h, n, d), dt, inv, (a_, c0_, c_)) in enumerate(grow_cases):
        kk = torch.randn(1, h, n, d, generator=gs).to(dt)
        vv = torch.randn(1, h, n, d, generator=gs).to(dt)
        ly = ref_kv.GrowingLayer()
        ly.update(kk.clone(), vv.clone())
        ly.splice(ref_match.Split(a_, c0_, c_), inv)
        key = f"grow{ci}"
        out[f"{key}_k"], out[f"{key}_v"] = store(kk), store(vv)
        out[f"{key}_kout"], out[f"{key}_vout"] = store(ly.keys), store(ly.values)
        meta["cases"][key] = {"split": [a_, c0_, c_], "d": d, "dtype": "f32" if dt == torch.float32 else "bf16",
                              "theta": 1e4 if d == 16 else 1e6}

    # 7) copy splice path (plain DynamicCache)
    kk = torch.randn(1, 2, 40, 16, generator=gs)
    vv = torch.randn(1, 2, 40, 16, generator=gs)
    cache = DynamicCache(config=Qwen3Config(num_hidden_layers=1))
    cache.layers[0].update(kk.clone(), vv.clone())
    ref_kv.splice(cache, ref_match.Split(10, 17, 20), inv16)
    out["copy_k"], out["copy_v"] = kk.numpy(), vv.numpy()
    out["copy_kout"], out["copy_vout"] = cache.layers[0].keys.numpy(), cache.layers[0].values.numpy()

    # 8) ragged decode: independent sequences through the reference plugin one at a time
    lengths = [1, 17, 300, 64, 129]
    for bi, n in enumerate(lengths):
        q = torch.randn(1, 8, 1, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16)
        v = torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16)
        out[f"rag{bi}_q"], out[f"rag{bi}_k"], out[f"rag{bi}_v"] = bits(q), bits(k), bits(v)
        out[f"rag{bi}_out"] = ref_decode(q.float(), k.float(), v.float(), workloads.SCALE).numpy()
    meta["ragged_lengths"] = lengths

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)

    # 9) split(): the reference's own rule cases plus seeded synthetic A.B.C / A.C.D requests
    cases = []
    A, B, C, D = [1, 2, 3], [7, 7], [4, 5, 6, 8, 9], [10, 11]
    for cached, new, ms, suf in [(A + B + C, A + C + D, 3, True), (A + B + C, A + C + D, 3, False),
                                 (A + C, A + C + D, 3, True), (A + C, A + C, 3, True), ([], [5, 6], 3, True),
                                 ([1], [1], 1, True), (A + B + C + [99, 98], A + C + D, 2, True)]:
        s = ref_match.split(cached, new, min_suffix=ms, suffix=suf)
        cases.append({"cached": cached, "new": new, "min_suffix": ms, "suffix": suf, "expect": [s.a, s.c0, s.c]})
    rng = np.random.default_rng(5)
    for _ in range(200):
        la, lb, lc, ld, lt = (int(x) for x in rng.integers(0, 40, 5))
        vocab = int(rng.integers(2, 12))
        A_ = rng.integers(0, vocab, la).tolist()
        B_ = rng.integers(0, vocab, lb).tolist()
        C_ = rng.integers(0, vocab, lc).tolist()
        D_ = rng.integers(0, vocab, ld).tolist()
        T_ = rng.integers(0, vocab, lt).tolist()
        ms = int(rng.integers(1, 9))
        suf = bool(rng.integers(0, 4))
        new = A_ + C_ + D_
        if not new:
            new = [0]
        s = ref_match.split(A_ + B_ + C_ + T_, new, min_suffix=ms, suffix=suf)
        cases.append({"cached": A_ + B_ + C_ + T_, "new": new, "min_suffix": ms, "suffix": suf,
                      "expect": [s.a, s.c0, s.c]})
    with open(os.path.join(HERE, "split_cases.json"), "w") as f:
        json.dump(cases, f)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", len(out), "arrays and", len(cases), "split cases")


if __name__ == "__main__":
    main()
