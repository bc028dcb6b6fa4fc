"""The CPU oracle against golden vectors recorded from the reference itself (CPU only).

These pin the oracle before it is trusted as the checker of the CUDA kernels: every function in
oracle/ is compared with the reference's own outputs (tests/golden/make_golden.py).
"""
import numpy as np
import pytest
import torch

import workloads
from helpers import ORACLE_ATOL, gold, meta, ref_cos_sin, sha, storage_dtype, values
from oracle.attention import attention_decode_ref, decode_attention_ref, merge_ref
from oracle.rope import f32_to_bf16_bits, round_to, shift_keys_f32, shift_keys_ref
from oracle.splice import copy_splice_ref, growing_splice_ref


@pytest.mark.parametrize("ci", range(10))
def test_decode_small_cases_match_reference(ci):
    G, M = gold(), meta()["cases"][f"dec{ci}"]
    q, k, v = (values(G[f"dec{ci}_{x}"]) for x in "qkv")
    out = attention_decode_ref(q, k, v, M["scale"])
    np.testing.assert_allclose(out, G[f"dec{ci}_out"], atol=ORACLE_ATOL, rtol=0)


def test_cfg1_inputs_pinned_and_output_matches():
    q, k, v = workloads.cfg1()
    assert [sha(q), sha(k), sha(v)] == meta()["cfg1_sha"]
    out = attention_decode_ref(q.numpy(), k.numpy(), v.numpy(), workloads.SCALE)
    np.testing.assert_allclose(out, gold()["cfg1_out_f32"], atol=ORACLE_ATOL, rtol=0)
    qb, kb, vb = (t.to(torch.bfloat16).float().numpy() for t in (q, k, v))
    out = attention_decode_ref(qb, kb, vb, workloads.SCALE)
    np.testing.assert_allclose(out, gold()["cfg1_out_bf16in"], atol=ORACLE_ATOL, rtol=0)


def test_16k_single_layer_matches():
    q, k, v = workloads.cfg1(n=16384)
    assert [sha(q), sha(k), sha(v)] == meta()["cfg16k_sha"]
    qb, kb, vb = (t.to(torch.bfloat16).float().numpy() for t in (q, k, v))
    out = attention_decode_ref(qb, kb, vb, workloads.SCALE, dtype=np.float32)
    np.testing.assert_allclose(out, gold()["cfg16k_out_bf16in"], atol=ORACLE_ATOL, rtol=0)


@pytest.mark.parametrize("ci", range(7))
def test_shift_bit_exact_with_reference_table(ci):
    G = gold()
    dt = storage_dtype(G[f"shift{ci}_in"])
    keys = values(G[f"shift{ci}_in"])
    res = shift_keys_ref(keys, dtype=dt, cos_sin=(G[f"shift{ci}_cos"], G[f"shift{ci}_sin"]))
    np.testing.assert_array_equal(res.view(np.uint32), values(G[f"shift{ci}_out"]).view(np.uint32))


@pytest.mark.parametrize("ci", range(7))
def test_shift_numpy_table_within_one_ulp(ci):
    """With numpy's own cos/sin the oracle stays within 1 ulp of the storage dtype."""
    G, M = gold(), meta()["cases"][f"shift{ci}"]
    dt = storage_dtype(G[f"shift{ci}_in"])
    inv = workloads.inv_freq(M["d"], M["theta"]).numpy()
    res = shift_keys_ref(values(G[f"shift{ci}_in"]), M["delta"], inv, dtype=dt)
    ref = values(G[f"shift{ci}_out"])
    if dt == "bf16":
        diff = np.abs(f32_to_bf16_bits(res).astype(np.int32) - f32_to_bf16_bits(ref).astype(np.int32))
        assert diff.max() <= 1
    elif dt == "f16":
        diff = np.abs(res.astype(np.float16).view(np.int16).astype(np.int32)
                      - ref.astype(np.float16).view(np.int16).astype(np.int32))
        assert diff.max() <= 1
    else:
        np.testing.assert_allclose(res, ref, rtol=4e-6, atol=4e-6)


def test_cfg2_splice_bit_exact_and_decode():
    G, Mt = gold(), meta()
    kc, vc = workloads.cfg2_cache()
    assert [sha(kc), sha(vc)] == Mt["cfg2_sha_in"]
    a, c0, c = workloads.CFG2_SPLIT
    cs = ref_cos_sin(-(c0 - a), workloads.inv_freq())
    kb, vb, n = growing_splice_ref(kc.float().numpy(), vc.float().numpy(), a, c0, c, dtype="bf16", cos_sin=cs)
    ks = torch.from_numpy(kb[:, :n]).to(torch.bfloat16)
    vs = torch.from_numpy(vb[:, :n]).to(torch.bfloat16)
    assert [sha(ks), sha(vs)] == Mt["cfg2_sha_spliced"]
    np.testing.assert_array_equal(f32_to_bf16_bits(kb[:, G["cfg2_rows"]]), G["cfg2_k_rows"])
    q = workloads.cfg2_query()
    assert sha(q) == Mt["cfg2_sha_q"]
    out = decode_attention_ref(q.float().numpy().reshape(8, 4, 128), kb[:, :n], vb[:, :n], workloads.SCALE)
    np.testing.assert_allclose(out.reshape(1, 1, 32, 128), G["cfg2_out"], atol=ORACLE_ATOL, rtol=0)


@pytest.mark.parametrize("ci", range(9))
def test_growing_splice_matches_reference(ci):
    G, M = gold(), meta()["cases"][f"grow{ci}"]
    a, c0, c = M["split"]
    dt = M["dtype"]
    inv = workloads.inv_freq(M["d"], M["theta"])
    cs = ref_cos_sin(-(c0 - a), inv)
    k, v = values(G[f"grow{ci}_k"])[0], values(G[f"grow{ci}_v"])[0]
    kb, vb, n = growing_splice_ref(k, v, a, c0, c, dtype=dt, cos_sin=cs)
    np.testing.assert_array_equal(kb[:, :n], values(G[f"grow{ci}_kout"])[0])
    np.testing.assert_array_equal(vb[:, :n], values(G[f"grow{ci}_vout"])[0])


def test_copy_splice_matches_reference():
    G = gold()
    cs = ref_cos_sin(-7, workloads.inv_freq(16, 1e4))
    k, v = copy_splice_ref(G["copy_k"][0], G["copy_v"][0], 10, 17, 20, dtype="f32", cos_sin=cs)
    np.testing.assert_array_equal(k, G["copy_kout"][0])
    np.testing.assert_array_equal(v, G["copy_vout"][0])


def test_ragged_cases_match_reference():
    G = gold()
    for bi, _ in enumerate(meta()["ragged_lengths"]):
        q, k, v = (values(G[f"rag{bi}_{x}"]) for x in "qkv")
        out = attention_decode_ref(q, k, v, workloads.SCALE)
        np.testing.assert_allclose(out, G[f"rag{bi}_out"], atol=ORACLE_ATOL, rtol=0)


def test_merge_of_partials_equals_whole():
    """LSE merge is exact: attention over [0, n) == merge of attention over any split of [0, n)."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal((8, 4, 64))
    k = rng.standard_normal((8, 500, 64))
    v = rng.standard_normal((8, 500, 64))
    whole = decode_attention_ref(q, k, v, 0.125)
    cuts = [0, 1, 130, 131, 400, 500]
    parts = [decode_attention_ref(q, k[:, lo:hi], v[:, lo:hi], 0.125, return_lse=True)
             for lo, hi in zip(cuts[:-1], cuts[1:])]
    o = np.stack([p[0].reshape(32, 64) for p in parts])
    lse = np.stack([p[1].reshape(32) for p in parts])
    merged, _ = merge_ref(o, lse)
    np.testing.assert_allclose(merged, whole.reshape(32, 64), atol=1e-12)


def test_oracle_plants_are_caught():
    """A planted mistake in the oracle (wrong rotation sign) must break bit-exactness."""
    G = gold()
    keys = values(G["shift0_in"])
    cs = (G["shift0_cos"], G["shift0_sin"])
    bad_sin = (cs[0], -cs[1])
    good = shift_keys_ref(keys, dtype="bf16", cos_sin=cs)
    bad = shift_keys_ref(keys, dtype="bf16", cos_sin=bad_sin)
    assert np.array_equal(good, values(G["shift0_out"]))
    assert not np.array_equal(bad, values(G["shift0_out"]))


def test_round_to_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    ours = round_to(x, "bf16")
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(ours, ref)
    f = shift_keys_f32(x.reshape(100, 100), 3, workloads.inv_freq(100, 1e4).numpy())
    assert f.dtype == np.float32


# ---- oracle/torch_ref.py: the reference's CPU path as torch expressions (the timed CPU baseline)
@pytest.mark.parametrize("ci", range(7))
def test_torch_ref_shift_bit_exact_with_reference(ci):
    from oracle.torch_ref import shift_keys as torch_shift
    G, M = gold(), meta()["cases"][f"shift{ci}"]
    dt = storage_dtype(G[f"shift{ci}_in"])
    keys = torch.from_numpy(values(G[f"shift{ci}_in"])).to({"bf16": torch.bfloat16, "f16": torch.float16,
                                                            "f32": torch.float32}[dt])
    out = torch_shift(keys, M["delta"], workloads.inv_freq(M["d"], M["theta"]))
    np.testing.assert_array_equal(out.float().numpy().view(np.uint32), values(G[f"shift{ci}_out"]).view(np.uint32))


def test_torch_ref_cfg2_splice_and_decode_match_reference():
    from oracle.torch_ref import folded_decode, growing_splice
    G, Mt = gold(), meta()
    kc, vc = workloads.cfg2_cache()
    a, c0, c = workloads.CFG2_SPLIT
    kb, vb = kc.clone()[None], vc.clone()[None]
    n = growing_splice(kb, vb, a, c0, c, workloads.inv_freq())
    assert [sha(kb[0, :, :n]), sha(vb[0, :, :n])] == Mt["cfg2_sha_spliced"]
    q = workloads.cfg2_query()
    out = folded_decode(q.float().reshape(1, 32, 1, 128), kb[:, :, :n].float(), vb[:, :, :n].float(), workloads.SCALE)
    np.testing.assert_allclose(out.numpy(), G["cfg2_out"], atol=ORACLE_ATOL, rtol=0)


def test_torch_ref_decode_matches_reference_cfg1():
    from oracle.torch_ref import folded_decode
    q, k, v = workloads.cfg1()
    out = folded_decode(q, k, v, workloads.SCALE)
    np.testing.assert_allclose(out.numpy().reshape(gold()["cfg1_out_f32"].shape), gold()["cfg1_out_f32"],
                               atol=ORACLE_ATOL, rtol=0)
