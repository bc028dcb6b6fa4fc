"""split() on the GPU (tc_split) against the host rule: every reference golden case and large
synthetic requests (needs a B200). Integer work: results must be identical."""
import numpy as np
import pytest
import torch

from helpers import split_cases
from threadcut_b200 import _lib
from threadcut_b200.match import Split, split, split_device

pytestmark = pytest.mark.gpu


def test_reference_golden_cases():
    cases = split_cases()
    assert len(cases) >= 200
    for case in cases:
        cached, new = case["cached"], case["new"]
        kw = {k: case[k] for k in ("min_suffix", "suffix") if k in case}
        if len(new) == 0:
            continue
        want = split(cached, new, **kw)
        got = split_device(cached, new, **kw)
        assert got == want, (case, got, want)
    assert _lib.device_errors(clear=True) == 0


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_large_spliced_requests(seed):
    """config-5-like request: a 128k cache, a 32k span pruned mid-context, a fresh tail; plus a
    second copy of part of C earlier in the cache (a tie between candidate starts)."""
    rng = np.random.default_rng(seed)
    cached = rng.integers(0, 151936, 131072).astype(np.int64)
    a, c0 = 49152, 81920
    cached[20000:20000 + 5000] = cached[c0:c0 + 5000]  # shorter duplicate of C's head before c0
    new = np.concatenate([cached[:a], cached[c0:], rng.integers(0, 151936, 300)])
    want = split(cached.tolist(), new.tolist())
    got = split_device(cached, new)
    assert got == want and got.a == a and got.c0 == c0, (got, want)
    # the same request as device tensors
    assert split_device(torch.as_tensor(cached, device="cuda"), torch.as_tensor(new, device="cuda")) == want


def test_degenerate_and_edge_inputs():
    z = [7] * 3000
    assert split_device(z, z[:2000] + [9] + z[:100]) == split(z, z[:2000] + [9] + z[:100])
    assert split_device(z, z) == split(z, z)
    rng = np.random.default_rng(4)
    cached = rng.integers(0, 50, 4000).tolist()  # small vocabulary: many candidate windows
    new = cached[:100] + cached[1000:3000] + cached[500:900]
    for ms in (1, 2, 8, 32):
        for suf in (True, False):
            assert split_device(cached, new, min_suffix=ms, suffix=suf) == split(cached, new, min_suffix=ms, suffix=suf)
    assert split_device([], [1, 2, 3]) == split([], [1, 2, 3])
    assert split_device([1, 2, 3], [1]) == split([1, 2, 3], [1]) == Split(0, 0, 0)
    with pytest.raises(ValueError):
        split_device([1, 2], [])
    assert _lib.device_errors(clear=True) == 0


def test_tie_between_candidate_starts_picks_the_first():
    rng = np.random.default_rng(5)
    cached = rng.integers(0, 151936, 20000)
    cached[5000:8001] = cached[15000:18001]  # C (and one token more) also occurs earlier, inside B
    new = np.concatenate([cached[:2000], cached[15000:18000]])
    want = split(cached.tolist(), new.tolist())
    assert want == Split(2000, 5000, 2999)
    assert split_device(cached, new) == want
