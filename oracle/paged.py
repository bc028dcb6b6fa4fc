"""Paged-cache oracle (numpy). Test infrastructure only; see oracle/__init__.py.

The paged layout has no reference code (threadcut README.md:141-144 names it as the next step);
its contract is that the logical cache equals the reference's contiguous cache after the same
updates and splices. So the checker is the reference's own cache model plus a gather:

  * `ListCache` keeps one contiguous [hkv, n, d] array per layer and applies appends and
    splices exactly as threadcut/kv.py:28-41 (via copy_splice_ref) and kv.py:64-77 (append);
  * `gather_ref` reads a paged pool back in run order, to compare with it element for element.
"""
import numpy as np

from .splice import copy_splice_ref


def gather_ref(pool, runs):
    """pool [pages, hkv, page_rows, d]; runs [(page, first row, rows), ...] -> [hkv, n, d]."""
    pool = np.asarray(pool)
    if len(runs) == 0:
        return np.zeros((pool.shape[1], 0, pool.shape[3]), dtype=pool.dtype)
    return np.concatenate([pool[p, :, r0:r0 + c, :] for p, r0, c in runs], axis=1)


class ListCache:
    """Contiguous K/V per layer (fp32 values of the stored dtype), the reference's cache model."""

    def __init__(self, layers, hkv, d):
        self.k = [np.zeros((hkv, 0, d), np.float32) for _ in range(layers)]
        self.v = [np.zeros((hkv, 0, d), np.float32) for _ in range(layers)]

    @property
    def n(self):
        return self.k[0].shape[1]

    def append(self, layer, k, v):
        """threadcut/kv.py:64-77: new rows [hkv, t, d] go after the last one."""
        self.k[layer] = np.concatenate((self.k[layer], np.asarray(k, np.float32)), axis=1)
        self.v[layer] = np.concatenate((self.v[layer], np.asarray(v, np.float32)), axis=1)

    def splice(self, a, c0, c, inv_freq=None, dtype="bf16", cos_sin=None):
        """threadcut/kv.py:28-41 on every layer."""
        for l in range(len(self.k)):
            self.k[l], self.v[l] = copy_splice_ref(self.k[l], self.v[l], a, c0, c, inv_freq, dtype, cos_sin)
