"""Decode attention sharded across GPUs (one process per GPU, torch.distributed over NCCL).

threadcut itself runs one sequence on one GPU (its Kaggle runs use two independent server
replicas, kaggle/run/run.py:66-70); sharding is new here. Decode attention splits two ways:

* by KV head (`HeadShardedDecode`): rank r owns heads [h0, h1) of the cache and the matching
  g query heads. The attention of a head needs nothing from other heads, so there is no exchange on
  the data path; `gather=True` all-gathers the per-rank outputs when every rank needs all heads.
* by sequence (`SeqShardedDecode`): rank r owns a contiguous token range of every head. Each rank
  computes its partial (o in fp32, log-sum-exp) with the decode kernel, the partials are
  all-gathered (hkv*g*(d+1)*4 bytes per rank, 16.5 KB for Qwen3-4B) and merged by log-sum-exp
  (tc_merge_partials) into the same output on every rank — the cross-GPU form of the slice merge
  of threadcut/flash_decode.py:68-69.

The shard planning and the gather are plain host logic (`head_shard`, `seq_shard`,
`gather_partials`), so they run on any backend; the kernels need CUDA.
"""
import torch
import torch.distributed as dist

from .flash_decode import decode_attention, decode_attention_partial, merge_partials

__all__ = ["head_shard", "seq_shard", "gather_partials", "HeadShardedDecode", "SeqShardedDecode"]


def _even(total, rank, world, align=1):
    """[lo, hi) of an even split of `total` items into `world` parts, boundaries on multiples of
    `align` (the last part takes the remainder)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    units = -(-total // align)
    lo = units * rank // world * align
    hi = units * (rank + 1) // world * align
    return min(lo, total), min(hi, total)


def head_shard(hkv, rank, world):
    """KV heads [h0, h1) owned by `rank`; every rank gets hkv // world heads (hkv must divide)."""
    if hkv % world:
        raise ValueError(f"{hkv} KV heads do not split evenly over {world} ranks")
    return _even(hkv, rank, world)


def seq_shard(n, rank, world, align=32):
    """Token range [t0, t1) of a length-n cache owned by `rank` (boundaries on 32-token tiles)."""
    return _even(n, rank, world, align)


def gather_partials(o_local, lse_local, group=None):
    """All-gather per-rank partials. o_local fp32 [rows, d], lse_local fp32 [rows] ->
    (o_parts [world, rows, d], lse_parts [world, rows]) in rank order."""
    world = dist.get_world_size(group)
    o_parts = [torch.empty_like(o_local) for _ in range(world)]
    l_parts = [torch.empty_like(lse_local) for _ in range(world)]
    dist.all_gather(o_parts, o_local.contiguous(), group=group)
    dist.all_gather(l_parts, lse_local.contiguous(), group=group)
    return torch.stack(o_parts), torch.stack(l_parts)


class HeadShardedDecode:
    """Decode attention over this rank's KV heads. q [hkv_local, g, d], k/v [hkv_local, n, d]."""

    def __init__(self, group=None):
        self.group = group

    def __call__(self, q, k, v, scale, gather=False):
        out = decode_attention(q, k, v, scale)
        if not gather:
            return out
        world = dist.get_world_size(self.group)
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out, group=self.group)
        return torch.cat(parts, dim=0)


class SeqShardedDecode:
    """Decode attention over this rank's token range of every head; returns the full output
    [hkv, g, d] (q's dtype) on every rank. q [hkv, g, d], k/v [hkv, n_local, d]."""

    def __init__(self, group=None):
        self.group = group

    def __call__(self, q, k, v, scale):
        hkv, g, d = q.shape
        o, lse = decode_attention_partial(q, k, v, scale)
        o_parts, l_parts = gather_partials(o.reshape(hkv * g, d), lse.reshape(hkv * g), self.group)
        out, _ = merge_partials(o_parts, l_parts, q.dtype)
        return out.reshape(hkv, g, d)
