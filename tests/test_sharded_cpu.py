"""Host logic of sharded decode on CPU: shard planning, and the gather + LSE merge on two `gloo`
ranks with oracle partials (the kernels need a GPU; the plumbing does not)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.attention import decode_attention_ref, merge_ref
from threadcut_b200.sharded import gather_partials, head_shard, seq_shard


def test_seq_shard_covers_and_aligns():
    for n in (1, 31, 32, 33, 4096, 98304, 131071):
        for world in (1, 2, 3, 4, 8):
            ranges = [seq_shard(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
                assert a1 == b0
            for lo, hi in ranges[:-1]:
                assert lo % 32 == 0 and hi % 32 == 0 and lo <= hi


def test_head_shard():
    assert [head_shard(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert head_shard(8, 0, 1) == (0, 8)
    with pytest.raises(ValueError):
        head_shard(8, 0, 3)
    with pytest.raises(ValueError):
        seq_shard(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)  # same global problem on every rank
        q = rng.standard_normal((8, 4, 64))
        k = rng.standard_normal((8, n, 64))
        v = rng.standard_normal((8, n, 64))
        # sequence sharding: partial over this rank's tokens, gather, merge
        t0, t1 = seq_shard(n, rank, world)
        o, lse = decode_attention_ref(q, k[:, t0:t1], v[:, t0:t1], 0.125, return_lse=True)
        o_parts, l_parts = gather_partials(torch.from_numpy(o.reshape(32, 64)).float(),
                                           torch.from_numpy(lse.reshape(32)).float())
        assert o_parts.shape == (world, 32, 64) and l_parts.shape == (world, 32)
        merged, _ = merge_ref(o_parts.numpy(), l_parts.numpy())
        whole = decode_attention_ref(q, k, v, 0.125).reshape(32, 64)
        seq_err = float(np.abs(merged - whole).max())
        # head sharding: this rank's heads, all-gathered in rank order
        h0, h1 = head_shard(8, rank, world)
        mine = torch.from_numpy(decode_attention_ref(q[h0:h1], k[h0:h1], v[h0:h1], 0.125)).float()
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        head_err = float(np.abs(torch.cat(parts).numpy() - decode_attention_ref(q, k, v, 0.125)).max())
        result_q.put((rank, seq_err, head_err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [700, 4097])
def test_two_gloo_ranks_gather_and_merge(n):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, seq_err, head_err in results:
        assert seq_err < 1e-5 and head_err < 1e-6
