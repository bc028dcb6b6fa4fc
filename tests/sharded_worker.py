"""torchrun worker for tests/test_sharded_gpu.py: sequence- and head-sharded decode on N GPUs
(NCCL) checked against the single-GPU kernel and the oracle on the same seeded problem."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)
from helpers import ATTN_ATOL, attn_error  # noqa: E402
from oracle.attention import decode_attention_ref  # noqa: E402
from threadcut_b200.flash_decode import decode_attention  # noqa: E402
from threadcut_b200.sharded import HeadShardedDecode, SeqShardedDecode, head_shard, seq_shard  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = True
    try:
        for n in (32768, 5000):
            g = torch.Generator().manual_seed(n)
            q = torch.randn(8, 4, 128, generator=g).to(torch.bfloat16)
            k = torch.randn(8, n, 128, generator=g).to(torch.bfloat16)
            v = torch.randn(8, n, 128, generator=g).to(torch.bfloat16)
            ref = decode_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), 128 ** -0.5,
                                       dtype=np.float32)
            single = decode_attention(q.to(dev), k.to(dev), v.to(dev), 128 ** -0.5).float().cpu().numpy()
            t0, t1 = seq_shard(n, rank, world)
            seq = SeqShardedDecode()(q.to(dev), k[:, t0:t1].to(dev), v[:, t0:t1].to(dev), 128 ** -0.5)
            h0, h1 = head_shard(8, rank, world)
            head = HeadShardedDecode()(q[h0:h1].to(dev), k[h0:h1].to(dev), v[h0:h1].to(dev), 128 ** -0.5, gather=True)
            torch.cuda.synchronize()
            e_seq = attn_error(seq.float().cpu().numpy(), ref, torch.bfloat16)
            e_head = attn_error(head.float().cpu().numpy(), ref, torch.bfloat16)
            e_single = attn_error(single, ref, torch.bfloat16)
            print(f"rank {rank} n {n}: seq {e_seq:.2e} head {e_head:.2e} single {e_single:.2e}", flush=True)
            ok &= e_seq <= ATTN_ATOL and e_head <= ATTN_ATOL and e_single <= ATTN_ATOL
        flag = torch.tensor([0 if ok else 1], device=dev)
        dist.all_reduce(flag)
        ok = flag.item() == 0
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
