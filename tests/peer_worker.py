"""torchrun worker: the peer-memory collectives (threadcut_b200.peer: AllReduce, the sums of the
tensor-parallel step; GatherMerge, the combine of a sequence-sharded decode) against the same
arithmetic through the collective library.

Every rank holds its own columns of a row-split projection (x_r [k], w_r [hidden, k]). Expected, as
torch would compute it: the fp32 partials x_r . w_r^T of all ranks (all-gathered with NCCL) summed in
rank order, rounded to bf16, added to the residual h (rounded) and RMS-normalised (Qwen3RMSNorm).
Checked over 7 sums in a row (both slots, several epochs): every rank ends with the same bits in h,
h and out are within a rounding step of the expected values, and no device wait ran out. The
residual form of the sums is checked against that form (check_residual)."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from threadcut_b200 import _lib  # noqa: E402
from threadcut_b200.peer import AllReduce  # noqa: E402


def rmsnorm(h, w, eps):
    hf = h.float()
    return w * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)).to(h.dtype)


def check(dev, world, rank, hidden=2560, k=512, rounds=7):
    eps = 1e-6
    ar = AllReduce(hidden, dev)
    g = torch.Generator(device=dev).manual_seed(1)  # shared: h and the norm weight equal on every rank
    h = torch.randn(1, hidden, generator=g, device=dev).to(torch.bfloat16)
    wn = (1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).to(torch.bfloat16)
    mine = torch.Generator(device=dev).manual_seed(100 + rank)
    h_ref = h.clone()
    out = torch.empty_like(h)
    worst = 0.0
    for i in range(rounds):
        x = torch.randn(1, k, generator=mine, device=dev).to(torch.bfloat16)
        w = (torch.randn(hidden, k, generator=mine, device=dev) / k ** 0.5).to(torch.bfloat16)
        ar.gemv(x, w)
        ar.add_rmsnorm(h, wn, out, eps)
        part = (x.float() @ w.float().t()).view(-1)
        every = torch.empty(world * hidden, device=dev)
        dist.all_gather_into_tensor(every, part)
        tot = every.view(world, hidden)[0].clone()
        for r in range(1, world):
            tot += every.view(world, hidden)[r]
        h_ref = (h_ref.float() + tot.to(torch.bfloat16).float()).to(torch.bfloat16)
        out_ref = rmsnorm(h_ref, wn, eps)
        worst = max(worst, float((h.float() - h_ref.float()).abs().max()))
        assert torch.allclose(h.float(), h_ref.float(), atol=0.05, rtol=0.02), (i, worst)
        assert torch.allclose(out.float(), out_ref.float(), atol=0.05, rtol=0.02), i
        h_ref = h.clone()  # continue from the kernel's bits (the comparison is per round)
        hs = torch.empty(world * hidden, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(hs, h.view(-1))
        assert all(torch.equal(hs.view(world, hidden)[r], h.view(-1)) for r in range(world)), i
    torch.cuda.synchronize(dev)
    errs = _lib.device_errors(clear=True)
    assert errs == 0, errs
    dist.barrier()
    ar.close()
    return {"rounds": rounds, "worst_h_diff": worst}


def check_residual(dev, world, rank, hidden=2560, k=512, n2=1536, rounds=7):
    """The residual form (AllReduce.gemv_residual, then gemv_norm of the next projection) against
    the two-kernel form on a copy of the residual, in the same region (the forms alternate sums):
    h bit-identical to gemv + add_rmsnorm on every rank and every round (both slots, several
    epochs), the same h bits on every rank, and the next projection of RMSNorm(h) equal on every
    rank and within a rounding step of tc_gemv of add_rmsnorm's output."""
    from threadcut_b200.tp import _gemv
    eps = 1e-6
    ar = AllReduce(hidden, dev)
    g = torch.Generator(device=dev).manual_seed(3)  # shared: h, the norm weight, the next projection
    h_a = torch.randn(1, hidden, generator=g, device=dev).to(torch.bfloat16)
    h_b = h_a.clone()
    wn = (1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).to(torch.bfloat16)
    w2 = (torch.randn(n2, hidden, generator=g, device=dev) / hidden ** 0.5).to(torch.bfloat16)
    mine = torch.Generator(device=dev).manual_seed(300 + rank)
    out_a = torch.empty_like(h_a)
    for i in range(rounds):
        swiglu = i % 2 == 1
        x = torch.randn(1, 2 * k if swiglu else k, generator=mine, device=dev).to(torch.bfloat16)
        w = (torch.randn(hidden, k, generator=mine, device=dev) / k ** 0.5).to(torch.bfloat16)
        ar.gemv(x, w, swiglu=swiglu)
        ar.add_rmsnorm(h_a, wn, out_a, eps)
        want = _gemv(out_a, w2)
        ar.gemv_residual(x, w, h_b, swiglu=swiglu)
        got = ar.gemv_norm(h_b, wn, w2, eps)
        torch.cuda.synchronize(dev)
        assert torch.equal(h_b, h_a), (i, float((h_b.float() - h_a.float()).abs().max()))
        diff = (got.float() - want.float()).abs()
        assert bool((diff <= 2 ** -6 * want.float().abs().clamp(min=1.0)).all()), (i, float(diff.max()))
        gs = torch.empty(world * n2, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(gs, got.view(-1))
        assert all(torch.equal(gs.view(world, n2)[r], got.view(-1)) for r in range(world)), i
    torch.cuda.synchronize(dev)
    errs = _lib.device_errors(clear=True)
    assert errs == 0, errs
    dist.barrier()
    ar.close()
    return {"residual_rounds": rounds}


def check_gather(dev, world, rank, rows=1152, d=128, rounds=5):
    """GatherMerge (tc_peer_gather_merge) against an NCCL all-gather of the same partials followed by
    flash_decode.merge_partials: the same bits on every rank, over several gathers (both slots)."""
    from threadcut_b200.flash_decode import merge_partials
    from threadcut_b200.peer import GatherMerge
    gm = GatherMerge(rows, d, dev)
    g = torch.Generator(device=dev).manual_seed(200 + rank)
    out = torch.empty(rows, d, dtype=torch.bfloat16, device=dev)
    lse_out = torch.empty(rows, device=dev)
    for i in range(rounds):
        o = torch.randn(rows, d, generator=g, device=dev)
        lse = torch.randn(rows, generator=g, device=dev) * 3
        if i == 1:
            lse[::7] = -float("inf")  # rows this rank's slice did not see
        gm(o, lse, out, lse_out)
        go = torch.empty(world * rows * d, device=dev)
        gl = torch.empty(world * rows, device=dev)
        dist.all_gather_into_tensor(go, o.view(-1))
        dist.all_gather_into_tensor(gl, lse)
        want, want_lse = merge_partials(go.view(world, rows, d), gl.view(world, rows), torch.bfloat16)
        torch.cuda.synchronize(dev)
        assert torch.equal(out, want), (i, float((out.float() - want.float()).abs().max()))
        assert torch.equal(lse_out, want_lse), i
    errs = _lib.device_errors(clear=True)
    assert errs == 0, errs
    dist.barrier()
    gm.close()
    return {"gathers": rounds}


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = True
    try:
        try:
            print(f"rank {rank}/{world}: {check(dev, world, rank)} {check_residual(dev, world, rank)} "
                  f"{check_gather(dev, world, rank)} "
                  f"{check_gather(dev, world, rank, rows=3, d=128, rounds=3)}", flush=True)
        except AssertionError as exc:
            print(f"rank {rank}/{world}: FAILED {exc}", flush=True)
            ok = False
        flag = torch.tensor([0 if ok else 1], device=dev)
        dist.all_reduce(flag)
        ok = flag.item() == 0
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
