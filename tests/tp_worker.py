"""Tensor-parallel decoder check, shared by the one-GPU test (test_engine_gpu.py) and the torchrun
worker of the multi-GPU test (test_sharded_gpu.py).

A small bf16 Qwen3 (head_dim 128, 4 query heads per KV head: the decode kernel's fast path) decodes
one token after a 300-token prompt. Expected: the HF forward with threadcut_b200's attention over
the whole prompt (same weights, same seed on every rank). Checked: same top-1 and correlated
logits (the partial sums of the sharded projections round differently in bf16), the step's token
equals the argmax of the gathered logits, and a CUDA graph of the step (NCCL all-reduces inside)
replays the eager token."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from transformers import AutoModelForCausalLM, Qwen3Config  # noqa: E402

from threadcut_b200 import attention as tc_attention  # noqa: E402
from threadcut_b200.kv import new_cache  # noqa: E402
from threadcut_b200.tp import TPDecoder  # noqa: E402


def check(dev, world=1, rank=0):
    """Returns a dict of the measured quantities; raises AssertionError on a mismatch."""
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=8192)
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation=tc_attention.NAME)
    model = model.to(dev).eval()
    ids = torch.randint(0, 512, (1, 301), generator=torch.Generator().manual_seed(3)).to(dev)
    with torch.no_grad():
        ref = model(input_ids=ids, past_key_values=new_cache(model.config), use_cache=True).logits[0, -1].float()
        cache = new_cache(model.config)
        model(input_ids=ids[:, :300], past_key_values=cache, use_cache=True)
        dec = TPDecoder(model, dev, world=world, rank=rank)
        for i, layer in enumerate(cache.layers):
            dec.load(i, layer.keys, layer.values)
        tok = ids[0, 300:]
        logits = dec.logits(tok, 300)
        dec.crop(300)
        eager = dec.step(tok, 300)
        dec.crop(300)
        graph, out = dec.capture(tok, 300)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        replayed = int(out)
        del graph
    corr = torch.corrcoef(torch.stack([logits, ref]))[0, 1].item()
    res = {"corr": corr, "max_abs": float((logits - ref).abs().max()), "top1": int(logits.argmax()),
           "ref_top1": int(ref.argmax()), "step": int(eager), "replayed": replayed}
    assert res["top1"] == res["ref_top1"], res
    assert corr > 0.999, res
    assert res["step"] == res["top1"] and res["replayed"] == res["step"], res
    return res


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = True
    try:
        try:
            print(f"rank {rank}/{world}: {check(dev, world, rank)}", flush=True)
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
