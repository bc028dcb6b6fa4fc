"""Tensor-parallel decoder check, shared by the one-GPU test (test_engine_gpu.py) and the torchrun
worker of the multi-GPU tests (test_sharded_gpu.py, any number of ranks).

A small bf16 Qwen3 (Qwen3-4B's attention shape: 8 KV heads, so 1, 2, 4 and 8 ranks all hold whole
heads, 4 query heads per KV head, head_dim 128; hidden 256, 2 layers) holds a
2,304-token prompt A.B.C in its cache, computed by stock transformers with SDPA attention. B (256
tokens) is pruned with kv.splice, leaving 2,048 rows. Expected next token: the same SDPA forward of
one more token over that spliced cache (the torch path the reference's engine tests compare with,
threadcut tests/test_core.py:93-101). TPDecoder loads the spliced cache (2,048 rows: every layer's
buffer exactly full, so the step's append must find room) and is captured in a CUDA graph at once.
Checked: the replayed token, the eager step's token and the argmax of the gathered logits equal the
SDPA top-1, and the logits correlate (the partial sums of the sharded projections round differently
in bf16)."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from transformers import AutoModelForCausalLM, DynamicCache, Qwen3Config  # noqa: E402

from threadcut_b200.kv import splice  # noqa: E402
from threadcut_b200.match import Split  # noqa: E402
from threadcut_b200.tp import TPDecoder  # noqa: E402


def check(dev, world=1, rank=0):
    """Returns a dict of the measured quantities; raises AssertionError on a mismatch."""
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=8192)
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation="sdpa")
    model = model.to(dev).eval()
    ids = torch.randint(0, 512, (1, 2305), generator=torch.Generator().manual_seed(3)).to(dev)
    s = Split(512, 768, 2304 - 768)
    n = s.a + s.c
    with torch.no_grad():
        cache = DynamicCache(config=model.config)
        model(input_ids=ids[:, :2304], past_key_values=cache, use_cache=True)
        splice(cache, s, model.model.rotary_emb.inv_freq)  # the reference's copy splice (kv.py:34-41)
        assert cache.get_seq_length() == n == 2048
        dec = TPDecoder(model, dev, world=world, rank=rank)
        for i, layer in enumerate(cache.layers):
            dec.load(i, layer.keys, layer.values)
        assert all(ly.kbuf.shape[-2] == n for ly in dec.layers)  # full: the step's row needs a grow
        tok = ids[0, 2304:]
        graph, out = dec.capture(tok, n)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        replayed = int(out)
        del graph
        eager = int(dec.step(tok, n))
        dec.crop(n)
        logits = dec.logits(tok, n)
        dec.crop(n)
        ref = model(input_ids=ids[:, 2304:], past_key_values=cache, use_cache=True).logits[0, -1].float()
    corr = torch.corrcoef(torch.stack([logits, ref]))[0, 1].item()
    res = {"corr": corr, "max_abs": float((logits - ref).abs().max()), "top1": int(logits.argmax()),
           "sdpa_top1": int(ref.argmax()), "step": eager, "replayed": replayed, "world": world}
    assert res["top1"] == res["sdpa_top1"], res
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
