"""The reference engine's sequence of calls into this path, made by the GPU tests.

threadcut/engine.py:21-104 is the caller of the hot path, not part of it: per request it asks
match.split for the reusable A and C (engine.py:51-52), either builds a fresh cache with
kv.new_cache or rewrites the cached one with kv.splice (engine.py:53-57), prefills the new tail in
chunks through the model (engine.py:41-49), then decodes greedily one token per forward
(engine.py:88-95). The package does not ship an engine: the reference's own engine binds to
threadcut_b200 unchanged (tests/test_host.py runs that binding on the reference's engine source in
the build container, where the checkout is available). The GPU box has no reference source, so the
tests drive the same calls, in the same order and with the same statistics, through `Session`.
"""
import torch

from threadcut_b200.kv import cache_bytes, new_cache, splice
from threadcut_b200.match import split


class Session:
    """One cached sequence over `model` (any device). layout: keyword arguments of new_cache
    (paged=..., max_tokens=...), empty for the process-wide default."""

    def __init__(self, model, stop_ids=(510, 511), min_suffix=4, prefill_chunk=7, max_ctx=32768, layout=None):
        self.model = model.eval()
        self.device = next(model.parameters()).device
        self.inv_freq = model.model.rotary_emb.inv_freq
        self.stop_ids = set(stop_ids)
        self.min_suffix, self.prefill_chunk, self.max_ctx = min_suffix, prefill_chunk, max_ctx
        self.layout = dict(layout or {})
        self.ids, self.cache = [], None

    @torch.no_grad()
    def prefill(self, ids, cache):
        """Logits [1, vocab] of the last of `ids` after running them on top of `cache` in chunks."""
        last = None
        for lo in range(0, len(ids), self.prefill_chunk):
            chunk = torch.tensor([ids[lo:lo + self.prefill_chunk]], device=self.device)
            out = self.model(input_ids=chunk, past_key_values=cache, use_cache=True, logits_to_keep=1)
            last = out.logits[:, -1]
        return last

    @torch.no_grad()
    def load(self, new_ids):
        """Cache := new_ids with the least recompute: (logits of the last id, reuse statistics)."""
        plan = None if self.cache is None else split(self.ids, new_ids, self.min_suffix, True)
        if plan is None or plan.a + plan.c == 0:
            self.cache = new_cache(self.model.config, **self.layout)
            kept = 0
        else:
            splice(self.cache, plan, self.inv_freq)
            kept = plan.a + plan.c
        logits = self.prefill(new_ids[kept:], self.cache)
        stats = {"prompt_tokens": len(new_ids), "reused_prefix": plan.a if plan else 0,
                 "reused_suffix": plan.c if plan else 0, "reused_tokens": kept,
                 "dropped_from_cache": len(self.ids) - kept, "computed_tokens": len(new_ids) - kept}
        self.ids = list(new_ids)
        return logits, stats

    @torch.no_grad()
    def generate(self, new_ids, max_new_tokens=16):
        """Greedy continuation of new_ids until a stop id or the budget: (tokens, statistics)."""
        budget = min(max_new_tokens, self.max_ctx - len(new_ids))
        logits, stats = self.load(new_ids)
        out, finish = [], "length"
        while len(out) < budget:
            nxt = int(logits.argmax(-1))
            if nxt in self.stop_ids:
                finish = "stop"
                break
            out.append(nxt)
            step = self.model(input_ids=torch.tensor([[nxt]], device=self.device), past_key_values=self.cache,
                              use_cache=True)
            logits = step.logits[:, -1]
        self.ids += out
        stats.update(completion_tokens=len(out), finish=finish, kv_tokens=self.cache.get_seq_length(),
                     kv_mb=cache_bytes(self.cache) / 2**20)
        return out, stats
