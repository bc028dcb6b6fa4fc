"""Benchmark of threadcut's decode hot path on B200: split-KV GQA flash-decode µs/layer and % of HBM
peak at 16k context (BASELINE metric), plus the RoPE-shift splice GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = decode attention for all 36 Qwen3-4B layers (one query token, 32 q / 8 KV heads,
head_dim 128, bf16) of one sequence, every layer its own K/V buffer. On N GPUs the sequence holds
16384 x N tokens and its KV heads are sharded over the GPUs (8 / N per GPU), so every GPU streams
67 MB per layer (36 x 67 MB = 2.4 GB per step, far above the 126 MB L2, so no flush is needed), and
the step ends with an all-gather of every layer's outputs to every rank. At N = 1 this is the 16k
decode; at N = 8 the 128k sequence with one KV head per GPU. `value` is µs per layer of the job
divided by N (µs per layer per 16k tokens of context: device time, CUDA events, the step replayed
from a CUDA graph, max over ranks), so the driver's v_1 / v_N is the weak-scaling efficiency.
`e2e` is the same metric through the public API (`threadcut_b200.flash_decode.decode_attention`,
one Python call per layer, and the all-gather) with each step's queries copied host->device from
pinned memory and the gathered outputs read back device->host inside the timed region.
`--impl reference` times the reference's CPU path (its torch decode expression on CPU tensors,
oracle/torch_ref.py, bf16, every host core) on the same workload and prints the same line with
"impl": "reference".
"""
import argparse
import json
import os
import statistics
import subprocess
import tempfile
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import workloads  # noqa: E402

METRIC = "flash-decode µs/layer & % of HBM peak (Qwen3-4B GQA, 16k ctx); shift GB/s"
WORKLOAD = ("cfg3-16k: 36-layer split-KV GQA decode of one sequence of 16384 x N tokens over N GPUs, 32 q / 8 kv "
            "heads, head_dim 128, KV heads sharded over the GPUs, one K/V buffer per layer")
N_CTX = 16384
LAYERS = workloads.LAYERS


def decode_bytes(n):
    """Algorithmic bytes of one decode launch: K+V (2 * 8 heads * n * 128 * 2 B) + q + o."""
    return 4096 * n + 16384


BYTES_PER_LAYER = decode_bytes(N_CTX)
SHIFT_BYTES_PER_LAYER = 4 * 4096 * 8 * 128 * 2  # K read+write and V read+write of |C| = 4096 rows
FALLBACK_HBM_GBS = 6650.0


def peaks():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------ clocks during the timed region
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, None

    def __enter__(self):
        try:
            # raw samples go to BENCH_CLOCKS_DIR when set (kept for inspection), else a temp folder
            out_dir = os.environ.get("BENCH_CLOCKS_DIR") or tempfile.mkdtemp(prefix="bench_clocks_")
            os.makedirs(out_dir, exist_ok=True)
            self.path = os.path.join(out_dir, f"clocks_gpu{self.index}.csv")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        load = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ distributed plumbing
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        if args.impl == "reference":
            return rank, local, world, None
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        return rank, local, world, dist
    if args.impl != "reference":
        torch.cuda.set_device(0)
    return 0, 0, 1, None


def max_over_ranks(x, dist):
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# ------------------------------------------------------------------ our arm
def build_layers(n, layers, dev, seed, heads=8):
    ks, vs = workloads.layer_kv(n, layers, dev, seed=seed, heads=heads)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    qs = [torch.randn(heads, 4, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(layers)]
    return qs, ks, vs


def capture_step(qs, ks, vs, outs, dev, stable=True, combine=None, lses=None):
    """CUDA graph of one step: the 36 decode launches through the C ABI with preallocated outputs.
    stable: declare rows [0, n-1) stable (tc_decode_attention_stable), as a decode step may: every
    row but the newest was written before the step; False runs plain tc_decode_attention.
    lses: None, or one fp32 [hl, 4] tensor per layer: then each launch computes the fp32 partial and
    its log-sum-exp (tc_decode_attention_partial_stable; outs fp32), a sequence shard's part.
    combine: None, or a function run after the launches inside the graph (the sharded step's
    combine: collectives and the merge)."""
    from threadcut_b200._lib import TC_BF16, check, lib, workspaces
    L = lib()
    n = ks[0].shape[1]
    hl = qs[0].shape[0]
    ws = workspaces.get(("decode", hl), dev, L.tc_decode_attention_workspace_size(1, hl, 4, 128, n, n, 0, TC_BF16))

    stable_rows = n - 1 if stable else 0

    def launch_all():
        st = torch.cuda.current_stream(dev).cuda_stream
        for i, (q, k, v, o) in enumerate(zip(qs, ks, vs, outs)):
            if lses is None:
                rc = L.tc_decode_attention_stable(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), hl, 4, 128,
                                                  n, q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0),
                                                  v.stride(1), o.stride(0), o.stride(1), workloads.SCALE, 0, TC_BF16,
                                                  stable_rows, ws.data_ptr(), ws.numel(), st)
            else:
                rc = L.tc_decode_attention_partial_stable(
                    q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lses[i].data_ptr(), hl, 4, 128, n,
                    q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1), o.stride(0),
                    o.stride(1), workloads.SCALE, 0, TC_BF16, stable_rows, ws.data_ptr(), ws.numel(), st)
            check("tc_decode_attention", rc)
        if combine is not None:
            combine()

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        launch_all()  # eager warm-up on the capture stream (kernel attributes, workspace, communicator)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s, capture_error_mode="thread_local"):
            launch_all()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    return graph


class SeqShardedStep:
    """Buffers and combine of a sequence-sharded decode step over `world` ranks: every rank holds a
    token slice of all 8 KV heads of every layer and computes per layer the fp32 partial and LSE of
    its slice (tc_decode_attention_partial_stable); the combine gathers the step's partials from all
    ranks and merges them by log-sum-exp (the merge of threadcut/flash_decode.py:68-69 over ranks)
    into the bf16 outputs of every layer on every rank: one tc_peer_gather_merge launch through peer
    memory (combine), or two NCCL all-gathers and tc_merge_partials (combine_nccl)."""

    def __init__(self, layers, dev, dist, world, hl=8):
        from threadcut_b200.peer import GatherMerge
        self.rows = layers * hl * 4
        self.po = torch.empty((layers, hl, 4, 128), dtype=torch.float32, device=dev)
        self.pl = torch.empty((layers, hl, 4), dtype=torch.float32, device=dev)
        self.go = torch.empty((world * self.po.numel(),), dtype=torch.float32, device=dev)
        self.gl = torch.empty((world * self.pl.numel(),), dtype=torch.float32, device=dev)
        self.out = torch.empty((self.rows, 128), dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty((self.rows,), dtype=torch.float32, device=dev)
        self.outs, self.lses = list(self.po.unbind(0)), list(self.pl.unbind(0))
        self.dist, self.world, self.dev = dist, world, dev
        self.gm = GatherMerge(self.rows, 128, dev)

    def combine(self):
        """Through peer memory: one tc_peer_gather_merge launch (push to every rank + merge)."""
        self.gm(self.po.view(self.rows, 128), self.pl.view(self.rows), self.out, self.lse)

    def combine_nccl(self):
        """The same through the collective library: two NCCL all-gathers and tc_merge_partials."""
        from threadcut_b200._lib import TC_BF16, check, lib
        self.dist.all_gather_into_tensor(self.go, self.po.view(-1))
        self.dist.all_gather_into_tensor(self.gl, self.pl.view(-1))
        check("tc_merge_partials", lib().tc_merge_partials(
            self.go.data_ptr(), self.gl.data_ptr(), self.out.data_ptr(), self.lse.data_ptr(), self.world, self.rows,
            128, self.out.stride(0), TC_BF16, torch.cuda.current_stream(self.dev).cuda_stream))

    def close(self):
        self.dist.barrier()
        self.gm.close()


def time_graph(graph, steps, warmup, dist):
    for _ in range(warmup):
        graph.replay()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    e1.synchronize()
    barrier(dist)
    return e0.elapsed_time(e1) / steps  # ms per step on this rank


def time_e2e(qs, ks, vs, steps, warmup, dist, dev, world=1):
    """Public-API path: pinned host queries -> device, 36 decode calls, outputs -> host. One GPU:
    decode_attention per layer. N GPUs (sequence shards): decode_attention_partial per layer over
    the rank's token slice, then peer.GatherMerge (the step's partials pushed to every rank and
    merged in one launch), the merged outputs read back."""
    from threadcut_b200.flash_decode import decode_attention, decode_attention_partial
    host_q = torch.stack([q.cpu() for q in qs]).pin_memory()
    dq = torch.empty_like(host_q, device=dev)
    host_out = torch.empty(host_q.shape, dtype=host_q.dtype).pin_memory()
    layers, hl = host_q.shape[0], host_q.shape[1]
    rows = layers * hl * 4
    gm = None
    if world > 1:
        from threadcut_b200.peer import GatherMerge
        gm = GatherMerge(rows, 128, dev)
    merged = torch.empty((rows, 128), dtype=torch.bfloat16, device=dev)

    n = ks[0].shape[1]

    def step():
        dq.copy_(host_q, non_blocking=True)
        if world == 1:
            outs = torch.stack([decode_attention(dq[i], ks[i], vs[i], workloads.SCALE, stable_rows=n - 1)
                                for i in range(layers)])
        else:
            parts = [decode_attention_partial(dq[i], ks[i], vs[i], workloads.SCALE, stable_rows=n - 1)
                     for i in range(layers)]
            outs = gm(torch.stack([o for o, _ in parts]).view(rows, 128),
                      torch.stack([lse for _, lse in parts]).view(rows), merged)
        host_out.copy_(outs.view(host_out.shape), non_blocking=True)

    for _ in range(warmup):
        step()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    e1.synchronize()
    barrier(dist)
    if gm is not None:
        gm.close()
    return e0.elapsed_time(e1) / steps, host_q.numel() * host_q.element_size(), host_out.numel() * 2


def time_shift(steps, warmup, dev, dist, layers=LAYERS):
    """Config 2 splice (Split(2048, 4096, 4096) of an 8192-token cache) on all layers, one in-place
    launch per step through the C ABI (arguments prepared once, a fresh epoch per call); returns ms
    per launch. Every step splices the same rows again, so the bytes moved are the same each time."""
    import ctypes
    from threadcut_b200._lib import TC_BF16, check, cos_sin_table, lib, workspaces
    L = lib()
    g = torch.Generator(device=dev).manual_seed(7)
    n = workloads.CFG2_N
    kbufs = [torch.randn(8, n, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(layers)]
    vbufs = [k.clone() for k in kbufs]
    a, c0, c = workloads.CFG2_SPLIT
    kp = (ctypes.c_void_p * layers)(*[k.data_ptr() for k in kbufs])
    vp = (ctypes.c_void_p * layers)(*[v.data_ptr() for v in vbufs])
    tab, tab_ptr = cos_sin_table(a - c0, workloads.inv_freq())
    ws = workspaces.get("splice-bench", dev, L.tc_splice_workspace_size(layers, 8, c))
    epoch = [0]

    def run():
        epoch[0] += 1
        check("tc_splice_inplace", L.tc_splice_inplace(kp, vp, layers, 8, 128, n, a, c0, c, n * 128, 128, tab_ptr,
                                                       TC_BF16, ws.data_ptr(), ws.numel(), epoch[0],
                                                       torch.cuda.current_stream(dev).cuda_stream))
    for _ in range(warmup):
        run()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    e1.synchronize()
    barrier(dist)
    del tab
    return e0.elapsed_time(e1) / steps


def time_sdpa_16k(qs, ks, vs, steps, warmup, dist):
    """GPU comparator on the same box: the reference's own torch decode path (folded GQA SDPA,
    threadcut/attention.py:41-42: q [1, hkv, g, d] against k/v [1, hkv, n, d]) over the same 36 layers,
    replayed from a CUDA graph. Returns ms per 36-layer step."""
    import torch.nn.functional as F
    dev = qs[0].device
    q4 = [q.unsqueeze(0) for q in qs]
    k4 = [k.unsqueeze(0) for k in ks]
    v4 = [v.unsqueeze(0) for v in vs]

    def launch_all():
        for q, k, v in zip(q4, k4, v4):
            F.scaled_dot_product_attention(q, k, v, scale=workloads.SCALE)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        launch_all()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            launch_all()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    ms = time_graph(graph, steps, warmup, dist)
    del graph
    return ms


def time_append_16k(qs, ks, vs, steps, warmup, dist):
    """One decode step's append + attention per layer over the 36 16k layers (the cache views end at
    the appended row), replayed from CUDA graphs two ways: fused (decode_attention_append: one
    launch writes the row and attends) and the reference's order (two row copies, then decode).
    Returns (fused ms, copy-then-decode ms) per 36-layer step."""
    from threadcut_b200.flash_decode import decode_attention, decode_attention_append
    dev = qs[0].device
    n = ks[0].shape[1]
    g = torch.Generator(device=dev).manual_seed(77)
    kn = [torch.randn(8, 128, generator=g, device=dev).to(torch.bfloat16) for _ in ks]
    vn = [torch.randn(8, 128, generator=g, device=dev).to(torch.bfloat16) for _ in ks]

    def fused():
        for q, k, v, a, b in zip(qs, ks, vs, kn, vn):
            decode_attention_append(q, k, v, a, b, workloads.SCALE, stable_rows=n - 1)

    def unfused():
        for q, k, v, a, b in zip(qs, ks, vs, kn, vn):
            k[:, n - 1] = a
            v[:, n - 1] = b
            decode_attention(q, k, v, workloads.SCALE, stable_rows=n - 1)

    out = []
    for fn in (fused, unfused):
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        out.append(time_graph(graph, steps, warmup, dist))
        del graph
    return out[0], out[1]


def time_paged(steps, warmup, dev, dist, layers=LAYERS):
    """Paged cache (threadcut_b200.paged): (1) a 36-layer decode step over 16,384 live tokens held
    in 64-row pages after a splice whose cut points fall inside pages (ragged runs), replayed from a
    CUDA graph; (2) the config-2 splice as a paged splice: B's pages dropped on the host and C's
    keys re-rotated in place (tc_paged_rotate_keys, all layers in one launch, the same C rows every
    step). Returns (decode ms per step, rotate ms per launch, rotate bytes per layer, host table
    splice us, tiles)."""
    import ctypes
    from threadcut_b200._lib import TC_BF16, check, cos_sin_table, lib
    from threadcut_b200.match import Split
    from threadcut_b200.paged import PagedKV, PageTable
    g = torch.Generator(device=dev).manual_seed(99)
    kv = PagedKV(layers, 8, 128, max_tokens=20000, page_rows=64, device=dev)
    kv.reserve(20000)
    for l in range(layers):
        kv.write(l, torch.randn(8, 20000, 128, generator=g, device=dev).to(torch.bfloat16),
                 torch.randn(8, 20000, 128, generator=g, device=dev).to(torch.bfloat16))
    kv.splice(Split(4010, 7626, 12374), workloads.inv_freq())  # n = 16384, runs start/end inside pages
    assert kv.n == N_CTX
    qs = [torch.randn(8, 4, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(layers)]

    stable = kv.n_tiles - 1  # as the headline's stable_rows = n - 1

    def launch_all():
        for l in range(layers):
            kv.decode(l, qs[l], workloads.SCALE, stable_tiles=stable)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        launch_all()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            launch_all()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    dec_ms = time_graph(graph, steps, warmup, dist)
    tiles = kv._tiles()[1]
    del graph, kv, qs
    torch.cuda.empty_cache()
    # (2) config-2 splice on a fresh 8192-token paged cache
    n = workloads.CFG2_N
    a, c0, c = workloads.CFG2_SPLIT
    kv = PagedKV(layers, 8, 128, max_tokens=n, page_rows=64, device=dev)
    kv.reserve(n)
    reps = 200
    tabs = []
    for _ in range(reps):
        tabs.append(PageTable(kv.table.num_pages, 64))
        tabs[-1].reserve(n)
    tabs[0].splice(Split(a, c0, c))  # first call pays numpy's lazy imports
    t0 = time.perf_counter()
    for tab in tabs[1:]:
        tab.splice(Split(a, c0, c))
    host_us = (time.perf_counter() - t0) / (reps - 1) * 1e6
    runs_c = kv.table._cut(c0, c0 + c)
    ct = PageTable.tiles_of(runs_c)
    ctiles = torch.from_numpy(ct).to(dev)
    cs, cs_ptr = cos_sin_table(a - c0, workloads.inv_freq())
    kp = (ctypes.c_void_p * layers)(*[t.data_ptr() for t in kv.k])
    L = lib()
    sp, sh, sr = kv._strides()

    def run():
        check("tc_paged_rotate_keys", L.tc_paged_rotate_keys(kp, layers, 8, 128, 64, kv.table.num_pages, sp, sh, sr,
                                                             ctiles.data_ptr(), ct.shape[0], cs_ptr, TC_BF16,
                                                             torch.cuda.current_stream(dev).cuda_stream))
    for _ in range(warmup):
        run()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    e1.synchronize()
    barrier(dist)
    rot_ms = e0.elapsed_time(e1) / steps
    del kv, cs
    torch.cuda.empty_cache()
    # (3) prefill of a 512-token chunk over a spliced 98k-token paged cache: straight over the pages
    # vs gather-then-contiguous-kernel (the gather is what a paged cache without it would pay)
    from threadcut_b200.prefill import prefill_attention
    kv = PagedKV(1, 8, 128, max_tokens=100000, page_rows=64, device=dev)
    kv.reserve(99000)
    kv.write(0, torch.randn(8, 99000, 128, generator=g, device=dev).to(torch.bfloat16),
             torch.randn(8, 99000, 128, generator=g, device=dev).to(torch.bfloat16))
    kv.splice(Split(1000, 1726, 97274), workloads.inv_freq())  # 98,274 tokens, runs cut inside pages
    kv.reserve(512)
    kv.write(0, torch.randn(8, 512, 128, generator=g, device=dev).to(torch.bfloat16),
             torch.randn(8, 512, 128, generator=g, device=dev).to(torch.bfloat16))
    q = torch.randn(1, 32, 512, 128, generator=g, device=dev).to(torch.bfloat16)

    def timed(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / reps
    pf_paged = timed(lambda: kv.prefill(0, q, workloads.SCALE))
    kc, vc = kv.gather(0)
    pf_contig = timed(lambda: prefill_attention(q, kc[None], vc[None], workloads.SCALE))
    pf_gather = timed(lambda: kv.gather(0))
    n_pf = kv.n
    del kv, kc, vc, q
    torch.cuda.empty_cache()
    return dec_ms, rot_ms, 2 * c * 8 * 128 * 2, host_us, tiles, (pf_paged, pf_contig, pf_gather, n_pf)


def time_split_128k(dev, reps=20):
    """split() of a config-5-like request (128k cached tokens, a 32k span pruned mid-context, a
    300-token fresh tail) on the device (tokens already on the GPU, result read back) and with the
    host rule on Python lists (the reference's path). Returns (device us, host us)."""
    import time
    import numpy as np
    from threadcut_b200.match import split, split_device
    rng = np.random.default_rng(0)
    cached = rng.integers(0, 151936, workloads.CFG5_CTX)
    new = np.concatenate([cached[:49152], cached[81920:], rng.integers(0, 151936, 300)])
    cd = torch.as_tensor(cached, device=dev, dtype=torch.int32)
    nd = torch.as_tensor(new, device=dev, dtype=torch.int32)
    want = split(cached.tolist(), new.tolist())
    for _ in range(3):
        assert split_device(cd, nd) == want
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        split_device(cd, nd)
    dev_us = (time.perf_counter() - t) / reps * 1e6
    cl, nl = cached.tolist(), new.tolist()
    t = time.perf_counter()
    for _ in range(3):
        split(cl, nl)
    host_us = (time.perf_counter() - t) / 3 * 1e6
    return dev_us, host_us


def bf16_peak():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def time_prefill(steps, warmup, dev, lq=512, lk=98304):
    """The engine's prefill after a splice (config-5-like: a 512-token chunk over a 98k-token cache,
    32 q / 8 kv heads, d 128): the tcgen05 GQA prefill kernel, SDPA's GQA mode, and the reference's
    own path (repeat_kv + SDPA with the explicit mask, threadcut/attention.py:43-46). Returns ms of
    each and the useful FLOPs (visible query-key pairs only)."""
    import torch.nn.functional as F
    from threadcut_b200.attention import repeat_kv
    from threadcut_b200.prefill import causal_offset_mask, prefill_attention
    g = torch.Generator(device=dev).manual_seed(88)
    q = torch.randn(1, 32, lq, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, 8, lk, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, 8, lk, 128, generator=g, device=dev).to(torch.bfloat16)
    mask = causal_offset_mask(lq, lk, dev)[None, None]

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / steps

    ours = timed(lambda: prefill_attention(q, k, v, workloads.SCALE))
    gqa = timed(lambda: F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=workloads.SCALE,
                                                       enable_gqa=True))
    ref = timed(lambda: F.scaled_dot_product_attention(q, repeat_kv(k, 4), repeat_kv(v, 4), attn_mask=mask,
                                                       scale=workloads.SCALE))
    pairs = lq * (lk - lq) + lq * (lq + 1) // 2
    return ours, gqa, ref, 4.0 * 32 * pairs * 128


def time_cfg5_step(steps, warmup, dev):
    """Config 5 end to end: random-init Qwen3-4B (bf16) whose 36-layer cache holds 131,072 tokens,
    spliced with Split(49152, 81920, 49152) (the pruned span dropped, the suffix re-rotated by -32768)
    to 98,304 tokens, then one greedy decode token per step through the HF model with
    threadcut_b200's attention plugin: forward + argmax read back to the host, as the reference's
    engine does per token (threadcut/engine.py:66-73). The appended row is cropped after each step
    so every step decodes at the same length. Timed three ways: eager (the engine's path), the same
    forward replayed from a CUDA graph, and eager with HF's SDPA attention (the stock torch path).
    Returns a dict of ms per token, the splice ms and the step's algorithmic bytes."""
    from transformers import AutoModelForCausalLM
    from threadcut_b200 import attention as tc_attention
    from threadcut_b200.kv import new_cache, splice
    from threadcut_b200.match import Split
    torch.manual_seed(0)
    cfg = workloads.qwen3_4b_config()
    with torch.device(dev):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation=tc_attention.NAME)
    model.eval()
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    ctx = workloads.CFG5_CTX
    lo, hi = workloads.CFG5_PRUNE
    s = Split(lo, hi, ctx - hi)
    cache = new_cache(cfg)
    gen = torch.Generator(device=dev).manual_seed(0)
    for layer in cache.layers:
        k = torch.randn(1, workloads.HKV, ctx, workloads.D, generator=gen, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, workloads.HKV, ctx, workloads.D, generator=gen, device=dev, dtype=torch.bfloat16)
        layer.update(k, v)
        del k, v
    warm = new_cache(cfg)  # a small splice first: the timed one then pays no first-launch setup
    for layer in warm.layers:
        layer.update(*(torch.zeros(1, workloads.HKV, 96, workloads.D, device=dev, dtype=torch.bfloat16),) * 2)
    splice(warm, Split(16, 48, 48), model.model.rotary_emb.inv_freq)
    del warm
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    splice(cache, s, model.model.rotary_emb.inv_freq)
    e1.record()
    e1.synchronize()
    splice_ms = e0.elapsed_time(e1)
    n = s.a + s.c
    x = torch.tensor([[1234]], device=dev)

    def crop():
        for layer in cache.layers:
            layer.crop(n)

    def eager():
        tok = model(input_ids=x, past_key_values=cache, use_cache=True).logits[0, -1].argmax()
        tok.item()
        crop()

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / steps

    def graph_ms(key):
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                tok = model(input_ids=x, past_key_values=cache, use_cache=True).logits[0, -1].argmax()
            crop()

            def replay():
                graph.replay()
                tok.item()

            out[key] = timed(replay)
            del graph
        except Exception as exc:  # a host op the capture cannot hold: report it, keep the eager number
            crop()
            out[key] = None
            out[key.replace("_ms", "_error")] = f"{type(exc).__name__}: {str(exc)[:160]}"

    out = {"splice_ms": splice_ms, "n": n, "weight_bytes": weight_bytes,
           "kv_bytes": LAYERS * decode_bytes(n)}
    with torch.no_grad():
        out["eager_ms"] = timed(eager)
        with torch.cuda.nvtx.range("cfg5_step"):  # one eager step, for a profiler's launch list
            eager()
        torch.cuda.synchronize(dev)
        graph_ms("graph_ms")
        # the same calls with the one-token step routed through the fused step (tp.accelerate)
        from threadcut_b200 import tp as tc_tp
        tc_tp.accelerate(model)
        out["fused_eager_ms"] = timed(eager)
        graph_ms("fused_graph_ms")
        tc_tp.restore(model)
        torch.cuda.empty_cache()
        model.set_attn_implementation("sdpa")
        for layer in cache.layers:
            layer.fuse_append = False  # SDPA reads the cache itself: appends must be written, not deferred
        out["sdpa_eager_ms"] = timed(eager)
        graph_ms("sdpa_graph_ms")
    del model, cache
    torch.cuda.empty_cache()
    return out


def kernel_family(name):
    """Short name of a device activity in a launch list: this library's kernels by name and
    template flags (the dtype dropped), everything else by its library."""
    base = name.split("(")[0].replace("void ", "").strip()
    if base.startswith("tc::"):
        return base.replace("__nv_bfloat16, ", "").replace("__nv_bfloat16", "").replace("<>", "")
    if "nccl" in base:
        return "nccl"
    if base.startswith("Memcpy") or base.startswith("Memset"):
        return base.split(" ")[0].lower()
    return "torch (argmax, embedding, cos/sin)"


def serial_launches(dec, tok, n, dev, rank, dist, timed, steps=3):
    """Launch list of the config-5 step (`dec`) with programmatic dependent launch off
    (tc_set_pdl(0) while capturing its graph), so each kernel runs alone and the per-kernel device
    times add up to the step: per kernel family, launches and µs per step and the share, recorded
    by torch.profiler's CUDA activity on rank 0 (every rank replays: the sums need all of them).
    Also the replay time of that graph (max over ranks), against which the overlapped graph's time
    shows what the overlap saves."""
    from torch.profiler import ProfilerActivity, profile
    from threadcut_b200._lib import lib
    prev = lib().tc_set_pdl(0)
    try:
        graph, out = dec.capture(tok, n)
    finally:
        lib().tc_set_pdl(prev)

    def replay():
        graph.replay()
        int(out)

    serial_ms = timed(replay)
    barrier(dist)
    prof = None
    if rank == 0:
        prof = profile(activities=[ProfilerActivity.CUDA])
        prof.start()
    for _ in range(steps):
        replay()
    torch.cuda.synchronize(dev)
    barrier(dist)
    res = {"graph_ms": round(serial_ms, 3)}
    if prof is not None:
        prof.stop()
        rows = {}
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA and ev.device_time_total > 0:
                r = rows.setdefault(kernel_family(ev.name), [0, 0.0])
                r[0] += 1
                r[1] += ev.device_time_total
        total = sum(r[1] for r in rows.values()) or 1.0
        res["kernel_us_per_step"] = round(total / steps, 1)
        res["kernels"] = [[k, round(c / steps, 1), round(us / steps, 1), round(us / total, 4)]
                          for k, (c, us) in sorted(rows.items(), key=lambda kv: -kv[1][1])]
    del graph
    return res


def time_cfg5_tp(steps, warmup, dev, dist, rank, world, launches=None, summary=True):
    """Config 5 over `world` GPUs: threadcut_b200.tp.TPDecoder (rank r holds KV heads
    head_shard(8, r, world), their query heads, 1/world of the MLP and of the vocabulary; two
    all-reduces per layer) decoding one greedy token of random-init Qwen3-4B over the 131,072-token
    cache spliced to 98,304 (each rank splices its own heads). Every rank first computes the
    expected token the torch way: HF's forward with SDPA attention over the full-head cache spliced
    the same way (the same seeded K/V on every rank), and the decoder's token is compared with it.
    Each timed step is the token's forward plus the next token read back to the host; the appended
    row is cropped after each step so every step decodes at the same length. Eager and replayed from
    a CUDA graph (the all-reduces inside it). Returns a dict (times max over ranks), with
    `launches_serial` (serial_launches) when `summary`."""
    from transformers import AutoModelForCausalLM
    from threadcut_b200.kv import new_cache, splice as kv_splice
    from threadcut_b200.match import Split
    from threadcut_b200.tp import TPDecoder
    torch.manual_seed(0)
    cfg = workloads.qwen3_4b_config()
    with torch.device(dev):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16, attn_implementation="sdpa")
    model.eval()
    dec = TPDecoder(model, dev, world=world, rank=rank)
    shard_bytes = sum(t.numel() * t.element_size() for w in dec.layers_w for t in vars(w).values()
                      if isinstance(t, torch.Tensor)) + dec.lm_head.numel() * dec.lm_head.element_size()
    inv = model.model.rotary_emb.inv_freq.detach().to(dev)
    ctx = workloads.CFG5_CTX
    lo, hi = workloads.CFG5_PRUNE
    s = Split(lo, hi, ctx - hi)
    n = s.a + s.c
    ref_cache = new_cache(model.config)  # GrowingLayers; no fused append under SDPA attention
    gen = torch.Generator(device=dev).manual_seed(0)
    for i in range(len(dec.layers)):
        k = torch.randn(1, workloads.HKV, ctx, workloads.D, generator=gen, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, workloads.HKV, ctx, workloads.D, generator=gen, device=dev, dtype=torch.bfloat16)
        dec.load(i, k, v)
        ref_cache.layers[i].update(k, v)
        del k, v
    tok = torch.tensor([1234], device=dev)
    with torch.no_grad():
        kv_splice(ref_cache, s, inv)
        ref_logits = model(input_ids=tok.view(1, 1), past_key_values=ref_cache, use_cache=True).logits[0, -1].float()
    ref_top1 = int(ref_logits.argmax())
    del model, ref_cache
    torch.cuda.empty_cache()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    dec.splice(s, inv)
    e1.record()
    e1.synchronize()
    splice_ms = max_over_ranks(e0.elapsed_time(e1), dist)

    def eager():
        int(dec.step(tok, n))
        dec.crop(n)

    def timed(fn):
        for _ in range(warmup):
            fn()
        barrier(dist)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        b.synchronize()
        barrier(dist)
        return max_over_ranks(a.elapsed_time(b) / steps, dist)

    with torch.no_grad():
        logits = dec.logits(tok, n)
        dec.crop(n)
        step_tok = int(dec.step(tok, n))
        dec.crop(n)
        corr = torch.corrcoef(torch.stack([logits, ref_logits]))[0, 1].item()
        ok = float(step_tok == ref_top1 and int(logits.argmax()) == ref_top1)
        top1_ok = -max_over_ranks(-ok, dist) == 1.0  # every rank agrees
        eager_ms = timed(eager)
        with torch.cuda.nvtx.range("cfg5_tp_step"):  # one eager step, for a profiler's launch list
            eager()
        torch.cuda.synchronize(dev)
        graph, out, cap = None, None, 1.0
        try:
            graph, out = dec.capture(tok, n)
        except Exception:  # a host op the capture cannot hold: every rank skips the replay
            cap = 0.0
        cap = -max_over_ranks(-cap, dist)  # min over ranks: replay only if every rank captured
        graph_ms, graph_tok = None, None
        if cap:
            def replay():
                graph.replay()
                int(out)

            graph_ms = timed(replay)
            graph_tok = int(out)
            if launches:  # every rank replays (the sums need all ranks); rank 0 records
                import contextlib
                from torch.profiler import ProfilerActivity, profile
                barrier(dist)
                ctx = profile(activities=[ProfilerActivity.CUDA]) if rank == 0 else contextlib.nullcontext()
                with ctx as prof:
                    for _ in range(3):
                        replay()
                barrier(dist)
                if rank == 0:
                    launch_list(prof, launches, 3)
        del graph
        nccl_ms = None
        # the same graph with the sums as separate launches: a GEMV, the collective library's
        # all-reduce (N > 1) and the residual add + norm kernel, then the next GEMV
        if dec.use_peer_sums:
            dec.use_peer_sums = False
            graph, out = dec.capture(tok, n)

            def replay():
                graph.replay()
                int(out)

            nccl_ms = timed(replay)
            ok = float(int(out) == ref_top1)
            top1_ok = top1_ok and -max_over_ranks(-ok, dist) == 1.0
            del graph
            dec.use_peer_sums = True
        serial = serial_launches(dec, tok, n, dev, rank, dist, timed) if (cap and summary) else None
    dec.close()
    del dec
    torch.cuda.empty_cache()
    return {"eager_ms": eager_ms, "graph_ms": graph_ms, "nccl_graph_ms": nccl_ms, "splice_ms": splice_ms,
            "launches_serial": serial, "world": world,
            "bytes": shard_bytes + LAYERS * (4096 // world * n + 16384 // world),
            "top1_ok": bool(top1_ok and (graph_tok is None or graph_tok == ref_top1)), "token": step_tok,
            "sdpa_token": ref_top1, "logit_corr": round(corr, 6),
            "logit_max_abs": round(float((logits - ref_logits).abs().max()), 4)}


def time_cfg4(steps, warmup, dev, dist, distinct=2):
    """Config 4: 64 ragged sequences (lengths uniform in [1024, 16384], seeded), one contiguous K/V
    cache per sequence and layer, one query token each. A step is 36 decode_attention_ragged launches
    cycling `distinct` layer caches (~2.3 GB each, far above L2), replayed from a CUDA graph. Returns
    (ms per step, algorithmic bytes per launch)."""
    from threadcut_b200.flash_decode import RaggedKV, decode_attention_ragged
    lengths = workloads.cfg4_lengths()
    g = torch.Generator(device=dev).manual_seed(44)
    kvs = []
    for _ in range(distinct):
        ks = [torch.randn(8, n, 128, generator=g, device=dev).to(torch.bfloat16) for n in lengths]
        vs = [torch.randn(8, n, 128, generator=g, device=dev).to(torch.bfloat16) for n in lengths]
        kvs.append(RaggedKV(ks, vs, lengths))
    q = torch.randn(len(lengths), 8, 4, 128, generator=g, device=dev).to(torch.bfloat16)

    def launch_all():
        for i in range(LAYERS):
            decode_attention_ragged(q, kvs[i % distinct], workloads.SCALE)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        launch_all()  # warm-up on the capture stream (its workspace exists before capture)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            launch_all()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    ms = time_graph(graph, steps, warmup, dist)
    del graph, kvs
    torch.cuda.empty_cache()
    return ms, 4096 * sum(lengths) + len(lengths) * 16384


def time_strong_128k(steps, warmup, dev, dist, rank, world, layers=LAYERS):
    """Strong scaling of one long sequence (config 5's 128k context, attention only), two ways.
    Head-sharded: the 8 KV heads are split over the ranks (head_shard), each rank decodes its heads
    for all layers, no collective. Sequence-sharded (N > 1): each rank holds all heads of a
    128k / N-token slice, computes each layer's partial, and the step ends with the combine
    (SeqShardedStep: all-gathers + one LSE merge). Returns (head ms, sequence ms or None) per
    36-layer step on this rank."""
    from threadcut_b200.sharded import head_shard
    n = workloads.CFG5_CTX
    h0, h1 = head_shard(workloads.HKV, rank, world)
    hl = h1 - h0
    g = torch.Generator(device=dev).manual_seed(5000 + rank)
    ks = [torch.randn(hl, n, 128, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(hl, n, 128, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
    qs = [torch.randn(hl, 4, 128, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
    outs = [torch.empty_like(q) for q in qs]
    graph = capture_step(qs, ks, vs, outs, dev)
    head_ms = time_graph(graph, steps, warmup, dist)
    del graph, ks, vs, qs
    torch.cuda.empty_cache()
    seq_ms = None
    if world > 1:
        nl = n // world
        ks = [torch.randn(8, nl, 128, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
        vs = [torch.randn(8, nl, 128, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
        gq = torch.Generator(device=dev).manual_seed(5999)
        qs = [torch.randn(8, 4, 128, generator=gq, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
        seq = SeqShardedStep(layers, dev, dist, world)
        graph = capture_step(qs, ks, vs, seq.outs, dev, lses=seq.lses, combine=seq.combine)
        seq_ms = time_graph(graph, steps, warmup, dist)
        del graph, ks, vs, qs
        seq.close()
        del seq
        torch.cuda.empty_cache()
    return head_ms, seq_ms


def cpu_threads():
    """Host cores this process may run on (its affinity mask), used as the CPU baseline's thread
    count at every N: torchrun sets OMP_NUM_THREADS=1, which would otherwise leave one core."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


_CPU_BUFS = {}


def cpu_layers(dtype, layers_in_memory=4):
    """Seeded 16k decode inputs on the host, built once per dtype: [(q, K, V)] x layers_in_memory."""
    if dtype not in _CPU_BUFS:
        g = torch.Generator().manual_seed(0)
        _CPU_BUFS[dtype] = [(torch.randn(1, 32, 1, 128, generator=g).to(dtype),
                             torch.randn(1, 8, N_CTX, 128, generator=g).to(dtype),
                             torch.randn(1, 8, N_CTX, 128, generator=g).to(dtype)) for _ in range(layers_in_memory)]
    return _CPU_BUFS[dtype]


def cpu_reference_us_per_layer(seconds=10.0, max_layers=None, dtype=torch.bfloat16):
    """The reference's CPU decode path (threadcut/attention.py:41-42: query heads folded, SDPA
    against the unexpanded cache; oracle/torch_ref.py) on 16k layers in `dtype`, with every host
    core. Returns (us per layer, layers timed, threads)."""
    from oracle.torch_ref import folded_decode
    threads = cpu_threads()
    torch.set_num_threads(threads)
    bufs = cpu_layers(dtype)
    layers_in_memory = len(bufs)
    with torch.no_grad():
        folded_decode(*bufs[0], workloads.SCALE)  # warm-up
        t0 = time.perf_counter()
        done = 0
        while True:
            q, k, v = bufs[done % layers_in_memory]
            folded_decode(q, k, v, workloads.SCALE)
            done += 1
            el = time.perf_counter() - t0
            if el >= seconds or (max_layers and done >= max_layers):
                break
    return el / done * 1e6, done, threads


def cpu_shift_us_per_layer(reps=20):
    """The reference's CPU splice (threadcut/kv.py:83-92: shift_keys of C plus the value clone,
    written back in place) of config 2, Split(2048, 4096, 4096) of an 8192-token bf16 layer, with
    every host core. Returns (median us per layer, threads)."""
    from oracle.torch_ref import growing_splice
    threads = cpu_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    a, c0, c = workloads.CFG2_SPLIT
    bufs = [(torch.randn(1, 8, workloads.CFG2_N, 128, generator=g).to(torch.bfloat16),
             torch.randn(1, 8, workloads.CFG2_N, 128, generator=g).to(torch.bfloat16)) for _ in range(4)]
    inv = workloads.inv_freq()
    growing_splice(*bufs[0], a, c0, c, inv)  # warm-up
    times = []
    for i in range(reps):
        kb, vb = bufs[i % len(bufs)]
        t0 = time.perf_counter()
        growing_splice(kb, vb, a, c0, c, inv)
        times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6, threads


def run_ours(args, rank, local, world, dist):
    dev = torch.device("cuda", local)
    hbm, peak_kind = peaks()
    # the step: one sequence of 16k * world tokens, 36 layers, sharded by token range over the
    # ranks: every rank holds all 8 KV heads of its own 16k-token slice (the same 67 MB per layer as
    # one GPU at 16k) and computes each layer's fp32 partial and LSE; the step ends with the combine
    # (all-gather of the step's partials + one LSE merge launch). At 1 GPU: the 16k headline.
    hl = workloads.HKV
    n_job = N_CTX * world
    rank_bytes = 512 * hl * N_CTX + 2048 * hl  # K+V of the rank's slice + q + o, one layer
    gq = torch.Generator(device=dev).manual_seed(1001)  # the sequence's queries: the same on every rank
    qs = [torch.randn(hl, 4, 128, generator=gq, device=dev).to(torch.bfloat16) for _ in range(LAYERS)]
    _, ks, vs = build_layers(N_CTX, LAYERS, dev, seed=1000 + rank)
    if world == 1:
        seq = None
        outs = [torch.empty_like(q) for q in qs]
        graph = capture_step(qs, ks, vs, outs, dev)
    else:
        seq = SeqShardedStep(LAYERS, dev, dist, world)
        graph = capture_step(qs, ks, vs, seq.outs, dev, lses=seq.lses, combine=seq.combine)
    with ClockSampler(local) as clk:
        ms = time_graph(graph, args.steps, args.warmup, dist)
    ms = max_over_ranks(ms, dist)
    us_layer_rank = ms * 1000.0 / LAYERS  # one rank's time per layer (incl. back-to-back gaps)
    value = ms * 1000.0 / (LAYERS * world)  # per 16k tokens of context per layer
    achieved = rank_bytes / (us_layer_rank * 1e-6) / 1e9
    nccl_ms = None
    if world > 1:  # the combine's share: the same decode launches without it, and with NCCL's
        g_nc = capture_step(qs, ks, vs, seq.outs, dev, lses=seq.lses)
        nocombine_ms = max_over_ranks(time_graph(g_nc, args.steps, args.warmup, dist), dist)
        del g_nc
        g_nc = capture_step(qs, ks, vs, seq.outs, dev, lses=seq.lses, combine=seq.combine_nccl)
        nccl_ms = max_over_ranks(time_graph(g_nc, args.steps, args.warmup, dist), dist)
        del g_nc
        g_plain = capture_step(qs, ks, vs, seq.outs, dev, stable=False, lses=seq.lses, combine=seq.combine)
    else:
        nocombine_ms = ms
        g_plain = capture_step(qs, ks, vs, outs, dev, stable=False)
    plain_ms = max_over_ranks(time_graph(g_plain, args.steps, args.warmup, dist), dist)
    del g_plain
    e2e_ms, h2d, d2h = time_e2e(qs, ks, vs, args.steps, args.warmup, dist, dev, world)
    e2e_ms = max_over_ranks(e2e_ms, dist)
    del graph, qs, ks, vs
    if seq is not None:
        seq.close()
    del seq
    torch.cuda.empty_cache()
    # the single-GPU 16k layers (replicated on every rank) for the comparators and the fused append
    qs, ks, vs = build_layers(N_CTX, LAYERS, dev, seed=1000 + rank)
    sdpa_ms = max_over_ranks(time_sdpa_16k(qs, ks, vs, args.steps, args.warmup, dist), dist)
    fused_ms, unfused_ms = time_append_16k(qs, ks, vs, args.steps, args.warmup, dist)
    fused_ms, unfused_ms = max_over_ranks(fused_ms, dist), max_over_ranks(unfused_ms, dist)
    del qs, ks, vs
    # context-length sweep of config 3 (same kernel, 4k and 32k), and the RoPE-shift splice
    sweep = {}
    for n in (4096, 32768):
        q2, k2, v2 = build_layers(n, LAYERS, dev, seed=2000 + n)
        o2 = [torch.empty_like(q) for q in q2]
        g2 = capture_step(q2, k2, v2, o2, dev)
        t = max_over_ranks(time_graph(g2, args.steps, args.warmup, dist), dist)
        sweep[str(n)] = {"us_per_layer": round(t * 1000 / LAYERS, 3),
                         "frac": round((4096 * n + 16384) / (t * 1e-3 / LAYERS) / 1e9 / hbm, 4)}
        del g2, q2, k2, v2, o2
    if world == 1:
        sweep[str(N_CTX)] = {"us_per_layer": round(us_layer_rank, 3), "frac": round(achieved / hbm, 4)}
    # configs 1 and 2 as decode steps: 1,536-token layers, and the 6,144 rows left after the
    # config-2 splice as views of 8,192-row buffers (the GrowingLayer layout after a splice)
    short = {}
    for name, n, cap in (("cfg1_1536", 1536, 1536), ("cfg2_6144_of_8192", 6144, 8192)):
        k2, v2 = workloads.layer_kv(n, LAYERS, dev, seed=3000 + n, cap=cap)
        gq2 = torch.Generator(device=dev).manual_seed(4000 + n)
        q2 = [torch.randn(8, 4, 128, generator=gq2, device=dev).to(torch.bfloat16) for _ in range(LAYERS)]
        o2 = [torch.empty_like(q) for q in q2]
        g2 = capture_step(q2, k2, v2, o2, dev)
        t = max_over_ranks(time_graph(g2, args.steps, args.warmup, dist), dist)
        short[name] = {"us_per_layer": round(t * 1000 / LAYERS, 3), "bytes_per_layer": 4096 * n + 16384,
                       "frac": round((4096 * n + 16384) / (t * 1e-3 / LAYERS) / 1e9 / hbm, 4)}
        del g2, q2, k2, v2, o2
    torch.cuda.empty_cache()
    shift_ms = max_over_ranks(time_shift(args.steps, args.warmup, dev, dist), dist)
    shift_gbs = SHIFT_BYTES_PER_LAYER * LAYERS / (shift_ms * 1e-3) / 1e9
    c4_ms, c4_bytes = time_cfg4(args.steps, args.warmup, dev, dist)
    c4_ms = max_over_ranks(c4_ms, dist)
    cfg4 = {"us_per_layer": round(c4_ms * 1000 / LAYERS, 3),
            "frac": round(c4_bytes / (c4_ms * 1e-3 / LAYERS) / 1e9 / hbm, 4), "bytes_per_layer": c4_bytes,
            "workload": "cfg4: 64 ragged sequences, lengths uniform in [1024,16384] (seeded), per-sequence bf16 "
                        "K/V caches, 32 q / 8 kv heads, d 128, 36 launches per step over 2 distinct layer caches"}
    pg_dec_ms, pg_rot_ms, pg_rot_bytes, pg_host_us, pg_tiles, pg_pf = time_paged(args.steps, args.warmup, dev, dist)
    pg_dec_ms, pg_rot_ms = max_over_ranks(pg_dec_ms, dist), max_over_ranks(pg_rot_ms, dist)
    split_dev_us, split_host_us = time_split_128k(dev)
    pf_ms, pf_gqa_ms, pf_ref_ms, pf_flops = time_prefill(min(args.steps, 10), args.warmup, dev)
    tc_peak, tc_peak_kind = bf16_peak()
    st_head, st_seq = time_strong_128k(args.steps, args.warmup, dev, dist, rank, world)
    st_head = max_over_ranks(st_head, dist)
    st_seq = max_over_ranks(st_seq, dist) if st_seq is not None else None
    best = min(st_head, st_seq) if st_seq is not None else st_head
    strong = {"us_per_layer": round(best * 1000 / LAYERS, 3), "n": workloads.CFG5_CTX,
              "head_sharded_us_per_layer": round(st_head * 1000 / LAYERS, 3),
              "seq_sharded_us_per_layer": None if st_seq is None else round(st_seq * 1000 / LAYERS, 3),
              "kv_heads_per_rank_head_sharded": workloads.HKV // world,
              "workload": "one 128k-token sequence, 36 layers, attention only, on N GPUs: head-sharded (8/N KV "
                          "heads per GPU, no collective) and sequence-sharded (all heads of a 128k/N-token slice per "
                          "GPU, partials all-gathered and LSE-merged once per step inside the graph); us_per_layer = "
                          "the faster; per-layer latency, max over ranks; speedup = the 1-GPU value / this",
              "frac_per_gpu": round(decode_bytes(workloads.CFG5_CTX) / world / (best * 1e-3 / LAYERS) / 1e9
                                    / hbm, 4)}
    cfg5 = None
    if world == 1:
        c5 = time_cfg5_step(min(args.steps, 10), args.warmup, dev)
        step_bytes = c5["weight_bytes"] + c5["kv_bytes"]
        rnd = lambda v: None if v is None else round(v, 3)  # noqa: E731
        cfg5 = {"eager_ms": rnd(c5["eager_ms"]), "graph_ms": rnd(c5["graph_ms"]),
                "fused_eager_ms": rnd(c5.get("fused_eager_ms")), "fused_graph_ms": rnd(c5.get("fused_graph_ms")),
                "sdpa_eager_ms": rnd(c5["sdpa_eager_ms"]), "sdpa_graph_ms": rnd(c5["sdpa_graph_ms"]),
                "splice_ms": rnd(c5["splice_ms"]),
                "n": c5["n"], "bytes_per_token": step_bytes,
                "ideal_ms": round(step_bytes / (hbm * 1e9) * 1e3, 3),
                "what": "one greedy decode token of random-init Qwen3-4B over the spliced 98,304-token cache "
                        "(131,072 tokens, Split(49152, 81920, 49152) timed once as splice_ms): HF forward with "
                        "threadcut_b200's attention + argmax read back, eager and replayed from a CUDA graph; "
                        "fused_*: the same model call after tp.accelerate(model) (the one-token step runs the fused "
                        "TPDecoder step at world 1 over the same cache), the call the reference's engine makes; vs "
                        "the same with HF's SDPA attention (under capture HF passes SDPA an explicit mask); ideal_ms = weights + K/V bytes at the measured HBM peak"}
        for key in ("graph_error", "fused_graph_error", "sdpa_graph_error"):
            if key in c5:
                cfg5[key] = c5[key]
    tp = time_cfg5_tp(min(args.steps, 10), args.warmup, dev, dist, rank, world)
    cfg5_tp = {"eager_ms": round(tp["eager_ms"], 3),
               "graph_ms": None if tp["graph_ms"] is None else round(tp["graph_ms"], 3),
               "splice_ms": round(tp["splice_ms"], 3), "bytes_per_rank": tp["bytes"],
               "ideal_ms": round(tp["bytes"] / (hbm * 1e9) * 1e3, 3),
               ("nccl_graph_ms" if world > 1 else "separate_sums_graph_ms"):
                   None if tp["nccl_graph_ms"] is None else round(tp["nccl_graph_ms"], 3),
               "top1_ok": tp["top1_ok"], "token": tp["token"], "sdpa_token": tp["sdpa_token"],
               "logit_corr": tp["logit_corr"], "logit_max_abs": tp["logit_max_abs"],
               "what": f"one greedy decode token of random-init Qwen3-4B over the spliced 98,304-token cache, "
                       f"tensor-parallel over {world} GPU(s) (threadcut_b200.tp.TPDecoder: KV heads, their query "
                       f"heads, 1/{world} of the MLP and vocabulary per rank; 2 sums over the ranks per layer through "
                       f"peer memory, each completed into the residual by the row-split projection, the next "
                       f"projection staging RMSNorm of it: 5 launches per layer (nccl_graph_ms, N > 1, or "
                       f"separate_sums_graph_ms, N = 1: the same graph with separate GEMV, NCCL all-reduce (N > 1) "
                       f"and residual add + norm launches instead)), next token "
                       f"read back each step; eager and CUDA graph; max over ranks; top1_ok: the eager, "
                       f"graph and gathered-logit tokens equal HF's SDPA forward over the same spliced full cache "
                       f"(sdpa_token) on every rank; ideal_ms = one rank's weight + K/V bytes at the measured HBM "
                       f"peak (collectives not counted); launches_serial: the step's graph captured with programmatic "
                       f"dependent launch off, its replay time and per-kernel-family launches, µs per step and "
                       f"shares on rank 0 (torch.profiler CUDA activity)",
               "launches_serial": tp["launches_serial"]}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        us16, nl16, thr = cpu_reference_us_per_layer(args.cpu_seconds / 2, dtype=torch.bfloat16)
        us32, nl32, _ = cpu_reference_us_per_layer(args.cpu_seconds / 2, dtype=torch.float32)
        sh_us, _ = cpu_shift_us_per_layer()
        cpu = {"value": round(min(us16, us32), 2), "unit": "us/layer", "cores": thr, "kind": "port",
               "bf16_us_per_layer": round(us16, 2), "fp32_us_per_layer": round(us32, 2),
               "sample": f"{nl16} bf16 + {nl32} fp32 layers of 16k decode through the reference's CPU decode "
                         f"expression (threadcut/attention.py:41-42: F.scaled_dot_product_attention(q.reshape(1,8,4,128), "
                         f"K, V, scale) on CPU tensors, oracle/torch_ref.py), 4 distinct layer buffers cycled, "
                         f"~{args.cpu_seconds:.0f}s; value = the faster dtype",
               "shift": {"us_per_layer": round(sh_us, 1),
                         "gbs": round(SHIFT_BYTES_PER_LAYER / (sh_us * 1e-6) / 1e9, 2),
                         "sample": "config-2 splice of one bf16 layer, median of 20: shift_keys of C + value "
                                   "clone written back (threadcut/kv.py:20-25,83-92 on CPU tensors)"}}
    traffic = None  # DRAM bytes per launch from the committed ncu capture of this kernel and size
    tpath = os.path.join(HERE, "profiles", "decode_16k_traffic.txt")
    if os.path.exists(tpath):
        for line in open(tpath):
            if line.startswith("dram_bytes_per_launch:"):
                traffic = int(line.split(":", 1)[1])
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "us/layer", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic: seeded N(0,1) K/V and queries",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "n": n_job, "batch": 1,
                   "tokens_per_gpu": N_CTX,
                   "l2": f"inputs larger than L2 (36 distinct {rank_bytes / 1e6:.0f} MB layers per GPU = "
                         f"{LAYERS * rank_bytes / 1e9:.1f} GB per step)",
                   "parallelism": f"sequence-sharded over {world} GPU(s): each GPU holds all 8 KV heads of its own "
                                  f"{N_CTX}-token slice of the {n_job}-token sequence" +
                                  (" and computes each layer's fp32 partial + LSE; the step ends with the combine "
                                   "(one tc_peer_gather_merge launch inside the graph: the 36 layers' partials pushed "
                                   "to every rank through peer memory and LSE-merged)" if world > 1 else ""),
                   "value": "us per layer of the job / world = us per layer per 16k tokens of context (at 1 GPU: "
                            "the 16k decode; at 8: the 128k sequence, 16k tokens per GPU)",
                   "stable_rows": "n-1: every row but the newest declared stable, as in a decode step "
                                  "(tc_decode_attention_stable); see no_stable_rows for the plain entry point"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic if world == 1 else None,
                     "peak_kind": peak_kind, "kernel": "decode_mma_kernel<bf16,128,1>", "bytes_per_launch": rank_bytes,
                     "per": "one GPU's launch (its token slice); the job's layer time per GPU includes the combine"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_ms * 1000.0 / (LAYERS * world), 3), "unit": "us/layer", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "threadcut_b200.flash_decode.decode_attention per layer" if world == 1 else
                       "threadcut_b200.flash_decode.decode_attention_partial per layer over the rank's token slice, "
                       "then threadcut_b200.peer.GatherMerge (the step's partials pushed to every rank and merged)"},
        "combine": None if world == 1 else {
            "us_per_layer_without": round(nocombine_ms * 1000.0 / LAYERS, 3),
            "us_per_layer_with": round(us_layer_rank, 3),
            "us_per_layer_with_nccl": round(nccl_ms * 1000.0 / LAYERS, 3),
            "what": "the step's 36 partial-decode launches without the combine, with it (one tc_peer_gather_merge "
                    "launch: partials pushed to every rank through peer memory and merged), and with NCCL's "
                    "all-gathers + tc_merge_partials instead"},
        "gpu_launches": args.steps * LAYERS,
        "clocks": clk.summary(),
        "shift": {"value": round(shift_gbs, 1), "unit": "GB/s", "frac": round(shift_gbs / hbm, 4),
                  "us_per_layer": round(shift_ms * 1000 / LAYERS, 3),
                  "workload": "cfg2 splice Split(2048,4096,4096) of an 8192-token bf16 cache, 36 layers in one "
                              "in-place launch; K rotated + V moved, read+write bytes"},
        "cfg3_sweep": sweep,
        "cfg1_cfg2_decode": dict(short, what="36-layer decode graphs (stable rows) of config 1's 1,536-token layers and "
                                              "of config 2's 6,144 rows after the splice (views of 8,192-row buffers); "
                                              "launch-bound at these sizes"),
        "cfg4_ragged": cfg4,
        "append_16k": {"fused_us_per_layer": round(fused_ms * 1000.0 / LAYERS, 3),
                       "copy_then_decode_us_per_layer": round(unfused_ms * 1000.0 / LAYERS, 3),
                       "what": "a decode step's K/V append + attention per 16k layer: decode_attention_append "
                               "(one launch) vs two row copies then decode_attention (the reference's order)"},
        "prefill_512x98k": {
            "tcgen05_ms": round(pf_ms, 4), "sdpa_gqa_ms": round(pf_gqa_ms, 4), "reference_path_ms": round(pf_ref_ms, 4),
            "tflops": round(pf_flops / (pf_ms * 1e-3) / 1e12, 1),
            "roofline": {"bound": "tensor", "achieved": round(pf_flops / (pf_ms * 1e-3) / 1e12, 1), "peak": tc_peak,
                         "unit": "TFLOP/s", "frac": round(pf_flops / (pf_ms * 1e-3) / 1e12 / tc_peak, 4),
                         "peak_kind": tc_peak_kind},
            "what": "prefill of a 512-token chunk over a 98,304-token cache (32 q / 8 kv heads, d 128, causal with "
                    "the cache offset): tc_prefill_attention vs SDPA GQA mode vs the reference's repeat_kv + SDPA"},
        "paged": {
            "decode_16k_us_per_layer": round(pg_dec_ms * 1000.0 / LAYERS, 3),
            "decode_16k_frac": round(BYTES_PER_LAYER / (pg_dec_ms * 1e-3 / LAYERS) / 1e9 / hbm, 4),
            "decode_tiles": pg_tiles,
            "splice_cfg2_us_per_layer": round(pg_rot_ms * 1000.0 / LAYERS, 3),
            "splice_cfg2_gbs": round(pg_rot_bytes * LAYERS / (pg_rot_ms * 1e-3) / 1e9, 1),
            "splice_cfg2_frac": round(pg_rot_bytes * LAYERS / (pg_rot_ms * 1e-3) / 1e9 / hbm, 4),
            "splice_cfg2_bytes_per_layer": pg_rot_bytes,
            "splice_cfg2_host_table_us": round(pg_host_us, 2),
            "prefill_512_ms": round(pg_pf[0], 4), "prefill_512_contiguous_ms": round(pg_pf[1], 4),
            "gather_ms": round(pg_pf[2], 4), "prefill_cache_tokens": pg_pf[3],
            "what": "paged K/V cache (64-row pages): decode of the 36-layer 16k step over ragged runs (a splice "
                    "cut inside pages), and the cfg2 splice Split(2048,4096,4096) as B's pages dropped on the "
                    "host + C's keys re-rotated in place (values never move: half the contiguous splice's bytes); "
                    "compare decode with the headline value and the splice with shift.us_per_layer; prefill: a 512-token "
                    "chunk over a spliced ~98k-token paged cache straight over the pages vs the contiguous kernel on "
                    "a gathered copy (gather_ms = that copy)"},
        "split_128k": {"device_us": round(split_dev_us, 1), "host_numpy_us": round(split_host_us, 1),
                       "what": "match.split of a 128k cached / 97k new request: tc_split (tokens on the GPU, "
                               "result read back, wall clock) vs the host rule on Python lists"},
        "no_stable_rows": {"us_per_layer": round(plain_ms * 1000.0 / LAYERS, 3),
                           "frac": round(rank_bytes / (plain_ms * 1e-3 / LAYERS) / 1e9 / hbm, 4),
                           "what": "the same 36-layer step through plain tc_decode_attention (nothing declared "
                                   "stable: K/V are read only after the preceding launch finished)"},
        "gpu_comparators": {"torch_sdpa_folded_16k": {
            "us_per_layer": round(sdpa_ms * 1000 / LAYERS, 3),
            "frac": round(BYTES_PER_LAYER / (sdpa_ms * 1e-3 / LAYERS) / 1e9 / hbm, 4),
            "what": "the reference's own torch decode path (folded GQA SDPA) on the same 36 layers, same GPU"}},
        "strong_128k": strong,
        "cfg5_step": cfg5,
        "cfg5_tp": cfg5_tp,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def time_gemv(steps, warmup, dev, n, k, layers):
    """tc_gemv alone: `layers` distinct bf16 weights [n, k] (the gate|up projection of one Qwen3-4B
    layer at 1 GPU by default, 99.6 MB; together far above L2), one launch per weight per step,
    replayed from a CUDA graph. The algorithmic bytes of a launch are the weight (x and out are a
    few KB). Returns µs per launch and GB/s."""
    from threadcut_b200 import tp
    g = torch.Generator(device=dev).manual_seed(3)
    ws = [(torch.randn(n, k, generator=g, device=dev) * k ** -0.5).to(torch.bfloat16) for _ in range(layers)]
    x = torch.randn(1, k, generator=g, device=dev).to(torch.bfloat16)

    def launch_all():
        for w in ws:
            tp._gemv(x, w)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        launch_all()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            launch_all()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    ms = time_graph(graph, steps, warmup, None)
    us = ms * 1000 / layers
    hbm, kind = peaks()
    gbs = n * k * 2 / (us * 1e-6) / 1e9
    del graph, ws
    return {"gemv_n": n, "gemv_k": k, "us_per_launch": round(us, 3), "gbs": round(gbs, 1),
            "frac": round(gbs / hbm, 4), "peak_kind": kind}


def time_gemv_chain(steps, warmup, dev, tp_world, layers, dist=None):
    """The projections of the tensor-parallel step alone, one GPU with the per-rank shapes of
    `tp_world` ranks (Qwen3-4B): per layer q|k|v with the input norm staged (tc_gemv_rmsnorm),
    o_proj completing its sum into the residual (tc_gemv_allreduce_residual, world 1), gate|up with
    the post-attention norm staged, down_proj of the SwiGLU activation completing its sum; the
    attention output is a fixed input. `layers` distinct weight sets, replayed from a CUDA graph,
    with programmatic dependent launch on and off. Returns µs per layer, the weight bytes per layer
    and the per-kernel serialized shares."""
    from torch.profiler import ProfilerActivity, profile
    from threadcut_b200._lib import lib
    from threadcut_b200.peer import AllReduce
    hid, inter, d = 2560, 9728 // tp_world, 128
    nq, nkv = 32 // tp_world, 8 // tp_world
    g = torch.Generator(device=dev).manual_seed(4)
    bf = torch.bfloat16

    def mat(n, k):
        return (torch.randn(n, k, generator=g, device=dev) * k ** -0.5).to(bf)

    ws = [(mat((nq + 2 * nkv) * d, hid), mat(hid, nq * d), mat(2 * inter, hid), mat(hid, inter)) for _ in range(layers)]
    norm = (1 + 0.1 * torch.randn(hid, generator=g, device=dev)).to(bf)
    o_in = torch.randn(1, nq * d, generator=g, device=dev).to(bf)
    h0 = torch.randn(1, hid, generator=g, device=dev).to(bf)
    ar = AllReduce(hid, dev, world=1)
    h = h0.clone()
    wbytes = sum(t.numel() * 2 for t in ws[0])

    def chain():
        h.copy_(h0)
        ar.gemv_residual(o_in, ws[0][1], h)  # records the first sums of squares
        for wq, wo, wgu, wd in ws:
            ar.gemv_norm(h, norm, wq, 1e-6)
            ar.gemv_residual(o_in, wo, h)
            act = ar.gemv_norm_swiglu(h, norm, wgu, 1e-6)  # gate/up rows taken as interleaved
            ar.gemv_residual(act[0], wd, h)

    res = {"tp_world": tp_world, "layers": layers, "weight_mb_per_layer": round(wbytes / 1e6, 2)}
    for mode in (1, 0):
        prev = lib().tc_set_pdl(mode)
        try:
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                chain()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(graph, stream=s):
                    chain()
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize()
        finally:
            lib().tc_set_pdl(prev)
        ms = time_graph(graph, steps, warmup, None)
        key = "pdl" if mode else "serial"
        res[key + "_us_per_layer"] = round(ms * 1000 / layers, 3)
        if not mode:
            prof = profile(activities=[ProfilerActivity.CUDA])
            prof.start()
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            prof.stop()
            rows = {}
            for ev in prof.events():
                if ev.device_type == torch.autograd.DeviceType.CUDA and ev.device_time_total > 0:
                    r = rows.setdefault(kernel_family(ev.name), [0, 0.0])
                    r[0] += 1
                    r[1] += ev.device_time_total
            res["serial_kernels"] = [[k, c // 3, round(us / c, 2)] for k, (c, us) in
                                     sorted(rows.items(), key=lambda kv: -kv[1][1])]
        del graph
    hbm, _ = peaks()
    res["pdl_frac"] = round(wbytes / (res["pdl_us_per_layer"] * 1e-6) / 1e9 / hbm, 4)
    torch.cuda.synchronize()
    ar.close()
    return res


def launch_list(prof, path, steps):
    """Kernel launch list of a torch.profiler run: per kernel name, launches, total device µs and
    share, from the CUDA activity records (the device's own start/end stamps; nothing replayed)."""
    rows = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and ev.device_time_total > 0:
            r = rows.setdefault(ev.name, [0, 0.0])
            r[0] += 1
            r[1] += ev.device_time_total
    total = sum(r[1] for r in rows.values()) or 1.0
    with open(path, "w") as f:
        f.write(f"# kernel launches of {steps} graph-replayed steps (torch.profiler CUDA activity)\n")
        f.write("kernel\tlaunches\ttotal_us\tshare\tavg_us\n")
        for name, (cnt, us) in sorted(rows.items(), key=lambda kv: -kv[1][1]):
            f.write(f"{name}\t{cnt}\t{us:.1f}\t{us / total:.4f}\t{us / cnt:.2f}\n")


def run_partial(args, rank, local, world, dist):
    """Profiling helper: one leg at a chosen size, no CPU baseline or e2e (not the bench contract)."""
    dev = torch.device("cuda", local)
    out = {"only": args.only, "layers": args.layers, "ctx": args.ctx, "steps": args.steps}
    if args.only == "decode":
        qs, ks, vs = build_layers(args.ctx, args.layers, dev, seed=1000 + rank, heads=args.heads)
        outs = [torch.empty_like(q) for q in qs]
        res = {}
        for name, stable in (("stable", True), ("plain", False)):
            graph = capture_step(qs, ks, vs, outs, dev, stable=stable)
            ms = max_over_ranks(time_graph(graph, args.steps, args.warmup, dist), dist)
            us = ms * 1000 / args.layers
            nbytes = 512 * args.heads * args.ctx + 2048 * args.heads
            res[name] = {"us_per_layer": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
            del graph
        out.update(heads=args.heads, **res)
    elif args.only == "cfg5tp":
        tp = time_cfg5_tp(args.steps, args.warmup, dev, dist, rank, world, launches=args.launches)
        out.update({k: (round(v, 3) if isinstance(v, float) else v) for k, v in tp.items()}, world=world)
    elif args.only == "gemv":
        out.update(time_gemv(args.steps, args.warmup, dev, args.gemv_n, args.gemv_k, args.layers))
    elif args.only == "gemvchain":
        out.update(time_gemv_chain(args.steps, args.warmup, dev, args.heads, args.layers))
    elif args.only == "cfg5":
        c5 = time_cfg5_step(args.steps, args.warmup, dev)
        out.update({k: (round(v, 3) if isinstance(v, float) else v) for k, v in c5.items()})
    else:
        ms = max_over_ranks(time_shift(args.steps, args.warmup, dev, dist, layers=args.layers), dist)
        out.update(us_per_layer=round(ms * 1000 / args.layers, 3),
                   gbs=round(SHIFT_BYTES_PER_LAYER * args.layers / (ms * 1e-3) / 1e9, 1))
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_reference(args, rank, world):
    """The reference arm: threadcut's own CPU path for this workload (the torch expressions of
    oracle/torch_ref.py) on rank 0 with every host core; other ranks exit without work. A step is
    the 36-layer 16k decode in bf16 (the faster of bf16 and fp32 on CPUs measured so far; fp32 is
    timed once beside it)."""
    if rank != 0:
        return
    per_step = []
    threads = cpu_threads()
    for i in range(args.warmup + args.steps):
        us, nl, threads = cpu_reference_us_per_layer(seconds=1e9, max_layers=LAYERS, dtype=torch.bfloat16)
        if i >= args.warmup:
            per_step.append(us * LAYERS / 1000.0)  # ms per 36-layer step
    us32, _, _ = cpu_reference_us_per_layer(seconds=1e9, max_layers=LAYERS, dtype=torch.float32)
    sh_us, _ = cpu_shift_us_per_layer()
    ms = statistics.mean(per_step)
    value = ms * 1000.0 / LAYERS
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "us/layer", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic: seeded N(0,1) K/V and queries",
        "impl": "reference",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "n": N_CTX, "batch": 1,
                   "parallelism": "rank 0 only (host CPU, every core of its affinity mask); one 16k-token layer "
                                  "per unit of the metric (the whole job at N GPUs is N such units per layer)"},
        "cpu_baseline": {"value": round(value, 2), "unit": "us/layer", "cores": threads, "kind": "port",
                         "fp32_us_per_layer": round(us32, 2),
                         "sample": "each step: 36 bf16 layers of 16k decode through the reference's CPU decode "
                                   "expression (threadcut/attention.py:41-42, F.scaled_dot_product_attention of the "
                                   "folded query on CPU tensors; oracle/torch_ref.py), 4 distinct layer buffers "
                                   "cycled",
                         "shift": {"us_per_layer": round(sh_us, 1),
                                   "gbs": round(SHIFT_BYTES_PER_LAYER / (sh_us * 1e-6) / 1e9, 2),
                                   "sample": "config-2 splice of one bf16 layer (threadcut/kv.py:20-25,83-92)"}},
        "e2e": {"value": round(value, 2), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--only", choices=["all", "decode", "shift", "cfg5", "cfg5tp", "gemv", "gemvchain"],
                    default="all",
                    help="profiling runs: time only the decode graph, the splice, the config-5 model step, its "
                         "tensor-parallel form, the step's GEMV, or its chain of projections with the sums in "
                         "residual form at one GPU (--heads = the tensor-parallel width whose shapes it uses; "
                         "smaller JSON line)")
    ap.add_argument("--launches", default=None,
                    help="profiling runs (cfg5tp): rank 0 writes the kernel launch list of 3 graph-replayed steps "
                         "(torch.profiler's CUDA activity records: device time per kernel, no replay) to this file")
    ap.add_argument("--gemv-n", type=int, default=19456, help="profiling runs (gemv): output rows")
    ap.add_argument("--gemv-k", type=int, default=2560, help="profiling runs (gemv): input length")
    ap.add_argument("--layers", type=int, default=LAYERS, help="profiling runs: layers per step")
    ap.add_argument("--ctx", type=int, default=N_CTX, help="profiling runs: context length")
    ap.add_argument("--heads", type=int, default=8, help="profiling runs (decode): KV heads per layer")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, local, world, dist = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.only != "all":
            run_partial(args, rank, local, world, dist)
        else:
            run_ours(args, rank, local, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
