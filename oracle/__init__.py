"""CPU oracle for threadcut_b200 — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's arithmetic for the hot path (threadcut, pure Python/torch;
nothing to compile, so there is no oracle/_ref build). Only tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py may import it, and only as the checker or the timed CPU baseline —
never as a product path. The package threadcut_b200 does not import it.

Parity is pinned: tests/test_oracle.py checks every function here against golden vectors produced
by the reference itself (tests/golden/make_golden.py imports the reference's threadcut package
in the build container, where the reference checkout is mounted, and records its outputs).

  attention.py  folded-GQA decode attention (threadcut/attention.py:35-42,47 and the math of
                threadcut/flash_decode.py:21-69), LSE merge (flash_decode.py:68-69)
  rope.py       rotate_half / shift_keys (threadcut/kv.py:15-25), bf16 round-to-nearest-even
  splice.py     GrowingLayer.splice and the copy splice (threadcut/kv.py:28-41, 83-92)
  paged.py      the reference's contiguous cache model (appends, splices) and a gather of a paged
                pool in run order, the checker of the paged layout (threadcut README.md:141-144)
"""
