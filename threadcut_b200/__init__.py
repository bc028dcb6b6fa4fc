"""threadcut_b200: B200-native (sm_100a) decode attention over a spliced KV cache.

Drop-in replacement for threadcut's hot path, module for module:
  threadcut.flash_decode -> threadcut_b200.flash_decode   (split-KV GQA decode kernel)
  threadcut.attention    -> threadcut_b200.attention      ("threadcut" transformers plugin)
  threadcut.kv           -> threadcut_b200.kv             (RoPE shift, splice, GrowingLayer)
  threadcut.match        -> threadcut_b200.match          (Split bookkeeping, host)
threadcut's engine (threadcut/engine.py) is the caller of these modules and runs over them unchanged;
it is not part of this package. The device code lives in csrc/ and is reached only through the C ABI of include/threadcut_b200.h
(libthreadcut_b200.so, built by `python -m threadcut_b200.build`).
"""
from .match import Split, lcp, split  # noqa: F401  (host only; importable without a GPU)

__version__ = "0.1.0"
