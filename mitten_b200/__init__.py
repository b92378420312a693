"""mitten_b200: a B200-native (sm_100a) paged-KV hot path for the mitten engine.

  mitten_b200.paged   device ops over torch tensors (append, page copy,
                      gather, decode and prefill attention, argmax)
  mitten_b200.host    page pool / radix cache / scheduler (C++ mirror)
  mitten_b200.build   in-tree build of libmitten_kv.so
Everything computes inside libmitten_kv.so (include/mitten_kv.h).
"""
__version__ = "0.1.0"
