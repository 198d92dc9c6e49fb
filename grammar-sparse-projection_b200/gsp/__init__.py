"""B200-native grammar-conditioned LM head (drop-in for the reference's ``gsp`` package).

Modules:
  gsp.triton_runtime  -- reference API for bitmask-conditioned logits (CUDA underneath)
  gsp.runtime         -- reference API for id-list projection (constrained_projection)
  gsp.vocab_parallel  -- the head sharded by vocabulary rows over several GPUs
"""
__all__ = ["triton_runtime", "runtime", "vocab_parallel"]
