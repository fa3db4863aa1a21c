"""voom_b200: B200-native (sm_100a) decode of vOOM's lossless BF16 weight-page
formats (bf16_rans, vpack/vpack2), fused with the MoE expert SwiGLU GEMV that
consumes the pages, plus the kv_paged spill/reload page codec.

Compute runs in libvoom_b200.so (hand-written CUDA for sm_100a) behind the C
ABI in include/voom_b200.h; the Python modules mirror the reference's
interfaces (formats.bf16_rans, formats.packed, formats.packed2,
runtime.weight_store, runtime.expert_batching, runtime.kv_paged).  The
reference's own WeightCache and consume_expert_batches stay in place and
drive these through their unchanged page API.
"""

__version__ = "0.1.0"
