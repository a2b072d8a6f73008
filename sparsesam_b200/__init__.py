"""B200-native (sm_100a) SparseSAM image-encoder hot path.

Stripe-Sort block-sparse attention with fused decomposed rel-pos bias and the
Residual-Consistency MLP, as hand-written tcgen05/TMA CUDA behind the C ABI in
include/sparsesam.h, registered through the reference's AlgoSpec/register()
patch API (sparsesam_b200.registry).
"""
__version__ = "0.1.0"
