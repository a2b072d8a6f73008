"""CPU restatement of the reference SparseSAM hot path — TEST INFRASTRUCTURE ONLY.

This package is the parity checker for the sm_100a kernels. Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may
import it; the product path (sparsesam_b200) never does and has no CPU
fallback.

  order.py     Morton order, Stripe-Sort permutation (fp64 scoring, lowest-index
               ties), A-shape mask parameters, keep-set selection   [numpy]
  attention.py dense restatement of the block-sparse rel-pos attention kernel
               (flash_attn.py:1519-1551 semantics)                  [torch fp32]
  encoder.py   SparseSAM-patched SAM ViT encoder forward
               (sam.py:168-290 + the SAM host model)                 [torch fp32]
  decoder.py   SAM-HQ box-prompted decode and mask resizing, the
               checker of the predictor around the encoder
               (eval_hq44k.py:87-129; SAM-HQ itself is unvendored)  [torch fp64]

Pinned against golden vectors produced by running the reference's own
algos/sparsesam code on CPU (tests/golden/make_golden.py).
"""
