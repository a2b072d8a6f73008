"""SparseSAM patch of the SAM ViT image encoder on the B200 kernels (see sam.py)."""
