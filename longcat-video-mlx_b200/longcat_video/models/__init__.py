"""BSA-path modules of the LongCat-Video DiT (attention hook, routing, kernels, RoPE)."""
