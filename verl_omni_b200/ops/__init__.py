"""Hot ops: each has a hand-written sm_100a CUDA kernel (CUDA tensors) and an fp32 torch oracle (CPU)."""
