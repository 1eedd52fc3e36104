"""sm_100a kernels behind thin Python wrappers.

Each op runs the in-tree CUDA extension for CUDA tensors (and fails loudly if it is not built)
and an fp32 PyTorch restatement for CPU tensors; the latter is the CPU test tier's oracle.
"""
