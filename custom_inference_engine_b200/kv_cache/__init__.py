"""Paged KV cache whose page scatter runs in the package's CUDA kernels."""
