"""Kernels (sm_100a via ctypes) and their PyTorch restatements."""
