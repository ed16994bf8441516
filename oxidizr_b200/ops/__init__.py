"""Op library: sm_100a kernels for CUDA tensors, PyTorch math for CPU tensors."""
