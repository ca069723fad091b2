"""fast_rfdetr.kernels: the reference's four kernel entry points (fast_rfdetr/kernels.py:53, :106, :165, :271) with
their signatures, on torch CUDA tensors, from kernelopt_b200.kernels."""
from kernelopt_b200.kernels import deform_attn, linear_gelu_f32, preprocess_gpu, residual_layernorm

__all__ = ["residual_layernorm", "preprocess_gpu", "deform_attn", "linear_gelu_f32"]
