"""GPU drop-in for the reference's penta_avx2_wrapper module: the same two
functions, on CUDA tensors, backed by pn_unpack and pn_matmul_i8w.

  penta_unpack(packed, K_orig)             -> (N, K_orig) int8 CUDA tensor
  penta_linear_avx2(x, w_int8, scale, bias) -> fp32 x . w^T * scale + bias

(penta_avx2_wrapper.py:42-94 of the reference; there they run the AVX2
kernel on the CPU and take or return numpy arrays.)"""
import torch

from penta_kernel import penta_linear_i8w, unpack_weights_i8


def penta_unpack(packed: torch.Tensor, K_orig: int) -> torch.Tensor:
    return unpack_weights_i8(packed, K_orig)


def penta_linear_avx2(x: torch.Tensor, w_int8: torch.Tensor, scale: float,
                      bias: torch.Tensor | None = None) -> torch.Tensor:
    return penta_linear_i8w(x, w_int8, scale, bias)
