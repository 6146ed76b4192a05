"""Fused B200 kernels and their functional API (drop-in for ``delta_phase.kernels``)."""
from .chunk_delta import (
    DeltaPhaseCudaFunction,
    DeltaPhaseTritonFunction,
    LaplaceCudaFunction,
    chunkwise_forward,
    complex_beta_chunkwise,
    cuda_available,
    decode_step,
    delta_phase_chunkwise_fused,
    gram_matrix_cuda,
    gram_matrix_triton,
    laplace_chunkwise,
    phasor,
    triton_available,
)

__all__ = [
    "delta_phase_chunkwise_fused",
    "triton_available",
    "DeltaPhaseTritonFunction",
    "DeltaPhaseCudaFunction",
    "LaplaceCudaFunction",
    "cuda_available",
    "chunkwise_forward",
    "complex_beta_chunkwise",
    "decode_step",
    "gram_matrix_cuda",
    "gram_matrix_triton",
    "laplace_chunkwise",
    "phasor",
]
