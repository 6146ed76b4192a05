"""delta_phase_b200 -- B200-native (sm_100a) DeltaPhase inference hot path.

Drop-in for the hot-path API of mcarbonell/delta-phase v1.3.0 (``delta_phase``):
the chunkwise complex delta-rule core, its decode step, the LaplacePhaseCore and the
spectral Lerp FFN, on hand-written CUDA kernels behind the C ABI of
``include/deltaphase_b200.h``.
"""
from .kernels import (
    DeltaPhaseCudaFunction,
    DeltaPhaseTritonFunction,
    cuda_available,
    decode_step,
    delta_phase_chunkwise_fused,
    gram_matrix_cuda,
    laplace_chunkwise,
    triton_available,
)
from .layers import (
    ComplexBetaDeltaPhaseBlock,
    DeltaPhaseHolographicBlock,
    LaplacePhaseCore,
    LearnableSubstrateLerpFFN,
    ShortCausalConv1D,
)
from .decode_graph import DecodeGraph
from .model import DeltaPhaseConfig, DeltaPhaseModel
from .spectral import create_dct2_matrix, create_haar_matrix, create_hadamard_matrix

__version__ = "0.1.0"
__all__ = [
    "DeltaPhaseConfig",
    "DeltaPhaseModel",
    "DecodeGraph",
    "DeltaPhaseHolographicBlock",
    "ComplexBetaDeltaPhaseBlock",
    "LearnableSubstrateLerpFFN",
    "ShortCausalConv1D",
    "LaplacePhaseCore",
    "create_hadamard_matrix",
    "create_dct2_matrix",
    "create_haar_matrix",
    "delta_phase_chunkwise_fused",
    "triton_available",
    "cuda_available",
    "DeltaPhaseTritonFunction",
    "DeltaPhaseCudaFunction",
    "gram_matrix_cuda",
    "decode_step",
    "laplace_chunkwise",
]
