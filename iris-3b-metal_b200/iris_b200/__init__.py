"""iris_b200: the Iris-3B denoiser hot path on B200 (sm_100a) kernels.

Public API (mirrors ``iris_metal``): :class:`CudaIris` (the per-step
forward, like ``MetalIris``), :mod:`iris_b200.kernels` (the fused-kernel API
of ``iris_metal.kernels``), the samplers in :mod:`iris_b200.sampling` and
:class:`DenoisePipeline`. The compute runs in ``libiris_b200.so`` (C ABI in
``include/iris_b200.h``).
"""

from iris_b200.config import ModelConfig, PixelStageConfig, baseline_step_config
from iris_b200.model import CudaIris, check_supported, require_finite
from iris_b200.pipeline import DenoisePipeline
from iris_b200.sampling import TURBO_SIGMAS, FlowDPMSolver, euler_cfg
from iris_b200.weights import IrisWeights, synthetic_state

__all__ = [
    "CudaIris",
    "DenoisePipeline",
    "FlowDPMSolver",
    "IrisWeights",
    "ModelConfig",
    "PixelStageConfig",
    "TURBO_SIGMAS",
    "baseline_step_config",
    "check_supported",
    "euler_cfg",
    "require_finite",
    "synthetic_state",
]
