"""B200-native (sm_100a) MagicMindNet optimizer step.

The hybrid AdamW + Newton-Schulz Muon optimizer of MagicMindNet's mmn-optim
crate, as hand-written CUDA kernels behind a C ABI (include/mmn_optim.h).
``optim`` mirrors the reference's per-call Rust API; ``step`` holds the
batched device-resident step and the trainer configuration; ``checkpoint``
saves and restores the optimizer state beside the reference's weight files.
"""
from ._native import CUDAError, KernelTimeoutError, MmnError, ShapeError  # noqa: F401
from .optim import (AdamW, AdamWConfig, GradAccumulator, HybridOptimizer, Muon,  # noqa: F401
                    MuonConfig, ParamKind, is_available, newton_schulz5, require_cuda)
from .step import (OptimizerStep, StepConfig, TrainConfig, chatbot_param_order,  # noqa: F401
                   classifier_param_order, diffusion_param_order, shard_plan, step_config_for)
from .checkpoint import load_state, save_state  # noqa: F401
from .failure import RankFailure, RankMonitor, RankTimeout  # noqa: F401

__all__ = ["AdamW", "AdamWConfig", "Muon", "MuonConfig", "HybridOptimizer", "ParamKind",
           "GradAccumulator", "newton_schulz5", "is_available", "require_cuda", "OptimizerStep",
           "StepConfig", "TrainConfig", "step_config_for", "chatbot_param_order", "shard_plan",
           "classifier_param_order", "diffusion_param_order",
           "save_state", "load_state", "RankMonitor", "RankFailure", "RankTimeout",
           "MmnError",
           "CUDAError", "ShapeError", "KernelTimeoutError"]
