"""swiftmoe_b200: B200-native (sm_100a) MoE-layer forward with SwiftMoE's module API.

    from swiftmoe_b200 import UltimateMoE, StandardMoE, BaselineMoE

The compute runs in libswiftmoe.so (hand-written CUDA, C ABI in include/swiftmoe.h);
PyTorch provides device memory, streams and torch.distributed.
"""
from .baseline_moe import BaselineMoE, StandardMoE, SwiGLUExpert
from .ultimate_moe import MoEAsyncCommHandler, UltimateMoE, setup_nccl_optimizations
from .dist_init import init_expert_parallel

__all__ = ["UltimateMoE", "StandardMoE", "BaselineMoE", "SwiGLUExpert", "MoEAsyncCommHandler",
           "setup_nccl_optimizations", "init_expert_parallel"]
__version__ = "0.1.0"
