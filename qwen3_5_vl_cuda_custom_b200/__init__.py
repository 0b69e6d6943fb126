"""B200-native (sm_100a) Qwen3-VL-MoE text decoder-layer forward.

Drop-in modules with the reference's API (luozoupi/Qwen3_5_VL_CUDA_CUSTOM):
CudaRMSNorm, CudaLinear, CudaEmbedding, TextMRoPE, CudaFullAttention,
CudaSparseMoE, CudaSwiGLUMLP, CudaTextDecoderLayer, CudaQwen3VLMoeModel.
The kernels live in libq35b200.so (C ABI: include/q35b200.h), built by
``python -m qwen3_5_vl_cuda_custom_b200.build``.
"""
from .configs import MoETextConfig, Qwen3VLConfig, TextConfig, VisionConfig  # noqa: F401
from .modules import (  # noqa: F401
    BoundMRoPE, CudaEmbedding, CudaFullAttention, CudaLinear, CudaRMSNorm, CudaSparseMoE,
    CudaSwiGLUMLP, CudaTextDecoderLayer, TextMRoPE,
)
from .models import CudaQwen3VLMoeModel  # noqa: F401
