"""npu_ai_b200: the npu-ai offload hot path (shape-agnostic bf16 GEMM + fused attention) on NVIDIA B200.

The reference (Tobynau/npu-ai) runs SD1.5's Linear layers and attention on an AMD XDNA1 NPU behind a Python
runner (`NpuGemm`, npu/xdna1_gemm.py) and three ComfyUI nodes. This package keeps that API and replaces the
device side with hand-written sm_100a kernels (tcgen05/TMEM/TMA) in libnpub200.so, reached through its C ABI
(include/npu_b200.h). There is no CPU fallback anywhere on the path.
"""
__version__ = "0.1.0"
