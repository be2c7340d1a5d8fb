"""B200-native quantized-linear hot path of comfy-quant-bench (ConvRot rotation + dynamic quantization,
packed-int4 x int8 tcgen05 GEMM, fused dequant epilogue, weight rotate-and-quantize).

The CUDA kernels live in ``libcq_b200.so`` (C ABI: ``include/cq_b200.h``); ``ops`` mirrors comfy-kitchen's
operator API on top of it, ``formats`` the packed-tensor layout, ``layout`` / ``comfy_ops`` the ComfyUI
plugin boundary, ``custom_op`` the torch.compile-safe opaque ops and ``dist`` the multi-GPU sharding.
"""
__version__ = "0.1.0"
