"""B200-native (sm_100a) k-quant dequant-GEMM and MoE layer.

``aipu_b200.ops`` is the torch-tensor front end of the C ABI in include/aipu_q4k.h;
``aipu_b200.q4k_ref`` / ``aipu_b200.glm_model_q4k_ref`` keep the reference's call signatures.
The CUDA library is built in-tree by ``python -m aipu_b200.build``.
"""
__version__ = "0.1.0"
