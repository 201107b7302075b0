"""lean_vllm_b200: B200-native disaggregated prefill->decode KV-cache transfer for lean-vLLM.

The package holds the kvx transport (CUDA kernels for sm_100a behind the C ABI of include/kvx.h, built into
libkvx.so) and the connector that puts it behind lean-vLLM's kv_transfer API.
"""

__version__ = "0.1.0"
