"""The KV connector API and the CUDA-IPC connector (drop-in for lean_vllm.kv_transfer)."""
