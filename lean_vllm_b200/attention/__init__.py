"""The per-token KV-cache store on sm_100a (the reference's lean_vllm/attention/triton_cache.py), fused with the
layer-by-layer push when peers are given."""
