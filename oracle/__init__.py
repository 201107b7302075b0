"""CPU oracle for the KV-cache transfer path. Test infrastructure only: never imported by lean_vllm_b200."""
