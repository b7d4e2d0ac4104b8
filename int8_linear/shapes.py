"""Linear-layer shapes, as (layers, K, N) for C[M, N] = A[M, K] @ W[N, K]^T.

The same table as the reference module int8_linear/shapes.py: the model
dimensions are facts about the models, not a design choice.
"""

SHAPES = {
    # Qwen3-1.7B: hidden 2048, intermediate 6144, 16 query and 8 KV heads of 128.
    "qwen3-1.7b": [
        ("q_proj, o_proj", 2048, 2048),
        ("k_proj, v_proj", 2048, 1024),
        ("gate_proj, up_proj", 2048, 6144),
        ("down_proj", 6144, 2048),
    ],
    # What vLLM runs for Qwen3-1.7B: q, k and v merged, gate and up merged.
    "qwen3-1.7b-vllm": [
        ("qkv_proj", 2048, 4096),
        ("o_proj", 2048, 2048),
        ("gate_up_proj", 2048, 12288),
        ("down_proj", 6144, 2048),
    ],
    # Llama-3-8B at TP1 with QKV and gate/up merged, as vLLM runs it.
    "llama-3-8b": [
        ("qkv_proj", 4096, 6144),
        ("o_proj", 4096, 4096),
        ("gate_up_proj", 4096, 28672),
        ("down_proj", 14336, 4096),
    ],
}
