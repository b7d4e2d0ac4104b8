"""One vLLM engine run of a Qwen3-1.7B-shaped W8A8 model with dummy weights (the f1 check).

    VLLM_ENABLE_V1_MULTIPROCESSING=0 python tests/vllm_served.py BACKEND OUT.json

BACKEND is `vllm_triton` (vLLM's own Triton int8 linear, unpatched) or `ours_fused`
(int8_linear.vllm_patch and int8_linear.vllm_fuse_patch applied first: this library's
GEMM behind the custom op, Qwen3's norms and SiLU feeding the linears pre-quantised), as
the reference's bench/e2e_vllm.py:77-94 builds them.  There is no checkpoint here, so the
model directory holds only a config.json: the public Qwen3-1.7B hyperparameters and the
compressed-tensors W8A8 scheme the reference's checkpoint uses (int8 per-channel
symmetric weights, dynamic per-token symmetric int8 activations, lm_head unquantised).
vLLM builds it with load_format="dummy", which leaves int8 parameters unset, so every
int8 weight and weight scale is then filled from a generator seeded by its name (the same
values in both backends).  The engine runs compiled with CUDA graphs, in-process (the
patches must reach the model).  Writes the prompt logprobs of a few token prompts, the
greedy tokens and the counters of both patches.
"""

from __future__ import annotations

import json
import os
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

QWEN3_1_7B = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 2048,
    "intermediate_size": 6144, "num_hidden_layers": 28, "num_attention_heads": 16,
    "num_key_value_heads": 8, "head_dim": 128, "hidden_act": "silu", "rms_norm_eps": 1e-6,
    "vocab_size": 151936, "max_position_embeddings": 40960, "rope_theta": 1000000,
    "rope_scaling": None, "tie_word_embeddings": True, "attention_bias": False,
    "attention_dropout": 0.0, "torch_dtype": "bfloat16", "use_sliding_window": False,
    "sliding_window": None, "max_window_layers": 28, "bos_token_id": 151643, "eos_token_id": 151645,
}
W8A8 = {
    "quant_method": "compressed-tensors", "format": "int-quantized", "quantization_status": "compressed",
    "ignore": ["lm_head"], "kv_cache_scheme": None, "global_compression_ratio": None,
    "config_groups": {"group_0": {
        "targets": ["Linear"], "output_activations": None,
        "weights": {"num_bits": 8, "type": "int", "symmetric": True, "strategy": "channel",
                    "dynamic": False, "group_size": None, "block_structure": None, "actorder": None,
                    "observer": "minmax", "observer_kwargs": {}},
        "input_activations": {"num_bits": 8, "type": "int", "symmetric": True, "strategy": "token",
                              "dynamic": True, "group_size": None, "block_structure": None,
                              "actorder": None, "observer": None, "observer_kwargs": {}},
    }},
}
PROMPTS = [[151643, 785, 6722, 315, 9625, 374, 12095, 13, 576, 1156, 3409, 304, 279, 1879, 572, 220],
           [8645, 1128, 264, 5175, 1965, 374, 13, 362, 5175, 1965, 374, 264, 821, 5944, 429, 14043],
           [750, 75698, 1445, 1648, 262, 421, 308, 2651, 220, 16, 25, 470, 308, 198, 262, 470]]


def fill_int8_weights(model) -> int:
    """Seeded int8 weights and positive per-channel scales for every quantised linear (the
    dummy loader leaves integer parameters unset).  Returns how many weights it set."""
    import zlib

    import torch

    count = 0
    for name, p in model.named_parameters():
        seed = zlib.crc32(name.encode())
        g = torch.Generator(device=p.device).manual_seed(seed)
        with torch.no_grad():
            if p.dtype == torch.int8:
                p.copy_(torch.randint(-127, 128, p.shape, generator=g, device=p.device, dtype=torch.int8))
                count += 1
            elif name.endswith("weight_scale"):
                p.copy_(torch.rand(p.shape, generator=g, device=p.device, dtype=torch.float32)
                        .to(p.dtype) * 1e-3 + 1e-4)
    return count


def main(backend: str, out_path: str) -> None:
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    os.environ.setdefault("VLLM_DISABLE_COMPILE_CACHE", "1")
    model_dir = Path(tempfile.mkdtemp(prefix="qwen3_w8a8_dummy_"))
    (model_dir / "config.json").write_text(json.dumps(dict(QWEN3_1_7B, quantization_config=W8A8)))

    if backend == "ours_fused":
        from int8_linear import vllm_fuse_patch, vllm_patch

        vllm_patch.patch_vllm()
        vllm_fuse_patch.patch_vllm()
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    llm = LLM(model=str(model_dir), load_format="dummy", linear_backend="triton", dtype="bfloat16",
              max_model_len=256, gpu_memory_utilization=0.3, seed=0, enable_prefix_caching=False,
              skip_tokenizer_init=True)
    filled = llm.apply_model(fill_int8_weights)[0]
    kernels = llm.apply_model(lambda m: sorted({type(getattr(getattr(x, "scheme", None), "kernel", None)).__name__
                                                for x in m.modules() if getattr(x, "scheme", None)}))[0]
    params = SamplingParams(temperature=0.0, max_tokens=8, logprobs=1, prompt_logprobs=1, detokenize=False)
    outs = llm.generate([TokensPrompt(prompt_token_ids=p) for p in PROMPTS], params)
    result = {"backend": backend, "int8_weights_filled": filled, "linear_kernels": kernels,
              "prompt_logprobs": [], "tokens": []}
    for o, prompt in zip(outs, PROMPTS):
        lp = []
        for pos, d in enumerate(o.prompt_logprobs or []):
            if d is None:
                continue
            lp.append(float(d[prompt[pos]].logprob))
        result["prompt_logprobs"].append(lp)
        result["tokens"].append(list(o.outputs[0].token_ids))
    if backend == "ours_fused":
        from int8_linear import vllm_fuse_patch, vllm_patch

        result.update(calls=vllm_patch.CALLS, fallbacks=vllm_patch.FALLBACKS,
                      prequant_calls=vllm_fuse_patch.PREQUANT_CALLS,
                      configs=len(vllm_patch.CONFIGS))
    Path(out_path).write_text(json.dumps(result))


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
