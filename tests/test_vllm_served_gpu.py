"""f1: the vLLM served path with both patches (int8_linear.vllm_patch, vllm_fuse_patch).

The reference runs patch_vllm() and vllm_fuse_patch.patch_vllm() on a real LLM
(bench/e2e_vllm.py:77-94).  Without its W8A8 checkpoint, tests/vllm_served.py builds a
Qwen3-1.7B-shaped W8A8 model with dummy weights (seeded int8 weights and scales, the same
in every run), once on vLLM's own Triton int8 linear and once with both patches, each in
its own process (the patches rebind module attributes).  Checked: the patched engine
really ran this library (CALLS > 0, PREQUANT_CALLS > 0, FALLBACKS == 0) under vLLM's
torch.compile + CUDA graphs, and its teacher-forced prompt logprobs match vLLM's within
the reference's 1% rule (max |difference| / max |logprob|, bench/bench_linear.py:185-192).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
HELPER = ROOT / "tests" / "vllm_served.py"


def vllm_loads() -> str | None:
    r = subprocess.run([sys.executable, "-c", "import vllm._C"], capture_output=True, text=True, timeout=300)
    return None if r.returncode == 0 else (r.stderr.strip().splitlines() or ["?"])[-1]


def run(backend: str, tmp: Path) -> dict:
    out = tmp / f"{backend}.json"
    env = dict(os.environ, VLLM_ENABLE_V1_MULTIPROCESSING="0", VLLM_DISABLE_COMPILE_CACHE="1")
    r = subprocess.run([sys.executable, str(HELPER), backend, str(out)], env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, f"{backend} failed:\n{r.stderr[-3000:]}"
    return json.loads(out.read_text())


def test_patched_vllm_serves_through_this_library(tmp_path):
    why = vllm_loads()
    if why:
        pytest.skip(f"vLLM's compiled ops do not load here: {why}")
    ref = run("vllm_triton", tmp_path)
    ours = run("ours_fused", tmp_path)
    (ROOT / "gpurun_out").mkdir(exist_ok=True)
    (ROOT / "gpurun_out" / "vllm_served.json").write_text(json.dumps({"ref": ref, "ours": ours}, indent=1))
    assert ref["int8_weights_filled"] == ours["int8_weights_filled"] == 28 * 4
    assert ours["calls"] > 0 and ours["prequant_calls"] > 0 and ours["fallbacks"] == 0, ours
    worst = scale = 0.0
    for a, b in zip(ours["prompt_logprobs"], ref["prompt_logprobs"]):
        assert len(a) == len(b) > 0
        for x, y in zip(a, b):
            worst = max(worst, abs(x - y))
            scale = max(scale, abs(y))
    assert worst <= 1e-2 * max(scale, 1e-6), (worst, scale)
