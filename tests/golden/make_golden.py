"""Writes tests/golden/golden.npz and golden.json from the REFERENCE's own functions.

    python tests/golden/make_golden.py --reference /path/to/int8-linear

Runs on a CPU in the build container, where the reference package is importable
(its Triton kernels are never run; only its torch reference functions are):
  tests/test_kernel.py:36-38      exact            (int32 product)
  tests/test_fused_quant.py:26-51 quant, ref_norm, ref_silu
  bench/bench_linear.py:146-150   quant_rows       (operand quantisation)
and the float64 layer of bench/bench_linear.py:164-165 / tests/test_kernel.py:68-69
computed from them.  Inputs come from tests/golden/recipes.py (seeded CPU
generators); the manifest records a SHA-256 of every input and output.  The tests
rebuild the inputs, check their hashes, and compare the oracle against these
outputs, so the committed fixtures pin the oracle without the reference present.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import recipes  # noqa: E402


def load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference repository (AshrithaG/int8-linear)")
    a = ap.parse_args()
    ref_root = Path(a.reference)
    sys.path.insert(0, str(ref_root))   # the reference package shadows nothing here
    tk = load_module(ref_root / "tests" / "test_kernel.py", "ref_test_kernel")
    tq = load_module(ref_root / "tests" / "test_fused_quant.py", "ref_test_fused_quant")
    bl = load_module(ref_root / "bench" / "bench_linear.py", "ref_bench_linear")
    torch.set_num_threads(4)

    arrays: dict[str, np.ndarray] = {}
    man: dict = {"reference": "AshrithaG/int8-linear", "torch": torch.__version__, "cases": {}}

    # --- BASELINE config 0 through the reference's quant_rows and exact
    x, w = recipes.config0()
    a_q, a_s = bl.quant_rows(x)
    w_q, w_s = bl.quant_rows(w)
    acc = tk.exact(a_q, w_q)
    term = acc.double() * a_s.double() * w_s.double().t()
    arrays.update({"c0_a_q": a_q.numpy(), "c0_a_s": a_s.numpy(), "c0_w_s": w_s.numpy(),
                   "c0_ref_bf16": bits(term.to(torch.bfloat16))})
    man["cases"]["config0"] = {"x": recipes.sha(x), "w": recipes.sha(w), "w_q": recipes.sha(w_q),
                               "acc": recipes.sha(acc), "ref": recipes.sha(term)}

    # --- exact int32 products at the reference test shapes
    for m, k, n in recipes.GEMM_SHAPES:
        ai, wi = recipes.ints((m, k), 1), recipes.ints((n, k), 2)
        out = tk.exact(ai, wi)
        man["cases"][f"exact_{m}x{k}x{n}"] = {"a": recipes.sha(ai), "w": recipes.sha(wi),
                                              "out": recipes.sha(out)}
        if m * n <= 8192:
            arrays[f"exact_{m}x{k}x{n}"] = out.numpy()

    # --- float64 scaled layer, the 16 cases of test_scaled_output_matches_float64
    for dtype in (torch.bfloat16, torch.float16):
        for per_row in (True, False):
            for per_col in (True, False):
                for use_bias in (True, False):
                    ai, wi, sa, sb, bias = recipes.scaled_case(dtype, per_row, per_col, use_bias)
                    t = tk.exact(ai, wi).double() * sa.double().reshape(-1, 1) * sb.double().reshape(1, -1)
                    r = t + bias.double() if use_bias else t
                    key = f"scaled_{str(dtype)[6:]}_{int(per_row)}{int(per_col)}{int(use_bias)}"
                    man["cases"][key] = {"term": recipes.sha(t), "ref": recipes.sha(r)}

    # --- fused quantisers through the reference's ref_norm / ref_silu
    for m, k in recipes.NORM_SHAPES:
        for has_res in (False, True):
            xx, rr, ww = recipes.norm_case(m, k, has_res)
            q, s, rout = tq.ref_norm(xx, rr, ww)
            key = f"norm_{m}x{k}_{int(has_res)}"
            arrays[key + "_q"], arrays[key + "_s"] = q.numpy(), s.numpy()
            man["cases"][key] = {"x": recipes.sha(xx), "w": recipes.sha(ww), "q": recipes.sha(q)}
            if rout is not None:
                man["cases"][key].update(r=recipes.sha(rr), rout=recipes.sha(rout))
    for m, i in recipes.SILU_SHAPES:
        for rnd in (False, True):
            gu = recipes.silu_case(m, i)
            q, s = tq.ref_silu(gu, rnd)
            key = f"silu_{m}x{i}_{int(rnd)}"
            arrays[key + "_q"], arrays[key + "_s"] = q.numpy(), s.numpy()
            man["cases"][key] = {"gu": recipes.sha(gu), "q": recipes.sha(q)}
    # outlier activations (bench/fuse_quant.py:52-57) through the plain quantiser
    xo = recipes.outlier_activations(64, 2048, 5)
    q, s = tq.quant(xo)
    arrays["outlier_q"], arrays["outlier_s"] = q.numpy(), s.numpy()
    man["cases"]["outlier_64x2048"] = {"x": recipes.sha(xo), "q": recipes.sha(q)}

    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(man, indent=1, sort_keys=True) + "\n")
    size = (HERE / "golden.npz").stat().st_size
    print(f"wrote {len(arrays)} arrays ({size / 1e6:.2f} MB) and {len(man['cases'])} cases")


if __name__ == "__main__":
    main()
