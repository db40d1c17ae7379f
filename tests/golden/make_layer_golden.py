"""Golden vectors for the draft layer's RMSNorm and SiLU-and-mul, made by
vLLM itself (the library whose Eagle3 layer the reference's draft model is).

Runs ``vllm.ir.ops.rms_norm`` and ``SiluAndMul.forward_native`` (plain torch,
CPU) from the vLLM installed in this image on seeded inputs and writes
``layer_ops.npz`` (inputs and outputs as float32 holding bf16 / fp16 values,
plus the vLLM version).  The reference pins vllm>=0.28.1rc1.dev319,<0.28.2
(pyproject.toml:13), which is not installed here; the image's vLLM is used.
Needs vLLM, so it runs in the build container, not on the GPU box; the CPU
test suite reads only the committed ``layer_ops.npz``.

    python tests/golden/make_layer_golden.py
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).with_name("layer_ops.npz")
CASES = {  # name: (dtype, rows, cols, scale)
    "rms_bf16": ("bf16", 8, 1024, 3.0),
    "rms_f16": ("f16", 5, 512, 1.5),
    "silu_bf16": ("bf16", 8, 2048, 4.0),
    "silu_f16": ("f16", 3, 1040, 3.0),
}
_T = {"bf16": torch.bfloat16, "f16": torch.float16}
EPS = 1e-6


def main() -> None:
    import vllm
    from vllm import ir
    from vllm.model_executor.layers.activation import SiluAndMul

    rng = np.random.default_rng(20261202)
    arrays = {"vllm_version": np.array(vllm.__version__), "eps": np.array(EPS)}
    for name, (dt, rows, cols, scale) in CASES.items():
        x = torch.from_numpy(rng.standard_normal((rows, cols), dtype=np.float32) * scale).to(_T[dt])
        if name.startswith("rms"):
            w = torch.from_numpy(rng.uniform(0.5, 1.5, cols).astype(np.float32)).to(_T[dt])
            y = ir.ops.rms_norm(x, w, EPS)
            arrays[f"{name}_w"] = w.float().numpy()
        else:
            y = SiluAndMul.forward_native(x)
        arrays[f"{name}_x"] = x.float().numpy()
        arrays[f"{name}_y"] = y.float().numpy()
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} (vLLM {vllm.__version__})")


if __name__ == "__main__":
    main()
