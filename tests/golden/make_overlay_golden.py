"""Generate tests/golden/overlay/ from the reference's own overlay writer.

The reference's ``tools/quantize.py`` (``quantize_file``, tools/quantize.py:
37-88) writes the ``uocr-q8-block32-v1`` overlay that
``QuantizedWeights::load`` (src/cpu/quantized.rs:304-362) reads: a
safetensors file with every eligible projection matrix as I8 plus
``<name>.q8_scales`` F32, and a JSON manifest beside it
(tools/quantize.py:83-99).  This script builds a small synthetic source
checkpoint (F32, BF16 and F16 matrices, eligible and ineligible names, tails
that are not a multiple of 32) and runs the reference's writer on it, so the
overlay loader and the package's writer are pinned to the reference's bytes
on machines where the reference is absent.

Usage:  python tests/golden/make_overlay_golden.py --reference <reference checkout>

Writes source.safetensors, overlay.safetensors and overlay.json under
tests/golden/overlay/.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "overlay")


def source_tensors(rng: np.random.Generator):
    """name -> torch tensor; eligible names per the reference's MATRIX
    pattern (tools/quantize.py:16) and eligible() (src/cpu/quantized.rs:262)."""
    import torch

    def mat(rows, cols, scale=1.0):
        v = rng.standard_normal((rows, cols)) * rng.uniform(0.05, 3.0, (rows, 1)) * scale
        return torch.from_numpy(v.astype(np.float32))

    z = mat(4, 40)
    z[1] = 0.0  # an all-zero row: zero scales
    return {
        "lm_head.weight": mat(6, 70),                                        # F32, tail 6
        "model.embed_tokens.weight": mat(6, 70),                             # not eligible
        "model.norm.weight": torch.ones(70),                                 # not eligible
        "model.layers.0.self_attn.q_proj.weight": mat(8, 33).to(torch.bfloat16),
        "model.layers.0.self_attn.o_proj.weight": mat(33, 8).to(torch.float16),
        "model.layers.0.mlp.gate_proj.weight": mat(12, 64),                  # dense FFN
        "model.layers.1.mlp.gate.weight": mat(4, 64).to(torch.bfloat16),     # router: not eligible
        "model.layers.1.mlp.shared_experts.up_proj.weight": mat(16, 64, 1e-3),
        "model.layers.1.mlp.experts.3.down_proj.weight": z.to(torch.bfloat16),
        "model.layers.1.mlp.experts.12.gate_proj.weight": mat(5, 1).to(torch.float16),
        "model.layers.1.self_attn.k_proj.bias": torch.ones(8),               # not eligible
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="reference checkout (contains tools/)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from safetensors.torch import save_file
    from tools.quantize import quantize_file  # the reference's own writer

    os.makedirs(OUT, exist_ok=True)
    rng = np.random.default_rng(20261202)
    with tempfile.TemporaryDirectory() as d:
        src = Path(d) / "source.safetensors"
        save_file(source_tensors(rng), str(src))
        out = Path(d) / "overlay.safetensors"
        manifest = quantize_file(src, out, chunk_rows=3)
        # tools/quantize.py:93-95: the manifest beside the overlay
        out.with_suffix(".json").write_text(json.dumps(manifest, indent=2) + "\n")
        for name in ("source.safetensors", "overlay.safetensors", "overlay.json"):
            shutil.copyfile(Path(d) / name, os.path.join(OUT, name))
    print(f"wrote {OUT}: {manifest['matrix_count']} matrices, {manifest['bytes']} bytes")


if __name__ == "__main__":
    main()
