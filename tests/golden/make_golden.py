"""Generate tests/golden/reference_outputs.npz from the reference itself.

Runs the reference engine's own hot-path sources (compiled from the reference
checkout into oracle/_ref by oracle/Makefile, scalar x86 build) on seeded
workloads from my-inference-engine_b200/workloads.py and stores, per case:

  <name>__meta    (ggml_type, rows, cols, seed)
  <name>__sha256  SHA-256 of the generated packed blocks (pins the generator)
  <name>__y       quantized_tensor_matvec_f32 output for x = make_activations(cols, seed)
  <name>__dq      *_dequantize_block output of the first blocks (up to 4096 values)
  <name>__Y       quantized_tensor_matmul_f32 output for P positions (some cases)

Usage (needs the reference checkout, so run it in the build container):
    python tests/golden/make_golden.py
"""
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


CASES = [
    # name, type, rows, cols, seed, batch
    ("q8_0_small", 8, 67, 160, 5, 3),
    ("q5_0_small", 6, 67, 160, 5, 3),
    ("q4_k_small", 12, 23, 768, 5, 3),
    ("q6_k_small", 14, 23, 768, 5, 3),
    ("cfg0_q8_0", 8, 4864, 896, 0, 0),
    ("cfg3_q5_0", 6, 4864, 896, 0, 2),
]


def main():
    wl = _load("wl", os.path.join(REPO, "my-inference-engine_b200", "workloads.py"))
    binding = _load("ob", os.path.join(REPO, "oracle", "binding.py"))
    binding.build(reference=True)
    ref = binding.Reference(binding.REF_SCALAR_SO)
    ref.set_threads(1)
    out = {}
    for name, gtype, rows, cols, seed, batch in CASES:
        blocks = wl.make_blocks(gtype, rows, cols, seed=seed)
        x = wl.make_activations(cols, seed=seed)
        nb = blocks.size // wl.BLOCK_BYTES[gtype]
        out[name + "__meta"] = np.array([gtype, rows, cols, seed], np.int64)
        out[name + "__sha256"] = np.frombuffer(hashlib.sha256(blocks.tobytes()).hexdigest().encode(), np.uint8)
        out[name + "__y"] = ref.matvec(gtype, blocks, rows, cols, x)
        be = wl.BLOCK_ELEMENTS[gtype]
        ndq = min(nb, 4096 // be)
        out[name + "__dq"] = ref.dequant(gtype, blocks, ndq)
        if batch:
            X = np.stack([wl.make_activations(cols, seed=seed + 100 + p) for p in range(batch)])
            out[name + "__Y"] = ref.matmul(gtype, blocks, rows, cols, X, batch)
        print(name, rows, cols, file=sys.stderr)
    np.savez_compressed(os.path.join(HERE, "reference_outputs.npz"), **out)


if __name__ == "__main__":
    main()
