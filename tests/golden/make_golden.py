"""Generates the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference tree (the fixtures are committed,
so the GPU box never needs the reference):

    python tests/golden/make_golden.py

Sources of truth:
  * oracle/_ref/libref_mlxcpu.so -- the reference's own MLX CPU kernels,
    compiled in place by oracle/Makefile: fp_qmm_t<float|bfloat16_t,16,4>
    (backend/cpu/quantized.cpp:491-533) and FromFP8/ToFP8
    (backend/cpu/unary_ops.h:120-173).
  * kat.json -- known-answer vectors restated from the reference's own tests
    (paths relative to the reference root):
      Tests/MLXFastTests/LagunaNVFP4KernelTests.swift:57-92   nibble order + E4M3 0x38/0x40
      Tests/MLXFastTests/NVFP4QuantizedMMTests.swift:100-154  low-nibble-first, scales 0x30/0x40
      Tests/MLXFastTests/LagunaNVFP4KernelTests.swift:152-330 routed gather over 256 experts
      Tests/MLXFastTests/NVFP4QuantizedMMTests.swift:372-379  deterministic source
The quantizer in MLX is a composition of array ops that cannot be built
without MLX's build system, so packed weights fed to the reference kernels
come from the restatement (oracle/nvfp4_oracle.c); the reference computes
the products.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle as O  # noqa: E402
from _util import det_source  # noqa: E402


def main() -> None:
    O.build()
    if not O.ref_available():
        raise SystemExit("reference shim not built: the reference tree is required")

    # --- FP8 codec: all 256 decodes, encodes on a seeded sweep + edge cases
    dec = np.array([O.ref_from_fp8(b) for b in range(256)], np.float32)
    rng = np.random.default_rng(1234)
    mags = np.exp2(rng.uniform(-14, 10, size=20000)).astype(np.float32)
    signs = np.where(rng.random(20000) < 0.5, -1, 1).astype(np.float32)
    edge = np.array([0.0, -0.0, 448, 464, 463.99, 480, 1e9, np.inf, -np.inf, np.nan, 2 ** -9, 2 ** -10,
                     3 * 2 ** -11, 2 ** -6, 1.5 * 2 ** -9, 0.0625, 240, 256, 272, 288], np.float32)
    enc_in = np.concatenate([mags * signs, edge]).astype(np.float32)
    enc = np.array([O.ref_to_fp8(float(v)) for v in enc_in], np.uint8)
    np.savez_compressed(os.path.join(HERE, "ref_fp8.npz"), decode=dec, encode_in=enc_in, encode_out=enc)

    # --- quantized matmul cases computed by the reference kernels
    cases = {}
    # (a) reference-test deterministic source, K=256
    w = det_source((64, 256), 59)
    c, s = O.fp_quantize(w)
    x = det_source((3, 256), 72)
    cases["det"] = dict(codes=c, scales=s, x=x, y_f32=O.ref_qmm_f32(x, c, s),
                        y_bf16path=O.ref_qmm_bf16(O.f32_to_bf16(x), c, s))
    # (b) N(0, 0.02) weights, N(0, 1) activations, M = 1 and 32
    w = (rng.standard_normal((128, 512), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    c, s = O.fp_quantize(w)
    for M in (1, 32):
        xb = O.f32_to_bf16(rng.standard_normal((M, 512), dtype=np.float32))
        xf = O.bf16_to_f32(xb)
        cases[f"normal_m{M}"] = dict(codes=c, scales=s, x=xf, y_f32=O.ref_qmm_f32(xf, c, s),
                                     y_bf16path=O.ref_qmm_bf16(xb, c, s))
    flat = {f"{k}/{n}": v for k, d in cases.items() for n, v in d.items()}
    np.savez_compressed(os.path.join(HERE, "ref_qmm.npz"), **flat)

    # --- known answers transcribed from the reference's tests
    base = [0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]
    kat = {
        "nibble_order": {
            "source": "Tests/MLXFastTests/LagunaNVFP4KernelTests.swift:57-92",
            "codes": [[0x76543210, 0xFEDCBA98], [0x76543210, 0xFEDCBA98]],
            "scales": [[0x38], [0x40]],
            "expected": [base, [2 * v for v in base]],
        },
        "low_nibble_first": {
            "source": "Tests/MLXFastTests/NVFP4QuantizedMMTests.swift:100-125",
            "nibbles": list(range(16)),
            "scales": [[0x38]],
            "expected": [base],
        },
        "group_scales": {
            "source": "Tests/MLXFastTests/NVFP4QuantizedMMTests.swift:127-154",
            "codes": [[0x22222222] * 4],
            "scales": [[0x30, 0x40]],
            "expected": [[0.5] * 16 + [2.0] * 16],
        },
        "routed_gather": {
            "source": "Tests/MLXFastTests/LagunaNVFP4KernelTests.swift:152-330",
            "n_experts": 256,
            "expert_code": "((e % 7) + 1) * 0x11111111",
            "scale": 0x38,
            "selected": [0, 7, 42, 255, 3, 128, 17, 99],
            "x_value": 0.25,
            "shapes": [[512, 2048], [2048, 512]],
            "tokens": [1, 8],
            "tolerance": 1e-4,
        },
    }
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kat, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
