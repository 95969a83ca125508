"""Generates tests/golden/golden.npz: small seeded inputs and the CPU oracle's
outputs for every hot-path function.  The reference (Rust) cannot be built in
this environment, so these vectors come from the oracle after it has been
pinned against the reference's own known-answer tests (tests/test_oracle.py);
they freeze that behaviour for regression and for the GPU parity tests.

Run:  python tests/golden/gen_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


def main():
    rng = np.random.default_rng(20240601)
    g = {}
    # f16 / bf16 bit patterns: specials + random
    specials = np.array([0x0000, 0x8000, 0x0001, 0x8001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x7BFF, 0x7C00, 0xFC00,
                         0x7C01, 0xFE00, 0x7FFF, 0x3555, 0x4000, 0x3800], np.uint16)
    h = np.concatenate([specials, rng.integers(0, 65536, 1007, dtype=np.uint16)])
    g["f16_bits"] = h
    g["f16_to_f32"] = O.f16_to_f32(h)
    g["bf16_to_f32"] = O.bf16_to_f32(h)
    x = (rng.standard_normal(1000) * 3e3).astype(np.float32)
    g["f32_in"] = x
    g["f32_to_f16"] = O.f32_to_f16(x)
    # Q8_0 / Q4_0 blocks (n not a multiple of 32 to cover the partial block)
    w = (rng.standard_normal(32 * 40 + 7) * 0.02).astype(np.float32)
    g["w"] = w
    q8 = O.quantize_q8_0(w)
    q4 = O.quantize_q4_0(w)
    g["q8_0_blocks"], g["q4_0_blocks"] = q8, q4
    g["q8_0_deq"] = O.dequantize_to_f32(q8, 8, w.size)
    g["q4_0_deq"] = O.dequantize_to_f32(q4, 2, w.size)
    # engine INT4
    s, p = O.quantize_q4(w, 32)
    g["eng_scales"], g["eng_packed"] = s, p
    g["eng_deq"] = O.dequant_layer(s, p, w.size, 32)
    # GEMV, both formats
    rows, cols = 48, 256
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    xv = rng.standard_normal(cols).astype(np.float32)
    es, ep = O.quantize_q4(W.ravel(), 32)
    g["gemv_x"], g["gemv_eng_scales"], g["gemv_eng_packed"] = xv, es, ep
    g["gemv_eng_y"] = O.gemv_4bit_into(es, ep, xv, rows, cols, 32)
    qb = O.quantize_q4_0(W.ravel())
    g["gemv_q4_0_blocks"] = qb
    g["gemv_q4_0_y"] = O.gemv_q4_0(qb, xv, rows, cols)
    np.savez_compressed(OUT, **g)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
