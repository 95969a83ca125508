"""Pins the CPU oracle (oracle/ah_oracle*.c) before anything is checked
against it: the reference's own known-answer tests, numpy's IEEE half
conversion over every bit pattern, independent numpy restatements of each
formula, the committed golden vectors, and the documented divergence of the
reference's AVX-512 kernels from its scalar semantics."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


# --- known answers from the reference's own tests --------------------------------

def test_f16_known_answers(oracle):
    # formats/gguf.rs:681-693
    v = oracle.f16_to_f32(np.array([0x3C00, 0x0000, 0xBC00, 0x4000, 0x3800], np.uint16))
    assert v.tolist() == [1.0, 0.0, -1.0, 2.0, 0.5]


def test_bf16_known_answers(oracle):
    # formats/gguf.rs:696-701
    v = oracle.bf16_to_f32(np.array([0x3F80, 0x0000], np.uint16))
    assert v.tolist() == [1.0, 0.0]


def test_q8_0_known_answer(oracle):
    # formats/gguf.rs:704-721: one block, d = f16 1.0, q = 0..31
    raw = np.concatenate([np.array([0x00, 0x3C], np.uint8), np.arange(32, dtype=np.uint8)])
    assert oracle.dequantize_to_f32(raw, 8, 32).tolist() == list(range(32))


def test_quantize_dequantize_roundtrip(oracle):
    # models/quantization.rs:536-556
    w = np.array([0.1, -0.2, 0.3, -0.4, 0.5, -0.6, 0.7, -0.8, 0.15, 0.25, -0.35, 0.45, -0.55, 0.65, -0.75, 0.85,
                  -0.95, 0.05, -0.15, 0.25, -0.35, 0.45, -0.55, 0.65, -0.75, 0.85, -0.95, 0.05, -0.15, 0.25,
                  -0.35, 0.45] + [0.0] * 32, np.float32)
    s, p = oracle.quantize_q4(w, 32)
    d = oracle.dequant_layer(s, p, w.size, 32)
    assert np.max(np.abs(w - d)) < 0.15


def test_zero_weights(oracle):
    # models/quantization.rs:558-566
    s, p = oracle.quantize_q4(np.zeros(64, np.float32), 32)
    assert np.all(np.abs(oracle.dequant_layer(s, p, 64, 32)) < 1e-6)


def test_packing(oracle):
    # models/quantization.rs:568-583
    w = np.zeros(32, np.float32)
    w[0], w[1] = 0.7, -0.7
    _, p = oracle.quantize_q4(w, 32)
    b = int(p[0])
    assert (b & 0x0F) - 8 > 0 and ((b >> 4) & 0x0F) - 8 < 0


def test_gemv_4bit_execution(oracle):
    # inference/math.rs:453-468 (constant weights 0.5, x = 1)
    s, p = oracle.quantize_q4(np.full(4 * 128, 0.5, np.float32), 32)
    out = oracle.gemv_4bit_into(s, p, np.ones(128, np.float32), 4, 128, 32)
    assert out[0] > 0


# --- IEEE conversions against numpy ------------------------------------------------

def test_f16_all_bit_patterns_vs_numpy(oracle):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ours = oracle.f16_to_f32(h)
    ref = h.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(bits(ours[~nan]), bits(ref[~nan]))
    # gguf.rs:111: every NaN becomes f32::NAN, then the sign is applied (-val)
    expect = np.where((h[nan] & 0x8000) != 0, 0xFFC00000, 0x7FC00000).astype(np.uint32)
    assert np.array_equal(bits(ours[nan]), expect)


def test_f32_to_f16_vs_numpy(oracle):
    rng = np.random.default_rng(7)
    x = np.concatenate([
        (rng.standard_normal(200000) * 3e4).astype(np.float32),
        (rng.standard_normal(200000) * 1e-5).astype(np.float32),
        rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32).view(np.float32),
        np.array([65504, 65519.996, 65520, 2.9802322e-08, 2.9802326e-08, 5.96e-8, -0.0, np.inf, -np.inf],
                 np.float32)])
    x = x[~np.isnan(x)]
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16(x), ref)


# --- numpy restatements of each formula -----------------------------------------------

def round_half_away(v):
    a = np.abs(v)
    f = np.floor(a)
    r = f + ((a - f) >= np.float32(0.5)).astype(np.float32)
    return np.copysign(r, v).astype(np.float32)


def np_quantize_q4(w, gs=32):
    """quantization.rs:369-404 in numpy float32 arithmetic."""
    n = w.size
    ng = (n + gs - 1) // gs
    pad = np.zeros(ng * gs, np.float32)
    pad[:n] = w
    g = pad.reshape(ng, gs)
    mx = np.max(np.abs(g), axis=1).astype(np.float32)
    scale = np.where(mx > 0, mx / np.float32(7.0), np.float32(0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, np.float32(1.0) / scale, np.float32(0)).astype(np.float32)
    q = round_half_away((g * inv[:, None]).astype(np.float32))
    q = np.where(scale[:, None] > 0, q, 0)
    q = (np.clip(q, -8, 7) + 8).astype(np.uint8).ravel()[:n]
    if n % 2:
        q = np.concatenate([q, np.zeros(1, np.uint8)])
    return scale, (q[0::2] | (q[1::2] << 4)).astype(np.uint8)


def test_quantize_q4_vs_numpy(oracle):
    rng = np.random.default_rng(3)
    for n in (32, 1000, 4096 * 3 + 17):
        w = (rng.standard_normal(n) * 0.02).astype(np.float32)
        w[::97] = 0.0
        s, p = oracle.quantize_q4(w, 32)
        s2, p2 = np_quantize_q4(w, 32)
        assert np.array_equal(bits(s), bits(s2))
        assert np.array_equal(p, p2)


def test_block_quantizers_vs_numpy(oracle):
    rng = np.random.default_rng(4)
    w = (rng.standard_normal(32 * 300) * 0.02).astype(np.float32)
    g = w.reshape(-1, 32)
    amax = np.max(np.abs(g), axis=1).astype(np.float32)
    for q4, div, bsz in ((False, 127.0, 34), (True, 8.0, 18)):
        d16 = (amax / np.float32(div)).astype(np.float16)
        d = d16.astype(np.float32)
        with np.errstate(divide="ignore"):
            idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0)).astype(np.float32)
        q = round_half_away((g * idv[:, None]).astype(np.float32))
        blocks = (oracle.quantize_q4_0(w) if q4 else oracle.quantize_q8_0(w)).reshape(-1, bsz)
        assert np.array_equal(blocks[:, :2].copy().view(np.uint16).ravel(), d16.view(np.uint16))
        if q4:
            qq = (np.clip(q + 8, 0, 15)).astype(np.uint8)
            assert np.array_equal(blocks[:, 2:], qq[:, 0::2] | (qq[:, 1::2] << 4))
        else:
            assert np.array_equal(blocks[:, 2:].view(np.int8), np.clip(q, -127, 127).astype(np.int8))


def test_dequant_vs_numpy(oracle):
    rng = np.random.default_rng(5)
    w = (rng.standard_normal(32 * 500) * 0.02).astype(np.float32)
    q8 = oracle.quantize_q8_0(w).reshape(-1, 34)
    d = q8[:, :2].copy().view(np.float16).astype(np.float32)
    ref = (d * q8[:, 2:].view(np.int8).astype(np.float32)).ravel()
    assert np.array_equal(bits(oracle.dequantize_to_f32(q8.ravel(), 8, w.size)), bits(ref))
    q4 = oracle.quantize_q4_0(w).reshape(-1, 18)
    d = q4[:, :2].copy().view(np.float16).astype(np.float32)
    nib = np.stack([q4[:, 2:] & 15, q4[:, 2:] >> 4], axis=2).reshape(-1, 32).astype(np.float32) - 8
    assert np.array_equal(bits(oracle.dequantize_to_f32(q4.ravel(), 2, w.size)), bits((d * nib).ravel()))
    s, p = oracle.quantize_q4(w, 32)
    nib = np.stack([p & 15, p >> 4], axis=1).ravel().astype(np.float32) - 8
    assert np.array_equal(bits(oracle.dequant_layer(s, p, w.size, 32)), bits(nib * np.repeat(s, 32)))


def test_gemv_vs_sequential_numpy(oracle):
    # math.rs:395-416: per row, sequential f32 sum of ((nib-8)*scale) * x[j]
    rng = np.random.default_rng(6)
    rows, cols = 24, 160  # cols % 32 == 0 and != 0 mod 128 (the scalar branch)
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    s, p = oracle.quantize_q4(W.ravel(), 32)
    nib = np.stack([p & 15, p >> 4], axis=1).ravel().astype(np.float32).reshape(rows, cols) - 8
    wd = (nib * np.repeat(s, 32).reshape(rows, cols)).astype(np.float32)
    acc = np.zeros(rows, np.float32)
    for j in range(cols):
        acc = (acc + (wd[:, j] * x[j]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(bits(oracle.gemv_4bit_into(s, p, x, rows, cols, 32)), bits(acc))
    # empty input zeroes the output (math.rs:264-267)
    assert np.all(oracle.gemv_4bit_into(s, p, np.zeros(0, np.float32), rows, 0, 32) == 0)


def test_gemv_ragged_group(oracle):
    # cols % group_size != 0: the last group of each row is short (math.rs:401-404)
    rng = np.random.default_rng(8)
    rows, cols, gs = 5, 50, 32
    n_gpr = 2
    s = (rng.random(rows * n_gpr) * 0.01).astype(np.float32)
    p = rng.integers(0, 256, (rows * cols + 1) // 2, dtype=np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    out = oracle.gemv_4bit_into(s, p, x, rows, cols, gs)
    for r in range(rows):
        acc = np.float32(0)
        for j in range(cols):
            lin = r * cols + j
            nb = (p[lin >> 1] >> (4 * (lin & 1))) & 15
            acc = np.float32(acc + np.float32(np.float32(np.float32(nb) - 8) * s[r * n_gpr + j // gs]) * x[j])
        assert bits(out[r]) == bits(acc)


def test_dequantize_to_f32_edge_semantics(oracle):
    raw = np.arange(34 * 2 + 10, dtype=np.uint8)
    assert oracle.dequantize_to_f32(raw[:12], 0, 100).size == 3          # F32 ignores element_count
    assert oracle.dequantize_to_f32(raw[:11], 1, 1).size == 5            # F16: raw_len / 2
    assert oracle.dequantize_to_f32(raw, 8, 1000).size == 64 + 8         # Q8_0 limited by raw bytes
    assert oracle.dequantize_to_f32(raw[:34 + 1], 8, 64).size == 32      # < 2 bytes of the next block
    assert oracle.dequantize_to_f32(raw[:18 + 5], 2, 64) is None         # Q4_0 truncated block: reference panics
    assert oracle.dequantize_to_f32(raw[:18 + 1], 2, 64).size == 32      # header absent: loop breaks
    z = oracle.dequantize_to_f32(raw, 99, 7)
    assert z.size == 7 and np.all(z == 0)                                # unknown dtype -> zeros


def test_rope_and_rmsnorm_vs_numpy(oracle):
    rng = np.random.default_rng(9)
    x = rng.standard_normal(128).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    ss = np.float32(0)
    for v in x:
        ss = np.float32(ss + np.float32(v * v))
    inv = np.float32(1) / np.sqrt(np.float32(ss / np.float32(128) + np.float32(1e-5)))
    assert np.allclose(oracle.rms_norm(x, w, 1e-5), (x * inv) * w, rtol=1e-6, atol=0)
    pos, base = 37, 5e5
    r = oracle.rope_head(x, pos, base)
    i = np.arange(64)
    th = pos * np.power(np.float64(base), -i / 64.0)
    x0, x1 = x[0::2].astype(np.float64), x[1::2].astype(np.float64)
    ref = np.empty(128)
    ref[0::2] = x0 * np.cos(th) - x1 * np.sin(th)
    ref[1::2] = x0 * np.sin(th) + x1 * np.cos(th)
    assert np.max(np.abs(r - ref)) < 1e-3


def test_argmax_first_max_wins(oracle):
    # inference/sampling.rs:4-14
    assert oracle.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert oracle.argmax(np.array([np.nan, -1, np.nan], np.float32)) == 1


# --- sampling.rs:17-64 with the uniform draw given ----------------------------------

def _sample_f64(logits, temperature, top_k, r):
    """An independent restatement in float64 with a stable sort: the pick and
    the distance of r from the nearest CDF boundary."""
    x = np.asarray(logits, np.float64)
    p = np.exp((x - x.max()) / temperature)
    order = sorted(range(x.size), key=lambda i: (-p[i], i))[:min(top_k, x.size)]
    cdf = np.cumsum(p[order]) / p[order].sum()
    j = int(np.searchsorted(cdf, r, side="right"))
    return order[min(j, len(order) - 1)], float(np.min(np.abs(cdf - r)))


def test_sample_matches_restatement(oracle):
    rng = np.random.default_rng(31)
    for n, temp, k in ((1000, 1.0, 40), (300, 0.5, 5), (64, 2.0, 64), (7, 1.0, 40), (500, 0.8, 1)):
        logits = (rng.standard_normal(n) * 3).astype(np.float32)
        for r in rng.random(60).astype(np.float32):
            got = oracle.sample(logits, temp, k, float(r))
            want, margin = _sample_f64(logits, temp, k, float(r))
            assert got == want or margin < 1e-5, (n, temp, k, r, got, want)


def test_sample_edge_cases(oracle):
    lg = np.array([1, 3, 3, 2], np.float32)
    assert oracle.sample(lg, 1.0, 1, 0.99) == 1  # top-1 is the first maximum
    assert oracle.sample(lg, 1.0, 40, 0.0) == 1  # r = 0: the first candidate
    assert oracle.sample(lg, 1.0, 2, 0.75) == 2  # the tie's second member
    # tiny temperature: only the two maxima keep weight, half each
    assert [oracle.sample(lg, 1e-30, 40, r) for r in (0.3, 0.49, 0.51, 0.999)] == [1, 1, 2, 2]
    # masked logits carry no weight
    masked = np.array([-np.inf, 0.0, -np.inf, 0.0], np.float32)
    assert {oracle.sample(masked, 1.0, 40, r) for r in (0.1, 0.6)} == {1, 3}


def test_sample_frequencies(oracle):
    # over many draws the picks follow the renormalised top-k softmax
    rng = np.random.default_rng(4)
    logits = (rng.standard_normal(200) * 1.5).astype(np.float32)
    k, temp, n = 8, 0.9, 20000
    picks = np.array([oracle.sample(logits, temp, k, oracle.sample_uniform(11, s, 0)) for s in range(n)])
    top = np.argsort(-logits, kind="stable")[:k]
    p = np.exp((logits[top] - logits.max()) / temp)
    p /= p.sum()
    assert set(np.unique(picks)) <= set(top.tolist())
    for i, pi in zip(top, p):
        f = np.mean(picks == i)
        assert abs(f - pi) <= 5 * np.sqrt(pi * (1 - pi) / n) + 1e-3, (i, f, pi)


def test_sample_uniform_matches_library(oracle):
    # the draw the device sampler uses (a host function of the C-ABI library,
    # no GPU needed) equals the oracle's restatement bit for bit
    from agent_harness_b200 import kernels as K
    O = oracle
    for seed, step, seq in ((0, 0, 0), (1, 5, 3), (2**63 + 17, 123456, 15), (42, 2**40, 7)):
        a, b = K.sample_uniform(seed, step, seq), O.sample_uniform(seed, step, seq)
        assert a == b, (seed, step, seq, a, b)
        assert 0.0 <= a < 1.0
    vals = np.array([O.sample_uniform(9, s, q) for s in range(200) for q in range(16)])
    assert abs(vals.mean() - 0.5) < 0.02 and vals.min() >= 0.0 and vals.max() < 1.0


# --- the reference's AVX-512 kernels, restated as-is for timing, diverge as documented --

def test_avx512_dequant_lane_permutation(oracle):
    rng = np.random.default_rng(10)
    w = (rng.standard_normal(256) * 0.02).astype(np.float32)
    s, p = oracle.quantize_q4(w, 32)
    scalar = oracle.dequant_layer(s, p, 256, 32)
    avx = np.empty(256, np.float32)
    oracle.lib().or_avx_dequant_layer(s, p, avx, 256)
    # unpacklo/hi_epi8 interleave within 128-bit lanes: output 16..31 receives
    # source elements 32..47 scaled by group 0, and so on.
    nib = np.stack([p & 15, p >> 4], axis=1).ravel().astype(np.float32) - 8
    src = np.concatenate([np.arange(0, 16), np.arange(32, 48), np.arange(64, 80), np.arange(96, 112),
                          np.arange(16, 32), np.arange(48, 64), np.arange(80, 96), np.arange(112, 128)])
    chunk = np.concatenate([src[:16], src[16:32], src[32:48], src[48:64], src[64:80], src[80:96], src[96:112],
                            src[112:128]])
    order = np.concatenate([chunk[0:16], chunk[16:32], chunk[32:48], chunk[48:64], chunk[64:80], chunk[80:96],
                            chunk[96:112], chunk[112:128]])
    lin = np.concatenate([order[0:64:1]])
    # first 32 outputs use scale 0 and source elements 0..15, 32..47
    assert np.array_equal(avx[:16], nib[0:16] * s[0])
    assert np.array_equal(avx[16:32], nib[32:48] * s[0])
    assert np.array_equal(avx[64:80], nib[16:32] * s[2])
    assert not np.array_equal(avx, scalar)
    del lin


def test_avx512_f16_even_element_quirk(oracle):
    h = (np.arange(16, dtype=np.uint16) + 0x3C00).astype(np.uint16)
    out = np.empty(16, np.float32)
    oracle.avx_f16_bytes_to_f32(h.view(np.uint8).copy(), out)
    ref = oracle.f16_to_f32(h)
    # lanes 0..7 take source elements 0, 2, 4, 6, 4, 6, 8, 10
    assert np.array_equal(out[:8], ref[[0, 2, 4, 6, 4, 6, 8, 10]])


# --- golden vectors ------------------------------------------------------------------

def test_golden_vectors(oracle):
    g = np.load(GOLDEN)
    assert np.array_equal(bits(oracle.f16_to_f32(g["f16_bits"])), bits(g["f16_to_f32"]))
    assert np.array_equal(bits(oracle.bf16_to_f32(g["f16_bits"])), bits(g["bf16_to_f32"]))
    assert np.array_equal(oracle.f32_to_f16(g["f32_in"]), g["f32_to_f16"])
    w = g["w"]
    assert np.array_equal(oracle.quantize_q8_0(w), g["q8_0_blocks"])
    assert np.array_equal(oracle.quantize_q4_0(w), g["q4_0_blocks"])
    assert np.array_equal(bits(oracle.dequantize_to_f32(g["q8_0_blocks"], 8, w.size)), bits(g["q8_0_deq"]))
    assert np.array_equal(bits(oracle.dequantize_to_f32(g["q4_0_blocks"], 2, w.size)), bits(g["q4_0_deq"]))
    s, p = oracle.quantize_q4(w, 32)
    assert np.array_equal(bits(s), bits(g["eng_scales"])) and np.array_equal(p, g["eng_packed"])
    assert np.array_equal(bits(oracle.dequant_layer(s, p, w.size, 32)), bits(g["eng_deq"]))
    y = oracle.gemv_4bit_into(g["gemv_eng_scales"], g["gemv_eng_packed"], g["gemv_x"], 48, 256, 32)
    assert np.array_equal(bits(y), bits(g["gemv_eng_y"]))
    y = oracle.gemv_q4_0(g["gemv_q4_0_blocks"], g["gemv_x"], 48, 256)
    assert np.array_equal(bits(y), bits(g["gemv_q4_0_y"]))
