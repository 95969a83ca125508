"""GPU parity: block dequantisation and the quantisers, bit-exact against the
oracle (formats/gguf.rs:434-535, models/quantization.rs:369-454)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_config_q8_0_full_size(cuda, oracle):
    # 4096 x 11008 weights ~ N(0, 0.02), seed 0 -> Q8_0 -> f32, bit-exact
    from agent_harness_b200 import kernels as K
    n = 4096 * 11008
    w = K.fill_normal(n, 0.0, 0.02, 0, device=cuda)
    blocks = K.quantize_q8_0(w)
    wh = w.cpu().numpy()
    bh = blocks.cpu().numpy()
    assert np.array_equal(bh, oracle.quantize_q8_0(wh))
    out = K.dequant_q8_0(blocks, n).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.dequantize_to_f32(bh, 8, n)))


def test_q4_0_and_engine_full_size(cuda, oracle):
    from agent_harness_b200 import kernels as K
    n = 4096 * 11008
    w = K.fill_normal(n, 0.0, 0.02, 2, device=cuda)
    wh = w.cpu().numpy()
    b4 = K.quantize_q4_0(w)
    b4h = b4.cpu().numpy()
    assert np.array_equal(b4h, oracle.quantize_q4_0(wh))
    assert np.array_equal(bits(K.dequant_q4_0(b4, n).cpu().numpy()), bits(oracle.dequantize_to_f32(b4h, 2, n)))
    s, p = K.quantize_q4(w, 32)
    so, po = oracle.quantize_q4(wh, 32)
    assert np.array_equal(bits(s.cpu().numpy()), bits(so)) and np.array_equal(p.cpu().numpy(), po)
    assert np.array_equal(bits(K.dequant_layer(s, p, n, 32).cpu().numpy()), bits(oracle.dequant_layer(so, po, n, 32)))


@pytest.mark.parametrize("n", [1, 31, 32, 33, 4095, 4096 * 32 + 7, 256 * 32 * 5 + 64])
def test_ragged_sizes(cuda, oracle, n):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(n)
    wh = (rng.standard_normal(n) * 0.02).astype(np.float32)
    w = torch.from_numpy(wh).to(cuda)
    for fmt, q, dq, code in (("q8", K.quantize_q8_0, K.dequant_q8_0, 8), ("q4", K.quantize_q4_0, K.dequant_q4_0, 2)):
        b = q(w)
        bh = b.cpu().numpy()
        ref_b = oracle.quantize_q8_0(wh) if fmt == "q8" else oracle.quantize_q4_0(wh)
        assert np.array_equal(bh, ref_b), fmt
        assert np.array_equal(bits(dq(b, n).cpu().numpy()), bits(oracle.dequantize_to_f32(bh, code, n))), fmt
    for gs in (32, 7, 64):
        s, p = K.quantize_q4(w, gs)
        so, po = oracle.quantize_q4(wh, gs)
        assert np.array_equal(bits(s.cpu().numpy()), bits(so)) and np.array_equal(p.cpu().numpy(), po), gs
        assert np.array_equal(bits(K.dequant_layer(s, p, n, gs).cpu().numpy()), bits(oracle.dequant_layer(so, po, n, gs)))


def test_misaligned_blocks(cuda, oracle):
    # blocks starting 2 bytes past a 16-byte boundary take the element-wise path
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(21)
    n = 128 * 32 * 9 + 40
    wh = (rng.standard_normal(n) * 0.02).astype(np.float32)
    for code, qz, bsz in ((8, oracle.quantize_q8_0, 34), (2, oracle.quantize_q4_0, 18)):
        bh = qz(wh)
        buf = torch.zeros(bh.size + 16, dtype=torch.uint8, device=cuda)
        buf[2:2 + bh.size] = torch.from_numpy(bh).to(cuda)
        view = buf[2:2 + bh.size]
        out = (K.dequant_q8_0 if code == 8 else K.dequant_q4_0)(view, n).cpu().numpy()
        assert np.array_equal(bits(out), bits(oracle.dequantize_to_f32(bh, code, n)))


def test_nan_inf_scales_bit_exact(cuda, oracle):
    # d = inf with q = 0 gives x86's default NaN 0xFFC00000; NaN d propagates quieted
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(22)
    nb = 128 * 4
    q8 = rng.integers(0, 256, (nb, 34), dtype=np.uint8)
    ds = np.array([0x7C00, 0xFC00, 0x7E00, 0xFC01, 0x7C01, 0x0001, 0x8000, 0x0000], np.uint16)
    q8[:, :2] = ds[np.arange(nb) % ds.size].view(np.uint8).reshape(-1, 2)
    q8[::3, 2:6] = 0
    q8h = q8.ravel().copy()
    out = K.dequant_q8_0(torch.from_numpy(q8h).to(cuda), nb * 32).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.dequantize_to_f32(q8h, 8, nb * 32)))
    q4 = rng.integers(0, 256, (nb * 2, 18), dtype=np.uint8)
    q4[:, :2] = ds[np.arange(nb * 2) % ds.size].view(np.uint8).reshape(-1, 2)
    q4[::2, 2:4] = 0x88
    q4h = q4.ravel().copy()
    out = K.dequant_q4_0(torch.from_numpy(q4h).to(cuda), nb * 64).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.dequantize_to_f32(q4h, 2, nb * 64)))
    # engine format: NaN scales with payloads, infinities
    s = np.array([np.inf, -np.inf, 0.0, 1.0], np.float32)
    s = np.concatenate([s, np.array([0x7F800001, 0xFF812345, 0x7FC00000], np.uint32).view(np.float32)])
    s = np.tile(s, 64)
    p = rng.integers(0, 256, s.size * 16, dtype=np.uint8)
    p[::5] = 0x88
    n = s.size * 32
    out = K.dequant_layer(torch.from_numpy(s).to(cuda), torch.from_numpy(p).to(cuda), n, 32).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.dequant_layer(s, p, n, 32)))


def test_dequantize_to_f32_dispatch(cuda, oracle):
    from agent_harness_b200 import kernels as K
    from agent_harness_b200._lib import AhError
    rng = np.random.default_rng(23)
    raw = rng.integers(0, 256, 34 * 50 + 13, dtype=np.uint8)
    # Q6_K approximate branch needs whole 210-byte blocks
    raw6 = rng.integers(0, 256, 210 * 9 + 100, dtype=np.uint8)
    for dtype, r, n in ((0, raw, 1000), (1, raw, 3), (30, raw, 10), (8, raw, 5000), (8, raw, 100), (2, raw[:18 * 40], 40 * 32),
                        (2, raw[:18 * 40 + 1], 4000), (13, raw6, 256 * 20), (13, raw6, 700), (77, raw, 123)):
        got = K.dequantize_to_f32(torch.from_numpy(r.copy()).to(cuda), dtype, n).cpu().numpy()
        ref = oracle.dequantize_to_f32(r, dtype, n)
        assert got.size == ref.size, (dtype, n)
        assert np.array_equal(bits(got), bits(ref)), (dtype, n)
    with pytest.raises(AhError):  # truncated Q4_0 block: the reference panics
        K.dequantize_to_f32(torch.from_numpy(raw[:18 * 3 + 7].copy()).to(cuda), 2, 200)


def test_golden_vectors(cuda):
    import os
    from agent_harness_b200 import kernels as K
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    w = torch.from_numpy(g["w"]).to(cuda)
    n = g["w"].size
    assert np.array_equal(K.quantize_q8_0(w).cpu().numpy(), g["q8_0_blocks"])
    assert np.array_equal(K.quantize_q4_0(w).cpu().numpy(), g["q4_0_blocks"])
    assert np.array_equal(bits(K.dequant_q8_0(torch.from_numpy(g["q8_0_blocks"]).to(cuda), n).cpu()), bits(g["q8_0_deq"]))
    assert np.array_equal(bits(K.dequant_q4_0(torch.from_numpy(g["q4_0_blocks"]).to(cuda), n).cpu()), bits(g["q4_0_deq"]))
    s, p = K.quantize_q4(w, 32)
    assert np.array_equal(bits(s.cpu()), bits(g["eng_scales"])) and np.array_equal(p.cpu().numpy(), g["eng_packed"])
    h = torch.from_numpy(g["f16_bits"].view(np.int16).copy()).to(cuda)
    assert np.array_equal(bits(K.f16_to_f32(h).cpu()), bits(g["f16_to_f32"]))


def test_host_dropins(cuda, oracle):
    from agent_harness_b200 import hostapi
    rng = np.random.default_rng(24)
    w = (rng.standard_normal(1000) * 0.02).astype(np.float32)
    s, p = hostapi.quantize(w, 32)
    so, po = oracle.quantize_q4(w, 32)
    assert np.array_equal(bits(s), bits(so)) and np.array_equal(p, po)
    res = np.empty(1000, np.float32)
    hostapi.dequant_layer(s, p, res, 32)
    assert np.array_equal(bits(res), bits(oracle.dequant_layer(so, po, 1000, 32)))
    for i in (0, 1, 31, 32, 999):
        assert bits(hostapi.dequant_weight(s, p, i, 32)) == bits(res[i])
    raw = oracle.quantize_q8_0(w)
    assert np.array_equal(bits(hostapi.dequantize_to_f32(raw, 8, 1000)), bits(oracle.dequantize_to_f32(raw, 8, 1000)))
