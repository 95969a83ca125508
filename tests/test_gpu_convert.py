"""GPU parity: f16/bf16 -> f32 and f32 -> f16 conversions, bit-exact against
the oracle (formats/gguf.rs:93-126 semantics, NaN bit patterns included)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_f16_all_bit_patterns(cuda, oracle):
    from agent_harness_b200 import kernels as K
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    d = torch.from_numpy(h.view(np.int16).copy()).to(cuda)
    out = K.f16_to_f32(d).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.f16_to_f32(h)))
    outb = K.bf16_to_f32(d).cpu().numpy()
    assert np.array_equal(bits(outb), bits(oracle.bf16_to_f32(h)))


@pytest.mark.parametrize("n", [1, 7, 8, 9, 1000, 4096 * 8 + 5])
@pytest.mark.parametrize("offset", [0, 1, 8])
def test_f16_sizes_and_alignment(cuda, oracle, n, offset):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(n + offset)
    h = rng.integers(0, 65536, n + offset, dtype=np.uint32).astype(np.uint16)
    d = torch.from_numpy(h.view(np.int16).copy()).to(cuda)[offset:]
    out = K.f16_to_f32(d).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.f16_to_f32(h[offset:])))


def test_f16_config_size(cuda, oracle):
    # 45 088 768 f16 values drawn N(0,1), seed 1 (the conversion benchmark's tensor)
    from agent_harness_b200 import kernels as K
    n = 4096 * 11008
    x = K.fill_normal(n, 0.0, 1.0, 1, device=cuda)
    h = K.f32_to_f16(x)
    out = K.f16_to_f32(h)
    hc = h.cpu().numpy().view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16(x.cpu().numpy()), hc)
    assert np.array_equal(bits(out.cpu().numpy()), bits(oracle.f16_to_f32(hc)))


def test_f32_to_f16_specials(cuda, oracle):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(11)
    x = np.concatenate([rng.integers(0, 2**32, 100003, dtype=np.uint64).astype(np.uint32).view(np.float32),
                        np.array([65504, 65519.996, 65520, 2.9802322e-08, 5.96e-8, -0.0, np.inf, -np.inf, np.nan],
                                 np.float32)])
    out = K.f32_to_f16(torch.from_numpy(x).to(cuda)).cpu().numpy().view(np.uint16)
    assert np.array_equal(out, oracle.f32_to_f16(x))


def test_host_dropins(cuda, oracle):
    from agent_harness_b200 import hostapi
    rng = np.random.default_rng(12)
    h = rng.integers(0, 65536, 4099, dtype=np.uint32).astype(np.uint16)
    raw = h.view(np.uint8).tobytes()
    assert np.array_equal(bits(hostapi.f16_bytes_to_f32(raw)), bits(oracle.f16_to_f32(h)))
    assert np.array_equal(bits(hostapi.bf16_bytes_to_f32(raw)), bits(oracle.bf16_to_f32(h)))
    assert hostapi.f16_bytes_to_f32(b"").size == 0
    assert hostapi.f16_to_f32(0x3C00) == 1.0 and hostapi.f16_to_f32(0xBC00) == -1.0
    assert hostapi.bf16_to_f32(0x3F80) == 1.0
