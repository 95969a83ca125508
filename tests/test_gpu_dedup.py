"""GPU parity of the DedupCount decode (models/dedup/) and of the fused load
path (decode + quantize + tiled repack), bit-exact against the oracle:

* decompress_all / decompress_all_global / decompress_with_remap element by
  element, including the reference's fallbacks for short sandbags and
  out-of-range indices, on aligned (vector) and misaligned (scalar) arrays;
* the remap path's panic cases surface as AH_EINVAL from the device error word;
* to_q4weight's device planes equal quantize() of the decoded values followed
  by the engine-format repack, at ragged and full decoder shapes."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def bits_equal(a, b):
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else a
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def compressed(oracle, n, std, pd=2, rounds=2, seed=0):
    w = (np.random.default_rng(seed).standard_normal(n) * std).astype(np.float32)
    return oracle.dedup_compress(w, pd, rounds)


def to_mine(ot, os_):
    from agent_harness_b200 import dedup as D
    t = D.DedupCountTensor(ot.prefixes, ot.tail_values, ot.count, ot.prefix_digits, ot.tail_digits,
                           ot.avg_precision_lost)
    return t, D.Sandbag(os_.prefix_idx, os_.tail_idx, os_.sign_bits, os_.count)


@pytest.mark.parametrize("n", [1, 7, 8, 1000, 65543])
def test_decompress_all_matches_oracle(cuda, oracle, n):
    ot, os_ = compressed(oracle, n, 0.03, seed=n)
    t, s = to_mine(ot, os_)
    assert bits_equal(t.decompress_all(s), oracle.dedup_decompress_all(ot, os_))


def test_decompress_all_fallbacks_and_misaligned(cuda, oracle):
    from agent_harness_b200 import dedup as D
    ot = oracle.DedupTensor([7, 2, 40], [11, 40000, 3], 45, 1, 4, -1e-6)
    rng = np.random.default_rng(1)
    os_ = oracle.Sandbag(rng.integers(0, 5, 37), rng.integers(0, 5, 29), rng.integers(0, 256, 3), 45)
    t, _ = to_mine(ot, os_)
    want = oracle.dedup_decompress_all(ot, os_)
    # device arrays one element into a larger allocation: not 16-byte aligned
    dev = torch.device("cuda")
    p = torch.zeros(38, dtype=torch.int16, device=dev)
    p[1:] = torch.as_tensor(os_.prefix_idx.view(np.int16))
    tt = torch.zeros(30, dtype=torch.int16, device=dev)
    tt[1:] = torch.as_tensor(os_.tail_idx.view(np.int16))
    got = t.decompress_all(D.Sandbag(p[1:], tt[1:], torch.as_tensor(os_.sign_bits), 45))
    assert bits_equal(got, want)
    assert bits_equal(t.decompress_all(D.Sandbag(os_.prefix_idx, os_.tail_idx, os_.sign_bits, 45)), want)


def test_host_drop_in(cuda, oracle):
    from agent_harness_b200 import _lib
    ot, os_ = compressed(oracle, 4099, 0.02, seed=5)
    out = np.empty(ot.count, np.float32)
    _lib.call("ah_host_dedup_decompress_all", ot.prefixes.ctypes.data, ot.prefixes.size, ot.tail_values.ctypes.data,
              ot.tail_values.size, ot.count, ot.prefix_digits, ot.tail_digits, ot.avg_precision_lost,
              os_.prefix_idx.ctypes.data, os_.prefix_idx.size, os_.tail_idx.ctypes.data, os_.tail_idx.size,
              os_.sign_bits.ctypes.data, os_.sign_bits.size, out.ctypes.data)
    assert bits_equal(out, oracle.dedup_decompress_all(ot, os_))


def _global(oracle, chunks):
    from agent_harness_b200 import dedup as D
    og = oracle.dedup_global_table_new([c[0] for c in chunks])
    rows = [og.row(i) for i in range(og.prefixes.size)]
    return og, D.GlobalTable(og.prefix_digits, og.prefixes, rows)


def test_decompress_all_global_matches_oracle(cuda, oracle):
    rng = np.random.default_rng(2)
    chunks = [oracle.dedup_compress((rng.standard_normal(n) * s).astype(np.float32), pd, 2)
              for n, s, pd in ((3001, 0.02, 2), (2000, 0.05, 2), (1500, 0.04, 1))]
    og, g = _global(oracle, chunks)
    for ot, os_ in chunks:
        t, s = to_mine(ot, os_)
        assert bits_equal(t.decompress_all_global(s, g), oracle.dedup_decompress_all_global(ot, os_, og))
    # a sandbag that runs out early and indices past the tables use the fallbacks
    ot, os_ = chunks[0]
    short = oracle.Sandbag(np.append(os_.prefix_idx[:100], 999), os_.tail_idx[:90], os_.sign_bits[:5], os_.count)
    t, s = to_mine(ot, short)
    assert bits_equal(t.decompress_all_global(s, g), oracle.dedup_decompress_all_global(ot, short, og))


def test_decompress_with_remap_matches_oracle(cuda, oracle):
    from agent_harness_b200 import _lib
    rng = np.random.default_rng(3)
    chunks = [oracle.dedup_compress((rng.standard_normal(2500) * 0.03).astype(np.float32), 2, 2) for _ in range(3)]
    og, g = _global(oracle, chunks)
    for ot, os_ in chunks:
        remap = oracle.dedup_build_chunk_remap(og, ot)
        t, s = to_mine(ot, os_)
        got = g.decompress_with_remap(s, t, remap)
        assert bits_equal(got, oracle.dedup_decompress_with_remap(og, os_, ot, remap))
    # a prefix index past the tensor's prefixes panics in the reference: AH_EINVAL here
    ot, os_ = chunks[0]
    bad = os_.prefix_idx.copy()
    bad[17] = ot.prefixes.size + 3
    t, s = to_mine(ot, oracle.Sandbag(bad, os_.tail_idx, os_.sign_bits, os_.count))
    g.decompress_with_remap(s, t, oracle.dedup_build_chunk_remap(og, ot))
    torch.cuda.synchronize()
    assert _lib.lib().ah_check_device_error(None) == -1  # AH_EINVAL
    assert _lib.lib().ah_check_device_error(None) == 0


@pytest.mark.parametrize("rows,cols", [(1, 32), (100, 96), (37, 4096), (4096, 14336)])
def test_to_q4weight_equals_quantize_then_repack(cuda, oracle, rows, cols):
    from agent_harness_b200 import dedup as D
    from agent_harness_b200 import kernels as K
    n = rows * cols
    if n <= 200_000:
        ot, os_ = compressed(oracle, n, 0.02, seed=rows)
        t, s = to_mine(ot, os_)
        dec = oracle.dedup_decompress_all(ot, os_)
        scales = np.empty((n + 31) // 32, np.float32)
        packed = np.empty((n + 1) // 2, np.uint8)
        oracle.lib().or_quantize_q4(dec, n, 32, scales, packed)
        ref = K.Q4Weight.from_engine(torch.as_tensor(scales).cuda(), torch.as_tensor(packed).cuda(), rows, cols)
    else:  # decoder shape: synthetic sandbag; the reference is the GPU's own bit-exact two-step path
        rng = np.random.default_rng(7)
        t = D.DedupCountTensor(np.arange(12) * 3, np.sort(rng.choice(60000, 900, replace=False)), n, 2, 3, 2e-6)
        s = D.Sandbag(torch.randint(0, 12, (n,), dtype=torch.int16, device="cuda"),
                      torch.randint(0, 900, (n,), dtype=torch.int16, device="cuda"),
                      torch.randint(0, 256, ((n + 7) // 8,), dtype=torch.uint8, device="cuda"), n)
        dec = t.decompress_all(s)
        sc, pk = K.quantize_q4(dec)
        ref = K.Q4Weight.from_engine(sc, pk, rows, cols)
    w = t.to_q4weight(s, rows, cols)
    torch.cuda.synchronize()
    n1, s1, f1 = w.planes()
    n2, s2, f2 = ref.planes()
    assert f1 and f2
    assert torch.equal(n1, n2)
    assert torch.equal(s1, s2)
    x = torch.randn(cols, device="cuda")
    assert torch.equal(w.gemv(x), ref.gemv(x))
    w.close()
    ref.close()
