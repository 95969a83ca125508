"""GPU parity: the tcgen05 prefill GEMM (all prompt tokens at once) against the
oracle's per-token scalar GEMV (inference/math.rs:382-418 applied per token, as
the reference's token-by-token prefill does, inference/mod.rs:550), plus a
torch fp32 matmul of the bit-exact dequantised weight at full size.
Tolerance (north star, prefill GEMM): normwise max|C - ref| / max|ref| <= 2e-3."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3


def relerr(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _weight(K, rows, cols, seed, cuda):
    blocks = K.synth_q4_0(rows, cols, 0.02, seed, device=cuda)
    return blocks, K.Q4Weight.from_q4_0(blocks, rows, cols)


def test_config_prefill_gemm_512x14336x4096(cuda, oracle):
    # W 14336x4096 ~ N(0,0.02) seed 4 as Q4_0; A 512x4096 ~ N(0,1) seed 5
    from agent_harness_b200 import kernels as K
    M, N, Kc = 512, 14336, 4096
    blocks, W = _weight(K, N, Kc, 4, cuda)
    a = K.fill_normal(M * Kc, 0.0, 1.0, 5, device=cuda).reshape(M, Kc)
    c = W.gemm(a)
    torch.cuda.synchronize()
    ch = c.cpu().numpy()
    assert np.all(np.isfinite(ch))
    # oracle on a token sample (first, last, both tile halves, ragged picks)
    rows = [0, 1, 127, 128, 255, 256, 300, 383, 384, 511]
    ah = a.cpu().numpy()
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), ah[rows], N)
    for i, r in enumerate(rows):
        assert relerr(ch[r], ref[i]) <= TOL, (r, relerr(ch[r], ref[i]))
    err_sample = relerr(ch[rows], ref)
    assert err_sample < 1e-3, err_sample
    # full size against torch fp32 on the bit-exact dequantised weight
    wf = K.dequant_q4_0(blocks, N * Kc).reshape(N, Kc)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        full = (a @ wf.t()).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert relerr(ch, full) <= TOL, relerr(ch, full)
    assert torch.equal(W.gemm(a), c)  # deterministic: same bits on a second call
    W.close()


@pytest.mark.parametrize("m,n,k", [(1, 16, 64), (7, 100, 96), (128, 208, 128), (129, 209, 64),
                                   (300, 3000, 4096 + 32), (256, 416, 512), (40, 14336 // 8, 1024)])
def test_ragged_shapes(cuda, oracle, m, n, k):
    from agent_harness_b200 import kernels as K
    blocks, W = _weight(K, n, k, m * 31 + n * 7 + k, cuda)
    a = K.fill_normal(m * k, 0.0, 1.0, m + k, device=cuda).reshape(m, k)
    c = W.gemm(a).cpu().numpy()
    assert c.shape == (m, n)
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), a.cpu().numpy(), n)
    assert relerr(c, ref) <= TOL, relerr(c, ref)
    W.close()


def test_strided_output_and_empty(cuda, oracle):
    from agent_harness_b200 import kernels as K
    m, n, k = 130, 224, 256
    blocks, W = _weight(K, n, k, 11, cuda)
    a = K.fill_normal(m * k, 0.0, 1.0, 12, device=cuda).reshape(m, k)
    big = torch.full((m, n + 40), 7.0, device=cuda)
    out = big[:, :n]
    from agent_harness_b200._lib import call
    from agent_harness_b200.kernels import _ptr, _stream
    import ctypes as C
    need = W.gemm_workspace_bytes(m)
    ws = torch.empty(need + 1024, dtype=torch.uint8, device=cuda)
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    call("ah_q4w_gemm", W.handle, _ptr(a), k, m, C.c_void_p(big.data_ptr()), n + 40, C.c_void_p(base), need,
         _stream(cuda))
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), a.cpu().numpy(), n)
    assert relerr(out.cpu().numpy(), ref) <= TOL
    assert torch.all(big[:, n:] == 7.0)  # columns past ldc's logical rows untouched
    # m == 0: no work, no error
    call("ah_q4w_gemm", W.handle, _ptr(a), k, 0, C.c_void_p(big.data_ptr()), n + 40, C.c_void_p(base), need,
         _stream(cuda))
    # workspace too small -> AH_EINVAL
    from agent_harness_b200._lib import AhError
    with pytest.raises(AhError):
        call("ah_q4w_gemm", W.handle, _ptr(a), k, m, C.c_void_p(big.data_ptr()), n + 40, C.c_void_p(base),
             need - 1, _stream(cuda))
    W.close()


def test_engine_format_weights(cuda, oracle):
    # engine storage (f32 scales, linear nibbles) through the same GEMM
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(21)
    m, n, k = 200, 96, 320
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    s, p = oracle.quantize_q4(w, 32)
    a = rng.standard_normal((m, k)).astype(np.float32)
    W = K.Q4Weight.from_engine(torch.from_numpy(s).to(cuda), torch.from_numpy(p).to(cuda), n, k)
    c = W.gemm(torch.from_numpy(a).to(cuda)).cpu().numpy()
    for i in (0, 57, 199):
        ref = oracle.gemv_4bit_into(s, p, a[i], n, k, 32)
        assert relerr(c[i], ref) <= TOL, i
    W.close()


def test_activation_scaling_extremes(cuda, oracle):
    # per-token power-of-two scaling keeps tiny and huge rows in f16 range
    from agent_harness_b200 import kernels as K
    m, n, k = 8, 64, 512
    blocks, W = _weight(K, n, k, 13, cuda)
    rng = np.random.default_rng(4)
    a = rng.standard_normal((m, k)).astype(np.float32)
    for i, sc in enumerate((1e-30, 1e-6, 1.0, 3e4, 1e30)):
        a[i] *= sc
    a[5] = 0.0
    a[6, 3] = np.nan
    c = W.gemm(torch.from_numpy(a).to(cuda)).cpu().numpy()
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), a, n)
    for i in range(5):
        assert relerr(c[i], ref[i]) <= TOL, i
    assert np.all(c[5] == 0)
    assert np.all(np.isnan(c[6]))
    assert relerr(c[7], ref[7]) <= TOL
    W.close()


def test_no_device_timeouts_recorded(cuda):
    from agent_harness_b200._lib import lib
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0
