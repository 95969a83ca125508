"""GPU parity: the tcgen05 batched decode GEMV (1..16 tokens, weights
dequantised into tensor memory, stream-K over persistent CTAs) against the
oracle's per-token scalar GEMV (inference/math.rs:382-418 per token, as the
reference's decode runs gemv_4bit_into for each sequence), plus a torch fp32
matmul of the bit-exact dequantised weight at the 70B projection shapes.
Tolerance (f16 tensor-core operands with f32 accumulation, as the
prefill GEMM): normwise max|y - ref| / max|ref| <= 2e-3."""
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


def _torch_ref(K, blocks, x, rows, cols):
    wf = K.dequant_q4_0(blocks, rows * cols).reshape(rows, cols)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return (x @ wf.t()).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("rows,cols", [(10240, 8192), (57344 // 8, 8192), (8192, 28672 // 8)])
def test_70b_projection_shapes_batch16(cuda, oracle, rows, cols):
    # the fused q|k|v (TP1), a gate/up slice and a down slice of the 70B widths
    from agent_harness_b200 import kernels as K
    B = 16
    blocks, W = _weight(K, rows, cols, rows + cols, cuda)
    x = K.fill_normal(B * cols, 0.0, 1.0, 7, device=cuda).reshape(B, cols)
    y = W.gemv_tc(x)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    assert np.all(np.isfinite(yh))
    # oracle on three tokens, torch fp32 on all sixteen
    picks = [0, 7, 15]
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), x.cpu().numpy()[picks], rows)
    for i, b in enumerate(picks):
        assert relerr(yh[b], ref[i]) <= TOL, (b, relerr(yh[b], ref[i]))
    full = _torch_ref(K, blocks, x, rows, cols)
    assert relerr(yh, full) <= TOL, relerr(yh, full)
    # deterministic: the stream-K partials are added in a fixed order
    assert torch.equal(W.gemv_tc(x), y)
    W.close()


@pytest.mark.parametrize("b,n,k", [(16, 16, 64), (9, 100, 96), (1, 208, 128), (13, 3000, 4096 + 32),
                                   (16, 1000, 2048), (12, 128, 64 * 300), (16, 16 * 1001, 512), (5, 7, 32)])
def test_ragged_shapes(cuda, oracle, b, n, k):
    # odd block-pair counts (zero-filled half steps), partial row blocks,
    # row blocks shared by many CTAs (few rows, long K) and one-step blocks
    from agent_harness_b200 import kernels as K
    blocks, W = _weight(K, n, k, b * 31 + n * 7 + k, cuda)
    x = K.fill_normal(b * k, 0.0, 1.0, b + k, device=cuda).reshape(b, k)
    y = W.gemv_tc(x).cpu().numpy()
    assert y.shape == (b, n)
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), x.cpu().numpy(), n)
    assert relerr(y, ref) <= TOL, relerr(y, ref)
    W.close()


def test_accumulate_and_strides(cuda, oracle):
    from agent_harness_b200 import kernels as K
    b, n, k = 11, 300, 1024
    blocks, W = _weight(K, n, k, 3, cuda)
    xs = K.fill_normal(b * (k + 64), 0.0, 1.0, 4, device=cuda).reshape(b, k + 64)
    x = xs[:, :k]
    big = torch.full((b, n + 24), 0.5, device=cuda)
    out = big[:, :n]
    W.gemv_tc(x, out=out, accumulate=True)
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), x.cpu().numpy(), n) + 0.5
    assert relerr(out.cpu().numpy(), ref) <= TOL
    assert torch.all(big[:, n:] == 0.5)  # entries past the rows untouched
    # batch outside 1..16 and a short workspace are refused before any launch
    from agent_harness_b200._lib import AhError, call
    from agent_harness_b200.kernels import _ptr, _stream
    import ctypes as C
    need = W.gemv_tc_workspace_bytes()
    ws = torch.empty(need + 1024, dtype=torch.uint8, device=cuda)
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    for batch, nbytes in ((17, need), (0, need), (b, need - 1)):
        with pytest.raises(AhError):
            call("ah_q4w_gemv_tc", W.handle, C.c_void_p(x.data_ptr()), k + 64, batch, C.c_void_p(out.data_ptr()),
                 n + 24, 0, C.c_void_p(base),
                 nbytes, _stream(cuda))
    W.close()


def test_engine_format_weights(cuda, oracle):
    # engine storage (f32 scales) through the same kernel
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(22)
    b, n, k = 16, 272, 640
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    s, p = oracle.quantize_q4(w, 32)
    x = rng.standard_normal((b, k)).astype(np.float32)
    W = K.Q4Weight.from_engine(torch.from_numpy(s).to(cuda), torch.from_numpy(p).to(cuda), n, k)
    y = W.gemv_tc(torch.from_numpy(x).to(cuda)).cpu().numpy()
    for i in (0, 9, 15):
        ref = oracle.gemv_4bit_into(s, p, x[i], n, k, 32)
        assert relerr(y[i], ref) <= TOL, i
    W.close()


def test_token_scaling_extremes(cuda, oracle):
    # per-token power-of-two scaling keeps tiny and huge rows in f16 range
    from agent_harness_b200 import kernels as K
    b, n, k = 8, 64, 512
    blocks, W = _weight(K, n, k, 13, cuda)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((b, k)).astype(np.float32)
    for i, sc in enumerate((1e-30, 1e-6, 1.0, 3e4, 1e30)):
        x[i] *= sc
    x[5] = 0.0
    x[6, 3] = np.nan
    y = W.gemv_tc(torch.from_numpy(x).to(cuda)).cpu().numpy()
    ref = oracle.gemm_q4_0(blocks.cpu().numpy(), x, n)
    for i in range(5):
        assert relerr(y[i], ref[i]) <= TOL, i
    assert np.all(y[5] == 0)
    assert np.all(np.isnan(y[6]))
    assert relerr(y[7], ref[7]) <= TOL
    W.close()


def test_matches_mma_sync_gemv(cuda):
    # the two decode GEMV paths agree within the f16 operand rounding
    from agent_harness_b200 import kernels as K
    b, n, k = 16, 4096, 4096
    blocks, W = _weight(K, n, k, 17, cuda)
    x = K.fill_normal(b * k, 0.0, 1.0, 18, device=cuda).reshape(b, k)
    y_tc = W.gemv_tc(x).cpu().numpy()
    y_ms = W.gemv(x).cpu().numpy()
    assert relerr(y_tc, y_ms) <= TOL
    W.close()


def test_no_device_timeouts_recorded(cuda):
    from agent_harness_b200._lib import lib
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0


def test_mma_rate_probe(cuda):
    # the diagnostic behind the kernel's design: an M=128 MMA with A in tensor
    # memory costs the same for N = 16 and N = 128 (within 10%), and issue
    # waits for completion (issue time >= 80% of completion time)
    import ctypes as C
    from agent_harness_b200._lib import AhError, call
    t = {}
    for n in (16, 128):
        out = (C.c_longlong * 3)()
        call("ah_debug_tc_mma_rate", 1, n, C.cast(out, C.c_void_p))
        assert out[0] > 0 and out[1] >= out[0] and out[2] > 0
        assert out[0] >= 0.8 * out[1]
        t[n] = out[1]
    assert abs(t[16] - t[128]) <= 0.1 * t[128]
    with pytest.raises(AhError):
        call("ah_debug_tc_mma_rate", 2, 16, C.cast((C.c_longlong * 3)(), C.c_void_p))  # the pair form needs N >= 32
