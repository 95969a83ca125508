"""GPU parity: the tcgen05 prefill GEMM (all prompt tokens at once) against the
oracle's per-token scalar GEMV (inference/math.rs:382-418 applied per token, as
the reference's token-by-token prefill does, inference/mod.rs:550), plus a
torch fp32 matmul of the bit-exact dequantised weight at full size.
Tolerance (prefill GEMM, f16 operands with f32 accumulation): normwise max|C - ref| / max|ref| <= 2e-3."""
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


def _silu(v):
    return v / (1.0 + np.exp(-v))


@pytest.mark.parametrize("m", [5, 130, 300])
def test_fused_epilogues_and_norm(cuda, oracle, m):
    # the prefill step's fusions through ah_q4w_gemm_ex against the oracle:
    # SwiGLU over an interleaved gate/up weight (inference/ffn.rs:155-174 per
    # token), the residual add (inference/mod.rs:505-545) and the RMSNorm
    # prologue (inference/math.rs:53-63); aligned rows take the bulk-copy
    # epilogue, rows of an odd stride the per-element stores
    from agent_harness_b200 import kernels as K
    n_embd, n_ff = 512, 384
    gate = K.synth_q4_0(n_ff, n_embd, 0.05, 11, device=cuda)
    up = K.synth_q4_0(n_ff, n_embd, 0.05, 12, device=cuda)
    down = K.synth_q4_0(n_embd, n_ff, 0.05, 13, device=cuda)
    blk = K.SwigluBlock.from_q4_0(gate, up, down, n_embd, n_ff)
    x = K.fill_normal(m * n_embd, 0.0, 1.0, 14, device=cuda).reshape(m, n_embd)
    xh = x.cpu().numpy()
    g = oracle.gemm_q4_0(gate.cpu().numpy(), xh, n_ff).astype(np.float64)
    u = oracle.gemm_q4_0(up.cpu().numpy(), xh, n_ff).astype(np.float64)
    ref_act = _silu(g) * u
    act = blk.gate_up.gemm(x, epilogue="swiglu")
    assert act.shape == (m, n_ff)
    assert relerr(act.cpu().numpy(), ref_act) <= TOL
    wide = torch.full((m, n_ff + 1), 7.0, device=cuda)
    blk.gate_up.gemm(x, out=wide[:, :n_ff], epilogue="swiglu")
    assert relerr(wide[:, :n_ff].cpu().numpy(), ref_act) <= TOL
    assert torch.all(wide[:, n_ff] == 7.0)
    # residual add into hidden rows
    h0 = K.fill_normal(m * n_embd, 0.0, 1.0, 15, device=cuda).reshape(m, n_embd)
    ref_h = h0.cpu().numpy() + oracle.gemm_q4_0(down.cpu().numpy(), act.cpu().numpy(), n_embd)
    h = h0.clone()
    blk.down.gemm(act, out=h, epilogue="add")
    assert relerr(h.cpu().numpy(), ref_h) <= TOL
    hw = torch.zeros(m, n_embd + 3, device=cuda)
    hw[:, :n_embd] = h0
    blk.down.gemm(act, out=hw[:, :n_embd], epilogue="add")
    assert relerr(hw[:, :n_embd].cpu().numpy(), ref_h) <= TOL
    assert torch.all(hw[:, n_embd:] == 0)
    # RMSNorm prologue (f16 norm weight), then SwiGLU
    w16 = K.synth_f16(n_embd, 1.0, 0.1, 16, device=cuda)
    wf = oracle.f16_to_f32(w16.cpu().numpy().view(np.uint16))
    xn = np.stack([oracle.rms_norm(xh[i], wf, 1e-5) for i in range(m)])
    gn = oracle.gemm_q4_0(gate.cpu().numpy(), xn, n_ff).astype(np.float64)
    un = oracle.gemm_q4_0(up.cpu().numpy(), xn, n_ff).astype(np.float64)
    act_n = blk.gate_up.gemm(x, epilogue="swiglu", norm_w=w16, eps=1e-5)
    assert relerr(act_n.cpu().numpy(), _silu(gn) * un) <= TOL
    y = K.Q4Weight.from_q4_0(down, n_embd, n_ff)
    yn = y.gemm(act, norm_w=K.synth_f16(n_ff, 1.0, 0.1, 17, device=cuda), eps=1e-6)
    wf2 = oracle.f16_to_f32(K.synth_f16(n_ff, 1.0, 0.1, 17, device=cuda).cpu().numpy().view(np.uint16))
    an = np.stack([oracle.rms_norm(act.cpu().numpy()[i], wf2, 1e-6) for i in range(m)])
    assert relerr(yn.cpu().numpy(), oracle.gemm_q4_0(down.cpu().numpy(), an, n_embd)) <= TOL
    y.close()
    blk.close()


def test_fused_epilogue_arguments_refused(cuda):
    from agent_harness_b200 import kernels as K
    from agent_harness_b200._lib import AhError
    W = K.Q4Weight.from_q4_0(K.synth_q4_0(24, 64, 0.05, 1, device=cuda), 24, 64)
    a = torch.zeros(4, 64, device=cuda)
    with pytest.raises(AhError):
        W.gemm(a, epilogue="swiglu")  # 24 rows: not whole 16-row gate/up tiles
    with pytest.raises(AhError):
        W.gemm(a, out=torch.zeros(4, 24), epilogue="add")  # host output
    W.close()
