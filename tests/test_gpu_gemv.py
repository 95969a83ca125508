"""GPU parity: the fused Q4 dequant+GEMV (inference/math.rs:255-418) against
the oracle's scalar GEMV.  Tolerance (the f32-accumulate parity bar): normwise relative error
max|y - ref| / max|ref| <= 1e-3 with f32 accumulation."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def relerr(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _q4_0_weight(K, rows, cols, seed, cuda):
    blocks = K.synth_q4_0(rows, cols, 0.02, seed, device=cuda)
    return blocks, K.Q4Weight.from_q4_0(blocks, rows, cols)


def test_config_gemv_4096(cuda, oracle):
    # W 4096x4096 ~ N(0,0.02) seed 2 as Q4_0; x ~ N(0,1) seed 3; batch 1
    from agent_harness_b200 import kernels as K
    blocks, W = _q4_0_weight(K, 4096, 4096, 2, cuda)
    x = K.fill_normal(4096, 0.0, 1.0, 3, device=cuda)
    y = W.gemv(x).cpu().numpy()
    ref = oracle.gemv_q4_0(blocks.cpu().numpy(), x.cpu().numpy(), 4096, 4096)
    err = relerr(y, ref)
    assert err <= TOL, err
    assert err < 1e-5  # the split-f16 tensor-core path is f32-grade in practice
    assert W.weight_bytes == 4096 * 128 * 18


@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 12, 16])
def test_batched(cuda, oracle, batch):
    from agent_harness_b200 import kernels as K
    rows, cols = 1024, 2048
    blocks, W = _q4_0_weight(K, rows, cols, 40 + batch, cuda)
    x = K.fill_normal(batch * cols, 0.0, 1.0, 50 + batch, device=cuda).reshape(batch, cols)
    y = W.gemv(x).cpu().numpy()
    bh, xh = blocks.cpu().numpy(), x.cpu().numpy()
    for b in range(batch):
        ref = oracle.gemv_q4_0(bh, xh[b], rows, cols)
        assert relerr(y[b], ref) <= TOL, (batch, b, relerr(y[b], ref))


@pytest.mark.parametrize("rows,cols", [(1, 32), (17, 64), (100, 96), (300, 4096 + 32), (16, 14336)])
def test_ragged_shapes(cuda, oracle, rows, cols):
    from agent_harness_b200 import kernels as K
    blocks, W = _q4_0_weight(K, rows, cols, rows * 7 + cols, cuda)
    x = K.fill_normal(cols, 0.0, 1.0, 9, device=cuda)
    y = W.gemv(x).cpu().numpy()
    assert y.shape == (rows,)
    ref = oracle.gemv_q4_0(blocks.cpu().numpy(), x.cpu().numpy(), rows, cols)
    assert relerr(y, ref) <= TOL


def test_large_batch_and_k(cuda, oracle):
    # batch 16 at K = 14336: 28 block pairs per cluster CTA (register ping-pong
    # over several batches); run twice (no state carried between calls).
    from agent_harness_b200 import kernels as K
    rows, cols, batch = 256, 14336, 16
    blocks, W = _q4_0_weight(K, rows, cols, 77, cuda)
    x = K.fill_normal(batch * cols, 0.0, 1.0, 78, device=cuda).reshape(batch, cols)
    bh, xh = blocks.cpu().numpy(), x.cpu().numpy()
    for _ in range(2):
        y = W.gemv(x).cpu().numpy()
        for b in (0, 7, 15):
            assert relerr(y[b], oracle.gemv_q4_0(bh, xh[b], rows, cols)) <= TOL


def test_activation_scaling_extremes(cuda, oracle):
    # tiny and large activations exercise the per-token power-of-two scaling
    from agent_harness_b200 import kernels as K
    rows, cols = 64, 1024
    blocks, W = _q4_0_weight(K, rows, cols, 5, cuda)
    bh = blocks.cpu().numpy()
    rng = np.random.default_rng(3)
    for scale in (1e-30, 1e-6, 1.0, 3e4, 1e30):
        xh = (rng.standard_normal(cols) * scale).astype(np.float32)
        y = W.gemv(torch.from_numpy(xh).to(cuda)).cpu().numpy()
        ref = oracle.gemv_q4_0(bh, xh, rows, cols)
        assert relerr(y, ref) <= TOL, scale
    xh = np.zeros(cols, np.float32)
    assert np.all(W.gemv(torch.from_numpy(xh).to(cuda)).cpu().numpy() == 0)
    xh[5] = np.nan
    assert np.all(np.isnan(W.gemv(torch.from_numpy(xh).to(cuda)).cpu().numpy()))


def test_engine_format_handle_and_direct(cuda, oracle):
    # the engine's own storage (f32 scales, linear nibbles), incl. a ragged group
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(31)
    for rows, cols in ((128, 4096), (33, 50), (64, 160)):
        Wf = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
        if cols % 32 == 0:
            s, p = oracle.quantize_q4(Wf, 32)
        else:  # per-row groups, as gemv_4bit_into reads them
            n_gpr = (cols + 31) // 32
            s = (rng.random(rows * n_gpr) * 0.01).astype(np.float32)
            p = rng.integers(0, 256, (rows * cols + 1) // 2, dtype=np.uint8)
        x = rng.standard_normal(cols).astype(np.float32)
        ref = oracle.gemv_4bit_into(s, p, x, rows, cols, 32)
        sd, pd, xd = (torch.from_numpy(a).to(cuda) for a in (s, p, x))
        W = K.Q4Weight.from_engine(sd, pd, rows, cols)
        assert relerr(W.gemv(xd).cpu().numpy(), ref) <= TOL, (rows, cols)
        out = torch.empty(rows, dtype=torch.float32, device=cuda)
        K.gemv_4bit_into(out, sd, pd, xd, rows, cols, 32)
        assert relerr(out.cpu().numpy(), ref) <= TOL, (rows, cols)


def test_engine_direct_any_group_size(cuda, oracle):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(32)
    rows, cols, gs = 40, 200, 24
    Wf = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    n_gpr = (cols + gs - 1) // gs
    s = (rng.random(rows * n_gpr) * 0.01).astype(np.float32)
    p = rng.integers(0, 256, (rows * cols + 1) // 2, dtype=np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    ref = oracle.gemv_4bit_into(s, p, x, rows, cols, gs)
    out = torch.empty(rows, dtype=torch.float32, device=cuda)
    K.gemv_4bit_into(out, *(torch.from_numpy(a).to(cuda) for a in (s, p, x)), rows, cols, gs)
    assert relerr(out.cpu().numpy(), ref) <= TOL
    # empty x -> zero output (math.rs:264-267)
    out.fill_(7.0)
    K.gemv_4bit_into(out, torch.from_numpy(s).to(cuda), torch.from_numpy(p).to(cuda),
                     torch.zeros(0, device=cuda), rows, 0, gs)
    assert torch.all(out == 0)
    del Wf


def test_host_dropin_gemv(cuda, oracle):
    from agent_harness_b200 import hostapi
    rng = np.random.default_rng(33)
    rows, cols = 512, 1024
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    s, p = hostapi.quantize(w, 32)
    x = rng.standard_normal(cols).astype(np.float32)
    out = np.empty(rows, np.float32)
    hostapi.gemv_4bit_into(out, s, p, x, rows, cols, 32)
    assert relerr(out, oracle.gemv_4bit_into(s, p, x, rows, cols, 32)) <= TOL
    out2 = np.empty(rows, np.float32)
    hostapi.matvec_4bit_into(out2[:64], s[: 64 * 2], p[: 64 * 32], x[:64], 64, 32)
    z = np.full(rows, 3.0, np.float32)
    hostapi.gemv_4bit_into(z, s, p, np.zeros(0, np.float32), rows, 0, 32)
    assert np.all(z == 0)


def test_golden_gemv(cuda):
    import os
    from agent_harness_b200 import kernels as K
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    x = torch.from_numpy(g["gemv_x"]).to(cuda)
    W = K.Q4Weight.from_q4_0(torch.from_numpy(g["gemv_q4_0_blocks"]).to(cuda), 48, 256)
    assert relerr(W.gemv(x).cpu().numpy(), g["gemv_q4_0_y"]) <= TOL
    W2 = K.Q4Weight.from_engine(torch.from_numpy(g["gemv_eng_scales"]).to(cuda),
                                torch.from_numpy(g["gemv_eng_packed"]).to(cuda), 48, 256)
    assert relerr(W2.gemv(x).cpu().numpy(), g["gemv_eng_y"]) <= TOL


@pytest.mark.parametrize("rows,cols,batch", [(1200, 96, 1), (1504, 4096 + 32, 1), (2048, 4096, 3),
                                             (4096, 14336, 1), (1216, 1024, 2), (12800, 256, 1), (9600, 512, 2)])
def test_many_row_tile_shapes(cuda, oracle, rows, cols, batch):
    # 75 .. 800 row tiles (cluster and rows schedules; rows mode from two tiles
    # per resident CTA), incl. K = 4096+32 columns (65 block pairs) and K = 14336
    from agent_harness_b200 import kernels as K
    blocks, W = _q4_0_weight(K, rows, cols, rows + cols + batch, cuda)
    x = K.fill_normal(batch * cols, 0.0, 1.0, 7 + batch, device=cuda).reshape(batch, cols)
    bh, xh = blocks.cpu().numpy(), x.cpu().numpy()
    for _ in range(2):  # two calls: no state carried between launches
        y = W.gemv(x).cpu().numpy()
        for b in range(batch):
            ref = oracle.gemv_q4_0(bh, xh[b], rows, cols)
            assert relerr(y[b], ref) <= TOL, (rows, cols, b, relerr(y[b], ref))
    from agent_harness_b200._lib import lib
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0


def test_many_row_tiles_engine_format(cuda, oracle):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(41)
    rows, cols = 1536, 512
    Wf = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    s, p = oracle.quantize_q4(Wf, 32)
    x = rng.standard_normal(cols).astype(np.float32)
    W = K.Q4Weight.from_engine(torch.from_numpy(s).to(cuda), torch.from_numpy(p).to(cuda), rows, cols)
    y = W.gemv(torch.from_numpy(x).to(cuda)).cpu().numpy()
    assert relerr(y, oracle.gemv_4bit_into(s, p, x, rows, cols, 32)) <= TOL


def test_batch_split_when_x_exceeds_shared_memory(cuda, oracle):
    # batch 16 x K 28672: the split of x needs more shared memory than one CTA
    # has, so the launch runs over token slices (each token independent)
    from agent_harness_b200 import kernels as K
    rows, cols, batch = 48, 28672, 16
    blocks, W = _q4_0_weight(K, rows, cols, 99, cuda)
    x = K.fill_normal(batch * cols, 0.0, 1.0, 98, device=cuda).reshape(batch, cols)
    y = W.gemv(x).cpu().numpy()
    bh, xh = blocks.cpu().numpy(), x.cpu().numpy()
    for b in (0, 5, 9, 15):
        assert relerr(y[b], oracle.gemv_q4_0(bh, xh[b], rows, cols)) <= TOL, b


@pytest.mark.parametrize("batch", [1, 5, 16])
def test_gemv_host_buffers_match_device_gemv(cuda, batch):
    # ah_q4w_gemv_host (host x in, host y out, synchronous; the gemv_4bit_into
    # calling convention on a resident weight) gives exactly the device GEMV's
    # result, on repeated calls through the same staging.
    from agent_harness_b200 import kernels as K
    rows, cols = 1000, 4096
    W = K.Q4Weight.from_q4_0(K.synth_q4_0(rows, cols, 0.02, 4, device="cuda"), rows, cols)
    for seed in (5, 6):
        x = K.fill_normal(batch * cols, 0.0, 1.0, seed, device="cuda").reshape(batch, cols)
        want = W.gemv(x).cpu()
        got = W.gemv_host(x.cpu().pin_memory())  # pinned: read and written by the kernels over the bus
        assert torch.equal(got, want)
        paged = torch.empty(batch, rows, dtype=torch.float32)
        got = W.gemv_host(x.cpu(), out=paged)  # pageable: through the copy engine
        assert torch.equal(got.reshape(batch, rows), want.reshape(batch, rows))
    W.close()
