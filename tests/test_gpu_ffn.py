"""GPU parity of the SwiGLU feed-forward block (inference/ffn.rs:155-174) and
the row-range scalar worker (inference/math.rs:382-418) through the C-ABI,
against the oracle's C restatements of the same functions.  Tolerance
(the f32-accumulate parity bar): normwise max|y - ref| / max|ref| <= 1e-3."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def relerr(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _ffn_weights(oracle, n_embd, n_ff, seed, gs=32):
    rng = np.random.default_rng(seed)
    out = []
    for rows, cols in ((n_ff, n_embd), (n_ff, n_embd), (n_embd, n_ff)):
        w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
        if cols % gs == 0:
            s, p = oracle.quantize_q4(w, gs)
        else:  # per-row groups as the GEMV reads them: scales [rows][ceil(cols/gs)]
            s = (rng.random(rows * ((cols + gs - 1) // gs)) * 0.004).astype(np.float32)
            p = rng.integers(0, 256, (rows * cols + 1) // 2, dtype=np.uint8)
        out += [s, p]
    x = rng.standard_normal(n_embd).astype(np.float32)
    return out, x


@pytest.mark.parametrize("n_embd,n_ff,gs", [(512, 1408, 32), (4096, 14336, 32), (100, 37, 24)])
def test_host_swiglu_matches_oracle(oracle, cuda, n_embd, n_ff, gs):
    from agent_harness_b200 import hostapi
    w, x = _ffn_weights(oracle, n_embd, n_ff, n_embd + n_ff, gs)
    ref_out, ref_g, ref_u, ref_a = oracle.swiglu_4bit_into(x, *w, n_embd, n_ff, gs)
    out = np.full(n_embd, np.nan, np.float32)
    sg, su, sa = (np.full(n_ff, np.nan, np.float32) for _ in range(3))
    hostapi.swiglu_4bit_into(out, x, *w, n_embd, n_ff, gs, sg, su, sa)
    for got, ref in ((sg, ref_g), (su, ref_u), (sa, ref_a), (out, ref_out)):
        assert relerr(got, ref) <= TOL, relerr(got, ref)


def test_swiglu_empty_shapes(cuda):
    from agent_harness_b200 import hostapi
    z = np.zeros(0, np.float32)
    out = np.full(4, 7.0, np.float32)
    sg, su, sa = (np.zeros(0, np.float32) for _ in range(3))
    # n_ff = 0: down . (empty act) zeroes out (math.rs:264-267)
    hostapi.swiglu_4bit_into(out, np.ones(4, np.float32), z, np.zeros(0, np.uint8), z, np.zeros(0, np.uint8),
                             np.zeros(4, np.float32), np.zeros(0, np.uint8), 4, 0, 32, sg, su, sa)
    assert np.all(out == 0)


def test_device_swiglu_and_tiled_block(oracle, cuda):
    from agent_harness_b200 import kernels as K
    n_embd, n_ff = 1024, 2816
    w, x = _ffn_weights(oracle, n_embd, n_ff, 91)
    ref_out, _, _, ref_a = oracle.swiglu_4bit_into(x, *w, n_embd, n_ff, 32)
    wd = [torch.from_numpy(a).to(cuda) for a in w]
    xd = torch.from_numpy(x).to(cuda)
    out = torch.empty(n_embd, device=cuda)
    sg, su, sa = (torch.empty(n_ff, device=cuda) for _ in range(3))
    K.swiglu_4bit_into(out, xd, *wd, n_embd, n_ff, 32, sg, su, sa)
    assert relerr(out.cpu().numpy(), ref_out) <= TOL
    assert relerr(sa.cpu().numpy(), ref_a) <= TOL
    # the decoder's form: interleaved gate/up GEMV with the SwiGLU epilogue + down GEMV
    blk = K.SwigluBlock.from_engine(*wd, n_embd, n_ff)
    rng = np.random.default_rng(5)
    for batch in (1, 3):
        xs = rng.standard_normal((batch, n_embd)).astype(np.float32)
        act = torch.empty(batch, n_ff, device=cuda)
        y = blk(torch.from_numpy(xs).to(cuda), act).cpu().numpy()
        for b in range(batch):
            r_out, _, _, r_act = oracle.swiglu_4bit_into(xs[b], *w, n_embd, n_ff, 32)
            assert relerr(act[b].cpu().numpy(), r_act) <= TOL
            assert relerr(y[b], r_out) <= TOL
    blk.close()


def test_tiled_block_from_q4_0(oracle, cuda):
    from agent_harness_b200 import kernels as K
    n_embd, n_ff = 512, 1024
    g = K.synth_q4_0(n_ff, n_embd, 0.02, 1, device=cuda)
    u = K.synth_q4_0(n_ff, n_embd, 0.02, 2, device=cuda)
    d = K.synth_q4_0(n_embd, n_ff, 0.02, 3, device=cuda)
    x = K.fill_normal(n_embd, 0.0, 1.0, 4, device=cuda)
    blk = K.SwigluBlock.from_q4_0(g, u, d, n_embd, n_ff)
    y = blk(x).cpu().numpy()
    xh = x.cpu().numpy()
    gg = oracle.gemv_q4_0(g.cpu().numpy(), xh, n_ff, n_embd)
    uu = oracle.gemv_q4_0(u.cpu().numpy(), xh, n_ff, n_embd)
    act = np.array([oracle.silu(float(a)) for a in gg], np.float32) * uu
    ref = oracle.gemv_q4_0(d.cpu().numpy(), act, n_embd, n_ff)
    assert relerr(y, ref) <= TOL
    blk.close()


@pytest.mark.parametrize("rows,cols,gs,ranges", [(300, 4096, 32, [(0, 300), (7, 123), (299, 300), (5, 5)]),
                                                 (41, 33, 32, [(1, 40), (3, 4)]),  # odd row starts: nibble phase
                                                 (64, 200, 24, [(10, 64)])])
def test_worker_scalar_row_ranges(oracle, cuda, rows, cols, gs, ranges):
    from agent_harness_b200 import hostapi
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(rows + cols)
    s = (rng.random(rows * ((cols + gs - 1) // gs)) * 0.004).astype(np.float32)
    p = rng.integers(0, 256, (rows * cols + 1) // 2, dtype=np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    for r0, r1 in ranges:
        ref = oracle.gemv_4bit_worker_scalar(s, p, x, r0, r1, cols, gs)
        out = np.full(r1 - r0, np.nan, np.float32)
        hostapi.gemv_4bit_parallel_worker_scalar(out, s, p, x, r0, r1, cols, gs)
        if r1 > r0:
            assert relerr(out, ref) <= TOL, (r0, r1)
        dev = torch.full((max(r1 - r0, 1),), float("nan"), device=cuda)
        K.gemv_4bit_rows(dev, torch.from_numpy(s).to(cuda), torch.from_numpy(p).to(cuda), torch.from_numpy(x).to(cuda),
                         r0, r1, cols, gs)
        if r1 > r0:
            assert relerr(dev[: r1 - r0].cpu().numpy(), ref) <= TOL
