"""GPU parity of the fused Q4 GEMV (batches of 1..4 tokens) on shapes that
stress its schedules: the benchmark shape, the 8B decoder's projections, an
odd block-pair count, ragged rows, fewer row tiles than SMs, a single padded
tile.  Against the oracle's scalar gemv (inference/math.rs:382-418) at the
1e-3 normwise tolerance, and repeated calls on the same input must give
bit-identical results (no state carried between launches)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def relerr(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.mark.parametrize("rows,cols,batch", [
    (4096, 4096, 1),        # the benchmark shape
    (4096, 4096, 4),
    (6144, 4096, 1),        # fused QKV of the 8B shape
    (4096, 14336, 1),       # down projection: 224 block pairs per tile
    (4096 + 16, 4096 + 32, 2),  # 65 block pairs (odd), one extra tile
    (1000, 2048, 3),        # ragged rows, 63 tiles: fewer tiles than SMs
    (2368, 1024, 1),        # 148 tiles exactly
    (2384, 1024, 1),        # 149 tiles
    (7, 64, 1),             # a single padded tile
    (3000, 96, 4),          # 2 block pairs per tile, 188 tiles
])
def test_shapes_match_oracle(cuda, oracle, rows, cols, batch):
    from agent_harness_b200 import kernels as K
    blocks = K.synth_q4_0(rows, cols, 0.02, rows * 3 + cols + batch, device=cuda)
    W = K.Q4Weight.from_q4_0(blocks, rows, cols)
    bh = blocks.cpu().numpy()
    outs = []
    for seed in (11, 12):
        x = K.fill_normal(batch * cols, 0.0, 1.0, seed, device=cuda).reshape(batch, cols)
        y = W.gemv(x).cpu().numpy().reshape(batch, rows)
        xh = x.cpu().numpy()
        for b in range(batch):
            ref = oracle.gemv_q4_0(bh, xh[b], rows, cols)
            err = relerr(y[b], ref)
            assert err <= TOL, (rows, cols, batch, b, err)
            assert err < 1e-5, err  # f32-grade split-f16 products
        outs.append((x, y))
    # the same input again: bit-identical
    x, y = outs[0]
    y2 = W.gemv(x).cpu().numpy().reshape(batch, rows)
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))
    from agent_harness_b200._lib import lib
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0
    W.close()


def test_engine_format_ragged_tiles(cuda, oracle):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(71)
    rows, cols = 2384, 2048
    Wf = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    s, p = oracle.quantize_q4(Wf, 32)
    W = K.Q4Weight.from_engine(torch.from_numpy(s).to(cuda), torch.from_numpy(p).to(cuda), rows, cols)
    for batch in (1, 4):
        x = rng.standard_normal((batch, cols)).astype(np.float32)
        y = W.gemv(torch.from_numpy(x).to(cuda)).cpu().numpy().reshape(batch, rows)
        for b in range(batch):
            assert relerr(y[b], oracle.gemv_4bit_into(s, p, x[b], rows, cols, 32)) <= TOL
    W.close()


def test_back_to_back_weights_share_nothing(cuda, oracle):
    # launches on different weights queued back to back (each prefetches its
    # weights under the previous one's tail) and on the same weight twice in a row
    from agent_harness_b200 import kernels as K
    shapes = [(4096, 4096), (2384, 1024), (4096, 4096), (1000, 2048)]
    ws, bs = [], []
    for i, (r, c) in enumerate(shapes):
        b = K.synth_q4_0(r, c, 0.02, 500 + i, device=cuda)
        bs.append(b.cpu().numpy())
        ws.append(K.Q4Weight.from_q4_0(b, r, c))
    xs = [K.fill_normal(c, 0.0, 1.0, 600 + i, device=cuda) for i, (r, c) in enumerate(shapes)]
    ys = [torch.empty(r, device=cuda) for r, _ in shapes]
    for _ in range(3):
        for W, x, y in zip(ws, xs, ys):
            W.gemv(x, out=y)
        ws[0].gemv(xs[0], out=ys[0])
    torch.cuda.synchronize()
    for (r, c), b, x, y in zip(shapes, bs, xs, ys):
        assert relerr(y.cpu().numpy(), oracle.gemv_q4_0(b, x.cpu().numpy(), r, c)) <= TOL
    for W in ws:
        W.close()
