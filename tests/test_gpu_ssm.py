"""GPU parity of the gated delta-net SSM block (inference/ssm.rs:171-296)
against the oracle restatement, over several tokens so that the conv window
and the per-head state carry across steps: outputs and states within 1e-4 of
their largest entry, the conv window within 1e-5 (f32 sums in a different
order)."""
import numpy as np
import pytest
import torch

from test_ssm_cpu import SMALL, ssm_weights

pytestmark = pytest.mark.gpu

QWEN_LIKE = dict(n_embd=1024, d_state=128, n_group=4, dt_rank=8, d_inner=1024, d_conv=4, eps=1e-6)
# a short, wide output projection (256 x 4096): several warps share each row
WIDE_OUT = dict(n_embd=256, d_state=128, n_group=2, dt_rank=32, d_inner=4096, d_conv=4, eps=1e-6)


@pytest.mark.parametrize("cfg", [SMALL, QWEN_LIKE, dict(SMALL, d_state=32, d_inner=128, d_conv=1), WIDE_OUT],
                         ids=["small", "head128", "no_conv_window", "wide_out_split_rows"])
def test_ssm_forward_matches_oracle(cuda, oracle, cfg):
    from agent_harness_b200.ssm import SsmBlock
    w = ssm_weights(cfg, 3)
    blk = SsmBlock(cfg, w)
    st = blk.new_state()
    nv, D = cfg["dt_rank"], cfg["d_state"]
    conv_dim = 2 * cfg["n_group"] * D + cfg["d_inner"]
    cs = np.zeros((max(cfg["d_conv"] - 1, 1), conv_dim), np.float32)
    ss = np.zeros((nv, D, D), np.float32)
    rng = np.random.default_rng(4)
    for step in range(5):
        x = rng.standard_normal(cfg["n_embd"]).astype(np.float32)
        got = blk.forward(torch.as_tensor(x), st).cpu().numpy()
        want = oracle.ssm_forward(cfg, w, cs, ss, x)
        assert np.max(np.abs(got - want)) <= 1e-4 * np.max(np.abs(want)), step
        gs = st.ssm_state.cpu().numpy()
        assert np.max(np.abs(gs - ss)) <= 1e-4 * max(np.max(np.abs(ss)), 1e-6), step
        if cfg["d_conv"] > 1:  # the window holds the raw projections (summed in another order)
            gc = st.conv_state.cpu().numpy()
            assert np.max(np.abs(gc - cs)) <= 1e-5 * max(np.max(np.abs(cs)), 1e-6), step
