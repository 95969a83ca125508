"""The gated delta-net SSM block oracle (inference/ssm.rs:171-296) on CPU.  The
reference has no tests of the block, so the C restatement is pinned against
an independent numpy float32 restatement of the same steps (summation order
aside: numpy's pairwise sums, hence a 1e-5 tolerance), over several tokens so
that the conv window and the delta-rule state carry across steps."""
import numpy as np
import pytest

from oracle import oracle as O

F = np.float32
SMALL = dict(n_embd=64, d_state=16, n_group=2, dt_rank=4, d_inner=64, d_conv=4, eps=1e-6)


def ssm_weights(cfg, seed):
    rng = np.random.default_rng(seed)
    hk, nk, nv = cfg["d_state"], cfg["n_group"], cfg["dt_rank"]
    hv = cfg["d_inner"] // nv
    key_dim, value_dim = hk * nk, hv * nv
    conv_dim = 2 * key_dim + value_dim
    d = cfg["n_embd"]

    def r(*shape, s=0.1):
        return (rng.standard_normal(shape) * s).astype(np.float32)

    return {"wqkv": r(conv_dim, d), "wqkv_gate": r(value_dim, d), "conv1d": r(conv_dim, cfg["d_conv"], s=0.5),
            "dt_bias": r(nv, s=0.5), "a": -np.abs(r(nv, s=1.0)), "alpha": r(nv, d), "beta": r(nv, d),
            "norm": (1.0 + r(hv, s=0.05)).astype(np.float32), "out": r(d, value_dim)}


def sigmoid(x):
    x = F(x)
    return F(1.0) / (F(1.0) + np.exp(-x)) if x >= 0 else np.exp(x) / (F(1.0) + np.exp(x))


def numpy_ssm(cfg, w, conv_state, S, x):
    hk, nk, nv = cfg["d_state"], cfg["n_group"], cfg["dt_rank"]
    hv = cfg["d_inner"] // nv
    key_dim = hk * nk
    eps = F(cfg["eps"])
    qkv = w["wqkv"] @ x
    z = w["wqkv_gate"] @ x
    beta = np.array([sigmoid(v) for v in w["beta"] @ x], np.float32)
    ar = w["alpha"] @ x + w["dt_bias"]
    gate = np.where(ar > 20, ar, np.log(F(1) + np.exp(ar))).astype(np.float32) * w["a"]
    dc = cfg["d_conv"]
    craw = (conv_state * w["conv1d"][:, :dc - 1].T).sum(0) + qkv * w["conv1d"][:, dc - 1]
    conv_state[:-1] = conv_state[1:].copy()
    conv_state[-1] = qkv
    cout = np.array([v * sigmoid(v) for v in craw], np.float32)
    q, k, v = cout[:key_dim].copy(), cout[key_dim:2 * key_dim].copy(), cout[2 * key_dim:]
    for h in range(nk):
        for t in (q, k):
            seg = t[h * hk:(h + 1) * hk]
            seg *= F(1) / max(np.sqrt((seg * seg).sum(dtype=np.float32)), eps)
    rep = nv // nk
    out_h = np.empty((nv, hv), np.float32)
    scale = F(1) / np.sqrt(F(hk))
    for h in range(nv):
        qh, kh, vh = q[(h // rep) * hk:][:hk] * scale, k[(h // rep) * hk:][:hk], v[h * hv:(h + 1) * hv]
        S[h] *= np.exp(gate[h])
        delta = (vh - S[h] @ kh) * beta[h]
        S[h] += np.outer(delta, kh)
        out_h[h] = S[h] @ qh
    res = np.empty(nv * hv, np.float32)
    for h in range(nv):
        oh = out_h[h]
        inv = F(1) / np.sqrt((oh * oh).sum(dtype=np.float32) / F(hv) + eps)
        zh = z[h * hv:(h + 1) * hv]
        res[h * hv:(h + 1) * hv] = oh * inv * w["norm"] * np.array([t * sigmoid(t) for t in zh], np.float32)
    return w["out"] @ res


def test_ssm_oracle_matches_numpy_over_steps(oracle):
    cfg = SMALL
    w = ssm_weights(cfg, 1)
    hk, nv = cfg["d_state"], cfg["dt_rank"]
    hv = cfg["d_inner"] // nv
    conv_dim = 2 * hk * cfg["n_group"] + hv * nv
    cs_o = np.zeros((cfg["d_conv"] - 1, conv_dim), np.float32)
    ss_o = np.zeros((nv, hv, hk), np.float32)
    cs_n, ss_n = cs_o.copy(), ss_o.copy()
    rng = np.random.default_rng(2)
    for step in range(6):
        x = rng.standard_normal(cfg["n_embd"]).astype(np.float32)
        got = O.ssm_forward(cfg, w, cs_o, ss_o, x)
        want = numpy_ssm(cfg, w, cs_n, ss_n, x)
        assert np.max(np.abs(got - want)) <= 1e-5 * max(1.0, np.max(np.abs(want))), step
        assert np.allclose(cs_o, cs_n, atol=1e-6) and np.allclose(ss_o, ss_n, atol=1e-5), step
    assert np.max(np.abs(ss_o)) > 0  # the state evolved


def test_ssm_oracle_rejects_mismatched_head_dims(oracle):
    cfg = dict(SMALL, d_inner=128)  # head_v_dim 32 != head_k_dim 16: the reference asserts
    w = ssm_weights(dict(SMALL), 1)
    with pytest.raises(ValueError):
        O.ssm_forward(cfg, w, np.zeros((3, 192), np.float32), np.zeros(4 * 32 * 16, np.float32),
                      np.zeros(64, np.float32))


def _pad4(n):
    return (n + 3) // 4 * 4


@pytest.mark.parametrize("cfg", [SMALL, dict(n_embd=2048, d_state=128, n_group=16, dt_rank=32, d_inner=4096,
                                             d_conv=4, eps=1e-6)], ids=["small", "n2048"])
def test_ssm_workspace_bytes_on_host(cfg):
    # host arithmetic of the C-ABI, no device needed: the step's intermediates
    # (conv output, z, the normed result, o) and beta, gate and the per-head
    # completion counters
    import ctypes as C
    from agent_harness_b200 import _lib
    from agent_harness_b200.ssm import _Cfg
    c = _Cfg(cfg["n_embd"], cfg["d_state"], cfg["n_group"], cfg["dt_rank"], cfg["d_inner"], cfg["d_conv"],
             cfg["eps"])
    n = C.c_size_t()
    _lib.call("ah_ssm_workspace_bytes", C.byref(c), C.byref(n))
    conv_dim = 2 * cfg["n_group"] * cfg["d_state"] + cfg["d_inner"]
    want = 4 * (_pad4(conv_dim) + 3 * _pad4(cfg["d_inner"]) + 3 * _pad4(cfg["dt_rank"]))
    assert n.value == want


@pytest.mark.parametrize("bad", [dict(d_inner=128),            # head_v_dim 32 != head_k_dim 16 (ssm.rs:239)
                                 dict(dt_rank=3, d_inner=48),   # v heads not a multiple of k heads
                                 dict(d_state=512, d_inner=2048),  # head dim above 256
                                 dict(n_embd=0)], ids=["head_dims", "head_groups", "head_dim_max", "zero_dim"])
def test_ssm_config_rejected_on_host(bad):
    import ctypes as C
    from agent_harness_b200 import _lib
    from agent_harness_b200.ssm import _Cfg
    cfg = dict(SMALL, **bad)
    c = _Cfg(cfg["n_embd"], cfg["d_state"], cfg["n_group"], cfg["dt_rank"], cfg["d_inner"], cfg["d_conv"],
             cfg["eps"])
    with pytest.raises(_lib.AhError):
        _lib.call("ah_ssm_workspace_bytes", C.byref(c), C.byref(C.c_size_t()))
