"""GPU parity: temperature + top-k sampling (inference/sampling.rs:17-64) on
the device against the oracle's sample() given the same uniform draw
r = sample_uniform(seed, step, sequence).  The pick is an index, so it must
match exactly; the one allowance is a draw within 1e-5 of a CDF boundary
(computed in float64), where CUDA's expf and the host's may round the
probabilities differently by an ulp."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MARGIN = 1e-5


def _margin(row, temp, k, r):
    x = np.asarray(row, np.float64)
    x = x[np.isfinite(x)] if np.isfinite(x).any() else x
    p = np.sort(np.exp((x - x.max()) / temp))[::-1][:k]
    cdf = np.cumsum(p) / p.sum()
    return float(np.min(np.abs(cdf - r)))


def _check(oracle, logits, temp, k, seed, step, got):
    bad = []
    for b in range(logits.shape[0]):
        r = oracle.sample_uniform(seed, step, b)
        want = oracle.sample(logits[b], temp, k, r)
        if int(got[b]) != want and _margin(logits[b], temp, k, r) >= MARGIN:
            bad.append((b, int(got[b]), want, r))
    assert not bad, bad[:5]


@pytest.mark.parametrize("batch,vocab,temp,k", [(16, 128256, 0.7, 40), (3, 32000, 1.0, 64), (1, 1000, 1.5, 1),
                                                (4, 10, 1.0, 40), (8, 151936, 0.9, 40), (2, 4097, 0.3, 17)])
def test_matches_oracle(cuda, oracle, batch, vocab, temp, k):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(batch * 7 + vocab)
    logits = (rng.standard_normal((batch, vocab)) * 2.5).astype(np.float32)
    d = torch.from_numpy(logits).to(cuda)
    for step in (0, 1, 977):
        got = K.sample_logits(d, temp, k, seed=5, step=step)
        _check(oracle, logits, temp, k, 5, step, got.cpu().numpy())
        # rows split over slice CTAs and rows walked by one CTA pick the same
        assert torch.equal(K.sample_logits(d, temp, k, seed=5, step=step, split=False), got)


def test_ties_and_masks(cuda, oracle):
    # rows whose k-th largest logit is shared by more entries than the slots
    # left (the ordered tie scan), by exactly as many (the unordered slots), a
    # constant row, and rows with -inf masks
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(3)
    V = 50000
    rows = [np.round(rng.standard_normal(V) * 2) / 2,  # ~20 levels: large ties
            np.where(np.arange(V) % 2 == 1, -0.0, 0.0),  # -0 and +0 tie
            np.full(V, -np.inf),
            rng.standard_normal(V)]
    exact = rng.standard_normal(V) - 10.0  # 38 distinct tops, then two copies of the 39th value
    exact[:38] = np.arange(38) + 1.0
    exact[1000] = exact[2000] = 0.5
    rows.append(exact)
    rows[2][[5, 17, 40000]] = [0.0, 1.0, 1.0]
    rows[3][rng.integers(0, V, 30000)] = -np.inf
    logits = np.stack(rows).astype(np.float32)
    d = torch.from_numpy(logits).to(cuda)
    for k in (1, 39, 40, 64):
        for step in range(4):
            got = K.sample_logits(d, 1.0, k, seed=17, step=step)
            _check(oracle, logits, 1.0, k, 17, step, got.cpu().numpy())
            assert torch.equal(K.sample_logits(d, 1.0, k, seed=17, step=step, split=False), got)
    # the constant row at top-k 40: one of the first 40 indices
    got = np.array([K.sample_logits(d[1:2], 1.0, 40, seed=s).item() for s in range(32)])
    assert got.min() >= 0 and got.max() < 40 and len(set(got.tolist())) > 10


def test_strided_rows_and_determinism(cuda, oracle):
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(8)
    big = torch.from_numpy((rng.standard_normal((6, 3000 + 40)) * 3).astype(np.float32)).to(cuda)
    view = big[:, :3000]
    a = K.sample_logits(view, 0.8, 40, seed=2, step=9)
    b = K.sample_logits(view, 0.8, 40, seed=2, step=9)
    assert torch.equal(a, b)
    _check(oracle, view.cpu().numpy(), 0.8, 40, 2, 9, a.cpu().numpy())
    c = torch.stack([K.sample_logits(view, 0.8, 40, seed=2, step=s) for s in range(10, 40)])
    assert len(torch.unique(c[:, 0])) > 1  # the draw moves with the step


def test_frequencies_follow_top_k_softmax(cuda):
    # 8192 sequences of one row: the picks follow the renormalised top-k softmax
    from agent_harness_b200 import kernels as K
    rng = np.random.default_rng(6)
    row = (rng.standard_normal(5000) * 1.2).astype(np.float32)
    n, k, temp = 8192, 6, 1.1
    d = torch.from_numpy(np.tile(row, (n, 1))).to(cuda)
    picks = K.sample_logits(d, temp, k, seed=3, step=1).cpu().numpy()
    top = np.argsort(-row, kind="stable")[:k]
    p = np.exp((row[top] - row.max()) / temp)
    p /= p.sum()
    assert set(np.unique(picks).tolist()) <= set(top.tolist())
    for i, pi in zip(top, p):
        f = float(np.mean(picks == i))
        assert abs(f - pi) <= 5 * np.sqrt(pi * (1 - pi) / n) + 1e-3, (i, f, pi)


def test_bad_arguments_refused(cuda):
    from agent_harness_b200 import kernels as K
    from agent_harness_b200._lib import AhError
    d = torch.zeros(2, 100, device=cuda)
    for temp, k in ((0.0, 40), (-1.0, 40), (1.0, 0), (1.0, 65)):
        with pytest.raises(AhError):
            K.sample_logits(d, temp, k)
    # a split row with a short workspace
    big = torch.zeros(2, 20000, device=cuda)
    need = K.sample_workspace_bytes(2, 20000)
    assert need > 0 and K.sample_workspace_bytes(2, 8191) == 0
    with pytest.raises(AhError):
        K.sample_logits(big, 1.0, 64, workspace=torch.empty(need - 16, dtype=torch.uint8, device=cuda))


def test_decoder_samples_its_own_logits(cuda, oracle):
    # every token the decode step samples is sample() of that step's logits
    # with the draw for (seed, position, sequence); generate repeats them
    from agent_harness_b200.model import Model, ModelConfig
    cfg = ModelConfig(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=64, vocab_size=1000,
                      max_seq=64, max_batch=2, rope_freq_base=10000.0, rms_eps=1e-5)
    m = Model(cfg)
    m.init_random(123, w_std=0.05)
    prompt = np.array([[3, 14, 159, 265, 358, 979], [2, 71, 828, 182, 845, 904]], np.int32)
    greedy = m.generate(prompt, 12)
    temp, k, seed = 0.9, 40, 21
    m.set_sampling(temp, k, seed)
    m.reset(2)
    for t in range(prompt.shape[1]):
        lg = m.forward(prompt[:, t]).cpu().numpy()
    chain = []
    for i in range(12):
        pos = m.position - 1
        tok = m.decode(1, 2).cpu().numpy()[0]
        _check(oracle, lg, temp, k, seed, pos, tok)
        chain.append(tok)
        lg = m.forward(tok).cpu().numpy()
    chain = np.stack(chain)
    gen = m.generate(prompt, 12)
    assert np.array_equal(gen, chain)
    assert np.array_equal(m.generate(prompt, 12), gen)
    m.set_sampling(temp, k, seed + 1)
    assert not np.array_equal(m.generate(prompt, 12), gen)
    m.set_sampling(0.0)
    assert np.array_equal(m.generate(prompt, 12), greedy)
    m.close()


def test_no_device_timeouts_recorded(cuda):
    from agent_harness_b200._lib import lib
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0
