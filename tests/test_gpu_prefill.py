"""GPU parity of the prompt prefill through the tcgen05 GEMMs (the decoder's
ah_model_set_prefill mode 1): the reference prefills one forward() per token
(inference/mod.rs:550); the GEMM prefill must leave the same state.  Checked
by the logits of the last prompt token (fed through the decode step after the
prefill) against the oracle at 1e-3 normwise, and greedy tokens identical to
the token-by-token path, including prompts split over several chunks."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3


def relerr(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _last_token_logits(m, prompt, mode):
    """Prefill prompt[:, :-1] in `mode`, then the last prompt token through the
    decode step; returns its logits [batch][vocab]."""
    m.set_prefill(mode)
    m.generate(prompt, 0)
    return m.forward(prompt[:, -1]).cpu().numpy()


def _oracle_last_logits(oracle, cfg, W, seq):
    from test_gpu_decoder import oracle_model
    o = oracle_model(oracle, cfg, W)
    for t, tok in enumerate(seq):
        lg = o.forward(int(tok), t)
    return lg


@pytest.mark.parametrize("batch,n_prompt", [(1, 12), (2, 40)])
def test_small_prefill_matches_oracle_and_token_path(cuda, oracle, batch, n_prompt):
    from test_gpu_decoder import SMALL, oracle_weights
    from agent_harness_b200.model import Model, ModelConfig
    cfg = ModelConfig(**SMALL)
    m = Model(cfg)
    m.init_random(123)
    W = oracle_weights(cfg, 123, cuda)
    prompt = np.random.default_rng(n_prompt).integers(0, cfg.vocab_size, (batch, n_prompt)).astype(np.int32)
    lg_gemm = _last_token_logits(m, prompt, 1)
    lg_tok = _last_token_logits(m, prompt, 0)
    for b in range(batch):
        ref = _oracle_last_logits(oracle, cfg, W, prompt[b])
        assert relerr(lg_gemm[b], ref) <= TOL, relerr(lg_gemm[b], ref)
        assert relerr(lg_gemm[b], lg_tok[b]) <= TOL
        assert int(np.argmax(lg_gemm[b])) == oracle.argmax(ref)
    m.set_prefill(1)
    a = m.generate(prompt, 10)
    m.set_prefill(0)
    t = m.generate(prompt, 10)
    assert np.array_equal(a, t)
    m.close()


def test_8b_width_prefill(cuda, oracle):
    from test_gpu_decoder import oracle_weights
    from agent_harness_b200.model import Model, ModelConfig
    cfg = ModelConfig(n_layer=2, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128,
                      vocab_size=128256, max_seq=160, max_batch=1, rope_freq_base=500000.0, rms_eps=1e-5)
    m = Model(cfg)
    m.init_random(6)
    W = oracle_weights(cfg, 6, cuda)
    prompt = np.random.default_rng(7).integers(0, cfg.vocab_size, (1, 130)).astype(np.int32)
    lg = _last_token_logits(m, prompt, 1)[0]
    ref = _oracle_last_logits(oracle, cfg, W, prompt[0])
    assert relerr(lg, ref) <= TOL, relerr(lg, ref)
    assert int(np.argmax(lg)) == oracle.argmax(ref)
    m.close()


def test_prefill_over_several_chunks(cuda):
    # batch 16: 128 positions per chunk, so a 300-token prompt takes three chunks
    # (the later chunks attend over cache rows the earlier ones wrote)
    from agent_harness_b200.model import Model, ModelConfig
    cfg = ModelConfig(n_layer=3, n_embd=256, n_ff=512, n_head=8, n_head_kv=2, head_dim=32, vocab_size=512,
                      max_seq=320, max_batch=16, rope_freq_base=10000.0, rms_eps=1e-5)
    m = Model(cfg)
    m.init_random(77)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, (16, 300)).astype(np.int32)
    lg_gemm = _last_token_logits(m, prompt, 1)
    lg_tok = _last_token_logits(m, prompt, 0)
    for b in range(16):
        assert relerr(lg_gemm[b], lg_tok[b]) <= TOL, (b, relerr(lg_gemm[b], lg_tok[b]))
    m.set_prefill(1)
    a = m.generate(prompt, 6)
    m.set_prefill(0)
    t = m.generate(prompt, 6)
    assert np.array_equal(a, t)
    m.close()
