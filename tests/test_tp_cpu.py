"""Tensor parallelism on CPU: world-2 gloo ranks run decoder steps with the
sharding the CUDA decoder uses (agent_harness_b200.model.shard_rows: q/k/v,
gate/up and LM-head rows, o/down columns), one all-reduce of the o and down
partials per block, and the argmax-candidate all-gather + first-maximum merge.
The gathered result must match the unsharded step (same NumPy arithmetic), and
the unsharded step must match the oracle decoder (inference/mod.rs:333-545)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CFG = dict(n_layer=2, n_embd=128, n_ff=256, n_head=4, n_head_kv=2, head_dim=32, vocab_size=512,
           rope_base=10000.0, eps=1e-5)
TOKENS = [5, 77, 300, 511]


def _weights(seed=11):
    """Full tensors in the decoder's formats (Q4_0 projections, f16 embeddings
    and norms) from one seeded generator; returns (f32 arrays for the NumPy
    steps, the oracle's weight dict)."""
    from oracle import oracle as O
    c = CFG
    rng = np.random.default_rng(seed)
    d, L = c["n_embd"], c["n_layer"]
    dq, dkv = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    W, OW = {}, {}

    def q4(rows, cols):
        w = (rng.standard_normal(rows * cols) * 0.05).astype(np.float32)
        blocks = O.quantize_q4_0(w)
        return O.dequantize_to_f32(blocks, 2, rows * cols).reshape(rows, cols), blocks

    def f16(n, mean, std):
        bits = (mean + std * rng.standard_normal(n)).astype(np.float16).view(np.uint16)
        return O.f16_to_f32(bits), bits

    W["emb"], OW["tok_embd"] = f16(c["vocab_size"] * d, 0.0, 1.0)
    W["emb"] = W["emb"].reshape(c["vocab_size"], d)
    W["out_norm"], OW["out_norm"] = f16(d, 1.0, 0.02)
    W["lm"], OW["lm_head"] = q4(c["vocab_size"], d)
    an, fn = [], []
    for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
        OW[name] = []
    for l in range(L):
        W[f"an{l}"], b1 = f16(d, 1.0, 0.02)
        W[f"fn{l}"], b2 = f16(d, 1.0, 0.02)
        an.append(b1)
        fn.append(b2)
        for key, name, shape in (("q", "wq", (dq, d)), ("k", "wk", (dkv, d)), ("v", "wv", (dkv, d)),
                                 ("o", "wo", (d, dq)), ("g", "wg", (c["n_ff"], d)), ("u", "wu", (c["n_ff"], d)),
                                 ("d", "wd", (d, c["n_ff"]))):
            W[f"{key}{l}"], blocks = q4(*shape)
            OW[name].append(blocks)
    OW["attn_norm"], OW["ffn_norm"] = np.concatenate(an), np.concatenate(fn)
    return W, OW


def _rms(x, w, eps):
    return (x / np.sqrt(np.mean(x * x, dtype=np.float32) + eps)).astype(np.float32) * w


def _rope(x, pos, base):  # adjacent pairs (2i, 2i+1), theta_i = pos * base^(-i/half)
    hd = x.shape[-1]
    half = hd // 2
    th = pos * base ** (-(np.arange(half, dtype=np.float32)) / half)
    c, s = np.cos(th).astype(np.float32), np.sin(th).astype(np.float32)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def _run(W, rank, world, allreduce, allgather):
    """Greedy steps over TOKENS then 3 generated tokens; returns (local logits
    per step, generated tokens)."""
    from agent_harness_b200.model import (LM_HEAD, WDOWN, WGATE, WK, WO, WQ, WUP, WV, ModelConfig, shard_rows)
    c = CFG
    mc = ModelConfig(c["n_layer"], c["n_embd"], c["n_ff"], c["n_head"], c["n_head_kv"], c["head_dim"],
                     c["vocab_size"])
    sh = shard_rows(mc, rank, world)
    rows = lambda k, t: t[sh[k][0]:sh[k][0] + sh[k][1]]                 # noqa: E731
    cols = lambda k, t: t[:, sh[k][2]:sh[k][2] + sh[k][3]]              # noqa: E731
    hd, nh, nkv = c["head_dim"], c["n_head"] // world, c["n_head_kv"] // world
    G = nh // nkv
    kv = {l: ([], []) for l in range(c["n_layer"])}
    logits_log, gen = [], []
    seq = list(TOKENS)
    for pos in range(len(TOKENS) + 3):
        tok = seq[pos]
        h = W["emb"][tok].copy()
        for l in range(c["n_layer"]):
            x = _rms(h, W[f"an{l}"], c["eps"])
            q = (rows(WQ, W[f"q{l}"]) @ x).reshape(nh, hd)
            k = (rows(WK, W[f"k{l}"]) @ x).reshape(nkv, hd)
            v = (rows(WV, W[f"v{l}"]) @ x).reshape(nkv, hd)
            q, k = _rope(q, pos, c["rope_base"]), _rope(k, pos, c["rope_base"])
            kv[l][0].append(k.astype(np.float16).astype(np.float32))  # f16 KV cache
            kv[l][1].append(v.astype(np.float16).astype(np.float32))
            K, V = np.stack(kv[l][0], 1), np.stack(kv[l][1], 1)  # [nkv][ctx][hd]
            att = np.empty((nh, hd), np.float32)
            for hh in range(nh):
                sc = K[hh // G] @ q[hh] / np.float32(np.sqrt(hd))
                p = np.exp(sc - sc.max())
                att[hh] = (p / p.sum()) @ V[hh // G]
            h = h + allreduce(cols(WO, W[f"o{l}"]) @ att.reshape(-1))
            x = _rms(h, W[f"fn{l}"], c["eps"])
            g, u = rows(WGATE, W[f"g{l}"]) @ x, rows(WUP, W[f"u{l}"]) @ x
            act = (g / (1 + np.exp(-g))) * u
            h = h + allreduce(cols(WDOWN, W[f"d{l}"]) @ act)
        lg = rows(LM_HEAD, W["lm"]) @ _rms(h, W["out_norm"], c["eps"])
        logits_log.append(lg)
        i = int(np.argmax(lg))
        cands = allgather((float(lg[i]), i + sh[LM_HEAD][0]))
        best = min(cands, key=lambda vi: (-vi[0], vi[1]))  # first global maximum
        if pos + 1 >= len(seq):
            seq.append(best[1])
            gen.append(best[1])
    return logits_log, gen


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, _ = _weights()

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        def allgather(pair):
            out = [None] * world
            dist.all_gather_object(out, pair)
            return out

        lg, gen = _run(W, rank, world, allreduce, allgather)
        q.put((rank, [x.tolist() for x in lg], gen))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sharding_plan_covers_every_row():
    from agent_harness_b200.model import LLAMA_70B, shard_rows
    for world in (2, 4, 8):
        parts = [shard_rows(LLAMA_70B, r, world) for r in range(world)]
        for kind in parts[0]:
            r0 = sorted((p[kind][0], p[kind][1], p[kind][2], p[kind][3]) for p in parts)
            if parts[0][kind][2] == 0 and parts[0][kind][3] == LLAMA_70B.n_embd:  # row split
                assert sum(x[1] for x in r0) == parts[0][kind][1] * world
                assert all(r0[i][0] + r0[i][1] == r0[i + 1][0] for i in range(world - 1))
            else:  # column split of o / down: K slices of whole 32-column blocks
                assert all(x[2] % 32 == 0 and x[3] % 32 == 0 for x in r0)
                assert all(r0[i][2] + r0[i][3] == r0[i + 1][2] for i in range(world - 1))


def test_world2_matches_unsharded_and_oracle(oracle):
    W, OW = _weights()
    ident = lambda a: a  # noqa: E731
    lg1, gen1 = _run(W, 0, 1, ident, lambda p: [p])
    # the unsharded NumPy steps against the oracle decoder on the same weights
    c = CFG
    om = oracle.OracleModel({"n_layer": c["n_layer"], "n_embd": c["n_embd"], "n_ff": c["n_ff"],
                             "n_head": c["n_head"], "n_head_kv": c["n_head_kv"], "head_dim": c["head_dim"],
                             "vocab": c["vocab_size"], "rope_base": c["rope_base"], "eps": c["eps"]}, OW, 16)
    seq = list(TOKENS) + gen1
    for pos in range(len(lg1)):
        ref = om.forward(int(seq[pos]), pos)
        assert np.max(np.abs(lg1[pos] - ref)) <= 1e-3 * np.max(np.abs(ref)), pos
        assert int(np.argmax(ref)) == int(np.argmax(lg1[pos]))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, lg, gen = q.get(timeout=240)
        res[r] = (lg, gen)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == res[1][1] == gen1
    for step in range(len(lg1)):
        full = np.concatenate([np.asarray(res[0][0][step]), np.asarray(res[1][0][step])])
        ref = lg1[step]
        assert np.max(np.abs(full - ref)) <= 1e-4 * np.max(np.abs(ref)), step


def _topk_sorted(values, idx, k):
    """The k largest by (value desc, index asc), as (value, index) pairs."""
    order = sorted(range(len(values)), key=lambda i: (-values[i], idx[i]))[:k]
    return [(values[i], idx[i]) for i in order]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sampling_candidate_merge_equals_global(oracle, world):
    # the tensor-parallel sampler's plan: each rank's top-k of its vocab slice
    # (global indices), the W*k candidates merged by (value desc, index asc),
    # then sample() over the merged top-k -- the same pick as sample() over
    # the full row, for every draw, including tied logits across ranks
    rng = np.random.default_rng(world)
    vocab, k, temp = 512, 40, 0.8
    for trial in range(6):
        row = (rng.standard_normal(vocab) * 2).astype(np.float32)
        if trial % 2:
            row = np.round(row * 2).astype(np.float32) / 2  # ties within and across slices
        per = vocab // world
        cands = []
        for r in range(world):
            sl = row[r * per:(r + 1) * per]
            cands += _topk_sorted(list(sl), list(range(r * per, (r + 1) * per)), k)
        merged = _topk_sorted([c[0] for c in cands], [c[1] for c in cands], k)
        glob = _topk_sorted(list(row), list(range(vocab)), k)
        assert [c[1] for c in merged] == [c[1] for c in glob]
        sub = np.array([c[0] for c in merged], np.float32)
        for r in rng.random(20).astype(np.float32):
            pick = merged[oracle.sample(sub, temp, k, float(r))][1]
            assert pick == oracle.sample(row, temp, k, float(r))
