"""GPU tensor parallelism: a 2-rank decoder (one process per GPU, NCCL
all-reduce per block, argmax-candidate all-gather) against the same model on
one GPU.  The ranks' vocab slices of the logits, concatenated, match the
single-GPU logits (1e-3 normwise, as the decoder parity bar) and greedy tokens
are identical on every rank and equal to the single-GPU ones.  Skipped on
boxes with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=64, vocab_size=1000, max_seq=64,
             max_batch=2, rope_freq_base=10000.0, rms_eps=1e-5)
PROMPT = np.array([[3, 14, 159, 265, 358, 979], [2, 71, 828, 182, 845, 904]], np.int32)
# long enough for the prefill GEMMs (with an all-reduce of the block outputs)
LONG = (np.arange(2 * 40, dtype=np.int32).reshape(2, 40) * 37 + 11) % 1000


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q, p2p=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from agent_harness_b200 import _lib
        from agent_harness_b200.model import Model, ModelConfig, nccl_unique_id
        _lib.check(_lib.lib().ah_device_init(rank))
        ids = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        m = Model(ModelConfig(**SMALL), device=f"cuda:{rank}", tp_rank=rank, tp_world=world, nccl_id=ids[0])
        m.init_random(123)
        if p2p:
            def allgather(blob):
                out = [None] * world
                dist.all_gather_object(out, blob)
                return out
            m.enable_peer_allreduce(allgather)
        m.reset(2)
        logits = [m.forward(PROMPT[:, t]).cpu().numpy() for t in range(PROMPT.shape[1])]
        gen = m.generate(PROMPT, 8)
        gen_long = m.generate(LONG, 6)
        m.generate(LONG, 0)
        last = m.forward(LONG[:, -1]).cpu().numpy()
        # temperature + top-k: per-rank candidates, all-gathered and merged
        m.set_sampling(0.8, 40, 99)
        m.reset(2)
        s_last = [m.forward(PROMPT[:, t]).cpu().numpy() for t in range(PROMPT.shape[1])][-1]
        s_tok = m.decode(1, 2).cpu().numpy()[0]
        s_gen = m.generate(PROMPT, 8)
        torch.cuda.synchronize()
        err = _lib.lib().ah_check_device_error(None)
        m.close()
        q.put((rank, logits, (gen, gen_long, last, s_last, s_tok, s_gen), err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("p2p", [False, True], ids=["nccl", "nvlink_peer"])
def test_tp2_matches_single_gpu(cuda, oracle, p2p):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, p2p)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, lg, gen, err = q.get(timeout=600)
        res[r] = (lg, gen, err)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][2] == 0 and res[1][2] == 0
    from agent_harness_b200.model import Model, ModelConfig
    m = Model(ModelConfig(**SMALL), device="cuda:0")
    m.init_random(123)
    m.reset(2)
    for t in range(PROMPT.shape[1]):
        ref = m.forward(PROMPT[:, t]).cpu().numpy()
        full = np.concatenate([res[0][0][t], res[1][0][t]], axis=1)
        err = np.max(np.abs(full - ref)) / np.max(np.abs(ref))
        assert err <= 1e-3, (t, err)
    gen1 = m.generate(PROMPT, 8)
    gen1_long = m.generate(LONG, 6)
    m.generate(LONG, 0)
    last1 = m.forward(LONG[:, -1]).cpu().numpy()
    m.close()
    (g0, gl0, la0, sl0, st0, sg0), (g1, gl1, la1, sl1, st1, sg1) = res[0][1], res[1][1]
    assert np.array_equal(g0, g1) and np.array_equal(g0, gen1)
    # the long prompt went through the tensor-parallel prefill GEMMs
    assert np.array_equal(gl0, gl1) and np.array_equal(gl0, gen1_long)
    full = np.concatenate([la0, la1], axis=1)
    assert np.max(np.abs(full - last1)) / np.max(np.abs(last1)) <= 1e-3
    # sampling: both ranks pick the same tokens, sample() of the full logits
    # (the ranks' slices concatenated) with the draw for (99, position 5, b)
    assert np.array_equal(st0, st1) and np.array_equal(sg0, sg1) and np.array_equal(sg0[0], st0)
    full = np.concatenate([sl0, sl1], axis=1)
    for b in range(2):
        r = oracle.sample_uniform(99, PROMPT.shape[1] - 1, b)
        assert st0[b] == oracle.sample(full[b], 0.8, 40, r), b


# batch 16 with every projection on the tcgen05 batched GEMV (min_batch 1):
# the o / down projections' peer-store epilogue (nvlink_peer) or their NCCL
# all-reduce, at widths whose row blocks several CTAs share (stream-K)
WIDE = dict(n_layer=2, n_embd=1024, n_ff=2048, n_head=8, n_head_kv=2, head_dim=128, vocab_size=1000, max_seq=32,
            max_batch=16, rope_freq_base=10000.0, rms_eps=1e-5)
PROMPT16 = (np.arange(16 * 5, dtype=np.int32).reshape(16, 5) * 53 + 7) % 1000


def _rank16(rank, world, port, q, p2p):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from agent_harness_b200 import _lib
        from agent_harness_b200.model import Model, ModelConfig, nccl_unique_id
        _lib.check(_lib.lib().ah_device_init(rank))
        ids = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        m = Model(ModelConfig(**WIDE), device=f"cuda:{rank}", tp_rank=rank, tp_world=world, nccl_id=ids[0])
        m.init_random(77)
        m.set_batched_gemv(1)
        if p2p:
            def allgather(blob):
                out = [None] * world
                dist.all_gather_object(out, blob)
                return out
            m.enable_peer_allreduce(allgather)
        m.reset(16)
        logits = [m.forward(PROMPT16[:, t]).cpu().numpy() for t in range(PROMPT16.shape[1])]
        gen = m.generate(PROMPT16, 4)
        torch.cuda.synchronize()
        err = _lib.lib().ah_check_device_error(None)
        m.close()
        q.put((rank, logits, gen, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("p2p", [False, True], ids=["nccl", "nvlink_peer"])
def test_tp2_batch16_tensor_core_gemv(cuda, p2p):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank16, args=(r, 2, port, q, p2p)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, lg, gen, err = q.get(timeout=600)
        res[r] = (lg, gen, err)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][2] == 0 and res[1][2] == 0
    from agent_harness_b200.model import Model, ModelConfig
    m = Model(ModelConfig(**WIDE), device="cuda:0")
    m.init_random(77)
    m.set_batched_gemv(1)
    m.reset(16)
    for t in range(PROMPT16.shape[1]):
        ref = m.forward(PROMPT16[:, t]).cpu().numpy()
        full = np.concatenate([res[0][0][t], res[1][0][t]], axis=1)
        for b in range(16):
            err = np.max(np.abs(full[b] - ref[b])) / np.max(np.abs(ref[b]))
            assert err <= 1e-3, (t, b, err)
    m.close()
    # the ranks merge their argmax candidates: identical tokens on both
    assert np.array_equal(res[0][1], res[1][1])
