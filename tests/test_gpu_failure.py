"""GPU: failure detection without a GPU fault.

Host side: ah_debug_inject_failure makes the nth device allocation, NCCL
communicator set-up or fused-GEMV launch fail as the real call would, and the
status must reach the caller with its message (AH_ENOMEM / AH_ENCCL /
AH_ECUDA) while the library stays usable.  Device side: the tensor-parallel
decoder's peer all-reduce step waits on a flag that nothing sets; its bounded
wait must give up (about 0.4 s), report AH_ETIMEOUT through the device error
word and leave the hidden state untouched.  No test faults, traps or hangs the
GPU.  The reference routes a failed GPU allocation to the host
(memory_controller/virtual_tensor_arena.rs:128-147); here the failure is a
status the caller sees.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inject(kind, nth):
    from agent_harness_b200._lib import call
    call("ah_debug_inject_failure", kind, nth)


def test_injected_allocation_failure_is_enomem(cuda):
    from agent_harness_b200 import kernels as K
    from agent_harness_b200._lib import AH_ENOMEM, AH_INJECT_ALLOC, AhError, lib
    blocks = K.synth_q4_0(64, 256, 0.02, 1, device=cuda)
    n0 = lib().ah_device_alloc_count()
    for nth in (1, 2):  # the nibble plane, then the scale plane (the first is freed again)
        _inject(AH_INJECT_ALLOC, nth)
        with pytest.raises(AhError) as e:
            K.Q4Weight.from_q4_0(blocks, 64, 256)
        assert e.value.status == AH_ENOMEM
        assert "cudaMalloc" in str(e.value)
    assert lib().ah_device_alloc_count() == n0 + 1  # only the nth=2 attempt's first plane was made
    _inject(AH_INJECT_ALLOC, 0)
    W = K.Q4Weight.from_q4_0(blocks, 64, 256)  # disarmed: works again
    x = K.fill_normal(256, 0.0, 1.0, 2, device=cuda)
    assert torch.isfinite(W.gemv(x)).all()
    W.close()


def test_injected_launch_failure_is_ecuda(cuda):
    from agent_harness_b200 import kernels as K
    from agent_harness_b200._lib import AH_ECUDA, AH_INJECT_LAUNCH, AhError
    W = K.Q4Weight.from_q4_0(K.synth_q4_0(128, 512, 0.02, 3, device=cuda), 128, 512)
    x = K.fill_normal(512, 0.0, 1.0, 4, device=cuda)
    ref = W.gemv(x)
    _inject(AH_INJECT_LAUNCH, 1)
    with pytest.raises(AhError) as e:
        W.gemv(x)
    assert e.value.status == AH_ECUDA and "injected" in str(e.value)
    torch.cuda.synchronize()
    assert torch.equal(W.gemv(x), ref)  # the next launch runs
    W.close()


def test_injected_nccl_failure_is_enccl(cuda):
    from agent_harness_b200._lib import AH_ENCCL, AH_INJECT_NCCL, AhError
    from agent_harness_b200.model import Model, ModelConfig
    cfg = ModelConfig(n_layer=1, n_embd=128, n_ff=256, n_head=4, n_head_kv=2, head_dim=32, vocab_size=256,
                      max_seq=16, max_batch=1)
    _inject(AH_INJECT_NCCL, 1)
    # rank 0 of 2: the injected failure comes before NCCL would wait for rank 1
    with pytest.raises(AhError) as e:
        Model(cfg, device=cuda, tp_rank=0, tp_world=2, nccl_id=bytes(128))
    assert e.value.status == AH_ENCCL and "injected" in str(e.value)
    _inject(AH_INJECT_NCCL, 0)


def test_peer_allreduce_wait_times_out_and_leaves_hidden(cuda):
    from agent_harness_b200._lib import AH_ETIMEOUT, call, lib
    from agent_harness_b200.kernels import _ptr, _stream
    world, batch, d = 2, 3, 256
    hidden = K_hidden = torch.randn(batch, d, device=cuda)
    before = hidden.clone()
    slots = torch.randn(world * d * batch, device=cuda)
    ss = torch.zeros(batch, d // 16, device=cuda)
    flags = torch.zeros(64, dtype=torch.int32, device=cuda)
    seq = torch.ones(1, dtype=torch.int32, device=cuda)
    flags[0] = 1  # rank 0 has signalled; rank 1 never does
    assert lib().ah_check_device_error(None) == 0
    call("ah_debug_residual_add_peer", _ptr(hidden), _ptr(slots), world, batch, d, _ptr(ss), _ptr(flags), _ptr(seq),
         _stream(cuda))
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == AH_ETIMEOUT
    assert b"gave up" in lib().ah_last_error()
    assert torch.equal(K_hidden, before)
    assert lib().ah_check_device_error(None) == 0  # the word was cleared
    # once every flag is set the same step completes: hidden += slot sums in rank order
    flags[1] = 1
    call("ah_debug_residual_add_peer", _ptr(hidden), _ptr(slots), world, batch, d, _ptr(ss), _ptr(flags), _ptr(seq),
         _stream(cuda))
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0
    s = slots.view(world, d, batch)
    ref = before + (s[0] + s[1]).t()
    assert torch.equal(hidden, ref)
    q = (ref * ref).view(batch, d // 16, 16)
    np.testing.assert_allclose(ss.cpu().numpy(), q.sum(-1).cpu().numpy(), rtol=1e-5)
