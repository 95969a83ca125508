"""GPU: the allocation-free prefill GEMM entry (workspace in a static per-device
buffer) against the workspace-taking ah_q4w_gemm on the same inputs, two calls
in a row each.  Collected last so it also runs after every other GPU test."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(W, a, out, dev):
    from agent_harness_b200._lib import call
    from agent_harness_b200.kernels import _ptr, _stream
    m, k = a.shape
    call("ah_q4w_gemm_noalloc", W.handle, _ptr(a), k, m, _ptr(out), out.shape[1], _stream(dev))


@pytest.mark.parametrize("m,n,k", [(512, 2048, 4096), (37, 3 * 208 + 5, 320), (129, 16, 64)])
def test_noalloc_matches_workspace_entry(cuda, m, n, k):
    from agent_harness_b200 import kernels as K
    blocks = K.synth_q4_0(n, k, 0.02, 1000 + m, device=cuda)
    W = K.Q4Weight.from_q4_0(blocks, n, k)
    a = K.fill_normal(m * k, 0.0, 1.0, 2000 + m, device=cuda).reshape(m, k)
    ref = W.gemm(a)
    for _ in range(2):
        out = torch.full((m, n), float("nan"), device=cuda)
        _noalloc(W, a, out, cuda)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    W.close()


def test_noalloc_rejects_oversize_and_accepts_empty(cuda):
    from agent_harness_b200 import kernels as K
    from agent_harness_b200._lib import AhError, call, lib
    from agent_harness_b200.kernels import _ptr, _stream
    n, k, m = 64, 4096, 1024
    W = K.Q4Weight.from_q4_0(K.synth_q4_0(n, k, 0.02, 7, device=cuda), n, k)
    # buffers of the full requested size, so that even a regressed size check
    # could not read or write outside them
    a = torch.zeros(m, k, device=cuda)
    out = torch.zeros(m, n, device=cuda)
    # 1024 tokens x 4096 columns need 8 MiB + 4 KiB of f16 tiles: over the
    # buffer, refused on the host before any launch
    n_alloc = lib().ah_device_alloc_count()
    with pytest.raises(AhError) as e:
        call("ah_q4w_gemm_noalloc", W.handle, _ptr(a), k, m, _ptr(out), n, _stream(cuda))
    assert e.value.status == -1
    call("ah_q4w_gemm_noalloc", W.handle, _ptr(a), k, 0, _ptr(out), n, _stream(cuda))  # no-op
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0
    assert lib().ah_device_alloc_count() == n_alloc
    assert torch.count_nonzero(out) == 0
    W.close()


_FRESH = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from agent_harness_b200 import kernels as K
from agent_harness_b200._lib import call, lib
from agent_harness_b200.kernels import _ptr, _stream
torch.cuda.set_device(0)
dev = torch.device("cuda:0")
m, n, k = 300, 1040, 2048
W = K.Q4Weight.from_q4_0(K.synth_q4_0(n, k, 0.02, 5, device=dev), n, k)
a = K.fill_normal(m * k, 0.0, 1.0, 6, device=dev).reshape(m, k)
outs = []
before = lib().ah_device_alloc_count()
for _ in range(2):
    out = torch.full((m, n), float("nan"), device=dev)
    call("ah_q4w_gemm_noalloc", W.handle, _ptr(a), k, m, _ptr(out), n, _stream(dev))
    torch.cuda.synchronize()
    outs.append(out)
after = lib().ah_device_alloc_count()
assert after == before, (before, after)
assert lib().ah_check_device_error(None) == 0
ref = W.gemm(a)
assert torch.equal(outs[0], ref) and torch.equal(outs[1], ref)
print("fresh ok", before, after)
"""


def test_noalloc_first_call_in_fresh_process_allocates_nothing(cuda):
    # A process that never called ah_device_init: the first calls on the
    # device must not allocate (not even the device error word) and must
    # match the workspace entry.
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH, root], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fresh ok" in r.stdout
