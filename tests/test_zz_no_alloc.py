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
    n, k = 64, 4096
    W = K.Q4Weight.from_q4_0(K.synth_q4_0(n, k, 0.02, 7, device=cuda), n, k)
    a = torch.zeros(1, k, device=cuda)
    out = torch.zeros(1, n, device=cuda)
    # 1024 tokens x 4096 columns need 8 MiB + 4 KiB of f16 tiles: over the
    # buffer, refused on the host before any launch
    with pytest.raises(AhError) as e:
        call("ah_q4w_gemm_noalloc", W.handle, _ptr(a), k, 1024, _ptr(out), n, _stream(cuda))
    assert e.value.status == -1
    call("ah_q4w_gemm_noalloc", W.handle, _ptr(a), k, 0, _ptr(out), n, _stream(cuda))  # no-op
    torch.cuda.synchronize()
    assert lib().ah_check_device_error(None) == 0
    W.close()
