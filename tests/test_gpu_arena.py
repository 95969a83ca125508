"""GPU test of the paged virtual tensor arena (memory_controller/
virtual_tensor_arena.rs) on CUDA virtual memory management: residency moves
(commit, routing past the GPU page budget, Move to the host pool, Drop,
re-commit) and the page GEMV (execute_layer_math) on GPU-resident and
host-resident pages, bit-identical to the device engine-format GEMV on the same
bytes and within 1e-5 of the oracle's gemv_4bit_into.  Only committed pages
are ever touched by a kernel."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

UNMAPPED, GPU, CPU = 0, 1, 2


def test_arena_residency_and_page_gemv(cuda, oracle):
    from agent_harness_b200 import _lib
    from agent_harness_b200 import kernels as K
    call = _lib.call
    g = C.c_size_t()
    call("ah_arena_page_granularity", C.byref(g))
    G = g.value
    n_pages = 6
    a = C.c_void_p()
    call("ah_arena_create", n_pages * G, G, 3, C.byref(a))

    def state(p):
        r, ptr = C.c_int(), C.c_void_p()
        call("ah_arena_page_state", a, p, C.byref(r), C.byref(ptr))
        return r.value, ptr.value

    try:
        for p in range(4):
            call("ah_arena_commit_page", a, p)
        assert [state(p)[0] for p in range(n_pages)] == [GPU, GPU, GPU, CPU, UNMAPPED, UNMAPPED]
        # one engine-format matrix filling a page exactly
        cols = 4096
        rows = 2 * G // cols
        w = (np.random.default_rng(3).standard_normal(rows * cols) * 0.05).astype(np.float32)
        scales, packed = oracle.quantize_q4(w)
        dev = torch.device("cuda")
        pool = torch.zeros(n_pages * G, dtype=torch.uint8).pin_memory()
        page0 = K._device_bytes(state(0)[1], G, dev)
        page0.copy_(torch.as_tensor(packed).to(dev))
        pool[3 * G:4 * G] = torch.as_tensor(packed)
        x = torch.randn(cols, device=dev)
        sc = torch.as_tensor(scales).to(dev)
        ref = K.gemv_4bit_into(torch.empty(rows, device=dev), sc, torch.as_tensor(packed).to(dev), x, rows, cols)
        want = oracle.gemv_4bit_into(scales, packed, x.cpu().numpy(), rows, cols)
        assert np.max(np.abs(ref.cpu().numpy() - want)) <= 1e-5 * np.max(np.abs(want))

        def page_gemv(p):
            out = torch.empty(rows, device=dev)
            call("ah_arena_gemv_4bit", a, p, C.c_void_p(pool.data_ptr()), C.c_void_p(out.data_ptr()),
                 C.c_void_p(sc.data_ptr()), C.c_void_p(x.data_ptr()), rows, cols, 32,
                 C.c_void_p(torch.cuda.current_stream().cuda_stream))
            return out

        assert torch.equal(page_gemv(0), ref)  # GPU resident
        assert torch.equal(page_gemv(3), ref)  # routed to the host at commit (budget of 3 GPU pages)
        # Move: the page's bytes land in the host pool and the GEMV reads them there
        call("ah_arena_evict_page", a, 0, 1, C.c_void_p(pool.data_ptr()), None)
        assert state(0)[0] == CPU
        assert np.array_equal(pool[:G].numpy(), packed)
        assert torch.equal(page_gemv(0), ref)
        # Drop: unmapped, and the GEMV refuses it (the reference panics)
        call("ah_arena_evict_page", a, 1, 0, None, None)
        assert state(1)[0] == UNMAPPED
        with pytest.raises(_lib.AhError):
            page_gemv(1)
        # a dropped page commits again under the budget (pages 1 and 2 on the GPU)
        call("ah_arena_commit_page", a, 1)
        assert state(1)[0] == GPU and state(1)[1] is not None
        torch.cuda.synchronize()
    finally:
        call("ah_arena_destroy", a)
