"""Device-tensor front-end of the C ABI (torch CUDA tensors in, tensors out).

torch supplies device memory and streams only; every computation below is one
of the library's sm_100a kernels.  All calls run on torch's current stream.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import AhError, call, lib

DTYPE_F32, DTYPE_F16, DTYPE_Q4_0, DTYPE_Q8_0, DTYPE_Q6_K, DTYPE_BF16 = 0, 1, 2, 8, 13, 30
GROUP_SIZE = 32


def _stream(dev: torch.device | None = None):
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _ptr(t: torch.Tensor):
    if not t.is_cuda:
        raise AhError(-1, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise AhError(-1, "expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


def _as_u8(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.contiguous().view(torch.uint8)


# --- conversions ---------------------------------------------------------------

def f16_to_f32(src: torch.Tensor) -> torch.Tensor:
    """formats/gguf.rs:93-120 semantics over f16 bit patterns (int16/uint16/float16)."""
    out = torch.empty(src.numel(), dtype=torch.float32, device=src.device)
    call("ah_f16_to_f32", _ptr(src), _ptr(out), src.numel(), _stream(src.device))
    return out


def bf16_to_f32(src: torch.Tensor) -> torch.Tensor:
    out = torch.empty(src.numel(), dtype=torch.float32, device=src.device)
    call("ah_bf16_to_f32", _ptr(src), _ptr(out), src.numel(), _stream(src.device))
    return out


def f32_to_f16(src: torch.Tensor) -> torch.Tensor:
    out = torch.empty(src.numel(), dtype=torch.int16, device=src.device)
    call("ah_f32_to_f16", _ptr(src), _ptr(out), src.numel(), _stream(src.device))
    return out


# --- dequantisation --------------------------------------------------------------

def dequant_q8_0(blocks: torch.Tensor, n: int, out: torch.Tensor | None = None) -> torch.Tensor:
    out = out if out is not None else torch.empty(n, dtype=torch.float32, device=blocks.device)
    call("ah_dequant_q8_0_f32", _ptr(blocks), _ptr(out), n, _stream(blocks.device))
    return out


def dequant_q4_0(blocks: torch.Tensor, n: int, out: torch.Tensor | None = None) -> torch.Tensor:
    out = out if out is not None else torch.empty(n, dtype=torch.float32, device=blocks.device)
    call("ah_dequant_q4_0_f32", _ptr(blocks), _ptr(out), n, _stream(blocks.device))
    return out


def dequant_layer(scales: torch.Tensor, packed: torch.Tensor, n: int, group_size: int = GROUP_SIZE) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=packed.device)
    call("ah_dequant_layer", _ptr(scales), _ptr(packed), _ptr(out), n, group_size, _stream(packed.device))
    return out


def dequantize_to_f32(raw: torch.Tensor, dtype: int, element_count: int) -> torch.Tensor:
    raw = _as_u8(raw)
    cap = max(element_count, raw.numel() // 2, 1)
    out = torch.empty(cap, dtype=torch.float32, device=raw.device)
    n_out = C.c_int64(0)
    call("ah_dequantize_to_f32", _ptr(raw), raw.numel(), dtype, element_count, _ptr(out), C.byref(n_out),
         _stream(raw.device))
    return out[: n_out.value]


# --- quantisers ---------------------------------------------------------------------

def quantize_q4(w: torch.Tensor, group_size: int = GROUP_SIZE):
    n = w.numel()
    gs = max(group_size, 1)
    scales = torch.empty((n + gs - 1) // gs, dtype=torch.float32, device=w.device)
    packed = torch.empty((n + 1) // 2, dtype=torch.uint8, device=w.device)
    call("ah_quantize_q4", _ptr(w), n, group_size, _ptr(scales), _ptr(packed), _stream(w.device))
    return scales, packed


def quantize_q8_0(w: torch.Tensor) -> torch.Tensor:
    n = w.numel()
    blocks = torch.empty(((n + 31) // 32) * 34, dtype=torch.uint8, device=w.device)
    call("ah_quantize_q8_0", _ptr(w), n, _ptr(blocks), _stream(w.device))
    return blocks


def quantize_q4_0(w: torch.Tensor) -> torch.Tensor:
    n = w.numel()
    blocks = torch.empty(((n + 31) // 32) * 18, dtype=torch.uint8, device=w.device)
    call("ah_quantize_q4_0", _ptr(w), n, _ptr(blocks), _stream(w.device))
    return blocks


# --- synthetic inputs ------------------------------------------------------------------

def fill_normal(n: int, mean: float, std: float, seed: int, device="cuda", index_offset: int = 0) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=device)
    call("ah_fill_normal", _ptr(out), n, mean, std, seed, index_offset, _stream(out.device))
    return out


def synth_q4_0(rows: int, cols: int, std: float, seed: int, device="cuda", row0: int = 0, col0: int = 0,
               full_cols: int | None = None) -> torch.Tensor:
    full_cols = cols if full_cols is None else full_cols
    blocks = torch.empty(rows * (cols // 32) * 18, dtype=torch.uint8, device=device)
    call("ah_synth_q4_0", _ptr(blocks), row0, rows, col0, cols, full_cols, std, seed, _stream(blocks.device))
    return blocks


def synth_f16(n: int, mean: float, std: float, seed: int, device="cuda", index_offset: int = 0) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.int16, device=device)
    call("ah_synth_f16", _ptr(out), n, mean, std, seed, index_offset, _stream(out.device))
    return out


# --- fused GEMV ----------------------------------------------------------------------------

class _DeviceBuffer:
    """A raw device allocation seen through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _device_bytes(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.as_tensor(_DeviceBuffer(ptr, int(nbytes)), device=device)


class Q4Weight:
    """A device-resident quantised matrix in the GEMV's tiled layout."""

    def __init__(self, handle: C.c_void_p, rows: int, cols: int, device: torch.device):
        self._h = handle
        self.rows, self.cols, self.device = rows, cols, device

    @classmethod
    def from_q4_0(cls, blocks: torch.Tensor, rows: int, cols: int) -> "Q4Weight":
        h = C.c_void_p()
        call("ah_q4w_from_q4_0", _ptr(blocks), rows, cols, C.byref(h), _stream(blocks.device))
        return cls(h, rows, cols, blocks.device)

    @classmethod
    def from_engine(cls, scales: torch.Tensor, packed: torch.Tensor, rows: int, cols: int) -> "Q4Weight":
        h = C.c_void_p()
        call("ah_q4w_from_engine", _ptr(scales), _ptr(packed), rows, cols, C.byref(h), _stream(packed.device))
        return cls(h, rows, cols, packed.device)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @property
    def weight_bytes(self) -> int:
        return int(lib().ah_q4w_weight_bytes(self._h))

    def planes(self):
        """Copies of the device planes (nibbles, scales) as uint8 tensors, and
        whether the scales are f32 (engine format) rather than f16 (Q4_0)."""
        nib, scl = C.c_void_p(), C.c_void_p()
        nb, sb = C.c_size_t(), C.c_size_t()
        f32 = C.c_int()
        call("ah_q4w_planes", self._h, C.byref(nib), C.byref(nb), C.byref(scl), C.byref(sb), C.byref(f32))
        return (_device_bytes(nib.value, nb.value, self.device).clone(),
                _device_bytes(scl.value, sb.value, self.device).clone(), bool(f32.value))

    def gemv(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y[b] = W @ x[b] for x of shape [cols] or [batch, cols] (batch <= 16)."""
        squeeze = x.dim() == 1
        xb = x.reshape(-1, self.cols)
        batch = xb.shape[0]
        if out is None:
            out = torch.empty(batch, self.rows, dtype=torch.float32, device=x.device)
        call("ah_q4w_gemv", self._h, _ptr(xb), _ptr(out), batch, _stream(x.device))
        return out.reshape(self.rows) if squeeze else out

    def gemv_host(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """y = W @ x for host tensors (pinned for asynchronous copies): copy in,
        GEMV on the resident weight, copy out, wait -- one library call."""
        assert not x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        xb = x.reshape(-1, self.cols)
        batch = xb.shape[0]
        if out is None:
            out = torch.empty(batch, self.rows, dtype=torch.float32).pin_memory()
        assert not out.is_cuda and out.is_contiguous() and out.numel() == batch * self.rows
        st = _stream(self.device) if stream is None else C.c_void_p(stream.cuda_stream)
        call("ah_q4w_gemv_host", self._h, C.c_void_p(xb.data_ptr()), C.c_void_p(out.data_ptr()), batch, st)
        return out.reshape(self.rows) if x.dim() == 1 else out

    def gemm_workspace_bytes(self, m: int) -> int:
        n = C.c_size_t()
        call("ah_q4w_gemm_workspace_bytes", self._h, m, C.byref(n))
        return int(n.value)

    def gemm(self, a: torch.Tensor, out: torch.Tensor | None = None,
             workspace: torch.Tensor | None = None, epilogue: str = "store", norm_w: torch.Tensor | None = None,
             eps: float = 1e-5) -> torch.Tensor:
        """C = A @ W^T on the tensor cores for A of shape [m, cols] f32 (prefill).
        epilogue "swiglu" (an interleaved gate/up weight): C = silu(gate) * up,
        [m, rows / 2]; "add": C += A @ W^T.  norm_w (f16 bits, cols): RMSNorm
        each row of A first."""
        assert a.dtype == torch.float32 and a.dim() == 2 and a.shape[1] == self.cols and a.stride(1) == 1
        m = a.shape[0]
        epi = {"store": 0, "swiglu": 1, "add": 2}[epilogue]
        if out is not None and (not out.is_cuda or out.dtype != torch.float32 or out.stride(1) != 1):
            raise AhError(-1, "expected a CUDA f32 output with unit-stride rows")
        if out is None:
            assert epi != 2, "the add epilogue needs out"
            out = torch.empty(m, self.rows // 2 if epi == 1 else self.rows, dtype=torch.float32, device=a.device)
        need = self.gemm_workspace_bytes(m)
        if workspace is None or workspace.numel() < need + 1024:
            workspace = torch.empty(need + 1024, dtype=torch.uint8, device=a.device)
        base = workspace.data_ptr()
        aligned = (base + 1023) // 1024 * 1024
        if epi == 0 and norm_w is None:
            call("ah_q4w_gemm", self._h, _ptr(a), a.stride(0), m, C.c_void_p(out.data_ptr()), out.stride(0),
                 C.c_void_p(aligned), need, _stream(a.device))
        else:
            call("ah_q4w_gemm_ex", self._h, _ptr(a), a.stride(0), m, C.c_void_p(out.data_ptr()), out.stride(0), epi,
                 _ptr(norm_w) if norm_w is not None else None, eps, C.c_void_p(aligned), need, _stream(a.device))
        return out

    def gemv_tc_workspace_bytes(self) -> int:
        n = C.c_size_t()
        call("ah_q4w_gemv_tc_workspace_bytes", self._h, C.byref(n))
        return n.value

    def gemv_tc(self, x: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
        """y = W x for 1..16 token rows x [batch, cols] f32 through the tcgen05
        batched GEMV (f16 operands, f32 accumulation); accumulate adds into out."""
        assert x.dtype == torch.float32 and x.dim() == 2 and x.shape[1] == self.cols and x.stride(1) == 1
        b = x.shape[0]
        if out is None:
            assert not accumulate
            out = torch.empty(b, self.rows, dtype=torch.float32, device=x.device)
        need = self.gemv_tc_workspace_bytes()
        if workspace is None or workspace.numel() < need + 1024:
            workspace = torch.empty(need + 1024, dtype=torch.uint8, device=x.device)
        base = workspace.data_ptr()
        aligned = (base + 1023) // 1024 * 1024
        assert x.is_cuda and out.is_cuda and out.dim() == 2 and out.stride(1) == 1 and out.shape[0] == b
        # row-strided views are fine: the entry point takes the row strides
        call("ah_q4w_gemv_tc", self._h, C.c_void_p(x.data_ptr()), x.stride(0), b, C.c_void_p(out.data_ptr()),
             out.stride(0), int(bool(accumulate)), C.c_void_p(aligned), need, _stream(x.device))
        return out

    def close(self):
        if self._h:
            lib().ah_q4w_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemv_4bit_into(out: torch.Tensor, scales: torch.Tensor, packed: torch.Tensor, x: torch.Tensor, rows: int,
                   cols: int, group_size: int = GROUP_SIZE) -> torch.Tensor:
    """inference/math.rs:255-295 on device tensors in the engine's own storage."""
    call("ah_gemv_4bit_into", _ptr(out), _ptr(scales), _ptr(packed), _ptr(x) if x.numel() else None, rows, cols,
         group_size, _stream(out.device))
    return out


def gemv_4bit_rows(out: torch.Tensor, scales: torch.Tensor, packed: torch.Tensor, x: torch.Tensor, row_start: int,
                   row_end: int, cols: int, group_size: int = GROUP_SIZE) -> torch.Tensor:
    """inference/math.rs:382-418 gemv_4bit_parallel_worker_scalar on device
    tensors: rows [row_start, row_end) of the full planes into out."""
    call("ah_gemv_4bit_rows", _ptr(out), _ptr(scales), _ptr(packed), _ptr(x), row_start, row_end, cols, group_size,
         _stream(out.device))
    return out


def swiglu_4bit_into(out: torch.Tensor, x: torch.Tensor, gate_scales, gate_packed, up_scales, up_packed,
                     down_scales, down_packed, n_embd: int, n_ff: int, group_size: int, scratch_gate: torch.Tensor,
                     scratch_up: torch.Tensor, scratch_act: torch.Tensor) -> torch.Tensor:
    """inference/ffn.rs:155-174 on device tensors in the engine's own storage."""
    call("ah_swiglu_4bit_into", _ptr(out), _ptr(x), _ptr(gate_scales), _ptr(gate_packed), _ptr(up_scales),
         _ptr(up_packed), _ptr(down_scales), _ptr(down_packed), n_embd, n_ff, group_size, _ptr(scratch_gate),
         _ptr(scratch_up), _ptr(scratch_act), _stream(out.device))
    return out


def sample_workspace_bytes(batch: int, vocab: int) -> int:
    return int(lib().ah_sample_workspace_bytes(batch, vocab))


def sample_logits(logits: torch.Tensor, temperature: float, top_k: int = 40, seed: int = 0, step: int = 0,
                  out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                  split: bool = True) -> torch.Tensor:
    """inference/sampling.rs:17-64 sample(row, temperature, top_k) for each row
    of a [batch, vocab] f32 device tensor; the draw of row b is
    sample_uniform(seed, step, b).  Returns int32 tokens [batch].  Rows are
    split over CTAs through a workspace (allocated here unless given);
    split=False walks each row with one CTA."""
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    if not logits.is_cuda or logits.dtype != torch.float32 or logits.stride(1) != 1:
        raise AhError(-1, "expected a CUDA f32 tensor with unit-stride rows")
    batch, vocab = logits.shape
    if out is None:
        out = torch.empty(batch, dtype=torch.int32, device=logits.device)
    ws, nbytes = None, 0
    if split:
        nbytes = sample_workspace_bytes(batch, vocab)
        if workspace is None and nbytes:
            workspace = torch.empty(nbytes, dtype=torch.uint8, device=logits.device)
        if nbytes:
            ws = _ptr(workspace)
            nbytes = workspace.numel() * workspace.element_size()
    call("ah_sample_logits", C.c_void_p(logits.data_ptr()), logits.stride(0), batch, vocab, temperature, top_k, seed,
         step, _ptr(out), ws, nbytes, _stream(logits.device))
    return out


def sample_uniform(seed: int, step: int, seq: int) -> float:
    """The draw in [0, 1) that sample_logits uses for sequence seq at step."""
    return lib().ah_sample_uniform(seed, step, seq)


class SwigluBlock:
    """The feed-forward block on resident tiled weights, as the decoder runs it:
    gate and up interleaved in one weight (one GEMV whose epilogue writes
    silu(gate) * up), then the down GEMV."""

    def __init__(self, gate_up: C.c_void_p, down: Q4Weight, n_embd: int, n_ff: int):
        self.gate_up = Q4Weight(gate_up, 2 * n_ff, n_embd, down.device)
        self.down, self.n_embd, self.n_ff = down, n_embd, n_ff

    @classmethod
    def from_engine(cls, gate_scales, gate_packed, up_scales, up_packed, down_scales, down_packed, n_embd: int,
                    n_ff: int) -> "SwigluBlock":
        h = C.c_void_p()
        call("ah_q4w_from_engine_gate_up", _ptr(gate_scales), _ptr(gate_packed), _ptr(up_scales), _ptr(up_packed),
             n_ff, n_embd, C.byref(h), _stream(gate_packed.device))
        return cls(h, Q4Weight.from_engine(down_scales, down_packed, n_embd, n_ff), n_embd, n_ff)

    @classmethod
    def from_q4_0(cls, gate_blocks, up_blocks, down_blocks, n_embd: int, n_ff: int) -> "SwigluBlock":
        h = C.c_void_p()
        call("ah_q4w_from_q4_0_gate_up", _ptr(gate_blocks), _ptr(up_blocks), n_ff, n_embd, C.byref(h),
             _stream(gate_blocks.device))
        return cls(h, Q4Weight.from_q4_0(down_blocks, n_embd, n_ff), n_embd, n_ff)

    def __call__(self, x: torch.Tensor, act: torch.Tensor | None = None) -> torch.Tensor:
        xb = x.reshape(-1, self.n_embd)
        batch = xb.shape[0]
        act = act if act is not None else torch.empty(batch, self.n_ff, dtype=torch.float32, device=x.device)
        out = torch.empty(batch, self.n_embd, dtype=torch.float32, device=x.device)
        call("ah_q4w_swiglu", self.gate_up.handle, self.down.handle, _ptr(xb), _ptr(act), _ptr(out), batch,
             _stream(x.device))
        return out.reshape(self.n_embd) if x.dim() == 1 else out

    def close(self):
        self.gate_up.close()
        self.down.close()
