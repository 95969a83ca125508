"""Host-slice mirrors of the reference's Rust API for the hot path.

Each function keeps the reference's name, argument meaning and behaviour on
empty input, takes host numpy arrays (the Rust slices) and runs on the GPU
through the synchronous ah_host_* entries of the C ABI.  No CPU fallback.

  models/quantization.rs : GROUP_SIZE, quantize, dequant_weight, dequant_layer,
                           packed_bytes, n_groups, quantized_bytes
  inference/math.rs      : gemv_4bit_into, matvec_4bit_into, gemv_4bit_parallel_worker_scalar
  inference/ffn.rs       : swiglu_4bit_into
  models/avx512_kernel.rs: f16_bytes_to_f32, bf16_bytes_to_f32
  models/formats/gguf.rs : f16_to_f32, bf16_to_f32, dequantize_to_f32
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import AhError, call, lib

GROUP_SIZE = 32  # models/quantization.rs:365


def _p(a: np.ndarray):
    return C.c_void_p(a.ctypes.data) if a.size else None


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# --- models/quantization.rs ---------------------------------------------------

def packed_bytes(n_elements: int) -> int:
    return int(lib().ah_packed_bytes(n_elements))


def n_groups(n_elements: int, group_size: int) -> int:
    return int(lib().ah_n_groups(n_elements, group_size))


def quantized_bytes(n_elements: int, group_size: int) -> int:
    return int(lib().ah_quantized_bytes(n_elements, group_size))


def quantize(weights: np.ndarray, group_size: int = GROUP_SIZE):
    """quantization.rs:369-404 -> (scales f32[n_groups], packed u8[ceil(n/2)])."""
    w = _c(weights, np.float32).ravel()
    gs = max(group_size, 1)
    scales = np.zeros((w.size + gs - 1) // gs, np.float32)
    packed = np.zeros((w.size + 1) // 2, np.uint8)
    if w.size:
        call("ah_host_quantize", _p(w), w.size, gs, _p(scales), _p(packed))
    return scales, packed


def dequant_layer(scales: np.ndarray, packed: np.ndarray, result: np.ndarray, group_size: int = GROUP_SIZE) -> None:
    """quantization.rs:439-454: fills `result` in place (scalar-path semantics)."""
    if result.dtype != np.float32 or not result.flags.c_contiguous:
        raise AhError(-1, "result must be a contiguous float32 array")
    s, p = _c(scales, np.float32), _c(packed, np.uint8)
    if result.size:
        call("ah_host_dequant_layer", _p(s), _p(p), _p(result), result.size, group_size)


def dequant_weight(scales: np.ndarray, packed: np.ndarray, index: int, group_size: int = GROUP_SIZE) -> float:
    """quantization.rs:407-420: one element, dequantised on the device from its
    byte and its group's scale."""
    gs = max(group_size, 1)
    s = np.array([scales[index // gs]], np.float32)
    p = np.array([packed[index // 2]], np.uint8)
    out = np.empty(2, np.float32)
    call("ah_host_dequant_layer", _p(s), _p(p), _p(out), 2, 2)
    return float(out[index % 2])


# --- inference/math.rs ---------------------------------------------------------------

def gemv_4bit_into(out: np.ndarray, scales: np.ndarray, packed: np.ndarray, x: np.ndarray, rows: int, cols: int,
                   group_size: int = GROUP_SIZE) -> None:
    """math.rs:255-295: out[r] = sum_j ((nib-8)*scale) * x[j]; empty input zeroes out."""
    if out.dtype != np.float32 or not out.flags.c_contiguous:
        raise AhError(-1, "out must be a contiguous float32 array")
    s, p, xv = _c(scales, np.float32), _c(packed, np.uint8), _c(x, np.float32)
    call("ah_host_gemv_4bit_into", _p(out), _p(s), _p(p), _p(xv), rows, cols, group_size)


def matvec_4bit_into(out, scales, packed, x, dim: int, group_size: int = GROUP_SIZE) -> None:
    """math.rs:205-214."""
    gemv_4bit_into(out, scales, packed, x, dim, dim, group_size)


def gemv_4bit_parallel_worker_scalar(out: np.ndarray, global_scales: np.ndarray, global_packed: np.ndarray,
                                     x: np.ndarray, row_start: int, row_end: int, cols: int,
                                     group_size: int = GROUP_SIZE) -> None:
    """math.rs:382-418: out[i - row_start] for rows [row_start, row_end) of the
    full matrix (the row-range worker gemv_4bit_into hands to each thread)."""
    if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < row_end - row_start:
        raise AhError(-1, "out must be a contiguous float32 array of row_end - row_start values")
    s, p, xv = _c(global_scales, np.float32), _c(global_packed, np.uint8), _c(x, np.float32)
    call("ah_host_gemv_4bit_worker_scalar", _p(out), _p(s), _p(p), _p(xv), row_start, row_end, cols, group_size)


# --- inference/ffn.rs -----------------------------------------------------------------

def swiglu_4bit_into(out: np.ndarray, input: np.ndarray, gate_scales, gate_packed, up_scales, up_packed, down_scales,
                     down_packed, n_embd: int, n_ff: int, group_size: int, scratch_gate: np.ndarray,
                     scratch_up: np.ndarray, scratch_act: np.ndarray) -> None:
    """ffn.rs:155-174: gate/up GEMVs, act = silu(gate) * up, out = down . act;
    the scratch slices receive the intermediates, as the reference's do."""
    for a, n in ((out, n_embd), (scratch_gate, n_ff), (scratch_up, n_ff), (scratch_act, n_ff)):
        if a.dtype != np.float32 or not a.flags.c_contiguous or a.size < n:
            raise AhError(-1, "out and scratch slices must be contiguous float32 arrays of their lengths")
    args = [_c(v, dt) for v, dt in ((input, np.float32), (gate_scales, np.float32), (gate_packed, np.uint8),
                                     (up_scales, np.float32), (up_packed, np.uint8), (down_scales, np.float32),
                                     (down_packed, np.uint8))]
    call("ah_host_swiglu_4bit_into", _p(out), *[_p(a) for a in args], n_embd, n_ff, group_size, _p(scratch_gate),
         _p(scratch_up), _p(scratch_act))


# --- models/avx512_kernel.rs / models/formats/gguf.rs ---------------------------------

def f16_bytes_to_f32(src: bytes | np.ndarray) -> np.ndarray:
    """avx512_kernel.rs:212-232 with the defined (gguf.rs:93-120) semantics."""
    b = np.frombuffer(src, np.uint8) if isinstance(src, (bytes, bytearray)) else _c(src, np.uint8).ravel()
    out = np.empty(b.size // 2, np.float32)
    if out.size:
        call("ah_host_f16_bytes_to_f32", _p(b), b.size, _p(out))
    return out


def bf16_bytes_to_f32(src: bytes | np.ndarray) -> np.ndarray:
    """avx512_kernel.rs:236-255."""
    b = np.frombuffer(src, np.uint8) if isinstance(src, (bytes, bytearray)) else _c(src, np.uint8).ravel()
    out = np.empty(b.size // 2, np.float32)
    if out.size:
        call("ah_host_bf16_bytes_to_f32", _p(b), b.size, _p(out))
    return out


def f16_to_f32(bits: int) -> float:
    """gguf.rs:93-120 for one value."""
    return float(f16_bytes_to_f32(np.array([bits], np.uint16).view(np.uint8))[0])


def bf16_to_f32(bits: int) -> float:
    """gguf.rs:124-126 for one value."""
    return float(bf16_bytes_to_f32(np.array([bits], np.uint16).view(np.uint8))[0])


def dequantize_to_f32(raw: bytes | np.ndarray, dtype: int, element_count: int) -> np.ndarray:
    """GGUFFile::dequantize_to_f32 (gguf.rs:434-535)."""
    b = np.frombuffer(raw, np.uint8) if isinstance(raw, (bytes, bytearray)) else _c(raw, np.uint8).ravel()
    cap = max(element_count, b.size // 2, 1)
    out = np.empty(cap, np.float32)
    n_out = C.c_size_t(0)
    call("ah_host_dequantize_to_f32", _p(b), b.size, dtype, element_count, _p(out), C.byref(n_out))
    return out[: n_out.value].copy()
