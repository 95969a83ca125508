"""ctypes front-end for the CPU oracle (oracle/ah_oracle*.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs, always as the checker or the timed CPU baseline
of the reference's own algorithm, never as a product code path.  Every
function forwards to the C restatement, which cites the reference's file:line.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libah_oracle.so")
_lib = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
i64 = C.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (system gcc, no FP contraction)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.or_f16_to_f32.argtypes = [C.c_uint16]; L.or_f16_to_f32.restype = C.c_float
        L.or_bf16_to_f32.argtypes = [C.c_uint16]; L.or_bf16_to_f32.restype = C.c_float
        L.or_f16_to_f32_scalar_asis.argtypes = [C.c_uint16]; L.or_f16_to_f32_scalar_asis.restype = C.c_float
        L.or_f32_to_f16.argtypes = [C.c_float]; L.or_f32_to_f16.restype = C.c_uint16
        L.or_f16_array_to_f32.argtypes = [u16p, f32p, i64]
        L.or_bf16_array_to_f32.argtypes = [u16p, f32p, i64]
        L.or_f32_array_to_f16.argtypes = [f32p, u16p, i64]
        L.or_dequantize_to_f32.argtypes = [u8p, i64, C.c_uint32, i64, f32p]; L.or_dequantize_to_f32.restype = i64
        L.or_packed_bytes.argtypes = [i64]; L.or_packed_bytes.restype = i64
        L.or_n_groups.argtypes = [i64, i64]; L.or_n_groups.restype = i64
        L.or_quantized_bytes.argtypes = [i64, i64]; L.or_quantized_bytes.restype = i64
        L.or_quantize_q4.argtypes = [f32p, i64, i64, f32p, u8p]
        L.or_dequant_weight.argtypes = [f32p, u8p, i64, i64]; L.or_dequant_weight.restype = C.c_float
        L.or_dequant_layer.argtypes = [f32p, u8p, f32p, i64, i64]
        L.or_quantize_q8_0.argtypes = [f32p, i64, u8p]
        L.or_quantize_q4_0.argtypes = [f32p, i64, u8p]
        L.or_gemv_4bit_worker_scalar.argtypes = [f32p, f32p, u8p, f32p, i64, i64, i64, i64]
        L.or_gemv_4bit_into.argtypes = [f32p, f32p, u8p, f32p, i64, i64, i64]
        L.or_gemv_q4_0.argtypes = [f32p, u8p, f32p, i64, i64]
        L.or_gemm_q4_0.argtypes = [f32p, u8p, f32p, i64, i64, i64]
        L.or_gemv_f32.argtypes = [f32p, f32p, f32p, i64, i64]
        L.or_rms_norm_into.argtypes = [f32p, f32p, f32p, i64, C.c_float]
        L.or_sigmoid.argtypes = [C.c_float]; L.or_sigmoid.restype = C.c_float
        L.or_silu.argtypes = [C.c_float]; L.or_silu.restype = C.c_float
        L.or_softmax.argtypes = [f32p, i64]
        L.or_rope_multi.argtypes = [f32p, i64, i64, np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS"), C.c_float]
        L.or_argmax.argtypes = [f32p, i64]; L.or_argmax.restype = C.c_uint32
        L.or_sample.argtypes = [f32p, i64, C.c_float, i64, C.c_float]; L.or_sample.restype = C.c_uint32
        L.or_swiglu_4bit_into.argtypes = [f32p, f32p, f32p, u8p, f32p, u8p, f32p, u8p, i64, i64, i64, f32p, f32p, f32p]
        L.or_model_forward.argtypes = [C.c_void_p, C.c_int32, i64, f32p]; L.or_model_forward.restype = C.c_int
        # AVX-512 as-is restatements (timing only)
        L.or_avx_gemv_4bit_into.argtypes = [f32p, f32p, u8p, f32p, i64, i64, i64, C.c_int]
        L.or_avx_gemv_4bit_worker.argtypes = [f32p, f32p, u8p, f32p, i64, i64, i64]
        L.or_avx_gemm_rows.argtypes = [f32p, f32p, u8p, f32p, i64, i64, i64, C.c_int]
        L.or_avx_dequant_layer.argtypes = [f32p, u8p, f32p, i64]
        L.or_avx_f16_bytes_to_f32.argtypes = [u8p, i64, f32p]; L.or_avx_f16_bytes_to_f32.restype = i64
        L.or_avx_bf16_bytes_to_f32.argtypes = [u8p, i64, f32p]; L.or_avx_bf16_bytes_to_f32.restype = i64
        # DedupCount codec
        u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
        i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
        L.or_dedup_compress.argtypes = [f32p, i64, C.c_int, C.c_int, u16p, u32p, C.POINTER(i64), u16p, u32p,
                                        C.POINTER(i64), C.POINTER(i64), C.POINTER(C.c_float), u16p, u16p, u8p]
        L.or_dedup_compress.restype = C.c_int
        L.or_dedup_decompress_all.argtypes = [u16p, i64, u16p, i64, i64, C.c_int, C.c_int, C.c_float, u16p, i64,
                                              u16p, i64, u8p, i64, f32p]
        L.or_dedup_decompress_all_global.argtypes = [u16p, i64, u16p, i64, i64, C.c_int, C.c_int, C.c_float, u16p,
                                                     i64, u16p, i64, u8p, i64, C.c_int, f32p, i64, u32p, u32p, f32p]
        L.or_dedup_decompress_all_global.restype = C.c_int
        L.or_dedup_global_table_new.argtypes = [C.c_int, i32p, u16p, i64p, u16p, i64p, f32p, u32p, u32p, i64]
        L.or_dedup_global_table_new.restype = i64
        L.or_dedup_build_chunk_remap.argtypes = [u16p, i64, u16p, i64, C.c_int, C.c_int, f32p, i64, u32p, u32p, u16p]
        L.or_dedup_decompress_with_remap.argtypes = [u16p, i64, C.c_int, C.c_int, C.c_float, u16p, i64, u16p, i64,
                                                     u8p, i64, i64, C.c_int, f32p, i64, u32p, u32p, u16p, i64, f32p]
        L.or_dedup_decompress_with_remap.restype = C.c_int
        L.or_ssm_forward.argtypes = [i64, i64, i64, i64, i64, i64, C.c_float] + [f32p] * 13
        L.or_ssm_forward.restype = C.c_int
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# --- conversions -----------------------------------------------------------

def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    bits = _c(bits, np.uint16)
    out = np.empty(bits.shape, np.float32)
    lib().or_f16_array_to_f32(bits.ravel(), out.ravel(), bits.size)
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    bits = _c(bits, np.uint16)
    out = np.empty(bits.shape, np.float32)
    lib().or_bf16_array_to_f32(bits.ravel(), out.ravel(), bits.size)
    return out


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().or_f32_array_to_f16(x.ravel(), out.ravel(), x.size)
    return out


def dequantize_to_f32(raw: np.ndarray, dtype: int, element_count: int) -> np.ndarray | None:
    """GGUFFile::dequantize_to_f32 semantics; None where the reference panics."""
    raw = _c(raw, np.uint8).ravel()
    cap = max(element_count, raw.size // 2 + 1, 1)
    out = np.empty(cap, np.float32)
    k = lib().or_dequantize_to_f32(raw if raw.size else np.zeros(1, np.uint8), raw.size, dtype, element_count, out)
    if k < 0:
        return None
    return out[:k].copy()


# --- engine INT4 format ----------------------------------------------------

def quantize_q4(w: np.ndarray, group_size: int = 32):
    w = _c(w, np.float32).ravel()
    n = w.size
    gs = max(group_size, 1)
    scales = np.empty((n + gs - 1) // gs, np.float32)
    packed = np.empty((n + 1) // 2, np.uint8)
    lib().or_quantize_q4(w if n else np.zeros(1, np.float32), n, group_size,
                         scales if scales.size else np.zeros(1, np.float32),
                         packed if packed.size else np.zeros(1, np.uint8))
    return scales, packed


def dequant_layer(scales, packed, n, group_size=32):
    out = np.empty(n, np.float32)
    lib().or_dequant_layer(_c(scales, np.float32), _c(packed, np.uint8), out, n, group_size)
    return out


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    w = _c(w, np.float32).ravel()
    blocks = np.empty(((w.size + 31) // 32) * 34, np.uint8)
    lib().or_quantize_q8_0(w, w.size, blocks)
    return blocks


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    w = _c(w, np.float32).ravel()
    blocks = np.empty(((w.size + 31) // 32) * 18, np.uint8)
    lib().or_quantize_q4_0(w, w.size, blocks)
    return blocks


# --- GEMV / GEMM -----------------------------------------------------------

def gemv_4bit_into(scales, packed, x, rows, cols, group_size=32) -> np.ndarray:
    out = np.zeros(rows, np.float32)
    x = _c(x, np.float32)
    lib().or_gemv_4bit_into(out, _c(scales, np.float32), _c(packed, np.uint8),
                            x if x.size else np.zeros(1, np.float32), rows, cols, group_size)
    return out


def gemv_4bit_worker_scalar(scales, packed, x, row_start, row_end, cols, group_size=32) -> np.ndarray:
    """inference/math.rs:382-418 on rows [row_start, row_end) of the full planes."""
    out = np.zeros(max(row_end - row_start, 0), np.float32)
    x = _c(x, np.float32)
    lib().or_gemv_4bit_worker_scalar(out if out.size else np.zeros(1, np.float32), _c(scales, np.float32),
                                     _c(packed, np.uint8), x if x.size else np.zeros(1, np.float32),
                                     row_start, row_end, cols, group_size)
    return out


def swiglu_4bit_into(inp, g_s, g_p, u_s, u_p, d_s, d_p, n_embd, n_ff, group_size=32):
    """inference/ffn.rs:155-174 -> (out, scratch_gate, scratch_up, scratch_act)."""
    out = np.zeros(max(n_embd, 1), np.float32)
    sg, su, sa = (np.zeros(max(n_ff, 1), np.float32) for _ in range(3))
    lib().or_swiglu_4bit_into(out, _c(inp, np.float32), _c(g_s, np.float32), _c(g_p, np.uint8), _c(u_s, np.float32),
                              _c(u_p, np.uint8), _c(d_s, np.float32), _c(d_p, np.uint8), n_embd, n_ff, group_size,
                              sg, su, sa)
    return out[:n_embd], sg[:n_ff], su[:n_ff], sa[:n_ff]


def gemv_q4_0(blocks, x, rows, cols) -> np.ndarray:
    out = np.empty(rows, np.float32)
    lib().or_gemv_q4_0(out, _c(blocks, np.uint8), _c(x, np.float32), rows, cols)
    return out


def gemm_q4_0(blocks, a, n) -> np.ndarray:
    a = _c(a, np.float32)
    m, k = a.shape
    out = np.empty((m, n), np.float32)
    lib().or_gemm_q4_0(out, _c(blocks, np.uint8), a, m, n, k)
    return out


def rms_norm(x, w, eps):
    x = _c(x, np.float32)
    out = np.empty_like(x)
    lib().or_rms_norm_into(out, x, _c(w, np.float32), x.size, eps)
    return out


def rope_head(x, pos, freq_base, sections=None):
    x = _c(x, np.float32).copy()
    if sections is None:
        sections = np.array([x.size // 2, 0, 0, 0], np.int32)
    lib().or_rope_multi(x, x.size, pos, _c(sections, np.int32), freq_base)
    return x


def sample(logits, temperature: float, top_k: int, r: float) -> int:
    """inference/sampling.rs:17-64 with the uniform draw r given."""
    logits = _c(logits, np.float32)
    return int(lib().or_sample(logits, logits.size, float(temperature), int(top_k), float(r)))


def sample_uniform(seed: int, step: int, seq: int) -> float:
    """The device sampler's draw for (seed, step, sequence): 24 bits of a
    splitmix64-style hash, mapped to [0, 1) as the reference maps its draw."""
    M = (1 << 64) - 1

    def mix(x):
        x = (x + 0x9E3779B97F4A7C15) & M
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M
        return x ^ (x >> 31)

    x = mix((seed ^ mix((step * 0x100000001B3 + seq) & M)) & M)
    return float(np.float32(x & 0xFFFFFF) / np.float32(16777216.0))


def argmax(logits) -> int:
    logits = _c(logits, np.float32)
    return int(lib().or_argmax(logits, logits.size))


def silu(v: float) -> float:
    return float(lib().or_silu(v))


# --- DedupCount codec (models/dedup/) ----------------------------------------

class DedupTensor:
    """DedupCountTensor's decode-relevant fields (dedup/tensor.rs:4-13):
    prefixes (u16), unique tail values (u16) and counts, count, prefix_digits,
    tail_digits, avg_precision_lost."""

    def __init__(self, prefixes, tail_values, count, prefix_digits, tail_digits, avg_precision_lost,
                 prefix_counts=None, tail_counts=None):
        self.prefixes = np.ascontiguousarray(prefixes, np.uint16)
        self.tail_values = np.ascontiguousarray(tail_values, np.uint16)
        self.count = int(count)
        self.prefix_digits = int(prefix_digits)
        self.tail_digits = int(tail_digits)
        self.avg_precision_lost = float(np.float32(avg_precision_lost))
        self.prefix_counts = prefix_counts
        self.tail_counts = tail_counts


class Sandbag:
    """Per-element indices (dedup/types.rs:14-21): prefix_idx, tail_idx (u16),
    sign_bits (one bit per element, LSB first) and count."""

    def __init__(self, prefix_idx, tail_idx, sign_bits, count):
        self.prefix_idx = np.ascontiguousarray(prefix_idx, np.uint16)
        self.tail_idx = np.ascontiguousarray(tail_idx, np.uint16)
        self.sign_bits = np.ascontiguousarray(sign_bits, np.uint8)
        self.count = int(count)


class GlobalTable:
    """dedup/types.rs:23-28: prefix_digits, f32 prefixes and tails_for_prefix
    (CSR: tail_off[n + 1], tails)."""

    def __init__(self, prefix_digits, prefixes, tail_off, tails):
        self.prefix_digits = int(prefix_digits)
        self.prefixes = np.ascontiguousarray(prefixes, np.float32)
        self.tail_off = np.ascontiguousarray(tail_off, np.uint32)
        self.tails = np.ascontiguousarray(tails, np.uint32)

    def row(self, gi):
        return self.tails[self.tail_off[gi]:self.tail_off[gi + 1]]


def _arr(a, dt):
    a = np.ascontiguousarray(a, dt)
    return a if a.size else np.zeros(1, dt)


def dedup_compress(w, prefix_digits: int, truncate_rounds: int):
    """DedupCountTensor::compress (compressor.rs:8-160, scalar tail path)."""
    w = _c(w, np.float32)
    n = w.size
    pre = np.zeros(65536, np.uint16); pc = np.zeros(65536, np.uint32)
    tv = np.zeros(65536, np.uint16); tc = np.zeros(65536, np.uint32)
    pidx = np.zeros(max(n, 1), np.uint16); tidx = np.zeros(max(n, 1), np.uint16)
    signs = np.zeros(max((n + 7) // 8, 1), np.uint8)
    np_, nt, td = i64(), i64(), i64()
    avg = C.c_float()
    rc = lib().or_dedup_compress(_arr(w, np.float32), n, prefix_digits, truncate_rounds, pre, pc, C.byref(np_), tv, tc,
                                 C.byref(nt), C.byref(td), C.byref(avg), pidx, tidx, signs)
    if rc != 0:
        raise MemoryError("oracle compress")
    t = DedupTensor(pre[:np_.value].copy(), tv[:nt.value].copy(), n, prefix_digits, td.value, avg.value,
                    pc[:np_.value].copy(), tc[:nt.value].copy())
    return t, Sandbag(pidx[:n].copy(), tidx[:n].copy(), signs[:(n + 7) // 8].copy(), n)


def dedup_decompress_all(t: DedupTensor, s: Sandbag) -> np.ndarray:
    """DedupCountTensor::decompress_all (decompressor.rs:7-27)."""
    out = np.empty(max(t.count, 1), np.float32)
    lib().or_dedup_decompress_all(_arr(t.prefixes, np.uint16), t.prefixes.size, _arr(t.tail_values, np.uint16),
                                  t.tail_values.size, t.count, t.prefix_digits, t.tail_digits, t.avg_precision_lost,
                                  _arr(s.prefix_idx, np.uint16), s.prefix_idx.size, _arr(s.tail_idx, np.uint16),
                                  s.tail_idx.size, _arr(s.sign_bits, np.uint8), s.sign_bits.size, out)
    return out[:t.count]


def dedup_decompress_all_global(t: DedupTensor, s: Sandbag, g: GlobalTable) -> np.ndarray:
    """DedupCountTensor::decompress_all_global (decompressor.rs:29-85); raises
    where the reference panics."""
    out = np.empty(max(t.count, 1), np.float32)
    rc = lib().or_dedup_decompress_all_global(
        _arr(t.prefixes, np.uint16), t.prefixes.size, _arr(t.tail_values, np.uint16), t.tail_values.size, t.count,
        t.prefix_digits, t.tail_digits, t.avg_precision_lost, _arr(s.prefix_idx, np.uint16), s.prefix_idx.size,
        _arr(s.tail_idx, np.uint16), s.tail_idx.size, _arr(s.sign_bits, np.uint8), s.sign_bits.size, g.prefix_digits,
        _arr(g.prefixes, np.float32), g.prefixes.size, _arr(g.tail_off, np.uint32), _arr(g.tails, np.uint32), out)
    if rc != 0:
        raise IndexError("decompress_all_global: index out of range (the reference panics)")
    return out[:t.count]


def dedup_global_table_new(chunks) -> GlobalTable:
    """GlobalTable::new (global_lookup.rs:7-59)."""
    n = len(chunks)
    if n == 0:
        return GlobalTable(0, np.zeros(0, np.float32), np.zeros(1, np.uint32), np.zeros(0, np.uint32))
    pd = np.array([c.prefix_digits for c in chunks], np.int32)
    npre = np.array([c.prefixes.size for c in chunks], np.int64)
    ntl = np.array([c.tail_values.size for c in chunks], np.int64)
    pre = _arr(np.concatenate([c.prefixes for c in chunks]), np.uint16)
    tl = _arr(np.concatenate([c.tail_values for c in chunks]), np.uint16)
    cap = int(max(1, ntl.sum() * max(1, npre.sum())))
    gp = np.zeros(65536, np.float32); off = np.zeros(65537, np.uint32); tails = np.zeros(min(cap, 1 << 26), np.uint32)
    ng = lib().or_dedup_global_table_new(n, pd, pre, npre, tl, ntl, gp, off, tails, tails.size)
    if ng < 0:
        raise MemoryError("global table capacity")
    return GlobalTable(int(pd[0]), gp[:ng].copy(), off[:ng + 1].copy(), tails[:off[ng]].copy())


def dedup_build_chunk_remap(g: GlobalTable, t: DedupTensor) -> np.ndarray:
    """GlobalTable::build_chunk_remap (global_lookup.rs:62-86)."""
    out = np.zeros(max(t.tail_values.size, 1), np.uint16)
    lib().or_dedup_build_chunk_remap(_arr(t.prefixes, np.uint16), t.prefixes.size, _arr(t.tail_values, np.uint16),
                                     t.tail_values.size, t.prefix_digits, g.prefix_digits,
                                     _arr(g.prefixes, np.float32), g.prefixes.size, _arr(g.tail_off, np.uint32),
                                     _arr(g.tails, np.uint32), out)
    return out[:t.tail_values.size]


def dedup_decompress_with_remap(g: GlobalTable, s: Sandbag, t: DedupTensor, remap) -> np.ndarray:
    """GlobalTable::decompress_with_remap with a remap (global_lookup.rs:89-113);
    raises where the reference panics."""
    remap = np.ascontiguousarray(remap, np.uint16)
    out = np.empty(max(s.count, 1), np.float32)
    rc = lib().or_dedup_decompress_with_remap(
        _arr(t.prefixes, np.uint16), t.prefixes.size, t.prefix_digits, t.tail_digits, t.avg_precision_lost,
        _arr(s.prefix_idx, np.uint16), s.prefix_idx.size, _arr(s.tail_idx, np.uint16), s.tail_idx.size,
        _arr(s.sign_bits, np.uint8), s.sign_bits.size, s.count, g.prefix_digits, _arr(g.prefixes, np.float32),
        g.prefixes.size, _arr(g.tail_off, np.uint32), _arr(g.tails, np.uint32), _arr(remap, np.uint16), remap.size,
        out)
    if rc != 0:
        raise IndexError("decompress_with_remap: index out of range (the reference panics)")
    return out[:s.count]


# --- gated delta-net SSM block (inference/ssm.rs) ------------------------------

SSM_WEIGHTS = ("wqkv", "wqkv_gate", "conv1d", "dt_bias", "a", "alpha", "beta", "norm", "out")


def ssm_forward(cfg: dict, w: dict, conv_state: np.ndarray, ssm_state: np.ndarray, x) -> np.ndarray:
    """SsmBlock::forward (ssm.rs:171-296) for one token; conv_state and
    ssm_state (float32 arrays) are updated in place."""
    out = np.empty(cfg["n_embd"], np.float32)
    rc = lib().or_ssm_forward(cfg["n_embd"], cfg["d_state"], cfg["n_group"], cfg["dt_rank"], cfg["d_inner"],
                              cfg["d_conv"], cfg["eps"], *[_c(w[k], np.float32) for k in SSM_WEIGHTS],
                              conv_state, ssm_state, _c(x, np.float32), out)
    if rc != 0:
        raise ValueError("ssm_forward: head_k_dim != head_v_dim (the reference asserts)")
    return out


# --- decoder ----------------------------------------------------------------

class _OrModel(C.Structure):
    _fields_ = [
        ("n_layer", i64), ("n_embd", i64), ("n_ff", i64), ("n_head", i64), ("n_head_kv", i64),
        ("head_dim", i64), ("vocab", i64), ("max_seq", i64),
        ("rope_base", C.c_float), ("eps", C.c_float),
        ("tok_embd", C.c_void_p), ("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("out_norm", C.c_void_p),
        ("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p),
        ("wg", C.c_void_p), ("wu", C.c_void_p), ("wd", C.c_void_p),
        ("lm_head", C.c_void_p), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p),
        ("k_cache_f32", C.c_void_p), ("v_cache_f32", C.c_void_p), ("engine", i64),
    ]


class OracleModel:
    """Host-side decoder oracle over Q4_0 blocks (inference/mod.rs:333-545).

    `weights` is a dict with numpy arrays: tok_embd/attn_norm/ffn_norm/out_norm
    (uint16 f16 bits) and per-layer lists wq..wd plus lm_head: uint8 Q4_0
    blocks, or with engine=True quantize()'s output as one uint8 blob per
    matrix (f32 scales [rows*cols/32] then packed [rows*cols/2]).
    """

    def __init__(self, cfg: dict, weights: dict, max_seq: int, engine: bool = False):
        self.cfg = cfg
        self._keep = []
        L = cfg["n_layer"]

        def ptr(a):
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            return a.ctypes.data

        def ptrs(lst):
            arr = (C.c_void_p * L)(*[ptr(a) for a in lst])
            self._keep.append(arr)
            return C.cast(arr, C.c_void_p).value

        hd = cfg["head_dim"]
        self.k_cache = np.zeros((L, cfg["n_head_kv"], max_seq, hd), np.uint16)
        self.v_cache = np.zeros_like(self.k_cache)
        self.k_cache_f32 = np.zeros(self.k_cache.shape, np.float32)
        self.v_cache_f32 = np.zeros(self.k_cache.shape, np.float32)
        self.m = _OrModel(L, cfg["n_embd"], cfg["n_ff"], cfg["n_head"], cfg["n_head_kv"], hd, cfg["vocab"], max_seq,
                          cfg["rope_base"], cfg["eps"],
                          ptr(weights["tok_embd"]), ptr(weights["attn_norm"]), ptr(weights["ffn_norm"]),
                          ptr(weights["out_norm"]),
                          ptrs(weights["wq"]), ptrs(weights["wk"]), ptrs(weights["wv"]), ptrs(weights["wo"]),
                          ptrs(weights["wg"]), ptrs(weights["wu"]), ptrs(weights["wd"]),
                          ptr(weights["lm_head"]), self.k_cache.ctypes.data, self.v_cache.ctypes.data,
                          self.k_cache_f32.ctypes.data, self.v_cache_f32.ctypes.data, 1 if engine else 0)

    def forward(self, token: int, pos: int) -> np.ndarray:
        logits = np.empty(self.cfg["vocab"], np.float32)
        rc = lib().or_model_forward(C.addressof(self.m), token, pos, logits)
        if rc != 0:
            raise ValueError("oracle forward rejected token/pos")
        return logits


# --- AVX-512 as-is (timing) -------------------------------------------------

def avx_gemv_4bit_into(out, scales, packed, x, rows, cols, nthreads):
    lib().or_avx_gemv_4bit_into(out, scales, packed, x, rows, cols, 32, nthreads)


def avx_f16_bytes_to_f32(src_u8, out):
    return lib().or_avx_f16_bytes_to_f32(src_u8, src_u8.size, out)
