"""DedupCount weight decoding on the GPU, with the reference's types and
method names (src/models/dedup/):

    DedupCountTensor.decompress_all(sandbag)            decompressor.rs:7-27
    DedupCountTensor.decompress_all_global(sandbag, g)  decompressor.rs:29-85
    GlobalTable.decompress_with_remap(sandbag, t, m)    global_lookup.rs:89-118

each returning a float32 device tensor, plus the load path the reference runs
per tensor in inference/mod.rs:255-271 (decompress, quantise with group 32),
fused into one kernel that yields a resident GEMV weight:

    DedupCountTensor.to_q4weight(sandbag, rows, cols, global_table=None, remap=None)

Sandbag arrays may be numpy arrays (uploaded) or device tensors.  There is no
CPU path: the CUDA library must be loaded.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .kernels import Q4Weight, _ptr, _stream

call = _lib.call


def _dev(a, dtype: torch.dtype, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        assert a.dtype == dtype, f"expected {dtype}, got {a.dtype}"
        return a.to(device).contiguous()
    return torch.as_tensor(np.ascontiguousarray(a)).to(dtype=dtype, device=device)


def _np(a, dtype) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.cpu().numpy()
    a = np.ascontiguousarray(a, dtype)
    return a if a.size else np.zeros(1, dtype)


class Sandbag:
    """Per-element indices (dedup/types.rs:14-21): prefix_idx and tail_idx
    (u16), sign_bits (one bit per element, LSB first) and count."""

    def __init__(self, prefix_idx, tail_idx, sign_bits, count: int):
        self.prefix_idx, self.tail_idx, self.sign_bits, self.count = prefix_idx, tail_idx, sign_bits, int(count)

    def on(self, device):
        """(prefix_idx, tail_idx, sign_bits) as device tensors (int16 / uint8 bit patterns)."""
        p = _dev(np.asarray(self.prefix_idx, np.uint16).view(np.int16) if not isinstance(self.prefix_idx, torch.Tensor)
                 else self.prefix_idx, torch.int16, device)
        t = _dev(np.asarray(self.tail_idx, np.uint16).view(np.int16) if not isinstance(self.tail_idx, torch.Tensor)
                 else self.tail_idx, torch.int16, device)
        s = _dev(self.sign_bits, torch.uint8, device)
        return p, t, s


class GlobalTable:
    """dedup/types.rs:23-28: prefix_digits, f32 prefixes and tails_for_prefix
    (a list of u32 lists, held in CSR form)."""

    def __init__(self, prefix_digits: int, prefixes, tails_for_prefix):
        self.prefix_digits = int(prefix_digits)
        self.prefixes = np.ascontiguousarray(prefixes, np.float32)
        rows = [np.asarray(r, np.uint32) for r in tails_for_prefix]
        self.tail_off = np.zeros(len(rows) + 1, np.uint32)
        self.tail_off[1:] = np.cumsum([r.size for r in rows]) if rows else []
        self.tails = np.concatenate(rows).astype(np.uint32) if rows else np.zeros(0, np.uint32)

    def decompress_with_remap(self, sandbag: Sandbag, tensor: "DedupCountTensor", remap=None, device="cuda"):
        """global_lookup.rs:89-118; without a remap this is tensor.decompress_all."""
        if remap is None:
            return tensor.decompress_all(sandbag, device)
        table = tensor._table_remap(self, remap)
        try:
            return tensor._decompress(table, sandbag, sandbag.count, device)
        finally:
            call("ah_dedup_table_destroy", table)


class DedupCountTensor:
    """The decode-relevant fields of dedup/tensor.rs:4-13: prefixes (u16),
    unique tail values (u16), count, prefix_digits, tail_digits and
    avg_precision_lost."""

    def __init__(self, prefixes, unique_tails, count: int, prefix_digits: int, tail_digits: int,
                 avg_precision_lost: float):
        self.prefixes = np.ascontiguousarray(prefixes, np.uint16)
        self.unique_tails = np.ascontiguousarray(unique_tails, np.uint16)
        self.count, self.prefix_digits, self.tail_digits = int(count), int(prefix_digits), int(tail_digits)
        self.avg_precision_lost = float(np.float32(avg_precision_lost))

    # -- decode tables (the reference's per-tensor lookups, flattened) --
    def _host_arrays(self):
        return _np(self.prefixes, np.uint16), _np(self.unique_tails, np.uint16)

    def _table_local(self):
        pre, tl = self._host_arrays()
        h = C.c_void_p()
        call("ah_dedup_table_local", pre.ctypes.data, self.prefixes.size, tl.ctypes.data, self.unique_tails.size,
             self.prefix_digits, self.tail_digits, self.avg_precision_lost, C.byref(h))
        return h

    def _table_global(self, g: GlobalTable):
        pre, tl = self._host_arrays()
        gp, go, gt = _np(g.prefixes, np.float32), _np(g.tail_off, np.uint32), _np(g.tails, np.uint32)
        h = C.c_void_p()
        call("ah_dedup_table_global", pre.ctypes.data, self.prefixes.size, tl.ctypes.data, self.unique_tails.size,
             self.prefix_digits, self.tail_digits, self.avg_precision_lost, g.prefix_digits, gp.ctypes.data,
             g.prefixes.size, go.ctypes.data, gt.ctypes.data, C.byref(h))
        return h

    def _table_remap(self, g: GlobalTable, remap):
        pre, _ = self._host_arrays()
        gp, go, gt = _np(g.prefixes, np.float32), _np(g.tail_off, np.uint32), _np(g.tails, np.uint32)
        rm = np.ascontiguousarray(remap, np.uint16)
        rmp = _np(rm, np.uint16)
        h = C.c_void_p()
        call("ah_dedup_table_remap", pre.ctypes.data, self.prefixes.size, self.prefix_digits, self.tail_digits,
             self.avg_precision_lost, g.prefix_digits, gp.ctypes.data, g.prefixes.size, go.ctypes.data,
             gt.ctypes.data, rmp.ctypes.data, rm.size, C.byref(h))
        return h

    def _decompress(self, table, sandbag: Sandbag, count: int, device) -> torch.Tensor:
        device = torch.device(device)
        p, t, s = sandbag.on(device)
        out = torch.empty(count, dtype=torch.float32, device=device)
        call("ah_dedup_decompress_f32", table, _ptr(p), p.numel(), _ptr(t), t.numel(), _ptr(s), s.numel(), count,
             _ptr(out), _stream(device))
        return out

    # -- the reference's methods --
    def decompress_all(self, sandbag: Sandbag, device="cuda") -> torch.Tensor:
        """decompressor.rs:7-27 (count = self.count)."""
        table = self._table_local()
        try:
            return self._decompress(table, sandbag, self.count, device)
        finally:
            call("ah_dedup_table_destroy", table)

    def decompress_all_global(self, sandbag: Sandbag, global_table: GlobalTable, device="cuda") -> torch.Tensor:
        """decompressor.rs:29-85 (count = self.count)."""
        table = self._table_global(global_table)
        try:
            return self._decompress(table, sandbag, self.count, device)
        finally:
            call("ah_dedup_table_destroy", table)

    def to_q4weight(self, sandbag: Sandbag, rows: int, cols: int, global_table: GlobalTable | None = None,
                    remap=None, device="cuda") -> Q4Weight:
        """Decode (local, global or remapped tables, as the loader chooses at
        convert/loader.rs:223-225) and quantise with group 32 into a resident
        engine-format weight, in one pass on the device."""
        if global_table is None:
            table = self._table_local()
        elif remap is None:
            table = self._table_global(global_table)
        else:
            table = self._table_remap(global_table, remap)
        device = torch.device(device)
        try:
            p, t, s = sandbag.on(device)
            h = C.c_void_p()
            call("ah_dedup_to_q4w", table, _ptr(p), p.numel(), _ptr(t), t.numel(), _ptr(s), s.numel(), rows, cols,
                 C.byref(h), _stream(device))
            return Q4Weight(h, rows, cols, device)
        finally:
            call("ah_dedup_table_destroy", table)
