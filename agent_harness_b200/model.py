"""Llama-shaped decoder on the C ABI (ah_model_*): the B200 counterpart of
agent_harness's InferenceEngine (inference/mod.rs) for Q4_0 weights."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import call, lib

# tensor kinds (include/ah_cuda.h)
TOK_EMBD, ATTN_NORM, FFN_NORM, OUT_NORM, WQ, WK, WV, WO, WGATE, WUP, WDOWN, LM_HEAD = range(12)


class _Cfg(C.Structure):
    _fields_ = [("n_layer", C.c_int32), ("n_embd", C.c_int32), ("n_ff", C.c_int32), ("n_head", C.c_int32),
                ("n_head_kv", C.c_int32), ("head_dim", C.c_int32), ("vocab_size", C.c_int32),
                ("max_seq", C.c_int32), ("max_batch", C.c_int32), ("rope_freq_base", C.c_float),
                ("rms_eps", C.c_float)]


@dataclass
class ModelConfig:
    """inference/config.rs:6-58 (the fields the decoder uses)."""
    n_layer: int
    n_embd: int
    n_ff: int
    n_head: int
    n_head_kv: int
    head_dim: int
    vocab_size: int
    max_seq: int = 4096
    max_batch: int = 1
    rope_freq_base: float = 500000.0
    rms_eps: float = 1e-5

    def to_c(self) -> _Cfg:
        return _Cfg(self.n_layer, self.n_embd, self.n_ff, self.n_head, self.n_head_kv, self.head_dim,
                    self.vocab_size, self.max_seq, self.max_batch, self.rope_freq_base, self.rms_eps)

    def shapes(self) -> dict:
        dq, dkv = self.n_head * self.head_dim, self.n_head_kv * self.head_dim
        return {WQ: (dq, self.n_embd), WK: (dkv, self.n_embd), WV: (dkv, self.n_embd), WO: (self.n_embd, dq),
                WGATE: (self.n_ff, self.n_embd), WUP: (self.n_ff, self.n_embd), WDOWN: (self.n_embd, self.n_ff),
                LM_HEAD: (self.vocab_size, self.n_embd)}


LLAMA_8B = ModelConfig(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128,
                       vocab_size=128256, max_seq=2304, max_batch=1, rope_freq_base=500000.0, rms_eps=1e-5)
LLAMA_70B = ModelConfig(n_layer=80, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, head_dim=128,
                        vocab_size=128256, max_seq=2176, max_batch=16, rope_freq_base=500000.0, rms_eps=1e-5)


def tensor_seed(seed: int, kind: int, layer: int) -> int:
    return int(lib().ah_model_tensor_seed(C.c_uint64(seed), kind, layer))


def nccl_unique_id() -> bytes:
    """A fresh NCCL id (128 bytes) for ah_model_create_tp; make it on one rank
    and share it (e.g. torch.distributed.broadcast_object_list)."""
    buf = C.create_string_buffer(128)
    call("ah_nccl_unique_id", buf, 128)
    return buf.raw


def shard_rows(cfg: ModelConfig, rank: int, world: int) -> dict:
    """Rows / columns of each full tensor that tensor-parallel rank `rank`
    holds: {kind: (row0, rows, col0, cols)} (row split for q, k, v, gate, up
    and the LM head; column split for o and down)."""
    dq, dkv = cfg.n_head * cfg.head_dim // world, cfg.n_head_kv * cfg.head_dim // world
    nff, nv, d = cfg.n_ff // world, cfg.vocab_size // world, cfg.n_embd
    return {WQ: (rank * dq, dq, 0, d), WK: (rank * dkv, dkv, 0, d), WV: (rank * dkv, dkv, 0, d),
            WO: (0, d, rank * dq, dq), WGATE: (rank * nff, nff, 0, d), WUP: (rank * nff, nff, 0, d),
            WDOWN: (0, d, rank * nff, nff), LM_HEAD: (rank * nv, nv, 0, d)}


class Model:
    """The decoder on one GPU, or rank `tp_rank` of a `tp_world`-way
    tensor-parallel group (pass the group's NCCL id from nccl_unique_id)."""

    def __init__(self, cfg: ModelConfig, device="cuda", tp_rank: int = 0, tp_world: int = 1,
                 nccl_id: bytes | None = None):
        self.cfg = cfg
        dev = torch.device(device)
        self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        torch.cuda.set_device(self.device)
        self._h = C.c_void_p()
        c = cfg.to_c()
        self.tp_rank, self.tp_world = tp_rank, tp_world
        if tp_world == 1:
            call("ah_model_create", C.byref(c), C.byref(self._h))
        else:
            if nccl_id is None or len(nccl_id) < 128:
                raise ValueError("tensor parallelism needs the group's 128-byte NCCL id")
            idb = C.create_string_buffer(bytes(nccl_id[:128]), 128)
            call("ah_model_create_tp", C.byref(c), tp_rank, tp_world, idb, C.byref(self._h))
        self.vocab_local = cfg.vocab_size // tp_world

    def enable_peer_allreduce(self, allgather):
        """Switch the block all-reduce from NCCL to stores into the other ranks'
        memory over NVLink.  `allgather(bytes) -> [bytes per rank]` shares this
        rank's 64-byte IPC handle (e.g. torch.distributed.all_gather_object)."""
        h = C.create_string_buffer(64)
        call("ah_model_ipc_handle", self._h, h, 64)
        hs = allgather(h.raw)
        buf = C.create_string_buffer(b"".join(bytes(x) for x in hs), 64 * len(hs))
        call("ah_model_ipc_open", self._h, buf, 64 * len(hs))

    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def init_random(self, seed: int, w_std=0.02, emb_std=1.0, norm_std=0.02):
        call("ah_model_init_random", self._h, C.c_uint64(seed), w_std, emb_std, norm_std)
        torch.cuda.synchronize(self.device)

    def load_tensor(self, kind: int, layer: int, data: torch.Tensor):
        call("ah_model_load_tensor", self._h, kind, layer, C.c_void_p(data.data_ptr()), self._stream())

    def load_tensor_engine(self, kind: int, layer: int, scales: torch.Tensor, packed: torch.Tensor):
        """A projection in quantize()'s engine format (f32 group-32 scales, packed nibbles)."""
        call("ah_model_load_tensor_engine", self._h, kind, layer, C.c_void_p(scales.data_ptr()),
             C.c_void_p(packed.data_ptr()), self._stream())

    def load_tensor_f32(self, kind: int, layer: int, data: torch.Tensor):
        """An f32 tensor: projections are quantized on the device (engine format),
        embeddings and norms stored as f16."""
        assert data.dtype == torch.float32 and data.is_cuda and data.is_contiguous()
        call("ah_model_load_tensor_f32", self._h, kind, layer, C.c_void_p(data.data_ptr()), self._stream())

    def reset(self, batch: int = 1):
        call("ah_model_reset", self._h, batch, self._stream())

    def forward(self, tokens) -> torch.Tensor:
        """One forward() per sequence; returns logits [batch][vocab] (this
        rank's vocab slice [batch][vocab/world] under tensor parallelism)."""
        t = torch.as_tensor(np.asarray(tokens, np.int32)).to(self.device)
        out = torch.empty(t.numel(), self.vocab_local, dtype=torch.float32, device=self.device)
        call("ah_model_forward", self._h, C.c_void_p(t.data_ptr()), C.c_void_p(out.data_ptr()), self._stream())
        return out

    def decode(self, n: int, batch: int) -> torch.Tensor:
        out = torch.empty(n, batch, dtype=torch.int32, device=self.device)
        call("ah_model_decode", self._h, n, C.c_void_p(out.data_ptr()), self._stream())
        return out

    def generate(self, prompt: np.ndarray, n_new: int) -> np.ndarray:
        """Greedy generate for prompt [batch][n_prompt]; returns [n_new][batch]."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        batch, n_prompt = p.shape
        out = np.zeros((n_new, batch), np.int32)
        call("ah_model_generate", self._h, p.ctypes.data_as(C.c_void_p), batch, n_prompt, n_new,
             out.ctypes.data_as(C.c_void_p), self._stream())
        return out

    def set_prefill(self, mode: int):
        """1 (default): long prompts through the prefill GEMMs; 0: one forward()
        per prompt token, as the reference (inference/mod.rs:550)."""
        call("ah_model_set_prefill", self._h, mode)

    def set_batched_gemv(self, min_batch: int):
        """Decode steps of at least min_batch sequences (default 9) run each
        projection on the tcgen05 batched GEMV where it is the faster one
        (large enough weights for the batch); 1: every projection, 17: never."""
        call("ah_model_set_batched_gemv", self._h, min_batch)

    def set_sampling(self, temperature: float, top_k: int = 40, seed: int = 0):
        """Next-token choice of generate/decode: temperature 0 is greedy
        (sampling.rs:4-14); above 0 temperature + top-k sampling
        (inference/mod.rs:552-553, sampling.rs:17-64) with the draw of
        sequence b at position p = kernels.sample_uniform(seed, p, b)."""
        call("ah_model_set_sampling", self._h, temperature, top_k, seed)

    @property
    def position(self) -> int:
        v = C.c_int(0)
        call("ah_model_position", self._h, C.byref(v))
        return v.value

    def close(self):
        if self._h:
            lib().ah_model_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
