"""The gated delta-net SSM block on the GPU, mirroring inference/ssm.rs:
SsmBlock (weights), SsmState (conv window and per-head state, zero at start,
as SsmState::new) and SsmBlock.forward(input, state) for one token.  There is
no CPU path: the CUDA library must be loaded."""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .kernels import _ptr, _stream

call = _lib.call
WEIGHTS = ("wqkv", "wqkv_gate", "conv1d", "dt_bias", "a", "alpha", "beta", "norm", "out")


class _Cfg(C.Structure):
    _fields_ = [("n_embd", C.c_int32), ("d_state", C.c_int32), ("n_group", C.c_int32), ("dt_rank", C.c_int32),
                ("d_inner", C.c_int32), ("d_conv", C.c_int32), ("rms_eps", C.c_float)]


class _W(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in WEIGHTS]


class SsmState:
    """conv_state [(d_conv - 1)][conv_dim] and ssm_state [dt_rank][d_state][d_state], f32, zero-initialised."""

    def __init__(self, cfg: dict, device="cuda"):
        conv_dim = 2 * cfg["n_group"] * cfg["d_state"] + cfg["d_inner"]
        self.conv_state = torch.zeros(max(cfg["d_conv"] - 1, 1), conv_dim, dtype=torch.float32, device=device)
        self.ssm_state = torch.zeros(cfg["dt_rank"], cfg["d_state"], cfg["d_state"], dtype=torch.float32,
                                     device=device)


class SsmBlock:
    """Weights as device f32 tensors in the reference's row-major shapes
    (wqkv [conv_dim][n_embd], wqkv_gate [d_inner][n_embd], conv1d
    [conv_dim][d_conv], dt_bias / a [dt_rank], alpha / beta [dt_rank][n_embd],
    norm [d_state], out [n_embd][d_inner])."""

    def __init__(self, cfg: dict, weights: dict, device="cuda"):
        self.cfg = dict(cfg)
        self.device = torch.device(device)
        self.w = {k: torch.as_tensor(weights[k], dtype=torch.float32).to(self.device).contiguous() for k in WEIGHTS}
        self._c = _Cfg(cfg["n_embd"], cfg["d_state"], cfg["n_group"], cfg["dt_rank"], cfg["d_inner"], cfg["d_conv"],
                       cfg["eps"])
        self._w = _W(*[self.w[k].data_ptr() for k in WEIGHTS])
        n = C.c_size_t()
        call("ah_ssm_workspace_bytes", C.byref(self._c), C.byref(n))
        self._ws = torch.empty((n.value + 3) // 4, dtype=torch.float32, device=self.device)

    def new_state(self) -> SsmState:
        return SsmState(self.cfg, self.device)

    def forward(self, x: torch.Tensor, state: SsmState, out: torch.Tensor | None = None) -> torch.Tensor:
        """ssm.rs:171-296: one token x [n_embd] -> [n_embd]; the state advances in place."""
        x = x.to(self.device, torch.float32).contiguous()
        if out is None:
            out = torch.empty(self.cfg["n_embd"], dtype=torch.float32, device=self.device)
        call("ah_ssm_forward", C.byref(self._c), C.byref(self._w), _ptr(state.conv_state), _ptr(state.ssm_state),
             _ptr(x), _ptr(out), _ptr(self._ws), self._ws.numel() * 4, _stream(self.device))
        return out
