"""Transition bridges ``out = x + MLP(RMSNorm(x))`` (API of
ssd/models/bridges.py:27-135).

Parameter names and shapes match the reference (``norm.weight``,
``mlp.body.{0,2}``, ``mlp.out_proj`` or ``mlp.{gate,up,out}_proj``), so its
``stage*.pt`` / ``online.pt`` checkpoints load unchanged. The forward runs on
the device through the GEMM kernels (RMSNorm -> in-projection + bias +
activation -> out-projection + bias + residual); there is no CPU path.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from ssd.config import BridgeConfig

ACTIVATIONS = ("silu", "gelu", "relu")


class RMSNorm(nn.Module):
    """Parameter holder for the bridge norm (bridges.py:27-37)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))


class _PlainMLP(nn.Module):
    """Linear/act stack then out_proj (bridges.py:40-54)."""

    def __init__(self, d_model: int, hidden: int, num_layers: int, activation: str, bias: bool):
        super().__init__()
        if num_layers not in (2, 3):
            raise ValueError(f"mlp bridge supports 2 or 3 layers, got {num_layers}")
        dims = [d_model] + [hidden] * (num_layers - 1)
        layers: list[nn.Module] = []
        for i in range(num_layers - 1):
            layers += [nn.Linear(dims[i], dims[i + 1], bias=bias), _Act(activation)]
        self.body = nn.Sequential(*layers)
        self.out_proj = nn.Linear(hidden, d_model, bias=bias)

    def linears(self) -> list[nn.Linear]:
        return [m for m in self.body if isinstance(m, nn.Linear)]


class _SwiGLU(nn.Module):
    """gate/up + SiLU-gated product + out_proj (bridges.py:57-65)."""

    def __init__(self, d_model: int, hidden: int, bias: bool):
        super().__init__()
        self.gate_proj = nn.Linear(d_model, hidden, bias=bias)
        self.up_proj = nn.Linear(d_model, hidden, bias=bias)
        self.out_proj = nn.Linear(hidden, d_model, bias=bias)


class _Act(nn.Module):
    """Parameter-free activation marker (keeps the reference's body indices)."""

    def __init__(self, name: str):
        super().__init__()
        self.name = name


class TransitionBridge(nn.Module):
    """Residual MLP bridge ``out = x + MLP(RMSNorm(x))`` (bridges.py:68-135)."""

    def __init__(self, d_model: int, hidden_dim: Optional[int] = None, num_layers: int = 2, mlp_type: str = "mlp",
                 activation: str = "silu", bias: bool = True, init_std: float = 1e-3, norm_eps: float = 1e-5,
                 dtype: torch.dtype = torch.float32):
        super().__init__()
        hidden = hidden_dim or d_model
        self.d_model = d_model
        self.hidden = hidden
        self.mlp_type = mlp_type
        self.activation = activation
        self.norm = RMSNorm(d_model, eps=norm_eps)
        if mlp_type == "mlp":
            if activation not in ACTIVATIONS:
                raise ValueError(f"unknown activation {activation!r}")
            self.mlp = _PlainMLP(d_model, hidden, num_layers, activation, bias)
        elif mlp_type == "swiglu":
            if num_layers != 2:
                raise ValueError("swiglu bridge is a fixed gate/up + down block; set num_layers=2")
            self.mlp = _SwiGLU(d_model, hidden, bias)
            self.activation = "silu"
        else:
            raise ValueError(f"unknown mlp_type {mlp_type!r}")
        self.reset_parameters(init_std)
        self.to(dtype)

    @classmethod
    def from_config(cls, d_model: int, cfg: BridgeConfig) -> "TransitionBridge":
        return cls(d_model=d_model, hidden_dim=cfg.hidden_dim, num_layers=cfg.num_layers, mlp_type=cfg.mlp_type,
                   activation=cfg.activation, bias=cfg.bias, init_std=cfg.init_std, norm_eps=cfg.norm_eps,
                   dtype=getattr(torch, cfg.dtype))

    @torch.no_grad()
    def reset_parameters(self, init_std: float = 1e-3) -> None:
        """Out-projection ~ N(0, init_std) (zero if 0), inner projections
        fan-in scaled, biases 0, norm 1 (bridges.py:118-129)."""
        for name, module in self.mlp.named_modules():
            if not isinstance(module, nn.Linear):
                continue
            if name == "out_proj":
                if init_std > 0:
                    nn.init.normal_(module.weight, std=init_std)
                else:
                    module.weight.zero_()
            else:
                nn.init.normal_(module.weight, std=1.0 / math.sqrt(module.in_features))
            if module.bias is not None:
                module.bias.zero_()
        self.norm.weight.fill_(1.0)

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [..., d] on the bridge's CUDA device -> same shape and dtype."""
        from ssd import ops
        from ssd.models.runner import run_bridge

        if not x.is_cuda or not self.norm.weight.is_cuda:
            raise ValueError("TransitionBridge.forward runs on the B200 kernels: move it and x to CUDA")
        shape, in_dtype = x.shape, x.dtype
        rows = x.reshape(-1, self.d_model)
        T = rows.shape[0]
        scratch = _BridgeScratch(self, T, x.device)
        scratch.resid.copy_(rows.to(self.norm.weight.dtype).float())
        ws = _workspace(x.device, T)
        run_bridge(self, scratch, T, ws)
        return scratch.resid.to(self.norm.weight.dtype).to(in_dtype).reshape(shape)


class _BridgeScratch:
    """Minimal scratch for a standalone bridge forward."""

    def __init__(self, bridge: TransitionBridge, T: int, device):
        dt = bridge.norm.weight.dtype
        self.resid = torch.zeros(T, bridge.d_model, dtype=torch.float32, device=device)
        self._xn = torch.zeros(T, bridge.d_model, dtype=dt, device=device)
        self._h = [torch.zeros(T, bridge.hidden, dtype=dt, device=device) for _ in range(2)]

        class _W:
            d = bridge.d_model

        self.w = _W

    def xn(self, dtype, cols):
        return self._xn

    def hid(self, dtype, cols, which=0):
        return self._h[which]


_WS: dict = {}


def _workspace(device, rows: int):
    from ssd import ops

    key = (str(device), max(64, rows))
    ws = _WS.get(key)
    if ws is None:
        _WS.clear()
        ws = ops.Workspace(device, max_rows=max(64, rows), vocab=1, max_head_rows=1)
        _WS[key] = ws
    return ws
