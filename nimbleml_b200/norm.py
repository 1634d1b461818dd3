"""RMSNorm on B200 — the norm whose output is the tied head's input.

Mirrors NimbleML/layers/rms_norm.py:9-90 (``RMSNorm(normalized_shape,
epsilon)`` with a learnable ``gamma``) over ``nimble_rmsnorm_forward /
_backward``: fp32 row statistics, one read and one write per element, and a
deterministic grad_gamma (per-block partial sums reduced in a fixed order).
"""
from __future__ import annotations

import torch

from nimbleml_b200.kernels.fused_tied_crossentropy import _TORCH_TO_NIMBLE, _stream_ptr, compute_dtype_of, native


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, eps):
        d = x.shape[-1]
        x2d = x.reshape(-1, d).contiguous()
        g = gamma.to(x.dtype).contiguous()
        y, ms, rms = rmsnorm_forward(x2d, g, eps)
        ctx.save_for_backward(x2d, g, ms, rms)
        ctx.eps = float(eps)
        ctx.gamma_dtype = gamma.dtype
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, grad):
        x2d, g, ms, rms = ctx.saved_tensors
        n, d = x2d.shape
        gx, gg = rmsnorm_backward(grad.reshape(n, d), x2d, g, ms, rms, ctx.eps)
        return gx.view(grad.shape), gg.to(ctx.gamma_dtype), None


def rmsnorm_forward(x2d: torch.Tensor, gamma: torch.Tensor, eps: float):
    """(y, ms, rms) of nimble_rmsnorm_forward for a contiguous (n, d) input; gamma in x's dtype."""
    n, d = x2d.shape
    y = torch.empty_like(x2d)
    ms = torch.empty(n, dtype=torch.float32, device=x2d.device)
    rms = torch.empty(n, dtype=torch.float32, device=x2d.device)
    native.call("nimble_rmsnorm_forward", x2d.data_ptr(), gamma.data_ptr(), n, d, float(eps),
                _TORCH_TO_NIMBLE[x2d.dtype], y.data_ptr(), ms.data_ptr(), rms.data_ptr(), _stream_ptr(x2d.device))
    return y, ms, rms


def rmsnorm_backward(grad2d: torch.Tensor, x2d: torch.Tensor, gamma: torch.Tensor, ms: torch.Tensor,
                     rms: torch.Tensor, eps: float):
    """(grad_x in x's dtype, grad_gamma fp32). An fp32 ``grad2d`` is read as is
    (the tied head's fp32 grad_hidden); other dtypes are cast to x's dtype."""
    n, d = x2d.shape
    if grad2d.dtype != torch.float32 and grad2d.dtype != x2d.dtype:
        grad2d = grad2d.to(x2d.dtype)
    gy = grad2d.contiguous()
    gx = torch.empty_like(x2d)
    gg = torch.empty(d, dtype=torch.float32, device=x2d.device)
    ws_bytes = native.rmsnorm_backward_workspace_size(n, d)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x2d.device)
    native.call("nimble_rmsnorm_backward", gy.data_ptr(), x2d.data_ptr(), gamma.data_ptr(), ms.data_ptr(),
                rms.data_ptr(), n, d, float(eps), _TORCH_TO_NIMBLE[x2d.dtype], _TORCH_TO_NIMBLE[gy.dtype],
                gx.data_ptr(), gg.data_ptr(), 0, ws.data_ptr(), ws_bytes, _stream_ptr(x2d.device))
    return gx, gg


def rms_norm(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """y = x / sqrt(mean(x^2, -1) + eps) * gamma."""
    if x.shape[-1] != gamma.shape[-1]:
        raise ValueError(f"Expected last dim {gamma.shape[-1]}, got {x.shape[-1]}")
    compute_dtype_of(x)
    return _RMSNormFn.apply(x, gamma, eps)


class RMSNorm(torch.nn.Module):
    """``RMSNorm(normalized_shape, epsilon=1e-5)`` with ``gamma`` initialised to ones."""

    def __init__(self, normalized_shape: int, epsilon: float = 1e-5, device=None, dtype=torch.float32):
        super().__init__()
        self.normalized_shape = int(normalized_shape)
        self.epsilon = float(epsilon)
        self.gamma = torch.nn.Parameter(torch.ones(self.normalized_shape, device=device, dtype=dtype))

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        if inputs.shape[-1] != self.normalized_shape:
            raise ValueError(f"Expected last dim {self.normalized_shape}, got {inputs.shape[-1]}")
        return rms_norm(inputs, self.gamma, self.epsilon)


__all__ = ["RMSNorm", "rms_norm", "rmsnorm_forward", "rmsnorm_backward"]
