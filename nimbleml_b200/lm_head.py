"""Tied LM-head logits on B200: the GEMM behind ``GPT.forward`` and ``generate``.

Mirrors ``GPT._tied_logits`` (NimbleML/models/gpt.py:139-181): logits =
x @ E^T over the last dimension with the backward
grad_x = grad @ E and grad_E = grad^T @ x (gpt.py:165-178), here as a
``torch.autograd.Function`` over ``nimble_tied_logits_forward / _backward``.
Training should use the fused loss (``CrossEntropyLoss.forward_tied``), which
never builds these logits; this module is for evaluation and sampling.

``last_token_logits`` returns only the logits of the last position of each
sequence, as ``generate`` consumes them (NimbleML/models/generate.py:101-111),
reading those rows of the hidden states in place through a row pitch.
"""
from __future__ import annotations

import torch

from nimbleml_b200._native_loader import native
from nimbleml_b200.kernels.fused_tied_crossentropy import _TORCH_TO_NIMBLE, _stream_ptr

_HALF = (torch.float16, torch.bfloat16)


def _padded(v: int, elem: int) -> int:
    per16 = 16 // elem
    return -(-v // per16) * per16


class _TiedLogits(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, weights):
        if x2d.dtype not in _HALF:
            raise ValueError("tied logits run in float16 or bfloat16")
        w = weights if weights.dtype == x2d.dtype else weights.to(x2d.dtype)
        w = w.contiguous()
        n, d = x2d.shape
        v = w.shape[0]
        vp = _padded(v, x2d.element_size())
        out = torch.empty((n, vp), dtype=x2d.dtype, device=x2d.device)
        native.call("nimble_tied_logits_forward", x2d.data_ptr(), x2d.stride(0), w.data_ptr(), n, d, v,
                    _TORCH_TO_NIMBLE[x2d.dtype], out.data_ptr(), vp, _TORCH_TO_NIMBLE[x2d.dtype],
                    _stream_ptr(x2d.device))
        ctx.save_for_backward(x2d, w)
        ctx.w_dtype = weights.dtype
        return out[:, :v]

    @staticmethod
    def backward(ctx, grad):
        x2d, w = ctx.saved_tensors
        n, d = x2d.shape
        v = w.shape[0]
        vp = _padded(v, x2d.element_size())
        g = torch.empty((n, vp), dtype=x2d.dtype, device=x2d.device)
        g[:, :v].copy_(grad)
        gx = torch.empty((n, d), dtype=x2d.dtype, device=x2d.device) if ctx.needs_input_grad[0] else None
        gw = torch.empty((v, d), dtype=ctx.w_dtype, device=x2d.device) if ctx.needs_input_grad[1] else None
        xc = x2d.contiguous()
        native.call("nimble_tied_logits_backward", g.data_ptr(), vp, xc.data_ptr(), w.data_ptr(), n, d, v,
                    _TORCH_TO_NIMBLE[x2d.dtype], gx.data_ptr() if gx is not None else None,
                    _TORCH_TO_NIMBLE[x2d.dtype], gw.data_ptr() if gw is not None else None,
                    _TORCH_TO_NIMBLE[ctx.w_dtype], 0, _stream_ptr(x2d.device))
        return gx, gw


def tied_logits(hidden: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """``hidden @ weights.T`` over the last dimension (GPT._tied_logits).

    Raises ValueError on a d_model mismatch, as the reference does
    (gpt.py:143-146). Returns logits of shape ``hidden.shape[:-1] + (V,)``.
    """
    v, d = weights.shape
    if hidden.shape[-1] != d:
        raise ValueError(f"d_model mismatch: activations {hidden.shape[-1]}, weights {d}")
    x2d = hidden.reshape(-1, d)
    if x2d.stride(-1) != 1 or x2d.stride(0) != d:
        x2d = x2d.contiguous()
    out = _TiedLogits.apply(x2d, weights)
    return out.reshape(*hidden.shape[:-1], v)


@torch.no_grad()
def last_token_logits(hidden_bsd: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """Logits of the last position of each sequence, (B, V), for sampling.

    Only B rows are multiplied: the kernel reads row S-1 of every sequence in
    place (row pitch S*d), so no (B, S, V) tensor and no gather copy.
    """
    if hidden_bsd.ndim != 3:
        raise ValueError("last_token_logits expects hidden of shape (batch, seq, d_model)")
    b, s, d = hidden_bsd.shape
    v = weights.shape[0]
    if weights.shape[1] != d:
        raise ValueError(f"d_model mismatch: activations {d}, weights {weights.shape[1]}")
    if hidden_bsd.dtype not in _HALF:
        raise ValueError("tied logits run in float16 or bfloat16")
    h = hidden_bsd.contiguous()
    w = (weights if weights.dtype == h.dtype else weights.to(h.dtype)).contiguous()
    vp = _padded(v, h.element_size())
    out = torch.empty((b, vp), dtype=h.dtype, device=h.device)
    last_row = h[:, s - 1, :]
    native.call("nimble_tied_logits_forward", last_row.data_ptr(), s * d, w.data_ptr(), b, d, v,
                _TORCH_TO_NIMBLE[h.dtype], out.data_ptr(), vp, _TORCH_TO_NIMBLE[h.dtype],
                _stream_ptr(h.device))
    return out[:, :v]


__all__ = ["tied_logits", "last_token_logits"]
