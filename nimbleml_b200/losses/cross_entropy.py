"""``CrossEntropyLoss.forward_tied`` on B200 — the autograd node of the path.

Mirrors NimbleML/losses/cross_entropy.py:109-192: one autograd node for the
tied head ``hidden @ E^T`` plus cross-entropy, mean over the rows whose label
is not ``ignore_index``, grads for both ``hidden`` and the tied embedding
weights. The reference's node is a closure on its own ``Tensor``; here it is
a ``torch.autograd.Function`` whose backward runs the sm_100a kernels, so
``E.grad`` accumulates with every other use of the tied matrix (the input
embedding lookup) exactly as ``Tensor._accumulate_grad`` does
(NimbleML/utils/tensor.py:334-350).

Differences from the reference, each deliberate:

* No logits are saved: the forward keeps (lse, n_valid) per token and the
  backward recomputes (the reference saves a copy of the N x V logits,
  cross_entropy.py:152).
* ``ignore_index`` rows are masked inside the kernels instead of
  boolean-indexing a copy of ``hidden`` (``filter_ignore_index``,
  NimbleML/losses/_ce_prepare.py:46-69), so there is no host sync. When every
  row is ignored the loss is 0 and both grads are exactly zero (the
  reference returns a detached zero scalar, so no grad is produced at all).
* ``grad_scale`` (the upstream grad of the loss) is read on the device.
"""
from __future__ import annotations

from typing import Optional

import torch

from nimbleml_b200.kernels.fused_tied_crossentropy import (
    _NO_IGNORE,
    CHECK_BOUNDS,
    TiedCEStats,
    _as_cuda,
    as_label_indices,
    check_status,
    combine,
    compute_dtype_of,
    round_tf32,
    shard_backward,
    shard_forward,
)


def tied_forward_core(h2d, weights, labels, ignore_index, vocab_offset, vocab_size, group):
    """Forward of the tied head + CE for one vocab shard (shared by the autograd nodes).

    Returns ``(loss, saved)``: the fp32 0-d loss and what ``tied_backward_core``
    needs — the operands in the compute dtype, the labels, the per-token lse
    and valid count, and (fp32) the TF32-rounded operand copies.
    """
    from nimbleml_b200 import vocab_parallel

    # The tensor cores read E in the hidden's dtype; fp32 master weights
    # are cast for the GEMMs but receive an fp32 grad straight from the
    # kernel epilogue.
    weights_in_dtype = weights.dtype
    if weights.dtype != h2d.dtype:
        weights = weights.to(h2d.dtype)
    weights = weights.contiguous()
    rounded = (round_tf32(h2d), round_tf32(weights)) if h2d.dtype == torch.float32 else None
    part = shard_forward(*(rounded or (h2d, weights)), labels, vocab_offset, rounded=rounded is not None)
    stats3 = vocab_parallel.gather_shard_stats(part, group)  # (3, P, N)
    _, _, lse, loss, valid = combine(stats3, labels, vocab_size, ignore_index)
    if CHECK_BOUNDS:
        check_status(h2d.device)
    saved = dict(h2d=h2d, weights=weights, labels=labels, lse=lse, valid=valid, rounded=rounded,
                 meta=(ignore_index, vocab_offset, vocab_size, group, weights_in_dtype))
    return loss, saved


def tied_backward_core(grad_out, saved, *, grad_buffer=None, grad_hidden_dtype=None):
    """(grad_hidden, grad_weights or None) of ``tied_forward_core``'s loss.

    With ``grad_buffer`` the shard's dE is added into it by the GEMM epilogue
    and None is returned for the weights. ``grad_hidden_dtype`` defaults to
    the compute dtype.
    """
    from nimbleml_b200 import vocab_parallel

    h2d, weights, labels = saved["h2d"], saved["weights"], saved["labels"]
    ignore_index, vocab_offset, vocab_size, group, w_dtype = saved["meta"]
    stats = TiedCEStats(lse=saved["lse"], valid_count=saved["valid"], ignore_index=ignore_index,
                        vocab_size=vocab_size, vocab_offset=vocab_offset, rounded=saved["rounded"])
    grad_w = grad_buffer if grad_buffer is not None else torch.empty(weights.shape, dtype=w_dtype,
                                                                     device=weights.device)
    gh_dtype = grad_hidden_dtype or h2d.dtype
    if vocab_parallel.world_size(group) > 1:
        grad_h, grad_w = vocab_parallel.sharded_backward(grad_out, h2d, weights, labels, stats, group,
                                                         grad_weights=grad_w, accumulate=grad_buffer is not None)
        if grad_h.dtype != gh_dtype:
            grad_h = grad_h.to(gh_dtype)
    else:
        grad_h, grad_w = shard_backward(grad_out, h2d, weights, labels, stats, grad_weights=grad_w,
                                        accumulate=grad_buffer is not None, grad_hidden_dtype=gh_dtype)
    if CHECK_BOUNDS:
        check_status(h2d.device)
    return grad_h, (None if grad_buffer is not None else grad_w)


class _TiedCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h2d, weights, labels, ignore_index, vocab_offset, vocab_size, group, grad_buffer=None):
        loss, ctx.saved = tied_forward_core(h2d, weights, labels, ignore_index, vocab_offset, vocab_size, group)
        ctx.grad_buffer = grad_buffer
        return loss

    @staticmethod
    def backward(ctx, grad_out):
        saved, buf = ctx.saved, ctx.grad_buffer
        ctx.saved = ctx.grad_buffer = None
        grad_h, grad_w = tied_backward_core(grad_out, saved, grad_buffer=buf)
        return grad_h, grad_w, None, None, None, None, None, None


def tied_cross_entropy(hidden2d, weights, labels, ignore_index: Optional[int] = None, *,
                       vocab_offset: int = 0, vocab_size: Optional[int] = None, group=None,
                       grad_weights_buffer: Optional[torch.Tensor] = None):
    """Functional form: mean CE of ``hidden2d @ weights^T`` against ``labels``.

    With ``group`` set (a torch.distributed process group), ``weights`` is
    this rank's vocab shard starting at class ``vocab_offset`` of a
    ``vocab_size`` vocabulary; every rank gets the same loss, the grad of its
    own shard and the full ``hidden`` grad.

    ``grad_weights_buffer``: an fp32 tensor of the weights' shape that the
    backward adds this loss's weight grad into (the tied matrix's one grad
    buffer, shared with the embedding lookup's scatter-add); autograd then
    gets no grad for ``weights``.
    """
    ign = _NO_IGNORE if ignore_index is None else int(ignore_index)
    if vocab_size is None:
        vocab_size = weights.shape[0]
    if grad_weights_buffer is not None and (grad_weights_buffer.dtype != torch.float32 or
                                            grad_weights_buffer.shape != weights.shape or
                                            not grad_weights_buffer.is_contiguous()):
        raise ValueError("grad_weights_buffer must be a contiguous float32 tensor of the weights' shape")
    return _TiedCrossEntropy.apply(hidden2d, weights, labels, ign, int(vocab_offset), int(vocab_size), group,
                                   grad_weights_buffer)


def _flatten_logits(logits):
    """(2-D view, out_shape) for 1-D / 2-D / 3-D logits (NimbleML/losses/_ce_prepare.py:9-29)."""
    if logits.ndim == 1:
        return logits.reshape(1, -1), logits.shape
    if logits.ndim == 2:
        return logits, logits.shape
    if logits.ndim == 3:
        return logits.reshape(-1, logits.shape[-1]), logits.shape
    raise ValueError("Cross-entropy expects 1D, 2D, or 3D logits.")


def _loss_dtype(compute_dtype):
    """The reference coerces the loss to its compute dtype (Tensor([loss], ()),
    NimbleML/utils/tensor.py:147-153); it has no bf16 (NumPy falls back to
    fp16, np_backend.py:164-166), so a bf16 computation returns fp32."""
    return torch.float32 if compute_dtype == torch.bfloat16 else compute_dtype


def _row_pitch_ok(x2d):
    return x2d.stride(-1) == 1 and (x2d.stride(0) * x2d.element_size()) % 16 == 0


class _LogitsCrossEntropy(torch.autograd.Function):
    """Cross-entropy over given logits (the untied head), HBM-bound row kernels."""

    @staticmethod
    def forward(ctx, x2d, labels, ignore_index):
        from nimbleml_b200.kernels.fused_tied_crossentropy import _TORCH_TO_NIMBLE, _stream_ptr, native, status_word

        if not _row_pitch_ok(x2d):
            x2d = x2d.contiguous()
        n, v = x2d.shape
        dev = x2d.device
        st = torch.empty((3, n), dtype=torch.float32, device=dev)
        lse = torch.empty(n, dtype=torch.float32, device=dev)
        sc = torch.empty(2, dtype=torch.float32, device=dev)
        native.call("nimble_ce_logits_forward", x2d.data_ptr(), x2d.stride(0), labels.data_ptr(), n, v,
                    _TORCH_TO_NIMBLE[x2d.dtype], ignore_index, st[0].data_ptr(), st[1].data_ptr(),
                    st[2].data_ptr(), lse.data_ptr(), sc[0:1].data_ptr(), sc[1:2].data_ptr(),
                    status_word(dev).data_ptr(), _stream_ptr(dev))
        if CHECK_BOUNDS:
            check_status(dev)
        ctx.save_for_backward(x2d, labels, lse, sc[1:2])
        ctx.ignore_index = ignore_index
        return sc[0]

    @staticmethod
    def backward(ctx, grad_out):
        from nimbleml_b200.kernels.fused_tied_crossentropy import _TORCH_TO_NIMBLE, _stream_ptr, native

        x2d, labels, lse, valid = ctx.saved_tensors
        n, v = x2d.shape
        gs = grad_out.reshape(1).float().contiguous()
        g = torch.empty_like(x2d, memory_format=torch.contiguous_format)
        native.call("nimble_ce_logits_backward", gs.data_ptr(), valid.data_ptr(), x2d.data_ptr(), x2d.stride(0),
                    labels.data_ptr(), lse.data_ptr(), n, v, _TORCH_TO_NIMBLE[x2d.dtype], ctx.ignore_index,
                    g.data_ptr(), g.stride(0), _stream_ptr(x2d.device))
        return g, None, None


class CrossEntropyLoss:
    """NimbleML's ``CrossEntropyLoss``: the fused tied head and CE over given logits."""

    def forward(self, logits, labels, ignore_index=None):
        """Mean cross-entropy of (classes,), (batch, classes) or (batch, seq, classes) logits.

        Mirrors NimbleML/losses/cross_entropy.py:31-107 (ignored rows are
        masked in the kernel; the loss is returned in the logits' dtype).
        """
        if not logits.is_cuda:
            raise RuntimeError("CrossEntropyLoss on B200 needs CUDA tensors; there is no CPU path")
        compute_dtype_of(logits)
        x2d, _ = _flatten_logits(logits)
        labels = as_label_indices(labels, batch_size=x2d.shape[0], device=logits.device)
        ign = _NO_IGNORE if ignore_index is None else int(ignore_index)
        return _LogitsCrossEntropy.apply(x2d, labels, ign).to(_loss_dtype(logits.dtype))

    def forward_tied(self, hidden, embedding_weights, labels, ignore_index=None):
        """Cross-entropy with tied ``hidden @ embedding_weights.T`` logits.

        ``hidden`` is (batch, seq, d_model); returns a 0-d loss tensor in the
        compute dtype, as the reference's ``Tensor([loss], ())`` coerces it
        (NimbleML/utils/tensor.py:147-153).
        """
        if hidden.ndim != 3:
            raise ValueError("forward_tied expects hidden of shape (batch, seq, d_model).")
        batch, seq_len, d_model = hidden.shape
        row_count = batch * seq_len
        compute_dtype_of(hidden)
        if not hidden.is_cuda:
            raise RuntimeError("forward_tied on B200 needs CUDA tensors; there is no CPU path")
        h2d = hidden.reshape(row_count, d_model)
        if not h2d.is_contiguous():
            h2d = h2d.contiguous()
        weights = embedding_weights
        if not weights.is_contiguous():
            weights = weights.contiguous()
        label_indices = as_label_indices(labels, batch_size=row_count, device=hidden.device)
        loss = tied_cross_entropy(h2d, weights, label_indices, ignore_index)
        return loss.to(_loss_dtype(hidden.dtype))

    def __call__(self, logits, labels, ignore_index=None):
        return self.forward(logits, labels, ignore_index=ignore_index)


__all__ = ["CrossEntropyLoss", "tied_cross_entropy", "_as_cuda"]
