"""Sampled softmax cross-entropy on B200 (NimbleML's ``SampledCrossEntropyLoss``).

Mirrors NimbleML/losses/sampled_cross_entropy.py:21-119 and
NimbleML/kernels/sampled_softmax.py:13-98: each row's softmax runs over its
true class (candidate column 0) plus ``num_samples`` negatives, and the
gradient scatters back into the full logits. The gather / softmax / scatter
run in ``nimble_sampled_ce_forward / _backward``.

Negatives are drawn on the host as the reference does, uniformly without
replacement from the classes other than the label; the random stream
differs from the reference's, so pass ``negative_indices`` for
reproducible parity.
"""
from __future__ import annotations

import numpy as np
import torch

from nimbleml_b200.kernels.fused_tied_crossentropy import (
    _NO_IGNORE, _TORCH_TO_NIMBLE, _stream_ptr, as_label_indices, check_status, compute_dtype_of, native,
    status_word, CHECK_BOUNDS)
from nimbleml_b200.losses.cross_entropy import _flatten_logits, _loss_dtype, _row_pitch_ok


def sample_negative_indices(vocab_size, label_indices, num_samples, *, rng=None):
    """(batch, num_samples) int64 negatives per row, never the row's label.

    Same contract and errors as NimbleML/kernels/sampled_softmax.py:13-42.
    """
    if vocab_size < 2:
        raise ValueError("vocab_size must be at least 2.")
    if num_samples < 1:
        raise ValueError("num_samples must be at least 1.")
    if num_samples >= vocab_size:
        raise ValueError("num_samples must be smaller than vocab_size.")
    labels = np.asarray(label_indices, dtype=np.int64).reshape(-1)
    gen = rng if hasattr(rng, "integers") else np.random.default_rng()
    out = np.empty((labels.size, num_samples), dtype=np.int64)
    for i, y in enumerate(labels):
        pick = gen.choice(vocab_size - 1, size=num_samples, replace=False)
        out[i] = pick + (pick >= y)  # skip the label: map [0, V-1) onto the other V-1 classes
    return out


class _SampledCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, cand, labels, ignore_index):
        if not _row_pitch_ok(x2d):
            x2d = x2d.contiguous()
        n, v = x2d.shape
        c = cand.shape[1]
        dev = x2d.device
        st = torch.empty((3, n), dtype=torch.float32, device=dev)
        lse = torch.empty(n, dtype=torch.float32, device=dev)
        sc = torch.empty(2, dtype=torch.float32, device=dev)
        native.call("nimble_sampled_ce_forward", x2d.data_ptr(), x2d.stride(0), cand.data_ptr(), labels.data_ptr(),
                    n, v, c, _TORCH_TO_NIMBLE[x2d.dtype], ignore_index, st[0].data_ptr(), st[1].data_ptr(),
                    st[2].data_ptr(), lse.data_ptr(), sc[0:1].data_ptr(), sc[1:2].data_ptr(),
                    status_word(dev).data_ptr(), _stream_ptr(dev))
        if CHECK_BOUNDS:
            check_status(dev)
        ctx.save_for_backward(x2d, cand, labels, lse, sc[1:2])
        ctx.ignore_index = ignore_index
        return sc[0]

    @staticmethod
    def backward(ctx, grad_out):
        x2d, cand, labels, lse, valid = ctx.saved_tensors
        n, v = x2d.shape
        gs = grad_out.reshape(1).float().contiguous()
        g = torch.empty((n, v), dtype=x2d.dtype, device=x2d.device)
        native.call("nimble_sampled_ce_backward", gs.data_ptr(), valid.data_ptr(), x2d.data_ptr(), x2d.stride(0),
                    cand.data_ptr(), labels.data_ptr(), lse.data_ptr(), n, v, cand.shape[1],
                    _TORCH_TO_NIMBLE[x2d.dtype], ctx.ignore_index, g.data_ptr(), v, _stream_ptr(x2d.device))
        return g, None, None, None


class SampledCrossEntropyLoss:
    """Cross-entropy over the true class plus sampled negatives per row."""

    def __call__(self, logits, labels, num_samples=32, negative_indices=None, rng=None, ignore_index=None):
        return self.forward(logits, labels, num_samples=num_samples, negative_indices=negative_indices, rng=rng,
                            ignore_index=ignore_index)

    def forward(self, logits, labels, *, num_samples=32, negative_indices=None, rng=None, ignore_index=None):
        if not logits.is_cuda:
            raise RuntimeError("SampledCrossEntropyLoss on B200 needs CUDA tensors; there is no CPU path")
        compute_dtype_of(logits)
        x2d, _ = _flatten_logits(logits)
        n, v = x2d.shape
        lab = as_label_indices(labels, batch_size=n, device=logits.device)
        if negative_indices is None:
            lab_host = lab.cpu().numpy()
            fill = 0 if ignore_index is None else int(ignore_index)
            safe = np.where(lab_host == fill, 0, lab_host) if ignore_index is not None else lab_host
            neg = sample_negative_indices(v, safe, num_samples, rng=rng)
        else:
            neg = np.asarray(negative_indices, dtype=np.int64)
            if neg.shape != (n, num_samples):
                raise ValueError(f"negative_indices must have shape ({n}, {num_samples}), got {neg.shape}.")
        neg_t = torch.as_tensor(neg, device=logits.device)
        cand = torch.cat([lab.clamp(min=0).view(-1, 1), neg_t], dim=1).contiguous()
        ign = _NO_IGNORE if ignore_index is None else int(ignore_index)
        return _SampledCE.apply(x2d, cand, lab, ign).to(_loss_dtype(logits.dtype))


__all__ = ["SampledCrossEntropyLoss", "sample_negative_indices"]
