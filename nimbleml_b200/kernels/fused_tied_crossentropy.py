"""Fused tied LM head + cross-entropy on B200 (drop-in for the reference kernels).

Same names, argument order and return shapes as
NimbleML/kernels/fused_tied_crossentropy.py:8-48, but no N x V buffer exists:

* ``fused_tied_crossentropy_forward(hidden, weights, label_indices)`` returns
  ``(loss, hidden, weights, stats, max_vals, sum_exp)``. Slot 4, which held
  the materialised logits in the reference, is a :class:`TiedCEStats` with the
  per-token log-sum-exp and the valid-row count; ``max_vals`` is (N, 1) and
  ``sum_exp`` is (N, 1) fp32, as in the reference's fp16 path
  (NimbleML/kernels/fused_crossentropy.py:21-23). ``loss`` is a 0-d fp32
  device tensor (``float(loss)`` gives the reference's Python float; keeping
  it on the device avoids the reference's per-step host sync at
  fused_crossentropy.py:29).
* ``fused_tied_crossentropy_backward(grad_scale, hidden, weights,
  label_indices, logits, max_vals, sum_exp)`` recomputes the logits with
  tensor cores and returns ``(grad_hidden, grad_weights)`` in the compute
  dtype, with G = (softmax - onehot) * grad_scale / n_valid as in
  fused_crossentropy.py:33-50.

Inputs are torch CUDA tensors (or anything ``torch.as_tensor`` accepts; host
arrays are copied to the current device). On a CUDA device every launch goes
through ``libnimbleml_tied_ce.so``; there is no CPU or library fallback, and a
missing library raises at import.

Device-side errors (a label outside [0, V), a bounded device wait that gave
up) are OR-ed into a per-device status word. Without any host sync, a label
error makes the loss NaN at once, and every call of the path first reads an
asynchronous pinned-memory copy of the word taken at the end of an earlier
call, raising if a bit is set. So an error raises at the latest a few calls
later; results of a call are undefined until a later check has passed.
``check_status`` reads the word synchronously (``NIMBLEML_CHECK_BOUNDS=1``
does that after every call).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch

from nimbleml_b200._native_loader import (
    DTYPE_BF16,
    DTYPE_F16,
    DTYPE_F32,
    DTYPE_TF32,
    STATUS_BAD_LABEL,
    STATUS_WAIT_TIMEOUT,
    native,
)

_TORCH_TO_NIMBLE = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}

# NIMBLEML_CHECK_BOUNDS=1 makes every call read the device status word (one
# host sync) and raise on out-of-range labels — the reference's bounds-check
# knob (NimbleML/kernels/embedding_scatter.py:9-22) applied to this path.
CHECK_BOUNDS = os.environ.get("NIMBLEML_CHECK_BOUNDS", "0") not in ("", "0", "false", "False")
# Per-slab budget (bytes) for the backward's G tile; 0 = library default.
SLAB_BYTES = int(os.environ.get("NIMBLEML_TIED_CE_SLAB_BYTES", "0"))


@dataclass
class TiedCEStats:
    """Per-token statistics saved by the forward in place of the N x V logits."""

    lse: torch.Tensor          # (N,) fp32 global log-sum-exp
    valid_count: torch.Tensor  # (1,) fp32 number of rows whose label != ignore_index
    ignore_index: int          # rows with this label contribute nothing
    vocab_size: int            # total vocabulary V
    vocab_offset: int = 0      # first global class id of the local weight shard
    # fp32 only: TF32-rounded copies of (hidden, weights) made by the forward,
    # reused by the backward so each pair of calls rounds once.
    rounded: Optional[tuple] = None


_status_words: dict = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The per-device int32 status word the kernels OR error bits into."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status_words.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _status_words[key] = buf
    return buf


def _raise_for(val: int) -> None:
    if val & STATUS_WAIT_TIMEOUT:
        raise RuntimeError("tied-CE kernel aborted: a bounded device wait timed out; "
                           "the outputs of the calls since the last check are undefined")
    if val & STATUS_BAD_LABEL:
        raise ValueError("label index out of range for the vocabulary")


def check_status(device: torch.device, *, clear: bool = True) -> int:
    """Reads (host sync) and optionally clears the device status word; raises on error bits."""
    buf = status_word(device)
    val = int(buf.item())
    if clear and val:
        buf.zero_()
        _monitor(device).pending = False  # an older asynchronous copy would repeat this value
    _raise_for(val)
    return val


class _StatusMonitor:
    """Asynchronous reads of one device's status word (no host sync).

    ``snapshot`` enqueues a copy of the word into pinned host memory on the
    current stream and records an event; ``poll`` looks at the copy only once
    that event has completed (``Event.query`` does not block), and raises
    (clearing the device word) when an error bit is set.
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = torch.cuda.Event()
        self.pending = False

    def snapshot(self) -> None:
        self.host.copy_(status_word(self.device), non_blocking=True)
        self.event.record(torch.cuda.current_stream(self.device))
        self.pending = True

    def poll(self) -> None:
        if not self.pending or not self.event.query():
            return
        self.pending = False
        val = int(self.host[0])
        if val:
            status_word(self.device).zero_()
            _raise_for(val)


_monitors: dict = {}


def _monitor(device: torch.device) -> _StatusMonitor:
    key = device.index if device.index is not None else torch.cuda.current_device()
    mon = _monitors.get(key)
    if mon is None:
        mon = _StatusMonitor(torch.device("cuda", key))
        _monitors[key] = mon
    return mon


def poll_status(device: torch.device) -> None:
    """Raises if an earlier call's status copy, already on the host, shows an error."""
    _monitor(device).poll()


def snapshot_status(device: torch.device) -> None:
    """Enqueues the asynchronous host copy of the status word read by poll_status."""
    _monitor(device).snapshot()


def round_tf32(x: torch.Tensor) -> torch.Tensor:
    """A TF32-rounded fp32 copy of ``x`` (nimble_round_tf32 on the device)."""
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    native.call("nimble_round_tf32", x.data_ptr(), out.data_ptr(), x.numel(), _stream_ptr(x.device))
    return out


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def compute_dtype_of(t: torch.Tensor) -> int:
    try:
        return _TORCH_TO_NIMBLE[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported compute dtype {t.dtype}; use float32, float16 or bfloat16") from None


def _as_cuda(x, dtype=None, device=None) -> torch.Tensor:
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    if device is None:
        device = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
    if dtype is not None and x.dtype != dtype:
        x = x.to(dtype)
    if x.device != device:
        x = x.to(device, non_blocking=True)
    return x.contiguous()


def as_label_indices(label_indices, *, batch_size: int, device: torch.device) -> torch.Tensor:
    """Flatten and validate int64 labels (NimbleML/utils/np_backend.py:193-208)."""
    if not hasattr(label_indices, "dtype") and hasattr(label_indices, "data"):
        label_indices = label_indices.data
    labels = _as_cuda(label_indices, dtype=torch.int64, device=device).reshape(-1)
    if labels.numel() != batch_size:
        raise ValueError(f"label count ({labels.numel()}) must match batch size ({batch_size}).")
    return labels


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def shard_forward(h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, vocab_offset: int = 0, *,
                  rounded: bool = False):
    """Per-token (max, sum-exp, target) over the columns of one weight shard.

    Returns a (3, N) fp32 tensor: rows are shard max, shard sum-exp and the
    target logit (0 where the label lies outside the shard). ``rounded``: fp32
    ``h`` and ``w`` already hold TF32 values (``round_tf32``) and are read in
    place.
    """
    n, d = h.shape
    v_local = w.shape[0]
    dt = compute_dtype_of(h)
    if rounded and dt == DTYPE_F32:
        dt = DTYPE_TF32
    poll_status(h.device)
    out = torch.empty((3, n), dtype=torch.float32, device=h.device)
    ws = _workspace(native.forward_workspace_size(n, d, v_local, dt), h.device)
    native.call(
        "nimble_tied_ce_forward", h.data_ptr(), w.data_ptr(), labels.data_ptr(), n, d, v_local,
        vocab_offset, dt, out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), ws.data_ptr(),
        ws.numel(), status_word(h.device).data_ptr(), _stream_ptr(h.device))
    return out


def combine(shard_stats: torch.Tensor, labels: torch.Tensor, vocab_size: int, ignore_index: int):
    """Merges (3, P, N) shard statistics into (max, sum_exp, lse, loss, valid_count)."""
    _, p, n = shard_stats.shape
    dev = shard_stats.device
    stats = shard_stats.contiguous()
    gmax = torch.empty(n, dtype=torch.float32, device=dev)
    gsum = torch.empty(n, dtype=torch.float32, device=dev)
    lse = torch.empty(n, dtype=torch.float32, device=dev)
    scalars = torch.empty(2, dtype=torch.float32, device=dev)
    native.call(
        "nimble_tied_ce_combine", stats[0].data_ptr(), stats[1].data_ptr(), stats[2].data_ptr(), p,
        labels.data_ptr(), n, vocab_size, ignore_index, gmax.data_ptr(), gsum.data_ptr(),
        lse.data_ptr(), scalars[0:1].data_ptr(), scalars[1:2].data_ptr(),
        status_word(dev).data_ptr(), _stream_ptr(dev))
    snapshot_status(dev)
    return gmax, gsum, lse, scalars[0], scalars[1:2]


def shard_backward(grad_scale: torch.Tensor, h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor,
                   stats: TiedCEStats, *, grad_hidden_dtype=None, grad_weights: Optional[torch.Tensor] = None,
                   accumulate: bool = False, slab_bytes: Optional[int] = None,
                   ready_event: Optional[torch.cuda.Event] = None, last_de_max_ctas: int = 0,
                   capped_fraction: float = 1.0):
    """(grad_hidden partial over this shard, grad_weights of the shard).

    ``slab_bytes`` bounds the vocab slab's G scratch (default: the
    NIMBLEML_TIED_CE_SLAB_BYTES environment value, else the library's 2 GiB).
    With ``ready_event`` the event is recorded as soon as grad_hidden is final
    and the first ``capped_fraction`` of the last slab's grad_weights rows run
    on at most ``last_de_max_ctas`` SMs (the rest on all SMs), so a
    collective on grad_hidden can overlap them.
    """
    n, d = h.shape
    v_local = w.shape[0]
    dt = compute_dtype_of(h)
    dev = h.device
    poll_status(dev)
    if stats.rounded is not None and dt == DTYPE_F32:
        h, w = stats.rounded  # the forward's TF32 copies: no second rounding pass
        dt = DTYPE_TF32
    gh_dtype = grad_hidden_dtype or h.dtype
    grad_h = torch.empty((n, d), dtype=gh_dtype, device=dev)
    if grad_weights is None:
        grad_weights = torch.empty((v_local, d), dtype=h.dtype, device=dev)
        accumulate = False
    slab = SLAB_BYTES if slab_bytes is None else int(slab_bytes)
    ws = _workspace(native.backward_workspace_size(n, d, v_local, dt, slab, overlap=ready_event is not None), dev)
    gs = grad_scale.reshape(-1)[:1].to(device=dev, dtype=torch.float32).contiguous()
    args = (gs.data_ptr(), h.data_ptr(), w.data_ptr(), labels.data_ptr(), stats.lse.data_ptr(),
            stats.valid_count.data_ptr(), n, d, v_local, stats.vocab_offset, stats.ignore_index, dt,
            grad_h.data_ptr(), _TORCH_TO_NIMBLE[gh_dtype], grad_weights.data_ptr(),
            _TORCH_TO_NIMBLE[grad_weights.dtype], 1 if accumulate else 0, slab, ws.data_ptr(), ws.numel(),
            status_word(dev).data_ptr(), _stream_ptr(dev))
    if ready_event is None:
        native.call("nimble_tied_ce_backward", *args)
    else:
        if ready_event.cuda_event == 0:
            ready_event.record()  # torch creates the CUDA event at its first record; the library re-records it
        native.call("nimble_tied_ce_backward_overlap", *args, ready_event.cuda_event, int(last_de_max_ctas),
                    float(capped_fraction))
    snapshot_status(dev)
    return grad_h, grad_weights


# Reference has no ignore_index at this level; labels equal to it (default
# -100, never a valid class id) simply never match a column.
_NO_IGNORE = -(2**63)


def fused_tied_crossentropy_forward(hidden, weights, label_indices, *, ignore_index: Optional[int] = None):
    """Mean CE from hidden states and tied embedding weights, without logits.

    Args:
        hidden: ``(batch, d_model)`` CUDA tensor in the compute dtype.
        weights: tied embedding matrix ``(vocab, d_model)``; cast to the
            hidden's dtype if it differs (the reference's ``on_device``).
        label_indices: int64 labels ``(batch,)``.
        ignore_index: optional label value whose rows are left out of the mean.

    Returns:
        tuple: ``(loss, hidden, weights, stats, max_vals, sum_exp)`` for backward.
    """
    h = _as_cuda(hidden)
    compute_dtype_of(h)
    w = _as_cuda(weights, dtype=h.dtype, device=h.device)
    if h.ndim != 2 or w.ndim != 2 or h.shape[1] != w.shape[1]:
        raise ValueError("hidden must be (batch, d_model) and weights (vocab, d_model)")
    n = h.shape[0]
    labels = as_label_indices(label_indices, batch_size=n, device=h.device)
    ign = _NO_IGNORE if ignore_index is None else int(ignore_index)
    rounded = (round_tf32(h), round_tf32(w)) if h.dtype == torch.float32 else None
    part = shard_forward(*(rounded or (h, w)), labels, rounded=rounded is not None)
    gmax, gsum, lse, loss, valid = combine(part.unsqueeze(1), labels, w.shape[0], ign)
    if CHECK_BOUNDS:
        check_status(h.device)
    stats = TiedCEStats(lse=lse, valid_count=valid, ignore_index=ign, vocab_size=w.shape[0], rounded=rounded)
    return loss, h, w, stats, gmax.view(n, 1), gsum.view(n, 1)


def fused_tied_crossentropy_backward(grad_scale, hidden, weights, label_indices, logits, max_vals, sum_exp):
    """Gradients w.r.t. hidden and tied weights from fused tied CE.

    Args:
        grad_scale: upstream gradient of the loss (Python float or a device
            scalar tensor; a tensor is read on the device, no host sync).
        logits: the :class:`TiedCEStats` returned by the forward. A plain
            placeholder is accepted too; the lse is then rebuilt from
            ``max_vals`` and ``sum_exp`` over all rows.

    Returns:
        tuple: ``(grad_hidden, grad_weights)`` in the compute dtype.
    """
    h = _as_cuda(hidden)
    w = _as_cuda(weights, dtype=h.dtype, device=h.device)
    n = h.shape[0]
    labels = as_label_indices(label_indices, batch_size=n, device=h.device)
    if isinstance(logits, TiedCEStats):
        stats = logits
    else:
        mx = _as_cuda(max_vals, dtype=torch.float32, device=h.device).reshape(-1)
        se = _as_cuda(sum_exp, dtype=torch.float32, device=h.device).reshape(-1)
        stats = TiedCEStats(lse=(mx + torch.log(se)).contiguous(),
                            valid_count=torch.full((1,), float(n), device=h.device),
                            ignore_index=_NO_IGNORE, vocab_size=w.shape[0])
    if not isinstance(grad_scale, torch.Tensor):
        grad_scale = torch.full((1,), float(grad_scale), dtype=torch.float32, device=h.device)
    grad_h, grad_w = shard_backward(grad_scale, h, w, labels, stats)
    if CHECK_BOUNDS:
        check_status(h.device)
    return grad_h, grad_w
