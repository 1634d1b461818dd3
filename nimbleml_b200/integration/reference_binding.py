"""Runs the reference NimbleML's own tied-CE path on the B200 kernels.

``install()`` rebinds ``fused_tied_crossentropy_forward`` /
``fused_tied_crossentropy_backward`` inside the reference package
(``NimbleML.kernels``, ``NimbleML.kernels.fused_tied_crossentropy`` and the
names ``NimbleML.losses.cross_entropy`` imported from there,
NimbleML/losses/cross_entropy.py:1-3) to the functions below. Those call the
pybind11 ``*_device`` entry points of ``nimbleml_tied_ce_native``
(``csrc/tied_ce_pybind.cpp``), which call the C ABI of
``libnimbleml_tied_ce.so``. Nothing else in the reference changes:
``GPT.compute_loss`` (NimbleML/models/gpt.py:123-137), ``forward_tied`` and
its ``_backward`` closure (NimbleML/losses/cross_entropy.py:109-192), and
``Tensor.backward`` through the native autograd runner
(NimbleML/utils/tensor.py:286-332, native/src/autograd.cpp:28-57) run as
they are.

The functions keep the reference's names, argument order and return arity
(NimbleML/kernels/fused_tied_crossentropy.py:8-48):

* forward returns ``(loss, hidden, weights, stats, max_vals, sum_exp)``;
  slot 4, the reference's N x V logits, is a float32 array of N + 1 values
  (the per-token log-sum-exp, then the valid-row count). ``forward_tied``
  copies that slot with ``_save_for_backward`` (cross_entropy.py:152), so it
  copies N + 1 floats instead of the logits.
* backward returns ``(grad_hidden, grad_weights)`` in the compute dtype.

Arrays may be NumPy (the reference's CPU backend: each call copies the
operands to the current CUDA device and the results back) or CuPy / any
``__cuda_array_interface__`` array on the device (zero-copy; the launch goes
on CuPy's current stream). The compute dtype is the reference's
``np_backend.dtype``: float32 runs on TF32 tensor cores, float16 on f16
tensor cores; float64 is rejected (no tensor-core path). Errors of the
native layer raise RuntimeError, as the reference's pybind layer does.
"""
from __future__ import annotations

import contextlib
import importlib
import sys
from typing import Optional

import numpy as np
import torch

from nimbleml_b200.build_native import LIB_DIR

if str(LIB_DIR) not in sys.path:
    sys.path.insert(0, str(LIB_DIR))
import nimbleml_tied_ce_native as _native  # noqa: E402  (built by nimbleml_b200.build_native)

# Labels that can never match a class id: the reference filters
# ignore_index rows before calling these functions (_ce_prepare.py:46-69).
_NO_IGNORE = -(2**63)
_DTYPES = {np.dtype(np.float32): (_native.DTYPE_F32, torch.float32),
           np.dtype(np.float16): (_native.DTYPE_F16, torch.float16)}

# Number of forward / backward calls served, for callers that want to check
# the reference really ran on these kernels.
calls = {"forward": 0, "backward": 0}


def _is_device_array(x) -> bool:
    return hasattr(x, "__cuda_array_interface__")


def _to_torch(x, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """A contiguous CUDA tensor for a NumPy array (copied) or a device array (zero-copy when possible)."""
    if isinstance(x, torch.Tensor):
        t = x
    elif _is_device_array(x):
        t = torch.as_tensor(x, device="cuda")
    else:
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(x)))
    if t.device.type != "cuda":
        t = t.to("cuda", non_blocking=False)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def _like(t: torch.Tensor, ref):
    """Returns ``t`` as the array kind of ``ref``: NumPy for NumPy inputs, CuPy for device arrays."""
    if _is_device_array(ref) and not isinstance(ref, torch.Tensor):
        import cupy as cp  # the reference's GPU backend (NimbleML/utils/np_backend.py:16-24)

        return cp.asarray(t)
    return t.cpu().numpy()


def _on_caller_stream(ref):
    """Context that puts every torch op and launch of a call on the caller's stream:
    CuPy's current stream for device arrays, torch's current stream otherwise."""
    if _is_device_array(ref) and not isinstance(ref, torch.Tensor):
        import cupy as cp

        return torch.cuda.stream(torch.cuda.ExternalStream(cp.cuda.get_current_stream().ptr))
    return contextlib.nullcontext()


def _compute_dtype():
    from NimbleML.utils import np_backend

    dt = np.dtype(np_backend.dtype)
    if dt not in _DTYPES:
        raise ValueError(f"the B200 tied-CE kernels compute in float32 (TF32) or float16, not {dt}")
    return dt, _DTYPES[dt]


def _status(dev_status: torch.Tensor) -> None:
    val = int(dev_status.item())
    if val & _native.STATUS_WAIT_TIMEOUT:
        raise RuntimeError("tied-CE kernel aborted: a bounded device wait timed out")
    if val & _native.STATUS_BAD_LABEL:
        raise IndexError("label index out of range for the vocabulary")


def fused_tied_crossentropy_forward(hidden, weights, label_indices):
    """Mean CE from hidden states and tied embedding weights, without logits.

    Same contract as NimbleML/kernels/fused_tied_crossentropy.py:8-24 except
    slot 4 (see the module docstring).
    """
    from NimbleML.utils import np_backend

    np_dt, (code, tdt) = _compute_dtype()
    h_arr = np_backend.on_device(hidden, dtype=np_dt)
    w_arr = np_backend.on_device(weights, dtype=np_dt)
    n, d = h_arr.shape
    v = w_arr.shape[0]
    y_arr = np_backend.as_label_indices(label_indices, batch_size=n)
    with _on_caller_stream(h_arr):
        h, w, y = _to_torch(h_arr, tdt), _to_torch(w_arr, tdt), _to_torch(y_arr, torch.int64)
        dev = h.device
        stream = torch.cuda.current_stream().cuda_stream
        st = torch.empty((3, n), dtype=torch.float32, device=dev)
        ws = torch.empty(max(1, _native.tied_ce_forward_workspace_size(n, d, v, code)), dtype=torch.uint8,
                         device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        _native.tied_ce_forward_device(h.data_ptr(), w.data_ptr(), y.data_ptr(), n, d, v, 0, code, st[0].data_ptr(),
                                       st[1].data_ptr(), st[2].data_ptr(), ws.data_ptr(), ws.numel(),
                                       status.data_ptr(), stream)
        mx = torch.empty(n, dtype=torch.float32, device=dev)
        se = torch.empty(n, dtype=torch.float32, device=dev)
        packed = torch.empty(n + 1, dtype=torch.float32, device=dev)  # [lse_0 .. lse_{N-1}, n_valid]
        loss = torch.empty(1, dtype=torch.float32, device=dev)
        _native.tied_ce_combine_device(st[0].data_ptr(), st[1].data_ptr(), st[2].data_ptr(), 1, y.data_ptr(), n, v,
                                       _NO_IGNORE, mx.data_ptr(), se.data_ptr(), packed.data_ptr(), loss.data_ptr(),
                                       packed[n:].data_ptr(), status.data_ptr(), stream)
        _status(status)  # one host read, as the reference's float(loss) (fused_crossentropy.py:29)
        calls["forward"] += 1
        # max / sum_exp as the reference returns them: (N, 1), sum_exp in fp32.
        return (float(loss.item()), h_arr, w_arr, _like(packed, h_arr), _like(mx.view(n, 1).to(tdt), h_arr),
                _like(se.view(n, 1), h_arr))


def fused_tied_crossentropy_backward(grad_scale, hidden, weights, label_indices, logits, max_vals, sum_exp):
    """(grad_hidden, grad_weights) of the tied CE, recomputing the logits on tensor cores.

    Same contract as NimbleML/kernels/fused_tied_crossentropy.py:27-48;
    ``logits`` is the packed (N + 1,) slot of the forward.
    """
    from NimbleML.utils import np_backend

    np_dt, (code, tdt) = _compute_dtype()
    h_arr = np_backend.on_device(hidden, dtype=np_dt)
    w_arr = np_backend.on_device(weights, dtype=np_dt)
    n, d = h_arr.shape
    v = w_arr.shape[0]
    y_arr = np_backend.as_label_indices(label_indices, batch_size=n)
    with _on_caller_stream(h_arr):
        h, w, y = _to_torch(h_arr, tdt), _to_torch(w_arr, tdt), _to_torch(y_arr, torch.int64)
        packed = _to_torch(logits, torch.float32).reshape(-1)
        if packed.numel() != n + 1:
            raise ValueError("logits must be the (N + 1,) statistics slot returned by this forward")
        dev = h.device
        stream = torch.cuda.current_stream().cuda_stream
        gs = torch.full((1,), float(grad_scale), dtype=torch.float32, device=dev)
        gh = torch.empty((n, d), dtype=tdt, device=dev)
        gw = torch.empty((v, d), dtype=tdt, device=dev)
        ws = torch.empty(max(1, _native.tied_ce_backward_workspace_size(n, d, v, code, 0)), dtype=torch.uint8,
                         device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        _native.tied_ce_backward_device(gs.data_ptr(), h.data_ptr(), w.data_ptr(), y.data_ptr(), packed.data_ptr(),
                                        packed[n:].data_ptr(), n, d, v, 0, _NO_IGNORE, code, gh.data_ptr(), code,
                                        gw.data_ptr(), code, False, 0, ws.data_ptr(), ws.numel(),
                                        status.data_ptr(), stream)
        _status(status)
        calls["backward"] += 1
        return _like(gh, h_arr), _like(gw, h_arr)


_MODULES = ("NimbleML.kernels", "NimbleML.kernels.fused_tied_crossentropy", "NimbleML.losses.cross_entropy")


def install():
    """Rebinds the reference's fused tied-CE names to the B200 kernels; returns the previous bindings."""
    previous = {}
    for name in _MODULES:
        mod = importlib.import_module(name)
        previous[name] = (mod.fused_tied_crossentropy_forward, mod.fused_tied_crossentropy_backward)
        mod.fused_tied_crossentropy_forward = fused_tied_crossentropy_forward
        mod.fused_tied_crossentropy_backward = fused_tied_crossentropy_backward
    return previous


def uninstall(previous) -> None:
    """Restores the bindings ``install`` returned."""
    for name, (fwd, bwd) in previous.items():
        mod = importlib.import_module(name)
        mod.fused_tied_crossentropy_forward = fwd
        mod.fused_tied_crossentropy_backward = bwd
