"""Load the required ``libnimbleml_tied_ce.so`` C-ABI library.

Mirrors NimbleML/_native_loader.py:20-28: there is no Python fallback for the
hot path. If the library is missing, importing this module raises
ImportError with the build command; if it is present but a call fails, the
wrapper raises RuntimeError with the library's own message (the reference's
pybind11 layer turns C++ ``std::runtime_error`` into RuntimeError the same
way, native/include/nimbleml/kernels.hpp:10-12).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from nimbleml_b200.build_native import LIB_PATH

_INSTALL_HINT = (
    "nimbleml_b200 requires the compiled library 'libnimbleml_tied_ce.so'.\n"
    "Build it from the repo root with:\n"
    "  python -m nimbleml_b200.build_native\n"
    "(needs nvcc from CUDA >= 12.8 for sm_100a)."
)

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2
DTYPE_TF32 = 3  # fp32 storage already rounded to TF32 (nimble_round_tf32)

STATUS_BAD_LABEL = 1
STATUS_WAIT_TIMEOUT = 2

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_size = ctypes.c_size_t
_c_vp = ctypes.c_void_p

# Exported symbol -> (restype, argtypes); kept in the order of
# include/nimbleml_tied_ce.h.
SIGNATURES = {
    "nimble_tied_ce_available": (_c_int, []),
    "nimble_tied_ce_last_error": (ctypes.c_char_p, []),
    "nimble_tied_ce_forward_workspace_size": (
        _c_int, [_c_i64, _c_i64, _c_i64, _c_int, ctypes.POINTER(_c_size)]),
    "nimble_tied_ce_forward": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_vp,
         _c_vp, _c_size, _c_vp, _c_vp]),
    "nimble_tied_ce_forward_noalloc": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp]),
    "nimble_tied_ce_combine": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp,
         _c_vp, _c_vp, _c_vp, _c_vp]),
    "nimble_tied_ce_backward_workspace_size": (
        _c_int, [_c_i64, _c_i64, _c_i64, _c_int, _c_size, ctypes.POINTER(_c_size)]),
    "nimble_tied_ce_backward_overlap_workspace_size": (
        _c_int, [_c_i64, _c_i64, _c_i64, _c_int, _c_size, ctypes.POINTER(_c_size)]),
    "nimble_round_tf32": (_c_int, [_c_vp, _c_vp, _c_i64, _c_vp]),
    "nimble_tied_ce_probe_wait_timeout": (_c_int, [ctypes.c_uint64, _c_vp, _c_vp]),
    "nimble_tied_logits_forward": (
        _c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_i64, _c_int, _c_vp]),
    "nimble_tied_logits_backward": (
        _c_int,
        [_c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_int, _c_vp, _c_int,
         _c_int, _c_vp]),
    "nimble_ce_logits_forward": (
        _c_int,
        [_c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_int, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
         _c_vp, _c_vp, _c_vp]),
    "nimble_ce_logits_backward": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64, _c_int, _c_i64, _c_vp, _c_i64,
         _c_vp]),
    "nimble_sampled_ce_forward": (
        _c_int,
        [_c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_i64, _c_vp, _c_vp, _c_vp,
         _c_vp, _c_vp, _c_vp, _c_vp, _c_vp]),
    "nimble_sampled_ce_backward": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_i64,
         _c_vp, _c_i64, _c_vp]),
    "nimble_rmsnorm_forward": (
        _c_int, [_c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_float, _c_int, _c_vp, _c_vp, _c_vp, _c_vp]),
    "nimble_rmsnorm_backward_workspace_size": (_c_int, [_c_i64, _c_i64, ctypes.POINTER(_c_size)]),
    "nimble_rmsnorm_backward": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_float, _c_int, _c_int, _c_vp, _c_vp,
         _c_int, _c_vp, _c_size, _c_vp]),
    "nimble_embedding_scatter_add_workspace_size": (_c_int, [_c_i64, _c_i64, ctypes.POINTER(_c_size)]),
    "nimble_embedding_scatter_add": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_size, _c_vp, _c_vp]),
    "nimble_adamw_step": (
        _c_int,
        [_c_vp, _c_vp, _c_int, _c_vp, _c_vp, _c_i64] + [ctypes.c_float] * 7 + [_c_vp, _c_int, _c_vp]),
    "nimble_tied_ce_backward": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_int, _c_vp, _c_int, _c_vp, _c_int, _c_int, _c_size, _c_vp, _c_size, _c_vp,
         _c_vp]),
    "nimble_tied_ce_backward_overlap": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_int, _c_vp, _c_int, _c_vp, _c_int, _c_int, _c_size, _c_vp, _c_size, _c_vp,
         _c_vp, _c_vp, _c_int, ctypes.c_float]),
}


class NativeLibrary:
    """ctypes view of the C ABI; every call is checked and raises on error."""

    def __init__(self, path: Path):
        self.path = Path(path)
        self.lib = ctypes.CDLL(str(self.path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    def last_error(self) -> str:
        msg = self.lib.nimble_tied_ce_last_error()
        return msg.decode() if msg else ""

    def call(self, name: str, *args) -> None:
        rc = getattr(self.lib, name)(*args)
        if rc != 0:
            raise RuntimeError(f"{name} failed ({rc}): {self.last_error()}")

    def available(self) -> bool:
        return bool(self.lib.nimble_tied_ce_available())

    def forward_workspace_size(self, n, d, v_local, dtype) -> int:
        out = _c_size(0)
        self.call("nimble_tied_ce_forward_workspace_size", n, d, v_local, dtype, ctypes.byref(out))
        return out.value

    def backward_workspace_size(self, n, d, v_local, dtype, slab_bytes=0, overlap=False) -> int:
        out = _c_size(0)
        name = "nimble_tied_ce_backward_overlap_workspace_size" if overlap else "nimble_tied_ce_backward_workspace_size"
        self.call(name, n, d, v_local, dtype, slab_bytes, ctypes.byref(out))
        return out.value

    def scatter_add_workspace_size(self, n, vocab_rows) -> int:
        out = _c_size(0)
        self.call("nimble_embedding_scatter_add_workspace_size", n, vocab_rows, ctypes.byref(out))
        return out.value

    def rmsnorm_backward_workspace_size(self, n, d) -> int:
        out = _c_size(0)
        self.call("nimble_rmsnorm_backward_workspace_size", n, d, ctypes.byref(out))
        return out.value


def load_native() -> NativeLibrary:
    if not LIB_PATH.exists():
        raise ImportError(_INSTALL_HINT)
    try:
        return NativeLibrary(LIB_PATH)
    except OSError as exc:
        raise ImportError(f"{_INSTALL_HINT}\n(load error: {exc})") from exc


native = load_native()

__all__ = ["native", "load_native", "NativeLibrary", "SIGNATURES", "DTYPE_F32", "DTYPE_F16",
           "DTYPE_BF16", "DTYPE_TF32", "STATUS_BAD_LABEL", "STATUS_WAIT_TIMEOUT"]
