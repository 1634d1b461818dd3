"""The C-ABI library loads without a GPU and exports what include/*.h declares."""
import ctypes
import re

import pytest

from conftest import REPO


def declared_symbols():
    names = set()
    for hdr in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", hdr.read_text(), flags=re.S)
        names |= set(re.findall(r"NIMBLE_API\s+[\w\s\*]+?\b(nimble_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"nimble_tied_ce_forward", "nimble_tied_ce_backward", "nimble_tied_ce_combine"} <= names


def test_library_exports_every_declared_symbol():
    from nimbleml_b200._native_loader import SIGNATURES, native

    lib = ctypes.CDLL(str(native.path))
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(SIGNATURES) == declared_symbols()


def test_workspace_queries_and_argument_errors():
    from nimbleml_b200._native_loader import DTYPE_F16, DTYPE_F32, native

    fwd = native.forward_workspace_size(32768, 4096, 128256, DTYPE_F16)
    # Per-tile (max, sumexp) pairs + target: far below one N x V logit buffer.
    assert fwd < 32768 * 128256 * 2 / 16
    bwd = native.backward_workspace_size(32768, 4096, 128256, DTYPE_F16)
    assert bwd < 32768 * 128256 * 2 / 2
    small = native.backward_workspace_size(32768, 4096, 128256, DTYPE_F16, 256 << 20)
    assert small < bwd
    assert native.forward_workspace_size(8192, 768, 50257, DTYPE_F32) > 0
    with pytest.raises(RuntimeError, match="sizes must be positive"):
        native.forward_workspace_size(8, 0, 10, DTYPE_F32)
    # Argument checks run before any device call.
    with pytest.raises(RuntimeError, match="dtype"):
        native.call("nimble_tied_ce_forward", 16, 16, 16, 4, 64, 100, 0, 7, 16, 16, 16, 16, 1 << 20,
                    None, None)
    with pytest.raises(RuntimeError, match="16 bytes"):
        native.call("nimble_tied_ce_forward", 16, 16, 16, 4, 3, 100, 0, DTYPE_F16, 16, 16, 16, 16,
                    1 << 20, None, None)
    assert native.last_error()


def test_available_is_false_without_gpu():
    import torch
    from nimbleml_b200._native_loader import native

    if not torch.cuda.is_available():
        assert native.available() is False


def test_pybind_module_exports_device_entry_points():
    """The pybind11 module (the reference extension's binding pattern) loads without a GPU."""
    import sys

    from nimbleml_b200._native_loader import DTYPE_F16, native
    from nimbleml_b200.build_native import LIB_DIR

    sys.path.insert(0, str(LIB_DIR))
    import nimbleml_tied_ce_native as m

    for name in ("tied_ce_available", "tied_ce_forward_device", "tied_ce_combine_device", "tied_ce_backward_device",
                 "tied_ce_forward_workspace_size", "tied_ce_backward_workspace_size"):
        assert callable(getattr(m, name)), name
    assert m.tied_ce_forward_workspace_size(4096, 1024, 50257, DTYPE_F16) == \
        native.forward_workspace_size(4096, 1024, 50257, DTYPE_F16)
    with pytest.raises(RuntimeError, match="sizes must be positive"):
        m.tied_ce_forward_workspace_size(8, 0, 10, DTYPE_F16)


def test_reference_binding_rebinds_the_reference_names():
    """install() swaps the fused tied-CE functions everywhere the reference looks them up."""
    import os
    import subprocess
    import sys

    ref = REPO / "baseline" / "_ref"
    if not (ref / "NimbleML" / "__init__.py").exists():
        pytest.skip("baseline/_ref holds no reference install")
    code = f"""
import sys
sys.path[:0] = [{str(ref)!r}, {str(REPO)!r}]
import NimbleML.kernels as K, NimbleML.kernels.fused_tied_crossentropy as F, NimbleML.losses.cross_entropy as C
from nimbleml_b200.integration import reference_binding as rb
orig = C.fused_tied_crossentropy_forward
prev = rb.install()
for mod in (K, F, C):
    assert mod.fused_tied_crossentropy_forward is rb.fused_tied_crossentropy_forward
    assert mod.fused_tied_crossentropy_backward is rb.fused_tied_crossentropy_backward
rb.uninstall(prev)
assert C.fused_tied_crossentropy_forward is orig
print("ok")
"""
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, NIMBLEML_DEVICE="cpu"),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stderr[-2000:]
