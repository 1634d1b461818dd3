"""The reference NimbleML's own training loss runs on the B200 kernels.

The unmodified reference package (installed offline into baseline/_ref from
the reference checkout) runs ``GPT.compute_loss`` + ``Tensor.backward`` —
its ``forward_tied`` node (NimbleML/losses/cross_entropy.py:109-192), its
Tensor autograd hook and its native autograd runner
(NimbleML/utils/tensor.py:286-332, native/src/autograd.cpp:28-57) — twice on
the tiny GPT of config 1 (NimbleML/models/gpt.py:123-137): once as shipped
(NumPy on the CPU), once after ``nimbleml_b200.integration.reference_binding
.install()`` rebinds its fused tied-CE functions to the pybind11 ``*_device``
entry points over the C ABI. Loss and every parameter grad must agree
within the fp32 / TF32 tolerances (loss 1e-5, grads 1e-3 relative), and the
bound kernels must actually have served the calls.

Each run is a fresh subprocess with NIMBLEML_DEVICE=cpu (the reference picks
its array backend at import). Skipped, with the reason, when baseline/_ref
does not hold the reference.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

REF = REPO / "baseline" / "_ref"


def _run_case(patched: bool, ignore: bool, out_path: str) -> None:
    """Body of one subprocess: the reference GPT's loss and grads, optionally on the B200 kernels."""
    import random

    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(REPO))
    from NimbleML import GPT, Tensor
    from NimbleML.utils import np_backend
    from NimbleML.utils import tensor as ref_tensor

    np_backend.set_dtype("float32")
    if patched:
        from nimbleml_b200.integration import reference_binding as rb

        rb.install()
    random.seed(0)
    np.random.seed(0)
    m = GPT(vocab_size=256, d_model=64, num_heads=4, num_layers=2, max_seq_len=32, fused_blocks=True)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 256, (2, 8), dtype=np.int64)
    lab = rng.integers(0, 256, (2, 8), dtype=np.int64)
    lab[0, 0] = 0
    lab[1, 7] = 255
    if ignore:
        lab[0, 2:5] = -1
    loss = m.compute_loss(Tensor.from_int64(ids, (2, 8)), Tensor.from_int64(lab, (2, 8)),
                          ignore_index=-1 if ignore else None)
    loss.backward()
    grads = [np.asarray(p.grad, dtype=np.float64).ravel() for p in m.parameters()]
    np.savez(out_path, loss=np.float64(loss.item()), n=len(grads), **{f"g{i}": g for i, g in enumerate(grads)})
    info = {"copies": ref_tensor._SAVE_FOR_BACKWARD_STATS["copies"]}
    if patched:
        info["calls"] = dict(rb.calls)
    with open(out_path + ".json", "w") as f:
        json.dump(info, f)


def _spawn(patched, ignore, tmp_path):
    out = str(tmp_path / f"case_{int(patched)}_{int(ignore)}.npz")
    env = dict(os.environ, NIMBLEML_DEVICE="cpu", NIMBLEML_DTYPE="float32")
    code = (f"import sys; sys.path.insert(0, {str(REPO / 'tests')!r}); "
            f"from test_reference_dropin_gpu import _run_case; _run_case({patched}, {ignore}, {out!r})")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    data = dict(np.load(out))
    with open(out + ".json") as f:
        info = json.load(f)
    return data, info


@pytest.mark.parametrize("ignore", [False, True])
def test_reference_compute_loss_on_b200_kernels(ignore, tmp_path):
    if not (REF / "NimbleML" / "__init__.py").exists():
        pytest.skip("baseline/_ref holds no reference install (pip install --no-index --no-deps --target "
                    "baseline/_ref <reference checkout>)")
    ref, _ = _spawn(False, ignore, tmp_path)
    ours, info = _spawn(True, ignore, tmp_path)
    assert info["calls"] == {"forward": 1, "backward": 1}
    assert int(ours["n"]) == int(ref["n"]) > 0
    loss_ref, loss = float(ref["loss"]), float(ours["loss"])
    assert abs(loss - loss_ref) <= 1e-5 * abs(loss_ref), (loss, loss_ref)
    # A grad that is zero in exact arithmetic (the attention key bias: softmax
    # ignores a shift shared by a query's scores) holds only rounding noise
    # (~1e-9) in both runs, so each grad's error is relative to its own norm
    # or, if larger, to 1e-6 of the norm of all grads.
    total = np.sqrt(sum(float(np.sum(ref[f"g{i}"] ** 2)) for i in range(int(ref["n"]))))
    for i in range(int(ref["n"])):
        g_ref, g = ref[f"g{i}"], ours[f"g{i}"]
        assert g.shape == g_ref.shape
        err = np.linalg.norm(g - g_ref) / max(np.linalg.norm(g_ref), 1e-6 * total)
        assert err <= 1e-3, (i, err, float(np.linalg.norm(g_ref)))
