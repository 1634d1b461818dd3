"""Every GEMM tiling mode gives the same results.

The tiling is chosen once per process from NIMBLEML_TIED_CE_WIDE /
NIMBLEML_TIED_CE_CTA_PAIRS, so each mode runs in a child process: fp16
forward + backward of a ragged case, checked against the float64 oracle and
against the default mode (loss 2e-3, grads 1e-2 relative).
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import REPO
from oracle import tied_ce_oracle as orc

pytestmark = pytest.mark.gpu

CHILD = r"""
import json, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from nimbleml_b200.kernels import fused_tied_crossentropy as k
from oracle import tied_ce_oracle as orc
h, e, y = orc.make_inputs(700, 320, 2900, seed=31, unit_rms=True)
hd = torch.as_tensor(h).cuda().half(); ed = torch.as_tensor(e).cuda().half(); yd = torch.as_tensor(y).cuda()
loss, hh, ww, st, mx, se = k.fused_tied_crossentropy_forward(hd, ed, yd)
dh, de = k.shard_backward(torch.ones(1, device="cuda"), hh, ww, yd, st, grad_hidden_dtype=torch.float32,
                          grad_weights=torch.empty(ww.shape, dtype=torch.float32, device="cuda"), slab_bytes=700 * 2 * 1024)
torch.cuda.synchronize()
assert k.check_status(hd.device) == 0
np.save(sys.argv[2], np.concatenate([[float(loss)], dh.double().cpu().numpy().ravel(), de.double().cpu().numpy().ravel()]))
"""

MODES = {
    "default": {},
    "all_128x256": {"NIMBLEML_TIED_CE_WIDE": "0"},
    "all_wide": {"NIMBLEML_TIED_CE_WIDE": "15"},
    "all_cta_pairs": {"NIMBLEML_TIED_CE_CTA_PAIRS": "15"},
}


def run_mode(env_extra, out):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO), str(out)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return np.load(out)


def test_all_tilings_agree(tmp_path):
    h, e, y = orc.make_inputs(700, 320, 2900, seed=31, unit_rms=True)
    import torch

    l64, dh64, de64, _, _ = orc.row_chunked_reference(torch.as_tensor(h).half().double().numpy(),
                                                      torch.as_tensor(e).half().double().numpy(), y)
    n_dh = dh64.size
    results = {name: run_mode(env, tmp_path / f"{name}.npy") for name, env in MODES.items()}
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    for name, r in results.items():
        assert abs(r[0] - l64) <= 2e-3 * l64, name
        assert rel(r[1:1 + n_dh], dh64.ravel()) <= 1e-2, name
        assert rel(r[1 + n_dh:], de64.ravel()) <= 1e-2, name
        assert rel(r[1:], results["default"][1:]) <= 1e-4, name
