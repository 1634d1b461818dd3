"""Tied LM-head logits (GPT._tied_logits) on the sm_100a GEMM vs the reference / oracle.

fp16 / bf16 inputs with fp32 accumulation; tolerance 1e-2 relative (the
fp16 grad tolerance of the parity tests), against the reference's fp32
golden (inputs rounded to the compute dtype first) and the float64 oracle.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import tied_ce_oracle as orc

pytestmark = pytest.mark.gpu
TOL = 1e-2


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_tiny_gpt_tied_logits_against_reference_golden():
    from nimbleml_b200.lm_head import tied_logits

    g = dict(np.load(GOLDEN / "tied_logits_c1.npz"))
    x = torch.as_tensor(g["x"]).cuda().half().requires_grad_(True)
    e = torch.as_tensor(g["e"]).cuda().float().requires_grad_(True)   # fp32 master weights
    out = tied_logits(x, e)
    assert out.shape == (2, 8, 256) and out.dtype == torch.float16
    out.backward(torch.as_tensor(g["grad_out"]).cuda().half())
    assert rel(out.detach().float().cpu(), g["logits"]) < TOL
    assert rel(x.grad.float().cpu(), g["dx"]) < TOL
    assert e.grad.dtype == torch.float32
    assert rel(e.grad.cpu(), g["de"]) < TOL


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(3, 77, 136, 1001), (2, 300, 256, 5003)])
def test_tied_logits_against_oracle(dtype, shape):
    from nimbleml_b200.lm_head import last_token_logits, tied_logits

    b, s, d, v = shape
    h, e, _ = orc.make_inputs(b * s, d, v, seed=b + s + v, unit_rms=True)
    gr = np.random.default_rng(5).standard_normal((b, s, v)).astype(np.float32)
    x = torch.as_tensor(h.reshape(b, s, d)).cuda().to(dtype).requires_grad_(True)
    w = torch.as_tensor(e).cuda().to(dtype).requires_grad_(True)
    gd = torch.as_tensor(gr).cuda().to(dtype)
    out = tied_logits(x, w)
    out.backward(gd)
    r = lambda t: t.detach().to(torch.float64).cpu().numpy()
    ref = orc.tied_logits_forward(r(x), r(w))
    dx, dw = orc.tied_logits_backward(r(gd), r(x), r(w))
    assert rel(r(out), ref) < TOL
    assert rel(r(x.grad), dx) < TOL and rel(r(w.grad), dw) < TOL
    last = last_token_logits(x.detach(), w.detach())
    assert last.shape == (b, v)
    assert torch.equal(last, out.detach()[:, -1, :])


def test_tied_logits_shape_errors():
    from nimbleml_b200.lm_head import tied_logits

    with pytest.raises(ValueError, match="d_model mismatch"):
        tied_logits(torch.zeros(2, 3, 8, device="cuda", dtype=torch.float16),
                    torch.zeros(10, 16, device="cuda", dtype=torch.float16))
