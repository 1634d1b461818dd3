"""Row kernels around the head (CE over logits, sampled CE, RMSNorm, embedding
grad, AdamW) against the reference's golden vectors and the float64 oracle.

Tolerances: fp32 inputs 1e-5 (loss) / 1e-4 (grads, no tensor cores involved);
fp16 / bf16 inputs 2e-3 (loss) / 1e-2 (grads), relative 2-norm.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import tied_ce_oracle as orc

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def g():
    return dict(np.load(GOLDEN / "row_kernels_f32.npz"))


def t(x, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(x)).cuda().to(dtype)


def test_ce_over_logits_reference_golden():
    from nimbleml_b200.losses import CrossEntropyLoss

    gd = g()
    x = t(gd["ce_logits"]).requires_grad_(True)
    loss = CrossEntropyLoss()(x, t(gd["ce_labels"], torch.int64), ignore_index=-1)
    loss.backward()
    assert abs(float(loss) - float(gd["ce_loss"])) <= 1e-5 * float(gd["ce_loss"])
    assert rel(x.grad.cpu(), gd["ce_grad"]) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 7), (130, 1001), (64, 50257)])
def test_ce_over_logits_half_vs_oracle(dtype, shape):
    from nimbleml_b200.losses import CrossEntropyLoss

    n, v = shape
    rng = np.random.default_rng(n + v)
    logits = (rng.standard_normal((n, v)) * 3).astype(np.float32)
    y = rng.integers(0, v, n)
    y[::5] = -1 if n > 1 else y[::5]
    x = t(logits, dtype).requires_grad_(True)
    loss = CrossEntropyLoss()(x, t(y, torch.int64), ignore_index=-1)
    loss.backward()
    xr = x.detach().double().cpu().numpy()
    l64, g64 = orc.ce_logits_loss_and_grad(xr, y, ignore_index=-1)
    assert abs(float(loss) - l64) <= 2e-3 * abs(l64)
    assert rel(x.grad.double().cpu(), g64) <= 1e-2


def test_sampled_ce_reference_golden_and_half():
    from nimbleml_b200.losses import SampledCrossEntropyLoss

    gd = g()
    x = t(gd["s_logits"]).requires_grad_(True)
    neg = gd["s_neg"]
    loss = SampledCrossEntropyLoss()(x, t(gd["s_labels"], torch.int64), num_samples=neg.shape[1],
                                     negative_indices=neg)
    loss.backward()
    assert abs(float(loss) - float(gd["s_loss"])) <= 1e-5 * float(gd["s_loss"])
    assert rel(x.grad.cpu(), gd["s_grad"]) <= 1e-4
    # fp16, larger, with sampled negatives and repeated candidates.
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((256, 3000)).astype(np.float32)
    y = rng.integers(0, 3000, 256)
    neg = rng.integers(0, 3000, (256, 40))
    xh = t(lg, torch.float16).requires_grad_(True)
    loss = SampledCrossEntropyLoss()(xh, t(y, torch.int64), num_samples=40, negative_indices=neg)
    loss.backward()
    l64, g64, _ = orc.sampled_ce_loss_and_grad(xh.detach().double().cpu().numpy(), y, neg)
    assert abs(float(loss) - l64) <= 2e-3 * l64
    assert rel(xh.grad.double().cpu(), g64) <= 1e-2


def test_sample_negative_indices_contract():
    from nimbleml_b200.losses import sample_negative_indices

    y = np.array([0, 5, 9, 3])
    neg = sample_negative_indices(10, y, 9, rng=np.random.default_rng(1))
    for i in range(4):
        assert y[i] not in neg[i] and len(set(neg[i])) == 9
    with pytest.raises(ValueError):
        sample_negative_indices(10, y, 10)


def test_rmsnorm_reference_golden():
    from nimbleml_b200.norm import rms_norm

    gd = g()
    x = t(gd["n_x"]).requires_grad_(True)
    gm = t(gd["n_gamma"]).requires_grad_(True)
    y = rms_norm(x, gm, 1e-5)
    y.backward(t(gd["n_gy"]))
    assert rel(y.detach().cpu(), gd["n_y"]) <= 1e-5
    assert rel(x.grad.cpu(), gd["n_gx"]) <= 1e-4
    assert rel(gm.grad.cpu(), gd["n_gg"]) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(3, 64), (1000, 4096), (37, 5000)])
def test_rmsnorm_vs_oracle(dtype, shape):
    from nimbleml_b200.norm import RMSNorm

    n, d = shape
    rng = np.random.default_rng(n * d)
    x = t(rng.standard_normal((n, d)) * 2, dtype).requires_grad_(True)
    layer = RMSNorm(d, device="cuda")
    with torch.no_grad():
        layer.gamma.copy_(t(1 + 0.1 * rng.standard_normal(d)))
    y = layer(x)
    gy = t(rng.standard_normal((n, d)), dtype)
    y.backward(gy)
    xr = x.detach().double().cpu().numpy()
    gr = layer.gamma.detach().to(dtype).double().cpu().numpy()
    y64, ms, rms = orc.rmsnorm_forward(xr, gr)
    gx64, gg64 = orc.rmsnorm_backward(gy.double().cpu().numpy(), xr, gr, ms, rms)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel(y.detach().double().cpu(), y64) <= tol
    assert rel(x.grad.double().cpu(), gx64) <= max(tol, 1e-4)
    assert rel(layer.gamma.grad.double().cpu(), gg64) <= max(tol, 1e-4)
    # Deterministic grad_gamma.
    layer.gamma.grad = None
    layer(x).backward(gy)
    g1 = layer.gamma.grad.clone()
    layer.gamma.grad = None
    layer(x).backward(gy)
    assert torch.equal(g1, layer.gamma.grad)


def test_embedding_scatter_add_and_adamw_reference_golden():
    from nimbleml_b200.embedding_grad import AdamW, embedding_scatter_add

    gd = g()
    gw = t(gd["e_gw"]).contiguous()
    embedding_scatter_add(gw, t(gd["e_ids"], torch.int64), t(gd["e_go"], torch.float16))
    ref = orc.embedding_scatter_add(gd["e_gw"], gd["e_ids"], gd["e_go"].astype(np.float16).astype(np.float32))
    assert rel(gw.cpu(), ref) <= 1e-6
    p = t(gd["a_w0"]).contiguous()
    copy = torch.empty(p.shape, dtype=torch.float16, device="cuda")
    opt = AdamW([p], learning_rate=1e-2, weight_decay=0.1, copies=[copy])
    for gr in gd["a_grads"]:
        p.grad = t(gr)
        opt.step()
    assert rel(p.cpu(), gd["a_w2"]) <= 1e-6
    assert rel(copy.float().cpu(), gd["a_w2"]) <= 1e-3
