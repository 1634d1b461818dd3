"""Pins the NumPy oracle to outputs of the reference itself (tests/golden)."""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle import tied_ce_oracle as orc


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300)


@pytest.mark.parametrize("name,dtype,tol", [
    ("small_f32", np.float32, 1e-6), ("small_f64", np.float64, 1e-12),
    ("ragged_f32", np.float32, 1e-6), ("tile_multi_f32", np.float32, 1e-6),
])
def test_kernel_level_matches_reference(name, dtype, tol):
    g = load(name)
    loss, h, w, logits, mx, se = orc.tied_forward(g["h"], g["e"], g["labels"], dtype)
    dh, de = orc.tied_backward(1.0, h, w, g["labels"], logits, mx, se)
    assert abs(loss - float(g["loss"])) <= tol * abs(float(g["loss"]))
    assert rel(mx.ravel(), g["max"]) <= tol
    assert rel(se.ravel(), g["sumexp"]) <= tol
    assert rel(dh, g["dh"]) <= tol
    assert rel(de, g["de"]) <= tol


def test_fp16_reference_path_restated():
    g = load("small_f16")
    h16, e16 = g["h"].astype(np.float16), g["e"].astype(np.float16)
    loss, h, w, logits, mx, se = orc.tied_forward(h16, e16, g["labels"], np.float16)
    dh, de = orc.tied_backward(1.0, h, w, g["labels"], logits, mx, se)
    # Same op order and dtypes as the reference's fp16 path: identical results
    # up to BLAS-vs-loop summation order in the fp16 matmul.
    assert abs(loss - float(g["ref16_loss"])) < 2e-3 * abs(float(g["ref16_loss"]))
    assert rel(dh, g["ref16_dh"]) < 5e-2
    assert rel(de, g["ref16_de"]) < 5e-2
    # The float64 run on fp16-rounded inputs (the fp16 parity target).
    l64, h64, w64, lg, mx64, se64 = orc.tied_forward(h16.astype(np.float64), e16.astype(np.float64),
                                                      g["labels"], np.float64)
    dh64, de64 = orc.tied_backward(1.0, h64, w64, g["labels"], lg, mx64, se64)
    assert abs(l64 - float(g["loss"])) < 1e-12 * l64
    assert rel(dh64, g["dh"]) < 1e-12 and rel(de64, g["de"]) < 1e-12


@pytest.mark.parametrize("name", ["ignore_f32", "all_ignored_f32"])
def test_forward_tied_ignore_index(name):
    g = load(name)
    n = int(g["b"]) * int(g["s"])
    loss, dh, de = orc.forward_tied_loss_and_grads(g["h"], g["e"], g["labels"], int(g["ignore_index"]))
    assert abs(loss - float(g["loss"])) <= 1e-6 * max(1.0, abs(float(g["loss"])))
    assert rel(dh, g["dh"]) <= 1e-6 or np.abs(g["dh"]).max() == 0 == np.abs(dh).max()
    assert rel(de, g["de"]) <= 1e-6 or np.abs(g["de"]).max() == 0 == np.abs(de).max()
    ignored = g["labels"] == int(g["ignore_index"])
    assert np.all(dh[ignored] == 0) and dh.shape == (n, int(g["d"]))


def test_tiny_gpt_head():
    g = load("c1_tiny_gpt")
    loss, dh, de = orc.forward_tied_loss_and_grads(g["h"], g["e"], g["labels"])
    assert abs(loss - float(g["loss"])) < 1e-6 * float(g["loss"])
    assert rel(dh, g["dh"]) < 1e-6 and rel(de, g["de"]) < 1e-6
    assert abs(float(g["model_loss"]) - 5.512688636779785) < 1e-6


@pytest.mark.parametrize("name", ["c2_slice_f32", "c3_slice_f16"])
def test_benchmark_shape_slices(name):
    g = load(name)
    n, d, v = int(g["n"]), int(g["d"]), int(g["v"])
    h, e, y = orc.make_inputs(n, d, v, seed=int(g["seed"]), unit_rms=bool(g["unit_rms"]))
    assert np.array_equal(y, g["labels"])
    if str(g["dtype"]) == "float16":
        h, e = h.astype(np.float16), e.astype(np.float16)
    loss, dh, de, mx, se = orc.row_chunked_reference(h, e, y, rows_per_chunk=64)
    tol = 1e-5 if str(g["dtype"]) == "float32" else 1e-10
    assert abs(loss - float(g["loss"])) < tol * loss
    assert rel(dh, g["dh"]) < 1e-3 if str(g["dtype"]) == "float32" else rel(dh, g["dh"]) < 1e-10
    rng = np.random.default_rng(int(g["seed"]) + 7)
    u_d = rng.standard_normal(d)
    u_v = rng.standard_normal(v)
    dtol = 1e-3 if str(g["dtype"]) == "float32" else 1e-9
    assert rel(de @ u_d, g["de_proj_d"]) < dtol
    assert rel(u_v @ de, g["de_proj_v"]) < dtol
    assert rel(de[g["de_rows_idx"]], g["de_rows"]) < dtol


@pytest.mark.parametrize("p", [1, 2, 3, 8])
def test_sharded_combine_equals_full(p):
    h, e, y = orc.make_inputs(40, 24, 203, seed=5, ignore_frac=0.2, ignore_index=-1)
    st = orc.sharded_stats(h, e, y, p)
    m, s, lse, loss, nv = orc.combine_stats(st, y, 203, ignore_index=-1)
    l64, dh, de, mx, se = orc.row_chunked_reference(h, e, y, ignore_index=-1)
    assert abs(loss - l64) < 1e-12 * l64
    assert np.allclose(m, mx) and np.allclose(s, se, rtol=1e-12)
    assert nv == int(np.sum(y != -1))


def test_tied_logits_head_matches_reference():
    g = load("tied_logits_c1")
    logits = orc.tied_logits_forward(g["x"], g["e"])
    dx, de = orc.tied_logits_backward(g["grad_out"], g["x"], g["e"])
    assert rel(logits, g["logits"]) < 1e-6
    assert rel(dx, g["dx"]) < 1e-6 and rel(de, g["de"]) < 1e-6


def test_row_kernel_restatements_match_reference():
    g = load("row_kernels_f32")
    lg = g["ce_logits"].reshape(-1, g["ce_logits"].shape[-1])
    loss, grad = orc.ce_logits_loss_and_grad(lg, g["ce_labels"], ignore_index=-1)
    assert abs(loss - float(g["ce_loss"])) < 1e-6 * float(g["ce_loss"])
    assert rel(grad, g["ce_grad"].reshape(lg.shape)) < 1e-6
    sloss, sgrad, _ = orc.sampled_ce_loss_and_grad(g["s_logits"], g["s_labels"], g["s_neg"])
    assert abs(sloss - float(g["s_loss"])) < 1e-6 * float(g["s_loss"])
    assert rel(sgrad, g["s_grad"]) < 1e-6
    y, ms, rms = orc.rmsnorm_forward(g["n_x"], g["n_gamma"])
    assert rel(y, g["n_y"]) < 1e-6 and rel(rms.ravel(), g["n_rms"]) < 1e-6
    gx, gg = orc.rmsnorm_backward(g["n_gy"], g["n_x"], g["n_gamma"], ms, rms)
    assert rel(gx, g["n_gx"]) < 1e-5 and rel(gg, g["n_gg"]) < 1e-5
    assert rel(orc.embedding_scatter_add(g["e_gw"], g["e_ids"], g["e_go"]), g["e_out"]) < 1e-6
    w, m, v = g["a_w0"].astype(np.float64), 0.0, 0.0
    for t, gr in enumerate(g["a_grads"], start=1):
        w, m, v = orc.adamw_step(w, gr.astype(np.float64), m, v, 1e-2, 0.9, 0.999, 1 - 0.9 ** t,
                                 1 - 0.999 ** t, 1e-8, 0.1)
    assert rel(w, g["a_w2"]) < 1e-6


def test_tied_embedding_composition_matches_reference():
    """Lookup + tied head + scatter-add into one grad, then AdamW (reference Embedding /
    forward_tied / AdamW), restated by the oracle in the reference's order."""
    g = load("tied_embedding_adamw_f32")
    e0, ids, y = g["e0"], g["ids"].reshape(-1), g["labels"]
    h = e0[ids]
    loss, dh, de_head = orc.forward_tied_loss_and_grads(h, e0, y, ignore_index=-1)
    assert abs(loss - float(g["loss"])) < 1e-6 * float(g["loss"])
    grad = orc.embedding_scatter_add(de_head.astype(np.float32), ids, dh.astype(np.float32))
    assert rel(grad, g["grad"]) < 1e-5
    w, m, v = orc.adamw_step(e0.astype(np.float64), g["grad"].astype(np.float64), 0.0, 0.0, float(g["lr"]),
                             float(g["b1"]), float(g["b2"]), 1 - float(g["b1"]), 1 - float(g["b2"]),
                             float(g["eps"]), float(g["wd"]))
    assert rel(w, g["e1"]) < 1e-6


def test_norm_head_composition_matches_reference():
    """Final RMSNorm then the tied head (reference RMSNorm + forward_tied), restated."""
    g = load("norm_head_f32")
    d = g["x"].shape[-1]
    x = g["x"].reshape(-1, d)
    yv, ms, rms = orc.rmsnorm_forward(x, g["gamma"], float(g["eps"]))
    loss, dy, de = orc.forward_tied_loss_and_grads(yv, g["e"], g["labels"])
    assert abs(loss - float(g["loss"])) < 1e-6 * float(g["loss"])
    assert rel(de, g["de"]) < 1e-5
    dx, dgamma = orc.rmsnorm_backward(dy, x, g["gamma"], ms, rms, float(g["eps"]))
    assert rel(dx, g["dx"].reshape(-1, d)) < 1e-5
    assert rel(dgamma, g["dgamma"]) < 1e-5
