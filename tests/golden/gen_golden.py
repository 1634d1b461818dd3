"""Generate golden vectors for the tied-CE path by running the REFERENCE itself.

Imports the reference NimbleML package (CPU backend) with its native
extension compiled from source by ``oracle/Makefile`` and records seeded
inputs and outputs of

* ``GPT.compute_loss`` + ``backward`` on the tiny GPT of config 1
  (NimbleML/models/gpt.py:123-137),
* ``fused_tied_crossentropy_forward / _backward``
  (NimbleML/kernels/fused_tied_crossentropy.py:8-48) in float32, float64 and
  float16,
* ``CrossEntropyLoss.forward_tied`` with ``ignore_index``
  (NimbleML/losses/cross_entropy.py:109-192),

as ``.npz`` files beside this script. Run in a container that has the
reference checkout (it is not needed afterwards):

    make -C oracle REF=<reference checkout>
    python tests/golden/gen_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import os
import random
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
from oracle.tied_ce_oracle import make_inputs  # noqa: E402


def _import_reference(ref: Path):
    os.environ["NIMBLEML_DEVICE"] = "cpu"
    sys.path.insert(0, str(REPO / "oracle" / "_ref"))
    sys.path.insert(0, str(ref))
    import NimbleML  # noqa: F401
    from NimbleML.utils import np_backend
    return np_backend


def kernel_case(nb, name, n, d, v, seed, dtype, unit_rms=False, store_inputs=True, force_edges=False):
    from NimbleML.kernels import fused_tied_crossentropy_backward, fused_tied_crossentropy_forward

    h, e, y = make_inputs(n, d, v, seed=seed, unit_rms=unit_rms)
    if force_edges:
        y[0], y[-1] = 0, v - 1
    out = {"n": n, "d": d, "v": v, "seed": seed, "unit_rms": unit_rms, "labels": y}
    if store_inputs:
        out.update(h=h, e=e)
    if dtype == "float16":
        # The parity target for fp16: the reference run in float64 on the
        # fp16-rounded inputs; the reference's own fp16 result is kept for
        # information (its backward flushes p/N to zero in fp16).
        h16, e16 = h.astype(np.float16), e.astype(np.float16)
        nb.set_dtype("float64")
        loss, hh, ww, logits, mx, se = fused_tied_crossentropy_forward(h16.astype(np.float64),
                                                                       e16.astype(np.float64), y)
        gh, gw = fused_tied_crossentropy_backward(1.0, hh, ww, y, logits, mx, se)
        out.update(loss=loss, max=mx.ravel(), sumexp=se.ravel(), dh=gh, de=gw)
        nb.set_dtype("float16")
        loss16, hh, ww, logits, mx, se = fused_tied_crossentropy_forward(h16, e16, y)
        gh16, gw16 = fused_tied_crossentropy_backward(1.0, hh, ww, y, logits, mx, se)
        out.update(ref16_loss=loss16, ref16_dh=gh16, ref16_de=gw16)
    else:
        nb.set_dtype(dtype)
        loss, hh, ww, logits, mx, se = fused_tied_crossentropy_forward(h, e, y)
        gh, gw = fused_tied_crossentropy_backward(1.0, hh, ww, y, logits, mx, se)
        out.update(loss=loss, max=mx.ravel(), sumexp=se.ravel(), dh=gh, de=gw)
    out["dtype"] = dtype
    return name, out


def projected(out, seed):
    """Replace a large dE with fixed projections (the fixture stays small)."""
    rng = np.random.default_rng(seed + 7)
    de = np.asarray(out.pop("de"), np.float64)
    u_d = rng.standard_normal(de.shape[1])
    u_v = rng.standard_normal(de.shape[0])
    rows = np.unique(np.concatenate([out["labels"][:16], rng.integers(0, de.shape[0], 16)]))
    out.update(de_proj_d=de @ u_d, de_proj_v=u_v @ de, de_rows_idx=rows, de_rows=de[rows],
               de_norm=np.linalg.norm(de))
    return out


def ignore_case(nb, name, b, s, d, v, seed, ignore_index, frac, dtype="float32"):
    from NimbleML.losses.cross_entropy import CrossEntropyLoss
    from NimbleML.utils.tensor import Tensor

    nb.set_dtype(dtype)
    h, e, y = make_inputs(b * s, d, v, seed=seed, ignore_frac=frac, ignore_index=ignore_index)
    ht = Tensor(h.ravel(), (b, s, d), requires_grad=True)
    et = Tensor(e.ravel(), (v, d), requires_grad=True)
    loss = CrossEntropyLoss().forward_tied(ht, et, y.reshape(b, s), ignore_index=ignore_index)
    loss.backward()
    dh = np.zeros((b * s, d), np.float32) if ht.grad is None else np.asarray(ht.grad).reshape(b * s, d)
    de = np.zeros((v, d), np.float32) if et.grad is None else np.asarray(et.grad).reshape(v, d)
    return name, {"b": b, "s": s, "d": d, "v": v, "seed": seed, "ignore_index": ignore_index,
                  "h": h, "e": e, "labels": y, "loss": loss.item(), "dh": dh, "de": de,
                  "grads_present": np.array([ht.grad is not None, et.grad is not None])}


def tiny_gpt_case(nb):
    from NimbleML import GPT, Tensor
    from NimbleML.losses.cross_entropy import CrossEntropyLoss

    nb.set_dtype("float32")
    random.seed(0)
    np.random.seed(0)
    m = GPT(vocab_size=256, d_model=64, num_heads=4, num_layers=2, max_seq_len=32, fused_blocks=True)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 256, (2, 8), dtype=np.int64)
    lab = rng.integers(0, 256, (2, 8), dtype=np.int64)
    loss = m.compute_loss(Tensor.from_int64(ids, (2, 8)), Tensor.from_int64(lab, (2, 8)))
    loss.backward()
    model_loss = loss.item()
    emb_grad_norm = float(np.linalg.norm(m.token_emb.weights.grad))
    hidden = np.asarray(m._hidden_states(Tensor.from_int64(ids, (2, 8)))._view()).astype(np.float32)
    e = np.asarray(m.token_emb.weights._view()).astype(np.float32)
    ht = Tensor(hidden.ravel(), (2, 8, 64), requires_grad=True)
    et = Tensor(e.ravel(), e.shape, requires_grad=True)
    head = CrossEntropyLoss().forward_tied(ht, et, lab)
    head.backward()
    return "c1_tiny_gpt", {"ids": ids, "labels": lab.ravel(), "model_loss": model_loss,
                           "model_emb_grad_norm": emb_grad_norm, "h": hidden.reshape(16, 64), "e": e,
                           "loss": head.item(), "dh": np.asarray(ht.grad).reshape(16, 64),
                           "de": np.asarray(et.grad).reshape(e.shape)}


def tied_logits_case(nb):
    """GPT._tied_logits forward and backward on the tiny GPT (config 1 sizes)."""
    from NimbleML import GPT, Tensor

    nb.set_dtype("float32")
    random.seed(0)
    np.random.seed(0)
    m = GPT(vocab_size=256, d_model=64, num_heads=4, num_layers=2, max_seq_len=32, fused_blocks=True)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((2, 8, 64), dtype=np.float32)
    g = rng.standard_normal((2, 8, 256), dtype=np.float32)
    xt = Tensor(x.ravel(), (2, 8, 64), requires_grad=True)
    m.token_emb.weights.zero_grad(set_to_none=True)
    out = m._tied_logits(xt)
    out.backward(g.ravel())
    e = np.asarray(m.token_emb.weights._view()).astype(np.float32)
    return "tied_logits_c1", {"x": x, "e": e, "grad_out": g, "logits": np.asarray(out._view()),
                              "dx": np.asarray(xt.grad).reshape(2, 8, 64),
                              "de": np.asarray(m.token_emb.weights.grad).reshape(e.shape),
                              "loss": 0.0}


def row_kernels_case(nb):
    """Reference outputs for the row kernels around the head (fp32)."""
    from NimbleML.kernels import (embedding_scatter_add, fused_rmsnorm_backward, fused_rmsnorm_forward,
                                  sampled_softmax_backward, sampled_softmax_forward)
    from NimbleML.losses.cross_entropy import CrossEntropyLoss
    from NimbleML.utils.tensor import Tensor

    nb.set_dtype("float32")
    rng = np.random.default_rng(3)
    out = {"loss": 0.0}
    # Untied CE on (B, S, V) logits with ignore_index=-1.
    logits = rng.standard_normal((3, 10, 77), dtype=np.float32) * 2
    labels = rng.integers(0, 77, (3, 10))
    labels[0, :3] = -1
    lt = Tensor(logits.ravel(), logits.shape, requires_grad=True)
    loss = CrossEntropyLoss().forward(lt, labels, ignore_index=-1)
    loss.backward()
    out.update(ce_logits=logits, ce_labels=labels, ce_loss=loss.item(),
               ce_grad=np.asarray(lt.grad).reshape(logits.shape))
    # Sampled softmax with fixed negatives (num_samples 7, V 50).
    sl = rng.standard_normal((12, 50), dtype=np.float32)
    sy = rng.integers(0, 50, 12)
    neg = np.stack([rng.choice(np.delete(np.arange(50), sy[i]), 7, replace=False) for i in range(12)])
    sloss, lg, cand, mx, se = sampled_softmax_forward(sl, sy, neg)
    sgrad = sampled_softmax_backward(1.0, lg, cand, mx, se)
    out.update(s_logits=sl, s_labels=sy, s_neg=neg, s_loss=sloss, s_grad=sgrad)
    # RMSNorm forward / backward.
    x = rng.standard_normal((9, 96), dtype=np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(96)).astype(np.float32)
    y, xs, ms, rms = fused_rmsnorm_forward(x, gamma, 1e-5)
    gy = rng.standard_normal((9, 96), dtype=np.float32)
    gx, gg = fused_rmsnorm_backward(gy, xs, gamma, ms, rms, 1e-5)
    out.update(n_x=x, n_gamma=gamma, n_y=y, n_ms=np.asarray(ms).ravel(), n_rms=np.asarray(rms).ravel(), n_gy=gy,
               n_gx=gx, n_gg=gg)
    # Embedding scatter-add with repeated ids.
    gw = rng.standard_normal((40, 24), dtype=np.float32)
    ids = rng.integers(0, 40, 64)
    ids[:8] = 5
    go = rng.standard_normal((64, 24), dtype=np.float32)
    res = embedding_scatter_add(gw.copy(), ids, go)
    out.update(e_gw=gw, e_ids=ids, e_go=go, e_out=np.asarray(res))
    # Two AdamW steps on one fp32 parameter (reference optimizer, CPU path).
    from NimbleML.optimizers import AdamW

    w0 = rng.standard_normal(300).astype(np.float32)
    grads = rng.standard_normal((2, 300)).astype(np.float32)
    prm = Tensor(w0.copy(), (300,), requires_grad=True)
    opt = AdamW([prm], learning_rate=1e-2, weight_decay=0.1)
    for g in grads:
        prm.grad = g.copy()
        opt.step()
    out.update(a_w0=w0, a_grads=grads, a_w2=np.asarray(prm.data).reshape(-1).copy())
    return "row_kernels_f32", out


def tied_embedding_case(nb):
    """The tied matrix used twice — input embedding lookup and tied LM head —
    through the reference's Embedding (NimbleML/layers/embedding.py:23-67,138-148),
    forward_tied (NimbleML/losses/cross_entropy.py:109-192) and one AdamW step
    (NimbleML/optimizers/adam.py:85-131,295-312), fp32. E.grad is the head's dE
    plus the lookup's scatter-add (with repeated ids)."""
    from NimbleML.layers import Embedding
    from NimbleML.losses.cross_entropy import CrossEntropyLoss
    from NimbleML.optimizers import AdamW
    from NimbleML.utils.tensor import Tensor

    nb.set_dtype("float32")
    np.random.seed(5)
    v, d, b, s = 300, 64, 4, 32
    emb = Embedding(v, d, init_std=0.5)
    rng = np.random.default_rng(6)
    ids = rng.integers(0, v, (b, s), dtype=np.int64)
    ids[:, ::4] = 7  # a frequent token: many rows scatter into one grad row
    labels = rng.integers(0, v, (b, s), dtype=np.int64)
    labels[0, :5] = -1
    e0 = np.asarray(emb.weights._view()).astype(np.float32).copy()
    h = emb(Tensor.from_int64(ids, (b, s)))
    loss = CrossEntropyLoss().forward_tied(h, emb.weights, labels, ignore_index=-1)
    loss.backward()
    grad = np.asarray(emb.weights.grad).reshape(v, d).astype(np.float32).copy()
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.999, 1e-8, 0.01
    opt = AdamW([emb.weights], learning_rate=lr, beta1=b1, beta2=b2, epsilon=eps, weight_decay=wd)
    opt.step()
    e1 = np.asarray(emb.weights._view()).astype(np.float32).copy()
    return "tied_embedding_adamw_f32", {"ids": ids, "labels": labels.ravel(), "e0": e0, "grad": grad, "e1": e1,
                                        "loss": loss.item(), "lr": lr, "b1": b1, "b2": b2, "eps": eps, "wd": wd}


def norm_head_case(nb):
    """The final RMSNorm feeding the tied head (NimbleML/models/gpt.py:67,90,
    NimbleML/layers/rms_norm.py:25-95) then forward_tied, fp32: loss and the
    grads of x, gamma and E."""
    from NimbleML.layers import RMSNorm
    from NimbleML.losses.cross_entropy import CrossEntropyLoss
    from NimbleML.utils.tensor import Tensor

    nb.set_dtype("float32")
    np.random.seed(8)
    v, d, b, s = 500, 128, 3, 40
    norm = RMSNorm(d)
    rng = np.random.default_rng(9)
    norm.gamma.data[...] = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    x = (2.0 * rng.standard_normal((b, s, d))).astype(np.float32)
    e = (0.05 * rng.standard_normal((v, d))).astype(np.float32)
    labels = rng.integers(0, v, (b, s), dtype=np.int64)
    xt = Tensor(x.ravel(), (b, s, d), requires_grad=True)
    et = Tensor(e.ravel(), (v, d), requires_grad=True)
    loss = CrossEntropyLoss().forward_tied(norm(xt), et, labels)
    loss.backward()
    return "norm_head_f32", {"x": x, "e": e, "gamma": np.asarray(norm.gamma.data).astype(np.float32).copy(),
                             "labels": labels.ravel(), "loss": loss.item(), "eps": norm.epsilon,
                             "dx": np.asarray(xt.grad).reshape(b, s, d), "de": np.asarray(et.grad).reshape(v, d),
                             "dgamma": np.asarray(norm.gamma.grad).reshape(d)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NIMBLEML_REFERENCE"),
                    help="the reference checkout (or set NIMBLEML_REFERENCE)")
    ap.add_argument("--only", nargs="*", help="write only these fixtures (file stems)")
    args = ap.parse_args()
    if not args.ref or not (Path(args.ref) / "NimbleML").is_dir():
        raise SystemExit("pass --ref <reference checkout> (or set NIMBLEML_REFERENCE); its native extension must "
                         "be built into oracle/_ref first: make -C oracle REF=<checkout>")
    nb = _import_reference(Path(args.ref))
    if args.only:
        makers = {"tied_embedding_adamw_f32": tied_embedding_case, "norm_head_f32": norm_head_case,
                  "c1_tiny_gpt": tiny_gpt_case, "tied_logits_c1": tied_logits_case,
                  "row_kernels_f32": row_kernels_case}
        for stem in args.only:
            name, data = makers[stem](nb)
            path = HERE / f"{name}.npz"
            np.savez_compressed(path, **{k: np.asarray(v) for k, v in data.items()})
            print(f"{path.name}: {path.stat().st_size / 1024:.0f} KiB, loss={float(data['loss']):.6f}")
        return
    cases = [
        tied_embedding_case(nb),
        norm_head_case(nb),
        tiny_gpt_case(nb),
        tied_logits_case(nb),
        row_kernels_case(nb),
        kernel_case(nb, "small_f32", 96, 64, 1000, 11, "float32"),
        kernel_case(nb, "small_f64", 96, 64, 1000, 11, "float64"),
        kernel_case(nb, "ragged_f32", 77, 40, 257, 12, "float32", force_edges=True),
        kernel_case(nb, "tile_multi_f32", 300, 192, 1300, 13, "float32", force_edges=True),
        kernel_case(nb, "small_f16", 64, 64, 2048, 14, "float16", unit_rms=True),
        ignore_case(nb, "ignore_f32", 4, 16, 32, 300, 15, -1, 0.25),
        ignore_case(nb, "all_ignored_f32", 2, 8, 32, 100, 16, -1, 1.01),
    ]
    name, c2 = kernel_case(nb, "c2_slice_f32", 64, 768, 50257, 21, "float32", store_inputs=False)
    cases.append((name, projected(c2, 21)))
    name, c3 = kernel_case(nb, "c3_slice_f16", 32, 2048, 32000, 31, "float16", unit_rms=True,
                           store_inputs=False)
    for k in ("ref16_dh", "ref16_de"):
        c3.pop(k)
    cases.append((name, projected(c3, 31)))
    for name, data in cases:
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **{k: np.asarray(v) for k, v in data.items()})
        print(f"{path.name}: {path.stat().st_size / 1024:.0f} KiB, loss={float(data['loss']):.6f}")


if __name__ == "__main__":
    main()
