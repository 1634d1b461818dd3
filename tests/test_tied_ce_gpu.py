"""Parity of the sm_100a tied-CE path against the oracle and the reference's golden vectors.

Tolerances (from the path's specification), relative, rel(a, b) = |a-b|_2 / |b|_2:
  fp32 inputs (TF32 tensor cores):  loss <= 1e-5, grads <= 1e-3
  fp16 / bf16 inputs:               loss <= 2e-3, grads <= 1e-2
fp16/bf16 results are compared with the reference's math run in float64 on
the same fp16/bf16-rounded inputs (the reference's own fp16 backward flushes
p/N to zero and is not a usable target).
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import tied_ce_oracle as orc

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-3), torch.float16: (2e-3, 1e-2), torch.bfloat16: (2e-3, 1e-2)}


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def golden(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def to_dev(x, dtype):
    return torch.as_tensor(np.ascontiguousarray(x)).to("cuda").to(dtype).contiguous()


def rounded64(x, dtype):
    """Host copy of x after rounding to the device compute dtype, as float64."""
    return torch.as_tensor(np.ascontiguousarray(x)).to(dtype).to(torch.float64).numpy()


def run_path(h, e, y, dtype, ignore_index=None, slab_bytes=None, grad_scale=1.0):
    """Forward + backward through the public kernels (C ABI underneath)."""
    from nimbleml_b200.kernels import fused_tied_crossentropy as k

    hd, ed = to_dev(h, dtype), to_dev(e, dtype)
    yd = torch.as_tensor(y).to("cuda")
    loss, hh, ww, stats, mx, se = k.fused_tied_crossentropy_forward(hd, ed, yd, ignore_index=ignore_index)
    gs = torch.full((1,), grad_scale, device="cuda")
    dh, de = k.shard_backward(gs, hh, ww, yd, stats, slab_bytes=slab_bytes)
    torch.cuda.synchronize()
    assert k.check_status(hd.device) == 0
    f = lambda t: t.double().cpu().numpy()
    return float(loss), f(mx).ravel(), f(se).ravel(), f(stats.lse), f(dh), f(de)


@pytest.fixture(autouse=True)
def _device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from nimbleml_b200._native_loader import native

    assert native.available(), "needs a compute capability 10.x device"
    yield


@pytest.mark.parametrize("name", ["small_f32", "ragged_f32", "tile_multi_f32"])
def test_fp32_goldens(name):
    g = golden(name)
    lt, gt = TOL[torch.float32]
    loss, mx, se, lse, dh, de = run_path(g["h"], g["e"], g["labels"], torch.float32)
    assert abs(loss - float(g["loss"])) <= lt * abs(float(g["loss"]))
    assert rel(mx, g["max"]) <= 1e-3
    assert rel(se, g["sumexp"]) <= 1e-3
    assert rel(dh, g["dh"]) <= gt
    assert rel(de, g["de"]) <= gt


def test_fp16_golden_against_float64_reference():
    g = golden("small_f16")
    lt, gt = TOL[torch.float16]
    loss, mx, se, lse, dh, de = run_path(g["h"], g["e"], g["labels"], torch.float16)
    assert abs(loss - float(g["loss"])) <= lt * float(g["loss"])
    assert rel(dh, g["dh"]) <= gt
    assert rel(de, g["de"]) <= gt
    # For information: the reference's own fp16 result is far less accurate.
    print("ref-fp16 dh rel err vs f64:", rel(g["ref16_dh"], g["dh"]), "ours:", rel(dh, g["dh"]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 8, 16), (257, 64, 513), (300, 136, 1000), (640, 256, 3000)])
def test_oracle_parity_dtypes_and_ragged_shapes(dtype, shape):
    n, d, v = shape
    h, e, y = orc.make_inputs(n, d, v, seed=n + d + v, unit_rms=True)
    y[0] = 0
    y[-1] = v - 1
    lt, gt = TOL[dtype]
    loss, mx, se, lse, dh, de = run_path(h, e, y, dtype)
    l64, dh64, de64, mx64, se64 = orc.row_chunked_reference(rounded64(h, dtype), rounded64(e, dtype), y)
    assert abs(loss - l64) <= lt * l64
    assert rel(lse, mx64 + np.log(se64)) <= lt
    assert rel(dh, dh64) <= gt
    assert rel(de, de64) <= gt


def test_multi_slab_backward_matches_single_slab():
    n, d, v = 384, 128, 2100
    h, e, y = orc.make_inputs(n, d, v, seed=9, unit_rms=True)
    one = run_path(h, e, y, torch.float16)
    # 256-column slabs: 9 slabs, dh accumulated in the fp32 scratch.
    many = run_path(h, e, y, torch.float16, slab_bytes=2 * 384 * 256)
    assert one[0] == many[0]
    # dh: fp32 partial sums over slabs vs one fp32 accumulation, then fp16
    # output rounding; dE rows of each slab are computed identically.
    assert rel(many[4], one[4]) < 2e-4
    assert np.array_equal(many[5], one[5])
    l64, dh64, de64, _, _ = orc.row_chunked_reference(rounded64(h, torch.float16), rounded64(e, torch.float16), y)
    assert rel(many[4], dh64) < 1e-2 and rel(many[5], de64) < 1e-2


def test_deterministic_bitwise():
    h, e, y = orc.make_inputs(500, 192, 1500, seed=4, unit_rms=True)
    a = run_path(h, e, y, torch.float16)
    b = run_path(h, e, y, torch.float16)
    assert a[0] == b[0]
    for x, z in zip(a[1:], b[1:]):
        assert np.array_equal(x, z)


def test_grad_scale_is_applied():
    h, e, y = orc.make_inputs(130, 64, 700, seed=5, unit_rms=True)
    a = run_path(h, e, y, torch.float32, grad_scale=1.0)
    b = run_path(h, e, y, torch.float32, grad_scale=0.25)
    assert rel(b[4], 0.25 * a[4]) < 1e-6 and rel(b[5], 0.25 * a[5]) < 1e-6


@pytest.mark.parametrize("name", ["ignore_f32", "all_ignored_f32"])
def test_forward_tied_autograd_ignore_index(name):
    from nimbleml_b200.losses import CrossEntropyLoss

    g = golden(name)
    b, s, d, v = int(g["b"]), int(g["s"]), int(g["d"]), int(g["v"])
    ign = int(g["ignore_index"])
    hid = to_dev(g["h"].reshape(b, s, d), torch.float32).requires_grad_(True)
    emb = to_dev(g["e"], torch.float32).requires_grad_(True)
    labels = torch.as_tensor(g["labels"].reshape(b, s)).cuda()
    loss = CrossEntropyLoss().forward_tied(hid, emb, labels, ignore_index=ign)
    loss.backward()
    torch.cuda.synchronize()
    lt, gt = TOL[torch.float32]
    assert abs(float(loss) - float(g["loss"])) <= lt * max(1.0, abs(float(g["loss"])))
    dh = hid.grad.reshape(b * s, d).double().cpu().numpy()
    de = emb.grad.double().cpu().numpy()
    ignored = g["labels"] == ign
    assert np.all(dh[ignored] == 0.0)
    if ignored.all():
        assert float(loss) == 0.0 and not dh.any() and not de.any()
    else:
        assert rel(dh, g["dh"]) <= gt and rel(de, g["de"]) <= gt


def test_tiny_gpt_head_config1():
    """Config 1: the tiny GPT's hidden states and tied E through forward_tied + backward."""
    from nimbleml_b200.losses import CrossEntropyLoss

    g = golden("c1_tiny_gpt")
    hid = to_dev(g["h"].reshape(2, 8, 64), torch.float32).requires_grad_(True)
    emb = to_dev(g["e"], torch.float32).requires_grad_(True)
    loss = CrossEntropyLoss().forward_tied(hid, emb, torch.as_tensor(g["labels"].reshape(2, 8)).cuda())
    loss.backward()
    lt, gt = TOL[torch.float32]
    assert abs(float(loss) - float(g["loss"])) <= lt * float(g["loss"])
    assert rel(hid.grad.reshape(16, 64).cpu().numpy(), g["dh"]) <= gt
    assert rel(emb.grad.cpu().numpy(), g["de"]) <= gt


def test_tied_grad_accumulates_with_embedding_lookup():
    """E.grad = head grad + lookup grad when E is also the input embedding."""
    from nimbleml_b200.losses import CrossEntropyLoss

    n, d, v = 64, 64, 500
    h, e, y = orc.make_inputs(n, d, v, seed=6)
    emb = to_dev(e, torch.float32).requires_grad_(True)
    ids = torch.as_tensor(y).cuda()
    hid = (emb[ids] + to_dev(h, torch.float32)).reshape(4, 16, d)
    loss = CrossEntropyLoss().forward_tied(hid, emb, torch.roll(ids, 1).reshape(4, 16))
    loss.backward()
    emb2 = to_dev(e, torch.float32).requires_grad_(True)
    hid2 = (emb2[ids] + to_dev(h, torch.float32)).reshape(4, 16, d)
    logits = hid2.reshape(n, d) @ emb2.T
    ref = torch.nn.functional.cross_entropy(logits.double(), torch.roll(ids, 1))
    ref.backward()
    assert abs(float(loss) - float(ref)) < 1e-5 * float(ref)
    assert rel(emb.grad.cpu().numpy(), emb2.grad.cpu().numpy()) < 1e-3


def test_bad_label_sets_status():
    from nimbleml_b200.kernels import fused_tied_crossentropy as k

    h, e, y = orc.make_inputs(40, 32, 100, seed=8)
    y[3] = 100  # == V: out of range, not ignore_index
    loss = k.fused_tied_crossentropy_forward(to_dev(h, torch.float32), to_dev(e, torch.float32),
                                             torch.as_tensor(y).cuda())[0]
    torch.cuda.synchronize()
    # Visible without reading the status word: the loss is NaN.
    assert np.isnan(float(loss))
    with pytest.raises(ValueError, match="out of range"):
        k.check_status(torch.device("cuda", torch.cuda.current_device()))


def test_bad_label_raises_on_a_later_call_without_sync():
    """The asynchronous status copy taken at the end of one call is read by a
    later call (no host sync in between) and raises there."""
    from nimbleml_b200.kernels import fused_tied_crossentropy as k

    h, e, y = orc.make_inputs(40, 32, 100, seed=8)
    yb = y.copy()
    yb[5] = -7  # negative, not ignore_index
    hd, ed = to_dev(h, torch.float16), to_dev(e, torch.float16)
    k.fused_tied_crossentropy_forward(hd, ed, torch.as_tensor(yb).cuda())
    torch.cuda.synchronize()  # only so the status copy has landed before the next call
    with pytest.raises(ValueError, match="out of range"):
        k.fused_tied_crossentropy_forward(hd, ed, torch.as_tensor(y).cuda())
    # Raising cleared the word: the path runs again.
    loss = k.fused_tied_crossentropy_forward(hd, ed, torch.as_tensor(y).cuda())[0]
    torch.cuda.synchronize()
    assert np.isfinite(float(loss)) and k.check_status(hd.device) == 0


@pytest.mark.parametrize("name,dtype", [("c2_slice_f32", torch.float32), ("c3_slice_f16", torch.float16)])
def test_benchmark_shape_slices_against_reference(name, dtype):
    g = golden(name)
    n, d, v = int(g["n"]), int(g["d"]), int(g["v"])
    h, e, y = orc.make_inputs(n, d, v, seed=int(g["seed"]), unit_rms=bool(g["unit_rms"]))
    lt, gt = TOL[dtype]
    loss, mx, se, lse, dh, de = run_path(h, e, y, dtype)
    assert abs(loss - float(g["loss"])) <= lt * float(g["loss"])
    assert rel(dh, g["dh"]) <= gt
    rng = np.random.default_rng(int(g["seed"]) + 7)
    u_d = rng.standard_normal(d)
    u_v = rng.standard_normal(v)
    assert rel(de @ u_d, g["de_proj_d"]) <= gt
    assert rel(u_v @ de, g["de_proj_v"]) <= gt
    assert rel(de[g["de_rows_idx"]], g["de_rows"]) <= gt


def test_config2_full_size_tf32():
    """Config 2 at full size (N=8192, d=768, V=50257, fp32/TF32) against the float64 oracle."""
    n, d, v = 8192, 768, 50257
    h, e, y = orc.make_inputs(n, d, v, seed=21)
    loss, mx, se, lse, dh, de = run_path(h, e, y, torch.float32)
    l64, dh64, de64, mx64, se64 = orc.row_chunked_reference(h, e, y, rows_per_chunk=512)
    lt, gt = TOL[torch.float32]
    assert abs(loss - l64) <= lt * l64
    assert rel(dh, dh64) <= gt
    assert rel(de, de64) <= gt


# The loss scale bench.py runs the fp16 backward with, 2^15: the largest power
# of two whose product with the upstream grad of the fp16 loss stays finite
# (a dynamic loss scaler settles there). With fp16 grad outputs and no scale,
# the dominant dh term -E_y / N (~6e-7 at N = 32768) would sit among fp16
# subnormals.
BENCH_GRAD_SCALE = 32768.0


def _full_size_sampled_parity(n, d, v, seed, *, grad_scale, out_dtype, n_rows=48, n_cls=8):
    """Forward + backward at full size with the given grad output dtype, then
    sampled rows / classes against float64 recomputed from the same inputs:
    per-row loss terms (lse - target) and lse at 2e-3, the loss as the mean of
    the device's per-row terms, dh rows and dE rows at 1e-2, and the
    size-independent identity sum_v dE[v] = 0. No N x V buffer may appear."""
    from nimbleml_b200.kernels import fused_tied_crossentropy as k

    h, e, y = orc.make_inputs(n, d, v, seed=seed, unit_rms=True)
    hd, ed = to_dev(h, torch.float16), to_dev(e, torch.float16)
    yd = torch.as_tensor(y).cuda()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    # The same calls bench.py times: shard forward, combine, shard backward.
    part = k.shard_forward(hd, ed, yd)
    _, _, lse_d, loss_d, valid = k.combine(part.unsqueeze(1), yd, v, k._NO_IGNORE)
    st = k.TiedCEStats(lse=lse_d, valid_count=valid, ignore_index=k._NO_IGNORE, vocab_size=v)
    gs = torch.full((1,), grad_scale, device="cuda")
    gw = None if out_dtype == torch.float16 else torch.empty((v, d), dtype=out_dtype, device="cuda")
    dh, de = k.shard_backward(gs, hd, ed, yd, st, grad_hidden_dtype=out_dtype, grad_weights=gw)
    torch.cuda.synchronize()
    assert k.check_status(hd.device) == 0
    peak_extra = torch.cuda.max_memory_allocated() - base
    assert peak_extra < n * v * 2, (peak_extra, n * v * 2)
    assert dh.dtype == out_dtype and de.dtype == out_dtype

    lse = lse_d.double().cpu().numpy()
    tgt = part[2].double().cpu().numpy()
    terms = lse - tgt
    # The loss is the fixed-order mean of the per-row terms (float64 sum on the device).
    assert abs(float(loss_d) - terms.mean()) <= 1e-6 * terms.mean()
    assert float(valid) == n

    rows = np.random.default_rng(0).choice(n, n_rows, replace=False)
    e64 = rounded64(e, torch.float16)
    s = rounded64(h[rows], torch.float16) @ e64.T
    mx = s.max(1, keepdims=True)
    lse64 = np.log(np.exp(s - mx).sum(1)) + mx[:, 0]
    terms64 = lse64 - s[np.arange(n_rows), y[rows]]
    assert rel(lse[rows], lse64) < 2e-3
    assert rel(terms[rows], terms64) < 2e-3
    assert np.max(np.abs(terms[rows] - terms64) / terms64) < 2e-3
    g = np.exp(s - lse64[:, None])
    g[np.arange(n_rows), y[rows]] -= 1.0
    dh_ref = (g * (grad_scale / n)) @ e64
    dhn = dh.double().cpu().numpy()
    assert np.all(np.isfinite(dhn))
    assert rel(dhn[rows], dh_ref) < 1e-2
    den = de.double()
    assert bool(torch.isfinite(den).all())
    colsum = den.sum(0).cpu().numpy()
    assert np.linalg.norm(colsum) < 1e-3 * float(den.norm())
    cls = np.random.default_rng(1).choice(v, n_cls, replace=False)
    hf = rounded64(h, torch.float16)
    pc = np.exp(hf @ e64[cls].T - lse[:, None])
    for j, c in enumerate(cls):
        pc[y == c, j] -= 1.0
    de_ref = (pc * (grad_scale / n)).T @ hf
    assert rel(den[torch.as_tensor(cls).cuda()].cpu().numpy(), de_ref) < 1e-2
    return float(loss_d)


def test_headline_shape_full_size_bench_configuration():
    """Config 4 at full size (N=32768, d=4096, V=128256, fp16) in the exact
    configuration bench.py times: fp16 dh and dE outputs under the 2^15 loss
    scale. Loss terms at 2e-3, grads at 1e-2 against float64."""
    loss = _full_size_sampled_parity(32768, 4096, 128256, 41, grad_scale=BENCH_GRAD_SCALE,
                                     out_dtype=torch.float16)
    assert abs(loss - np.log(128256)) < 1.0


def test_headline_shape_full_size_fp32_grads():
    """Config 4 at full size with fp32 grad outputs and grad_scale 1 (the
    unscaled grads, ~1e-6, are below fp16's normal range)."""
    _full_size_sampled_parity(32768, 4096, 128256, 43, grad_scale=1.0, out_dtype=torch.float32)


def test_config3_full_size_bench_configuration():
    """Config 3 at full size (N=16384, d=2048, V=32000, fp16) as bench.py runs it."""
    _full_size_sampled_parity(16384, 2048, 32000, 31, grad_scale=BENCH_GRAD_SCALE, out_dtype=torch.float16,
                              n_rows=64, n_cls=16)


def test_overlap_entry_point_matches_backward():
    """nimble_tied_ce_backward_overlap (event after grad_hidden, capped last dE
    GEMM) gives bit-identical results to nimble_tied_ce_backward."""
    from nimbleml_b200.kernels import fused_tied_crossentropy as k

    n, d, v = 640, 256, 3001
    h, e, y = orc.make_inputs(n, d, v, seed=12, unit_rms=True)
    hd, ed, yd = to_dev(h, torch.float16), to_dev(e, torch.float16), torch.as_tensor(y).cuda()
    loss, hh, ww, st, mx, se = k.fused_tied_crossentropy_forward(hd, ed, yd)
    one = torch.ones(1, device="cuda")
    # Same slabs in both (a 1024-column budget): bit-identical results.
    slab = 640 * 2 * 1024
    a = k.shard_backward(one, hh, ww, yd, st, grad_hidden_dtype=torch.float32, slab_bytes=slab)
    ev = torch.cuda.Event()
    ev.record()
    b = k.shard_backward(one, hh, ww, yd, st, grad_hidden_dtype=torch.float32, ready_event=ev, last_de_max_ctas=20,
                         slab_bytes=slab)
    # The last dE GEMM split into a capped part and an uncapped part.
    b2 = k.shard_backward(one, hh, ww, yd, st, grad_hidden_dtype=torch.float32, ready_event=ev, last_de_max_ctas=20,
                          slab_bytes=slab, capped_fraction=0.4)
    torch.cuda.synchronize()
    assert ev.query()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert torch.equal(a[0], b2[0]) and torch.equal(a[1], b2[1])
    # Default budget: the overlap entry point (a shard of a split vocabulary)
    # takes the shard in one slab, the plain backward in two; both match float64.
    c = k.shard_backward(one, hh, ww, yd, st, grad_hidden_dtype=torch.float32, ready_event=ev, last_de_max_ctas=20)
    torch.cuda.synchronize()
    l64, dh64, de64, _, _ = orc.row_chunked_reference(rounded64(h, torch.float16), rounded64(e, torch.float16), y)
    for dh, de in (a, c):
        assert rel(dh.double().cpu().numpy(), dh64) < 1e-2
        assert rel(de.double().cpu().numpy(), de64) < 1e-2
    assert torch.equal(a[1], c[1])  # dE rows: the same K loop over the tokens whatever the slab


def test_empty_batch():
    """No tokens: loss 0 with no valid rows, an all-zero tied grad, an empty hidden grad
    (the reference divides 0 by 0 here; this path returns the defined 0)."""
    from nimbleml_b200.kernels import fused_tied_crossentropy as k
    from nimbleml_b200.losses import CrossEntropyLoss

    e = to_dev(np.random.default_rng(0).standard_normal((100, 64)) * 0.02, torch.float16)
    h = torch.empty((0, 64), dtype=torch.float16, device="cuda")
    y = torch.empty((0,), dtype=torch.int64, device="cuda")
    loss, hh, ww, st, mx, se = k.fused_tied_crossentropy_forward(h, e, y)
    dh, de = k.fused_tied_crossentropy_backward(1.0, hh, ww, y, st, mx, se)
    torch.cuda.synchronize()
    assert float(loss) == 0.0 and float(st.valid_count) == 0.0
    assert dh.shape == (0, 64) and de.shape == (100, 64) and not de.any()
    hid = torch.empty((0, 4, 64), dtype=torch.float16, device="cuda", requires_grad=True)
    emb = e.clone().requires_grad_(True)
    out = CrossEntropyLoss().forward_tied(hid, emb, torch.empty((0, 4), dtype=torch.int64, device="cuda"))
    out.backward()
    assert float(out) == 0.0 and not emb.grad.any() and hid.grad.shape == (0, 4, 64)
    lg = torch.empty((0, 10), dtype=torch.float16, device="cuda", requires_grad=True)
    l2 = CrossEntropyLoss()(lg, torch.empty((0,), dtype=torch.int64, device="cuda"))
    l2.backward()
    assert float(l2) == 0.0 and lg.grad.shape == (0, 10)
