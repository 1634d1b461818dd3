"""The allocation-free forward entry point, called through the C ABI.

``nimble_tied_ce_forward_noalloc`` serves callers that cannot allocate device
memory (for example a host runtime whose GPU memory is owned by another
framework's pool): its per-tile scratch is a fixed 64 MiB array inside the
library. Its results must match ``nimble_tied_ce_forward``, which uses a
caller-provided workspace, on consecutive calls (the shared array keeps the
previous call's contents). This file is named to be collected last.
"""
import numpy as np
import pytest
import torch

from oracle import tied_ce_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the tightest relative tolerance of the parity tests (fp32 loss)


def _forward_both(native, n, d, v, seed, dtype=torch.float16):
    from nimbleml_b200._native_loader import DTYPE_F16, DTYPE_F32

    code = DTYPE_F16 if dtype == torch.float16 else DTYPE_F32
    h, e, y = orc.make_inputs(n, d, v, seed=seed, unit_rms=True)
    hd = torch.as_tensor(h).cuda().to(dtype).contiguous()
    ed = torch.as_tensor(e).cuda().to(dtype).contiguous()
    yd = torch.as_tensor(y).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    ref = torch.empty((3, n), dtype=torch.float32, device="cuda")
    ws_bytes = native.forward_workspace_size(n, d, v, code)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    native.call("nimble_tied_ce_forward", hd.data_ptr(), ed.data_ptr(), yd.data_ptr(), n, d, v, 0, code,
                ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr(), ws.data_ptr(), ws_bytes,
                status.data_ptr(), stream)

    out = torch.full((3, n), float("nan"), dtype=torch.float32, device="cuda")
    native.call("nimble_tied_ce_forward_noalloc", hd.data_ptr(), ed.data_ptr(), yd.data_ptr(), n, d, v, 0,
                code, out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), status.data_ptr(), stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return ref.double().cpu().numpy(), out.double().cpu().numpy()


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def test_noalloc_forward_matches_workspace_forward_on_consecutive_calls():
    from nimbleml_b200._native_loader import native

    # Two calls in a row with different shapes: the second must not see the
    # first call's leftovers in the shared scratch array.
    for n, d, v, seed in [(1000, 256, 5000, 1), (333, 128, 1200, 2)]:
        ref, out = _forward_both(native, n, d, v, seed)
        assert np.all(np.isfinite(out))
        for row in range(3):
            assert _rel(out[row], ref[row]) <= TOL, (n, d, v, row)


def test_noalloc_forward_fp32_keeps_rounded_operands_in_its_scratch():
    from nimbleml_b200._native_loader import native

    # fp32 inputs: the TF32-rounded copies of hidden and weights also live in
    # the built-in array, after the per-tile pairs.
    for n, d, v, seed in [(500, 128, 3000, 3), (700, 64, 2000, 4)]:
        ref, out = _forward_both(native, n, d, v, seed, dtype=torch.float32)
        assert np.all(np.isfinite(out))
        for row in range(3):
            assert _rel(out[row], ref[row]) <= TOL, (n, d, v, row)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from nimbleml_b200._native_loader import DTYPE_F16, native

    n, d, v = 32768, 4096, 128256  # needs ~131 MB of per-tile scratch
    h = torch.empty((8, d), dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="64 MiB"):
        native.call("nimble_tied_ce_forward_noalloc", h.data_ptr(), h.data_ptr(), h.data_ptr(), n, d, v, 0,
                    DTYPE_F16, h.data_ptr(), h.data_ptr(), h.data_ptr(), None,
                    torch.cuda.current_stream().cuda_stream)
