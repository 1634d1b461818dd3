"""Failure detection without a GPU fault.

A bounded device wait that nothing satisfies must give up, report
NIMBLE_STATUS_WAIT_TIMEOUT through the status word, and leave the CUDA
context usable (a forward afterwards still matches the oracle).
"""
import time

import numpy as np
import pytest
import torch

from oracle import tied_ce_oracle as orc

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    from nimbleml_b200._native_loader import STATUS_WAIT_TIMEOUT, native

    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    native.call("nimble_tied_ce_probe_wait_timeout", 50_000_000, status.data_ptr(),
                torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(status.item()) & STATUS_WAIT_TIMEOUT
    assert 0.04 < dt < 1.5
    # The context is intact: the path still runs and matches the oracle.
    from nimbleml_b200.kernels import fused_tied_crossentropy as k

    h, e, y = orc.make_inputs(200, 128, 700, seed=3, unit_rms=True)
    loss = k.fused_tied_crossentropy_forward(torch.as_tensor(h).cuda().half(), torch.as_tensor(e).cuda().half(),
                                             torch.as_tensor(y).cuda())[0]
    l64 = orc.row_chunked_reference(torch.as_tensor(h).half().double().numpy(),
                                    torch.as_tensor(e).half().double().numpy(), y)[0]
    assert abs(float(loss) - l64) < 2e-3 * l64


def test_check_status_raises_on_timeout_bit():
    from nimbleml_b200._native_loader import STATUS_WAIT_TIMEOUT
    from nimbleml_b200.kernels import fused_tied_crossentropy as k

    dev = torch.device("cuda", torch.cuda.current_device())
    k.status_word(dev).fill_(STATUS_WAIT_TIMEOUT)
    with pytest.raises(RuntimeError, match="timed out"):
        k.check_status(dev)
    assert k.check_status(dev) == 0


def test_probe_argument_checks():
    from nimbleml_b200._native_loader import native

    with pytest.raises(RuntimeError, match="limit_ns"):
        native.call("nimble_tied_ce_probe_wait_timeout", 0, 16, None)
    with pytest.raises(RuntimeError, match="null status"):
        native.call("nimble_tied_ce_probe_wait_timeout", 1000, None, None)
