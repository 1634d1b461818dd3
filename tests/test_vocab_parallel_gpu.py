"""Vocab-sharded tied CE over NCCL against the single-GPU path (needs >= 2 GPUs).

Each rank owns ceil(V/P) rows of E; the loss must equal the 1-GPU loss, every
rank must hold the same loss and the full grad_hidden, and the shards' dE
rows must equal the matching rows of the 1-GPU dE (fp16 inputs; tolerances as
in the parity tests: loss 2e-3, grads 1e-2 relative — in practice the only
differences are the fp32 dh all-reduce order and fp16 output rounding).
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import tied_ce_oracle as orc

pytestmark = pytest.mark.gpu

N, D, V = 1536, 512, 10007  # V prime: uneven shards


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from nimbleml_b200.vocab_parallel import VocabParallelTiedHead

        h, e, y = orc.make_inputs(N, D, V, seed=77, unit_rms=True, ignore_frac=0.1, ignore_index=-1)
        hd = torch.as_tensor(h).cuda().half().requires_grad_(True)
        ed = torch.as_tensor(e).cuda().half()
        head = VocabParallelTiedHead(ed, V, group=dist.group.WORLD)
        w = head.weights.clone().requires_grad_(True)
        head.weights = w
        loss = head.loss(hd, torch.as_tensor(y).cuda(), ignore_index=-1)
        loss.backward()
        torch.cuda.synchronize()
        q.put((rank, head.vocab_offset, float(loss), hd.grad.float().cpu().numpy(), w.grad.float().cpu().numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_vocab_parallel_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from nimbleml_b200.losses.cross_entropy import tied_cross_entropy

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0

    h, e, y = orc.make_inputs(N, D, V, seed=77, unit_rms=True, ignore_frac=0.1, ignore_index=-1)
    hd = torch.as_tensor(h).cuda().half().requires_grad_(True)
    ed = torch.as_tensor(e).cuda().half().requires_grad_(True)
    loss = tied_cross_entropy(hd, ed, torch.as_tensor(y).cuda(), -1)
    loss.backward()
    ref_loss = float(loss)
    ref_dh = hd.grad.float().cpu().numpy()
    ref_de = ed.grad.float().cpu().numpy()

    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    assert res[0][2] == res[1][2]                      # identical loss on every rank
    assert np.array_equal(res[0][3], res[1][3])         # identical grad_hidden on every rank
    for rank, off, l_r, dh_r, de_r in res:
        assert abs(l_r - ref_loss) <= 1e-6 * ref_loss
        assert rel(dh_r, ref_dh) <= 1e-2
        assert rel(de_r, ref_de[off:off + de_r.shape[0]]) <= 1e-2
    assert sum(r[4].shape[0] for r in res) == V
