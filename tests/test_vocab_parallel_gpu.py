"""Vocab-sharded tied CE over NCCL against the float64 oracle (needs >= P GPUs).

Each of P ranks (2, 4, 8) owns ceil(V/P) rows of E; every rank must hold the
same loss and the same full grad_hidden, the loss and grad_hidden must match
the reference math run in float64 on the fp16-rounded inputs, and each
shard's dE rows must match the matching rows of the float64 dE (tolerances
of the fp16 parity tests: loss 2e-3, grads 1e-2 relative).
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


@pytest.mark.parametrize("world", [2, 4, 8])
def test_vocab_parallel_matches_float64_oracle(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
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
    h64 = torch.as_tensor(h).half().double().numpy()
    e64 = torch.as_tensor(e).half().double().numpy()
    ref_loss, ref_dh, ref_de, _, _ = orc.row_chunked_reference(h64, e64, y, ignore_index=-1)

    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    for r in res[1:]:
        assert r[2] == res[0][2]                        # identical loss on every rank
        assert np.array_equal(r[3], res[0][3])          # identical grad_hidden on every rank
    for rank, off, l_r, dh_r, de_r in res:
        assert abs(l_r - ref_loss) <= 2e-3 * ref_loss
        assert rel(dh_r, ref_dh) <= 1e-2
        assert rel(de_r, ref_de[off:off + de_r.shape[0]]) <= 1e-2
    assert sum(r[4].shape[0] for r in res) == V


def _rank_tied_embedding(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from conftest import GOLDEN
        from nimbleml_b200.gpt_head import TiedEmbedding
        from nimbleml_b200.vocab_parallel import shard_range

        g = dict(np.load(GOLDEN / "tied_embedding_adamw_f32.npz"))
        v = g["e0"].shape[0]
        off, rows = shard_range(v, rank, world)
        te = TiedEmbedding(torch.as_tensor(g["e0"][off:off + rows]).cuda(), v, vocab_offset=off,
                           compute_dtype=torch.float32, group=dist.group.WORLD, learning_rate=float(g["lr"]),
                           beta1=float(g["b1"]), beta2=float(g["b2"]), epsilon=float(g["eps"]),
                           weight_decay=float(g["wd"]))
        ids = torch.as_tensor(g["ids"]).cuda()
        loss = te.loss(te.lookup(ids), torch.as_tensor(g["labels"]).cuda().view(ids.shape), ignore_index=-1)
        loss.backward()
        grad = te.grad.cpu().numpy().copy()
        te.step()
        torch.cuda.synchronize()
        q.put((rank, off, float(loss), grad, te.master.cpu().numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_tied_embedding_grad_and_adamw_match_reference(world):
    """Vocab-sharded tied embedding (lookup all_reduce, sharded head, one fp32
    grad buffer per shard, AdamW per shard) against the reference's
    Embedding + forward_tied + AdamW golden (fp32 / TF32 tolerances)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import sys

    from conftest import GOLDEN, REPO

    sys.path.insert(0, str(REPO / "tests"))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_tied_embedding, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    g = dict(np.load(GOLDEN / "tied_embedding_adamw_f32.npz"))
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    grad = np.concatenate([r[3] for r in res])
    master = np.concatenate([r[4] for r in res])
    assert all(r[2] == res[0][2] for r in res)
    assert abs(res[0][2] - float(g["loss"])) <= 1e-5 * float(g["loss"])
    assert rel(grad, g["grad"]) <= 1e-3
    assert rel(master.astype(np.float64) - g["e0"], g["e1"].astype(np.float64) - g["e0"]) <= 1e-2
