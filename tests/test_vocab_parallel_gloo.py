"""Host logic of the vocab-parallel path on CPU ranks (gloo, world_size 2)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import tied_ce_oracle as orc


def test_shard_range_covers_vocab():
    from nimbleml_b200.vocab_parallel import shard_range

    for v, p in [(128256, 8), (32000, 8), (50257, 8), (50257, 3), (7, 8)]:
        spans = [shard_range(v, r, p) for r in range(p)]
        assert spans[0][0] == 0
        assert sum(n for _, n in spans) == v
        for (o0, n0), (o1, _) in zip(spans, spans[1:]):
            assert o0 + n0 == o1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nimbleml_b200.vocab_parallel import gather_shard_stats, reduce_grad_hidden, shard_range

        n, d, v = 33, 16, 101
        h, e, y = orc.make_inputs(n, d, v, seed=3, ignore_frac=0.25, ignore_index=-1)
        off, rows = shard_range(v, rank, world)
        # Local shard statistics exactly as the device kernel defines them.
        s = h.astype(np.float64) @ e[off:off + rows].astype(np.float64).T
        local = np.zeros((3, n))
        local[0] = s.max(axis=1)
        local[1] = np.exp(s - local[0][:, None]).sum(axis=1)
        inside = (y >= off) & (y < off + rows)
        local[2, inside] = s[inside, y[inside] - off]
        group = dist.group.WORLD
        stats = gather_shard_stats(torch.from_numpy(local), group).numpy()
        m, se, lse, loss, nv = orc.combine_stats(stats, y, v, ignore_index=-1)
        # Partial grad_hidden of the shard: G_r E_r with the global lse.
        g = np.exp(s - lse[:, None])
        g[inside, y[inside] - off] -= 1.0
        g[y == -1] = 0.0
        g /= nv
        dh = torch.from_numpy(g @ e[off:off + rows].astype(np.float64))
        reduce_grad_hidden(dh, group)
        result_q.put((rank, loss, dh.numpy()))
    finally:
        dist.destroy_process_group()


def test_gloo_two_rank_exchange_matches_single_device_math():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 2000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    h, e, y = orc.make_inputs(33, 16, 101, seed=3, ignore_frac=0.25, ignore_index=-1)
    loss, dh, de, _, _ = orc.row_chunked_reference(h, e, y, ignore_index=-1)
    for _, l_r, dh_r in results:
        assert abs(l_r - loss) < 1e-12 * loss
        assert np.allclose(dh_r, dh, rtol=1e-10, atol=1e-14)
    # Every rank holds bit-identical results.
    assert results[0][1] == results[1][1]
    assert np.array_equal(results[0][2], results[1][2])


def _host_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nimbleml_b200.vocab_parallel import VocabParallelTiedHead

        h = torch.arange(13 * 4, dtype=torch.float32).view(13, 4)
        head = VocabParallelTiedHead(torch.zeros(10, 4), 10, group=dist.group.WORLD)
        q.put((rank, head.hidden_from_host(h).clone()))
    finally:
        dist.destroy_process_group()


def test_hidden_from_host_assembles_all_rows():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28500 + os.getpid() % 1000
    procs = [ctx.Process(target=_host_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = torch.arange(13 * 4, dtype=torch.float32).view(13, 4)
    for _, got in res:
        assert torch.equal(got, want)


def _lookup_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nimbleml_b200.gpt_head import TiedEmbedding
        from nimbleml_b200.vocab_parallel import shard_range

        v, d = 37, 8  # uneven shards
        e = torch.arange(v * d, dtype=torch.float32).reshape(v, d) / 7.0
        off, rows = shard_range(v, rank, world)
        te = TiedEmbedding(e[off:off + rows].clone(), v, vocab_offset=off, compute_dtype=torch.float32,
                           group=dist.group.WORLD)
        ids = torch.tensor([[0, 36, 18, 19], [5, 5, 30, 17]])
        out = te.lookup(ids).detach()
        result_q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


def test_gloo_vocab_parallel_lookup_assembles_every_row_exactly():
    """The tied embedding's vocab-parallel lookup: each rank gathers its own
    rows (zeros elsewhere) and one all_reduce assembles exact rows everywhere."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29300 + os.getpid() % 500
    procs = [ctx.Process(target=_lookup_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    e = torch.arange(37 * 8, dtype=torch.float32).reshape(37, 8) / 7.0
    ids = torch.tensor([[0, 36, 18, 19], [5, 5, 30, 17]])
    for _, out in res:
        assert np.array_equal(out, e[ids].numpy())


def test_tied_embedding_argument_checks():
    from nimbleml_b200.gpt_head import TiedEmbedding
    from nimbleml_b200.vocab_parallel import dh_reduce_dtype

    with pytest.raises(ValueError, match="float32"):
        TiedEmbedding(torch.zeros((4, 8), dtype=torch.float16), 10)
    with pytest.raises(ValueError, match="inside the vocabulary"):
        TiedEmbedding(torch.zeros((4, 8)), 10, vocab_offset=8)
    te = TiedEmbedding(torch.ones((4, 8)), 10, vocab_offset=6, compute_dtype=torch.float16)
    assert te.weight.dtype == torch.float16 and te.grad.dtype == torch.float32 and te.rows == 4
    # The grad_hidden reduction dtype: bf16 partials for 16-bit inputs, fp32 for fp32.
    assert dh_reduce_dtype(torch.float16) == torch.bfloat16
    assert dh_reduce_dtype(torch.bfloat16) == torch.bfloat16
    assert dh_reduce_dtype(torch.float32) == torch.float32
