"""Benchmark of the fused tied LM-head cross-entropy (forward + backward).

Default workload: config 4 of the path's specification (the headline):
N = 32768 tokens (4 x 8192), d = 4096, V = 128256, fp16, h unit-RMS rows from
N(0,1), E ~ N(0, 0.02^2), labels ~ U[0, V). One "step" is one forward and
backward of the tied head over those N tokens. With --gpus P > 1 (launched by
torchrun, one rank per GPU) the vocabulary is sharded P ways and the total
work stays fixed (strong scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4|c3|c2]
    python bench.py --impl reference ...   # the reference's CPU algorithm

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "tied LM-head+CE fwd+bwd tokens/s (V=128256,d=4096) at 1–8 B200; % TC peak"
DATASHEET_DENSE_F16_TFLOPS = 2250.0
DATASHEET_DENSE_TF32_TFLOPS = 1100.0

CONFIGS = {
    "c4": dict(workload="config 4: large-vocab fused tied CE fwd+bwd (headline)", n=32768, d=4096,
               v=128256, dtype="float16", unit_rms=True, batch=4, seq=8192),
    "c3": dict(workload="config 3: fused tied CE fwd+bwd", n=16384, d=2048, v=32000, dtype="float16",
               unit_rms=True, batch=16, seq=1024),
    "mid": dict(workload="profiling case: config-4 d with N=4096, V=32768 (inputs > L2)", n=4096, d=4096,
                v=32768, dtype="float16", unit_rms=True, batch=1, seq=4096),
    "mid_bf16": dict(workload="profiling case: config-4 d with N=4096, V=32768, bf16 (inputs > L2)", n=4096,
                     d=4096, v=32768, dtype="bfloat16", unit_rms=True, batch=1, seq=4096),
    "c2": dict(workload="config 2: standalone fused tied CE fwd+bwd, fp32 on TF32", n=8192, d=768,
               v=50257, dtype="float32", unit_rms=False, batch=8, seq=1024),
}
DTYPE_TAG = {"float16": "f16", "float32": "f32", "bfloat16": "bf16"}


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d["bf16_tflops_sustained"], d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def _profile_traffic(config_name):
    """DRAM bytes per launch of the forward GEMM from the committed ncu summary, if any."""
    p = REPO / "profiles" / f"tc_gemm_ce_fwd_{config_name}.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("dram_bytes_per_launch_full_size")
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.bus_id = (bus_id or "").lower()
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            if self.bus_id and self.bus_id[-12:] not in parts[1].lower():
                continue
            rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][3]) if rows[0][3].replace(".", "").isdigit() else None,
                "samples": len(rows), "reasons": sorted(reasons)}


def _dist_setup(gpus):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if gpus > 1 and world != gpus:
        raise SystemExit(f"--gpus {gpus} needs torchrun with {gpus} ranks (WORLD_SIZE={world})")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return rank, local, world


# Upstream grad of the loss for the fp16 backward: 2^15, a dynamic loss
# scaler's settled scale (2^16 times the upstream grad of an fp16 loss
# overflows). Unscaled fp16 grads at N = 32768 would fall among fp16
# subnormals; tests/test_tied_ce_gpu.py pins this exact configuration.
GRAD_SCALE = {"float16": 32768.0, "bfloat16": 1.0, "float32": 1.0}


def all_host_threads():
    """Lets NumPy's BLAS use every host core the process may run on.

    torchrun exports OMP_NUM_THREADS=1 to every rank; OpenBLAS reads it when
    NumPy is imported, so it is overridden before that import, and
    threadpoolctl raises a pool that was already created. Returns the thread
    count the BLAS pool reports.
    """
    n = len(os.sched_getaffinity(0))
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = str(n)
    try:
        import threadpoolctl

        threadpoolctl.threadpool_limits(n, user_api="blas")
        pools = [p["num_threads"] for p in threadpoolctl.threadpool_info() if p.get("user_api") == "blas"]
        return max(pools) if pools else n
    except Exception:
        return n


def reference_kernels():
    """The unmodified reference's own fused tied-CE functions on its CPU
    (NumPy) backend, from the offline install in baseline/_ref, or None."""
    ref = REPO / "baseline" / "_ref"
    if not (ref / "NimbleML" / "__init__.py").exists():
        return None
    os.environ["NIMBLEML_DEVICE"] = "cpu"
    os.environ["NIMBLEML_DTYPE"] = "float32"
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    from NimbleML.kernels import fused_tied_crossentropy_backward, fused_tied_crossentropy_forward

    return fused_tied_crossentropy_forward, fused_tied_crossentropy_backward


def cpu_reference_sample(cfg, seconds=12.0, max_rows=4096):
    """A bounded CPU sample of the workload for the reference arm and the
    cpu_baseline: the reference's own NimbleML.kernels.fused_tied_crossentropy_*
    (NIMBLEML_DEVICE=cpu, fp32, BLAS on all host threads) when baseline/_ref
    holds it, else the oracle's restatement of the same algorithm. Returns
    (step callable, rows, sample description, kind, threads)."""
    threads = all_host_threads()
    import numpy as np

    ref = reference_kernels()
    rng = np.random.default_rng(1234)
    e = (rng.standard_normal((cfg["v"], cfg["d"]), dtype=np.float32) * np.float32(0.02))

    def make(rows):
        h = rng.standard_normal((rows, cfg["d"]), dtype=np.float32)
        if cfg["unit_rms"]:
            h /= np.sqrt(np.mean(h * h, axis=1, keepdims=True))
        y = rng.integers(0, cfg["v"], rows, dtype=np.int64)
        return h, y

    if ref is not None:
        fwd, bwd = ref
        kind = "reference"
        what = ("the reference's own NimbleML.kernels.fused_tied_crossentropy_forward/_backward "
                "(baseline/_ref, NIMBLEML_DEVICE=cpu)")

        def run(h, y):
            loss, hh, ww, logits, mx, se = fwd(h, e, y)
            bwd(1.0, hh, ww, y, logits, mx, se)
    else:
        from oracle import tied_ce_oracle as orc

        kind = "port"
        what = ("the reference algorithm restated in oracle/tied_ce_oracle.py "
                "(NimbleML/kernels/fused_*crossentropy.py)")

        def run(h, y):
            loss, hh, ww, logits, mx, se = orc.tied_forward(h, e, y, np.float32)
            orc.tied_backward(1.0, hh, ww, y, logits, mx, se)

    rows = 32
    h, y = make(rows)
    run(h, y)  # first call pays one-time costs (page faults, BLAS pool start)
    t0 = time.perf_counter()
    run(h, y)
    dt = time.perf_counter() - t0
    rows = int(min(max_rows, max(32, rows * seconds / max(dt, 1e-3))))
    rows = max(32, rows // 32 * 32)
    h, y = make(rows)
    sample = (f"{rows} of {cfg['n']} token rows at full d={cfg['d']}, V={cfg['v']}; {what} in NumPy fp32 with "
              f"{threads} BLAS threads (the reference's fp16 NumPy matmul has no BLAS path)")
    return (lambda: run(h, y)), rows, sample, kind, threads


def run_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    step, rows, sample, kind, threads = cpu_reference_sample(cfg, seconds=6.0)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    t = statistics.mean(times)
    value = rows / t
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["workload"], "n_tokens": cfg["n"], "d_model": cfg["d"], "vocab": cfg["v"],
                   "sample_rows": rows, "parallelism": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def full_loss64(h, e_local, labels, v_off, world, group, chunk=512):
    """The mean loss over all N rows in float64, recomputed on the device a row
    chunk at a time (never more than chunk x V_local logits); at P > 1 each
    rank reduces its vocab shard and the per-row (max, sum-exp, target)
    triples are merged over ranks."""
    import torch
    import torch.distributed as dist

    n = h.shape[0]
    e64 = e_local.double()
    v_local = e_local.shape[0]
    st = torch.zeros((3, n), dtype=torch.float64, device=h.device)
    for i in range(0, n, chunk):
        s = h[i:i + chunk].double() @ e64.T
        mx = s.max(1).values
        st[0, i:i + chunk] = mx
        st[1, i:i + chunk] = torch.exp(s - mx[:, None]).sum(1)
        y = labels[i:i + chunk] - v_off
        own = (y >= 0) & (y < v_local)
        idx = own.nonzero()[:, 0]
        st[2, i + idx] = s[idx, y[own]]
        del s
    if world > 1:
        allst = torch.empty((world, 3, n), dtype=torch.float64, device=h.device)
        dist.all_gather_into_tensor(allst, st, group=group)
    else:
        allst = st[None]
    m = allst[:, 0].max(0).values
    lse = m + torch.log((allst[:, 1] * torch.exp(allst[:, 0] - m)).sum(0))
    return float((lse - allst[:, 2].sum(0)).mean())


def sampled_parity(h, e_local, labels, v, v_off, world, group, stats3, lse, loss, dh, de, scale,
                   n_rows=32, n_cls=8):
    """Checks the last timed step's results on every rank against float64
    recomputed on the device from the same inputs: the loss over all N rows,
    sampled rows' lse and loss terms (lse - target), the loss as the mean of
    the device's per-row terms, and sampled rows of grad_hidden and of this
    rank's grad_weights shard (relative 2-norms). Tolerances follow the
    compute dtype (fp16 / bf16: loss 2e-3, grads 1e-2; fp32 on TF32: loss
    1e-5, grads 1e-3; per-row terms at ten times the loss tolerance, as the
    loss averages their rounding). Rank-local errors are maxed over ranks."""
    import torch
    import torch.distributed as dist

    dev = h.device
    n = h.shape[0]
    fp32 = h.dtype == torch.float32
    loss64 = full_loss64(h, e_local, labels, v_off, world, group)
    g = torch.Generator(device="cpu").manual_seed(5)
    rows = torch.randperm(n, generator=g)[:n_rows].to(dev)
    e64 = e_local.double()
    s_loc = h[rows].double() @ e64.T                                     # (R, v_local)
    if world > 1:
        per = -(-v // world)
        pad = torch.full((n_rows, per), float("-inf"), dtype=torch.float64, device=dev)
        pad[:, : s_loc.shape[1]] = s_loc
        allp = torch.empty((world, n_rows, per), dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(allp, pad, group=group)
        s_full = allp.permute(1, 0, 2).reshape(n_rows, world * per)[:, :v]
    else:
        s_full = s_loc
    y = labels[rows]
    lse64 = torch.logsumexp(s_full, dim=1)
    terms64 = lse64 - s_full.gather(1, y[:, None])[:, 0]
    tgt = stats3[2].double().sum(0)                                      # (N,) target logit
    terms = lse.double() - tgt
    rel = lambda a, b: float((a - b).norm() / b.norm())
    out = {"loss_rel": abs(float(loss) - loss64) / abs(loss64),
           "lse_rel": rel(lse.double()[rows], lse64), "loss_terms_rel": rel(terms[rows], terms64),
           "loss_vs_mean_terms_rel": abs(float(loss) - float(terms.mean())) / float(terms.mean())}
    # grad_hidden rows: sum over shards of G_rows . E_shard (float64).
    gl = torch.exp(s_loc - lse64[:, None])
    yl = y - v_off
    own = (yl >= 0) & (yl < e_local.shape[0])
    gl[own.nonzero()[:, 0], yl[own]] -= 1.0
    dh_ref = (gl * (scale / n)) @ e64
    if world > 1:
        dist.all_reduce(dh_ref, group=group)
    out["dh_rel"] = rel(dh.double()[rows], dh_ref)
    # grad_weights rows of this rank's shard.
    cls = torch.randperm(e_local.shape[0], generator=g)[:n_cls].to(dev)
    h64 = h.double()
    pc = torch.exp(h64 @ e64[cls].T - lse.double()[:, None])
    pc -= (labels[:, None] == (cls[None, :] + v_off)).double()
    de_ref = (pc * (scale / n)).T @ h64
    out["de_rel"] = rel(de.double()[cls], de_ref)
    del h64, pc
    keys = ("loss_rel", "lse_rel", "loss_terms_rel", "loss_vs_mean_terms_rel", "dh_rel", "de_rel")
    errs = torch.tensor([out[k] for k in keys], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(errs, op=dist.ReduceOp.MAX, group=group)
    out = {k: float(x) for k, x in zip(keys, errs.tolist())}
    lt, gt = (1e-5, 1e-3) if fp32 else (2e-3, 1e-2)
    tol = {"loss_rel": lt, "lse_rel": lt, "loss_terms_rel": 10 * lt, "loss_vs_mean_terms_rel": 1e-6,
           "dh_rel": gt, "de_rel": gt}
    out["ok"] = all(out[k] <= tol[k] and math.isfinite(out[k]) for k in keys)
    out["tolerances"] = tol
    out["sample"] = (f"loss over all {n} rows; {n_rows} token rows and {n_cls} vocab rows per rank sampled; float64 on "
                     f"the device; max over ranks")
    return out


def run_c5(args):
    """`--config c5`: prints config 5's own JSON line (see c5_measure)."""
    print(json.dumps(c5_measure(args.steps, args.warmup)), flush=True)


def c5_measure(steps, warmup):
    """Config 5: one GPT training step (24 layers, d=1024, 16 heads, seq 1024,
    batch 8, V=50257, fp16 autocast) with clip_grad_norm(1.0) and AdamW;
    reports the head's share of step time and memory.

    The trunk is a plain torch harness (embedding + learned positions,
    pre-norm blocks with SDPA attention and a GELU MLP). This library runs the
    tied matrix E end to end — TiedEmbedding's lookup, the final RMSNorm fused
    with the tied head + CE, the one fp32 E grad buffer shared by the head's
    dE and the lookup's deterministic scatter-add — and the AdamW update of
    every parameter (nimble_adamw_step over fp32 masters; E's fp16 copy is
    rewritten in the same pass). The loss scale is a static 2^15. Random
    init, synthetic ids.
    """
    import torch
    import torch.nn.functional as F

    from nimbleml_b200.embedding_grad import AdamW
    from nimbleml_b200.gpt_head import TiedEmbedding, norm_tied_cross_entropy

    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    V, D, H, L, S, B = 50257, 1024, 16, 24, 1024, 8
    loss_scale = 32768.0

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.n1 = torch.nn.RMSNorm(D, device=dev)
            self.n2 = torch.nn.RMSNorm(D, device=dev)
            self.qkv = torch.nn.Linear(D, 3 * D, bias=False, device=dev)
            self.o = torch.nn.Linear(D, D, bias=False, device=dev)
            self.up = torch.nn.Linear(D, 4 * D, bias=False, device=dev)
            self.down = torch.nn.Linear(4 * D, D, bias=False, device=dev)

        def forward(self, x):
            q, k, v = self.qkv(self.n1(x)).view(B, S, 3, H, D // H).permute(2, 0, 3, 1, 4)
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            x = x + self.o(a.transpose(1, 2).reshape(B, S, D))
            return x + self.down(F.gelu(self.up(self.n2(x)), approximate="tanh"))

    class GPT(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.emb = TiedEmbedding(torch.randn(V, D, device=dev) * 0.02, V, compute_dtype=torch.float16,
                                     learning_rate=3e-4, weight_decay=0.01)
            self.pos = torch.nn.Parameter(torch.randn(S, D, device=dev) * 0.02)
            self.blocks = torch.nn.ModuleList([Block() for _ in range(L)])
            self.ln_gamma = torch.nn.Parameter(torch.ones(D, device=dev))

        def hidden(self, ids):
            x = self.emb.lookup(ids).float() + self.pos
            for blk in self.blocks:
                x = blk(x)
            return x.half()

        def compute_loss(self, ids, labels):
            return self.emb.loss(self.hidden(ids), labels, norm_gamma=self.ln_gamma)

    model = GPT()
    params = list(model.parameters())
    opt = AdamW(params, learning_rate=3e-4, weight_decay=0.01)
    gen = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, V, (B, S), device=dev, generator=gen)
    labels = torch.randint(0, V, (B, S), device=dev, generator=gen)

    def step():
        opt.zero_grad(set_to_none=True)
        model.emb.zero_grad()
        with torch.autocast("cuda", dtype=torch.float16):
            loss = model.compute_loss(ids, labels)
        (loss * loss_scale).backward()
        grads = [p.grad for p in params] + [model.emb.grad]
        torch._foreach_mul_(grads, 1.0 / loss_scale)
        total = torch.linalg.vector_norm(torch.stack(torch._foreach_norm(grads)))
        torch._foreach_mul_(grads, torch.clamp(1.0 / (total + 1e-6), max=1.0))  # clip_grad_norm(1.0)
        opt.step()
        model.emb.step()
        return loss

    def timed(fn, k):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / k

    step_ms = timed(step, steps)
    torch.cuda.reset_peak_memory_stats(dev)
    step()
    torch.cuda.synchronize()
    step_peak = torch.cuda.max_memory_allocated(dev)

    with torch.no_grad():
        x = model.hidden(ids)
    xh = x.detach().requires_grad_(True)
    gamma = model.ln_gamma.detach().requires_grad_(True)
    w = model.emb.weight
    buf = torch.zeros_like(model.emb.grad)

    def head_ours():
        xh.grad = None
        gamma.grad = None
        norm_tied_cross_entropy(xh, gamma, w, labels, grad_weights_buffer=buf).backward()

    wt = w.detach().clone().requires_grad_(True)

    def head_torch():
        xh.grad = None
        wt.grad = None
        gamma.grad = None
        y = F.rms_norm(xh, (D,), gamma.half(), 1e-5)
        logits = (y.view(-1, D) @ wt.T).float()
        F.cross_entropy(logits, labels.view(-1)).backward()

    def peak(fn):
        fn()
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated(dev)
        torch.cuda.reset_peak_memory_stats(dev)
        fn()
        torch.cuda.synchronize()
        return torch.cuda.max_memory_allocated(dev) - base

    head_ms = timed(head_ours, steps)
    torch_ms = timed(head_torch, steps)
    line = {
        "metric": "GPT training step tokens/s (config 5: 24L, d=1024, V=50257, batch 8 x 1024, fp16)",
        "value": B * S / (step_ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
        "warmup": warmup, "ms_per_step": step_ms, "higher_is_better": True, "dtype": "f16",
        "data": "synthetic, random init",
        "config": {"workload": "config 5 harness: torch trunk; this library's tied embedding (lookup, shared fp32 "
                               "grad, deterministic scatter), final RMSNorm fused with the tied head, AdamW",
                   "vocab": V, "d_model": D, "layers": L, "heads": H, "batch": B, "seq_len": S,
                   "loss_scale": loss_scale},
        "head": {"ms_fwd_bwd": head_ms, "share_of_step": head_ms / step_ms,
                 "what": "final RMSNorm + tied head + CE, forward and backward",
                 "peak_extra_bytes": int(peak(head_ours)),
                 "materialised_torch_head_ms": torch_ms,
                 "materialised_torch_head_peak_extra_bytes": int(peak(head_torch)),
                 "head_tflops": 8.0 * B * S * D * V / (head_ms / 1e3) / 1e12},
        "step_peak_bytes": int(step_peak),
    }
    del model, opt
    torch.cuda.empty_cache()
    return line


def run_rows(args):
    """HBM-bound row kernels around the head: achieved GB/s (algorithmic bytes
    per launch / CUDA-event time per launch, inputs larger than L2) against
    the measured copy bandwidth. Not the headline metric."""
    import torch

    from nimbleml_b200.embedding_grad import embedding_scatter_add
    from nimbleml_b200.kernels import fused_tied_crossentropy as k
    from nimbleml_b200.losses.cross_entropy import CrossEntropyLoss
    from nimbleml_b200.norm import rmsnorm_backward, rmsnorm_forward

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _, _, hbm, peak_kind = _peaks()
    g = torch.Generator(device=dev).manual_seed(3)
    out = {}

    def timed(fn, nbytes, name, reps=None):
        reps = args.rows_reps if reps is None else min(reps, args.rows_reps)
        for _ in range(min(3, reps)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        out[name] = {"ms": ms, "bytes": int(nbytes), "gb_s": nbytes / ms / 1e6, "frac_of_hbm": nbytes / ms / 1e6 / hbm}

    n, d = 32768, 4096
    x = torch.randn((n, d), generator=g, device=dev).half()
    gamma = (1 + 0.1 * torch.randn(d, generator=g, device=dev)).half()
    y, ms_, rms = rmsnorm_forward(x, gamma, 1e-5)
    timed(lambda: rmsnorm_forward(x, gamma, 1e-5), 2 * n * d * 2 + 8 * n, "rmsnorm_forward f16 32768x4096")
    gy = torch.randn((n, d), generator=g, device=dev)
    timed(lambda: rmsnorm_backward(gy, x, gamma, ms_, rms, 1e-5), n * d * (4 + 2 + 2) + 8 * n,
          "rmsnorm_backward fp32 grad -> f16 grad_x 32768x4096")
    del y, gy
    nl, vl = 8192, 50257
    logits = torch.randn((nl, vl), generator=g, device=dev).half()
    lab = torch.randint(0, vl, (nl,), generator=g, device=dev)
    ce = CrossEntropyLoss()
    timed(lambda: ce(logits, lab), nl * vl * 2, "ce_logits_forward f16 8192x50257")
    lg = logits.detach().requires_grad_(True)
    loss = ce(lg, lab)
    timed(lambda: torch.autograd.grad(loss, lg, retain_graph=True), 2 * nl * vl * 2,
          "ce_logits_backward f16 8192x50257")
    del logits, lg, loss
    vv = 16384 if args.rows_small else 128256
    ids = torch.randint(0, vv, (n,), generator=g, device=dev)
    touched = int(torch.unique(ids).numel())
    gw = torch.zeros((vv, d), device=dev)
    timed(lambda: embedding_scatter_add(gw, ids, x), n * d * 2 + touched * d * 8 + n * 24,
          f"embedding_scatter_add f16 rows 32768x4096 -> fp32 {vv}x4096")
    del gw
    from nimbleml_b200.gpt_head import TiedEmbedding

    te = TiedEmbedding(torch.randn((vv, d), generator=g, device=dev) * 0.02, vv, compute_dtype=torch.float16)
    te.grad.normal_(generator=g)
    timed(te.step, vv * d * 30, f"adamw_step fp32 master + fp16 copy {vv}x4096", reps=5)
    del te
    src = torch.randn((vv, d), generator=g, device=dev)
    timed(lambda: k.round_tf32(src), vv * d * 8, f"round_tf32 {vv}x4096")
    line = {"metric": "HBM-bound row kernels: achieved GB/s", "unit": "GB/s", "n_gpus": 1,
            "peak": hbm, "peak_kind": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
            "timing": "CUDA events, mean of repeated launches after 3 warm-ups; inputs larger than L2",
            "kernels": out}
    print(json.dumps(line), flush=True)


def launches_per_step(cfg, world, slab_bytes):
    """Kernels of libnimbleml_tied_ce.so launched by one step on one rank."""
    n, d = cfg["n"], cfg["d"]
    v_local = -(-cfg["v"] // world)
    es = 4 if cfg["dtype"] == "float32" else 2
    cols = (slab_bytes or (2 << 30)) // (es * n)
    cols = max(256, cols // 256 * 256)
    if world == 1:  # one GPU: at least two slabs (no buffer holds half the logits)
        cols = min(cols, -(-((v_local + 1) // 2) // 256) * 256)
    else:  # a shard of a split vocabulary: the byte budget alone
        cols = min(cols, -(-v_local // 256) * 256)
    n_slabs = -(-v_local // cols)
    k = 2 + 1 + 3 * n_slabs  # fwd GEMM + row reduce, combine, 3 GEMMs per slab
    if cfg["dtype"] == "float32":
        k += 2  # tf32 rounding of h and E, once per forward + backward
    return k, n_slabs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--warmup-seconds", type=float, default=4.0,
                    help="keep warming up until this much time has passed, so every N is measured at "
                         "steady-state power and clocks")
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS) + ["c5", "rows"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--also", default="c3,c2",
                    help="with the default config 4: also device-time these configurations (comma list, '' for none)")
    ap.add_argument("--no-c5", dest="also_c5", action="store_false",
                    help="with the default config 4 on one GPU: skip the config-5 training-step measurement")
    ap.add_argument("--rows-reps", type=int, default=20, help="--config rows: timed launches per kernel")
    ap.add_argument("--rows-small", action="store_true",
                    help="--config rows: a 16384-row vocabulary for the scatter / AdamW / rounding kernels "
                         "(device footprint of a few GB, for profiler captures)")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="profiling aid: one process computes rank 0's vocab shard of this many ranks through "
                         "the sharded backward entry point, with no collectives (not a bench line)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.config == "rows":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the row-kernel report has no reference arm"}))
            return
        run_rows(args)
        return
    if args.config == "c5":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 5 is a GPU training harness; the "
                              "reference's CPU path cannot run a 24-layer GPT step in minutes"}))
            return
        run_c5(args)
        return
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        run_reference_arm(args, cfg)
        return

    import torch
    import torch.distributed as dist

    from nimbleml_b200.kernels import fused_tied_crossentropy as k
    from nimbleml_b200 import vocab_parallel as vp
    from nimbleml_b200.losses.cross_entropy import CrossEntropyLoss

    rank, local, world = _dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    group = dist.group.WORLD if world > 1 else None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def device_bench(cfg, steps, warmup, warmup_seconds, sample_clocks, do_parity):
        """Device-timed steps of one configuration with inputs resident (the
        `value` measurement); returns its inputs, timings and parity."""
        dtype = getattr(torch, cfg["dtype"])
        n, d, v = cfg["n"], cfg["d"], cfg["v"]
        emulate = args.shard_of if world == 1 and args.shard_of > 1 else 1
        v_off, v_local = vp.shard_range(v, rank, world * emulate)
        scale = GRAD_SCALE[cfg["dtype"]]

        gen = torch.Generator(device=dev)
        gen.manual_seed(1234)  # identical h / labels on every rank
        h = torch.randn((n, d), generator=gen, device=dev, dtype=torch.float32)
        if cfg["unit_rms"]:
            h = h * torch.rsqrt(h.pow(2).mean(dim=1, keepdim=True))
        h = h.to(dtype).contiguous()
        labels = torch.randint(0, v, (n,), generator=gen, device=dev, dtype=torch.int64)
        gen_e = torch.Generator(device=dev)
        gen_e.manual_seed(99 + rank)
        e_local = (torch.randn((v_local, d), generator=gen_e, device=dev) * 0.02).to(dtype).contiguous()
        ign = k._NO_IGNORE
        gscale = torch.full((1,), scale, device=dev)

        # Per-phase CUDA events of the timed steps (current stream unless noted).
        phases = []

        def step(record=False):
            ev = None
            if record:
                names = ["start", "fwd_end", "combine_end", "compute_end", "comm_start", "comm_end", "end"]
                ev = {nm: torch.cuda.Event(enable_timing=True) for nm in names}
                ev["start"].record()
            rounded = (k.round_tf32(h), k.round_tf32(e_local)) if dtype == torch.float32 else None
            part = k.shard_forward(*(rounded or (h, e_local)), labels, v_off, rounded=rounded is not None)
            if record:
                ev["fwd_end"].record()
            stats3 = vp.gather_shard_stats(part, group)
            _, _, lse, loss, valid = k.combine(stats3, labels, v, ign)
            if record:
                ev["combine_end"].record()
            st = k.TiedCEStats(lse=lse, valid_count=valid, ignore_index=ign, vocab_size=v, vocab_offset=v_off,
                               rounded=rounded)
            if world > 1:
                dh, de = vp.sharded_backward(gscale, h, e_local, labels, st, group, phase_events=ev)
            elif emulate > 1:
                ready = torch.cuda.Event()
                sms = torch.cuda.get_device_properties(dev).multi_processor_count
                dh, de = k.shard_backward(gscale, h, e_local, labels, st, grad_hidden_dtype=vp.dh_reduce_dtype(dtype),
                                          ready_event=ready, last_de_max_ctas=max(1, sms - vp.COMM_SMS),
                                          capped_fraction=vp.CAPPED_FRACTION)
                if record:
                    ev["compute_end"].record()
                    ev["end"].record()
            else:
                dh, de = k.shard_backward(gscale, h, e_local, labels, st)
                if record:
                    ev["compute_end"].record()
                    ev["end"].record()
            if record:
                phases.append(ev)
            return stats3, lse, loss, dh, de

        # Warm-up: W steps, then more until --warmup-seconds have passed (the same
        # count on every rank), so short multi-GPU runs are not timed before the
        # GPUs reach their power-capped steady state.
        t_w = time.perf_counter()
        for _ in range(warmup):
            step()
        barrier()
        per_step = (time.perf_counter() - t_w) / warmup
        extra = max(0, math.ceil((warmup_seconds - (time.perf_counter() - t_w)) / max(per_step, 1e-4)))
        if world > 1:
            t = torch.tensor([extra], device=dev, dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            extra = int(t[0])
        for _ in range(extra):
            step()
        barrier()
        warmup_steps = warmup + extra
        assert k.check_status(dev) == 0
        bus = None
        try:
            pr = torch.cuda.get_device_properties(dev)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
        except Exception:
            pass
        sampler = ClockSampler(bus) if rank == 0 and sample_clocks else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        torch.cuda.reset_peak_memory_stats(dev)
        mem0 = torch.cuda.memory_allocated(dev)
        barrier()
        t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_start.record()
        for _ in range(steps):
            last = step(record=True)
        t_end.record()
        barrier()
        clocks = sampler.stop() if sampler else None
        elapsed = t_start.elapsed_time(t_end) / 1e3
        peak_extra = torch.cuda.max_memory_allocated(dev) - mem0
        assert k.check_status(dev) == 0

        def mean_ms(a, b):
            return statistics.mean(ev[a].elapsed_time(ev[b]) for ev in phases)

        phase_ms = {"forward_gemm_and_row_reduce": mean_ms("start", "fwd_end"),
                    "stats_exchange_and_combine": mean_ms("fwd_end", "combine_end"),
                    "backward_gemms": mean_ms("combine_end", "compute_end"),
                    "exposed_grad_hidden_reduction": mean_ms("compute_end", "end")}
        if world > 1:
            phase_ms["grad_hidden_all_reduce"] = mean_ms("comm_start", "comm_end")
            phase_ms["all_reduce_start_after_backward_start"] = mean_ms("combine_end", "comm_start")
        fwd_ms = phase_ms["forward_gemm_and_row_reduce"]
        if world > 1:
            keys = sorted(phase_ms)
            t = torch.tensor([elapsed] + [phase_ms[x] for x in keys], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            elapsed = float(t[0])
            phase_ms = {x: float(val) for x, val in zip(keys, t[1:].tolist())}
            fwd_ms = phase_ms["forward_gemm_and_row_reduce"]

        parity = None
        if do_parity and emulate == 1:
            stats3, lse, loss, dh, de = last
            parity = sampled_parity(h, e_local, labels, v, v_off, world, group, stats3, lse, loss, dh, de, scale)
        del last
        return dict(h=h, labels=labels, e_local=e_local, v_off=v_off, v_local=v_local, scale=scale, dtype=dtype,
                    elapsed=elapsed, phase_ms=phase_ms, fwd_ms=fwd_ms, parity=parity, peak_extra=peak_extra,
                    clocks=clocks, warmup_steps=warmup_steps, emulate=emulate)

    R = device_bench(cfg, args.steps, args.warmup, args.warmup_seconds, True, not args.no_parity)
    h, labels, e_local, v_off, v_local = R["h"], R["labels"], R["e_local"], R["v_off"], R["v_local"]
    scale, dtype, elapsed, phase_ms, fwd_ms = R["scale"], R["dtype"], R["elapsed"], R["phase_ms"], R["fwd_ms"]
    parity, peak_extra, clocks, warmup_steps = R["parity"], R["peak_extra"], R["clocks"], R["warmup_steps"]
    emulate = R["emulate"]
    n, d, v = cfg["n"], cfg["d"], cfg["v"]
    del R

    # ---- end to end through the public API: host inputs, H2D copy, loss D2H.
    e2e = None
    if not args.no_e2e:
        h_host = h.cpu().pin_memory()
        y_host = labels.cpu().pin_memory()
        w_param = e_local.clone().requires_grad_(True)
        head = vp.VocabParallelTiedHead(None, v, group=group, shard=w_param) if world > 1 else None
        lossfn = CrossEntropyLoss()

        # Inputs are double-buffered on the device and step i+1's copies run on
        # a side stream while step i computes (a prefetching input pipeline;
        # every timed step still copies its own inputs). Several GPUs: each
        # rank copies 1/P of h from the host, an NVLink all_gather assembles
        # the rest.
        copy_stream = torch.cuda.Stream(dev)
        main_stream = torch.cuda.current_stream(dev)
        hbuf = [torch.empty_like(h) for _ in range(2)]
        ybuf = [torch.empty_like(labels) for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]

        def prefetch(i):
            with torch.cuda.stream(copy_stream):
                if head is None:
                    hbuf[i % 2].copy_(h_host, non_blocking=True)
                else:
                    # This rank's 1/P of the rows from pinned host memory, the
                    # rest by one NVLink all_gather (NCCL keeps collectives in
                    # issue order, so it cannot cross the backward's all_reduce).
                    full = head.hidden_from_host(h_host)
                    full.record_stream(main_stream)  # used there by step i
                    hbuf[i % 2] = full
                ybuf[i % 2].copy_(y_host, non_blocking=True)
                ready[i % 2].record(copy_stream)

        def e2e_step(i, k):
            w_param.grad = None
            if i == 0:
                prefetch(0)
            if i + 1 < k:
                prefetch(i + 1)  # buffer (i+1)%2 is free: step i-1 ended with a host sync
            torch.cuda.current_stream(dev).wait_event(ready[i % 2])
            hd = hbuf[i % 2].detach().requires_grad_(True)
            yd = ybuf[i % 2]
            if head is None:
                loss = lossfn.forward_tied(hd.view(cfg["batch"], cfg["seq"], d), w_param, yd)
            else:
                loss = head.loss(hd, yd)
            (loss * scale).backward()  # the same loss scale as the device-timed step
            return float(loss)

        for i in range(args.warmup):
            e2e_step(i, args.warmup)
        barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_step(i, args.steps)
        barrier()
        te = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([te], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            te = float(t[0])
        e2e = {"value": n * args.steps / te, "unit": "tokens/s",
               "h2d_bytes_per_step": h_host.numel() * h_host.element_size() // world + y_host.numel() * 8,
               "d2h_bytes_per_step": 4, "bytes_are": "per rank"}

    # ---- the other configurations of the path, device-timed at the same N
    # (config 3 fp16, config 2 fp32 on TF32), each with its own parity check.
    also = {}
    also_ok = True
    if args.also and args.config == "c4" and emulate == 1:
        for name in [x for x in args.also.split(",") if x]:
            c = CONFIGS[name]
            torch.cuda.empty_cache()
            r = device_bench(c, 20, 3, 2.0, False, not args.no_parity)
            st = r["elapsed"] / 20
            also[name] = {"workload": c["workload"], "value": c["n"] / st, "unit": "tokens/s", "ms_per_step": st * 1e3,
                          "steps": 20, "warmup": r["warmup_steps"], "dtype": DTYPE_TAG[c["dtype"]],
                          "n_tokens": c["n"], "d_model": c["d"], "vocab": c["v"],
                          "step_tflops_per_gpu": 8.0 * c["n"] * c["d"] * r["v_local"] / st / 1e12,
                          "phases_ms": r["phase_ms"], "parity": r["parity"]}
            if r["parity"] is not None and not r["parity"]["ok"]:
                also_ok = False
            del r
        if world == 1 and args.also_c5:
            # Config 5: one GPT training step (one GPU) around this library's head.
            torch.cuda.empty_cache()
            also["c5"] = c5_measure(5, 3)

    if rank != 0:
        dist.barrier() if world > 1 else None
        dist.destroy_process_group() if world > 1 else None
        if (parity is not None and not parity["ok"]) or not also_ok:
            sys.exit(3)
        return

    burst, sustained, hbm, peak_kind = _peaks()
    step_s = elapsed / args.steps
    flops_step_rank = 8.0 * n * d * v_local
    flops_fwd_launch = 2.0 * n * d * v_local
    fwd_tflops = flops_fwd_launch / (fwd_ms / 1e3) / 1e12
    step_tflops = flops_step_rank / step_s / 1e12
    datasheet = DATASHEET_DENSE_TF32_TFLOPS if cfg["dtype"] == "float32" else DATASHEET_DENSE_F16_TFLOPS
    k_launch, n_slabs = launches_per_step(cfg, world, k.SLAB_BYTES)
    traffic = _profile_traffic(args.config) if world == 1 else None
    line = {
        "metric": METRIC if emulate == 1 else f"profiling: rank-0 shard of {emulate} on one GPU, no collectives",
        "value": n / step_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": warmup_steps, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": DTYPE_TAG[cfg["dtype"]], "data": "synthetic",
        "config": {"workload": cfg["workload"], "n_tokens": n, "batch": cfg["batch"], "seq_len": cfg["seq"],
                   "d_model": d, "vocab": v, "parallelism": f"vocab-sharded x{world}" if world > 1 else "1 GPU",
                   "l2": "inputs larger than L2 (h %.0f MB, E %.0f MB), no flush" % (
                       n * d * h.element_size() / 1e6, v * d * h.element_size() / 1e6),
                   "grad_scale": scale,
                   "grad_dtypes": {"grad_hidden": (DTYPE_TAG[str(vp.dh_reduce_dtype(dtype)).replace("torch.", "")]
                                                   + " (all-reduced)") if world > 1 else DTYPE_TAG[cfg["dtype"]],
                                   "grad_weights": DTYPE_TAG[cfg["dtype"]]},
                   "last_de_capped_fraction": vp.CAPPED_FRACTION if world > 1 else None,
                   "backward_slabs": n_slabs, "warmup_seconds": args.warmup_seconds},
        "roofline": {"bound": "tensor", "kernel": "tc_gemm_tn_kernel<EPI_CE_FWD> (+ ce_row_reduce_kernel)",
                     "achieved": fwd_tflops, "peak": sustained, "unit": "TFLOP/s",
                     "frac": fwd_tflops / sustained, "peak_kind": f"{peak_kind} sustained bf16 cuBLAS",
                     "traffic": traffic, "flops_per_launch": flops_fwd_launch,
                     "step_tflops_per_gpu": step_tflops, "step_frac_of_measured": step_tflops / sustained,
                     "step_frac_of_datasheet_dense": step_tflops / datasheet},
        "phases_ms": phase_ms,
        "parity": parity,
        "gpu_launches": k_launch * args.steps,
        "clocks": clocks,
        "memory": {"peak_extra_bytes": int(peak_extra), "materialised_logits_bytes": n * v * h.element_size(),
                   "reference_style_peak_bytes": 3 * n * v * h.element_size()},
        "e2e": e2e,
        "also": also or None,
    }
    if world == 1 and not args.no_cpu_baseline:
        step_fn, rows, sample, kind, threads = cpu_reference_sample(cfg)
        step_fn()
        t0 = time.perf_counter()
        step_fn()
        tc = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": rows / tc, "unit": "tokens/s", "cores": threads, "kind": kind,
                                "sample": sample}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if (parity is not None and not parity["ok"]) or not also_ok:
        print("parity check FAILED: " + json.dumps({"headline": parity, "also": also}), file=sys.stderr, flush=True)
        sys.exit(3)


if __name__ == "__main__":
    main()
