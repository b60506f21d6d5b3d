"""Benchmark of the LongSpark drafting round on B200 (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload: Qwen3-8B-shaped drafter (H=4096, 32/8 heads,
I=12288, V=151936, 1 drafter layer, 5 tapped layers, Markov rank 256), batch 1,
paged KV cache (page 16, shuffled page table) at 1K/8K/32K/64K/128K context,
W=1024, S=256, 16-token verify block (anchor + 15 proposals).  A step is one
full round: view refresh of a 16-row commit over the 5 tapped layers, the
parallel drafter pass, the Markov greedy chain and the accept check, replayed
as one CUDA graph.  Weights and inputs are synthetic (seeded N(0, 0.02) weights,
N(0, 1) K/V); the 1.9 GB of weights streamed per round exceed the 126 MB L2, so
no flush is needed between steps.  ``value`` is the headline context (128K).

Multi-GPU (``torchrun --nproc-per-node N``): requests shard across GPUs with
no cross-GPU traffic (each rank runs its own batch), so scaling is weak and
``value`` sums the ranks' tokens over the max-over-ranks time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "draft-round latency (µs) + HBM GB/s vs ctx 1K–128K; tokens/s at 1/2/4/8 B200"
CONTEXTS = (1024, 8192, 32768, 65536, 131072)
HEADLINE_CTX = 131072


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sweep-steps", type=int, default=300)
    ap.add_argument("--load-seconds", type=float, default=0.5,
                    help="untimed load before the timed steps, so clock samples see the GPU busy")
    ap.add_argument("--contexts", type=str, default=",".join(str(c) for c in CONTEXTS),
                    help="comma-separated context lengths of the sweep (the headline is the largest)")
    ap.add_argument("--batch-sweep", type=str, default="8,32,128",
                    help="BASELINE config 4 concurrency sweep: requests per GPU (contexts U[2K, 32K]); '' to skip")
    ap.add_argument("--tp", action="store_true",
                    help="BASELINE config 5: the 14B drafter tensor-parallel over the torchrun ranks (batch 32, 64K "
                         "context), fused peer-store allreduce vs NCCL allreduce")
    ap.add_argument("--no-tp", action="store_true",
                    help="at N > 1, skip the config-5 tensor-parallel section of the request-sharded line")
    ap.add_argument("--tp-batch", type=int, default=32)
    ap.add_argument("--tp-ctx", type=int, default=65536)
    ap.add_argument("--calls", action="store_true",
                    help="diagnostic: device time of every native call of one eager round (one GPU), not a bench line")
    ap.add_argument("--calls-shape", default="cfg2", help="cfg2, or cfg5-tpN: the per-rank shapes of config 5 at TP N")
    ap.add_argument("--calls-ctx", type=int, default=4096)
    ap.add_argument("--calls-prefill", action="store_true",
                    help="with --calls: also one ls_prefill_summary over every request's whole prefix per round")
    ap.add_argument("--calls-temperature", type=float, default=0.0,
                    help="> 0: the round includes the sampled chain (DraftEngine.sample)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=__import__("datetime").timedelta(seconds=300))
    return rank, world, local


def dist_max(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU oracle baseline (bounded sample of the same workload)
# ---------------------------------------------------------------------------

def host_cores():
    """Cores this process may run on (its affinity mask)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_round_sample(shape, ctx, rounds, seed=0, warmup=0, threads=None):
    """Time the numpy oracle (fp32, the reference drafter's CPU path restated)
    on ``rounds`` drafting rounds of the workload, after ``warmup`` untimed
    rounds, with the BLAS pool set to ``threads`` (default: every core of the
    affinity mask) whatever the launcher set OMP_NUM_THREADS to.  Returns
    (median seconds per round, BLAS threads in use)."""
    import numpy  # noqa: F401  (the BLAS pool must be loaded for the limit to reach it)
    from threadpoolctl import threadpool_info, threadpool_limits
    threads = threads or host_cores()
    with threadpool_limits(limits=threads, user_api="blas"):
        used = [d["num_threads"] for d in threadpool_info() if d.get("user_api") == "blas"]
        sec = _cpu_rounds(shape, ctx, rounds, seed, warmup)
    return sec, (max(used) if used else 1)


def _cpu_rounds(shape, ctx, rounds, seed, warmup):
    import numpy as np
    import oracle as O

    rng = np.random.default_rng(seed)
    H, Hq, Hkv, I, V, L, S, Wn = (shape.hidden, shape.q_heads, shape.kv_heads, shape.inter, shape.vocab,
                                  shape.tap_layers, shape.slots, shape.window)

    def nrm(*s, std=0.02):
        return (rng.standard_normal(s, dtype=np.float32) * std).astype(np.float32)

    W = {"draft_state_encoder.proj.net.0.weight": nrm(H, L * H), "draft_state_encoder.proj.net.2.weight": nrm(H, H),
         "draft_state_encoder.norm.weight": np.ones(H, np.float32),
         "parallel_shifted_input.position_embedding.weight": nrm(shape.block, H),
         "parallel_shifted_input.proj.net.0.weight": nrm(H, 2 * H), "parallel_shifted_input.proj.net.2.weight": nrm(H, H),
         "parallel_shifted_input.norm.weight": np.ones(H, np.float32),
         "model.embed_tokens.weight": nrm(V, H), "lm_head.weight": nrm(V, H), "model.norm.weight": np.ones(H, np.float32),
         "parallel_markov_head.markov_w1.weight": nrm(V, shape.markov_rank),
         "parallel_markov_head.markov_w2.weight": nrm(V, shape.markov_rank)}
    for j in range(shape.draft_layers):
        p = f"parallel_qwen_layers.{j}."
        W.update({p + "self_attn.q_proj.weight": nrm(Hq * 128, H), p + "self_attn.k_proj.weight": nrm(Hkv * 128, H),
                  p + "self_attn.v_proj.weight": nrm(Hkv * 128, H), p + "self_attn.o_proj.weight": nrm(H, Hq * 128),
                  p + "self_attn.q_norm.weight": np.ones(128, np.float32),
                  p + "self_attn.k_norm.weight": np.ones(128, np.float32),
                  p + "mlp.gate_proj.weight": nrm(I, H), p + "mlp.up_proj.weight": nrm(I, H),
                  p + "mlp.down_proj.weight": nrm(H, I), p + "input_layernorm.weight": np.ones(H, np.float32),
                  p + "post_attention_layernorm.weight": np.ones(H, np.float32)})
    qg = nrm(L, Hq, S, 128)
    win_k = rng.standard_normal((1, Hkv, Wn, 128), dtype=np.float32)
    win_v = rng.standard_normal((1, Hkv, Wn, 128), dtype=np.float32)
    out = nrm(1, L, Hq, S, 128, std=0.1)
    lse = np.full((1, L, Hq, S), 10.0, np.float32)
    new_k = rng.standard_normal((L, 1, shape.max_commit, Hkv, 128), dtype=np.float32)
    new_v = rng.standard_normal((L, 1, shape.max_commit, Hkv, 128), dtype=np.float32)
    hidden = rng.standard_normal((1, L, H), dtype=np.float32)
    inv = (1.0 / (np.float32(shape.rope_theta) ** (np.arange(0, 128, 2, dtype=np.float32) / 128))).astype(np.float32)
    osh = O.DraftShapeOracle(H, Hq, Hkv, 128, shape.block, shape.mask_token_id)
    target = rng.integers(0, V, (1, shape.block + 1))
    times = []
    for i in range(warmup + rounds):
        t0 = time.perf_counter()
        out, lse = O.refresh_views(out, lse, np.array([0]), qg, new_k, new_v, np.array([shape.max_commit]),
                                   128 ** -0.5)
        views = [dict(qg=qg[j], summary_out=out[:, j], win_k=win_k, win_v=win_v, win_len=np.array([Wn]))
                 for j in range(shape.draft_layers)]
        base, _ = O.draft_pass(W, osh, np.array([7]), np.array([ctx]), hidden, views, inv, "fp32")
        toks, _ = O.markov_sample(base, np.array([7]), W, "fp32")
        O.accept_lengths(target, toks)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return statistics.median(times)


def cpu_cfg1_row():
    """BASELINE config 1, the primary CPU row: one fp32 round of the oracle
    at the Qwen3-4B shape (H=2560, 4K context, W=512, S=64, 16-token verify
    block, one tapped and one drafter layer), median of 5 rounds after 2
    warm-up rounds, on every host core."""
    from longspark_b200.config import CFG1
    sec, threads = cpu_round_sample(CFG1.shape, 4096, rounds=5, warmup=2)
    return {"value": round(CFG1.shape.block / sec, 2), "unit": "draft tokens/s", "ms_per_round": round(sec * 1e3, 1),
            "cores": threads, "kind": "port",
            "sample": "BASELINE config 1 (Qwen3-4B shape, 4K context, W=512, S=64, B=16, batch 1): median of 5 fp32 "
                      "rounds of the numpy restatement after 2 warm-ups"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def build_round(shape, ctx, batch, dev, seed):
    import torch
    from longspark_b200.engine import DraftEngine, DraftWeights, GraphedDraft, ViewPools
    from longspark_b200.synthetic import make_views, make_weights

    gen = torch.Generator(device=dev).manual_seed(seed)
    W = make_weights(shape, device=dev, gen=gen)
    v = make_views(shape, batch, ctx, device=dev, gen=gen, extra_rows=shape.max_commit)
    pools = ViewPools(kv_k=v["kv_k"], kv_v=v["kv_v"], page_table=v["page_table"], summary_out=v["summary_out"],
                      summary_lse=v["summary_lse"], hidden=v["hidden"])
    eng = DraftEngine(shape, DraftWeights(shape, W, dev), pools, max_batch=batch, device=dev)
    del W
    g = GraphedDraft(eng, batch, with_refresh=True, with_target=True, slots_are_rows=True)
    commit = torch.full((batch,), shape.max_commit, dtype=torch.int32, device=dev)
    target = torch.randint(0, shape.vocab, (batch, shape.block + 1), device=dev, generator=gen)
    g.load(slots=torch.arange(batch, dtype=torch.int32, device=dev), seq_lens=v["seq_lens"], anchors=v["anchors"],
           page_table=v["page_table"], commit_lens=commit, target=target)
    return eng, g, v


def concurrency_round(shape, batch, dev, seed, steps=30, view_peak=None):
    """one graph-replayed round for ``batch`` requests with
    per-request contexts uniform in [2K, 32K]; returns (ms per round, status,
    view-kernel timings when ``view_peak`` is given, else None)."""
    import torch
    from longspark_b200.engine import DraftEngine, DraftWeights, GraphedDraft, ViewPools
    from longspark_b200.synthetic import make_views, make_weights

    gen = torch.Generator(device=dev).manual_seed(seed)
    W = make_weights(shape, device=dev, gen=gen)
    weights = DraftWeights(shape, W, dev)
    del W
    ctxs = torch.randint(2048, 32769, (batch,), generator=torch.Generator().manual_seed(seed + batch)).tolist()
    v = make_views(shape, batch, ctxs, device=dev, gen=gen, extra_rows=shape.max_commit)
    pools = ViewPools(kv_k=v["kv_k"], kv_v=v["kv_v"], page_table=v["page_table"], summary_out=v["summary_out"],
                      summary_lse=v["summary_lse"], hidden=v["hidden"])
    eng = DraftEngine(shape, weights, pools, max_batch=batch, device=dev)
    g = GraphedDraft(eng, batch, with_refresh=True, with_target=True, slots_are_rows=True)
    g.load(slots=torch.arange(batch, dtype=torch.int32, device=dev), seq_lens=v["seq_lens"], anchors=v["anchors"],
           page_table=v["page_table"],
           commit_lens=torch.full((batch,), shape.max_commit, dtype=torch.int32, device=dev),
           target=torch.randint(0, shape.vocab, (batch, shape.block + 1), device=dev, generator=gen))
    g.capture()
    ms = time_graph(g, steps, 3, 1)
    status = eng.device_status()
    views = time_view_kernels(eng, g, view_peak) if view_peak else None
    del g, eng, pools, v, weights
    torch.cuda.empty_cache()
    return ms, status, views


def view_kernel_bytes(shape, eng, g):
    """Algorithmic HBM bytes of one refresh launch and one attention launch
    for the graph's batch: what each must read or write at least once.
    Refresh, per request and tapped layer: the committed K/V rows, the fp32
    state (output + lse) read and written; plus the bf16 state copy of the
    drafter layers; the learned queries once per launch.  Attention, per
    request (drafter layer 0): the window K/V rows (up to W), the bf16
    summary values, q/k/v of the block in and its output out, the window's
    page ids; the learned queries (the summary keys) once per launch."""
    s = shape
    B = g.batch
    lens = g.seq_lens[:B].tolist()
    commits = g.commit_lens[:B].tolist()
    D = s.head_dim
    qg_layer = s.q_heads * s.slots * D * 2
    refresh = s.tap_layers * qg_layer
    attn = qg_layer
    for n, c in zip(lens, commits):
        refresh += s.tap_layers * (2 * c * s.kv_heads * D * 2 + 2 * s.q_heads * s.slots * (D + 1) * 4)
        refresh += s.draft_layers * s.q_heads * s.slots * D * 2
        w = min(n, s.window)
        attn += (2 * w * s.kv_heads * D * 2 + s.q_heads * s.slots * D * 2 + (w + 15) // 16 * 4
                 + s.block * (s.q_heads + 2 * s.kv_heads) * D * 2 + s.block * s.q_heads * D * 2)
    return refresh, attn


def time_view_kernels(eng, g, hbm_peak, reps=20):
    """The refresh (every tapped layer) and the drafter attention (layer 0)
    launched alone on the round's live buffers, each launch after a 256 MiB
    write (twice the L2) and bracketed by its own CUDA events; median ms per
    launch, achieved GB/s of the algorithmic bytes and the fraction of the
    measured HBM copy peak."""
    import torch
    from longspark_b200 import ops
    s, p, b = eng.shape, eng.pools, eng.buf
    B = g.batch
    v = s.view_layer(0)

    def refresh():
        eng.refresh(slots=g.slots, seq_lens=g.seq_lens, commit_lens=g.commit_lens, page_table=g.page_table, batch=B)

    def attention():
        ops.draft_attention(qkv=b["qkv"], block=s.block, kv_k=p.kv_k[v], kv_v=p.kv_v[v], page_table=g.page_table,
                            seq_lens=g.seq_lens, window=s.window, learned_query=eng.w.learned_query[v],
                            state_out=p.summary_out[:, v], slots=g.slots, out=b["attn"], workspace=eng.attn_ws,
                            q_heads=s.q_heads, kv_heads=s.kv_heads, ring_pages=p.ring_pages,
                            softmax_scale=s.head_dim ** -0.5, status=b["status"], batch=B,
                            state_bf16=p.summary_bf16[:, v])

    # the refresh folds the same rows again at every launch: keep the state
    saved = (p.summary_out.clone(), p.summary_lse.clone(), p.summary_bf16.clone())
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=eng.device)
    st = torch.cuda.current_stream()
    rb, ab = view_kernel_bytes(s, eng, g)
    out = {}
    for name, fn, nbytes in (("refresh", refresh, rb), ("attention", attention, ab)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for e0, e1 in ev:
            flush.fill_(1)
            e0.record(st)
            fn()
            e1.record(st)
        torch.cuda.synchronize()
        ts = sorted(e0.elapsed_time(e1) for e0, e1 in ev)
        ms = ts[len(ts) // 2]
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 2), "algorithmic_bytes": int(nbytes), "gbs": round(gbs, 1),
                     "frac": round(gbs / hbm_peak, 3)}
    p.summary_out.copy_(saved[0])
    p.summary_lse.copy_(saved[1])
    p.summary_bf16.copy_(saved[2])
    out["status"] = eng.device_status()
    del flush
    return out


def algorithmic_bytes(shape, eng, batch):
    """HBM bytes a round must move (one pass over every streamed weight, the
    summary state read+write, learned queries, window K/V, new rows)."""
    s = shape
    w = eng.w.nbytes()
    refresh = s.tap_layers * (2 * s.max_commit * s.kv_heads * 128 * 2 + s.q_heads * s.slots * 128 * 2
                              + 2 * s.q_heads * s.slots * 129 * 4)
    attn = s.draft_layers * (2 * s.window * s.kv_heads * 128 * 2 + s.q_heads * s.slots * 128 * (4 + 2))
    return w + batch * (refresh + attn)


def time_graph(g, steps, warmup, world, load_seconds=0.0):
    """Mean ms per replay over exactly ``steps`` replays (CUDA events on the
    launching stream), after ``warmup`` replays plus, when ``load_seconds`` > 0,
    enough extra untimed replays to keep the GPU busy that long (so clock
    samples taken around the timed region see it under load)."""
    import torch
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if load_seconds > 0:
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < load_seconds:
            for _ in range(50):
                g.replay()
            torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    barrier(world)
    return e0.elapsed_time(e1) / steps  # ms


def time_dominant_kernel(eng, reps=20):
    """CUDA-event duration of the vocabulary-projection GEMM (the largest single
    weight stream of the round) launched on the current stream with the round's
    live buffers; returns ms per launch."""
    import torch
    from longspark_b200 import _native as N
    from longspark_b200 import ops
    b, w, s = eng.buf, eng.w, eng.shape
    M = eng.max_batch * s.block

    def launch():
        ops.gemm(b["xn"], w.lm_head, b["logits"], workspace=eng.gemm_ws, epilogue=N.EPI_LMHEAD, rows=M,
                 tile_max=b["tile_max"], tile_arg=b["tile_arg"])

    # Each launch is bracketed by its own events, with a 256 MiB write (twice the
    # L2) before it, so no launch starts on L2-resident weights or overlaps the
    # tail of the previous one.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for e0, e1 in ev:
        flush.fill_(1)
        e0.record(st)
        launch()
        e1.record(st)
    torch.cuda.synchronize()
    return sum(e0.elapsed_time(e1) for e0, e1 in ev) / reps


def time_prefill_summary(eng, v, batch, reps=5):
    """ls_prefill_summary over the whole synthetic prefix of every request
    (the state a prefill packet would carry): ms per launch (CUDA events,
    after one warm-up launch) and the algorithmic FLOPs of one launch
    (4 * D flops per (learned query, prefix key): q.k and p.v)."""
    import torch
    s = eng.shape
    slots = torch.arange(batch, dtype=torch.int32, device=eng.device)
    lens = v["seq_lens"][:batch]
    eng.prefill_summary(slots=slots, seq_lens=lens, page_table=v["page_table"], batch=batch)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        eng.prefill_summary(slots=slots, seq_lens=lens, page_table=v["page_table"], batch=batch)
    e1.record(st)
    torch.cuda.synchronize()
    flops = 4.0 * s.head_dim * s.tap_layers * s.q_heads * s.slots * float(lens.sum().item())
    return e0.elapsed_time(e1) / reps, flops, eng.device_status()


def time_sampled_round(eng, g, steps=50):
    """T > 0 round (LongSparkDraft.propose(temperature > 0)): the drafter pass
    (with the refresh) plus the 15-step sampled chain, one CUDA graph; ms per
    replay and the HBM bytes the chain adds per round (the Markov w2 matrix
    once per step, the reference's algorithm)."""
    import torch
    s, b = eng.shape, eng.buf
    B = g.batch

    def run():
        g._run()
        eng.sample(g.anchors, temperature=0.8, seed=12345, batch=B)

    side = torch.cuda.Stream(device=eng.device)
    side.wait_stream(torch.cuda.current_stream(eng.device))
    with torch.cuda.stream(side):
        run()
    torch.cuda.current_stream(eng.device).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        run()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    del graph
    chain_bytes = s.block * (eng.w.w2.numel() * 2 if eng.w.w2 is not None else 0)
    return e0.elapsed_time(e1) / steps, chain_bytes, eng.device_status()


def time_export(shape, dev, batch=32, reps=20):
    """ls_export_rows for one decode step at the cfg2 shapes: ``batch``
    requests x max_commit rows of every tapped layer gathered from a target
    pool and stored into a drafter pool on the same GPU (LongSparkDraft's ring
    layout), plus the boundary hidden states; median ms per launch over
    ``reps`` launches, each after a 256 MiB L2 flush, and the bytes it moves.
    The argument block is staged once; the timed region holds the launch
    alone, queued behind the flush so the GPU does not wait on the host."""
    import torch
    from longspark_b200.export import ExportDestination, prepare_export
    s = shape
    L, H, c, ring = s.tap_layers, s.kv_heads, s.max_commit, s.window // 16
    rows = batch * c
    gen = torch.Generator(device=dev).manual_seed(5)
    src_k = [torch.randn(4 * rows, H, 128, device=dev, generator=gen).to(torch.bfloat16) for _ in range(L)]
    src_v = [torch.randn(4 * rows, H, 128, device=dev, generator=gen).to(torch.bfloat16) for _ in range(L)]
    loc = torch.randperm(4 * rows, device=dev, generator=gen)[:rows]
    pool_k = torch.zeros(L, batch * ring, 16, H, 128, dtype=torch.bfloat16, device=dev)
    pool_v = torch.zeros_like(pool_k)
    hid = torch.zeros(batch, L * s.hidden, dtype=torch.bfloat16, device=dev)
    last_hidden = torch.randn(batch, L, s.hidden, device=dev, generator=gen).to(torch.bfloat16)
    slots = torch.arange(batch, dtype=torch.int32, device=dev)
    table = (slots[:, None] * ring + torch.arange(ring, dtype=torch.int32, device=dev)[None]).contiguous()
    lens = torch.full((batch,), 32768 + c, dtype=torch.int32, device=dev)
    dest = ExportDestination(kv_k=pool_k.data_ptr(), kv_v=pool_v.data_ptr(), pool_pages=batch * ring, heads=H,
                             tap_layers=L, ring_pages=ring, page_table=table, seq_lens=lens, slots=slots,
                             hidden_pool=hid.data_ptr(), capacity=batch, hidden=s.hidden)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    counts = [c] * batch
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    prep = prepare_export(dest, src_k=src_k, src_v=src_v, locations=loc, counts=counts, last_hidden=last_hidden,
                          status=status)
    ts = []
    for i in range(reps + 2):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        prep.launch()
        e1.record()
        torch.cuda.synchronize()
        if i >= 2:
            ts.append(e0.elapsed_time(e1))
    ts.sort()
    moved = 2 * (2 * L * rows * H * 128 * 2) + 2 * batch * L * s.hidden * 2  # K and V read + written, hidden
    return ts[len(ts) // 2], moved, int(status.item())


def count_launches(eng, g):
    """Kernels of one round, counted from the native calls of an eager run."""
    from longspark_b200 import _native as N
    counts = {"ls_row_norm_bound": 1}
    seen = []
    orig = N.call

    def counting(name, *args):
        seen.append(name)
        return orig(name, *args)

    N.call = counting
    try:
        g._run()
    finally:
        N.call = orig
    return sum(counts.get(n, 1) for n in seen)


def e2e_api(shape, batch, steps, warmup, dev, world):
    """Through the drop-in API: per step, the committed K/V rows, boundary hidden
    state and metadata go host->device (pinned), ``update`` folds them,
    ``propose`` drafts, and the tokens come back device->host."""
    import torch
    from longspark_b200.draft import LongSparkDraft
    from longspark_b200.synthetic import make_weights

    gen = torch.Generator(device=dev).manual_seed(7)
    W = make_weights(shape, device=dev, gen=gen)
    cfg = dict(draft_device=dev.index or 0, max_running_requests=batch, draft_state_gib=16.0, cuda_graph=True,
               graph_batch_sizes=(batch,))
    d = LongSparkDraft(cfg, weights=W, shape=shape, materialize_logits=True)
    del W
    L, Hkv, Hq, S, Wn = shape.tap_layers, shape.kv_heads, shape.q_heads, shape.slots, shape.window
    ids = [f"r{i}" for i in range(batch)]
    length = HEADLINE_CTX
    pk = torch.randn(L, batch * Wn, Hkv, 128).to(torch.bfloat16)
    d.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=[length] * batch, commit_lens=[Wn] * batch,
                  export_counts=[Wn] * batch, keys=pk, values=pk.clone(),
                  last_hidden=torch.randn(batch, L, shape.hidden).to(torch.bfloat16),
                  global_output=0.1 * torch.randn(batch, L, Hq, S, 128), global_lse=torch.full((batch, L, Hq, S), 11.0)),
             prefill=True)
    c = shape.max_commit
    keys = torch.randn(L, batch * c, Hkv, 128).to(torch.bfloat16).pin_memory()
    vals = torch.randn(L, batch * c, Hkv, 128).to(torch.bfloat16).pin_memory()
    hid = torch.randn(batch, L, shape.hidden).to(torch.bfloat16).pin_memory()
    anchors = torch.randint(0, shape.vocab, (batch,)).pin_memory()
    h2d = keys.numel() * 2 + vals.numel() * 2 + hid.numel() * 2 + anchors.numel() * 8 + batch * 4 * 5
    d2h = batch * shape.block * 8

    def step():
        nonlocal length
        length += c
        d.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=[length] * batch, commit_lens=[c] * batch,
                      export_counts=[c] * batch, keys=keys, values=vals, last_hidden=hid))
        toks, logits, _ = d.propose(ids, anchors, 0.0)  # logits [B, P, V] bf16 stay on the device
        return toks.cpu()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1) / steps
    wall = (time.perf_counter() - t0) / steps * 1e3
    status = d.device_status()
    return max(ms, wall), h2d, d2h, status


def run_b200(args):
    import torch
    from longspark_b200.config import CFG2

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shape = CFG2.shape
    batch = args.batch
    peaks = {}
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        peaks = json.loads(pp.read_text())
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    tensor_peak = float(peaks.get("bf16_tflops", 1590.0))
    tensor_peak_sustained = float(peaks.get("bf16_tflops_sustained", 1400.0))

    # context sweep (each context its own synthetic cache; same weights seed)
    sweep = []
    headline = None
    contexts = sorted(int(c) for c in args.contexts.split(","))
    head_ctx = contexts[-1]
    for ctx in contexts:
        eng, g, v = build_round(shape, ctx, batch, dev, seed=1000 + rank)
        g.capture()
        steps = args.steps if ctx == head_ctx else args.sweep_steps
        if ctx == head_ctx:
            with ClockSampler(local) as clk:
                ms = time_graph(g, steps, max(3, args.warmup), world, load_seconds=args.load_seconds)
            ms_max = dist_max(ms, world)
            launches = count_launches(eng, g)
            status = eng.device_status()
            dom_ms = time_dominant_kernel(eng)
            abytes = algorithmic_bytes(shape, eng, batch)
            pf_ms, pf_flops, pf_status = time_prefill_summary(eng, v, batch)
            sr_ms, sr_bytes, sr_status = time_sampled_round(eng, g)
            ex_ms, ex_bytes, ex_status = time_export(shape, dev)
            views = time_view_kernels(eng, g, hbm_peak)
            headline = dict(views=views, ms=ms_max, clocks=clk.summary(), launches=launches, status=status, dom_ms=dom_ms,
                            abytes=abytes, eng=eng, prefill=(pf_ms, pf_flops, pf_status),
                            sampled=(sr_ms, sr_bytes, sr_status), export=(ex_ms, ex_bytes, ex_status))
        else:
            ms_max = dist_max(time_graph(g, steps, 3, world), world)
            abytes = algorithmic_bytes(shape, eng, batch)
        sweep.append({"ctx": ctx, "round_us": round(ms_max * 1e3, 1),
                      "hbm_gbs": round(abytes / (ms_max * 1e-3) / 1e9, 1)})
        if ctx != head_ctx:
            del eng, g, v
            torch.cuda.empty_cache()

    ms = headline["ms"]
    tokens_per_round = batch * shape.block
    value = tokens_per_round * world / (ms * 1e-3)
    eng = headline["eng"]
    lm_bytes = eng.w.lm_head.numel() * 2 + batch * shape.block * shape.hidden * 2 + \
        batch * shape.block * shape.vocab * 2
    dom_gbs = lm_bytes / (headline["dom_ms"] * 1e-3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / "lm_head_gemm_traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get("dram_bytes_per_launch")

    e2e = None
    if not args.no_e2e:
        del headline["eng"], eng
        torch.cuda.empty_cache()
        e_ms, h2d, d2h, e_status = e2e_api(shape, batch, max(5, args.steps // 2), 3, dev, world)
        e_ms = dist_max(e_ms, world)
        e2e = {"value": round(tokens_per_round * world / (e_ms * 1e-3), 1), "unit": "draft tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms, 4),
               "path": "LongSparkDraft.update(batch packet from pinned host) + propose(T=0) returning tokens and "
                       "the Markov-corrected logits [B, 15, V] (a device tensor, as the reference returns) + "
                       "tokens.cpu()",
               "device_status": e_status}

    batch_sweep = []
    views32 = None
    for bs in [int(x) for x in args.batch_sweep.split(",") if x.strip()]:
        ms_b, st_b, vk = concurrency_round(shape, bs, dev, seed=2000 + rank, view_peak=hbm_peak if bs == 32 else None)
        ms_b = dist_max(ms_b, world)
        views32 = vk or views32
        batch_sweep.append({"requests_per_gpu": bs, "round_us": round(ms_b * 1e3, 1),
                            "draft_tokens_per_s": round(bs * shape.block * world / (ms_b * 1e-3), 1),
                            "device_status": st_b})

    tp = None
    if world > 1 and not args.no_tp:
        # BASELINE config 5 on the same ranks: the drafter split by KV-head
        # group, the fused peer-store allreduce against GEMM + NCCL
        results, roof, parity, meta = tp_bench(args, rank, world, dev)
        tp = {"config": meta, "modes": results, "parity": parity, "projection_roofline": roof,
              "projection_roofline_note": TP_ROOF_NOTE,
              "what": "cfg5 (14B, batch 32, 64K context) tensor-parallel over these ranks: whole rounds in one CUDA "
                      "graph with the fused exchange (fp32 / bf16 partials) and with GEMM + NCCL allreduce, the two "
                      "row-parallel projections alone (us per launch, max over ranks)"}

    cpu = cpu1 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, threads = cpu_round_sample(shape, HEADLINE_CTX, rounds=3, warmup=1)
        cpu = {"value": round(tokens_per_round / sec, 2), "unit": "draft tokens/s", "cores": threads, "kind": "port",
               "sample": f"median of 3 fp32 rounds (after 1 warm-up) of the numpy oracle at the cfg2 shapes, "
                         f"{sec:.3f} s/round"}
        cpu1 = cpu_cfg1_row()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "draft tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) paged K/V, shuffled 16-row pages)",
            "config": {"workload": "cfg2-qwen3-8b drafter round (BASELINE configs[1])", "batch_per_gpu": batch,
                       "hidden": shape.hidden, "q_heads": shape.q_heads, "kv_heads": shape.kv_heads,
                       "inter": shape.inter, "vocab": shape.vocab, "tap_layers": shape.tap_layers,
                       "draft_layers": shape.draft_layers, "window": shape.window, "slots": shape.slots,
                       "verify_block": shape.block + 1, "draft_rows": shape.block, "markov_rank": shape.markov_rank,
                       "headline_ctx": head_ctx, "parallelism": f"request-sharded x{world}",
                       "l2": "inputs larger than L2 (1.9 GB of weights streamed per round)",
                       "graph": "refresh + drafter pass + Markov chain + accept in one CUDA graph"},
            "round_latency_us": round(ms * 1e3, 1),
            "ctx_sweep": sweep,
            "batch_sweep": batch_sweep,
            "batch_sweep_note": ("BASELINE config 4: per-request contexts uniform in [2K, 32K], 16 committed rows "
                                 "per request per round, requests sharded over GPUs (value per box)"),
            "round_hbm_gbs": round(headline["abytes"] / (ms * 1e-3) / 1e9, 1),
            "round_algorithmic_bytes": headline["abytes"],
            "roofline": {"bound": "hbm", "kernel": "vocabulary projection GEMM (tcgen05, LS_EPI_LMHEAD)",
                         "achieved": round(dom_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(dom_gbs / hbm_peak, 3), "peak_source": peak_src,
                         "traffic": traffic, "algorithmic_bytes_per_launch": lm_bytes,
                         "launch_ms": round(headline["dom_ms"], 4)},
            "view_kernels": {
                "what": "refresh (5 tapped layers) and drafter attention (1 layer) launched alone on the round's "
                        "buffers, median of 20 launches, each after a 256 MiB L2 flush; algorithmic bytes: state "
                        "read+write, committed rows, bf16 state copy, window K/V, summary values, q/k/v/out, "
                        "learned queries once per launch; frac of the measured HBM copy peak",
                "cfg2_batch1_ctx": head_ctx, "cfg2_batch1": headline["views"],
                "cfg4_32_requests": views32},
            "tensor_parallel": tp,
            "cpu_baseline": cpu,
            "cpu_baseline_cfg1": cpu1,
            "prefill_summary": {
                "what": "ls_prefill_summary: fp32 (output, lse) of the 5 x 32 x 256 learned queries over the whole "
                        f"{head_ctx}-token prefix (replaces the target's FA3 summary pass)",
                "ms": round(headline["prefill"][0], 3),
                "tflops": round(headline["prefill"][1] / (headline["prefill"][0] * 1e-3) / 1e12, 1),
                "roofline": {"bound": "tensor", "peak": tensor_peak, "unit": "TFLOP/s",
                             "frac": round(headline["prefill"][1] / (headline["prefill"][0] * 1e-3) / 1e12
                                           / tensor_peak, 3),
                             "peak_sustained": tensor_peak_sustained,
                             "frac_sustained": round(headline["prefill"][1] / (headline["prefill"][0] * 1e-3) / 1e12
                                                     / tensor_peak_sustained, 3),
                             "note": "tcgen05 with scores and accumulators in TMEM (128-query tiles), the "
                                     "softmax weights as a bf16 high part + residual (P.V issued twice: "
                                     "executed tensor work is 1.5x the algorithmic); algorithmic flops = "
                                     "4 * 128 per (query, key); peak = burst cuBLAS bf16, peak_sustained = the "
                                     "seconds-long figure (the kernel runs for milliseconds)"},
                "device_status": headline["prefill"][2]},
            "sampled_round": {
                "what": "temperature 0.8: drafter pass with the refresh, then the 15-step chain (per step one "
                        "Markov-bias GEMM over the whole vocabulary and one Gumbel-max draw), one CUDA graph",
                "round_us": round(headline["sampled"][0] * 1e3, 1),
                "draft_tokens_per_s": round(tokens_per_round * world / (headline["sampled"][0] * 1e-3), 1),
                "hbm_gbs": round((headline["abytes"] + headline["sampled"][1]) / (headline["sampled"][0] * 1e-3)
                                 / 1e9, 1),
                "algorithmic_bytes": headline["abytes"] + headline["sampled"][1],
                "device_status": headline["sampled"][2]},
            "export_rows": {
                "what": "ls_export_rows: one decode step's accepted rows (32 requests x 16 rows x 5 tapped layers, "
                        "K and V) gathered from a target pool and stored into a drafter pool on the same GPU, plus "
                        "the boundary hidden states; median over 20 launches, each after a 256 MiB L2 flush",
                "us": round(headline["export"][0] * 1e3, 2),
                "bytes": headline["export"][1],
                "gbs": round(headline["export"][1] / (headline["export"][0] * 1e-3) / 1e9, 1),
                "device_status": headline["export"][2]},
            "e2e": e2e,
            "gpu_launches": headline["launches"] * args.steps,
            "gpu_launches_per_step": headline["launches"],
            "device_status": headline["status"],
            "clocks": headline["clocks"],
            "clocks_note": "nvidia-smi every 100 ms from 0.5 s of untimed load before the timed steps to their end",
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def tp_parity(rank, world, dev, all_gather, bar, batch=2, contexts=(3000, 700)):
    """A short check before the TP timings: one round (refresh of a 16-row
    commit + pass + chain) of the config-5 drafter on ``batch`` small requests,
    tensor-parallel with the fused fp32 exchange, against the one-GPU engine
    on the same weights and views (run on rank 0).  Returns tokens equal, the
    largest logit difference in bf16 steps, and both device statuses."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from longspark_b200 import _native as N
    from longspark_b200.config import CFG3
    from longspark_b200.engine import DraftEngine, DraftWeights, ViewPools
    from longspark_b200.synthetic import make_views, make_weights
    from longspark_b200.tp import TPDraftEngine, shard_state_dict, shard_views

    shape = CFG3.shape
    gen = torch.Generator(device=dev).manual_seed(77)  # identical on every rank
    W = make_weights(shape, device=dev, gen=gen, norm_jitter=0.05)
    v = make_views(shape, batch, list(contexts), device=dev, gen=gen, extra_rows=shape.max_commit)
    commit = torch.full((batch,), shape.max_commit, dtype=torch.int32, device=dev)
    lens = v["seq_lens"] + commit
    slots = torch.arange(batch, dtype=torch.int32, device=dev)
    M = batch * shape.block
    vl = shard_views(v, shape, rank, world)
    pools = ViewPools(kv_k=vl["kv_k"], kv_v=vl["kv_v"], page_table=v["page_table"], summary_out=vl["summary_out"],
                      summary_lse=vl["summary_lse"], hidden=v["hidden"])
    eng = TPDraftEngine(shape, {k: t.clone() for k, t in shard_state_dict(W, shape, rank, world).items()}, pools,
                        batch, rank=rank, world=world, device=dev, all_gather=all_gather, barrier=bar,
                        allreduce="fused", wire=N.TP_WIRE_F32, pg=dist.group.WORLD)
    eng.round(slots=slots, seq_lens=lens, commit_lens=commit, anchors=v["anchors"], page_table=v["page_table"],
              batch=batch)
    torch.cuda.synchronize()
    tp_status = eng.device_status()
    tp_tokens = eng.buf["tokens"][:batch].cpu().numpy()
    shards = [None] * world
    dist.all_gather_object(shards, eng.buf["logits"][:M].float().cpu().numpy())
    eng.close()
    del eng, pools
    result = None
    if rank == 0:
        one = DraftEngine(shape, DraftWeights(shape, W, dev),
                          ViewPools(kv_k=v["kv_k"], kv_v=v["kv_v"], page_table=v["page_table"],
                                    summary_out=v["summary_out"], summary_lse=v["summary_lse"], hidden=v["hidden"]),
                          max_batch=batch, device=dev)
        one.round(slots=slots, seq_lens=lens, commit_lens=commit, anchors=v["anchors"], page_table=v["page_table"],
                  batch=batch)
        torch.cuda.synchronize()
        ref = one.buf["logits"][:M].float().cpu().numpy()
        got = np.concatenate(shards, axis=1)
        step = 2.0 ** (np.floor(np.log2(np.abs(ref).max())) - 7)
        steps = float(np.abs(got - ref).max() / step)
        equal = bool(np.array_equal(tp_tokens, one.buf["tokens"][:batch].cpu().numpy()))
        result = {"what": f"config-5 drafter, {batch} requests (contexts {list(contexts)}), one round with a "
                          "16-row refresh: fused fp32 TP against the one-GPU engine",
                  "tokens_equal": equal, "logits_max_diff_bf16_steps": round(steps, 2),
                  "parity": equal and steps <= 4.0, "device_status": [tp_status, one.device_status()]}
        del one
    del W, v
    torch.cuda.empty_cache()
    bar()
    return result


def run_tp(args):
    """BASELINE config 5 as its own bench line (``--tp``): see ``tp_bench``."""
    import torch
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    results, roof, parity, meta = tp_bench(args, rank, world, dev)
    if rank == 0:
        line = {
            "metric": "cfg5 TP drafter round: draft tokens/s per box (fused peer-store allreduce vs NCCL)",
            "value": results["fused_f32"]["draft_tokens_per_s"], "unit": "draft tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": round(results["fused_f32"]["round_us"] / 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) paged K/V of this rank's heads)",
            "config": meta, "modes": results, "parity": parity, "projection_roofline": roof,
            "projection_roofline_note": TP_ROOF_NOTE,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


TP_ROOF_NOTE = ("target = max(weight bytes / measured HBM copy GB/s, bytes this rank sends over NVLink / 770 GB/s "
                "measured peer copy); fp32 partials + bf16 results")


def tp_bench(args, rank, world, dev):
    """one rank per GPU, the 14B-shaped drafter split by
    KV-head group.  Times the whole round (refresh + pass + sharded Markov chain
    + accept, one CUDA graph) with the row-parallel projections fused with the
    peer-store allreduce (fp32 and bf16 partials) and with a plain GEMM followed
    by an NCCL allreduce, plus the two decoder-layer projections alone, after a
    short parity check against the one-GPU engine (N > 1).  Returns (mode
    results, projection roofline, parity, config); every rank takes the same
    steps."""
    import torch
    import torch.distributed as dist
    from longspark_b200 import _native as N
    from longspark_b200 import ops
    from longspark_b200.config import CFG3
    from longspark_b200.engine import GraphedDraft, ViewPools
    from longspark_b200.synthetic import make_views, make_weights
    from longspark_b200.tp import TPDraftEngine, dist_helpers, local_shape, shard_state_dict

    shape = CFG3.shape
    batch, ctx = args.tp_batch, args.tp_ctx
    loc = local_shape(shape, world)
    if world > 1:
        all_gather, bar = dist_helpers()
    else:
        all_gather, bar = (lambda b: [b]), (lambda: None)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    nvlink_gbs = 770.0  # measured peer copy per direction on this pool
    parity = tp_parity(rank, world, dev, all_gather, bar) if world > 1 else None

    gen = torch.Generator(device=dev).manual_seed(5)  # the same on every rank: replicated inputs agree
    W = make_weights(shape, device=dev, gen=gen)
    Wl = {k: t.clone() for k, t in shard_state_dict(W, shape, rank, world).items()}
    del W
    torch.cuda.empty_cache()
    # this rank's heads of the paged pool and summary state, generated directly
    v = make_views(loc, batch, ctx, device=dev, gen=gen, extra_rows=shape.max_commit)
    pools = ViewPools(kv_k=v["kv_k"], kv_v=v["kv_v"], page_table=v["page_table"], summary_out=v["summary_out"],
                      summary_lse=v["summary_lse"], hidden=v["hidden"])
    commit = torch.full((batch,), shape.max_commit, dtype=torch.int32, device=dev)
    target = torch.randint(0, shape.vocab, (batch, shape.block + 1), device=dev, generator=gen)
    slots = torch.arange(batch, dtype=torch.int32, device=dev)
    M = batch * shape.block

    def round_ms(eng, graphed=True):
        g = GraphedDraft(eng, batch, with_refresh=True, with_target=True, slots_are_rows=True)
        g.load(slots=slots, seq_lens=v["seq_lens"], anchors=v["anchors"], page_table=v["page_table"],
               commit_lens=commit, target=target)
        if graphed:
            g.capture()
            ms = time_graph(g, args.steps, max(3, args.warmup), world)
        else:
            for _ in range(max(3, args.warmup)):
                g._run()
            torch.cuda.synchronize()
            barrier(world)
            st = torch.cuda.current_stream()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(args.steps):
                g._run()
            e1.record(st)
            torch.cuda.synchronize()
            barrier(world)
            ms = e0.elapsed_time(e1) / args.steps
        tokens = eng.buf["tokens"][:batch].clone()
        del g
        return dist_max(ms, world), tokens

    def projections(eng, mode):
        """us per launch of o_proj and down_proj with their allreduce (graph of
        20 launches each; 'gemm' = the local GEMM alone, no reduction)."""
        b, L = eng.buf, eng.w.layers[0]
        out = {}
        for name, x, w_ in (("o_proj", b["attn"], L["o"]), ("down_proj", b["act"], L["down"])):
            def launch():
                if mode == "fused":
                    ops.gemm_allreduce(x, w_, b["h"], group=eng.group, workspace=eng.gemm_ws, wire=eng.wire,
                                       epilogue=N.EPI_RESIDUAL, residual=b["h"], rows=M, status=b["status"])
                elif mode == "nccl":
                    ops.gemm(x, w_, b["g"], workspace=eng.gemm_ws, rows=M, status=b["status"])
                    dist.all_reduce(b["g"][:M])
                else:
                    ops.gemm(x, w_, b["g"], workspace=eng.gemm_ws, rows=M, status=b["status"])
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(3):
                    launch()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                for _ in range(20):
                    launch()
            for _ in range(3):
                gr.replay()
            torch.cuda.synchronize()
            barrier(world)
            st = torch.cuda.current_stream()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(10):
                gr.replay()
            e1.record(st)
            torch.cuda.synchronize()
            barrier(world)
            out[name] = round(dist_max(e0.elapsed_time(e1) / 200 * 1e3, world), 2)
            del gr
        return out

    results = {}
    for mode, wire in (("fused", N.TP_WIRE_F32), ("fused", N.TP_WIRE_BF16), ("nccl", N.TP_WIRE_BF16)):
        if mode == "nccl" and world == 1:
            continue
        eng = TPDraftEngine(shape, Wl, pools, batch, rank=rank, world=world, device=dev, all_gather=all_gather,
                            barrier=bar, allreduce=mode, wire=wire, pg=dist.group.WORLD if world > 1 else None)
        key = mode if mode == "nccl" else f"fused_{'bf16' if wire == N.TP_WIRE_BF16 else 'f32'}"
        try:
            ms, _ = round_ms(eng, graphed=True)
            graphed = True
        except RuntimeError as e:  # NCCL capture unsupported here: time it eagerly
            if mode != "nccl":
                raise
            torch.cuda.synchronize()
            ms, _ = round_ms(eng, graphed=False)
            graphed = False
        status = eng.device_status()
        try:
            proj = projections(eng, mode if world > 1 else "gemm")
        except RuntimeError as e:
            proj = {"error": str(e)[:200]}
        gemm_only = projections(eng, "gemm") if key == "fused_f32" else None
        results[key] = {"round_us": round(ms * 1e3, 1),
                        "draft_tokens_per_s": round(M / (ms * 1e-3), 1), "graphed": graphed,
                        "device_status": status, "projection_us": proj}
        if gemm_only is not None:
            results["gemm_only_projection_us"] = gemm_only
        eng.close()
        del eng
        pools.summary_bf16 = None
        torch.cuda.empty_cache()
        barrier(world)

    head = results["fused_f32"]
    # fused projection roofline: the slower of the weight stream (HBM) and the
    # NVLink bytes a rank must send (its partials of the tiles others own and
    # the results of its own tiles to every other rank; receives are symmetric)
    H = shape.hidden
    roof = {}
    for name, kdim in (("o_proj", loc.q_heads * 128), ("down_proj", loc.inter)):
        wbytes = H * kdim * 2
        link = (world - 1) / world * M * H * (4 + 2) if world > 1 else 0
        t_us = max(wbytes / (hbm_peak * 1e9), link / (nvlink_gbs * 1e9)) * 1e6
        got = head["projection_us"][name]
        roof[name] = {"target_us": round(t_us, 2), "achieved_us": got, "frac": round(t_us / got, 3),
                      "weight_bytes": wbytes, "nvlink_bytes_sent": int(link)}
    meta = {"workload": "cfg5-qwen3-14b drafter, tensor-parallel by KV-head group (BASELINE configs[4])",
            "batch": batch, "ctx": ctx, "tp": world, "hidden": shape.hidden, "q_heads": shape.q_heads,
            "kv_heads": shape.kv_heads, "inter": shape.inter, "vocab": shape.vocab,
            "window": shape.window, "slots": shape.slots, "verify_block": shape.block + 1,
            "parallelism": f"tp{world}", "l2": "inputs larger than L2 (weights and K/V of every round)",
            "nccl_nvls": os.environ.get("NCCL_NVLS_ENABLE", "default")}
    del Wl, v, pools
    torch.cuda.empty_cache()
    return results, roof, parity, meta


def run_calls(args):
    """Per-native-call device time of an eager round on one GPU: CUDA events
    around every C-ABI call, median over ``--steps`` rounds (first discarded).
    ``--calls-shape cfg5-tpN`` uses the per-rank shapes of config 5 at TP N
    (that rank's heads and intermediate slice, the full vocabulary)."""
    import torch
    from longspark_b200 import _native as N
    from longspark_b200.config import CFG2, CFG3
    from longspark_b200.tp import local_shape
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.calls_shape == "cfg2":
        shape = CFG2.shape
    elif args.calls_shape.startswith("cfg5-tp"):
        shape = local_shape(CFG3.shape, int(args.calls_shape[len("cfg5-tp"):]))
    else:
        raise SystemExit(f"unknown --calls-shape {args.calls_shape}")
    eng, g, v = build_round(shape, args.calls_ctx, args.batch, dev, seed=1000)
    orig = N.call
    records = []

    def timed(name, *a):
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        r = orig(name, *a)
        e1.record(st)
        records.append((name, e0, e1))
        return r

    N.call = timed
    per = {}
    try:
        for _ in range(max(2, min(args.steps, 20))):
            records.clear()
            g._run()
            if args.calls_prefill:
                eng.prefill_summary(slots=torch.arange(args.batch, dtype=torch.int32, device=dev),
                                    seq_lens=v["seq_lens"][:args.batch], page_table=v["page_table"], batch=args.batch)
            if args.calls_temperature > 0:
                eng.sample(g.anchors, temperature=args.calls_temperature, seed=7, batch=args.batch)
            torch.cuda.synchronize()
            for i, (name, e0, e1) in enumerate(records):
                per.setdefault((i, name), []).append(e0.elapsed_time(e1) * 1e3)
    finally:
        N.call = orig
    print(f"# {args.calls_shape}: {shape.q_heads} q / {shape.kv_heads} KV heads, H={shape.hidden}, I={shape.inter}, "
          f"V={shape.vocab}, batch {args.batch}, ctx {args.calls_ctx}; median us per call (eager, events)")
    tot = 0.0
    for (i, name), ts in sorted(per.items()):
        m = statistics.median(ts[1:])
        tot += m
        print(f"{i:2d} {name:28s} {m:9.1f}")
    print(f"sum {tot:.1f} us; device status {eng.device_status()}")


def run_reference(args):
    """The reference arm: the reference drafter's CPU path (numpy restatement,
    fp32) on the host cores, same metric/unit/config; rank 0 only.  One
    process with its BLAS pool on every core of its affinity mask at every N
    (torchrun sets OMP_NUM_THREADS=1 for its ranks; the pool is set here
    explicitly, and the line reports the threads the pool actually used)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from longspark_b200.config import CFG2
    shape = CFG2.shape
    steps = max(1, min(args.steps, 5))
    warm = min(args.warmup, 1)
    sec, threads = cpu_round_sample(shape, HEADLINE_CTX, rounds=steps, warmup=warm)
    value = shape.block / sec
    line = {"metric": METRIC, "value": round(value, 2), "unit": "draft tokens/s", "impl": "reference",
            "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": round(sec * 1e3, 1), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic",
            "config": {"workload": "cfg2-qwen3-8b drafter round (BASELINE configs[1])", "batch_per_gpu": 1,
                       "headline_ctx": HEADLINE_CTX,
                       "host": f"one process on {host_cores()} host cores at every N (rank 0 of {world})"},
            "cpu_baseline": {"value": round(value, 2), "unit": "draft tokens/s", "cores": threads, "kind": "port",
                             "sample": f"median of {steps} fp32 rounds (after {warm} warm-up) of the numpy "
                                       "restatement of the reference drafter (refresh + pass + Markov chain + "
                                       "accept) at the cfg2 shapes"},
            "cpu_baseline_cfg1": cpu_cfg1_row(),
            "e2e": {"value": round(value, 2), "unit": "draft tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.tp:
        run_tp(args)
    elif args.calls:
        run_calls(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
