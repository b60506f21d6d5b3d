"""Per-rank bodies of the tensor-parallel GPU tests (one process per GPU,
started with torch.multiprocessing.spawn by test_gpu_tp.py).  Rank 0 checks
against the oracle; every rank checks that all ranks hold the same result.
A failing check raises, which ends the spawn with the traceback."""

import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

import oracle as O
from gpu_util import assert_bf16_close, to_np, tokens_exact_or_tied
from longspark_b200 import _native as N
from longspark_b200 import ops
from longspark_b200.config import DraftShape
from longspark_b200.engine import DraftEngine, DraftWeights, GraphedDraft, ViewPools
from longspark_b200.synthetic import make_views, make_weights, rope_inv_freq
from longspark_b200.tp import (SymmetricHeap, TPDraftEngine, TPGroup, dist_helpers, shard_state_dict, shard_views,
                               vocab_shards)

# splits over 2, 4 and 8 ranks (8 KV heads, 1024 = 8 x 128 hidden, 256 vocabulary tiles)
TP_SMALL = DraftShape(hidden=1024, q_heads=16, kv_heads=8, inter=2048, vocab=32768, tap_layers=2, draft_layers=1,
                      slots=64, window=512, block=15, max_commit=16, markov_rank=64, mask_token_id=32000)


def init(rank, world, port):
    # NCCL without NVLink SHARP: a rank that exits on a failed check must not
    # leave memory bound to a multicast object behind on the other GPUs
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    return torch.device("cuda", rank)


def finish(objs=()):
    torch.cuda.synchronize()
    dist.barrier()
    for o in objs:
        o.close() if hasattr(o, "close") else None
    dist.destroy_process_group()


def same_on_all_ranks(t, what):
    """Every rank's tensor equals rank 0's, bit for bit."""
    x = t.contiguous()
    got = [torch.empty_like(x) for _ in range(dist.get_world_size())]
    dist.all_gather(got, x)
    for r, y in enumerate(got):
        assert torch.equal(y.view(torch.uint8) if y.dtype == torch.bfloat16 else y,
                           x.view(torch.uint8) if x.dtype == torch.bfloat16 else x), f"{what}: rank {r} differs"


# ----------------------------------------------------------------------------
# ls_gemm_allreduce against the oracle's row-parallel linear
# ----------------------------------------------------------------------------

GEMM_CASES = [  # rows, k (total), n_out, epilogue, wire
    (16, 1024, 512, "store", "f32"),
    (37, 1536, 640, "residual", "f32"),
    (37, 1536, 640, "residual", "bf16"),
    (480, 2048, 1024, "residual", "f32"),
    (480, 1024, 2048, "store", "bf16"),
    (3, 1024, 256, "store", "f32"),
]


def gemm_worker(rank, world, port):
    dev = init(rank, world, port)
    all_gather, barrier = dist_helpers()
    sync = max(N.lib().ls_tp_sync_bytes(world, r, n, 0) for r, _, n, _, _ in GEMM_CASES)
    heap = SymmetricHeap(sync + (64 << 20), rank=rank, world=world, device=dev, all_gather=all_gather)
    group = TPGroup(heap, sync, barrier=barrier)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for ci, (rows, k, n, epi, wire) in enumerate(GEMM_CASES):
        g = torch.Generator().manual_seed(100 + ci)
        x = (torch.randn(rows, k, generator=g) * 0.5).to(torch.bfloat16)
        w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
        res = torch.randn(rows, n, generator=g).to(torch.bfloat16)
        ks = k // world
        xr = x[:, rank * ks:(rank + 1) * ks].contiguous().to(dev)
        wr = ops.TiledWeight(w[:, rank * ks:(rank + 1) * ks].contiguous().to(dev))
        saved = heap.used
        out = heap.carve((rows, n), torch.bfloat16)
        out.copy_(res.to(dev) if epi == "residual" else torch.zeros(rows, n, dtype=torch.bfloat16))
        ws = torch.zeros(max(1, ops.gemm_workspace_bytes(rows, ks, n)), dtype=torch.uint8, device=dev)
        wire_c = N.TP_WIRE_BF16 if wire == "bf16" else N.TP_WIRE_F32
        reps = 3
        for _ in range(reps):  # in place: out <- out + sum (residual) or out <- sum (store)
            ops.gemm_allreduce(xr, wr, out, group=group, workspace=ws, wire=wire_c,
                               epilogue=N.EPI_RESIDUAL if epi == "residual" else N.EPI_STORE,
                               residual=out if epi == "residual" else None, rows=rows, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"case {ci}: device status {int(status.item())}"
        same_on_all_ranks(out, f"case {ci} output")
        if rank == 0:
            ref = O.row_parallel_linear(x.float().numpy(), w.float().numpy(), "bf16", (world, wire))
            cur = res.float().numpy() if epi == "residual" else None
            for _ in range(reps):
                cur = ref if cur is None or epi == "store" else O.bf16_round(cur + ref)
            # fp32 accumulation order inside each rank's partial is the only difference
            assert_bf16_close(to_np(out), cur, steps=1.0 * reps, exact_frac=0.97, what=f"case {ci} {epi} {wire}")
        heap.used = saved
    # the same launch replayed from a CUDA graph: flags and slots are reused
    rows, k, n = 64, 2048, 1024
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(rows, k, generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    ks = k // world
    xr = x[:, rank * ks:(rank + 1) * ks].contiguous().to(dev)
    wr = ops.TiledWeight(w[:, rank * ks:(rank + 1) * ks].contiguous().to(dev))
    out = heap.carve((rows, n), torch.bfloat16)
    ws = torch.zeros(max(1, ops.gemm_workspace_bytes(rows, ks, n)), dtype=torch.uint8, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.gemm_allreduce(xr, wr, out, group=group, workspace=ws, rows=rows, status=status)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        ops.gemm_allreduce(xr, wr, out, group=group, workspace=ws, rows=rows, status=status)
    for i in range(20):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(out.view(torch.uint8), eager.view(torch.uint8)), f"graph replay {i} differs from eager"
    same_on_all_ranks(out, "graph replay output")
    del graph
    finish([group.heap])


# ----------------------------------------------------------------------------
# vocabulary-sharded Markov chain against the one-GPU kernel
# ----------------------------------------------------------------------------

def markov_worker(rank, world, port):
    dev = init(rank, world, port)
    all_gather, barrier = dist_helpers()
    B, P, V, R = 6, 15, 32768, 64
    M = B * P
    T, shards = vocab_shards(V, world)
    heap = SymmetricHeap(256 + M * T * 128 * 2 + 2 * M * T * 4 + (4 << 20), rank=rank, world=world, device=dev,
                         all_gather=all_gather)
    group = TPGroup(heap, 4096 * 64, barrier=barrier)
    v0, nv = shards[rank]
    nt = nv // 128
    logits_sh = heap.carve((M, T * 128), torch.bfloat16).view(-1)[:M * nv].view(M, nv)
    tmax_sh = heap.carve((M, T), torch.float32).view(-1)[:M * nt].view(M, nt)
    targ_sh = heap.carve((M, T), torch.int32).view(-1)[:M * nt].view(M, nt)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(ops.markov_workspace_bytes(B, P), dtype=torch.uint8, device=dev)
    ws1 = torch.zeros_like(ws)
    for case in ("markov", "argmax", "ties", "flat"):
        g = torch.Generator().manual_seed({"markov": 1, "argmax": 2, "ties": 3, "flat": 4}[case])
        full = torch.randn(M, V, generator=g) * 2.0
        if case == "ties":
            full = torch.round(full * 2.0) / 2.0  # many exact ties, across shards too
        if case == "flat":
            full = torch.zeros(M, V)  # every token in the band: the step-by-step fallback
        full = full.to(torch.bfloat16).to(dev)
        tiles = full.view(M, V // 128, 128).float()
        tmax = tiles.max(-1).values.contiguous()
        targ = (tiles.argmax(-1).int() + torch.arange(V // 128, device=dev, dtype=torch.int32) * 128).contiguous()
        logits_sh.copy_(full[:, v0:v0 + nv])
        tmax_sh.copy_(tmax[:, v0 // 128:v0 // 128 + nt])
        targ_sh.copy_(targ[:, v0 // 128:v0 // 128 + nt] - v0)  # shard-local ids, as the LM-head epilogue writes
        w1 = w2 = b1 = b2 = None
        if case != "argmax":
            w1 = (torch.randn(V, R, generator=g) * 0.3).to(torch.bfloat16).to(dev)
            w2 = (torch.randn(V, R, generator=g) * 0.3).to(torch.bfloat16).to(dev)
            b1 = torch.zeros(1, device=dev)
            b2 = torch.zeros(1, device=dev)
            ops.row_norm_bound(w1, b1)
            ops.row_norm_bound(w2, b2)
        anchors = torch.randint(0, V, (B,), generator=g).to(dev)
        tok_tp = torch.zeros(B, P, dtype=torch.int64, device=dev)
        tok_1 = torch.zeros(B, P, dtype=torch.int64, device=dev)
        ops.tp_barrier(group, slot=1, status=status)
        ops.markov_argmax(base=logits_sh, tile_max=tmax_sh, tile_arg=targ_sh, anchors=anchors, tokens=tok_tp,
                          block=P, workspace=ws, w1=w1, w2=w2, w1_bound=b1, w2_bound=b2, status=status,
                          group=group, tiles_per_shard=T, vocab=V)
        ops.markov_argmax(base=full, tile_max=tmax, tile_arg=targ, anchors=anchors, tokens=tok_1, block=P,
                          workspace=ws1, w1=w1, w2=w2, w1_bound=b1, w2_bound=b2, status=status)
        # nobody overwrites a shard before every rank has read it
        ops.tp_barrier(group, slot=1, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"{case}: device status {int(status.item())}"
        assert torch.equal(tok_tp, tok_1), f"{case}: sharded tokens differ from the one-GPU kernel"
        same_on_all_ranks(tok_tp, f"{case} tokens")
    finish([group.heap])


# ----------------------------------------------------------------------------
# tensor-parallel drafting round against the oracle
# ----------------------------------------------------------------------------

def _oracle_logits(shape, Wn, v, prec, tp):
    views = O.build_views(to_np(v["kv_k"]), to_np(v["kv_v"]), v["page_table"].numpy(), v["seq_lens"].numpy(),
                          v["summary_out"].numpy(), Wn["global16_raw256_reference.global_query_generator.learned_query"],
                          shape.window, shape.draft_layers, prec=prec)
    osh = O.DraftShapeOracle(shape.hidden, shape.q_heads, shape.kv_heads, 128, shape.block, shape.mask_token_id,
                             shape.rms_eps, shape.final_eps)
    base, _ = O.draft_pass(Wn, osh, v["anchors"].numpy(), v["seq_lens"].numpy().astype(np.int64),
                           to_np(v["hidden"]), views, rope_inv_freq(shape).numpy(), prec, tp=tp)
    return base


def engine_worker(rank, world, port, allreduce, wire):
    dev = init(rank, world, port)
    all_gather, barrier = dist_helpers()
    shape = TP_SMALL
    batch = 3
    W = make_weights(shape, seed=21, norm_jitter=0.05)
    v = make_views(shape, batch, [900, 40, 2500], seed=22)
    Wl = shard_state_dict(W, shape, rank, world)
    vl = shard_views(v, shape, rank, world)
    pools = ViewPools(kv_k=vl["kv_k"].to(dev), kv_v=vl["kv_v"].to(dev), page_table=vl["page_table"].to(dev),
                      summary_out=vl["summary_out"].to(dev), summary_lse=vl["summary_lse"].to(dev),
                      hidden=vl["hidden"].to(dev))
    wire_c = N.TP_WIRE_BF16 if wire == "bf16" else N.TP_WIRE_F32
    eng = TPDraftEngine(shape, Wl, pools, batch, rank=rank, world=world, device=dev, all_gather=all_gather,
                        barrier=barrier, allreduce=allreduce, wire=wire_c, pg=dist.group.WORLD)
    slots = torch.arange(batch, dtype=torch.int32, device=dev)
    args = dict(slots=slots, seq_lens=v["seq_lens"].to(dev), anchors=v["anchors"].to(dev),
                page_table=v["page_table"].to(dev))
    eng.draft(**args)
    torch.cuda.synchronize()
    assert eng.device_status() == 0, f"device status {eng.device_status()}"
    M = batch * shape.block
    tokens = eng.buf["tokens"][:batch].clone()
    same_on_all_ranks(tokens, "draft tokens")
    shard = to_np(eng.buf["logits"][:M])
    shards = [None] * world
    dist.all_gather_object(shards, shard)
    if allreduce == "fused":
        # the same pass replayed from a CUDA graph, 10 times: same tokens, status 0
        gd = GraphedDraft(eng, batch, with_refresh=False, with_target=False, slots_are_rows=False)
        gd.load(**args)
        gd.capture()
        for i in range(10):
            eng.buf["tokens"].zero_()
            gd.replay()
            torch.cuda.synchronize()
            assert eng.device_status() == 0
            assert torch.equal(eng.buf["tokens"][:batch], tokens), f"graph replay {i} tokens differ"
        del gd
    if rank == 0:
        gl = np.concatenate(shards, axis=1).reshape(batch, shape.block, shape.vocab)
        Wn = {k: t.float().numpy() for k, t in W.items()}
        ref16 = _oracle_logits(shape, Wn, v, "bf16", (world, wire if allreduce == "fused" else "bf16"))
        # NCCL sums bf16 partials with its own rounding order, hence the wider band
        assert_bf16_close(gl, ref16, steps=4.0 if allreduce == "fused" else 8.0,
                          exact_frac=0.3 if allreduce == "fused" else 0.15, what=f"TP {allreduce}/{wire} logits")
        _, corrected = O.markov_sample(ref16, v["anchors"].numpy(), Wn, "bf16", forced=tokens.cpu().numpy())
        ties = tokens_exact_or_tied(tokens.cpu().numpy(), corrected, what=f"TP {allreduce}/{wire} tokens")
        assert ties <= 3
    finish([eng])


# ----------------------------------------------------------------------------
# Target-side export: every rank stores its KV-head slice into rank 0's pool
# ----------------------------------------------------------------------------

def export_worker(rank, world, port):
    """Each rank plays one target TP rank holding heads [r*h, (r+1)*h) of the
    target pool and exports them with ls_export_rows into the drafter pool on
    rank 0 (a symmetric-heap buffer, reached from the other ranks through its
    IPC mapping); rank 0 then holds the full-head rows (oracle gather + store)."""
    from longspark_b200.export import ExportDestination, export_rows

    dev = init(rank, world, port)
    g = torch.Generator().manual_seed(77)
    L, H, R, B = 2, 8, 3000, 3
    counts = [5, 16, 1]
    lens = torch.tensor([500, 37, 1200], dtype=torch.int32)
    stride = (int(lens.max()) + 15) // 16
    pages = B * stride + 4
    src_k = torch.randn(L, R, H, 128, generator=g).to(torch.bfloat16)
    src_v = torch.randn(L, R, H, 128, generator=g).to(torch.bfloat16)
    loc = torch.randperm(R, generator=g)[:sum(counts)]
    table = torch.randperm(pages, generator=g)[:B * stride].view(B, stride).to(torch.int32)
    ag, _ = dist_helpers()
    pool_bytes = L * pages * 16 * H * 128 * 2
    heap = SymmetricHeap(2 * pool_bytes, rank=rank, world=world, device=dev, all_gather=ag)
    pk = heap.carve((L, pages, 16, H, 128), torch.bfloat16)
    pv = heap.carve((L, pages, 16, H, 128), torch.bfloat16)
    pk.fill_(-2.0)
    pv.fill_(-2.0)
    torch.cuda.synchronize()
    dist.barrier()
    dest = ExportDestination(kv_k=heap.peers[0] + heap.offset_of(pk), kv_v=heap.peers[0] + heap.offset_of(pv),
                             pool_pages=pages, heads=H, tap_layers=L, ring_pages=0, page_table=table.to(dev),
                             seq_lens=lens.to(dev), slots=torch.zeros(B, dtype=torch.int32, device=dev))
    h = H // world
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    export_rows(dest, src_k=[src_k[l, :, rank * h:(rank + 1) * h].contiguous().to(dev) for l in range(L)],
                src_v=[src_v[l, :, rank * h:(rank + 1) * h].contiguous().to(dev) for l in range(L)],
                locations=loc, counts=counts, head_offset=rank * h, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"rank {rank}: status {int(status.item())}"
    dist.barrier()  # every rank's stores have completed
    if rank == 0:
        fill = torch.full((L, pages, 16, H, 128), -2.0).to(torch.bfloat16)
        bits = lambda t: t.cpu().view(torch.int16).numpy().copy()  # noqa: E731  (fresh arrays: the oracle writes)
        ref_k, ref_v = O.export_rows(bits(fill), bits(fill), bits(src_k), bits(src_v), loc.numpy(), counts,
                                     lens.numpy(), table.numpy())
        np.testing.assert_array_equal(bits(pk), ref_k)
        np.testing.assert_array_equal(bits(pv), ref_v)
    finish([heap])
