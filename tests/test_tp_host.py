"""Host logic of the tensor-parallel drafter, on the CPU: the shape checks and
shard plans, the oracle's row-parallel linear, and a world-size-2 gloo run in
which each rank projects with its own shard of the weights and the ranks sum
their partials in rank order, reproducing the oracle's row-parallel result
bit for bit (the data flow ls_gemm_allreduce implements on the GPU)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from longspark_b200.config import CFG3, DraftShape
from longspark_b200.synthetic import make_views, make_weights
from longspark_b200.tp import check_tp_shape, local_shape, shard_state_dict, shard_views, vocab_shards

SMALL = DraftShape(hidden=512, q_heads=8, kv_heads=4, inter=1024, vocab=4096 + 128, tap_layers=2, draft_layers=1,
                   slots=64, window=512, block=15, max_commit=16, markov_rank=64, mask_token_id=4000)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_vocab_shards_cover_qwen_vocab(world):
    T, shards = vocab_shards(151936, world)
    assert shards[0][0] == 0
    for (a, n), (b, _) in zip(shards, shards[1:]):
        assert a + n == b and n == T * 128
    assert shards[-1][0] + shards[-1][1] == 151936
    assert all(n > 0 and n % 128 == 0 for _, n in shards)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config5_shape_splits(world):
    """the 14B drafter over TP 2/4/8 by KV-head group."""
    shape = CFG3.shape
    check_tp_shape(shape, world)
    loc = local_shape(shape, world)
    assert loc.kv_heads * world == 8 and loc.q_heads * world == 40 and loc.group == 5
    assert loc.inter * world == shape.inter and loc.hidden == shape.hidden


def test_bad_splits_raise():
    with pytest.raises(ValueError):
        check_tp_shape(CFG3.shape, 3)
    with pytest.raises(ValueError):
        check_tp_shape(CFG3.shape.with_(kv_heads=4, q_heads=20), 8)
    with pytest.raises(ValueError):
        check_tp_shape(CFG3.shape, 16)


def test_shards_reassemble_full_weights():
    W = make_weights(SMALL, seed=2)
    world = 2
    parts = [shard_state_dict(W, SMALL, r, world) for r in range(world)]
    for k, full in W.items():
        got = [p[k] for p in parts]
        if all(g.shape == full.shape for g in got):
            assert all(torch.equal(g, full) for g in got), k  # replicated
            continue
        if k.endswith("learned_query"):
            cat = torch.cat(got, dim=1)
        elif full.ndim == 2 and got[0].shape[1] != full.shape[1]:
            cat = torch.cat(got, dim=1)
        else:
            cat = torch.cat(got, dim=0)
        assert torch.equal(cat, full), k
    # q/k/v rows of rank r are its heads: the k_proj rows of rank 1 start at KV head 2
    D = SMALL.head_dim
    assert torch.equal(parts[1]["parallel_qwen_layers.0.self_attn.k_proj.weight"],
                       W["parallel_qwen_layers.0.self_attn.k_proj.weight"][2 * D:4 * D])


def test_shard_views_take_rank_heads():
    v = make_views(SMALL, 2, [100, 300], seed=3)
    s = shard_views(v, SMALL, 1, 2)
    assert torch.equal(s["kv_k"], v["kv_k"][:, :, :, 2:4])
    assert torch.equal(s["summary_out"], v["summary_out"][:, :, 4:8])
    assert torch.equal(s["page_table"], v["page_table"])


def test_row_parallel_linear_oracle():
    rng = np.random.default_rng(0)
    x = O.bf16_round(rng.standard_normal((7, 256)).astype(np.float32))
    w = O.bf16_round(rng.standard_normal((128, 256)).astype(np.float32) * 0.05)
    assert np.array_equal(O.row_parallel_linear(x, w, "bf16", (1, "f32")), O.linear(x, w, "bf16"))
    y2 = O.row_parallel_linear(x, w, "fp32", (2, "f32"))
    np.testing.assert_allclose(y2, O.linear(x, w, "fp32"), rtol=1e-5, atol=1e-5)
    p0 = O.bf16_round(x[:, :128] @ w[:, :128].T)
    p1 = O.bf16_round(x[:, 128:] @ w[:, 128:].T)
    assert np.array_equal(O.row_parallel_linear(x, w, "fp32", (2, "bf16")), (p0 + p1).astype(np.float32))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_projections(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W = make_weights(SMALL, seed=4)
        Wl = {k: t.float().numpy() for k, t in shard_state_dict(W, SMALL, rank, world).items()}
        Wf = {k: t.float().numpy() for k, t in W.items()}
        rng = np.random.default_rng(5)
        H, D, I = SMALL.hidden, SMALL.head_dim, SMALL.inter
        x_attn = O.bf16_round(rng.standard_normal((9, SMALL.q_heads * D)).astype(np.float32))
        x_act = O.bf16_round(rng.standard_normal((9, I)).astype(np.float32))
        x_h = O.bf16_round(rng.standard_normal((9, H)).astype(np.float32))
        hq = SMALL.q_heads // world
        Is = I // world
        Hs = H // world
        cases = {
            "o_proj": (x_attn[:, rank * hq * D:(rank + 1) * hq * D], "parallel_qwen_layers.0.self_attn.o_proj.weight"),
            "down": (x_act[:, rank * Is:(rank + 1) * Is], "parallel_qwen_layers.0.mlp.down_proj.weight"),
            "enc2": (x_h[:, rank * Hs:(rank + 1) * Hs], "draft_state_encoder.proj.net.2.weight"),
        }
        full_x = {"o_proj": x_attn, "down": x_act, "enc2": x_h}
        res = {}
        for name, (xs, key) in cases.items():
            for wire in ("f32", "bf16"):
                part = np.matmul(xs, Wl[key].T, dtype=np.float32)
                if wire == "bf16":
                    part = O.bf16_round(part)
                parts = [None] * world
                dist.all_gather_object(parts, part)
                acc = parts[0]
                for p in parts[1:]:
                    acc = (acc + p).astype(np.float32)
                got = O.bf16_round(acc)
                ref = O.row_parallel_linear(full_x[name], Wf[key], "bf16", (world, wire))
                res[f"{name}/{wire}"] = bool(np.array_equal(got, ref))
        # vocabulary-parallel LM head: every rank's logits are its slice of the full projection
        lm = np.matmul(x_h, Wl["lm_head.weight"].T, dtype=np.float32)
        _, shards = vocab_shards(SMALL.vocab, world)
        v0, n = shards[rank]
        res["lm_head"] = bool(np.allclose(lm, np.matmul(x_h, Wf["lm_head.weight"][v0:v0 + n].T), atol=0, rtol=0))
        out[rank] = res
    finally:
        dist.destroy_process_group()


def test_two_rank_row_parallel_projections_gloo():
    world = 2
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_rank_projections, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        assert all(res[r].values()), res[r]


def test_tp_entry_points_validate_without_gpu():
    """Argument errors come back as status codes before any CUDA call."""
    import ctypes as C

    from longspark_b200 import _native as N
    lib = N.lib()
    assert lib.ls_tp_sync_bytes(2, 480, 5120, N.TP_WIRE_F32) > lib.ls_tp_sync_bytes(2, 480, 5120, N.TP_WIRE_BF16)
    assert lib.ls_tp_sync_bytes(0, 480, 5120, 0) == 0
    assert lib.ls_tp_sync_bytes(9, 480, 5120, 0) == 0
    assert lib.ls_tp_sync_bytes(2, 480, 5000, 0) == 0  # n_out not a multiple of 128
    assert lib.ls_tp_sync_bytes(2, 480, 5120, 7) == 0  # unknown wire format
    # exchange slots: ceil(tiles / world) * world slots of one token tile each,
    # for the widest need over every token tile a plan can pick (multiples of 16
    # up to 256 for 480 rows)
    need = max(-(-(40 * -(-480 // bn)) // 8) * 8 * bn * 128 for bn in range(16, 257, 16))
    assert lib.ls_tp_sync_bytes(8, 480, 5120, 0) - lib.ls_tp_sync_bytes(8, 480, 5120, 1) == need * 2
    g = N.TpGroup(world=0, rank=0, heap=(C.c_void_p * 8)(), heap_bytes=1 << 20, sync_offset=0)
    a = N.GemmArgs()
    assert lib.ls_gemm_allreduce(None, C.byref(a), C.byref(g), 0, None, 0) == 1
    assert b"world" in lib.ls_last_error()
    heaps = (C.c_void_p * 8)(0x100000, 0x200000)
    g = N.TpGroup(world=2, rank=1, heap=heaps, heap_bytes=1 << 20, sync_offset=0)
    a.epilogue = N.EPI_QKV
    assert lib.ls_gemm_allreduce(None, C.byref(a), C.byref(g), 0, None, 0) == 3  # unsupported epilogue
    assert lib.ls_tp_barrier(None, C.byref(g), 16, None) == 1  # slot out of range
    m = N.MarkovArgs(base=0x100100, tile_max=0x100200, tile_arg=0x100300, vocab=4096, batch=1, block=1)
    assert lib.ls_markov_argmax_tp(None, C.byref(m), C.byref(g), 8, None, 0) == 1  # 16 tiles cannot cover 32
    g.sync_offset = 100  # not 256-byte aligned
    assert lib.ls_tp_barrier(None, C.byref(g), 0, None) == 1
