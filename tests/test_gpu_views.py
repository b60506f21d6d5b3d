"""View refresh, drafter attention and greedy sampling kernels against the oracle."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import assert_bf16_close, to_np, tokens_exact_or_tied
from longspark_b200 import _native as N
from longspark_b200 import ops
from longspark_b200.config import DraftShape
from longspark_b200.synthetic import make_views

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


# --------------------------------------------------------------------------
# (a) refresh
# --------------------------------------------------------------------------

@pytest.mark.parametrize("q_heads,kv_heads,slots,max_commit,batch", [
    (32, 8, 16, 8, 3), (40, 8, 16, 8, 3), (32, 8, 256, 16, 3), (40, 8, 64, 16, 3),
    (40, 8, 256, 32, 8),  # 2560 units: several per persistent CTA, up to 32 rows
    (32, 8, 80, 5, 12),   # a 16-slot last chunk in every head
])
def test_refresh_chain_matches_oracle(q_heads, kv_heads, slots, max_commit, batch):
    """The reference's own protocol (tests/gpu/test_gqa5_attention.py:20-50):
    random bf16 queries and rows, random initial state, permuted pool slots,
    accept lengths ((arange(B) + step) % V) + 1, chained steps, tolerance 3e-5."""
    g = torch.Generator().manual_seed(980426)
    L, steps = 2, 12
    shape = DraftShape(hidden=512, q_heads=q_heads, kv_heads=kv_heads, inter=512, vocab=1024, tap_layers=L,
                       draft_layers=1, slots=slots, window=256, block=7, max_commit=max_commit, markov_rank=0,
                       mask_token_id=0)
    capacity = batch + 3
    ctx0 = [37, 300, 1000, 64, 17, 2048, 5, 999, 100, 16, 31, 700][:batch]
    v = make_views(shape, batch, ctx0, seed=5, extra_rows=steps * max_commit, gen=g)
    q = torch.randn(L, q_heads, slots, 128, generator=g).to(torch.bfloat16)
    out0 = torch.randn(capacity, L, q_heads, slots, 128, generator=g)
    lse0 = torch.randn(capacity, L, q_heads, slots, generator=g)
    slot_ids = torch.randperm(capacity, generator=g)[:batch].to(torch.int32)
    dev = "cuda"
    kv_k, kv_v, table = v["kv_k"].to(dev), v["kv_v"].to(dev), v["page_table"].to(dev)
    st_out, st_lse, qd = out0.to(dev), lse0.to(dev), q.to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ref_out, ref_lse = out0.numpy().copy(), lse0.numpy().copy()
    kk, vv = O.from_bf16_bits(v["kv_k"].view(torch.int16).numpy()), O.from_bf16_bits(v["kv_v"].view(torch.int16).numpy())
    lens = np.array(ctx0)
    for step in range(steps):
        commit = (np.arange(batch) + step) % max_commit + 1
        lens = lens + commit
        ops.refresh_views(kv_k=kv_k, kv_v=kv_v, page_table=table,
                          seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev),
                          commit_lens=torch.tensor(commit, dtype=torch.int32, device=dev),
                          slots=slot_ids.to(dev), learned_query=qd, state_out=st_out, state_lse=st_lse,
                          max_commit=max_commit, status=status)
        # oracle: the same rows gathered from the pool
        nk = np.zeros((L, batch, max_commit, kv_heads, 128), np.float32)
        nv = np.zeros_like(nk)
        for b in range(batch):
            for r in range(commit[b]):
                pos = lens[b] - commit[b] + r
                page = int(v["page_table"][b, pos // 16])
                nk[:, b, r] = kk[:, page, pos % 16]
                nv[:, b, r] = vv[:, page, pos % 16]
        ref_out, ref_lse = O.refresh_views(ref_out, ref_lse, slot_ids.numpy(), to_np(q), nk, nv, commit,
                                           128 ** -0.5)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    np.testing.assert_allclose(to_np(st_out), ref_out, rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(to_np(st_lse), ref_lse, rtol=3e-5, atol=3e-5)


def test_refresh_bad_page_leaves_request_untouched():
    """A committed row on a page id outside the pool: the status word reads
    LS_DEV_BAD_INDEX, that request's state is unchanged, the other requests
    (units before and after it in every CTA's range) match the oracle."""
    g = torch.Generator().manual_seed(7)
    L, batch, Hq, Hkv, S, V = 2, 6, 32, 8, 256, 16
    shape = DraftShape(hidden=512, q_heads=Hq, kv_heads=Hkv, inter=512, vocab=1024, tap_layers=L, draft_layers=1,
                       slots=S, window=256, block=7, max_commit=V, markov_rank=0, mask_token_id=0)
    ctx = [100, 200, 300, 400, 500, 600]
    v = make_views(shape, batch, ctx, seed=9, extra_rows=V, gen=g)
    q = torch.randn(L, Hq, S, 128, generator=g).to(torch.bfloat16)
    out0 = torch.randn(batch, L, Hq, S, 128, generator=g)
    lse0 = torch.randn(batch, L, Hq, S, generator=g)
    commit = np.full(batch, V)
    lens = np.array(ctx) + commit
    table = v["page_table"].clone()
    bad_b = 3
    table[bad_b, (lens[bad_b] - 1) // 16] = int(v["kv_k"].shape[1])  # one past the pool
    dev = "cuda"
    st_out, st_lse = out0.to(dev), lse0.to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.refresh_views(kv_k=v["kv_k"].to(dev), kv_v=v["kv_v"].to(dev), page_table=table.to(dev),
                      seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev),
                      commit_lens=torch.tensor(commit, dtype=torch.int32, device=dev),
                      slots=torch.arange(batch, dtype=torch.int32, device=dev), learned_query=q.to(dev),
                      state_out=st_out, state_lse=st_lse, max_commit=V, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 110
    kk, vv = O.from_bf16_bits(v["kv_k"].view(torch.int16).numpy()), O.from_bf16_bits(v["kv_v"].view(torch.int16).numpy())
    nk = np.zeros((L, batch, V, Hkv, 128), np.float32)
    nv = np.zeros_like(nk)
    for b in range(batch):
        for r in range(V):
            pos = lens[b] - V + r
            page = int(v["page_table"][b, pos // 16])
            nk[:, b, r] = kk[:, page, pos % 16]
            nv[:, b, r] = vv[:, page, pos % 16]
    ref_out, ref_lse = O.refresh_views(out0.numpy().copy(), lse0.numpy().copy(), np.arange(batch), to_np(q), nk, nv,
                                       commit, 128 ** -0.5)
    go, gl = to_np(st_out), to_np(st_lse)
    assert np.array_equal(go[bad_b], out0[bad_b].numpy()) and np.array_equal(gl[bad_b], lse0[bad_b].numpy())
    keep = [b for b in range(batch) if b != bad_b]
    np.testing.assert_allclose(go[keep], ref_out[keep], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(gl[keep], ref_lse[keep], rtol=3e-5, atol=3e-5)


def test_reference_api_scores_and_merge():
    """cache_position_scores + merge_accepted_positions_ with the reference's
    argument conventions (fixed [B, 8] locations, page-size-one value cache)."""
    g = torch.Generator().manual_seed(7)
    batch, hq, hkv, s, rows = 3, 40, 8, 16, 8
    dev = "cuda"
    query = torch.randn(1, hq, s, 128, generator=g).to(torch.bfloat16).to(dev).expand(batch, -1, -1, -1)
    capacity = batch + 2
    out = torch.randn(capacity, hq, s, 128, generator=g).to(dev)
    lse = torch.randn(capacity, hq, s, generator=g).to(dev)
    slots = torch.tensor([4, 0, 2], dtype=torch.int32, device=dev)
    exp_out, exp_lse = to_np(out)[[4, 0, 2]], to_np(lse)[[4, 0, 2]]
    for step in range(4):
        keys = torch.randn(batch, rows, hkv, 128, generator=g).to(torch.bfloat16).to(dev)
        values = torch.randn(batch, rows, hkv, 128, generator=g).to(torch.bfloat16).to(dev)
        sc = torch.empty(batch, hq, s, rows, device=dev)
        ops.cache_position_scores(layer_id=0, global_query=query, new_keys=keys, output=sc,
                                  softmax_scale=128 ** -0.5)
        ref_sc = O.position_scores(np.broadcast_to(to_np(query[:1]), (batch, hq, s, 128)), to_np(keys), 128 ** -0.5)
        np.testing.assert_allclose(to_np(sc), ref_sc, rtol=2e-5, atol=2e-5)
        lens = ((torch.arange(batch) + step) % rows + 1).to(torch.int32).to(dev)
        locs = torch.arange(batch * rows, device=dev).reshape(batch, rows)
        ops.merge_accepted_positions_(state_output=out, state_lse=lse, position_scores=sc,
                                      value_cache=values.reshape(batch * rows, 1, hkv, 128),
                                      accepted_cache_locs=locs, accept_lens=lens, accept_offsets=None,
                                      state_slots=slots)
        exp_out, exp_lse = O.merge_accepted(exp_out, exp_lse, ref_sc, to_np(values), lens.cpu().numpy())
    np.testing.assert_allclose(to_np(out)[[4, 0, 2]], exp_out, rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(to_np(lse)[[4, 0, 2]], exp_lse, rtol=3e-5, atol=3e-5)


@pytest.mark.parametrize("batch", [1, 3, 64])
def test_reference_protocol_gqa5_sixteen_steps(batch):
    """The reference's own refresh test protocol (tests/gpu/test_gqa5_attention.py:
    20-50): seed 980426, GQA-5 queries [1, 40, 16, 128] expanded over the
    batch, keys/values [B, 8, 8, 128], pool capacity batch + 3 with permuted
    slots, accept lengths ((arange(B) + step) % 8) + 1, 16 chained steps;
    scores within 2e-5, the merged (out, lse) within 3e-5."""
    g = torch.Generator().manual_seed(980426)
    hq, hkv, s, rows = 40, 8, 16, 8
    dev = "cuda"
    query = torch.randn(1, hq, s, 128, generator=g).to(torch.bfloat16).to(dev).expand(batch, -1, -1, -1)
    capacity = batch + 3
    out = torch.randn(capacity, hq, s, 128, generator=g).to(dev)
    lse = torch.randn(capacity, hq, s, generator=g).to(dev)
    perm = torch.randperm(capacity, generator=g)[:batch]
    slots = perm.to(torch.int32).to(dev)
    out0 = to_np(out)
    exp_out, exp_lse = out0[perm.numpy()], to_np(lse)[perm.numpy()]
    qn = np.broadcast_to(to_np(query[:1]), (batch, hq, s, 128))
    for step in range(16):
        keys = torch.randn(batch, rows, hkv, 128, generator=g).to(torch.bfloat16).to(dev)
        values = torch.randn(batch, rows, hkv, 128, generator=g).to(torch.bfloat16).to(dev)
        sc = torch.empty(batch, hq, s, rows, device=dev)
        ops.cache_position_scores(layer_id=0, global_query=query, new_keys=keys, output=sc,
                                  softmax_scale=128 ** -0.5)
        ref_sc = O.position_scores(qn, to_np(keys), 128 ** -0.5)
        np.testing.assert_allclose(to_np(sc), ref_sc, rtol=2e-5, atol=2e-5)
        lens = ((torch.arange(batch) + step) % rows + 1).to(torch.int32).to(dev)
        locs = torch.arange(batch * rows, device=dev).reshape(batch, rows)
        ops.merge_accepted_positions_(state_output=out, state_lse=lse, position_scores=sc,
                                      value_cache=values.reshape(batch * rows, 1, hkv, 128),
                                      accepted_cache_locs=locs, accept_lens=lens, accept_offsets=None,
                                      state_slots=slots)
        exp_out, exp_lse = O.merge_accepted(exp_out, exp_lse, ref_sc, to_np(values), lens.cpu().numpy())
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(out)[perm.numpy()], exp_out, rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(to_np(lse)[perm.numpy()], exp_lse, rtol=3e-5, atol=3e-5)
    others = np.setdiff1d(np.arange(capacity), perm.numpy())
    np.testing.assert_array_equal(to_np(out)[others], out0[others])  # pool entries of no request: untouched


# --------------------------------------------------------------------------
# (b) attention
# --------------------------------------------------------------------------

@pytest.mark.parametrize("q_heads,kv_heads,slots,window,block,contexts", [
    (8, 2, 16, 256, 7, (300, 100)),
    (32, 8, 64, 512, 15, (4096,)),
    (40, 8, 256, 2048, 15, (5000, 1999)),
    (32, 8, 256, 1024, 15, (1024, 17, 3000)),
    # many requests: two CTAs per SM, 64-row window sub-chunks, one warp per head
    (32, 8, 256, 1024, 15, tuple(900 + 37 * i for i in range(40))),
    (40, 8, 256, 2048, 15, tuple(2100 + 301 * i for i in range(12))),
    (8, 2, 16, 256, 7, tuple(5 + 23 * i for i in range(30))),
    # streaming instantiation (>= 64 request x KV-head units): short windows
    # (a partial 64-row stage, an empty one), a 16-slot summary
    (32, 8, 64, 512, 15, (0, 3, 64, 65, 511, 512, 513, 4000, 77)),
    (40, 8, 256, 2048, 15, tuple(1 + 555 * i for i in range(9))),
    (8, 2, 16, 256, 7, tuple(5 + 23 * i for i in range(33))),
])
def test_attention_matches_oracle(q_heads, kv_heads, slots, window, block, contexts):
    """Both instantiations against the oracle: the cluster kernel below 64
    (request, KV head) units, the streaming kernel from 64 on (the engine's
    bf16 summary copy is passed, as the engine does)."""
    _attention_case(q_heads, kv_heads, slots, window, block, contexts)


def _attention_case(q_heads, kv_heads, slots, window, block, contexts):
    g = torch.Generator().manual_seed(11)
    batch = len(contexts)
    shape = DraftShape(hidden=512, q_heads=q_heads, kv_heads=kv_heads, inter=512, vocab=1024, tap_layers=1,
                       draft_layers=1, slots=slots, window=window, block=block, max_commit=block + 1,
                       markov_rank=0, mask_token_id=0)
    v = make_views(shape, batch, list(contexts), seed=3, gen=g)
    qkv = torch.randn(batch * block, (q_heads + 2 * kv_heads) * 128, generator=g).to(torch.bfloat16)
    qg = (0.3 * torch.randn(q_heads, slots, 128, generator=g)).to(torch.bfloat16)
    dev = "cuda"
    out = torch.empty(batch * block, q_heads * 128, dtype=torch.bfloat16, device=dev)
    ws = torch.zeros(ops.attention_workspace_bytes(batch, q_heads, kv_heads, window, slots), dtype=torch.uint8,
                     device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    slots_t = torch.arange(batch, dtype=torch.int32, device=dev)
    state = v["summary_out"][:, 0].to(dev)
    ops.draft_attention(qkv=qkv.to(dev), block=block, kv_k=v["kv_k"][0].to(dev), kv_v=v["kv_v"][0].to(dev),
                        page_table=v["page_table"].to(dev), seq_lens=v["seq_lens"].to(dev), window=window,
                        learned_query=qg.to(dev), state_out=state, slots=slots_t, out=out,
                        workspace=ws, q_heads=q_heads, kv_heads=kv_heads, status=status,
                        state_bf16=state.to(torch.bfloat16).contiguous())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    x = to_np(qkv).reshape(batch, block, -1, 128)
    q = x[:, :, :q_heads].transpose(0, 2, 1, 3)
    k = x[:, :, q_heads:q_heads + kv_heads].transpose(0, 2, 1, 3)
    vl = x[:, :, q_heads + kv_heads:].transpose(0, 2, 1, 3)
    views = O.build_views(to_np(v["kv_k"]), to_np(v["kv_v"]), v["page_table"].numpy(), v["seq_lens"].numpy(),
                          v["summary_out"].numpy(), to_np(qg)[None], window, 1)
    w0 = views[0]
    ref = O.attend(q, k, vl, w0["qg"], w0["summary_out"], w0["win_k"], w0["win_v"], w0["win_len"], "bf16")
    ref = ref.transpose(0, 2, 1, 3).reshape(batch * block, q_heads * 128)
    assert_bf16_close(to_np(out), ref, steps=2.0, exact_frac=0.5, what="attention")


def test_attention_stream_kernel_at_every_batch_size():
    """The streaming instantiation forced for every case of the test above
    (LONGSPARK_B200_ATTN=stream, read once per process: a child process)."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    here = Path(__file__).resolve().parent
    env = dict(os.environ, LONGSPARK_B200_ATTN="stream")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        f"{here / 'test_gpu_views.py'}::test_attention_matches_oracle"],
                       env=env, cwd=str(here.parent), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


# --------------------------------------------------------------------------
# greedy chain + accept
# --------------------------------------------------------------------------

@pytest.mark.parametrize("rank,wstd", [(0, 0.02), (64, 0.02), (256, 0.02), (64, 0.3)])
def test_markov_chain_matches_oracle(rank, wstd):
    """wstd 0.3 makes the bias bound cover most of the vocabulary, so the
    candidate lists overflow and the exact step-by-step path runs."""
    g = torch.Generator().manual_seed(21 + rank)
    batch, block, vocab = 3, 15, 151936
    dev = "cuda"
    base = (1.3 * torch.randn(batch * block, vocab, generator=g)).to(torch.bfloat16)
    # plant exact ties and near-ties in a few rows
    base[0, 77] = base[0].max()
    base[1, 5] = base[1].max()
    base[1, 90000] = base[1].max()
    bl = base.to(dev)
    tmax = torch.empty(batch * block, vocab // 128, device=dev)
    targ = torch.empty(batch * block, vocab // 128, dtype=torch.int32, device=dev)
    lv = to_np(bl).reshape(batch * block, vocab // 128, 128)
    tmax.copy_(torch.from_numpy(lv.max(-1)))
    targ.copy_(torch.from_numpy((lv.argmax(-1) + np.arange(vocab // 128)[None] * 128).astype(np.int32)))
    anchors = torch.randint(0, vocab, (batch,), generator=g)
    W = {}
    w1 = w2 = b1 = b2 = None
    if rank:
        w1 = (wstd * torch.randn(vocab, rank, generator=g)).to(torch.bfloat16).to(dev)
        w2 = (wstd * torch.randn(vocab, rank, generator=g)).to(torch.bfloat16).to(dev)
        b1, b2 = torch.zeros(1, device=dev), torch.zeros(1, device=dev)
        ops.row_norm_bound(w1, b1)
        ops.row_norm_bound(w2, b2)
        W = {"parallel_markov_head.markov_w1.weight": to_np(w1), "parallel_markov_head.markov_w2.weight": to_np(w2)}
    tokens = torch.empty(batch, block, dtype=torch.int64, device=dev)
    target = torch.randint(0, vocab, (batch, block + 1), generator=g)
    acc = torch.empty(batch, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(ops.markov_workspace_bytes(batch, block), dtype=torch.uint8, device=dev)
    ops.markov_argmax(base=bl, tile_max=tmax, tile_arg=targ, anchors=anchors.to(dev), tokens=tokens, block=block,
                      workspace=ws, w1=w1, w2=w2, w1_bound=b1, w2_bound=b2, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    gt = tokens.cpu().numpy()
    # oracle, teacher-forced on the GPU's own chain so a flipped near-tie does not cascade
    toks, corrected = O.markov_sample(to_np(bl).reshape(batch, block, vocab), anchors.numpy(), W, "bf16", forced=gt)
    ties = tokens_exact_or_tied(gt, corrected, what=f"markov rank {rank}")
    assert ties <= 2
    # accept check against a target that agrees on a known prefix
    k = torch.tensor([0, 4, block])
    tgt = torch.where(torch.arange(block + 1)[None] < k[:, None], torch.cat([tokens.cpu(), tokens.cpu()[:, -1:]], 1),
                      (torch.cat([tokens.cpu(), tokens.cpu()[:, -1:]], 1) + 1) % vocab)
    ops.accept_lengths(tgt.to(dev), tokens, acc)
    assert acc.cpu().tolist() == k.tolist()
    np.testing.assert_array_equal(O.accept_lengths(tgt.numpy(), gt)[0], k.numpy())
