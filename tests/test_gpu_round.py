"""Whole drafting round (state encoder -> shifted input -> decoder layers ->
vocabulary projection -> Markov greedy chain -> accept check) against the
oracle, plus CUDA-graph replay and the drop-in ``LongSparkDraft`` API."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import assert_bf16_close, bf16_step, to_np, tokens_exact_or_tied
from longspark_b200.config import DraftShape
from longspark_b200.draft import LongSparkDraft
from longspark_b200.engine import DraftEngine, DraftWeights, GraphedDraft, ViewPools
from longspark_b200.synthetic import make_views, make_weights, rope_inv_freq

pytestmark = pytest.mark.gpu

# the unmodified reference's bf16-vs-fp32 distance on the config-1 logits (max
# over all 151,936 logits of the drafter pass, measured with the reference)
CFG1_REFERENCE_DRIFT = 0.042

SMALL = DraftShape(hidden=512, q_heads=8, kv_heads=2, inter=1024, vocab=4096, tap_layers=2, draft_layers=2,
                   slots=64, window=512, block=15, max_commit=16, markov_rank=64, mask_token_id=4000)


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _np_weights(W):
    return {k: v.float().numpy() for k, v in W.items()}


def _oracle_pass(shape, Wn, v, prec):
    views = O.build_views(to_np(v["kv_k"]), to_np(v["kv_v"]), v["page_table"].numpy(), v["seq_lens"].numpy(),
                          v["summary_out"].numpy(), Wn["global16_raw256_reference.global_query_generator.learned_query"],
                          shape.window, shape.draft_layers, prec=prec)
    osh = O.DraftShapeOracle(shape.hidden, shape.q_heads, shape.kv_heads, 128, shape.block, shape.mask_token_id,
                             shape.rms_eps, shape.final_eps)
    base, _ = O.draft_pass(Wn, osh, v["anchors"].numpy(), v["seq_lens"].numpy().astype(np.int64),
                           to_np(v["hidden"]), views, rope_inv_freq(shape).numpy(), prec)
    return base


def _engine(shape, W, v, batch):
    dev = torch.device("cuda")
    w = DraftWeights(shape, W, dev)
    pools = ViewPools(kv_k=v["kv_k"].to(dev), kv_v=v["kv_v"].to(dev), page_table=v["page_table"].to(dev),
                      summary_out=v["summary_out"].to(dev), summary_lse=v["summary_lse"].to(dev),
                      hidden=v["hidden"].to(dev))
    return DraftEngine(shape, w, pools, max_batch=batch, device=dev)


def _run_and_compare(shape, contexts, seed, *, fp32_tol=None):
    batch = len(contexts)
    W = make_weights(shape, seed=seed, norm_jitter=0.05)
    v = make_views(shape, batch, list(contexts), seed=seed + 1)
    eng = _engine(shape, W, v, batch)
    dev = eng.device
    slots = torch.arange(batch, dtype=torch.int32, device=dev)
    eng.draft(slots=slots, seq_lens=v["seq_lens"].to(dev), anchors=v["anchors"].to(dev),
              page_table=v["page_table"].to(dev))
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    M = batch * shape.block
    gpu_logits = to_np(eng.buf["logits"][:M]).reshape(batch, shape.block, shape.vocab)
    gpu_tokens = eng.buf["tokens"][:batch].cpu().numpy()
    Wn = _np_weights(W)
    ref16 = _oracle_pass(shape, Wn, v, "bf16")
    # same rounding points as the bf16 reference: differences come only from fp32
    # accumulation order (and the chunked softmax), a few bf16 steps at most
    assert_bf16_close(gpu_logits, ref16, steps=4.0, exact_frac=0.3, what="logits vs bf16 reference")
    _, corrected = O.markov_sample(ref16, v["anchors"].numpy(), Wn, "bf16", forced=gpu_tokens)
    ties = tokens_exact_or_tied(gpu_tokens, corrected, what="draft tokens")
    if fp32_tol is not None:
        ref32 = _oracle_pass(shape, Wn, v, "fp32")
        own = float(np.abs(ref16 - ref32).max())  # the reference's own bf16-vs-fp32 drift, for the message
        err = float(np.abs(gpu_logits - ref32).max())
        assert err <= fp32_tol, f"logits vs fp32 reference: {err:.4f} > {fp32_tol} (reference bf16 drift {own:.4f})"
    return ties


def test_round_small_matches_oracle():
    assert _run_and_compare(SMALL, (700, 37, 2000), seed=3, fp32_tol=3e-2) <= 2


def test_round_small_gqa5_matches_oracle():
    shape = SMALL.with_(q_heads=10, tap_layers=1, draft_layers=1, slots=256, window=1024, markov_rank=0)
    assert _run_and_compare(shape, (1500, 5), seed=4, fp32_tol=3e-2) <= 2


def test_round_config1_matches_oracle():
    """BASELINE config 1 shapes: Qwen3-4B drafter (H=2560, 32/8 heads, I=9728,
    V=151936), 4K context, W=512, S=64, 16-token verify block (15 drafter rows)."""
    from longspark_b200.config import CFG1
    shape = CFG1.shape
    W = make_weights(shape, seed=0)
    v = make_views(shape, 1, [4096], seed=1, pool_pages=512)
    eng = _engine(shape, W, v, 1)
    dev = eng.device
    eng.draft(slots=torch.zeros(1, dtype=torch.int32, device=dev), seq_lens=v["seq_lens"].to(dev),
              anchors=v["anchors"].to(dev), page_table=v["page_table"].to(dev))
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    gl = to_np(eng.buf["logits"][:shape.block]).reshape(1, shape.block, shape.vocab)
    gt = eng.buf["tokens"][:1].cpu().numpy()
    Wn = _np_weights(W)
    del W
    ref16 = _oracle_pass(shape, Wn, v, "bf16")
    assert_bf16_close(gl, ref16, steps=4.0, exact_frac=0.3, what="cfg1 logits vs bf16 reference")
    _, corrected = O.markov_sample(ref16, v["anchors"].numpy(), Wn, "bf16", forced=gt)
    assert tokens_exact_or_tied(gt, corrected, what="cfg1 tokens") <= 2
    # Against fp32: the unmodified reference's own bf16 run is 0.042 (max over
    # every logit) from its fp32 run at these dimensions, above the 3e-2 of the
    # bf16-vs-fp32 bound; a path that rounds where the reference rounds cannot be
    # closer, so config 1 is held to the reference's own measured distance.
    ref32 = _oracle_pass(shape, Wn, v, "fp32")
    err = float(np.abs(gl - ref32).max())
    assert err <= max(3e-2, CFG1_REFERENCE_DRIFT), f"cfg1 logits vs fp32 reference: {err:.4f}"
    print(f"cfg1 (P=15): logits vs the fp32 restatement {err:.4f}, its own bf16 run "
          f"{float(np.abs(ref16 - ref32).max()):.4f}")


def test_round_with_refresh_and_graph_replay():
    """refresh + pass inside one CUDA graph equals the eager sequence, and the
    refreshed summary matches the oracle."""
    shape = SMALL
    batch = 2
    W = make_weights(shape, seed=9, norm_jitter=0.05)
    v = make_views(shape, batch, [900, 333], seed=10, extra_rows=64)
    dev = torch.device("cuda")
    e1 = _engine(shape, W, v, batch)
    e2 = _engine(shape, W, v, batch)
    slots = torch.arange(batch, dtype=torch.int32, device=dev)
    commit = torch.tensor([16, 3], dtype=torch.int32, device=dev)
    lens = v["seq_lens"].to(dev) + commit
    table = v["page_table"].to(dev)
    anchors = v["anchors"].to(dev)
    target = torch.randint(0, shape.vocab, (batch, shape.block + 1), device=dev)
    e1.round(slots=slots, seq_lens=lens, commit_lens=commit, anchors=anchors, page_table=table, target=target)
    g = GraphedDraft(e2, batch, with_refresh=True, with_target=True)
    g.load(slots=slots, seq_lens=lens, anchors=anchors, page_table=table, commit_lens=commit, target=target)
    # the warm-up run inside capture() performs one real refresh: restore the state first
    state = (e2.pools.summary_out.clone(), e2.pools.summary_lse.clone(), e2.pools.summary_bf16.clone())
    g.capture()
    e2.pools.summary_out.copy_(state[0])
    e2.pools.summary_lse.copy_(state[1])
    e2.pools.summary_bf16.copy_(state[2])
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(e1.buf["tokens"][:batch], e2.buf["tokens"][:batch])
    assert torch.equal(e1.buf["logits"][:batch * shape.block], e2.buf["logits"][:batch * shape.block])
    assert torch.equal(e1.pools.summary_out, e2.pools.summary_out)
    # the bf16 copy the attention reads is the rounded fp32 state
    assert torch.equal(e1.pools.summary_bf16, e1.pools.summary_out[:, :shape.draft_layers].to(torch.bfloat16))
    assert e1.device_status() == 0 and e2.device_status() == 0
    # summary vs oracle
    kk, vv = to_np(v["kv_k"]), to_np(v["kv_v"])
    c = commit.cpu().numpy()
    L = lens.cpu().numpy()
    nk = np.zeros((shape.tap_layers, batch, shape.max_commit, shape.kv_heads, 128), np.float32)
    nv = np.zeros_like(nk)
    for b in range(batch):
        for r in range(c[b]):
            pos = L[b] - c[b] + r
            page = int(v["page_table"][b, pos // 16])
            nk[:, b, r] = kk[:, page, pos % 16]
            nv[:, b, r] = vv[:, page, pos % 16]
    ro, rl = O.refresh_views(v["summary_out"].numpy(), v["summary_lse"].numpy(), np.arange(batch),
                             to_np(W["global16_raw256_reference.global_query_generator.learned_query"]), nk, nv, c,
                             128 ** -0.5)
    np.testing.assert_allclose(to_np(e1.pools.summary_out), ro, rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(to_np(e1.pools.summary_lse), rl, rtol=3e-5, atol=3e-5)
    acc = e1.buf["accept"][:batch].cpu().numpy()
    np.testing.assert_array_equal(acc, O.accept_lengths(target.cpu().numpy(), e1.buf["tokens"][:batch].cpu().numpy())[0])


@pytest.mark.parametrize("q_heads,kv_heads,slots_are_rows", [(8, 2, False), (10, 2, True)])
def test_native_round_entry_matches_engine(q_heads, kv_heads, slots_are_rows):
    """ls_draft_round (the whole round as one C-ABI call) against the Python
    engine's launch sequence on the same buffers: refresh, two drafter layers
    on different tapped layers, the Markov chain and the accept check; tokens,
    accept lengths, base logits and the refreshed summary state bit for bit."""
    shape = DraftShape(hidden=512, q_heads=q_heads, kv_heads=kv_heads, inter=1024, vocab=4096, tap_layers=2,
                       draft_layers=2, slots=64, window=512, block=15, max_commit=16, markov_rank=64,
                       mask_token_id=4000)
    batch = 3
    W = make_weights(shape, seed=21, norm_jitter=0.05)
    v = make_views(shape, batch, [900, 333, 2000], seed=22, extra_rows=64)
    dev = torch.device("cuda")
    e1 = _engine(shape, W, v, batch)
    e2 = _engine(shape, W, v, batch)
    slots = (torch.arange(batch, dtype=torch.int32, device=dev) if slots_are_rows
             else torch.tensor([2, 0, 1], dtype=torch.int32, device=dev))
    commit = torch.tensor([16, 3, 9], dtype=torch.int32, device=dev)
    lens = v["seq_lens"].to(dev) + commit
    table = v["page_table"].to(dev)
    anchors = v["anchors"].to(dev)
    target = torch.randint(0, shape.vocab, (batch, shape.block + 1), device=dev)
    kw = dict(slots=slots, seq_lens=lens, commit_lens=commit, anchors=anchors, page_table=table, target=target,
              slots_are_rows=slots_are_rows)
    e1.draft(**kw)
    e2.draft_native(**kw)
    torch.cuda.synchronize()
    M = batch * shape.block
    assert e1.device_status() == 0 and e2.device_status() == 0
    assert torch.equal(e1.buf["tokens"][:batch], e2.buf["tokens"][:batch])
    assert torch.equal(e1.buf["accept"][:batch], e2.buf["accept"][:batch])
    assert torch.equal(e1.buf["logits"][:M], e2.buf["logits"][:M])
    assert torch.equal(e1.pools.summary_out, e2.pools.summary_out)
    assert torch.equal(e1.pools.summary_lse, e2.pools.summary_lse)
    assert torch.equal(e1.pools.summary_bf16, e2.pools.summary_bf16)


def test_longspark_draft_api_prefill_update_propose():
    """The drop-in API: prefill packets (window rows + summary), decode updates in
    the batch message format, proposals; checked against the oracle on the same
    ring-window contents."""
    shape = SMALL.with_(window=256, tap_layers=2, draft_layers=2)
    W = make_weights(shape, seed=31, norm_jitter=0.05)
    cfg = dict(draft_device=0, max_running_requests=4, draft_state_gib=1.0, cuda_graph=True,
               graph_batch_sizes=(1, 2, 4))
    d = LongSparkDraft(cfg, weights=W, shape=shape)
    g = torch.Generator().manual_seed(32)
    L, Hkv, Hq, S = shape.tap_layers, shape.kv_heads, shape.q_heads, shape.slots
    ids, lengths = ["a", "b"], [300, 90]
    # full synthetic histories (rows 0..len+extra) for both requests
    hist = {i: (torch.randn(L, n + 64, Hkv, 128, generator=g).to(torch.bfloat16),
                torch.randn(L, n + 64, Hkv, 128, generator=g).to(torch.bfloat16)) for i, n in zip(ids, lengths)}
    gout = 0.1 * torch.randn(2, L, Hq, S, 128, generator=g)
    glse = torch.randn(2, L, Hq, S, generator=g) + 5.0
    hidden = torch.randn(2, L, shape.hidden, generator=g).to(torch.bfloat16)
    cnt = [min(n, shape.window) for n in lengths]
    keys = torch.cat([hist[i][0][:, n - c:n] for i, n, c in zip(ids, lengths, cnt)], dim=1)
    vals = torch.cat([hist[i][1][:, n - c:n] for i, n, c in zip(ids, lengths, cnt)], dim=1)
    d.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=lengths, commit_lens=cnt, export_counts=cnt,
                  keys=keys, values=vals, last_hidden=hidden, global_output=gout, global_lse=glse), prefill=True)
    with pytest.raises(RuntimeError, match="out-of-order"):
        d.update(dict(format="longspark_state_batch_v1", ids=["a"], lengths=[305], commit_lens=[4],
                      export_counts=[4], keys=keys[:, :4], values=vals[:, :4], last_hidden=hidden[:1]))
    # one decode commit
    commit = [5, 16]
    new_len = [n + c for n, c in zip(lengths, commit)]
    keys2 = torch.cat([hist[i][0][:, n:n + c] for i, n, c in zip(ids, lengths, commit)], dim=1)
    vals2 = torch.cat([hist[i][1][:, n:n + c] for i, n, c in zip(ids, lengths, commit)], dim=1)
    hidden2 = torch.randn(2, L, shape.hidden, generator=g).to(torch.bfloat16)
    d.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=new_len, commit_lens=commit,
                  export_counts=commit, keys=keys2, values=vals2, last_hidden=hidden2))
    anchors = [7, 4095]
    tokens, logits, q = d.propose(ids, anchors, 0.0)
    assert q is None and tokens.shape == (2, shape.block) and logits.shape == (2, shape.block, shape.vocab)
    assert d.graph_stats()["replays"] >= 1
    assert d.device_status() == 0
    # oracle on the same data
    Wn = _np_weights(W)
    qg = Wn["global16_raw256_reference.global_query_generator.learned_query"]
    out_np, lse_np = gout.numpy().copy(), glse.numpy().copy()
    nk = np.zeros((L, 2, shape.max_commit, Hkv, 128), np.float32)
    nv = np.zeros_like(nk)
    for b, (i, n, c) in enumerate(zip(ids, lengths, commit)):
        nk[:, b, :c] = to_np(hist[i][0][:, n:n + c])
        nv[:, b, :c] = to_np(hist[i][1][:, n:n + c])
    out_np, lse_np = O.refresh_views(out_np, lse_np, np.arange(2), qg, nk, nv, np.array(commit), 128 ** -0.5)
    views = []
    for j in range(shape.draft_layers):
        wk = np.zeros((2, Hkv, shape.window, 128), np.float32)
        wv = np.zeros_like(wk)
        wl = []
        for b, (i, n) in enumerate(zip(ids, new_len)):
            m = min(n, shape.window)
            wk[b, :, :m] = to_np(hist[i][0][j, n - m:n]).transpose(1, 0, 2)
            wv[b, :, :m] = to_np(hist[i][1][j, n - m:n]).transpose(1, 0, 2)
            wl.append(m)
        views.append(dict(qg=qg[j], summary_out=out_np[:, j], win_k=wk, win_v=wv, win_len=np.array(wl)))
    osh = O.DraftShapeOracle(shape.hidden, Hq, Hkv, 128, shape.block, shape.mask_token_id)
    base, _ = O.draft_pass(Wn, osh, np.array(anchors), np.array(new_len), to_np(hidden2), views,
                           rope_inv_freq(shape).numpy(), "bf16")
    gt = tokens.cpu().numpy()
    toks_ref, corrected = O.markov_sample(base, np.array(anchors), Wn, "bf16", forced=gt)
    assert tokens_exact_or_tied(gt, corrected, what="api tokens") <= 2
    assert_bf16_close(to_np(logits), corrected, steps=4.0, exact_frac=0.3, what="api corrected logits")
    # T > 0 on the same state: sampled tokens with their proposal probabilities
    # (LS engine/draft.py:284-286), corrected logits as at T = 0 for the sampled chain
    t2, l2, q2 = d.propose(ids, anchors, 0.8)
    assert q2 is not None and q2.shape == (2, shape.block) and l2.shape == (2, shape.block, shape.vocab)
    assert ((q2 > 0) & (q2 <= 1)).all() and ((t2 >= 0) & (t2 < shape.vocab)).all()
    assert d.device_status() == 0
    _, q_ref, corr_ref, _ = O.markov_sample_gumbel(to_np(d.engine.buf["logits"][:2 * shape.block]).reshape(
        2, shape.block, shape.vocab), np.array(anchors), Wn, "bf16", 0.8, 0, forced=t2.cpu().numpy())
    assert_bf16_close(to_np(l2), corr_ref, steps=1.0, exact_frac=0.98, what="api T>0 corrected logits")
    t3, _, _ = d.propose(ids, anchors, 0.8)  # a fresh seed each proposal
    assert not torch.equal(t2, t3)
    d.release(["a"])
    assert 1 in d.free_slots or 0 in d.free_slots


def test_step_graph_capture_with_collector_pressure():
    """A drafter whose captured graphs sit in a reference cycle is dropped;
    then, with Python's cyclic collector set to run at every allocation, a
    second drafter captures its step graph (``capture_guard`` keeps automatic
    collection out of the capture) and proposes the same tokens as a drafter
    that runs eagerly on the same inputs."""
    import gc

    shape = SMALL.with_(window=256)
    W = make_weights(shape, seed=41, norm_jitter=0.05)
    g = torch.Generator().manual_seed(42)
    L, Hkv, Hq, S = shape.tap_layers, shape.kv_heads, shape.q_heads, shape.slots
    ids, n = ["x", "y"], 200
    hist = torch.randn(L, 2 * (n + 16), Hkv, 128, generator=g).to(torch.bfloat16)

    def drive(use_graph):
        cfg = dict(draft_device=0, max_running_requests=2, draft_state_gib=0.5, cuda_graph=use_graph)
        d = LongSparkDraft(cfg, weights=W, shape=shape)
        d.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=[n, n], commit_lens=[n, n],
                      export_counts=[n, n], keys=hist[:, :2 * n], values=hist[:, :2 * n],
                      last_hidden=torch.ones(2, L, shape.hidden, dtype=torch.bfloat16),
                      global_output=torch.zeros(2, L, Hq, S, 128), global_lse=torch.full((2, L, Hq, S), 3.0)),
                 prefill=True)
        d.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=[n + 16, n + 16], commit_lens=[16, 16],
                      export_counts=[16, 16], keys=hist[:, 2 * n:], values=hist[:, 2 * n:],
                      last_hidden=torch.ones(2, L, shape.hidden, dtype=torch.bfloat16)))
        tokens, logits, _ = d.propose(ids, [5, 9], 0.0)
        torch.cuda.synchronize()
        assert d.device_status() == 0
        return d, tokens, logits

    d1, _, _ = drive(True)
    d1.cycle = d1  # unreachable after the del below, collectable only by the cyclic collector
    del d1
    old = gc.get_threshold()
    gc.set_threshold(1, 1, 1)
    try:
        d2, t2, l2 = drive(True)
        assert d2.graph_stats()["replays"] >= 1
    finally:
        gc.set_threshold(*old)
        gc.collect()
    _, t3, l3 = drive(False)
    assert torch.equal(t2, t3)
    assert torch.equal(l2, l3)
