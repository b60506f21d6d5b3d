"""Temperature > 0 proposals: the sampling step against the oracle's Gumbel-max
restatement (same counter-based noise), the sampled distribution against
softmax(logits / T), and the whole step loop (Markov-corrected step logits by
GEMM, then the draw) against the oracle's chain."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import assert_bf16_close, to_np
from longspark_b200 import ops
from longspark_b200.config import DraftShape
from longspark_b200.engine import DraftEngine, DraftWeights, ViewPools
from longspark_b200.synthetic import make_views, make_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _oracle_step(row, T, seed, b, t):
    z = (row.astype(np.float32) / np.float32(T)).astype(np.float32)
    u = O.gumbel_hash_uniform(seed, b, t, np.arange(row.shape[0]))
    key = (z + -np.log(-np.log(u))).astype(np.float32)
    tok = int(np.argmax(key))
    top2 = np.partition(key, -2)[-2:]
    e = np.exp(z - z.max())
    return tok, float(e[tok] / e.sum(dtype=np.float32)), float(top2[1] - top2[0])


@pytest.mark.parametrize("vocab,T", [(32768, 0.7), (151936, 1.0), (1000, 2.5)])
def test_sample_step_matches_oracle(vocab, T):
    B, P = 6, 15
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(vocab)
    logits = (torch.randn(B, P, vocab, generator=g) * 3.0).to(torch.bfloat16)
    lg = logits.to(dev)
    tokens = torch.zeros(B, P, dtype=torch.int64, device=dev)
    q = torch.zeros(B, P, dtype=torch.float32, device=dev)
    prev = torch.zeros(B, dtype=torch.int32, device=dev)
    ws = torch.zeros(ops.sample_step_workspace_bytes(B), dtype=torch.uint8, device=dev)
    seed = 0x1234_5678_9ABC_DEF0
    for t in (0, 7, 14):
        ops.sample_step(logits=lg[:, t], step=t, block=P, temperature=T, seed=seed, tokens=tokens, workspace=ws,
                        q=q, prev=prev)
    torch.cuda.synchronize()
    gt, gq, gp = tokens.cpu().numpy(), q.cpu().numpy(), prev.cpu().numpy()
    ln = logits.float().numpy()
    for t in (0, 7, 14):
        for b in range(B):
            tok, qq, gap = _oracle_step(ln[b, t], T, seed, b, t)
            if gap > 1e-4:  # float32 log / exp of the two libraries agree far inside this margin
                assert gt[b, t] == tok, (b, t)
            np.testing.assert_allclose(gq[b, t], qq if gt[b, t] == tok else gq[b, t], rtol=2e-5)
    assert (gp == gt[:, 14]).all()


def test_sampled_tokens_follow_softmax():
    """4096 requests with the same logits row, 6 seeds: 24576 draws against
    softmax(logits / T) (max standardized deviation of the 64 frequencies)."""
    B, V, T = 4096, 64, 0.8
    dev = torch.device("cuda")
    row = torch.linspace(-2.0, 2.0, V)
    logits = row.to(torch.bfloat16)[None].expand(B, V).contiguous().to(dev)
    tokens = torch.zeros(B, 1, dtype=torch.int64, device=dev)
    ws = torch.zeros(ops.sample_step_workspace_bytes(B), dtype=torch.uint8, device=dev)
    counts = np.zeros(V)
    for seed in range(6):
        ops.sample_step(logits=logits, step=0, block=1, temperature=T, seed=seed + 1, tokens=tokens, workspace=ws)
        torch.cuda.synchronize()
        counts += np.bincount(tokens[:, 0].cpu().numpy(), minlength=V)
    z = row.to(torch.bfloat16).float().numpy() / T
    p = np.exp(z - z.max())
    p /= p.sum()
    n = counts.sum()
    dev_std = (counts - n * p) / np.sqrt(n * p * (1 - p))
    assert np.abs(dev_std).max() < 4.5, dev_std


def test_engine_sample_matches_oracle_chain():
    shape = DraftShape(hidden=512, q_heads=8, kv_heads=2, inter=1024, vocab=4096, tap_layers=2, draft_layers=1,
                       slots=64, window=512, block=15, max_commit=16, markov_rank=64, mask_token_id=4000)
    batch = 3
    dev = torch.device("cuda")
    W = make_weights(shape, seed=11, norm_jitter=0.05)
    v = make_views(shape, batch, [700, 90, 1500], seed=12)
    pools = ViewPools(kv_k=v["kv_k"].to(dev), kv_v=v["kv_v"].to(dev), page_table=v["page_table"].to(dev),
                      summary_out=v["summary_out"].to(dev), summary_lse=v["summary_lse"].to(dev),
                      hidden=v["hidden"].to(dev))
    eng = DraftEngine(shape, DraftWeights(shape, W, dev), pools, max_batch=batch, device=dev)
    anchors = v["anchors"].to(dev)
    eng.draft(slots=torch.arange(batch, dtype=torch.int32, device=dev), seq_lens=v["seq_lens"].to(dev),
              anchors=anchors, page_table=v["page_table"].to(dev))
    base = to_np(eng.buf["logits"][:batch * shape.block]).reshape(batch, shape.block, shape.vocab)
    T, seed = 0.9, 987654321
    corr = eng.sample(anchors, temperature=T, seed=seed)
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    gt = eng.buf["tokens"][:batch].cpu().numpy()
    gq = eng.buf["q"][:batch].cpu().numpy()
    Wn = {k: t.float().numpy() for k, t in W.items()}
    # the oracle's chain over the same base logits, fed the GPU's tokens
    toks, q, ref_corr, gap = O.markov_sample_gumbel(base, anchors.cpu().numpy(), Wn, "bf16", T, seed, forced=gt)
    # corrected step logits: one GEMM per step, fp32 accumulation order only
    assert_bf16_close(to_np(corr), ref_corr, steps=1.0, exact_frac=0.98, what="corrected step logits")
    sure = gap > 1e-2  # a corrected logit one bf16 step off can move a key by ~1e-2 / T
    assert (gt[sure] == toks[sure]).all()
    assert sure.mean() > 0.9
    np.testing.assert_allclose(gq[gt == toks], q[gt == toks], rtol=1e-3)


# ----------------------------------------------------------------------------
# T > 0 verification: two-phase rejection sampling (ls_rejection_sample)
# ----------------------------------------------------------------------------

def test_rejection_sampling_matches_reference(golden_dir):
    """Accept lengths and bonus tokens equal to the reference's
    ``decide_acceptance`` + ``finish_sampling`` run with the same uniforms
    (fixtures from the unmodified reference): 64 requests at V=4096 and 8 at
    V=151936 with 7 and 15 proposals, including requests that reject where the
    residual has zero mass (the fallback to the target row)."""
    import sys
    sys.path.insert(0, str(golden_dir))
    from sampling_inputs import CASES, sampling_logits

    z = np.load(golden_dir / "rejection_sampling.npz")
    dev = torch.device("cuda")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for case, (batch, block, vocab, temp, seed, sd, sn, same) in CASES.items():
        target, draft = sampling_logits(batch, block, vocab, seed, sd, sn, same)
        p = case + "_"
        lengths, bonus = ops.rejection_sample(
            candidates=torch.from_numpy(z[p + "candidates"]).to(dev), sampled_q=torch.from_numpy(z[p + "q"]).to(dev),
            target_logits=target.to(dev), draft_logits=draft.to(dev), temperature=temp,
            uniforms=torch.from_numpy(z[p + "uniforms"]).to(dev), final_uniforms=torch.from_numpy(z[p + "final"]).to(dev),
            status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        np.testing.assert_array_equal(lengths.cpu().numpy(), z[p + "lengths"], err_msg=case)
        np.testing.assert_array_equal(bonus.cpu().numpy(), z[p + "bonus"], err_msg=case)


@pytest.mark.parametrize("batch,block,vocab,temp", [(33, 16, 8192, 0.3), (5, 1, 151936, 2.0), (3, 15, 151936, 0.8)])
def test_rejection_sampling_matches_oracle(batch, block, vocab, temp):
    """Random drafts and verify passes with consistent q (from the drafter's
    own distribution), against the oracle restatement; strided views of
    larger logit buffers, as the engine hands them over."""
    g = torch.Generator().manual_seed(batch * 131 + block)
    draft = (2.0 * torch.randn(batch, block, vocab, generator=g)).to(torch.bfloat16)
    target = (draft.float()[:, list(range(block)) + [block - 1]] +
              0.4 * torch.randn(batch, block + 1, vocab, generator=g)).to(torch.bfloat16)
    probs = torch.softmax(draft.float() / temp, -1)
    cand = torch.multinomial(probs.view(-1, vocab), 1, generator=g).view(batch, block)
    q = probs.gather(-1, cand[..., None]).squeeze(-1)
    u = torch.rand(batch, block, generator=g)
    uf = torch.rand(batch, generator=g)
    dev = torch.device("cuda")
    pad = torch.zeros(batch, block + 1, vocab + 64, dtype=torch.bfloat16)
    pad[..., :vocab] = target
    lengths, bonus = ops.rejection_sample(candidates=cand.to(dev), sampled_q=q.to(dev),
                                          target_logits=pad.to(dev)[..., :vocab], draft_logits=draft.to(dev),
                                          temperature=temp, uniforms=u.to(dev), final_uniforms=uf.to(dev))
    want_l, want_b = O.rejection_sample(target.float().numpy(), draft.float().numpy(), cand.numpy(), q.numpy(), temp,
                                        u.numpy(), uf.numpy())
    np.testing.assert_array_equal(lengths.cpu().numpy(), want_l)
    np.testing.assert_array_equal(bonus.cpu().numpy(), want_b)


def test_rejection_sampling_argument_errors():
    """The reference's shape errors (LS engine/sampling.py:21-25, 41-43) and a
    candidate outside the vocabulary (device status LS_DEV_BAD_TOKEN)."""
    dev = torch.device("cuda")
    b, p, v = 2, 3, 256
    t = torch.zeros(b, p + 1, v, dtype=torch.bfloat16, device=dev)
    d = torch.zeros(b, p, v, dtype=torch.bfloat16, device=dev)
    c = torch.zeros(b, p, dtype=torch.int64, device=dev)
    q = torch.full((b, p), 0.5, device=dev)
    u = torch.full((b, p), 0.5, device=dev)
    uf = torch.full((b,), 0.5, device=dev)
    with pytest.raises(ValueError, match="proposal positions"):
        ops.rejection_sample(candidates=c, sampled_q=q[:, :2], target_logits=t, draft_logits=d, temperature=1.0,
                             uniforms=u, final_uniforms=uf)
    with pytest.raises(ValueError, match="plus one bonus row"):
        ops.rejection_sample(candidates=c, sampled_q=q, target_logits=t[:, :p], draft_logits=d, temperature=1.0,
                             uniforms=u, final_uniforms=uf)
    with pytest.raises(ValueError, match="one final uniform"):
        ops.rejection_sample(candidates=c, sampled_q=q, target_logits=t, draft_logits=d, temperature=1.0,
                             uniforms=u, final_uniforms=uf[:1])
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    c[1, 0] = v + 5
    lengths, bonus = ops.rejection_sample(candidates=c, sampled_q=q, target_logits=t, draft_logits=d, temperature=1.0,
                                          uniforms=u, final_uniforms=uf, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 111
    # flat logits: p = 1/256 for every token, u * q = 0.25 >= p rejects at 0;
    # the residual p - q_row is zero, so the draw falls back to the target row
    assert lengths.tolist() == [0, 0]
    assert bonus.tolist() == [128, 128]  # cumsum reaches 0.5 at index 127: 128 prefixes <= u
