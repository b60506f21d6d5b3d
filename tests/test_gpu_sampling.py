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
