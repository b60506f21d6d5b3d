"""a Qwen3-14B-shaped drafter (H=5120, 40 query / 8 KV heads,
so GQA 5, SwiGLU 17408) at 128K context with W=2048, S=256 and a 16-token
verify block, driven through 200 consecutive rounds of incremental refresh and
drafting over 5 tapped layers.  Every round the summary state (out, lse) must
follow the oracle's incremental refresh chain, the bf16 logits must lie within
a few bf16 steps of the oracle's pass on the oracle's own state, and the
Markov-greedy tokens must equal the oracle's own (un-forced) chain, a tie in
the oracle's bf16 logits being the one accepted difference (counted and
printed).
"""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import assert_bf16_close, compare_chain_with_reference, to_np
from longspark_b200.config import CFG3
from longspark_b200.engine import DraftEngine, DraftWeights, ViewPools
from longspark_b200.synthetic import make_views, make_weights, rope_inv_freq

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _rows(pool, table, positions):
    """[L_tap, n, Hkv, 128] fp32 rows of a paged pool at `positions` (request 0)."""
    pos = torch.as_tensor(positions, dtype=torch.long, device=pool.device)
    pages = table[0].long()[pos // 16]
    return pool[:, pages, pos % 16].float().cpu().numpy()


def test_chain_config3_200_rounds():
    shape = CFG3.shape
    rounds = 200
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(3)
    commits = [1 + (7 * t) % 16 for t in range(rounds)]
    ctx0 = 131072
    W = make_weights(shape, device=dev, gen=gen, norm_jitter=0.05)
    v = make_views(shape, 1, [ctx0], device=dev, gen=gen, extra_rows=sum(commits))
    pools = ViewPools(kv_k=v["kv_k"], kv_v=v["kv_v"], page_table=v["page_table"], summary_out=v["summary_out"].clone(),
                      summary_lse=v["summary_lse"].clone(), hidden=v["hidden"])
    eng = DraftEngine(shape, DraftWeights(shape, W, dev), pools, max_batch=1, device=dev)
    Wn = {k: t.float().cpu().numpy() for k, t in W.items()}
    del W
    qg = Wn["global16_raw256_reference.global_query_generator.learned_query"]
    osh = O.DraftShapeOracle(shape.hidden, shape.q_heads, shape.kv_heads, 128, shape.block, shape.mask_token_id,
                             shape.rms_eps, shape.final_eps)
    inv_freq = rope_inv_freq(shape).numpy()
    hidden = v["hidden"].float().cpu().numpy()
    ro = v["summary_out"].cpu().numpy()
    rl = v["summary_lse"].cpu().numpy()
    slots = torch.zeros(1, dtype=torch.int32, device=dev)
    table = v["page_table"]
    anchors_all = torch.randint(0, shape.vocab, (rounds,), generator=torch.Generator().manual_seed(4))
    length = ctx0
    checked = 0
    ties = []
    for t, c in enumerate(commits):
        length += c
        anchors = anchors_all[t:t + 1]
        eng.round(slots=slots, seq_lens=torch.tensor([length], dtype=torch.int32, device=dev),
                  commit_lens=torch.tensor([c], dtype=torch.int32, device=dev), anchors=anchors.to(dev),
                  page_table=table)
        # oracle: the same committed rows folded into its own chain
        new = np.arange(length - c, length)
        nk = np.zeros((shape.tap_layers, 1, shape.max_commit, shape.kv_heads, 128), np.float32)
        nv = np.zeros_like(nk)
        nk[:, 0, :c] = _rows(v["kv_k"], table, new)
        nv[:, 0, :c] = _rows(v["kv_v"], table, new)
        ro, rl = O.refresh_views(ro, rl, np.array([0]), qg, nk, nv, np.array([c]), 128 ** -0.5)
        torch.cuda.synchronize()
        assert eng.device_status() == 0, f"round {t}"
        np.testing.assert_allclose(to_np(pools.summary_out), ro, rtol=1e-4, atol=1e-4,
                                   err_msg=f"summary out after round {t}")
        np.testing.assert_allclose(to_np(pools.summary_lse), rl, rtol=1e-4, atol=1e-4,
                                   err_msg=f"summary lse after round {t}")
        win = np.arange(length - shape.window, length)
        view_layer = shape.view_layer(0)
        wk = _rows(v["kv_k"], table, win)[view_layer].transpose(1, 0, 2)[None]  # [1, Hkv, W, 128]
        wv = _rows(v["kv_v"], table, win)[view_layer].transpose(1, 0, 2)[None]
        views = [dict(qg=qg[view_layer], summary_out=ro[:, view_layer], win_k=wk, win_v=wv,
                      win_len=np.array([shape.window]))]
        ref16, _ = O.draft_pass(Wn, osh, anchors.numpy(), np.array([length]), hidden, views, inv_freq, "bf16")
        gl = to_np(eng.buf["logits"][:shape.block]).reshape(1, shape.block, shape.vocab)
        gt = eng.buf["tokens"][:1].cpu().numpy()
        # every logit within 4 bf16 steps of the bf16 oracle; with H = 5120 and
        # I = 17408 the longer fp32 reductions leave fewer bit-identical values
        # than at the 4B shape (measured 23% at round 0), hence the lower floor
        assert_bf16_close(gl, ref16, steps=4.0, exact_frac=0.15, what=f"config 3 logits, round {t}")
        ref_tokens, corrected = O.markov_sample(ref16, anchors.numpy(), Wn, "bf16")
        top = np.argsort(-corrected, axis=-1, kind="stable")[..., :4]
        ties += [(t,) + x[1:] for x in compare_chain_with_reference(
            gt, ref_tokens, np.take_along_axis(corrected, top, axis=-1), top, what=f"config 3 tokens, round {t}")]
        checked += 1
    print(f"config 3: {rounds} rounds x {shape.block} tokens against the oracle's own chain; rounds whose chain "
          f"took a tie of the oracle's bf16 logits: {len(ties)} {ties}")
    assert checked == rounds
