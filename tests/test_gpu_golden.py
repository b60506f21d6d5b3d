"""The CUDA path against the reference's own outputs (golden fixtures written
by ``tests/golden/make_golden.py`` from the unmodified reference on the CPU),
with no oracle in between.

* The reference contract (Global16 / Raw256 / Local7: S=16, W=256, P=7) and a
  widened GQA-5 shape (S=64, W=512), inputs stored in the fixtures.
* Config-1 dimensions (Qwen3-4B, 4K context) at P=7, inputs regenerated from
  the fixture's seeds.
* Chained runs at config-3 dimensions (Qwen3-14B, W=2048, S=256, 128K
  context, 200 rounds: refresh of each round's commit, then the pass) and
  config-2 dimensions (Qwen3-8B, W=1024, S=256, 128K), one tapped and one
  drafter layer (the reference needs a drafter layer per tapped layer).

Bars: draft tokens equal to the reference's, where the only accepted
difference is a tie in the reference's own bf16 logits (its top-2 at most one
bf16 step apart; the count is printed); bf16 base logits within a few bf16
steps of the reference's bf16 run; bf16 base logits within 3e-2 of the
reference's fp32 run, except where the reference's own bf16 run is further
than that from its fp32 run (config 1 and the chained runs: the measured
distances and the bounds are stated below).
"""

import numpy as np
import pytest
import torch

import oracle as O
from golden.chain_inputs import chain_views, chain_weights, committed_rows
from gpu_util import bf16_step, compare_chain_with_reference, to_np
from longspark_b200.config import DraftShape
from longspark_b200.engine import DraftEngine, DraftWeights, ViewPools
from longspark_b200.synthetic import make_views, make_weights

pytestmark = pytest.mark.gpu

# north-star bound on the bf16 logits against the reference's fp32 output
FP32_TOL = 3e-2
# Config 1 (H=2560, V=151936): the reference's own bf16 run is 0.0370 away from
# its fp32 run on the fixture's logits (max over the ids both runs rank in
# their top 32, all 7 steps); no implementation that rounds where the
# reference rounds can be closer, so this config is held to that distance.
CFG1_REFERENCE_DRIFT = 0.0370
# The chained fixtures' larger dimensions put the top logits at 6-8.1, where one
# bf16 step is 0.031-0.062 and rounding an exact value to bf16 alone can move
# it by up to 0.031.  Measured on the fixtures (the logits both of the
# reference's runs rank in their top 4, every round and step): the reference's
# own bf16 run is, from its fp32 run, at most / on average
#   config-2 dimensions: 0.0435 / 0.0122   (largest |logit| 6.2)
#   config-3 dimensions: 0.0594 / 0.0135   (largest |logit| 8.1)
# These configs are held to: max <= the reference's own max plus one bf16 step
# at the largest logit (the GPU's bf16 value may sit one step from the
# reference's bf16 value, which the bf16 comparison bounds), and mean <= 1.25x
# the reference's own mean.
CHAIN_REFERENCE_DRIFT = {"chain_cfg2_p7": (0.0435, 0.0122, 0.03125), "chain_cfg3_p7": (0.0594, 0.0135, 0.0625)}
# Token ties: one bf16 step between the reference's top two everywhere but the
# 200-round config-3 chain, where the GPU's summary state has followed its own
# fp32 summation order for up to 200 refreshes and its logits sit up to 2 bf16
# steps from the reference's (measured: one flip at 2 steps, round 154); the
# count and gap of every flip are printed.
CHAIN_TIE_STEPS = {"chain_cfg2_p7": 1.0, "chain_cfg3_p7": 2.0}
# bf16 logits against the reference's bf16 run: the rounding points are the
# reference's, only the fp32 accumulation order differs, and a one-step
# difference in an intermediate propagates; at most this many bf16 steps (at
# the largest logit magnitude)
BF16_STEPS = 4.0


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _bf16_tensor(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _shape_from(arr, max_commit=None):
    h, hq, hkv, inter, vocab, tap, drf, slots, window, block, rank, mask = [int(x) for x in arr]
    return DraftShape(hidden=h, q_heads=hq, kv_heads=hkv, inter=inter, vocab=vocab, tap_layers=tap,
                      draft_layers=drf, slots=slots, window=window, block=block,
                      max_commit=max_commit or block + 1, markov_rank=rank, mask_token_id=mask)


def _engine(shape, W, views, batch):
    dev = torch.device("cuda")
    pools = ViewPools(kv_k=views["kv_k"].to(dev), kv_v=views["kv_v"].to(dev), page_table=views["page_table"].to(dev),
                      summary_out=views["summary_out"].to(dev).contiguous(),
                      summary_lse=views["summary_lse"].to(dev).contiguous(), hidden=views["hidden"].to(dev))
    return DraftEngine(shape, DraftWeights(shape, W, dev), pools, max_batch=batch, device=dev)


def _top(x, k):
    ids = np.argsort(-x, axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(x, ids, axis=-1), ids


@pytest.mark.parametrize("stem", ["draft_small_ref", "draft_small_gqa5_s64_w512"])
def test_pass_matches_reference_fixture(golden_dir, stem):
    """One drafter pass on the fixture's own inputs: base logits against the
    reference's bf16 and fp32 runs, Markov-greedy tokens against the
    reference's bf16 tokens."""
    z = np.load(golden_dir / f"{stem}_inputs.npz")
    g16 = np.load(golden_dir / f"{stem}_bf16.npz")
    g32 = np.load(golden_dir / f"{stem}_fp32.npz")
    shape = _shape_from(g16["shape"])
    W = {k[3:]: _bf16_tensor(z[k]) for k in z.files if k.startswith("w::")}
    B = int(z["anchors"].shape[0])
    views = dict(kv_k=_bf16_tensor(z["kv_k"]), kv_v=_bf16_tensor(z["kv_v"]),
                 page_table=torch.from_numpy(z["table"]), summary_out=torch.from_numpy(z["summary_out"]),
                 summary_lse=torch.zeros(z["summary_out"].shape[:-1]), hidden=_bf16_tensor(z["hidden"]))
    eng = _engine(shape, W, views, B)
    dev = eng.device
    anchors = torch.from_numpy(z["anchors"]).to(dev)
    eng.draft(slots=torch.arange(B, dtype=torch.int32, device=dev), seq_lens=torch.from_numpy(z["seq_lens"]).to(dev),
              anchors=anchors, page_table=views["page_table"].to(dev))
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    P, V = shape.block, shape.vocab
    base = to_np(eng.buf["logits"][:B * P]).reshape(B, P, V)
    tokens = eng.buf["tokens"][:B].cpu().numpy()
    ref16 = O.from_bf16_bits(g16["base_logits"])
    err16 = float(np.abs(base - ref16).max())
    exact = float((base == ref16).mean())
    assert err16 <= BF16_STEPS * bf16_step(ref16), f"{stem}: bf16 logits {err16:.4g} from the reference's bf16 run"
    err32 = float(np.abs(base - g32["base_logits"]).max())
    assert err32 <= FP32_TOL, f"{stem}: bf16 logits {err32:.4g} from the reference's fp32 run (> {FP32_TOL})"
    corr = O.from_bf16_bits(g16["corrected"])
    vals, ids = _top(corr, 4)
    ties = compare_chain_with_reference(tokens, g16["tokens"], vals, ids, what=stem)
    print(f"{stem}: tokens {tokens.tolist()} reference {g16['tokens'].tolist()}; ties {ties}; bf16 logits "
          f"max |diff| {err16:.4g} ({exact:.3f} bit-identical), vs fp32 {err32:.4g}")
    # corrected logits of the rows whose chain is the reference's
    out = torch.empty(B * P, V, dtype=torch.bfloat16, device=dev)
    eng.corrected_logits(anchors, out, batch=B)
    gc = to_np(out).reshape(B, P, V)
    same = [b for b in range(B) if np.array_equal(tokens[b], g16["tokens"][b])]
    if same:
        e = float(np.abs(gc[same] - corr[same]).max())
        assert e <= BF16_STEPS * bf16_step(corr), f"{stem}: corrected logits {e:.4g} from the reference"


def test_pass_config1_dimensions_matches_reference(golden_dir):
    """Config-1 dimensions (H=2560, 32/8 heads, I=9728, V=151936, 4K context,
    S=64, W=512) at the reference's P=7; inputs regenerated from the seeds the
    fixture was made with."""
    g16 = np.load(golden_dir / "draft_cfg1_p7_bf16.npz")
    g32 = np.load(golden_dir / "draft_cfg1_p7_fp32.npz")
    shape = _shape_from(g16["shape"])
    seed = int(g16["seed"])
    W = make_weights(shape, seed=seed, norm_jitter=float(g16["norm_jitter"]))
    v = make_views(shape, 1, [int(c) for c in g16["contexts"]], seed=seed + 1)
    eng = _engine(shape, W, v, 1)
    del W
    dev = eng.device
    eng.draft(slots=torch.zeros(1, dtype=torch.int32, device=dev), seq_lens=v["seq_lens"].to(dev),
              anchors=v["anchors"].to(dev), page_table=v["page_table"].to(dev))
    torch.cuda.synchronize()
    assert eng.device_status() == 0
    P, V = shape.block, shape.vocab
    base = to_np(eng.buf["logits"][:P]).reshape(1, P, V)
    tokens = eng.buf["tokens"][:1].cpu().numpy()
    at16 = np.take_along_axis(base, g16["base_top_ids"], axis=-1)
    err16 = float(np.abs(at16 - g16["base_top_values"]).max())
    assert err16 <= BF16_STEPS * bf16_step(g16["base_top_values"]), f"cfg1: {err16:.4g} from the bf16 run"
    at32 = np.take_along_axis(base, g32["base_top_ids"], axis=-1)
    err32 = float(np.abs(at32 - g32["base_top_values"]).max())
    assert err32 <= max(FP32_TOL, CFG1_REFERENCE_DRIFT), f"cfg1: {err32:.4g} from the reference's fp32 run"
    ties = compare_chain_with_reference(tokens, g16["tokens"], g16["corrected_top_values"],
                                        g16["corrected_top_ids"], what="cfg1")
    print(f"cfg1 p7: tokens {tokens.tolist()}; ties {ties}; top-32 logits vs bf16 run {err16:.4g}, "
          f"vs fp32 run {err32:.4g} (reference's own drift {CFG1_REFERENCE_DRIFT})")


@pytest.mark.parametrize("name", ["chain_cfg2_p7", "chain_cfg3_p7"])
def test_chain_matches_reference_every_round(golden_dir, name):
    """Every round: refresh the summary with the round's committed rows, run
    the pass, compare the tokens with the reference's tokens of that round
    (the reference ran the same chain: its own fp32 summary updates, its own
    bf16 pass), the base logits at the reference's top-4 ids with its bf16 and
    fp32 runs, and the summary state with the oracle's chain (pinned to the
    reference by the refresh fixtures); the summary lse after the first and the
    last round also against the reference's own."""
    g = np.load(golden_dir / f"{name}.npz")
    shape = _shape_from(g["shape"], max_commit=8)
    rounds, ctx0, seed = int(g["rounds"]), int(g["ctx0"]), int(g["seed"])
    W = chain_weights(shape, seed)
    v = chain_views(shape, ctx0, rounds, seed + 1)
    views = dict(kv_k=v["kv_k"], kv_v=v["kv_v"], page_table=v["page_table"], summary_out=v["summary_out"],
                 summary_lse=v["summary_lse"], hidden=v["hidden"][0])
    qg = W["global16_raw256_reference.global_query_generator.learned_query"].float().numpy()
    eng = _engine(shape, W, views, 1)
    del W
    dev = eng.device
    pools = eng.pools
    P, V = shape.block, shape.vocab
    slots = torch.zeros(1, dtype=torch.int32, device=dev)
    table = pools.page_table
    ro, rl = v["summary_out"].numpy().copy(), v["summary_lse"].numpy().copy()
    all_ties, worst16, worst32, worst_state, d32 = [], 0.0, 0.0, 0.0, []
    for t in range(rounds):
        c, n = int(v["commits"][t]), int(v["lengths"][t])
        pools.hidden[0].copy_(v["hidden"][t][0])
        anchors = v["anchors"][t:t + 1].to(dev)
        eng.round(slots=slots, seq_lens=torch.tensor([n], dtype=torch.int32, device=dev),
                  commit_lens=torch.tensor([c], dtype=torch.int32, device=dev), anchors=anchors, page_table=table)
        torch.cuda.synchronize()
        assert eng.device_status() == 0, f"{name} round {t}"
        # summary state against the oracle's chain
        nk = committed_rows(v["kv_k"], v["page_table"], n, c, shape.max_commit).float().numpy()
        nv = committed_rows(v["kv_v"], v["page_table"], n, c, shape.max_commit).float().numpy()
        ro, rl = O.refresh_views(ro, rl, np.array([0]), qg, nk, nv, np.array([c]), 128 ** -0.5)
        go, gl = to_np(pools.summary_out), to_np(pools.summary_lse)
        np.testing.assert_allclose(go, ro, rtol=1e-4, atol=1e-4, err_msg=f"{name}: summary out, round {t}")
        np.testing.assert_allclose(gl, rl, rtol=1e-4, atol=1e-4, err_msg=f"{name}: summary lse, round {t}")
        worst_state = max(worst_state, float(np.abs(gl - rl).max()))
        if t == 0:
            np.testing.assert_allclose(gl, g["lse_first"], rtol=1e-4, atol=1e-4)
        if t == rounds - 1:
            np.testing.assert_allclose(gl, g["lse_last"], rtol=1e-4, atol=1e-4)
        # tokens and logits against the reference's round t
        base = to_np(eng.buf["logits"][:P]).reshape(1, P, V)
        tokens = eng.buf["tokens"][:1].cpu().numpy()
        ties = compare_chain_with_reference(tokens, g["tokens"][t][None], g["corr_vals"][t][None],
                                            g["corr_ids"][t][None], what=f"{name} round {t}",
                                            max_steps=CHAIN_TIE_STEPS[name])
        all_ties += [(t,) + x[1:] for x in ties]
        at16 = np.take_along_axis(base[0], g["base_ids"][t], axis=-1)
        e16 = float(np.abs(at16 - g["base_vals"][t]).max())
        assert e16 <= BF16_STEPS * bf16_step(g["base_vals"][t]), f"{name} round {t}: {e16:.4g} from bf16 run"
        at32 = np.take_along_axis(base[0], g["base32_ids"][t], axis=-1)
        e32 = float(np.abs(at32 - g["base32_vals"][t]).max())
        ref_max, ref_mean, step = CHAIN_REFERENCE_DRIFT[name]
        assert e32 <= max(FP32_TOL, ref_max + step), f"{name} round {t}: {e32:.4g} from the reference's fp32 run"
        worst16, worst32 = max(worst16, e16), max(worst32, e32)
        d32.append(np.abs(at32 - g["base32_vals"][t]).ravel())
    mean32 = float(np.concatenate(d32).mean())
    print(f"{name}: {rounds} rounds x {P} tokens; rounds whose chain took a tie of the reference: {len(all_ties)} "
          f"{all_ties}; top-4 logits vs bf16 run <= {worst16:.4g}, vs fp32 run max {worst32:.4g} mean {mean32:.4g} "
          f"(the reference's own bf16 run: max {ref_max}, mean {ref_mean}); summary lse vs oracle <= "
          f"{worst_state:.3g}")
    assert mean32 <= 1.25 * ref_mean, f"{name}: mean distance to the fp32 run {mean32:.4g}"
