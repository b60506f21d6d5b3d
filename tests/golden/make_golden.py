"""Generate golden input/output fixtures by running the UNMODIFIED LongSpark
reference on the CPU.

Usage (needs a read-only LongSpark checkout; default path below):

    LONGSPARK_REFERENCE=/path/to/LongSpark python tests/golden/make_golden.py

Nothing here is imported by the tests or the product; the tests only read the
``.npz`` files this script writes next to itself.  What runs:

* ``reference_position_scores`` + ``reference_merge_accepted_positions``
  (``vendor/sglang/python/sglang/srt/speculative/global16_raw256_incremental.py``,
  loaded by file path because the ``sglang`` package ``__init__`` needs
  ``orjson``) chained over steps, following the reference's own GPU test
  protocol (``tests/gpu/test_gqa5_attention.py:20-50``: seed 980426, random
  bf16 queries/keys/values, random initial state, permuted pool slots, accept
  lengths ``(arange(B) + step) % V + 1``).  The module's row-count constants are
  widened for the benchmark shapes (S=64/256, V=16); the functions read them at
  call time, so the reference code runs unchanged.
* ``DraftFreeKVModel._forward_global16_raw256`` (paged branch) +
  ``sample_parallel_tokens`` (``vendor/specforge/modeling/draft/draftfreekv.py``)
  with a paged ``attend`` context written in terms of the reference's own
  ``attention_statistics_from_4d`` and ``merge_normalized_attention``, mirroring
  ``Global16Raw256PagedDraftContext.attend``'s PyTorch path
  (``vendor/sglang/python/sglang/srt/speculative/global16_raw256.py:1598-1638``,
  the FA3 window source replaced by the same statistics function).
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch
from torch import nn

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("LONGSPARK_REFERENCE", "/root/reference"))
sys.path.insert(0, str(REF / "vendor"))
sys.path.insert(0, str(HERE.parents[1]))

from specforge.modeling.draft import DraftFreeKVConfig, DraftFreeKVModel  # noqa: E402
from specforge.modeling.draft.global16_raw256 import (  # noqa: E402
    attention_statistics_from_4d, merge_normalized_attention)

from longspark_b200.config import DraftShape  # noqa: E402
from longspark_b200.synthetic import make_views, make_weights, rope_inv_freq  # noqa: E402


def load_incremental():
    path = REF / "vendor/sglang/python/sglang/srt/speculative/global16_raw256_incremental.py"
    spec = importlib.util.spec_from_file_location("ls_ref_incremental", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def bits(t):
    """bf16 tensor -> uint16 numpy bit pattern."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


# --------------------------------------------------------------------------
# Refresh (incremental summary) fixtures
# --------------------------------------------------------------------------

def refresh_fixture(name, *, q_heads, kv_heads, slots, verify_rows, batches, steps, seed=980426):
    inc = load_incremental()
    inc.GLOBAL_ROWS = slots
    inc.VERIFY_ROWS = verify_rows
    torch.manual_seed(seed)
    out = {}
    for batch in batches:
        query = torch.randn(1, q_heads, slots, 128, dtype=torch.bfloat16)
        capacity = batch + 3
        output = torch.randn(capacity, q_heads, slots, 128)
        lse = torch.randn(capacity, q_heads, slots)
        slot_ids = torch.randperm(capacity)[:batch].to(torch.int32)
        st_out, st_lse = output[slot_ids].clone(), lse[slot_ids].clone()
        keys_all, vals_all, lens_all, first_scores = [], [], [], None
        for step in range(steps):
            keys = torch.randn(batch, verify_rows, kv_heads, 128, dtype=torch.bfloat16)
            values = torch.randn_like(keys)
            scores = inc.reference_position_scores(global_query=query.expand(batch, -1, -1, -1),
                                                   new_keys=keys, softmax_scale=128 ** -0.5)
            if first_scores is None:
                first_scores = scores.numpy()
            lens = ((torch.arange(batch) + step) % verify_rows + 1).to(torch.int32)
            st_out, st_lse = inc.reference_merge_accepted_positions(
                state_output=st_out, state_lse=st_lse, position_scores=scores,
                accepted_values=values, accept_lens=lens)
            keys_all.append(bits(keys)); vals_all.append(bits(values)); lens_all.append(lens.numpy())
        p = f"b{batch}_"
        out.update({p + "query": bits(query[0]), p + "output0": output[slot_ids].numpy(),
                    p + "lse0": lse[slot_ids].numpy(),
                    p + "slots": slot_ids.numpy(), p + "keys": np.stack(keys_all),
                    p + "values": np.stack(vals_all), p + "lens": np.stack(lens_all),
                    p + "scores0": first_scores, p + "final_output": st_out.numpy(),
                    p + "final_lse": st_lse.numpy()})
    out["meta"] = np.array([q_heads, kv_heads, slots, verify_rows, steps] + list(batches))
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print("wrote", name)


# --------------------------------------------------------------------------
# Drafter pass fixtures
# --------------------------------------------------------------------------

class FinalNorm(nn.Module):
    """Stand-in for the target's SGLang RMSNorm: a weight plus ``variance_epsilon``,
    which routes ``_prepare_logits_hidden`` to ``F.rms_norm`` as in serving."""

    def __init__(self, weight, eps):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.variance_epsilon = eps


class PagedViews:
    """A paged ``attend`` context over per-tapped-layer pools (page size 16)."""

    def __init__(self, qg, summary_out, kv_k, kv_v, table, seq_lens, window, batch):
        self.qg, self.summary_out = qg, summary_out
        self.kv_k, self.kv_v, self.table, self.seq_lens = kv_k, kv_v, table, seq_lens
        self.window = window
        self.cuda_graph_static_inputs = False
        self.position_ids_are_scheduler_owned = True
        self.batch = batch

    def _window(self, pool, layer):
        rows, lens = [], []
        for b in range(self.batch):
            n = min(int(self.seq_lens[b]), self.window)
            pos = torch.arange(int(self.seq_lens[b]) - n, int(self.seq_lens[b]))
            r = pool[layer][self.table[b, pos // 16].long(), pos % 16]  # [n, Hkv, D]
            pad = torch.zeros((self.window - n,) + r.shape[1:], dtype=r.dtype)
            rows.append(torch.cat([r, pad]).transpose(0, 1))
            lens.append(n)
        return torch.stack(rows), torch.tensor(lens)

    def attend(self, *, layer_index, query, local_keys, local_values, local_attention_mask):
        b, hq, p, d = query.shape
        gk = self.qg[layer_index][None].expand(b, -1, -1, -1).to(query.dtype)
        gv = self.summary_out[:, layer_index].to(query.dtype)
        gmask = torch.ones(b, p, gk.shape[2], dtype=torch.bool)
        g = attention_statistics_from_4d(query=query, keys=gk, values=gv, attention_mask=gmask)
        wk, lens = self._window(self.kv_k, layer_index)
        wv, _ = self._window(self.kv_v, layer_index)
        wmask = (torch.arange(self.window)[None, :] < lens[:, None])[:, None, :].expand(b, p, -1)
        w = attention_statistics_from_4d(query=query, keys=wk.to(query.dtype), values=wv.to(query.dtype),
                                         attention_mask=wmask.contiguous())
        loc = attention_statistics_from_4d(query=query, keys=local_keys, values=local_values,
                                           attention_mask=local_attention_mask)

        def norm(st):
            visible = st.normalizer > 0
            safe = st.normalizer.clamp_min(torch.finfo(st.normalizer.dtype).tiny)
            lse = torch.where(visible, st.max_logits + torch.log(safe), torch.full_like(safe, float("-inf")))
            return st.output(), lse

        merged, _ = merge_normalized_attention((norm(g), norm(w), norm(loc)))
        return merged.to(dtype=query.dtype)


def reference_model(shape: DraftShape, W, dtype):
    """The reference drafter (``DraftFreeKVModel``, parallel_shifted_qwen +
    Global16/Raw256) loaded with the reference-named weights ``W``, plus the
    three target modules the pass uses (embedding, LM head, final norm)."""
    cfg = DraftFreeKVConfig(
        target_layer_ids=list(range(shape.tap_layers)), num_target_layers=max(8, shape.tap_layers + 1),
        block_size=7, hidden_size=shape.hidden, num_key_value_heads=shape.kv_heads, head_dim=128,
        vocab_size=shape.vocab, draft_mode="parallel_shifted_qwen", mask_token_id=shape.mask_token_id,
        parallel_mixer_layers=shape.draft_layers, parallel_markov_rank=shape.markov_rank,
        qwen_intermediate_size=shape.inter, qwen_num_attention_heads=shape.q_heads,
        qwen_rope_theta=shape.rope_theta, qwen_rms_norm_eps=shape.rms_eps,
        global16_raw256_enabled=True)
    model = DraftFreeKVModel(cfg).eval()
    sd = model.state_dict()
    for k in list(sd):
        if k in W and W[k].shape == sd[k].shape:
            sd[k] = W[k].to(torch.float32)
    model.load_state_dict(sd)
    model = model.to(dtype)
    for j in range(shape.draft_layers):  # non-persistent buffer: restore the fp32 RoPE table
        model.parallel_qwen_layers[j].self_attn.inv_freq = rope_inv_freq(shape)
    emb = nn.Embedding.from_pretrained(W["model.embed_tokens.weight"].to(dtype), freeze=True)
    head = nn.Linear(shape.hidden, shape.vocab, bias=False)
    head.weight = nn.Parameter(W["lm_head.weight"].to(dtype), requires_grad=False)
    fnorm = FinalNorm(W["model.norm.weight"].to(dtype), shape.final_eps)
    return model, emb, head, fnorm


def draft_fixture(name, shape: DraftShape, *, contexts, seed, dtype, store_weights=True,
                  norm_jitter=0.05, store_logits=True):
    assert shape.block == 7, "the reference drafter pass is fixed to Local7"
    batch = len(contexts)
    W = make_weights(shape, seed=seed, norm_jitter=norm_jitter)
    model, emb, head, fnorm = reference_model(shape, W, dtype)

    v = make_views(shape, batch, list(contexts), seed=seed + 1, pool_pages=None, extra_rows=0)
    kv_k, kv_v, table, seq_lens = v["kv_k"], v["kv_v"], v["page_table"], v["seq_lens"]
    hidden, anchors, summary_out = v["hidden"], v["anchors"], v["summary_out"]
    qg = W["global16_raw256_reference.global_query_generator.learned_query"]

    views = PagedViews(qg.to(dtype), summary_out, kv_k.to(dtype), kv_v.to(dtype), table, seq_lens,
                       shape.window, batch)
    with torch.no_grad():
        base = model._forward_global16_raw256(
            keys=None, values=None, attention_mask=None, kv_source_indices=None,
            anchor_attention_mask=None, current_hidden_states=hidden.to(dtype),
            current_token_ids=anchors, current_position_ids=seq_lens.long(),
            teacher_forcing_token_ids=None, target_final_norm=fnorm, target_embed_tokens=emb,
            target_lm_head=head, candidate_token_ids=None, apply_markov_correction=False,
            global16_paged_context=views)
        # Serving keeps base logits in the model dtype before the Markov chain
        # (``install_bfloat16_markov_projection``); F.linear already rounded them.
        base = base.to(dtype)
        tokens, corrected = model.sample_parallel_tokens(base, first_previous_token_ids=anchors,
                                                         temperature=0.0)
    out = dict(seed=np.array(seed), contexts=np.array(contexts), dtype=np.array(str(dtype)),
               tokens=tokens.numpy(),
               shape=np.array([shape.hidden, shape.q_heads, shape.kv_heads, shape.inter, shape.vocab,
                               shape.tap_layers, shape.draft_layers, shape.slots, shape.window,
                               shape.block, shape.markov_rank, shape.mask_token_id]),
               norm_jitter=np.array(norm_jitter))
    if store_logits:
        out["base_logits"] = base.float().numpy() if dtype == torch.float32 else bits(base)
        out["corrected"] = corrected.float().numpy() if dtype == torch.float32 else bits(corrected)
    else:
        # Large vocabularies: keep the top-32 of every row and the row max.
        bf = base.float()
        top = torch.topk(bf, 32, dim=-1)
        out["base_top_values"] = top.values.numpy()
        out["base_top_ids"] = top.indices.numpy()
        cf = corrected.float()
        ctop = torch.topk(cf, 32, dim=-1)
        out["corrected_top_values"] = ctop.values.numpy()
        out["corrected_top_ids"] = ctop.indices.numpy()
    if store_weights:
        # Small fixtures carry their inputs (once per seed, shared by the fp32 and
        # bf16 outputs); large ones are regenerated from the seeds.
        inputs = {"w::" + k: bits(t) for k, t in W.items()}
        inputs.update(kv_k=bits(kv_k), kv_v=bits(kv_v), table=table.numpy(), hidden=bits(hidden),
                      anchors=anchors.numpy(), summary_out=summary_out.numpy(), seq_lens=seq_lens.numpy())
        np.savez_compressed(HERE / f"{name.rsplit('_', 1)[0]}_inputs.npz", **inputs)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print("wrote", name, "tokens", tokens.tolist())


def chain_fixture(name, shape: DraftShape, *, ctx0, rounds, seed, topk=4):
    """A chained run of the reference: every round folds that round's committed
    rows into the fp32 summary (``reference_position_scores`` +
    ``reference_merge_accepted_positions`` per tapped layer), then runs the
    drafter pass on the refreshed views in bf16 and in fp32 and the greedy
    Markov chain of the bf16 pass.  Inputs come from ``chain_inputs`` (seeds
    ``seed`` and ``seed + 1``); the fixture keeps per round the bf16 tokens,
    the top-``topk`` (value, id) pairs of the bf16 corrected and base logits
    and of the fp32 base logits, and the summary lse after the first and the
    last round."""
    from chain_inputs import chain_views, chain_weights, committed_rows

    assert shape.block == 7, "the reference drafter pass is fixed to Local7"
    inc = load_incremental()
    inc.GLOBAL_ROWS = shape.slots
    inc.VERIFY_ROWS = shape.max_commit
    W = chain_weights(shape, seed)
    v = chain_views(shape, ctx0, rounds, seed + 1)
    m16 = reference_model(shape, W, torch.bfloat16)
    m32 = reference_model(shape, W, torch.float32)
    qg = W["global16_raw256_reference.global_query_generator.learned_query"]  # [L, Hq, S, D] bf16
    out, lse = v["summary_out"].clone(), v["summary_lse"].clone()
    L = shape.tap_layers
    rec = {k: [] for k in ("tokens", "corr_vals", "corr_ids", "base_vals", "base_ids", "base32_vals",
                           "base32_ids")}
    lse_first = None
    for t in range(rounds):
        c, n = int(v["commits"][t]), int(v["lengths"][t])
        nk = committed_rows(v["kv_k"], v["page_table"], n, c, shape.max_commit)
        nv = committed_rows(v["kv_v"], v["page_table"], n, c, shape.max_commit)
        for layer in range(L):
            sc = inc.reference_position_scores(global_query=qg[layer][None], new_keys=nk[layer],
                                               softmax_scale=128 ** -0.5)
            o, s_ = inc.reference_merge_accepted_positions(
                state_output=out[:, layer].contiguous(), state_lse=lse[:, layer].contiguous(), position_scores=sc,
                accepted_values=nv[layer], accept_lens=torch.tensor([c], dtype=torch.int32))
            out[:, layer], lse[:, layer] = o, s_
        if lse_first is None:
            lse_first = lse.clone()
        lens = torch.tensor([n], dtype=torch.int32)
        anchors = v["anchors"][t:t + 1]
        for dtype, (model, emb, head, fnorm) in ((torch.bfloat16, m16), (torch.float32, m32)):
            views = PagedViews(qg.to(dtype), out, v["kv_k"].to(dtype), v["kv_v"].to(dtype), v["page_table"], lens,
                               shape.window, 1)
            with torch.no_grad():
                base = model._forward_global16_raw256(
                    keys=None, values=None, attention_mask=None, kv_source_indices=None,
                    anchor_attention_mask=None, current_hidden_states=v["hidden"][t].to(dtype),
                    current_token_ids=anchors, current_position_ids=lens.long(),
                    teacher_forcing_token_ids=None, target_final_norm=fnorm, target_embed_tokens=emb,
                    target_lm_head=head, candidate_token_ids=None, apply_markov_correction=False,
                    global16_paged_context=views).to(dtype)
                if dtype == torch.bfloat16:
                    tokens, corrected = model.sample_parallel_tokens(base, first_previous_token_ids=anchors,
                                                                     temperature=0.0)
                    ct = torch.topk(corrected.float(), topk, dim=-1)
                    bt = torch.topk(base.float(), topk, dim=-1)
                    rec["tokens"].append(tokens[0].numpy())
                    rec["corr_vals"].append(ct.values[0].numpy())
                    rec["corr_ids"].append(ct.indices[0].numpy())
                    rec["base_vals"].append(bt.values[0].numpy())
                    rec["base_ids"].append(bt.indices[0].numpy())
                else:
                    bt = torch.topk(base.float(), topk, dim=-1)
                    rec["base32_vals"].append(bt.values[0].numpy())
                    rec["base32_ids"].append(bt.indices[0].numpy())
        if t % 20 == 0:
            print(name, "round", t, "tokens", rec["tokens"][-1].tolist(), flush=True)
    fix = {k: np.stack(x) for k, x in rec.items()}
    fix.update(seed=np.array(seed), ctx0=np.array(ctx0), rounds=np.array(rounds),
               shape=np.array([shape.hidden, shape.q_heads, shape.kv_heads, shape.inter, shape.vocab,
                               shape.tap_layers, shape.draft_layers, shape.slots, shape.window,
                               shape.block, shape.markov_rank, shape.mask_token_id]),
               lse_first=lse_first.numpy(), lse_last=lse.numpy())
    np.savez_compressed(HERE / f"{name}.npz", **fix)
    print("wrote", name)


def load_sampling():
    """``src/longspark/engine/sampling.py`` by file path (it imports torch only)."""
    path = REF / "src/longspark/engine/sampling.py"
    spec = importlib.util.spec_from_file_location("ls_ref_sampling", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def sampling_fixture(name="rejection_sampling"):
    """Two-phase rejection sampling of the reference (``decide_acceptance`` then
    ``finish_sampling`` with given uniforms, ``src/longspark/engine/
    sampling.py:19-57``) driven as the target does (``engine/target.py:478-491``,
    q rows from the drafter's corrected logits as at :613-614), on the inputs
    of ``sampling_inputs.CASES``; the proposal probabilities q are the
    reference drafter's (``engine/draft.py:284-286``).  Stores per case the
    candidates, q, uniforms, accept lengths and bonus tokens."""
    from sampling_inputs import CASES, sampling_draws, sampling_logits

    smp = load_sampling()
    out = {}
    for case, (batch, block, vocab, temp, seed, sd, sn, same) in CASES.items():
        target, draft = sampling_logits(batch, block, vocab, seed, sd, sn, same)
        cand, uniforms, final = sampling_draws(draft, temp, seed)
        cand_t = torch.from_numpy(cand)
        q = torch.softmax(draft.float() / temp, -1).gather(-1, cand_t[..., None]).squeeze(-1)
        # the requests whose target rows equal the drafter's claim q = 1: they
        # reject where u >= p, and the residual there has zero mass (the
        # reference's fallback to the target row)
        q[:same] = 1.0
        decision = smp.decide_acceptance(candidates=cand_t, sampled_q=q,
                                         target_probs=torch.softmax(target.float() / temp, -1),
                                         uniforms=torch.from_numpy(uniforms))
        rows = decision.rejected_rows
        q_rows = torch.softmax(draft[rows, decision.rejection_positions].float() / temp, -1)
        bonus = smp.finish_sampling(decision, q_rows, uniforms=torch.from_numpy(final))
        p = case + "_"
        out.update({p + "candidates": cand, p + "q": q.numpy(), p + "uniforms": uniforms, p + "final": final,
                    p + "lengths": decision.lengths.numpy(), p + "bonus": bonus.numpy()})
        print(case, "lengths", decision.lengths.tolist(), "bonus", bonus.tolist())
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print("wrote", name)


def main(which=("refresh", "draft", "chain", "sampling")):
    torch.set_num_threads(os.cpu_count() or 1)
    sys.path.insert(0, str(HERE))
    if "sampling" in which:
        sampling_fixture()
    if "chain" in which:
        base = dict(tap_layers=1, draft_layers=1, slots=256, block=7, max_commit=8)
        # Qwen3-14B dimensions (1 drafter layer, W=2048, S=256,
        # 128K context, 200 chained rounds) at the reference's Local7 block
        chain_fixture("chain_cfg3_p7", DraftShape(hidden=5120, q_heads=40, kv_heads=8, inter=17408, window=2048,
                                                  **base), ctx0=131072, rounds=200, seed=300)
        # Qwen3-8B dimensions (W=1024, S=256, 128K context)
        chain_fixture("chain_cfg2_p7", DraftShape(hidden=4096, q_heads=32, kv_heads=8, inter=12288, window=1024,
                                                  **base), ctx0=131072, rounds=8, seed=200)
    if "refresh" in which:
        refresh_fixtures()
    if "draft" in which:
        draft_fixtures()


def refresh_fixtures():
    refresh_fixture("refresh_gqa4_ref", q_heads=32, kv_heads=8, slots=16, verify_rows=8,
                    batches=(1, 2), steps=8)
    refresh_fixture("refresh_gqa5_ref", q_heads=40, kv_heads=8, slots=16, verify_rows=8,
                    batches=(1, 2), steps=8)
    refresh_fixture("refresh_gqa4_s64_v16", q_heads=16, kv_heads=4, slots=64, verify_rows=16,
                    batches=(1,), steps=6)


def draft_fixtures():
    small = DraftShape(hidden=256, q_heads=8, kv_heads=2, inter=512, vocab=1024, tap_layers=2,
                       draft_layers=2, slots=16, window=256, block=7, max_commit=8, markov_rank=64,
                       mask_token_id=1000)
    for dt, tag in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        draft_fixture(f"draft_small_ref_{tag}", small, contexts=(300, 100), seed=11, dtype=dt)
        draft_fixture(f"draft_small_gqa5_s64_w512_{tag}",
                      small.with_(q_heads=10, slots=64, window=512, tap_layers=1, draft_layers=1),
                      contexts=(700, 37), seed=12, dtype=dt)
    cfg1 = DraftShape(hidden=2560, q_heads=32, kv_heads=8, inter=9728, tap_layers=1, draft_layers=1,
                      slots=64, window=512, block=7, max_commit=8)
    for dt, tag in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        draft_fixture(f"draft_cfg1_p7_{tag}", cfg1, contexts=(4096,), seed=0, dtype=dt,
                      store_weights=False, norm_jitter=0.0, store_logits=False)


if __name__ == "__main__":
    main(tuple(sys.argv[1:]) or ("refresh", "draft", "chain", "sampling"))
