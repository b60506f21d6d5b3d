"""numpy restatement of LongSpark's per-round drafting path (test oracle only).

Every function names the reference lines it follows.  Paths are relative to the
LongSpark project root; abbreviations:

* ``SF`` = ``vendor/specforge/modeling/draft/``
* ``SP`` = ``vendor/sglang/python/sglang/srt/speculative/``
* ``LS`` = ``src/longspark/``

Precision.  ``prec="bf16"`` reproduces the rounding points of the reference
drafter run in bfloat16 (the serving dtype): every ``nn.Linear`` output,
activation, residual sum and normalisation result is rounded to bf16 where the
PyTorch reference rounds it, while reductions accumulate in fp32.
``prec="fp32"`` turns every rounding point into the identity, which is the
reference model run in float32.  Arrays are float32 throughout; in bf16 mode
they only ever hold bf16-representable values.

Shapes follow the reference: B requests, P drafter rows (``block_size``), Hq
query heads, Hkv KV heads, D head dim, S summary slots, W window rows, V
committed rows per round at most.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

__all__ = [
    "bf16_round", "bf16_bits", "from_bf16_bits", "rnd",
    "linear", "row_parallel_linear", "silu", "rmsnorm_hf", "rmsnorm_fused", "feed_forward",
    "state_encoder", "shifted_input", "rope_tables", "apply_rotary",
    "attention_statistics", "statistics_as_normalized", "merge_normalized_attention",
    "window_positions", "gather_window", "export_rows", "attend", "decoder_layer", "project_logits",
    "markov_sample", "markov_sample_gumbel", "gumbel_hash_uniform", "greedy_argmax", "accept_lengths",
    "softmax_t", "rejection_sample", "position_scores", "merge_accepted",
    "full_prefix_state", "refresh_views", "draft_pass", "build_views", "DraftShapeOracle",
]


# ----------------------------------------------------------------------------
# bf16 emulation
# ----------------------------------------------------------------------------

def bf16_round(x):
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    out = r.view(np.float32).reshape(x.shape)
    return np.where(np.isnan(x), x, out)


def bf16_bits(x):
    """bfloat16 bit pattern (uint16) of float32 values (rounded to nearest even)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits):
    """float32 values of a uint16 bfloat16 bit-pattern array."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def rnd(x, prec):
    return bf16_round(x) if prec == "bf16" else np.asarray(x, dtype=np.float32)


# ----------------------------------------------------------------------------
# Dense building blocks
# ----------------------------------------------------------------------------

def linear(x, w, prec):
    """``nn.Linear`` without bias: fp32 accumulation, output in the model dtype."""
    return rnd(np.matmul(x, w.T, dtype=np.float32), prec)


def row_parallel_linear(x, w, prec, tp=None):
    """A row-parallel ``nn.Linear`` over ``tp = (world, wire)`` ranks: rank r
    holds the k-slice ``[r*K/world, (r+1)*K/world)`` of the input features and
    of ``w``; each rank's fp32 partial crosses the wire as fp32
    (``wire == "f32"``) or rounded to bf16 (``"bf16"``, what a bf16
    RowParallelLinear + bf16 allreduce does: SGLang
    ``srt/layers/linear.py`` RowParallelLinear, reduce_results), and the
    partials are added in rank order in fp32 before the output rounding.
    ``tp=None`` or world 1 is ``linear``.  The drafter itself has no tensor
    parallelism in the reference (forced TP1,
    SP global16_native_draft_executor.py:1101-1105): this is the split the
    tensor-parallel kernels implement, restated for their parity tests."""
    if tp is None or tp[0] == 1:
        return linear(x, w, prec)
    world, wire = tp
    k = w.shape[1]
    ks = k // world
    acc = None
    for r in range(world):
        part = np.matmul(x[..., r * ks:(r + 1) * ks], w[:, r * ks:(r + 1) * ks].T, dtype=np.float32)
        if wire == "bf16":
            part = bf16_round(part)
        acc = part if acc is None else (acc + part).astype(np.float32)
    return rnd(acc, prec)


def silu(x, prec):
    """``F.silu`` (computed in fp32, rounded once to the input dtype)."""
    x = np.asarray(x, dtype=np.float32)
    return rnd(x / (np.float32(1.0) + np.exp(-x)), prec)


def rmsnorm_hf(x, w, eps, prec):
    """SpecForge ``RMSNorm`` (SF draftfreekv.py:1518-1530); the SGLang
    ``RMSNorm(cast_x_before_out_mul=True)`` the serving path swaps in
    (SP draft_free_kv_runner.py:20-65, ``srt/layers/layernorm.py:454-500``) has the
    same rounding: normalise in fp32, round, multiply by the weight in bf16."""
    x = np.asarray(x, dtype=np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    normalized = rnd(x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))), prec)
    return rnd(normalized * w, prec)


def rmsnorm_fused(x, w, eps, prec):
    """``F.rms_norm`` as used on the target final norm by ``_prepare_logits_hidden``
    (SF draftfreekv.py:3607-3647): one rounding of ``x * rstd * w``."""
    x = np.asarray(x, dtype=np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return rnd(x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))) * w, prec)


def feed_forward(x, w1, w2, prec, tp=None):
    """``FeedForward`` = Linear -> SiLU -> Linear (SF draftfreekv.py:1498-1516);
    under ``tp`` the second Linear is row-parallel (``row_parallel_linear``)."""
    return row_parallel_linear(silu(linear(x, w1, prec), prec), w2, prec, tp)


def state_encoder(hidden, W, prec, eps=1e-6, tp=None):
    """``DraftStateEncoder.forward`` (SF draftfreekv.py:1533-1540).

    hidden: [B, L_tap, H] -> [B, H]."""
    b = hidden.shape[0]
    x = hidden.reshape(b, -1)
    y = feed_forward(x, W["draft_state_encoder.proj.net.0.weight"],
                     W["draft_state_encoder.proj.net.2.weight"], prec, tp)
    return rmsnorm_hf(y, W["draft_state_encoder.norm.weight"], eps, prec)


def shifted_input(anchors, latest, W, block, mask_token_id, prec, eps=1e-6, tp=None):
    """``ParallelShiftedInput.forward`` (SF draftfreekv.py:1658-1739).

    Token layout ``[x_t, MASK, ...]`` embedded with the target embedding, plus
    the learned position embedding (bf16 add), concatenated with the latest
    state, FeedForward(2H -> H -> H), RMSNorm.  Returns [B, P, H]."""
    b = anchors.shape[0]
    emb = W["model.embed_tokens.weight"]
    ids = np.full((b, block), mask_token_id, dtype=np.int64)
    ids[:, 0] = anchors
    tok = emb[ids]
    tok = rnd(tok + W["parallel_shifted_input.position_embedding.weight"][None, :block], prec)
    lat = np.broadcast_to(latest[:, None, :], tok.shape)
    x = np.concatenate([tok, lat], axis=-1)
    y = feed_forward(x, W["parallel_shifted_input.proj.net.0.weight"],
                     W["parallel_shifted_input.proj.net.2.weight"], prec, tp)
    return rmsnorm_hf(y, W["parallel_shifted_input.norm.weight"], eps, prec)


def rope_tables(positions, inv_freq, prec):
    """``_position_embeddings`` (SF draftfreekv.py:1996-2007): fp32 phase,
    cos/sin cast to the model dtype.  positions [B, P] -> cos, sin [B, P, D]."""
    f = positions.astype(np.float32)[..., None] * inv_freq.astype(np.float32)[None, None, :]
    e = np.concatenate([f, f], axis=-1)
    return rnd(np.cos(e), prec), rnd(np.sin(e), prec)


def apply_rotary(x, cos, sin, prec):
    """``_apply_rotary`` (SF draftfreekv.py:2009-2017) with ``_rotate_half``
    (:1887-1889).  x [B, H, P, D]; cos/sin [B, P, D].  Each bf16 product and the
    sum are rounded, as the elementwise bf16 ops of the reference are."""
    c = cos[:, None]
    s = sin[:, None]
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return rnd(rnd(x * c, prec) + rnd(rot * s, prec), prec)


# ----------------------------------------------------------------------------
# Attention statistics (online-softmax algebra)
# ----------------------------------------------------------------------------

def attention_statistics(q, k, v, mask, prec):
    """``_attention_statistics`` (SF global16_raw256.py:445-539) for one layer
    (``attention_statistics_from_4d``, :361-393).

    q [B, Hq, R, D]; k, v [B, Hk, T, D] (Hq % Hk == 0, consecutive query heads
    share a KV head); mask [B, R, T] bool.  Returns (max_logits, normalizer,
    weighted_values) with shapes [B, Hq, R], [B, Hq, R], [B, Hq, R, D].

    In bf16 mode the scores einsum and the weights-by-values einsum produce
    bf16 outputs (fp32 accumulation), as torch bf16 einsum does."""
    b, hq, r, d = q.shape
    hk, t = k.shape[1], k.shape[2]
    g = hq // hk
    qg = q.reshape(b, hk, g, r, d)
    scores = rnd(np.einsum("bhgrd,bhtd->bhgrt", qg, k, dtype=np.float32), prec)
    scores = (scores * np.float32(d ** -0.5)).reshape(b, hq, r, t)
    m4 = mask[:, None, :, :]
    visible = mask.any(axis=-1)[:, None, :]
    masked = np.where(m4, scores, -np.inf)
    mx = masked.max(axis=-1)
    safe = np.where(visible, mx, 0.0).astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        w = np.exp(scores - safe[..., None])
    w = np.where(m4, w, 0.0).astype(np.float32)
    normalizer = w.sum(axis=-1, dtype=np.float32)
    wg = rnd(w, prec).reshape(b, hk, g, r, t)
    wv = rnd(np.einsum("bhgrt,bhtd->bhgrd", wg, v, dtype=np.float32), prec).reshape(b, hq, r, d)
    return np.where(visible, mx, 0.0).astype(np.float32), normalizer, wv.astype(np.float32)


def statistics_as_normalized(stats):
    """``_statistics_as_normalized`` (SP global16_raw256.py:196-203) with
    ``AttentionStatistics.output`` (SF global16_raw256.py:349-358)."""
    mx, norm, wv = stats
    tiny = np.finfo(np.float32).tiny
    safe = np.maximum(norm, tiny).astype(np.float32)
    lse = np.where(norm > 0, mx + np.log(safe), -np.inf).astype(np.float32)
    return (wv / safe[..., None]).astype(np.float32), lse


def merge_normalized_attention(parts):
    """``merge_normalized_attention`` (SF global16_raw256.py:396-442), fp32."""
    lses = np.stack([lse for _, lse in parts]).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        mx = lses.max(axis=0)
        mxs = np.where(np.isfinite(mx), mx, 0.0)
        merged = (mxs + np.log(np.exp(lses - mxs).sum(axis=0))).astype(np.float32)
    safe = np.where(np.isfinite(merged), merged, 0.0).astype(np.float32)
    out = np.zeros_like(parts[0][0], dtype=np.float32)
    for o, lse in parts:
        with np.errstate(invalid="ignore", over="ignore"):
            c = np.where(np.isfinite(lse), np.exp(lse - safe), 0.0).astype(np.float32)
        out = out + c[..., None] * o
    return out.astype(np.float32), merged


# ----------------------------------------------------------------------------
# Window (recent K/V rows) through a paged cache
# ----------------------------------------------------------------------------

def window_positions(length, window):
    """Chronological positions of the recent window: the last ``min(len, W)``
    committed positions (``ring_page_table``, LS engine/draft.py:14-21;
    ``_build_raw256_page_table``, SP global16_raw256.py:1307-1361)."""
    n = min(int(length), int(window))
    return np.arange(int(length) - n, int(length), dtype=np.int64)


def gather_window(pool, page_table_row, length, window, page_size, ring_pages=0):
    """Rows of one tapped layer's paged pool [pages, page, Hkv, D] at the window
    positions.  Physical row of position p = ``table[p // page] * page + p % page``
    (the page-size-16 statement of ``_build_raw256_page_table_kernel``,
    SP global16_raw256_draft_fused.py:35-65); with ``ring_pages > 0`` the logical
    page is taken modulo the ring (the drafter-owned ring of LS engine/draft.py:98,257).
    Returns [Hkv, n, D]."""
    pos = window_positions(length, window)
    lp = pos // page_size
    if ring_pages:
        lp = lp % ring_pages
    pages = page_table_row[lp]
    rows = pool[pages, pos % page_size]  # [n, Hkv, D]
    return np.ascontiguousarray(rows.transpose(1, 0, 2))


def export_rows(pool_k, pool_v, src_k, src_v, locations, counts, seq_lens, page_table, ring_pages=0,
                head_offset=0, page_size=16):
    """The target-side export restated: the target gathers ``k[locations]`` /
    ``v[locations]`` per tapped layer (``TargetModel._kv_rows``, LS
    engine/target.py:213-228; ``gather_selected_kv``, LS engine/state_export.py:
    14-47) and the drafter stores row i of request b at position
    ``seq_lens[b] - counts[b] + i`` of its window (``LongSparkDraft.update``,
    LS engine/draft.py:207-212, 257-260), here through the paged table as in
    ``gather_window``.  pool_k/pool_v [L, pages, page, H, D] (updated in place,
    heads [head_offset, head_offset + h)); src_k/src_v [L, rows, h, D];
    locations request-major."""
    off = 0
    for b, c in enumerate(counts):
        for i in range(int(c)):
            pos = int(seq_lens[b]) - int(c) + i
            lp = pos // page_size
            if ring_pages:
                lp %= ring_pages
            page = int(page_table[b][lp])
            src = int(locations[off + i])
            h = src_k.shape[2]
            pool_k[:, page, pos % page_size, head_offset:head_offset + h] = src_k[:, src]
            pool_v[:, page, pos % page_size, head_offset:head_offset + h] = src_v[:, src]
        off += int(c)
    return pool_k, pool_v


def attend(q, k_loc, v_loc, qg, summary_out, win_k, win_v, win_len, prec):
    """``Global16Raw256PagedDraftContext.attend`` in its PyTorch form
    (SP global16_raw256.py:1598-1638): three sources, each reduced by
    ``attention_statistics_from_4d`` and merged by ``merge_normalized_attention``.

    q [B, Hq, P, D]; k_loc, v_loc [B, Hkv, P, D] (local rows, all-visible mask,
    SP global16_raw256.py:1407-1411); qg [Hq, S, D] learned summary queries
    (keys of the global source, one per query head); summary_out [B, Hq, S, D]
    fp32 (values, cast to the model dtype); win_k, win_v [B, Hkv, Wmax, D] with
    ``win_len[b]`` valid rows.  Returns [B, Hq, P, D] in the model dtype."""
    b, hq, p, d = q.shape
    s = qg.shape[1]
    gkeys = np.broadcast_to(qg[None], (b,) + qg.shape)
    gvals = rnd(summary_out, prec)
    gmask = np.ones((b, p, s), dtype=bool)
    g_out, g_lse = statistics_as_normalized(attention_statistics(q, gkeys, gvals, gmask, prec))
    wmax = win_k.shape[2]
    wmask = np.broadcast_to((np.arange(wmax)[None, :] < np.asarray(win_len)[:, None])[:, None, :], (b, p, wmax))
    w_out, w_lse = statistics_as_normalized(attention_statistics(q, win_k, win_v, wmask, prec))
    lmask = np.ones((b, p, p), dtype=bool)
    l_out, l_lse = statistics_as_normalized(attention_statistics(q, k_loc, v_loc, lmask, prec))
    merged, _ = merge_normalized_attention([(g_out, g_lse), (w_out, w_lse), (l_out, l_lse)])
    return rnd(merged, prec)


# ----------------------------------------------------------------------------
# Decoder layer, logits, sampling
# ----------------------------------------------------------------------------

def decoder_layer(h, cos, sin, Wl, view, shape, prec, tp=None):
    """One drafter decoder layer.

    ``Qwen3KVFreeParallelDecoderLayer.forward_global16_raw256`` (SF
    draftfreekv.py:2292-2308) with its attention
    ``Qwen3KVFreeParallelAttention.forward_global16_raw256`` (:2096-2173) and
    MLP ``Qwen3SwiGLUMLP`` (:1871-1884): ``F.silu(gate)`` is rounded to bf16,
    then multiplied by ``up`` and rounded again.  (The SGLang serving executor's
    fused ``SiluAndMul``, SP global16_native_draft_executor.py:628-633, rounds once
    instead; this restatement follows the PyTorch drafter it is pinned against.)

    h [B, P, H]; view = dict(qg, summary_out, win_k, win_v, win_len).  Under
    ``tp`` the o_proj and down_proj are row-parallel (``row_parallel_linear``);
    head-parallel attention and column-parallel projections compute the same
    values as one GPU."""
    b, p, hdim = h.shape
    hq, hkv, d = shape.q_heads, shape.kv_heads, shape.head_dim
    eps = shape.rms_eps
    x = rmsnorm_hf(h, Wl["input_layernorm.weight"], eps, prec)
    q = linear(x, Wl["self_attn.q_proj.weight"], prec).reshape(b, p, hq, d)
    k = linear(x, Wl["self_attn.k_proj.weight"], prec).reshape(b, p, hkv, d)
    v = linear(x, Wl["self_attn.v_proj.weight"], prec).reshape(b, p, hkv, d)
    q = rmsnorm_hf(q, Wl["self_attn.q_norm.weight"], eps, prec).transpose(0, 2, 1, 3)
    k = rmsnorm_hf(k, Wl["self_attn.k_norm.weight"], eps, prec).transpose(0, 2, 1, 3)
    v = v.transpose(0, 2, 1, 3)
    q = apply_rotary(q, cos, sin, prec)
    k = apply_rotary(k, cos, sin, prec)
    a = attend(q, k, v, view["qg"], view["summary_out"], view["win_k"], view["win_v"],
               view["win_len"], prec)
    a = np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(b, p, hq * d)
    h = rnd(h + row_parallel_linear(a, Wl["self_attn.o_proj.weight"], prec, tp), prec)
    x = rmsnorm_hf(h, Wl["post_attention_layernorm.weight"], eps, prec)
    gate = linear(x, Wl["mlp.gate_proj.weight"], prec)
    up = linear(x, Wl["mlp.up_proj.weight"], prec)
    act = rnd(silu(gate, prec) * up, prec)
    return rnd(h + row_parallel_linear(act, Wl["mlp.down_proj.weight"], prec, tp), prec)


def project_logits(h, W, final_eps, prec):
    """Target final norm + vocabulary projection: ``_prepare_logits_hidden``
    (SF draftfreekv.py:3607-3647, ``F.rms_norm``) then the bf16 projection
    installed by ``install_bfloat16_markov_projection`` (SP
    global16_markov_precision.py:71-136): logits stay in the model dtype."""
    x = rmsnorm_fused(h, W["model.norm.weight"], final_eps, prec)
    return linear(x, W["lm_head.weight"], prec)


def greedy_argmax(x):
    """``torch.argmax`` on the last axis: the first maximal index wins."""
    return np.argmax(x, axis=-1).astype(np.int64)


def markov_sample(base_logits, anchors, W, prec, forced=None):
    """Greedy ``DSparkVanillaMarkovHead.sample_block_tokens`` (SF
    draftfreekv.py:2366-2407): for each step, ``bias = w2(w1[prev])`` in the model
    dtype, ``step = base[:, t] + bias`` (rounded), ``tok = argmax(step)``, and the
    sampled token feeds the next step.  Without a Markov head
    (``parallel_markov_rank == 0``) this is ``base_logits.argmax(-1)``
    (``sample_parallel_tokens``, :3545-3578).

    ``forced`` ([B, P] tokens) feeds the given tokens back instead of the
    sampled ones, so a comparison can continue past a tie without diverging.
    Returns (tokens [B, P] int64, corrected logits [B, P, V])."""
    w1 = W.get("parallel_markov_head.markov_w1.weight")
    if w1 is None:
        return greedy_argmax(base_logits), base_logits
    w2 = W["parallel_markov_head.markov_w2.weight"]
    b, p, _ = base_logits.shape
    prev = np.asarray(anchors, dtype=np.int64)
    toks = np.zeros((b, p), dtype=np.int64)
    corrected = np.zeros_like(base_logits)
    for t in range(p):
        bias = linear(w1[prev], w2, prec)
        step = rnd(base_logits[:, t] + bias, prec)
        corrected[:, t] = step
        toks[:, t] = greedy_argmax(step)
        prev = toks[:, t] if forced is None else np.asarray(forced[:, t], dtype=np.int64)
    return toks, corrected


def gumbel_hash_uniform(seed, b, t, v):
    """Uniform in (0, 1) from a counter-based hash of (seed, request b, step t,
    token v): the random source of the tensor-core-free T > 0 sampler.  Two
    rounds of the lowbias32 integer mixer (C. Wellons) over a linear mix of the
    counters; 24 bits of the result, centred in their interval.  uint32
    arithmetic, identical to the CUDA side."""
    M = np.uint64(0xFFFFFFFF)
    s = np.uint64(seed)
    seed_lo = s & M
    seed_hi = (s >> np.uint64(32)) & M

    def mix(x):
        x = x & M
        x ^= x >> np.uint64(16)
        x = (x * np.uint64(0x7FEB352D)) & M
        x ^= x >> np.uint64(15)
        x = (x * np.uint64(0x846CA68B)) & M
        x ^= x >> np.uint64(16)
        return x

    v = np.asarray(v, dtype=np.uint64)
    x = ((v * np.uint64(0x9E3779B1)) & M) ^ ((np.uint64(t) * np.uint64(0x85EBCA77)) & M) \
        ^ ((np.uint64(b) * np.uint64(0xC2B2AE3D)) & M) ^ seed_lo
    x = mix(mix(x) ^ seed_hi)
    return (((x >> np.uint64(8)).astype(np.float64) + 0.5) * 2.0 ** -24).astype(np.float32)


def markov_sample_gumbel(base_logits, anchors, W, prec, temperature, seed, forced=None):
    """``DSparkVanillaMarkovHead.sample_block_tokens`` at T > 0 (SF
    draftfreekv.py:2366-2407) and the proposal probability of
    ``LongSparkDraft.propose`` (LS engine/draft.py:284-286): per step,
    ``step = bf16(base[t] + bf16(w2 . w1[prev]))``, a token drawn from
    ``softmax(step / T)`` feeds the next step, and ``q = softmax(step / T)[tok]``.
    The reference draws with ``torch.multinomial``; here the draw is the
    Gumbel-max of ``step / T + g`` with ``g = -log(-log(u))`` and ``u`` from
    ``gumbel_hash_uniform(seed, b, t, v)`` -- the same distribution, and a
    reproducible one.  ``forced`` ([B, P]) feeds the given tokens back as the
    previous tokens (to follow a chain past a near-tie).  Returns tokens
    [B, P] int64, q [B, P] fp32, corrected logits [B, P, V] and the gap
    between the two largest keys per step [B, P]."""
    w1 = W.get("parallel_markov_head.markov_w1.weight")
    w2 = W.get("parallel_markov_head.markov_w2.weight")
    b_n, p_n, vocab = base_logits.shape
    prev = np.asarray(anchors, dtype=np.int64).copy()
    toks = np.zeros((b_n, p_n), dtype=np.int64)
    q = np.zeros((b_n, p_n), dtype=np.float32)
    corrected = np.zeros_like(base_logits)
    temp = np.float32(temperature)
    ids = np.arange(vocab)
    gap = np.zeros((b_n, p_n), dtype=np.float32)
    for t in range(p_n):
        if w1 is None:
            step = base_logits[:, t]
        else:
            step = rnd(base_logits[:, t] + linear(w1[prev], w2, prec), prec)
        corrected[:, t] = step
        for b in range(b_n):
            z = (step[b].astype(np.float32) / temp).astype(np.float32)
            u = gumbel_hash_uniform(seed, b, t, ids)
            g = -np.log(-np.log(u))
            key = (z + g).astype(np.float32)
            tok = int(np.argmax(key))
            top2 = np.partition(key, -2)[-2:]
            gap[b, t] = top2[1] - top2[0]
            m = z.max()
            e = np.exp(z - m)
            q[b, t] = e[tok] / e.sum(dtype=np.float32)
            toks[b, t] = tok
        prev = toks[:, t].copy() if forced is None else np.asarray(forced[:, t], dtype=np.int64)
    return toks, q, corrected, gap


def accept_lengths(target_tokens, draft_tokens):
    """Greedy accept check (LS engine/target.py:472-477):
    ``accept = (target[:, :P] == draft).cumprod(1).sum(1)``; bonus token =
    ``target[accept]``; commit length = accept + 1."""
    t = np.asarray(target_tokens, dtype=np.int64)
    d = np.asarray(draft_tokens, dtype=np.int64)
    p = d.shape[1]
    acc = np.cumprod(t[:, :p] == d, axis=1).sum(axis=1).astype(np.int64)
    bonus = t[np.arange(t.shape[0]), acc] if t.shape[1] > p else None
    return acc, bonus


def softmax_t(logits, temperature):
    """``torch.softmax(logits.float() / T, -1)`` in float32 as torch computes it
    on the CPU: the scaled logits by IEEE division, their maximum subtracted,
    exponentials multiplied by the reciprocal of their sum."""
    z = np.asarray(logits, dtype=np.float32) / np.float32(temperature)
    e = np.exp(z - z.max(axis=-1, keepdims=True))
    return (e * (np.float32(1) / e.sum(axis=-1, keepdims=True, dtype=np.float32))).astype(np.float32)


def rejection_sample(target_logits, draft_logits, candidates, sampled_q, temperature, uniforms, final_uniforms):
    """Two-phase exact rejection sampling of a verified block at T > 0 (LS
    engine/sampling.py:19-57, driven from LS engine/target.py:478-491 and
    :613-614).

    Phase one, ``decide_acceptance``: with ``p = softmax(target / T)`` over the
    P + 1 verify rows, proposal t is accepted when ``u[t] * q[t] < p[t,
    cand[t]]``; the accept length is the number of leading accepted
    proposals.  Phase two, ``finish_sampling``: a request that rejected at
    position L draws its bonus token from the residual ``max(p[L] - q_row, 0)``
    renormalised (``q_row = softmax(draft[L] / T)``, the drafter's corrected
    logits; the target row itself when the residual mass is at most 1e-8); a
    request that accepted all P draws from ``p[P]``.  The draw is the
    reference's inverse CDF with the given final uniform:
    ``count(u >= cumsum(probs))`` clamped to V - 1, the cumulative sum taken in
    float64 and rounded to float32 as ``torch.cumsum`` does on the CPU.

    target_logits [B, P + 1, V], draft_logits [B, P, V] (any float dtype
    values), candidates [B, P] int, sampled_q, uniforms [B, P] float32,
    final_uniforms [B] float32.  Returns (lengths [B] int64, bonus [B] int64)."""
    tl = np.asarray(target_logits, dtype=np.float32)
    dl = np.asarray(draft_logits, dtype=np.float32)
    cand = np.asarray(candidates, dtype=np.int64)
    b_n, p_n = cand.shape
    vocab = tl.shape[-1]
    probs = softmax_t(tl, temperature)
    sel = np.take_along_axis(probs[:, :p_n], cand[..., None], axis=-1)[..., 0]
    accept = (np.asarray(uniforms, np.float32) * np.asarray(sampled_q, np.float32)) < sel
    lengths = np.cumprod(accept.astype(np.int64), axis=1).sum(axis=1)
    bonus = np.zeros(b_n, dtype=np.int64)
    for b in range(b_n):
        L = int(lengths[b])
        row = probs[b, L]
        if L < p_n:
            q_row = softmax_t(dl[b, L], temperature)
            residual = np.maximum(row - q_row, np.float32(0))
            mass = residual.sum(dtype=np.float32)
            if mass > np.float32(1e-8):
                row = residual / np.maximum(mass, np.float32(1e-30))
        cdf = np.cumsum(row.astype(np.float64)).astype(np.float32)
        bonus[b] = min(int((np.float32(final_uniforms[b]) >= cdf).sum()), vocab - 1)
    return lengths.astype(np.int64), bonus


# ----------------------------------------------------------------------------
# Summary state (view refresh)
# ----------------------------------------------------------------------------

def position_scores(global_query, new_keys, scale):
    """``reference_position_scores`` (SP global16_raw256_incremental.py:50-87),
    with the row count V as a parameter.  global_query [B, Hq, S, D];
    new_keys [B, V, Hkv, D] -> scores [B, Hq, S, V] fp32."""
    b, hq, s, d = global_query.shape
    hkv = new_keys.shape[2]
    g = hq // hkv
    q = global_query.astype(np.float32).reshape(b, hkv, g, s, d)
    k = new_keys.astype(np.float32).transpose(0, 2, 1, 3)
    sc = np.einsum("bhrgd,bhwd->bhrgw", q, k, dtype=np.float32) * np.float32(scale)
    return sc.reshape(b, hq, s, new_keys.shape[1]).astype(np.float32)


def merge_accepted(state_output, state_lse, scores, accepted_values, accept_lens):
    """``reference_merge_accepted_positions`` (SP
    global16_raw256_incremental.py:90-166): online-softmax merge of the first
    ``accept_lens[b]`` rows into the fp32 ``(output, lse)`` state.

    state_output [B, Hq, S, D]; state_lse [B, Hq, S]; scores [B, Hq, S, V];
    accepted_values [B, V, Hkv, D] (padded); accept_lens [B] in [1, V]."""
    b, hq, s, d = state_output.shape
    vrows = scores.shape[-1]
    acc = np.asarray(accept_lens)
    if np.any(acc < 1) or np.any(acc > vrows):
        raise ValueError("commit length must be between one and the verify width")
    valid = np.arange(vrows)[None, :] < acc[:, None]
    masked = np.where(valid[:, None, None, :], scores, -np.inf).astype(np.float32)
    dmax = masked.max(axis=-1)
    dlse = dmax + np.log(np.exp(masked - dmax[..., None]).sum(axis=-1))
    prior = state_lse.astype(np.float32)
    mx = np.maximum(prior, dlse)
    mxs = np.where(np.isfinite(mx), mx, 0.0)
    merged = (mxs + np.log(np.exp(prior - mxs) + np.exp(dlse - mxs))).astype(np.float32)
    prior_w = np.exp(prior - merged).astype(np.float32)
    delta_w = np.where(valid[:, None, None, :], np.exp(masked - merged[..., None]), 0.0).astype(np.float32)
    hkv = accepted_values.shape[2]
    g = hq // hkv
    wts = delta_w.reshape(b, hkv, g, s, vrows)
    vals = accepted_values.astype(np.float32).transpose(0, 2, 1, 3)
    delta = np.einsum("bhrgw,bhwd->bhrgd", wts, vals, dtype=np.float32).reshape(b, hq, s, d)
    out = state_output.astype(np.float32) * prior_w[..., None] + delta
    return out.astype(np.float32), merged


def full_prefix_state(query, keys, values, length, chunk=4096):
    """Full-prefix summary ``(output, lse)`` of the S learned queries over the
    first ``length`` rows, in fp32 (``global_state_from_full_prefix``, SF
    global16_raw256.py:829-869, key-chunked as ``_attention_statistics``
    :472-497; the serving prefill computes the same quantity with FA3,
    LS engine/target.py:230-253).

    query [Hq, S, D]; keys/values [T, Hkv, D]. Returns out [Hq, S, D], lse [Hq, S]."""
    hq, s, d = query.shape
    hkv = keys.shape[1]
    g = hq // hkv
    q = query.astype(np.float32).reshape(hkv, g, s, d)
    m = np.full((hkv, g, s), -np.inf, dtype=np.float32)
    l = np.zeros((hkv, g, s), dtype=np.float32)
    acc = np.zeros((hkv, g, s, d), dtype=np.float32)
    for start in range(0, int(length), chunk):
        stop = min(int(length), start + chunk)
        k = keys[start:stop].astype(np.float32).transpose(1, 0, 2)
        v = values[start:stop].astype(np.float32).transpose(1, 0, 2)
        sc = np.einsum("hgsd,htd->hgst", q, k, dtype=np.float32) * np.float32(d ** -0.5)
        cm = sc.max(axis=-1)
        nm = np.maximum(m, cm)
        scale = np.exp(m - nm)
        pw = np.exp(sc - nm[..., None])
        l = l * scale + pw.sum(axis=-1)
        acc = acc * scale[..., None] + np.einsum("hgst,htd->hgsd", pw, v, dtype=np.float32)
        m = nm
    out = (acc / l[..., None]).reshape(hq, s, d)
    lse = (m + np.log(l)).reshape(hq, s)
    return out.astype(np.float32), lse.astype(np.float32)


def refresh_views(state_out, state_lse, slots, qg, new_keys, new_values, commit_lens, scale):
    """One round of the view refresh over all tapped layers, in place on copies
    of the pools: per tapped layer ``reference_position_scores`` then
    ``reference_merge_accepted_positions`` (the loop of LS engine/draft.py:215-256).

    state_out [n_slots, L_tap, Hq, S, D]; state_lse [n_slots, L_tap, Hq, S];
    slots [B]; qg [L_tap, Hq, S, D]; new_keys/new_values [L_tap, B, V, Hkv, D]
    (rows past ``commit_lens[b]`` are padding); commit_lens [B].
    Returns the updated (state_out, state_lse)."""
    out = state_out.copy()
    lse = state_lse.copy()
    b = len(slots)
    for layer in range(qg.shape[0]):
        q = np.broadcast_to(qg[layer][None], (b,) + qg[layer].shape)
        sc = position_scores(q, new_keys[layer], scale)
        o, l = merge_accepted(out[slots, layer], lse[slots, layer], sc, new_values[layer], commit_lens)
        out[slots, layer] = o
        lse[slots, layer] = l
    return out, lse


# ----------------------------------------------------------------------------
# Whole drafter pass
# ----------------------------------------------------------------------------

@dataclass
class DraftShapeOracle:
    hidden: int
    q_heads: int
    kv_heads: int
    head_dim: int
    block: int
    mask_token_id: int
    rms_eps: float = 1e-6
    final_eps: float = 1e-6


def build_views(kv_k, kv_v, table, seq_lens, summary_out, learned_query, window, layers,
                page_size=16, ring_pages=0, prec="bf16"):
    """Per-drafter-layer view dicts for ``draft_pass``: drafter layer j reads
    tapped layer j's window (gathered through the page table) and summary.

    kv_k/kv_v [L_tap, pages, page, Hkv, D]; table [B, max_pages];
    summary_out [B, L_tap, Hq, S, D]; learned_query [L_tap, Hq, S, D]."""
    b = len(seq_lens)
    hkv, d = kv_k.shape[-2], kv_k.shape[-1]
    views = []
    for j in range(layers):
        wk = np.zeros((b, hkv, window, d), dtype=np.float32)
        wv = np.zeros_like(wk)
        lens = []
        for i in range(b):
            rk = gather_window(kv_k[j], table[i], seq_lens[i], window, page_size, ring_pages)
            rv = gather_window(kv_v[j], table[i], seq_lens[i], window, page_size, ring_pages)
            n = rk.shape[1]
            wk[i, :, :n] = rk
            wv[i, :, :n] = rv
            lens.append(n)
        views.append(dict(qg=rnd(learned_query[j], prec), summary_out=summary_out[:, j],
                          win_k=wk, win_v=wv, win_len=np.asarray(lens)))
    return views


def draft_pass(W, shape, anchors, positions, hidden, views, inv_freq, prec, tp=None):
    """``_forward_parallel_shifted_qwen_global16_raw256`` (SF
    draftfreekv.py:3231-3353) followed by the logits projection: returns
    bf16-rounded (or fp32) base logits [B, P, V] and the final block states.

    anchors [B] (the last accepted token ``x_t``), positions [B] (its position,
    i.e. the committed length), hidden [B, L_tap, H] (boundary state), views: one
    dict per drafter layer (see ``decoder_layer``).  ``tp = (world, wire)``: the
    tensor-parallel split of the four row-parallel projections (state-encoder
    and shifted-input second Linears, o_proj, down_proj)."""
    latest = state_encoder(hidden, W, prec, tp=tp)
    h = shifted_input(np.asarray(anchors), latest, W, shape.block, shape.mask_token_id, prec, tp=tp)
    pos = np.asarray(positions, dtype=np.int64)[:, None] + np.arange(shape.block)[None, :]
    cos, sin = rope_tables(pos, inv_freq, prec)
    j = 0
    while f"parallel_qwen_layers.{j}.self_attn.q_proj.weight" in W:
        Wl = {k[len(f"parallel_qwen_layers.{j}."):]: v for k, v in W.items()
              if k.startswith(f"parallel_qwen_layers.{j}.")}
        h = decoder_layer(h, cos, sin, Wl, views[j], shape, prec, tp)
        j += 1
    return project_logits(h, W, shape.final_eps, prec), h
