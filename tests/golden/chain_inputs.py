"""Seeded inputs of a chained drafting run (weights, a compact paged pool,
per-round commits, anchors and boundary hidden states), shared by the fixture
generator (``make_golden.py``, which runs the reference on them) and the GPU
tests (which run the kernels on them and compare with the stored outputs).

numpy's PCG64 stream is the same on every machine and fast enough to rebuild
a Qwen3-14B-shaped drafter in seconds, so the fixtures store seeds and
outputs, not the inputs themselves.

The pool is compact: a run of R rounds starting at context ``ctx0`` only ever
reads positions ``[ctx0 - W, ctx0 + sum(commits))`` (the window at round 0
and every committed row after it), so only those positions have pages of
their own, drawn in shuffled order; the page-table entries of the older
prefix point at spare pages that nothing reads.  Positions, page-table
columns and RoPE angles are those of the full context.
"""

from __future__ import annotations

import math

import numpy as np
import torch

PAGE = 16


def _bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16)


def chain_commits(rounds, max_commit):
    """Committed rows per round (anchor + accepted), cycling through [1, max_commit]."""
    return [1 + (5 * t + 3) % max_commit for t in range(rounds)]


def chain_weights(shape, seed, std=0.02, norm_jitter=0.05):
    """Reference-named drafter + target-module weights, bf16, N(0, std); RMSNorm
    weights 1 + N(0, norm_jitter)."""
    rng = np.random.default_rng(seed)
    H, Hq, Hkv, D, I, V = shape.hidden, shape.q_heads, shape.kv_heads, shape.head_dim, shape.inter, shape.vocab

    def nrm(*s):
        return _bf16(rng.standard_normal(s, dtype=np.float32) * np.float32(std))

    def norm(n):
        return _bf16(1.0 + rng.standard_normal(n, dtype=np.float32) * np.float32(norm_jitter))

    W = {"draft_state_encoder.proj.net.0.weight": nrm(H, shape.tap_layers * H),
         "draft_state_encoder.proj.net.2.weight": nrm(H, H), "draft_state_encoder.norm.weight": norm(H),
         "parallel_shifted_input.position_embedding.weight": nrm(shape.block, H),
         "parallel_shifted_input.proj.net.0.weight": nrm(H, 2 * H),
         "parallel_shifted_input.proj.net.2.weight": nrm(H, H), "parallel_shifted_input.norm.weight": norm(H)}
    for j in range(shape.draft_layers):
        p = f"parallel_qwen_layers.{j}."
        W[p + "self_attn.q_proj.weight"] = nrm(Hq * D, H)
        W[p + "self_attn.k_proj.weight"] = nrm(Hkv * D, H)
        W[p + "self_attn.v_proj.weight"] = nrm(Hkv * D, H)
        W[p + "self_attn.o_proj.weight"] = nrm(H, Hq * D)
        W[p + "self_attn.q_norm.weight"] = norm(D)
        W[p + "self_attn.k_norm.weight"] = norm(D)
        W[p + "mlp.gate_proj.weight"] = nrm(I, H)
        W[p + "mlp.up_proj.weight"] = nrm(I, H)
        W[p + "mlp.down_proj.weight"] = nrm(H, I)
        W[p + "input_layernorm.weight"] = norm(H)
        W[p + "post_attention_layernorm.weight"] = norm(H)
    W["global16_raw256_reference.global_query_generator.learned_query"] = nrm(shape.tap_layers, Hq, shape.slots, D)
    if shape.markov_rank:
        W["parallel_markov_head.markov_w1.weight"] = nrm(V, shape.markov_rank)
        W["parallel_markov_head.markov_w2.weight"] = nrm(V, shape.markov_rank)
    W["model.embed_tokens.weight"] = nrm(V, H)
    W["lm_head.weight"] = nrm(V, H)
    W["model.norm.weight"] = norm(H)
    return W


def chain_views(shape, ctx0, rounds, seed):
    """Compact pool, page table, initial summary state and per-round inputs of
    one request.  Returns a dict of CPU tensors: kv_k, kv_v ``[L, pages, 16,
    Hkv, 128]`` bf16, page_table ``[1, cols]`` int32, summary_out ``[1, L, Hq,
    S, 128]`` fp32, summary_lse ``[1, L, Hq, S]`` fp32, hidden ``[rounds, 1, L,
    H]`` bf16, anchors ``[rounds]`` int64, commits ``[rounds]`` int32 and
    lengths ``[rounds]`` int32 (committed length after each round's commit)."""
    rng = np.random.default_rng(seed)
    L, Hkv, D, Hq, S = shape.tap_layers, shape.kv_heads, shape.head_dim, shape.q_heads, shape.slots
    commits = chain_commits(rounds, shape.max_commit)
    end = ctx0 + sum(commits)
    live_lo = max(0, ctx0 - shape.window) // PAGE
    live_hi = math.ceil(end / PAGE)
    n_live = live_hi - live_lo
    spare = 8
    pages = n_live + spare
    kv_k = _bf16(rng.standard_normal((L, pages, PAGE, Hkv, D), dtype=np.float32))
    kv_v = _bf16(rng.standard_normal((L, pages, PAGE, Hkv, D), dtype=np.float32))
    perm = rng.permutation(pages).astype(np.int32)
    table = np.empty((1, live_hi), np.int32)
    table[0, live_lo:] = perm[:n_live]
    table[0, :live_lo] = perm[n_live + np.arange(live_lo) % spare]  # never read
    out = (rng.standard_normal((1, L, Hq, S, D), dtype=np.float32) * np.float32(0.1))
    lse = (np.float32(math.log(ctx0)) + rng.standard_normal((1, L, Hq, S), dtype=np.float32))
    hidden = _bf16(rng.standard_normal((rounds, 1, L, shape.hidden), dtype=np.float32))
    anchors = rng.integers(0, shape.vocab, rounds).astype(np.int64)
    lengths = ctx0 + np.cumsum(commits)
    return dict(kv_k=kv_k, kv_v=kv_v, page_table=torch.from_numpy(table), summary_out=torch.from_numpy(out),
                summary_lse=torch.from_numpy(lse), hidden=hidden, anchors=torch.from_numpy(anchors),
                commits=torch.tensor(commits, dtype=torch.int32), lengths=torch.from_numpy(lengths.astype(np.int32)))


def committed_rows(pool, table, length, count, max_commit):
    """``[L, 1, max_commit, Hkv, 128]`` rows at positions ``[length - count,
    length)`` of request 0 (zero-padded past ``count``)."""
    pos = torch.arange(length - count, length)
    pages = table[0].long()[pos // PAGE]
    rows = pool[:, pages, pos % PAGE]  # [L, count, Hkv, D]
    out = torch.zeros((pool.shape[0], 1, max_commit) + tuple(pool.shape[3:]), dtype=pool.dtype)
    out[:, 0, :count] = rows
    return out
