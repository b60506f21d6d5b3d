"""Seeded synthetic drafter weights and views (no checkpoints or datasets exist here).

Generation follows the benchmark recipe: every projection, embedding and the
learned summary queries are N(0, 0.02); RMSNorm weights are ones (the modules'
own initialisation) unless ``norm_jitter`` perturbs them for tests; target K/V
rows are N(0, 1) in a paged pool whose pages are randomly permuted; token ids
are uniform over the vocabulary.  One ``torch.Generator`` drives everything in
a fixed order (weights, KV, page permutation, ids), so a seed reproduces the
same tensors on the same device type.  CPU and CUDA generators give different
streams: parity tests generate on the CPU and copy, the benchmark generates on
the GPU directly.

Weight names are the reference state-dict names (``DraftFreeKVModel`` plus the
three target modules ``model.embed_tokens``, ``lm_head``, ``model.norm``).
"""

from __future__ import annotations

import math

import torch

from .config import DraftShape


def _normal(gen, shape, std, device, dtype=torch.bfloat16):
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=gen)
    return t.to(dtype)


def make_weights(shape: DraftShape, *, seed=0, device="cpu", std=0.02, norm_jitter=0.0,
                 gen=None):
    """Reference-named drafter + target-module weights, bf16."""
    gen = gen or torch.Generator(device=device).manual_seed(seed)
    H, Hq, Hkv, D, I, V = (shape.hidden, shape.q_heads, shape.kv_heads, shape.head_dim,
                           shape.inter, shape.vocab)
    W = {}

    def norm(n):
        if norm_jitter:
            return (1.0 + _normal(gen, (n,), norm_jitter, device, torch.float32)).to(torch.bfloat16)
        return torch.ones(n, dtype=torch.bfloat16, device=device)

    W["draft_state_encoder.proj.net.0.weight"] = _normal(gen, (H, shape.tap_layers * H), std, device)
    W["draft_state_encoder.proj.net.2.weight"] = _normal(gen, (H, H), std, device)
    W["draft_state_encoder.norm.weight"] = norm(H)
    W["parallel_shifted_input.position_embedding.weight"] = _normal(gen, (shape.block, H), std, device)
    W["parallel_shifted_input.proj.net.0.weight"] = _normal(gen, (H, 2 * H), std, device)
    W["parallel_shifted_input.proj.net.2.weight"] = _normal(gen, (H, H), std, device)
    W["parallel_shifted_input.norm.weight"] = norm(H)
    for j in range(shape.draft_layers):
        p = f"parallel_qwen_layers.{j}."
        W[p + "self_attn.q_proj.weight"] = _normal(gen, (Hq * D, H), std, device)
        W[p + "self_attn.k_proj.weight"] = _normal(gen, (Hkv * D, H), std, device)
        W[p + "self_attn.v_proj.weight"] = _normal(gen, (Hkv * D, H), std, device)
        W[p + "self_attn.o_proj.weight"] = _normal(gen, (H, Hq * D), std, device)
        W[p + "self_attn.q_norm.weight"] = norm(D)
        W[p + "self_attn.k_norm.weight"] = norm(D)
        W[p + "mlp.gate_proj.weight"] = _normal(gen, (I, H), std, device)
        W[p + "mlp.up_proj.weight"] = _normal(gen, (I, H), std, device)
        W[p + "mlp.down_proj.weight"] = _normal(gen, (H, I), std, device)
        W[p + "input_layernorm.weight"] = norm(H)
        W[p + "post_attention_layernorm.weight"] = norm(H)
    W["global16_raw256_reference.global_query_generator.learned_query"] = _normal(
        gen, (shape.tap_layers, Hq, shape.slots, D), std, device)
    if shape.markov_rank:
        W["parallel_markov_head.markov_w1.weight"] = _normal(gen, (V, shape.markov_rank), std, device)
        W["parallel_markov_head.markov_w2.weight"] = _normal(gen, (V, shape.markov_rank), std, device)
    W["model.embed_tokens.weight"] = _normal(gen, (V, H), std, device)
    W["lm_head.weight"] = _normal(gen, (V, H), std, device)
    W["model.norm.weight"] = norm(H)
    return W


def rope_inv_freq(shape: DraftShape, device="cpu"):
    """fp32 RoPE inverse frequencies ``1 / theta ** (arange(0, D, 2) / D)``
    (``Qwen3KVFreeParallelAttention.__init__``,
    ``vendor/specforge/modeling/draft/draftfreekv.py:1986-1994``)."""
    d = shape.head_dim
    return 1.0 / (float(shape.rope_theta) ** (torch.arange(0, d, 2, dtype=torch.float32, device=device) / d))


def make_views(shape: DraftShape, batch, contexts, *, seed=1, device="cpu", pool_pages=None,
               extra_rows=0, gen=None, summary="random"):
    """Paged target KV pool (one per tapped layer), page tables, boundary
    hidden states, summary state and anchors for ``batch`` requests.

    contexts: committed length per request (int or list).  Each request gets
    ``ceil((len + extra_rows) / 16)`` pages drawn from a random permutation of
    the pool.  ``summary="random"`` fills the (output, lse) state with plausible
    random values; ``"zero"`` leaves output 0 / lse -inf (an empty prefix)."""
    gen = gen or torch.Generator(device=device).manual_seed(seed)
    if isinstance(contexts, int):
        contexts = [contexts] * batch
    ps = shape.page_size
    need = [math.ceil((c + extra_rows) / ps) for c in contexts]
    max_pages = max(need)
    total = sum(need)
    pool_pages = pool_pages or total
    if pool_pages < total:
        raise ValueError("pool too small for the requested contexts")
    L, Hkv, D = shape.tap_layers, shape.kv_heads, shape.head_dim
    kv_k = _normal(gen, (L, pool_pages, ps, Hkv, D), 1.0, device)
    kv_v = _normal(gen, (L, pool_pages, ps, Hkv, D), 1.0, device)
    perm = torch.randperm(pool_pages, generator=gen, device=device).to(torch.int32)
    table = torch.zeros(batch, max_pages, dtype=torch.int32, device=device)
    o = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[o:o + n]
        o += n
    hidden = _normal(gen, (batch, L, shape.hidden), 1.0, device)
    anchors = torch.randint(0, shape.vocab, (batch,), generator=gen, device=device, dtype=torch.int64)
    S, Hq = shape.slots, shape.q_heads
    if summary == "random":
        out = _normal(gen, (batch, L, Hq, S, D), 0.1, device, torch.float32)
        lse = (torch.log(torch.tensor(contexts, dtype=torch.float32, device=device))[:, None, None, None]
               + _normal(gen, (batch, L, Hq, S), 1.0, device, torch.float32))
    else:
        out = torch.zeros(batch, L, Hq, S, D, dtype=torch.float32, device=device)
        lse = torch.full((batch, L, Hq, S), float("-inf"), dtype=torch.float32, device=device)
    return dict(kv_k=kv_k, kv_v=kv_v, page_table=table,
                seq_lens=torch.tensor(contexts, dtype=torch.int32, device=device),
                hidden=hidden, anchors=anchors, summary_out=out, summary_lse=lse)


def geometric_accept(gen, batch, block, p=0.25, device="cpu"):
    """Accepted-prefix lengths k ~ Geometric(p) on {0, 1, ...} clipped to ``block``
    (mean 3 for p = 1/4)."""
    u = torch.rand(batch, generator=gen, device=device, dtype=torch.float64)
    k = torch.floor(torch.log1p(-u) / math.log1p(-p)).to(torch.int64)
    return k.clamp_max(block)


def target_from_draft(draft, k, vocab):
    """Target tokens whose greedy accept length against ``draft`` is exactly ``k``:
    ``target[:k] = draft[:k]``, ``target[k] != draft[k]``; one extra (bonus) column."""
    b, p = draft.shape
    ar = torch.arange(p + 1, device=draft.device)[None, :]
    padded = torch.cat([draft, draft[:, -1:]], dim=1)
    other = (padded + 1) % vocab
    return torch.where(ar < k[:, None], padded, other)
