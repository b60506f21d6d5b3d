"""Tensor-level wrappers over the C ABI (shape/dtype checks, then one native launch).

Functions named after the reference keep the reference's keyword arguments,
argument meaning and ``ValueError`` contracts:

* ``cache_position_scores`` / ``merge_accepted_positions_`` mirror
  ``vendor/sglang/python/sglang/srt/speculative/global16_raw256_incremental.py:400-584``
  (generalised: any S, any verify width up to 32, any GQA group);
* ``refresh_views`` is the fused, paged form of the per-tapped-layer loop of
  ``LongSparkDraft._update_delta`` (``src/longspark/engine/draft.py:215-260``);
* ``draft_attention`` replaces ``Global16Raw256PagedDraftContext.attend``
  (``.../global16_raw256.py:1431-1647``).

All launches go to the current CUDA stream of the tensors' device; nothing is
allocated on the device here.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _native as N


def _p(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("longspark_b200 kernels require CUDA tensors")


class TiledWeight:
    """A [n_out, k] bf16 weight re-laid into the tensor-core tile order
    (``ls_tile_weight``): 128 x 64 tiles, contiguous per tile, pre-swizzled, so
    the GEMM streams each tile with one contiguous bulk copy."""

    def __init__(self, w):
        if w.dtype != torch.bfloat16 or w.ndim != 2 or w.shape[0] % 128 or w.shape[1] % 64:
            raise ValueError("tiled weights must be bf16 [n_out % 128 == 0, k % 64 == 0]")
        self.n_out, self.k = w.shape
        w = w.contiguous()
        self.data = torch.empty_like(w)
        N.call("ls_tile_weight", _stream(w.device), _p(w), _p(self.data), self.n_out, self.k)
        self.shape = (self.n_out, self.k)
        self.device = w.device

    def numel(self):
        return self.data.numel()

    def element_size(self):
        return 2


def _gemm_args(x, w, out, *, workspace, epilogue=N.EPI_STORE, rows=None, residual=None, q_heads=0, kv_heads=0,
               q_norm_w=None, k_norm_w=None, norm_eps=1e-6, positions=None, inv_freq=None, rope_table=None,
               tile_max=None, tile_arg=None, base=None, status=None):
    tiled = isinstance(w, TiledWeight)
    wt = w.data if tiled else w
    _require_cuda(x, wt, out, workspace)
    if x.dtype != torch.bfloat16 or wt.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("gemm operands must be bf16")
    if x.stride(-1) != 1 or out.stride(-1) != 1 or not wt.is_contiguous():
        raise ValueError("gemm operands must be contiguous along K")
    rows = x.shape[0] if rows is None else rows
    n_out, k = w.shape
    a = N.GemmArgs(x=_p(x), w=_p(wt), w_layout=N.W_TILED if tiled else N.W_ROWMAJOR, rows=rows, k=k, n_out=n_out,
                   x_ld=x.stride(0),
                   epilogue=epilogue, out=_p(out), out_ld=out.stride(0), residual=_p(residual),
                   res_ld=0 if residual is None else residual.stride(0), q_heads=q_heads, kv_heads=kv_heads,
                   q_norm_w=_p(q_norm_w), k_norm_w=_p(k_norm_w), norm_eps=norm_eps, positions=_p(positions),
                   inv_freq=_p(inv_freq), rope_table=_p(rope_table), tile_max=_p(tile_max), tile_arg=_p(tile_arg), base=_p(base),
                   base_ld=0 if base is None else base.stride(0), status=_p(status))
    return a


def gemm(x, w, out, *, workspace, **kw):
    """out = epilogue(x[:rows] @ w.T) on the tcgen05 tensor cores (see ``ls_gemm``).
    ``w`` is a row-major [n_out, k] bf16 tensor or a ``TiledWeight``.  Keywords:
    epilogue, rows, residual, q_heads, kv_heads, q_norm_w, k_norm_w, norm_eps,
    positions, inv_freq, rope_table, tile_max, tile_arg, base, status."""
    a = _gemm_args(x, w, out, workspace=workspace, **kw)
    N.call("ls_gemm", _stream(x.device), C.byref(a), _p(workspace), workspace.numel() * workspace.element_size())
    return out


def gemm_allreduce(x, w, out, *, group, workspace, wire=N.TP_WIRE_F32, **kw):
    """Row-parallel GEMM fused with the allreduce of its output over the
    tensor-parallel ``group`` (``ls_gemm_allreduce``): ``x``/``w`` are this rank's
    k-slice, ``out`` (inside the group's heap) receives the sum over ranks with
    the STORE or RESIDUAL epilogue on every rank."""
    a = _gemm_args(x, w, out, workspace=workspace, **kw)
    N.call("ls_gemm_allreduce", _stream(x.device), C.byref(a), C.byref(group.struct), wire, _p(workspace),
           workspace.numel() * workspace.element_size())
    return out


def tp_barrier(group, *, slot=0, status=None, device=None):
    """Device-side barrier over the tensor-parallel group (``ls_tp_barrier``)."""
    N.call("ls_tp_barrier", _stream(device if device is not None else group.device), C.byref(group.struct), slot,
           _p(status))


def gemm_workspace_bytes(rows, k, n_out):
    return int(N.lib().ls_gemm_workspace_bytes(rows, k, n_out))


def rmsnorm(x, w, out, eps, *, mode=0, rows=None, w2=None, out2=None):
    """mode 0: SpecForge RMSNorm rounding; mode 1: ``F.rms_norm`` rounding.
    With ``w2``/``out2`` a second norm of ``out`` follows in the same launch."""
    _require_cuda(x, w, out)
    rows = x.shape[0] if rows is None else rows
    N.call("ls_rmsnorm", _stream(x.device), _p(x), x.stride(0), _p(w), _p(out), out.stride(0), rows,
           x.shape[-1], float(eps), int(mode), _p(w2), _p(out2), 0 if out2 is None else out2.stride(0))
    return out


def shifted_input(anchors, seq_lens, positions, embed, pos_emb, latest, out, *, block, mask_token_id, status=None,
                  inv_freq=None, rope_table=None, batch=None, latest_norm_w=None, norm_eps=1e-6):
    """``latest_norm_w``: ``latest`` is the state encoder's output before its
    RMSNorm, which is applied here."""
    _require_cuda(anchors, embed, pos_emb, latest, out)
    batch = anchors.shape[0] if batch is None else batch
    N.call("ls_shifted_input", _stream(out.device), _p(anchors), _p(seq_lens), _p(positions), _p(inv_freq),
           _p(rope_table), _p(embed), _p(pos_emb), _p(latest), _p(latest_norm_w), float(norm_eps), _p(out), batch,
           block, embed.shape[1], embed.shape[0], mask_token_id, _p(status))
    return out


def gather_rows(src, idx, out, rows=None, status=None):
    rows = idx.shape[0] if rows is None else rows
    row_bytes = src[0].numel() * src.element_size()
    N.call("ls_gather_rows", _stream(out.device), _p(src), src.shape[0], _p(idx), _p(out), rows, row_bytes,
           _p(status))
    return out


# ---------------------------------------------------------------------------
# (a) view refresh
# ---------------------------------------------------------------------------

def cache_position_scores(*, layer_id, global_query, new_keys, output, softmax_scale, softcap=0.0):
    """Scores of the learned summary queries against new target K rows.

    global_query [B, Hq, S, D] bf16 (batch stride may be 0), new_keys
    [B, V, Hkv, D] bf16, output [B, Hq, S, V] fp32."""
    _require_cuda(global_query, new_keys, output)
    if global_query.ndim != 4 or new_keys.ndim != 4:
        raise ValueError("Global query and new Target keys must be rank-4")
    batch, q_heads, slots, head_dim = global_query.shape
    if new_keys.shape[0] != batch or head_dim != 128 or new_keys.shape[-1] != 128:
        raise ValueError("Global summary score shape is incompatible with the new keys")
    rows, kv_heads = new_keys.shape[1], new_keys.shape[2]
    if q_heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    if output.shape != (batch, q_heads, slots, rows) or output.dtype != torch.float32:
        raise ValueError("score output workspace has the wrong shape or dtype")
    if global_query.dtype != torch.bfloat16 or new_keys.dtype != torch.bfloat16:
        raise ValueError("Global queries and Target keys must be bf16")
    if float(softcap) != 0.0:
        raise ValueError("softcap is not used by Qwen3 drafters")
    if global_query.stride(-1) != 1 or global_query.stride(-2) != 128 or not new_keys.is_contiguous() \
            or not output.is_contiguous():
        raise ValueError("Global query rows, keys and output must be contiguous")
    N.call("ls_position_scores", _stream(output.device), _p(global_query), global_query.stride(0),
           global_query.stride(1), _p(new_keys), _p(output), batch, q_heads, kv_heads, slots, rows,
           float(softmax_scale))
    return output


def merge_accepted_positions_(*, state_output, state_lse, position_scores, value_cache, accepted_cache_locs,
                              accept_lens, accept_offsets, state_slots=None, status=None):
    """Online-softmax merge of accepted value rows into the persistent state, in place.

    value_cache [N, 1, Hkv, D] bf16 (page-size-one rows); accepted_cache_locs
    either fixed [B, V] or flat with int32 ``accept_offsets``."""
    _require_cuda(state_output, state_lse, position_scores, value_cache, accepted_cache_locs, accept_lens)
    capacity, q_heads, slots, head_dim = state_output.shape
    batch = position_scores.shape[0]
    rows = position_scores.shape[-1]
    if state_output.dtype != torch.float32 or state_lse.dtype != torch.float32 \
            or position_scores.dtype != torch.float32:
        raise ValueError("state, LSE and cached scores must use FP32")
    if state_lse.shape != (capacity, q_heads, slots) or head_dim != 128:
        raise ValueError("state output/LSE shapes do not match")
    if position_scores.shape != (batch, q_heads, slots, rows):
        raise ValueError("cached score shape is invalid")
    if value_cache.ndim != 4 or value_cache.shape[1] != 1 or value_cache.shape[-1] != 128:
        raise ValueError("accepted Target V must come from a page-size-one cache")
    kv_heads = value_cache.shape[2]
    if q_heads % kv_heads:
        raise ValueError("Target V cache does not match the GQA state")
    if accept_lens.shape != (batch,) or accept_lens.dtype != torch.int32:
        raise ValueError("accept_lens must be one int32 value per request")
    if accepted_cache_locs.ndim == 2:
        if accepted_cache_locs.shape != (batch, rows):
            raise ValueError("fixed verify cache locations must have shape [batch, rows]")
        locs = accepted_cache_locs.to(torch.int64).contiguous()
    elif accepted_cache_locs.ndim == 1:
        if accept_offsets is None or accept_offsets.dtype != torch.int32 or accept_offsets.shape[0] < batch:
            raise ValueError("compact cache locations require int32 accept offsets")
        idx = (accept_offsets[:batch].to(torch.int64)[:, None]
               + torch.arange(rows, device=accept_lens.device)[None, :])
        idx = idx.clamp_max(accepted_cache_locs.numel() - 1)
        locs = accepted_cache_locs.to(torch.int64)[idx].contiguous()
    else:
        raise ValueError("accepted cache locations must be compact flat or fixed [batch, rows]")
    if state_slots is not None and (state_slots.shape != (batch,) or state_slots.dtype != torch.int32):
        raise ValueError("state_slots must be one int32 pool index per request")
    if state_slots is None and capacity != batch:
        raise ValueError("batch-local state must have one row per request")
    if not value_cache.is_contiguous():
        raise ValueError("value cache must be contiguous")
    N.call("ls_merge_accepted", _stream(state_output.device), _p(state_output), state_output.stride(0),
           _p(state_lse), state_lse.stride(0), _p(position_scores.contiguous()), _p(value_cache), _p(locs),
           _p(accept_lens), _p(state_slots), batch, q_heads, kv_heads, slots, rows, _p(status))


def refresh_views(*, kv_k, kv_v, page_table, seq_lens, commit_lens, slots, learned_query, state_out, state_lse,
                  max_commit, ring_pages=0, softmax_scale=128 ** -0.5, status=None, batch=None, state_bf16=None):
    """Fused paged view refresh over all tapped layers (see ``ls_refresh_views``).

    kv_k/kv_v [L_tap, pages, 16, Hkv, 128] bf16; page_table [B, max_pages]
    int32; seq_lens/commit_lens/slots [B] int32; learned_query
    [L_tap, Hq, S, 128] bf16; state_out [cap, L_tap, Hq, S, 128] fp32;
    state_lse [cap, L_tap, Hq, S] fp32."""
    _require_cuda(kv_k, kv_v, page_table, seq_lens, commit_lens, slots, learned_query, state_out, state_lse)
    L, pages, ps, hkv, d = kv_k.shape
    if ps != 16 or d != 128 or kv_v.shape != kv_k.shape:
        raise ValueError("KV pool must be [layers, pages, 16, kv_heads, 128]")
    _, hq, s, _ = learned_query.shape
    if state_out.shape[1:] != (L, hq, s, 128) or state_lse.shape[1:] != (L, hq, s):
        raise ValueError("summary state does not match the learned queries")
    for t, name in ((page_table, "page_table"), (seq_lens, "seq_lens"), (commit_lens, "commit_lens"),
                    (slots, "slots")):
        if t.dtype != torch.int32:
            raise ValueError(f"{name} must be int32")
    batch = seq_lens.shape[0] if batch is None else batch
    a = N.RefreshArgs(kv_k=_p(kv_k), kv_v=_p(kv_v), pool_pages=pages, page_table=_p(page_table),
                      table_stride=page_table.stride(0), ring_pages=ring_pages, seq_lens=_p(seq_lens),
                      commit_lens=_p(commit_lens), slots=_p(slots), learned_query=_p(learned_query),
                      state_out=_p(state_out), state_lse=_p(state_lse), state_bf16=_p(state_bf16),
                      bf16_layers=0 if state_bf16 is None else state_bf16.shape[1], capacity=state_out.shape[0],
                      batch=batch, tap_layers=L,
                      q_heads=hq, kv_heads=hkv, slots_per_head=s, max_commit=max_commit,
                      softmax_scale=float(softmax_scale), status=_p(status))
    N.call("ls_refresh_views", _stream(state_out.device), C.byref(a))


def prefill_summary(*, kv_k, kv_v, page_table, seq_lens, slots, learned_query, state_out, state_lse,
                    softmax_scale=128 ** -0.5, status=None, batch=None, state_bf16=None):
    """Full-prefix summary state (``ls_prefill_summary``): for each request b,
    every tapped layer and query head, the (output, lse) of the learned
    queries over pool rows [0, seq_lens[b]) written at slot ``slots[b]``.

    kv_k/kv_v [L_tap, pages, 16, Hkv, 128] bf16 holding the whole prefix;
    page_table [B, max_pages] int32; learned_query [L_tap, Hq, S, 128] bf16;
    state_out [cap, L_tap, Hq, S, 128] fp32; state_lse [cap, L_tap, Hq, S]."""
    _require_cuda(kv_k, kv_v, page_table, seq_lens, slots, learned_query, state_out, state_lse)
    L, pages, ps, hkv, d = kv_k.shape
    if ps != 16 or d != 128 or kv_v.shape != kv_k.shape:
        raise ValueError("KV pool must be [layers, pages, 16, kv_heads, 128]")
    _, hq, s, _ = learned_query.shape
    if state_out.shape[1:] != (L, hq, s, 128) or state_lse.shape[1:] != (L, hq, s):
        raise ValueError("summary state does not match the learned queries")
    for t, name in ((page_table, "page_table"), (seq_lens, "seq_lens"), (slots, "slots")):
        if t.dtype != torch.int32:
            raise ValueError(f"{name} must be int32")
    batch = seq_lens.shape[0] if batch is None else batch
    a = N.PrefillArgs(kv_k=_p(kv_k), kv_v=_p(kv_v), pool_pages=pages, page_table=_p(page_table),
                      table_stride=page_table.stride(0), seq_lens=_p(seq_lens), slots=_p(slots),
                      learned_query=_p(learned_query), state_out=_p(state_out), state_lse=_p(state_lse),
                      state_bf16=_p(state_bf16), bf16_layers=0 if state_bf16 is None else state_bf16.shape[1],
                      capacity=state_out.shape[0], batch=batch, tap_layers=L, q_heads=hq, kv_heads=hkv,
                      slots_per_head=s, softmax_scale=float(softmax_scale), status=_p(status))
    N.call("ls_prefill_summary", _stream(state_out.device), C.byref(a))


def window_scatter(*, keys, values, row_offsets, counts, seq_lens, kv_k, kv_v, page_table, ring_pages=0,
                   last_hidden=None, hidden_pool=None, slots=None, status=None, batch=None):
    """Packet K/V rows -> paged pool at their positions; last hidden -> slot pool.
    ``keys``/``values`` [L, total_rows, Hkv, 128]: request b owns rows
    [row_offsets[b], row_offsets[b] + counts[b])."""
    L, total, hkv, d = keys.shape if keys is not None else (kv_k.shape[0], 0, kv_k.shape[3], 128)
    if batch is None:
        batch = counts.shape[0] if counts is not None else slots.shape[0]
    hidden = hidden_pool.shape[-1] if hidden_pool is not None else 0
    N.call("ls_window_scatter", _stream(kv_k.device), _p(keys), _p(values), total, _p(row_offsets), _p(counts),
           _p(seq_lens), _p(kv_k), _p(kv_v), kv_k.shape[1], _p(page_table),
           page_table.stride(0) if page_table is not None else 0, ring_pages, _p(last_hidden), _p(hidden_pool),
           0 if hidden_pool is None else hidden_pool.shape[0], _p(slots), batch, L, hkv, hidden, _p(status))


# ---------------------------------------------------------------------------
# (b) drafter attention, sampling, accept
# ---------------------------------------------------------------------------

def attention_workspace_bytes(batch, q_heads, kv_heads, window, slots):
    return int(N.lib().ls_attention_workspace_bytes(batch, q_heads, kv_heads, window, slots))


def draft_attention(*, qkv, block, kv_k, kv_v, page_table, seq_lens, window, learned_query, state_out, slots, out,
                    workspace, q_heads, kv_heads, ring_pages=0, softmax_scale=128 ** -0.5, status=None,
                    batch=None, state_bf16=None):
    """Block queries over [summary | window | local].  qkv [B*P, (Hq+2Hkv)*128]
    (rotated q, rotated k, v); kv_k/kv_v one tapped layer [pages, 16, Hkv, 128];
    learned_query [Hq, S, 128]; state_out [cap, ..., Hq, S, 128] fp32 (entry of
    request b at slot slots[b]); out [B*P, Hq*128] bf16."""
    _require_cuda(qkv, kv_k, kv_v, page_table, seq_lens, learned_query, state_out, slots, out, workspace)
    batch = seq_lens.shape[0] if batch is None else batch
    a = N.AttentionArgs(qkv=_p(qkv), block=block, kv_k=_p(kv_k), kv_v=_p(kv_v), pool_pages=kv_k.shape[0],
                        page_table=_p(page_table),
                        table_stride=page_table.stride(0), ring_pages=ring_pages, seq_lens=_p(seq_lens),
                        window=window, learned_query=_p(learned_query), state_out=_p(state_out),
                        state_stride=state_out.stride(0), state_bf16=_p(state_bf16),
                        state_bf16_stride=0 if state_bf16 is None else state_bf16.stride(0),
                        slots=_p(slots), capacity=state_out.shape[0],
                        slots_per_head=learned_query.shape[1],
                        batch=batch, q_heads=q_heads, kv_heads=kv_heads, softmax_scale=float(softmax_scale),
                        out=_p(out), status=_p(status))
    N.call("ls_draft_attention", _stream(out.device), C.byref(a), _p(workspace),
           workspace.numel() * workspace.element_size())
    return out


def markov_workspace_bytes(batch, block):
    return int(N.lib().ls_markov_workspace_bytes(batch, block))


def markov_argmax(*, base, tile_max, tile_arg, anchors, tokens, block, workspace, w1=None, w2=None, w1_bound=None,
                  w2_bound=None, target=None, accept_out=None, status=None, batch=None, group=None,
                  tiles_per_shard=None, vocab=None):
    """Greedy Markov chain (or plain argmax without a head) over bf16 base logits.
    With a tensor-parallel ``group``, ``base``/``tile_max``/``tile_arg`` are this
    rank's vocabulary shard (``tiles_per_shard`` 128-token tiles per rank, the
    full ``vocab``), inside the group's heap (``ls_markov_argmax_tp``)."""
    _require_cuda(base, tile_max, tile_arg, anchors, tokens, workspace)
    batch = anchors.shape[0] if batch is None else batch
    a = N.MarkovArgs(base=_p(base), tile_max=_p(tile_max), tile_arg=_p(tile_arg), w1=_p(w1), w2=_p(w2),
                     w1_row_bound=_p(w1_bound), w2_row_bound=_p(w2_bound), rank=0 if w1 is None else w1.shape[1],
                     anchors=_p(anchors), tokens=_p(tokens), target=_p(target),
                     target_ld=0 if target is None else target.stride(0), accept_out=_p(accept_out), batch=batch,
                     block=block, vocab=base.shape[-1] if vocab is None else vocab, status=_p(status))
    if group is not None:
        N.call("ls_markov_argmax_tp", _stream(tokens.device), C.byref(a), C.byref(group.struct), tiles_per_shard,
               _p(workspace), workspace.numel() * workspace.element_size())
        return tokens
    N.call("ls_markov_argmax", _stream(tokens.device), C.byref(a), _p(workspace),
           workspace.numel() * workspace.element_size())
    return tokens


def sample_step_workspace_bytes(batch):
    return N.lib().ls_sample_step_workspace_bytes(batch)


def sample_step(*, logits, step, block, temperature, seed, tokens, workspace, q=None, prev=None, status=None,
                batch=None):
    """One step of the T > 0 chain (``ls_sample_step``): ``logits`` [B, V] view
    (row stride = its stride(0)) of the step's bf16 logits; writes column
    ``step`` of ``tokens`` [B, block] int64 and ``q`` [B, block] fp32, and
    ``prev`` [B] int32."""
    _require_cuda(logits, tokens, workspace)
    if logits.dtype != torch.bfloat16 or logits.stride(-1) != 1:
        raise ValueError("step logits must be bf16 with unit stride along the vocabulary")
    batch = logits.shape[0] if batch is None else batch
    a = N.SampleStepArgs(logits=_p(logits), logits_ld=logits.stride(0), batch=batch, vocab=logits.shape[-1],
                         block=block, step=step, temperature=float(temperature), seed=int(seed) & (2 ** 64 - 1),
                         tokens=_p(tokens), q=_p(q), prev=_p(prev), status=_p(status))
    N.call("ls_sample_step", _stream(tokens.device), C.byref(a), _p(workspace),
           workspace.numel() * workspace.element_size())


def rejection_sample(*, candidates, sampled_q, target_logits, draft_logits, temperature, uniforms, final_uniforms,
                     lengths=None, bonus=None, status=None):
    """T > 0 verification of a drafted block (``ls_rejection_sample``): the
    reference's ``decide_acceptance`` + ``finish_sampling``
    (``src/longspark/engine/sampling.py:19-57``) in one launch.

    candidates [B, P] int64 (the drafted tokens), sampled_q [B, P] fp32 (their
    proposal probabilities), target_logits [B, P + 1, V] bf16 (the verify
    pass), draft_logits [B, P, V] bf16 (the drafter's corrected logits, whose
    softmax at the rejection position is the q row of phase two), uniforms
    [B, P] and final_uniforms [B] fp32.  Returns (lengths [B], bonus [B])
    int64 device tensors.  Shape errors raise ``ValueError`` with the
    reference's messages."""
    b, p = candidates.shape
    if sampled_q.shape != (b, p) or uniforms.shape != (b, p):
        raise ValueError("sampled q and uniforms must match the seven proposal positions")
    if tuple(target_logits.shape[:2]) != (b, p + 1):
        raise ValueError("target must verify proposal width plus one bonus row")
    if final_uniforms.shape != (b,):
        raise ValueError("one final uniform is required per request")
    if tuple(draft_logits.shape[:2]) != (b, p) or draft_logits.shape[-1] != target_logits.shape[-1]:
        raise ValueError("draft logits must cover the proposal positions over the target's vocabulary")
    for t, dt in ((target_logits, torch.bfloat16), (draft_logits, torch.bfloat16), (candidates, torch.int64),
                  (sampled_q, torch.float32), (uniforms, torch.float32), (final_uniforms, torch.float32)):
        if t.dtype != dt:
            raise ValueError(f"expected {dt} inputs, got {t.dtype}")
    _require_cuda(candidates, sampled_q, target_logits, draft_logits, uniforms, final_uniforms)
    tl = target_logits if target_logits.stride(-1) == 1 and target_logits.stride(1) * (p + 1) == \
        target_logits.stride(0) else target_logits.contiguous()
    dl = draft_logits if draft_logits.stride(-1) == 1 and draft_logits.stride(1) * p == draft_logits.stride(0) \
        else draft_logits.contiguous()
    dev = candidates.device
    lengths = torch.empty(b, dtype=torch.int64, device=dev) if lengths is None else lengths
    bonus = torch.empty(b, dtype=torch.int64, device=dev) if bonus is None else bonus
    a = N.RejectionArgs(target_logits=_p(tl), target_ld=tl.stride(1), draft_logits=_p(dl), draft_ld=dl.stride(1),
                        candidates=_p(candidates.contiguous()), sampled_q=_p(sampled_q.contiguous()),
                        uniforms=_p(uniforms.contiguous()), final_uniforms=_p(final_uniforms.contiguous()),
                        temperature=float(temperature), batch=b, block=p, vocab=tl.shape[-1], lengths=_p(lengths),
                        bonus=_p(bonus), status=_p(status))
    N.call("ls_rejection_sample", _stream(dev), C.byref(a))
    return lengths, bonus


def accept_lengths(target, draft, out):
    """Greedy accepted-prefix length (``src/longspark/engine/target.py:472-477``)."""
    _require_cuda(target, draft, out)
    if target.dtype != torch.int64 or draft.dtype != torch.int64 or out.dtype != torch.int64:
        raise ValueError("accept check works on int64 token ids")
    b, p = draft.shape
    if target.shape[0] != b or target.shape[1] < p:
        raise ValueError("target tokens must cover the draft block")
    N.call("ls_accept", _stream(out.device), _p(target), target.stride(0), _p(draft.contiguous()), _p(out), b, p)
    return out


def row_norm_bound(m, out):
    N.call("ls_row_norm_bound", _stream(m.device), _p(m), m.shape[0], m.shape[1], _p(out))
    return out
