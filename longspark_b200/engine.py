"""Drafting-round executor: weights in kernel layout, persistent view pools,
preallocated workspaces, the kernel sequence of one round, CUDA graphs.

The sequence mirrors ``DraftFreeKVModel._forward_parallel_shifted_qwen_global16_raw256``
(``vendor/specforge/modeling/draft/draftfreekv.py:3231-3353``) as served by
``Global16NativeDraftExecutor`` (``vendor/sglang/python/sglang/srt/speculative/
global16_native_draft_executor.py:548-645``), plus the Markov greedy chain
(``draftfreekv.py:2366-2407``) and the accept check
(``src/longspark/engine/target.py:472-477``); every step is one native launch.
"""

from __future__ import annotations

import contextlib
import ctypes as C
import gc
import math
from dataclasses import dataclass, field

import torch

from . import _native as N
from . import ops
from .config import DraftShape


def _interleave_gate_up(gate, up):
    """[I, H] x2 -> [2I, H] with 64 gate rows then the 64 up rows of the same
    outputs per 128-row tile (what the LS_EPI_GATEUP epilogue expects)."""
    i, h = gate.shape
    g = gate.view(i // 64, 64, h)
    u = up.view(i // 64, 64, h)
    return torch.stack([g, u], dim=1).reshape(2 * i, h).contiguous()


class DraftWeights:
    """Drafter + target-module weights in the layout the kernels read.

    Built from a reference-named state dict (``DraftFreeKVModel`` names plus
    ``model.embed_tokens.weight``, ``lm_head.weight``, ``model.norm.weight``)."""

    def __init__(self, shape: DraftShape, W: dict, device, inv_freq=None):
        self.shape = shape
        dev = torch.device(device)

        def t(name):
            return W[name].to(device=dev, dtype=torch.bfloat16).contiguous()

        def tiled(w):
            # GEMM weights live in the tensor-core tile order (ls_tile_weight)
            out = ops.TiledWeight(w)
            del w
            return out

        self.enc_w1 = tiled(t("draft_state_encoder.proj.net.0.weight"))
        self.enc_w2 = tiled(t("draft_state_encoder.proj.net.2.weight"))
        self.enc_norm = t("draft_state_encoder.norm.weight")
        self.pos_emb = t("parallel_shifted_input.position_embedding.weight")
        self.sh_w1 = tiled(t("parallel_shifted_input.proj.net.0.weight"))
        self.sh_w2 = tiled(t("parallel_shifted_input.proj.net.2.weight"))
        self.sh_norm = t("parallel_shifted_input.norm.weight")
        self.layers = []
        for j in range(shape.draft_layers):
            p = f"parallel_qwen_layers.{j}."
            self.layers.append(dict(
                qkv=tiled(torch.cat([t(p + "self_attn.q_proj.weight"), t(p + "self_attn.k_proj.weight"),
                                     t(p + "self_attn.v_proj.weight")], dim=0)),
                o=tiled(t(p + "self_attn.o_proj.weight")),
                q_norm=t(p + "self_attn.q_norm.weight"), k_norm=t(p + "self_attn.k_norm.weight"),
                in_norm=t(p + "input_layernorm.weight"), post_norm=t(p + "post_attention_layernorm.weight"),
                gate_up=tiled(_interleave_gate_up(t(p + "mlp.gate_proj.weight"), t(p + "mlp.up_proj.weight"))),
                down=tiled(t(p + "mlp.down_proj.weight"))))
        self.learned_query = t("global16_raw256_reference.global_query_generator.learned_query")
        self.embed = t("model.embed_tokens.weight")
        self.lm_head = tiled(t("lm_head.weight"))
        self.final_norm = t("model.norm.weight")
        if shape.markov_rank:
            self.w1 = t("parallel_markov_head.markov_w1.weight")
            self.w2 = t("parallel_markov_head.markov_w2.weight")
            # tile copy for the full-vocabulary bias GEMMs (T > 0 chain, corrected
            # logits); the greedy chain gathers rows of the row-major copy
            self.w2_tiled = ops.TiledWeight(self.w2)
            self.w1_bound = torch.zeros(1, dtype=torch.float32, device=dev)
            self.w2_bound = torch.zeros(1, dtype=torch.float32, device=dev)
            ops.row_norm_bound(self.w1, self.w1_bound)
            ops.row_norm_bound(self.w2, self.w2_bound)
        else:
            self.w1 = self.w2 = self.w1_bound = self.w2_bound = self.w2_tiled = None
        if inv_freq is None:
            d = shape.head_dim
            inv_freq = 1.0 / (float(shape.rope_theta) ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        self.inv_freq = inv_freq.to(device=dev, dtype=torch.float32).contiguous()

    def nbytes(self):
        """Weight bytes streamed by one round (each GEMM matrix once).  The
        Markov w1/w2 are not streamed: the chain gathers only the rows of its
        band candidates (a few KiB)."""
        mats = [self.enc_w1, self.enc_w2, self.sh_w1, self.sh_w2, self.lm_head]
        for L in self.layers:
            mats += [L["qkv"], L["o"], L["gate_up"], L["down"]]
        return sum(m.numel() * m.element_size() for m in mats)


@dataclass
class ViewPools:
    """Persistent per-request views: the paged K/V pool of the tapped layers
    (the target's cache, or a drafter-owned ring), page tables, the fp32
    summary state and the boundary hidden states, indexed by pool slot."""
    kv_k: torch.Tensor          # [L_tap, pages, 16, Hkv, 128] bf16
    kv_v: torch.Tensor
    page_table: torch.Tensor    # [capacity, table_stride] int32 (by slot)
    summary_out: torch.Tensor   # [capacity, L_tap, Hq, S, 128] fp32
    summary_lse: torch.Tensor   # [capacity, L_tap, Hq, S] fp32
    hidden: torch.Tensor        # [capacity, L_tap, H] bf16
    ring_pages: int = 0         # > 0: page_table rows are rings of this many pages
    summary_bf16: torch.Tensor = None  # [capacity, L_draft, Hq, S, 128] bf16 copy the attention reads

    def sync_summary_bf16(self, slots=None):
        """Refresh the bf16 copy from the fp32 state (after the state was set by
        other means than the refresh kernel, e.g. a prefill)."""
        if self.summary_bf16 is None:
            return
        n = self.summary_bf16.shape[1]
        if slots is None:
            self.summary_bf16.copy_(self.summary_out[:, :n])
        else:
            idx = slots.long()
            self.summary_bf16.index_copy_(0, idx, self.summary_out.index_select(0, idx)[:, :n].to(torch.bfloat16))


class DraftEngine:
    """Executes drafting rounds for up to ``max_batch`` requests.

    Inputs of a round (device tensors; ``B`` = batch): ``slots`` [B] int32 (pool
    slot of each request), ``seq_lens`` [B] int32 (committed length = position of
    the anchor), ``commit_lens`` [B] int32 (rows committed since the last round,
    refresh only), ``anchors`` [B] int64, ``page_table`` [B, table_stride] int32
    (per-request rows, batch order), optional ``target`` [B, >=P] int64."""

    def __init__(self, shape: DraftShape, weights: DraftWeights, pools: ViewPools, max_batch: int, device):
        self.shape = shape
        self.w = weights
        self.pools = pools
        self.max_batch = max_batch
        self.device = torch.device(device)
        s = shape
        B, P = max_batch, s.block
        M = B * P
        H, Hq, Hkv, I, V = s.hidden, s.q_heads, s.kv_heads, s.inter, s.vocab
        dev = self.device
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.buf = dict(
            enc_in=torch.zeros(B, s.tap_layers * H, **bf), t=torch.zeros(B, H, **bf), u=torch.zeros(B, H, **bf),
            xsh=torch.zeros(M, 2 * H, **bf), f1=torch.zeros(M, H, **bf),
            g=torch.zeros(M, H, **bf), h=torch.zeros(M, H, **bf), xn=torch.zeros(M, H, **bf),
            qkv=torch.zeros(M, (Hq + 2 * Hkv) * 128, **bf), attn=torch.zeros(M, Hq * 128, **bf),
            act=torch.zeros(M, I, **bf), logits=torch.zeros(M, V, **bf),
            tile_max=torch.zeros(M, V // 128, dtype=torch.float32, device=dev),
            tile_arg=torch.zeros(M, V // 128, dtype=torch.int32, device=dev),
            positions=torch.zeros(M, dtype=torch.int32, device=dev),
            rope=torch.zeros(M, 128, dtype=torch.float32, device=dev),
            tokens=torch.zeros(B, P, dtype=torch.int64, device=dev),
            accept=torch.zeros(B, dtype=torch.int64, device=dev),
            status=torch.zeros(1, dtype=torch.int32, device=dev),
        )
        gemm_shapes = [(B, s.tap_layers * H, H), (B, H, H), (M, 2 * H, H), (M, H, H),
                       (M, H, (Hq + 2 * Hkv) * 128), (M, Hq * 128, H), (M, H, 2 * I), (M, I, H), (M, H, V)]
        if s.markov_rank:
            gemm_shapes += [(M, s.markov_rank, V), (B, s.markov_rank, V)]
        # the largest token count needs the largest stream-K workspace (token tile,
        # tile count and grid all grow with it)
        ws = max(ops.gemm_workspace_bytes(r0, k, n) for (r0, k, n) in gemm_shapes)
        self.gemm_ws = torch.zeros(ws, dtype=torch.uint8, device=dev)
        self.attn_ws = torch.zeros(max(1, ops.attention_workspace_bytes(B, Hq, Hkv, s.window, s.slots)),
                                   dtype=torch.uint8, device=dev)
        self.markov_ws = torch.zeros(max(1, ops.markov_workspace_bytes(B, P)), dtype=torch.uint8, device=dev)
        if pools.summary_bf16 is None:
            pools.summary_bf16 = torch.empty(pools.summary_out.shape[0], s.draft_layers, Hq, s.slots, 128,
                                             dtype=torch.bfloat16, device=dev)
            pools.sync_summary_bf16()
        self.graphs = {}
        self.graph_replays = 0
        # a full round issues the view refresh after the first layer's QKV
        # projection, whose tail it overlaps (measured ~2 us faster than first)
        self.refresh_after_qkv = True

    # ------------------------------------------------------------------ refresh
    def refresh(self, *, slots, seq_lens, commit_lens, page_table, batch=None):
        """Fold the rows committed at [seq_lens - commit_lens, seq_lens) into the summary."""
        p = self.pools
        ops.refresh_views(kv_k=p.kv_k, kv_v=p.kv_v, page_table=page_table, seq_lens=seq_lens,
                          commit_lens=commit_lens, slots=slots, learned_query=self.w.learned_query,
                          state_out=p.summary_out, state_lse=p.summary_lse, max_commit=self.shape.max_commit,
                          ring_pages=p.ring_pages, softmax_scale=self.shape.head_dim ** -0.5,
                          status=self.buf["status"], batch=batch, state_bf16=p.summary_bf16)

    def prefill_summary(self, *, slots, seq_lens, page_table, batch=None):
        """Compute the summary state of requests from their whole prefix in the
        pool (``ls_prefill_summary``), replacing the state the target would
        export with a prefill packet; the pool must hold the whole prefix."""
        p = self.pools
        ops.prefill_summary(kv_k=p.kv_k, kv_v=p.kv_v, page_table=page_table, seq_lens=seq_lens, slots=slots,
                            learned_query=self.w.learned_query, state_out=p.summary_out, state_lse=p.summary_lse,
                            softmax_scale=self.shape.head_dim ** -0.5, status=self.buf["status"], batch=batch,
                            state_bf16=p.summary_bf16)

    # ------------------------------------------------------------------ drafter
    def draft(self, *, slots, seq_lens, anchors, page_table, target=None, batch=None, slots_are_rows=False,
              commit_lens=None):
        """One parallel drafter pass: writes ``buf['tokens']`` [B, P] (and
        ``buf['accept']`` [B] when ``target`` is given) and bf16 base logits.
        ``slots_are_rows``: the caller guarantees ``slots == arange(B)``, so the
        boundary hidden states are read in place instead of gathered.
        ``commit_lens``: fold the committed rows into the summary in the same
        pass (a full round).  With ``refresh_after_qkv`` (the default) the
        refresh is issued after the first layer's QKV projection: nothing
        before the attention reads the summary."""
        s, w, p, b = self.shape, self.w, self.pools, self.buf
        B = anchors.shape[0] if batch is None else batch
        P = s.block
        M = B * P
        if commit_lens is not None and not self.refresh_after_qkv:
            self.refresh(slots=slots, seq_lens=seq_lens, commit_lens=commit_lens, page_table=page_table, batch=B)
        H, Hq, Hkv = s.hidden, s.q_heads, s.kv_heads
        ws = self.gemm_ws
        st = b["status"]
        # state encoder
        if slots_are_rows:
            enc_in = p.hidden.view(p.hidden.shape[0], -1)
        else:
            enc_in = b["enc_in"]
            ops.gather_rows(p.hidden.view(p.hidden.shape[0], -1), slots, enc_in, rows=B, status=st)
        ops.gemm(enc_in, w.enc_w1, b["t"], workspace=ws, epilogue=N.EPI_SILU, rows=B, status=st)
        ops.gemm(b["t"], w.enc_w2, b["u"], workspace=ws, rows=B, status=st)
        # shifted input (the encoder's output RMSNorm is applied inside)
        ops.shifted_input(anchors, seq_lens, b["positions"], w.embed, w.pos_emb, b["u"], b["xsh"],
                          block=P, mask_token_id=s.mask_token_id, status=st, inv_freq=w.inv_freq,
                          rope_table=b["rope"], batch=B, latest_norm_w=w.enc_norm, norm_eps=s.rms_eps)
        ops.gemm(b["xsh"], w.sh_w1, b["f1"], workspace=ws, epilogue=N.EPI_SILU, rows=M, status=st)
        ops.gemm(b["f1"], w.sh_w2, b["g"], workspace=ws, rows=M, status=st)
        # shifted-input norm and the first layer's input norm in one launch
        ops.rmsnorm(b["g"], w.sh_norm, b["h"], s.rms_eps, mode=0, rows=M, w2=w.layers[0]["in_norm"], out2=b["xn"])
        for j, L in enumerate(w.layers):
            v = s.view_layer(j)
            if j > 0:
                ops.rmsnorm(b["h"], L["in_norm"], b["xn"], s.rms_eps, mode=0, rows=M)
            ops.gemm(b["xn"], L["qkv"], b["qkv"], workspace=ws, epilogue=N.EPI_QKV, rows=M, q_heads=Hq,
                     kv_heads=Hkv, q_norm_w=L["q_norm"], k_norm_w=L["k_norm"], norm_eps=s.rms_eps,
                     positions=b["positions"], inv_freq=w.inv_freq, rope_table=b["rope"], status=st)
            if j == 0 and commit_lens is not None and self.refresh_after_qkv:
                self.refresh(slots=slots, seq_lens=seq_lens, commit_lens=commit_lens, page_table=page_table,
                             batch=B)
            ops.draft_attention(qkv=b["qkv"], block=P, kv_k=p.kv_k[v], kv_v=p.kv_v[v], page_table=page_table,
                                seq_lens=seq_lens, window=s.window, learned_query=w.learned_query[v],
                                state_out=p.summary_out[:, v], slots=slots, out=b["attn"], workspace=self.attn_ws,
                                q_heads=Hq, kv_heads=Hkv, ring_pages=p.ring_pages,
                                softmax_scale=s.head_dim ** -0.5, status=st, batch=B,
                                state_bf16=p.summary_bf16[:, v] if p.summary_bf16 is not None else None)
            ops.gemm(b["attn"], L["o"], b["h"], workspace=ws, epilogue=N.EPI_RESIDUAL, rows=M, residual=b["h"],
                     status=st)
            ops.rmsnorm(b["h"], L["post_norm"], b["xn"], s.rms_eps, mode=0, rows=M)
            ops.gemm(b["xn"], L["gate_up"], b["act"], workspace=ws, epilogue=N.EPI_GATEUP, rows=M, status=st)
            ops.gemm(b["act"], L["down"], b["h"], workspace=ws, epilogue=N.EPI_RESIDUAL, rows=M,
                     residual=b["h"], status=st)
        ops.rmsnorm(b["h"], w.final_norm, b["xn"], s.final_eps, mode=1, rows=M)
        ops.gemm(b["xn"], w.lm_head, b["logits"], workspace=ws, epilogue=N.EPI_LMHEAD, rows=M,
                 tile_max=b["tile_max"], tile_arg=b["tile_arg"], status=st)
        ops.markov_argmax(base=b["logits"], tile_max=b["tile_max"], tile_arg=b["tile_arg"], anchors=anchors,
                          tokens=b["tokens"], block=P, workspace=self.markov_ws, w1=w.w1, w2=w.w2,
                          w1_bound=w.w1_bound, w2_bound=w.w2_bound, target=target,
                          accept_out=b["accept"] if target is not None else None, status=st, batch=B)

    def draft_native(self, *, slots, seq_lens, anchors, page_table, target=None, batch=None, slots_are_rows=False,
                     commit_lens=None):
        """``draft`` as one C-ABI call (``ls_draft_round``): the same launches
        issued from the library's C++ side, for hosts that bind the library
        directly; writes the same buffers."""
        s, w, p, b = self.shape, self.w, self.pools, self.buf
        B = anchors.shape[0] if batch is None else batch
        if not hasattr(self, "_round_layers"):
            layers = (N.RoundLayer * len(w.layers))()
            for j, L in enumerate(w.layers):
                layers[j] = N.RoundLayer(in_norm=ops._p(L["in_norm"]), qkv=ops._p(L["qkv"].data),
                                         q_norm=ops._p(L["q_norm"]), k_norm=ops._p(L["k_norm"]),
                                         o=ops._p(L["o"].data), post_norm=ops._p(L["post_norm"]),
                                         gate_up=ops._p(L["gate_up"].data), down=ops._p(L["down"].data),
                                         view=s.view_layer(j))
            self._round_layers = layers
        a = N.RoundArgs(
            hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads, inter=s.inter, vocab=s.vocab,
            tap_layers=s.tap_layers, slots_per_head=s.slots, window=s.window, block=s.block,
            max_commit=s.max_commit, markov_rank=s.markov_rank, mask_token_id=s.mask_token_id,
            rms_eps=s.rms_eps, final_eps=s.final_eps, n_layers=len(w.layers),
            layers=C.cast(self._round_layers, C.POINTER(N.RoundLayer)),
            enc_w1=ops._p(w.enc_w1.data), enc_w2=ops._p(w.enc_w2.data), enc_norm=ops._p(w.enc_norm),
            embed=ops._p(w.embed), pos_emb=ops._p(w.pos_emb), sh_w1=ops._p(w.sh_w1.data),
            sh_w2=ops._p(w.sh_w2.data), sh_norm=ops._p(w.sh_norm), final_norm=ops._p(w.final_norm),
            lm_head=ops._p(w.lm_head.data), markov_w1=ops._p(w.w1), markov_w2=ops._p(w.w2),
            w1_bound=ops._p(w.w1_bound), w2_bound=ops._p(w.w2_bound), inv_freq=ops._p(w.inv_freq),
            kv_k=ops._p(p.kv_k), kv_v=ops._p(p.kv_v), pool_pages=p.kv_k.shape[1], ring_pages=p.ring_pages,
            learned_query=ops._p(w.learned_query), summary_out=ops._p(p.summary_out),
            summary_lse=ops._p(p.summary_lse), summary_bf16=ops._p(p.summary_bf16),
            bf16_layers=0 if p.summary_bf16 is None else p.summary_bf16.shape[1],
            hidden_pool=ops._p(p.hidden), capacity=p.summary_out.shape[0],
            batch=B, slots=ops._p(slots), seq_lens=ops._p(seq_lens), commit_lens=ops._p(commit_lens),
            page_table=ops._p(page_table), table_stride=page_table.stride(0), anchors=ops._p(anchors),
            target=ops._p(target), target_ld=0 if target is None else target.stride(0),
            slots_are_rows=1 if slots_are_rows else 0, tokens=ops._p(b["tokens"]), accept=ops._p(b["accept"]),
            logits=ops._p(b["logits"]), status=ops._p(b["status"]))
        need = int(N.lib().ls_round_workspace_bytes(C.byref(a)))
        if getattr(self, "round_ws", None) is None or self.round_ws.numel() < need:
            self.round_ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=self.device)
        a.workspace = ops._p(self.round_ws)
        a.workspace_bytes = self.round_ws.numel()
        N.call("ls_draft_round", ops._stream(self.device), C.byref(a))

    def sample(self, anchors, *, temperature, seed, corrected=None, batch=None):
        """Sampled (T > 0) proposals from the base logits of the last pass, the
        reference's step loop (``sample_block_tokens``, SF draftfreekv.py:
        2366-2407): for each step t the Markov-corrected step logits are one
        tcgen05 GEMM of the previous tokens' w1 rows against w2 with the
        LS_EPI_MARKOV_ADD epilogue, written into ``corrected`` [B*P, V] (the
        ``corrected`` tensor the reference returns), then ``ls_sample_step``
        draws the token from softmax(step / T) and its probability q.  Writes
        ``buf['tokens']`` [B, P] and ``buf['q']`` [B, P]; returns ``corrected``
        viewed [B, P, V] (the base logits themselves without a Markov head)."""
        s, b, w = self.shape, self.buf, self.w
        B = anchors.shape[0] if batch is None else batch
        P, V = s.block, s.vocab
        M = B * P
        dev = self.device
        if "sample_ws" not in b:
            b["sample_ws"] = torch.zeros(max(256, ops.sample_step_workspace_bytes(self.max_batch)),
                                         dtype=torch.uint8, device=dev)
            b["prev"] = torch.zeros(self.max_batch, dtype=torch.int32, device=dev)
            b["q"] = torch.zeros(self.max_batch, P, dtype=torch.float32, device=dev)
            if w.w1 is not None:
                b["xw"] = torch.zeros(self.max_batch, s.markov_rank, dtype=torch.bfloat16, device=dev)
        st = b["status"]
        prev = b["prev"][:B]
        prev.copy_(anchors[:B])
        base = b["logits"][:M].view(B, P, V)
        if w.w1 is not None:
            if corrected is None:
                if "corrected" not in b:
                    b["corrected"] = torch.empty(self.max_batch * P, V, dtype=torch.bfloat16, device=dev)
                corrected = b["corrected"]
            corr = corrected[:M].view(B, P, V)
        else:
            corr = base
        for t in range(P):
            if w.w1 is not None:
                ops.gather_rows(w.w1, prev, b["xw"], rows=B, status=st)
                ops.gemm(b["xw"], w.w2_tiled, corr[:, t], workspace=self.gemm_ws, epilogue=N.EPI_MARKOV_ADD, rows=B,
                         base=base[:, t], status=st)
            ops.sample_step(logits=corr[:, t], step=t, block=P, temperature=temperature, seed=seed,
                            tokens=b["tokens"], workspace=b["sample_ws"], q=b["q"], prev=prev, status=st, batch=B)
        return corr

    def corrected_logits(self, anchors, out, batch=None):
        """Markov-corrected logits of the last pass, ``base + bias(prev)`` per step
        (the ``corrected`` tensor of ``sample_block_tokens``)."""
        s, b, w = self.shape, self.buf, self.w
        B = anchors.shape[0] if batch is None else batch
        M = B * s.block
        if w.w1 is None:
            out[:M].copy_(b["logits"][:M])
            return out
        prev = torch.cat([anchors[:B, None], b["tokens"][:B, :-1]], dim=1).reshape(-1)
        x = w.w1.index_select(0, prev)
        ops.gemm(x, w.w2_tiled, out, workspace=self.gemm_ws, epilogue=N.EPI_MARKOV_ADD, rows=M, base=b["logits"],
                 status=b["status"])
        return out

    def round(self, *, slots, seq_lens, commit_lens, anchors, page_table, target=None, batch=None,
              slots_are_rows=False):
        """One full drafting round: the committed rows are folded into the
        summary and the drafter pass runs (see ``draft``)."""
        self.draft(slots=slots, seq_lens=seq_lens, anchors=anchors, page_table=page_table, target=target,
                   batch=batch, slots_are_rows=slots_are_rows, commit_lens=commit_lens)

    # ------------------------------------------------------------------ status
    def device_status(self):
        """Device status word (0 = ok); synchronises."""
        return int(self.buf["status"].item())

    def clear_status(self):
        self.buf["status"].zero_()


@contextlib.contextmanager
def capture_guard():
    """Keep Python's cyclic garbage collector off while a CUDA graph is being
    captured (``torch.cuda.graph`` collects just before capture begins): an
    unreachable object collected mid-capture — say an earlier drafter that
    owns CUDA graphs and events — would destroy them inside the capture,
    which CUDA rejects and which invalidates the capture."""
    was = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was:
            gc.enable()


class GraphedDraft:
    """CUDA graph of one drafter pass (optionally preceded by the refresh) for a
    fixed batch size.  Inputs are copied into static buffers before replay; the
    whole round — every kernel of the pass, including the greedy Markov chain
    the reference runs eagerly — replays as one graph."""

    def __init__(self, engine: DraftEngine, batch: int, *, with_refresh: bool, with_target: bool,
                 slots_are_rows: bool = False):
        self.engine = engine
        self.slots_are_rows = slots_are_rows
        self.batch = batch
        dev = engine.device
        tstride = engine.pools.page_table.shape[1]
        self.slots = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.seq_lens = torch.ones(batch, dtype=torch.int32, device=dev)
        self.commit_lens = torch.ones(batch, dtype=torch.int32, device=dev)
        self.anchors = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.page_table = torch.zeros(batch, tstride, dtype=torch.int32, device=dev)
        self.target = (torch.zeros(batch, engine.shape.block + 1, dtype=torch.int64, device=dev)
                       if with_target else None)
        self.with_refresh = with_refresh
        self.graph = None

    def _run(self):
        e = self.engine
        e.draft(slots=self.slots, seq_lens=self.seq_lens, anchors=self.anchors, page_table=self.page_table,
                target=self.target, batch=self.batch, slots_are_rows=self.slots_are_rows,
                commit_lens=self.commit_lens if self.with_refresh else None)

    def load(self, *, slots, seq_lens, anchors, page_table, commit_lens=None, target=None):
        self.slots.copy_(slots, non_blocking=True)
        self.seq_lens.copy_(seq_lens, non_blocking=True)
        self.anchors.copy_(anchors, non_blocking=True)
        self.page_table.copy_(page_table, non_blocking=True)
        if commit_lens is not None:
            self.commit_lens.copy_(commit_lens, non_blocking=True)
        if target is not None and self.target is not None:
            self.target.copy_(target, non_blocking=True)

    def capture(self):
        """Capture on a side stream; the inputs currently loaded must be valid
        (the capture does not run the kernels, but a warm-up eager run does)."""
        s = torch.cuda.Stream(device=self.engine.device)
        s.wait_stream(torch.cuda.current_stream(self.engine.device))
        with torch.cuda.stream(s):
            self._run()  # warm-up: kernel attributes, lazy module loading
        torch.cuda.current_stream(self.engine.device).wait_stream(s)
        torch.cuda.synchronize(self.engine.device)
        self.graph = torch.cuda.CUDAGraph()
        with capture_guard(), torch.cuda.graph(self.graph, stream=s):
            self._run()
        return self

    def replay(self):
        self.graph.replay()
        self.engine.graph_replays += 1
