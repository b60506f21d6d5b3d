"""Tensor parallelism of the drafting round over NVLink, one process per GPU.

The reference runs its drafter on one GPU (TP1 is forced at
``vendor/sglang/python/sglang/srt/speculative/global16_native_draft_executor.py:1101-1105``).
This module splits the same round over ``world`` GPUs by KV-head group, the
way the target model's tensor parallelism already splits the K/V it hands
over (``src/longspark/engine/target.py:139-144`` all-gathers per-rank head
shards):

* rank r keeps KV heads ``[r*Hkv/w, (r+1)*Hkv/w)`` and their query heads:
  its slice of the paged K/V pool, of the summary state and of the learned
  queries, so the view refresh and the attention need no communication;
* column-parallel projections (QKV, gate_up, the first Linear of the state
  encoder and of the shifted input) keep the rank's output features;
* the four row-parallel projections (o_proj, down_proj, and the second
  Linears of the state encoder and shifted input) end in
  ``ls_gemm_allreduce``: the GEMM's epilogue peer-stores its tile partials to
  the tile's owner rank, which sums them and peer-stores the result to every
  rank (``allreduce="fused"``), or a plain GEMM followed by
  ``torch.distributed.all_reduce`` over NCCL (``allreduce="nccl"``, the
  baseline);
* the LM head is vocabulary-parallel (128-token tiles split over the ranks);
  after a device barrier every rank runs the same Markov chain, reading the
  band tiles it needs from the owning rank's memory (``ls_markov_argmax_tp``),
  so all ranks hold the same tokens with no gather of the logits.

Buffers that peers write or read live in a ``SymmetricHeap``: one CUDA IPC
allocation per rank, mapped into every rank's process.
"""

from __future__ import annotations

import ctypes as C
import math

import torch

from . import _native as N
from . import ops
from .config import DraftShape
from .engine import DraftWeights, ViewPools

# ----------------------------------------------------------------------------
# Sharding plan (pure host logic)
# ----------------------------------------------------------------------------


def check_tp_shape(shape: DraftShape, world: int):
    """Raise ValueError unless the shape splits evenly over ``world`` ranks in
    the units the kernels need."""
    if world < 1 or world > N.TP_MAX_RANKS:
        raise ValueError(f"tensor-parallel world must be in [1, {N.TP_MAX_RANKS}]")
    H, I = shape.hidden, shape.inter
    if shape.kv_heads % world:
        raise ValueError(f"{shape.kv_heads} KV heads do not split over {world} ranks")
    if H % (128 * world):
        raise ValueError(f"hidden {H} must split into multiples of 128 over {world} ranks")
    if I % (64 * world):
        raise ValueError(f"intermediate {I} must split into multiples of 64 over {world} ranks")
    n_tiles = shape.vocab // 128
    T = math.ceil(n_tiles / world)
    if T * (world - 1) >= n_tiles:
        raise ValueError(f"vocabulary of {n_tiles} tiles leaves a rank without tiles over {world} ranks")


def vocab_shards(vocab: int, world: int):
    """(tiles per shard T, [(first token, token count) per rank]) of the
    vocabulary-parallel LM head: rank s holds 128-token tiles
    [s*T, min((s+1)*T, vocab/128))."""
    n_tiles = vocab // 128
    T = math.ceil(n_tiles / world)
    out = []
    for s in range(world):
        t0 = s * T
        t1 = min(n_tiles, t0 + T)
        out.append((t0 * 128, (t1 - t0) * 128))
    return T, out


def local_shape(shape: DraftShape, world: int) -> DraftShape:
    """The per-rank shape: the rank's query/KV heads and intermediate slice
    (hidden and vocabulary stay global)."""
    check_tp_shape(shape, world)
    return shape.with_(q_heads=shape.q_heads // world, kv_heads=shape.kv_heads // world, inter=shape.inter // world)


def shard_state_dict(W: dict, shape: DraftShape, rank: int, world: int) -> dict:
    """Rank ``rank``'s slice of a reference-named drafter state dict (views, no
    copies).  Replicated: norms, embeddings, Markov w1/w2, boundary-state
    projections' inputs."""
    check_tp_shape(shape, world)
    H, D = shape.hidden, shape.head_dim
    hq, hkv = shape.q_heads // world, shape.kv_heads // world
    Hs, Is = H // world, shape.inter // world

    def rows(t, n):  # output-feature slice of a [n_out, k] weight
        return t[rank * n:(rank + 1) * n]

    def cols(t, n):  # input-feature slice
        return t[:, rank * n:(rank + 1) * n]

    out = {}
    for k, t in W.items():
        if k == "draft_state_encoder.proj.net.0.weight" or k == "parallel_shifted_input.proj.net.0.weight":
            out[k] = rows(t, Hs)
        elif k == "draft_state_encoder.proj.net.2.weight" or k == "parallel_shifted_input.proj.net.2.weight":
            out[k] = cols(t, Hs)
        elif k.endswith("self_attn.q_proj.weight"):
            out[k] = rows(t, hq * D)
        elif k.endswith("self_attn.k_proj.weight") or k.endswith("self_attn.v_proj.weight"):
            out[k] = rows(t, hkv * D)
        elif k.endswith("self_attn.o_proj.weight"):
            out[k] = cols(t, hq * D)
        elif k.endswith("mlp.gate_proj.weight") or k.endswith("mlp.up_proj.weight"):
            out[k] = rows(t, Is)
        elif k.endswith("mlp.down_proj.weight"):
            out[k] = cols(t, Is)
        elif k == "global16_raw256_reference.global_query_generator.learned_query":
            out[k] = t[:, rank * hq:(rank + 1) * hq]
        elif k == "lm_head.weight":
            _, shards = vocab_shards(shape.vocab, world)
            v0, n = shards[rank]
            out[k] = t[v0:v0 + n]
        else:
            out[k] = t
    return out


def shard_views(v: dict, shape: DraftShape, rank: int, world: int) -> dict:
    """Rank ``rank``'s slice of ``synthetic.make_views`` output: its KV heads of
    the paged pool and its query heads of the summary state (copies, so the
    rank's pool is contiguous as a head-sharded target cache would be)."""
    hkv = shape.kv_heads // world
    hq = shape.q_heads // world
    out = dict(v)
    out["kv_k"] = v["kv_k"][:, :, :, rank * hkv:(rank + 1) * hkv].contiguous()
    out["kv_v"] = v["kv_v"][:, :, :, rank * hkv:(rank + 1) * hkv].contiguous()
    out["summary_out"] = v["summary_out"][:, :, rank * hq:(rank + 1) * hq].contiguous()
    out["summary_lse"] = v["summary_lse"][:, :, rank * hq:(rank + 1) * hq].contiguous()
    return out


# ----------------------------------------------------------------------------
# Symmetric heap and group
# ----------------------------------------------------------------------------


def _round_up(x, a):
    return (x + a - 1) // a * a


class _CudaSpan:
    """A raw device range exposed through ``__cuda_array_interface__`` so torch
    can wrap it without a copy; holds its owner alive."""

    def __init__(self, owner, ptr, nbytes):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


class SymmetricHeap:
    """One ``ls_ipc_alloc`` of the same size on every rank, every peer's mapped
    with ``ls_ipc_open``.  ``carve`` hands out tensors at the same offset on
    every rank (call it in the same order with the same sizes everywhere).

    ``all_gather(bytes) -> list[bytes]`` exchanges the 64-byte IPC handles
    (e.g. ``torch.distributed.all_gather_object``)."""

    ALIGN = 256

    def __init__(self, nbytes, *, rank, world, device, all_gather):
        self.device = torch.device(device)
        self.rank, self.world = rank, world
        self.nbytes = _round_up(int(nbytes), 1 << 21)
        ptr = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        with torch.cuda.device(self.device):
            N.call("ls_ipc_alloc", self.nbytes, C.byref(ptr), handle)
        self.ptr = ptr.value
        self.peers = []
        self._opened = []
        try:
            handles = all_gather(bytes(handle))
            if len(handles) != world:
                raise RuntimeError(f"handle exchange returned {len(handles)} handles for {world} ranks")
            with torch.cuda.device(self.device):
                for p, h in enumerate(handles):
                    if p == rank:
                        self.peers.append(self.ptr)
                        continue
                    q = C.c_void_p()
                    buf = (C.c_ubyte * 64).from_buffer_copy(h)
                    N.call("ls_ipc_open", buf, C.byref(q))
                    self._opened.append(q.value)
                    self.peers.append(q.value)
        except BaseException:
            self._release()
            raise
        self.used = 0

    def carve(self, shape, dtype):
        """A tensor of ``shape``/``dtype`` at the next free (256-byte aligned) offset."""
        n = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
        off = self.used
        if off + n > self.nbytes:
            raise RuntimeError(f"symmetric heap of {self.nbytes} bytes exhausted ({off} + {n})")
        self.used = _round_up(off + n, self.ALIGN)
        raw = torch.as_tensor(_CudaSpan(self, self.ptr + off, max(n, 1)), device=self.device)
        return raw[:n].view(dtype).view(shape)

    def offset_of(self, t):
        return t.data_ptr() - self.ptr

    def _release(self):
        with torch.cuda.device(self.device):
            for q in self._opened:
                N.lib().ls_ipc_close(C.c_void_p(q))
            self._opened = []
            if self.ptr:
                N.lib().ls_ipc_free(C.c_void_p(self.ptr))
                self.ptr = 0

    def close(self, barrier=None):
        """Unmap the peers and free this rank's heap.  ``barrier()`` (a host
        barrier over the ranks) runs first, so no peer still reads this memory."""
        torch.cuda.synchronize(self.device)
        if barrier is not None:
            barrier()
        self._release()


class TPGroup:
    """A tensor-parallel group: rank, world, the symmetric heap and the
    ``ls_tp_group`` struct the kernels take.  The sync region (flags and
    exchange slots) is carved first, so it sits at offset 0 of every heap."""

    def __init__(self, heap: SymmetricHeap, sync_bytes: int, barrier=None):
        self.heap = heap
        self.rank, self.world, self.device = heap.rank, heap.world, heap.device
        self.sync = heap.carve((max(int(sync_bytes), 256),), torch.uint8)
        if heap.offset_of(self.sync) != 0:
            raise RuntimeError("the sync region must be the heap's first allocation")
        self.sync.zero_()
        torch.cuda.synchronize(self.device)
        self.struct = N.TpGroup(world=self.world, rank=self.rank,
                                heap=(C.c_void_p * N.TP_MAX_RANKS)(*heap.peers, *([None] * (N.TP_MAX_RANKS - self.world))),
                                heap_bytes=heap.nbytes, sync_offset=0)
        if barrier is not None:
            barrier()  # every rank's flags are zero before any rank launches a TP kernel

    def reset(self, barrier):
        """Zero the sync region after a peer wait gave up (LS_DEV_TIMEOUT_PEER)."""
        torch.cuda.synchronize(self.device)
        barrier()
        self.sync.zero_()
        torch.cuda.synchronize(self.device)
        barrier()


def dist_helpers(pg=None):
    """(all_gather, barrier) callables over a torch.distributed process group."""
    import torch.distributed as dist

    def all_gather(b):
        out = [None] * dist.get_world_size(pg)
        dist.all_gather_object(out, b, group=pg)
        return out

    def barrier():
        dist.barrier(group=pg)

    return all_gather, barrier


# ----------------------------------------------------------------------------
# Engine
# ----------------------------------------------------------------------------


class TPDraftEngine:
    """One rank of a tensor-parallel drafting round.  Same inputs and outputs as
    ``engine.DraftEngine`` (every rank gets the same slots, lengths, anchors and
    page table, and ends with the same tokens), over this rank's head / feature
    / vocabulary shards.

    ``W_local``: ``shard_state_dict`` of the full state dict for this rank;
    ``pools``: this rank's ``ViewPools`` (``shard_views``); ``allreduce``:
    "fused" (``ls_gemm_allreduce``) or "nccl" (GEMM, then
    ``torch.distributed.all_reduce`` on ``pg``); ``wire``: partial format of the
    fused allreduce."""

    def __init__(self, shape: DraftShape, W_local: dict, pools: ViewPools, max_batch: int, *, rank, world, device,
                 all_gather, barrier, allreduce="fused", wire=N.TP_WIRE_F32, pg=None):
        if allreduce not in ("fused", "nccl"):
            raise ValueError("allreduce must be 'fused' or 'nccl'")
        self.shape = shape
        self.world, self.rank = world, rank
        self.loc = local_shape(shape, world)
        self.device = torch.device(device)
        self.allreduce, self.wire, self.pg = allreduce, wire, pg
        self.barrier = barrier
        s, ls_ = shape, self.loc
        self.w = DraftWeights(ls_, W_local, self.device)
        self.pools = pools
        self.max_batch = max_batch
        B, P = max_batch, s.block
        M = B * P
        H, V = s.hidden, s.vocab
        self.T, self.vshards = vocab_shards(V, world)
        self.n_vocab_local = self.vshards[rank][1]
        hq, hkv, Is, Hs = ls_.q_heads, ls_.kv_heads, ls_.inter, H // world
        dev = self.device
        bf = dict(dtype=torch.bfloat16, device=dev)
        # symmetric heap: sync region, then the buffers peers write (allreduce
        # outputs) or read (logits shard and tile maxima), same sizes on every rank
        sync = max(N.lib().ls_tp_sync_bytes(world, r, H, wire) for r in (B, M))
        Tv = self.T * 128
        heap_bytes = (sync + 4096 + (B + 2 * M) * H * 2 + M * Tv * 2 + 2 * M * self.T * 4 + 8 * 4096)
        heap = SymmetricHeap(heap_bytes, rank=rank, world=world, device=dev, all_gather=all_gather)
        self.group = TPGroup(heap, sync, barrier=barrier)
        nl = self.n_vocab_local
        self.buf = dict(
            u=heap.carve((B, H), torch.bfloat16), g=heap.carve((M, H), torch.bfloat16),
            h=heap.carve((M, H), torch.bfloat16),
            logits=heap.carve((M, Tv), torch.bfloat16).view(-1)[:M * nl].view(M, nl),
            tile_max=heap.carve((M, self.T), torch.float32).view(-1)[:M * (nl // 128)].view(M, nl // 128),
            tile_arg=heap.carve((M, self.T), torch.int32).view(-1)[:M * (nl // 128)].view(M, nl // 128),
            enc_in=torch.zeros(B, s.tap_layers * H, **bf), t=torch.zeros(B, Hs, **bf),
            xsh=torch.zeros(M, 2 * H, **bf), f1=torch.zeros(M, Hs, **bf), xn=torch.zeros(M, H, **bf),
            qkv=torch.zeros(M, (hq + 2 * hkv) * 128, **bf), attn=torch.zeros(M, hq * 128, **bf),
            act=torch.zeros(M, Is, **bf),
            positions=torch.zeros(M, dtype=torch.int32, device=dev),
            rope=torch.zeros(M, 128, dtype=torch.float32, device=dev),
            tokens=torch.zeros(B, P, dtype=torch.int64, device=dev),
            accept=torch.zeros(B, dtype=torch.int64, device=dev),
            status=torch.zeros(1, dtype=torch.int32, device=dev),
        )
        for k in ("u", "g", "h", "logits", "tile_max", "tile_arg"):
            self.buf[k].zero_()
        gemm_shapes = [(B, s.tap_layers * H, Hs), (B, Hs, H), (M, 2 * H, Hs), (M, Hs, H),
                       (M, H, (hq + 2 * hkv) * 128), (M, hq * 128, H), (M, H, 2 * Is), (M, Is, H), (M, H, nl)]
        ws = max(ops.gemm_workspace_bytes(r0, k, n) for (r0, k, n) in gemm_shapes)
        self.gemm_ws = torch.zeros(ws, dtype=torch.uint8, device=dev)
        self.attn_ws = torch.zeros(max(1, ops.attention_workspace_bytes(B, hq, hkv, s.window, s.slots)),
                                   dtype=torch.uint8, device=dev)
        self.markov_ws = torch.zeros(max(1, ops.markov_workspace_bytes(B, P)), dtype=torch.uint8, device=dev)
        if pools.summary_bf16 is None:
            pools.summary_bf16 = torch.empty(pools.summary_out.shape[0], s.draft_layers, hq, s.slots, 128,
                                             dtype=torch.bfloat16, device=dev)
            pools.sync_summary_bf16()
        self.graph_replays = 0
        self.refresh_after_qkv = True
        torch.cuda.synchronize(dev)
        barrier()

    # ------------------------------------------------------------------ pieces
    def _row_parallel(self, x, w, out, rows, residual=None):
        """out = sum over ranks of x_r . w_r^T (+ residual), on every rank."""
        epi = N.EPI_RESIDUAL if residual is not None else N.EPI_STORE
        st = self.buf["status"]
        if self.allreduce == "fused":
            ops.gemm_allreduce(x, w, out, group=self.group, workspace=self.gemm_ws, wire=self.wire, epilogue=epi,
                               rows=rows, residual=residual, status=st)
            return
        import torch.distributed as dist
        if residual is not None and self.rank == 0:
            ops.gemm(x, w, out, workspace=self.gemm_ws, epilogue=N.EPI_RESIDUAL, rows=rows, residual=residual,
                     status=st)
        else:
            ops.gemm(x, w, out, workspace=self.gemm_ws, epilogue=N.EPI_STORE, rows=rows, status=st)
        dist.all_reduce(out[:rows], group=self.pg)

    def refresh(self, *, slots, seq_lens, commit_lens, page_table, batch=None):
        p = self.pools
        ops.refresh_views(kv_k=p.kv_k, kv_v=p.kv_v, page_table=page_table, seq_lens=seq_lens,
                          commit_lens=commit_lens, slots=slots, learned_query=self.w.learned_query,
                          state_out=p.summary_out, state_lse=p.summary_lse, max_commit=self.shape.max_commit,
                          ring_pages=p.ring_pages, softmax_scale=self.shape.head_dim ** -0.5,
                          status=self.buf["status"], batch=batch, state_bf16=p.summary_bf16)

    def draft(self, *, slots, seq_lens, anchors, page_table, target=None, batch=None, slots_are_rows=False,
              commit_lens=None):
        """One drafter pass on this rank (see ``DraftEngine.draft``); every rank
        must call it with the same arguments."""
        s, ls_, w, p, b = self.shape, self.loc, self.w, self.pools, self.buf
        B = anchors.shape[0] if batch is None else batch
        P = s.block
        M = B * P
        ws = self.gemm_ws
        st = b["status"]
        if commit_lens is not None and not self.refresh_after_qkv:
            self.refresh(slots=slots, seq_lens=seq_lens, commit_lens=commit_lens, page_table=page_table, batch=B)
        if slots_are_rows:
            enc_in = p.hidden.view(p.hidden.shape[0], -1)
        else:
            enc_in = b["enc_in"]
            ops.gather_rows(p.hidden.view(p.hidden.shape[0], -1), slots, enc_in, rows=B, status=st)
        ops.gemm(enc_in, w.enc_w1, b["t"], workspace=ws, epilogue=N.EPI_SILU, rows=B, status=st)
        self._row_parallel(b["t"], w.enc_w2, b["u"], B)
        ops.shifted_input(anchors, seq_lens, b["positions"], w.embed, w.pos_emb, b["u"], b["xsh"],
                          block=P, mask_token_id=s.mask_token_id, status=st, inv_freq=w.inv_freq,
                          rope_table=b["rope"], batch=B, latest_norm_w=w.enc_norm, norm_eps=s.rms_eps)
        ops.gemm(b["xsh"], w.sh_w1, b["f1"], workspace=ws, epilogue=N.EPI_SILU, rows=M, status=st)
        self._row_parallel(b["f1"], w.sh_w2, b["g"], M)
        ops.rmsnorm(b["g"], w.sh_norm, b["h"], s.rms_eps, mode=0, rows=M, w2=w.layers[0]["in_norm"], out2=b["xn"])
        for j, L in enumerate(w.layers):
            v = s.view_layer(j)
            if j > 0:
                ops.rmsnorm(b["h"], L["in_norm"], b["xn"], s.rms_eps, mode=0, rows=M)
            ops.gemm(b["xn"], L["qkv"], b["qkv"], workspace=ws, epilogue=N.EPI_QKV, rows=M, q_heads=ls_.q_heads,
                     kv_heads=ls_.kv_heads, q_norm_w=L["q_norm"], k_norm_w=L["k_norm"], norm_eps=s.rms_eps,
                     positions=b["positions"], inv_freq=w.inv_freq, rope_table=b["rope"], status=st)
            if j == 0 and commit_lens is not None and self.refresh_after_qkv:
                self.refresh(slots=slots, seq_lens=seq_lens, commit_lens=commit_lens, page_table=page_table,
                             batch=B)
            ops.draft_attention(qkv=b["qkv"], block=P, kv_k=p.kv_k[v], kv_v=p.kv_v[v], page_table=page_table,
                                seq_lens=seq_lens, window=s.window, learned_query=w.learned_query[v],
                                state_out=p.summary_out[:, v], slots=slots, out=b["attn"], workspace=self.attn_ws,
                                q_heads=ls_.q_heads, kv_heads=ls_.kv_heads, ring_pages=p.ring_pages,
                                softmax_scale=s.head_dim ** -0.5, status=st, batch=B,
                                state_bf16=p.summary_bf16[:, v] if p.summary_bf16 is not None else None)
            self._row_parallel(b["attn"], L["o"], b["h"], M, residual=b["h"])
            ops.rmsnorm(b["h"], L["post_norm"], b["xn"], s.rms_eps, mode=0, rows=M)
            ops.gemm(b["xn"], L["gate_up"], b["act"], workspace=ws, epilogue=N.EPI_GATEUP, rows=M, status=st)
            self._row_parallel(b["act"], L["down"], b["h"], M, residual=b["h"])
        ops.rmsnorm(b["h"], w.final_norm, b["xn"], s.final_eps, mode=1, rows=M)
        ops.gemm(b["xn"], w.lm_head, b["logits"], workspace=ws, epilogue=N.EPI_LMHEAD, rows=M,
                 tile_max=b["tile_max"], tile_arg=b["tile_arg"], status=st)
        ops.tp_barrier(self.group, slot=0, status=st, device=self.device)
        ops.markov_argmax(base=b["logits"], tile_max=b["tile_max"], tile_arg=b["tile_arg"], anchors=anchors,
                          tokens=b["tokens"], block=P, workspace=self.markov_ws, w1=w.w1, w2=w.w2,
                          w1_bound=w.w1_bound, w2_bound=w.w2_bound, target=target,
                          accept_out=b["accept"] if target is not None else None, status=st, batch=B,
                          group=self.group, tiles_per_shard=self.T, vocab=s.vocab)

    def round(self, *, slots, seq_lens, commit_lens, anchors, page_table, target=None, batch=None,
              slots_are_rows=False):
        self.draft(slots=slots, seq_lens=seq_lens, anchors=anchors, page_table=page_table, target=target,
                   batch=batch, slots_are_rows=slots_are_rows, commit_lens=commit_lens)

    def device_status(self):
        return int(self.buf["status"].item())

    def clear_status(self):
        self.buf["status"].zero_()

    def close(self):
        """Free the symmetric heap (host barrier first)."""
        self.group.heap.close(barrier=self.barrier)
