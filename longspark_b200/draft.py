"""Drop-in drafter: the ``LongSparkDraft`` host API of ``src/longspark/engine/draft.py:72-291``
on the B200 kernels.

Kept from the reference: the constructor's keyword interface, ``update(packets,
prefill=...)`` with the ``longspark_state_batch_v1`` batch message
(``src/longspark/engine/state_export.py:50-66``) or per-request packet dicts,
``propose(ids, anchors, temperature) -> (tokens [B, P] int64, logits [B, P, V],
q)``, ``release(ids)``, ``graph_stats()``, and the attributes ``capacity``,
``device``, ``allocated_state_bytes``, ``position_audit``.  The error contract
is the reference's: ``RuntimeError("out-of-order LongSpark state commit")``
when ``previous + commit_len != length`` or the commit length is out of range,
``RuntimeError`` for an unavailable or already-owned slot, ``ValueError`` for a
batch whose tensors disagree with its metadata.

What changes is underneath: the recent window lives in page-granular rings
(16-row pages) read in place by the attention kernel, the summary refresh and
the window scatter are two launches for the whole batch, and the drafter pass
(state encoder through the Markov greedy chain) replays as one CUDA graph.
"""

from __future__ import annotations

import json
import math
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

from . import ops
from .config import DraftShape
from .engine import DraftEngine, DraftWeights, GraphedDraft, ViewPools, capture_guard
from .requests import RequestTable, unpack_packets

GIB = 1 << 30


def _cfg(config, name, default=None):
    if isinstance(config, dict):
        return config.get(name, default)
    return getattr(config, name, default)


def load_weights(model_path, draft_path):
    """Reference-named weights from safetensors: the drafter checkpoint plus the
    target's ``model.embed_tokens``, ``lm_head`` (tied to the embedding when
    ``tie_word_embeddings``) and ``model.norm`` (``src/longspark/engine/draft.py:24-48``)."""
    from safetensors.torch import load_file

    W = {}
    for f in sorted(Path(draft_path).glob("*.safetensors")):
        W.update(load_file(str(f)))
    root = Path(model_path)
    cfg = json.loads((root / "config.json").read_text())
    index = root / "model.safetensors.index.json"
    wmap = json.loads(index.read_text())["weight_map"] if index.exists() else {}
    names = ("model.embed_tokens.weight", "lm_head.weight", "model.norm.weight")
    cache = {}
    for name in names:
        if name == "lm_head.weight" and cfg.get("tie_word_embeddings"):
            W[name] = W["model.embed_tokens.weight"]
            continue
        fname = wmap.get(name, "model.safetensors")
        if fname not in cache:
            cache[fname] = load_file(str(root / fname))
        W[name] = cache[fname][name]
    return W, cfg


def shape_from_checkpoint(draft_path, target_cfg, **overrides):
    """``DraftShape`` from a DraftFreeKV ``config.json`` (``vendor/specforge/modeling/draft/
    draftfreekv.py:1211-1460`` field names) and the target's config."""
    c = json.loads((Path(draft_path) / "config.json").read_text())
    kw = dict(hidden=c["hidden_size"], q_heads=c.get("qwen_num_attention_heads"), kv_heads=c["num_key_value_heads"],
              head_dim=c.get("head_dim", 128), inter=c.get("qwen_intermediate_size"), vocab=c["vocab_size"],
              tap_layers=len(c["target_layer_ids"]), draft_layers=c.get("parallel_mixer_layers", 5),
              slots=c.get("global_memory_slots", 16), window=c.get("raw_target_rows", 256),
              block=c.get("block_size", 7), max_commit=c.get("max_accepted_tokens", 8),
              markov_rank=c.get("parallel_markov_rank", 0), mask_token_id=c["mask_token_id"],
              rms_eps=c.get("qwen_rms_norm_eps", 1e-6), final_eps=target_cfg.get("rms_norm_eps", 1e-6),
              rope_theta=c.get("qwen_rope_theta", 1_000_000.0))
    kw.update(overrides)
    return DraftShape(**kw)


class LongSparkDraft:
    """B200 drafter with the reference ``LongSparkDraft`` interface.

    ``config`` supplies ``draft_device``, ``max_running_requests``,
    ``draft_state_gib``, ``cuda_graph``, ``graph_batch_sizes`` (attribute or key
    access).  Weights come from ``model_path``/``draft_path`` (safetensors), or
    directly from ``weights`` (a reference-named state dict) with ``shape``."""

    def __init__(self, config, *, model_path=None, draft_path=None, target_ready=None, shape=None,
                 weights=None, materialize_logits=True):
        self.device = torch.device("cuda", int(_cfg(config, "draft_device", 0)))
        torch.cuda.set_device(self.device)
        if weights is None:
            if model_path is None or draft_path is None:
                raise ValueError("LongSparkDraft needs model_path and draft_path, or weights and shape")
            weights, target_cfg = load_weights(model_path, draft_path)
            shape = shape or shape_from_checkpoint(draft_path, target_cfg)
        if shape is None:
            raise ValueError("a DraftShape is required with explicit weights")
        self.shape = shape
        self.position_audit = dict(position_variant=_cfg(config, "position_variant", "native"),
                                   theta=shape.rope_theta, layer_count=shape.draft_layers, weights_changed=False)
        self.weights = DraftWeights(shape, weights, self.device)
        s = shape
        ring = s.window // s.page_size
        per_request = s.tap_layers * s.window * s.kv_heads * s.head_dim * 2 * 2
        per_request += s.tap_layers * s.q_heads * s.slots * (s.head_dim + 1) * 4
        per_request += s.tap_layers * s.hidden * 2
        budget = int(float(_cfg(config, "draft_state_gib", 8.0)) * GIB)
        self.capacity = min(int(_cfg(config, "max_running_requests", 64)), budget // per_request)
        if self.capacity < 1:
            raise ValueError("draft state budget cannot fit one LongSpark request")
        n = self.capacity
        dev = self.device
        table = (torch.arange(n, dtype=torch.int32, device=dev)[:, None] * ring
                 + torch.arange(ring, dtype=torch.int32, device=dev)[None, :])
        self.pools = ViewPools(
            kv_k=torch.zeros(s.tap_layers, n * ring, s.page_size, s.kv_heads, s.head_dim, dtype=torch.bfloat16,
                             device=dev),
            kv_v=torch.zeros(s.tap_layers, n * ring, s.page_size, s.kv_heads, s.head_dim, dtype=torch.bfloat16,
                             device=dev),
            page_table=table.contiguous(),
            summary_out=torch.zeros(n, s.tap_layers, s.q_heads, s.slots, s.head_dim, dtype=torch.float32,
                                    device=dev),
            summary_lse=torch.full((n, s.tap_layers, s.q_heads, s.slots), float("-inf"), dtype=torch.float32,
                                   device=dev),
            hidden=torch.zeros(n, s.tap_layers, s.hidden, dtype=torch.bfloat16, device=dev),
            ring_pages=ring)
        self.allocated_state_bytes = sum(t.numel() * t.element_size() for t in (
            self.pools.kv_k, self.pools.kv_v, self.pools.summary_out, self.pools.summary_lse, self.pools.hidden))
        self.engine = DraftEngine(s, self.weights, self.pools, max_batch=n, device=dev)
        self.table = RequestTable(n, s.max_commit, s.window)
        self.materialize_logits = materialize_logits
        self.use_graph = bool(_cfg(config, "cuda_graph", True))
        sizes = _cfg(config, "graph_batch_sizes", ()) or ()
        self.graph_sizes = sorted({b for b in sizes if b <= n} | {n})
        self.graphs = {}
        self.fallbacks = 0
        self._logits = None
        # T > 0: every proposal draws with a fresh seed derived from this one
        self._temperature = 0.0
        self._sample_seed = int(_cfg(config, "seed", 0))
        self._sample_round = 0
        # Step path: a decode update stages its rows and metadata and launches
        # nothing; the next propose for the same requests replays one graph
        # (page-table gather, window scatter, drafter pass with the refresh).
        rows = n * s.max_commit
        self._stage_k = torch.zeros(s.tap_layers, rows, s.kv_heads, s.head_dim, dtype=torch.bfloat16, device=dev)
        self._stage_v = torch.zeros_like(self._stage_k)
        self._stage_h = torch.zeros(n, s.tap_layers * s.hidden, dtype=torch.bfloat16, device=dev)
        # metadata block: slots, lengths, counts, offsets (int32 x n each), anchors (int64 x n)
        self._meta_bytes = 4 * 4 * n + 8 * n
        self._meta_host = torch.zeros(self._meta_bytes, dtype=torch.uint8).pin_memory()
        hb = self._meta_host.numpy()  # numpy views of the pinned block: writes cost no torch op
        self._meta_np = (hb[:4 * n].view(np.int32), hb[4 * n:8 * n].view(np.int32), hb[8 * n:12 * n].view(np.int32),
                         hb[12 * n:16 * n].view(np.int32), hb[16 * n:].view(np.int64))
        self._meta_dev = torch.zeros(self._meta_bytes, dtype=torch.uint8, device=dev)
        self._meta_done = torch.cuda.Event()  # the last copy out of the host block has run
        self._meta_done.record()
        self._pending = None  # (ids, batch) of a staged, not yet applied decode update
        self._pending_in_pool = None  # (slots, lengths, counts) of rows exported in place, not yet folded
        self._step_graphs = {}

    # ------------------------------------------------------------------ state
    @property
    def requests(self):
        return self.table.requests

    @property
    def free_slots(self):
        return self.table.free_slots

    # ------------------------------------------------------------------ staging
    def _meta_views(self, t):
        """(slots, lengths, counts, offsets, anchors) views of a metadata block."""
        n = self.capacity
        i32 = t[:16 * n].view(torch.int32)
        return i32[:n], i32[n:2 * n], i32[2 * n:3 * n], i32[3 * n:], t[16 * n:].view(torch.int64)

    def _host_meta(self):
        """numpy views (slots, lengths, counts, offsets, anchors) of the pinned
        host metadata block, once its previous copy has run."""
        self._meta_done.synchronize()
        return self._meta_np

    def _push_meta(self):
        self._meta_dev.copy_(self._meta_host, non_blocking=True)
        self._meta_done.record()

    def _flush(self):
        """Apply a staged decode update now (window scatter + refresh)."""
        if self._pending_in_pool is not None:
            slot_t, lens_t, cnt_t = self._pending_in_pool
            self._pending_in_pool = None
            table = self.pools.page_table.index_select(0, slot_t)
            self.engine.refresh(slots=slot_t, seq_lens=lens_t, commit_lens=cnt_t, page_table=table,
                                batch=slot_t.shape[0])
        if self._pending is None:
            return
        ids, B = self._pending
        self._pending = None
        self._push_meta()
        slot_t, lens_t, cnt_t, off_t, _ = (v[:B] for v in self._meta_views(self._meta_dev))
        table = self.pools.page_table.index_select(0, slot_t)
        st = self.engine.buf["status"]
        ops.window_scatter(keys=self._stage_k, values=self._stage_v, row_offsets=off_t, counts=cnt_t, seq_lens=lens_t,
                           kv_k=self.pools.kv_k, kv_v=self.pools.kv_v, page_table=table,
                           ring_pages=self.pools.ring_pages, last_hidden=self._stage_h, hidden_pool=self.pools.hidden,
                           slots=slot_t, status=st, batch=B)
        self.engine.refresh(slots=slot_t, seq_lens=lens_t, commit_lens=cnt_t, page_table=table, batch=B)

    def export_destination(self, ids, lengths, commit_lens, device=None):
        """Where a target stores this decode step's rows in place
        (``export.export_rows``): validates the commit exactly as the
        matching ``update`` will (unknown request, out-of-order commit) and
        returns the pool addresses, the requests' page-table rows, slots and
        post-commit lengths, with the index arrays on ``device`` (the exporting
        GPU; peer access to this drafter's GPU is enabled from it).  After the
        export has run, ``update`` with a message whose ``keys`` is None
        (``export_counts`` = ``commit_lens``) folds the rows into the summary."""
        from .export import ExportDestination, enable_peer_access

        meta = [dict(id=i, length=n, commit_len=c) for i, n, c in zip(ids, lengths, commit_lens, strict=True)]
        self._flush()
        slot_list = self.table.check_decode(meta, list(commit_lens))
        dev = self.device
        slots = torch.tensor(slot_list, dtype=torch.int32, device=dev)
        p, s = self.pools, self.shape
        dest = ExportDestination(
            kv_k=p.kv_k.data_ptr(), kv_v=p.kv_v.data_ptr(), pool_pages=p.kv_k.shape[1], heads=s.kv_heads,
            tap_layers=s.tap_layers, ring_pages=p.ring_pages, page_table=p.page_table.index_select(0, slots),
            seq_lens=torch.tensor(list(lengths), dtype=torch.int32, device=dev), slots=slots,
            hidden_pool=p.hidden.data_ptr(), capacity=p.hidden.shape[0], hidden=s.hidden, keepalive=p)
        if device is not None and torch.device(device) != dev:
            enable_peer_access(device, dev)
            dest = dest.to(device)
        return dest

    @torch.inference_mode()
    def update(self, packets, *, prefill=False):
        meta, counts, keys, values, hidden, extra = unpack_packets(packets)
        if not meta:
            return
        self._flush()
        dev = self.device
        if keys is None:
            # rows and hidden states already stored in place by the target
            # (export.export_rows into export_destination): fold them in at the
            # next proposal
            if prefill:
                raise ValueError("prefill messages carry their rows and summary state")
            commit = self.table.decode(meta, counts)
            self._pending_in_pool = (torch.tensor(commit.slots, dtype=torch.int32, device=dev),
                                     torch.tensor(commit.lengths, dtype=torch.int32, device=dev),
                                     torch.tensor(commit.counts, dtype=torch.int32, device=dev))
            return
        if prefill:
            if "global_output" not in extra:
                raise ValueError("prefill packets must carry global_output / global_lse")
            commit = self.table.prefill(meta, counts)
        else:
            commit = self.table.decode(meta, counts)
        B = len(meta)
        if not prefill:
            # stage rows and metadata; the next propose of these requests applies them
            total = keys.shape[1]
            self._stage_k[:, :total].copy_(keys, non_blocking=True)
            self._stage_v[:, :total].copy_(values, non_blocking=True)
            self._stage_h[:B].copy_(hidden.reshape(B, -1), non_blocking=True)
            slot_h, lens_h, cnt_h, off_h, _ = self._host_meta()
            slot_h[:B] = commit.slots
            lens_h[:B] = commit.lengths
            cnt_h[:B] = commit.counts
            off_h[:B] = commit.offsets
            self._pending = (tuple(m["id"] for m in meta), B)
            return
        slot_t = torch.tensor(commit.slots, dtype=torch.int32, device=dev)
        lens_t = torch.tensor(commit.lengths, dtype=torch.int32, device=dev)
        cnt_t = torch.tensor(commit.counts, dtype=torch.int32, device=dev)
        off_t = torch.tensor(commit.offsets, dtype=torch.int32, device=dev)
        table = self.pools.page_table.index_select(0, slot_t)
        st = self.engine.buf["status"]
        ops.window_scatter(keys=keys.to(dev, torch.bfloat16).contiguous(),
                           values=values.to(dev, torch.bfloat16).contiguous(), row_offsets=off_t, counts=cnt_t,
                           seq_lens=lens_t, kv_k=self.pools.kv_k, kv_v=self.pools.kv_v, page_table=table,
                           ring_pages=self.pools.ring_pages, last_hidden=hidden.to(dev, torch.bfloat16).contiguous(),
                           hidden_pool=self.pools.hidden, slots=slot_t, status=st)
        self.pools.summary_out.index_copy_(0, slot_t.long(), extra["global_output"].to(dev, torch.float32))
        self.pools.summary_lse.index_copy_(0, slot_t.long(), extra["global_lse"].to(dev, torch.float32))
        self.pools.sync_summary_bf16(slot_t)

    # ------------------------------------------------------------------ propose
    def _graph_for(self, batch):
        for size in self.graph_sizes:
            if size >= batch:
                if size not in self.graphs:
                    self.graphs[size] = GraphedDraft(self.engine, size, with_refresh=False, with_target=False)
                    self.graphs[size].load(slots=self._pad_slots(size), seq_lens=self._pad_lens(size),
                                           anchors=torch.zeros(size, dtype=torch.int64, device=self.device),
                                           page_table=self.pools.page_table[:1].expand(size, -1))
                    self.graphs[size].capture()
                return self.graphs[size]
        return None

    def _pad_slots(self, size):
        return torch.zeros(size, dtype=torch.int32, device=self.device)

    def _pad_lens(self, size):
        return torch.ones(size, dtype=torch.int32, device=self.device)

    @torch.inference_mode()
    def _step_graph(self, B, with_logits):
        """Graph of one full step for exactly B requests: page-table gather,
        window scatter of the staged rows, drafter pass with the refresh, and
        with ``with_logits`` the corrected logits of the greedy chain."""
        g = self._step_graphs.get((B, with_logits))
        if g is None:
            g = StepGraph(self, B, with_logits=with_logits)
            self._step_graphs[(B, with_logits)] = g
        return g

    def _logits_buffer(self):
        if self._logits is None:
            s = self.shape
            self._logits = torch.empty(self.capacity * s.block, s.vocab, dtype=torch.bfloat16, device=self.device)
        return self._logits

    def propose(self, ids, anchors, temperature):
        if temperature < 0:
            raise ValueError("temperature must be >= 0")
        self._temperature = float(temperature)
        dev = self.device
        B = len(ids)
        if self._pending is not None and self.use_graph and self._pending[0] == tuple(ids):
            self.table.lookup(ids)  # the reference's unknown-request error
            _, _, _, _, anc_h = self._host_meta()
            on_device = torch.is_tensor(anchors) and anchors.is_cuda
            if not on_device:
                anc_h[:B] = anchors.reshape(-1).numpy() if torch.is_tensor(anchors) else np.asarray(anchors)
            self._pending = None
            self._push_meta()
            if on_device:  # device anchors (e.g. the target's bonus tokens): no host round trip
                self._meta_views(self._meta_dev)[4][:B].copy_(anchors.reshape(-1))
            # at T = 0 the corrected logits of the greedy chain are part of the step graph
            with_logits = self.materialize_logits and self._temperature == 0
            g = self._step_graph(B, with_logits)
            g.replay()
            self.engine.graph_replays += 1
            return self._propose_outputs(B, self._meta_views(self._meta_dev)[4][:B], B, logits_ready=with_logits)
        self._flush()
        slot_list, len_list = self.table.lookup(ids)
        slots = torch.tensor(slot_list, dtype=torch.int32, device=dev)
        lengths = torch.tensor(len_list, dtype=torch.int32, device=dev)
        anchor_t = torch.as_tensor(anchors, dtype=torch.long).to(dev)
        table = self.pools.page_table.index_select(0, slots)
        graph = self._graph_for(B) if self.use_graph else None
        if graph is not None:
            size = graph.batch
            if size > B:  # pad by repeating the last request (its outputs are discarded)
                pad = size - B
                slots = torch.cat([slots, slots[-1:].expand(pad)])
                lengths = torch.cat([lengths, lengths[-1:].expand(pad)])
                anchor_t = torch.cat([anchor_t, anchor_t[-1:].expand(pad)])
                table = torch.cat([table, table[-1:].expand(pad, -1)])
            graph.load(slots=slots, seq_lens=lengths, anchors=anchor_t, page_table=table)
            graph.replay()
            run_batch, run_anchors = size, anchor_t
        else:
            self.engine.draft(slots=slots, seq_lens=lengths, anchors=anchor_t, page_table=table, batch=B)
            run_batch, run_anchors = B, anchor_t
        return self._propose_outputs(B, run_anchors, run_batch)

    def _propose_outputs(self, B, run_anchors, run_batch, logits_ready=False):
        if self._temperature > 0:
            return self._sampled_outputs(B, run_anchors, run_batch)
        tokens = self.engine.buf["tokens"][:B].clone()
        logits = None
        if self.materialize_logits:
            s = self.shape
            if not logits_ready:
                self.engine.corrected_logits(run_anchors, self._logits_buffer(), batch=run_batch)
            logits = self._logits[:B * s.block].view(B, s.block, s.vocab).clone()
        return tokens, logits, None

    def _sampled_outputs(self, B, run_anchors, run_batch):
        """T > 0: the step loop over the pass's base logits (``DraftEngine.sample``)
        with a fresh seed per proposal; returns (tokens, corrected logits or
        None, q) like ``LongSparkDraft.propose`` (LS engine/draft.py:281-286)."""
        s = self.shape
        self._sample_round += 1
        seed = (self._sample_seed * 0x9E3779B97F4A7C15 + self._sample_round) & (2 ** 64 - 1)
        corr = self.engine.sample(run_anchors[:run_batch], temperature=self._temperature, seed=seed,
                                  corrected=self._logits_buffer() if self.materialize_logits else None,
                                  batch=run_batch)
        tokens = self.engine.buf["tokens"][:B].clone()
        q = self.engine.buf["q"][:B].clone()
        logits = corr[:B].clone() if self.materialize_logits else None
        return tokens, logits, q

    def release(self, ids):
        self._flush()
        self.table.release(ids)

    def graph_stats(self):
        return dict(replays=self.engine.graph_replays, captured_batch_sizes=sorted(self.graphs),
                    fallbacks=self.fallbacks)

    def device_status(self):
        """Device status word of the kernels (0 = ok); synchronises."""
        return self.engine.device_status()


class StepGraph:
    """CUDA graph of one full drafting step for a fixed batch B, reading the
    drafter's staged rows and metadata block: gather of the requests' page-table
    rows, window scatter of the committed K/V rows and boundary hidden states,
    then the drafter pass with the view refresh (``DraftEngine.draft``), and
    with ``with_logits`` the Markov-corrected logits of the greedy chain into
    the drafter's logits buffer (``DraftEngine.corrected_logits``)."""

    def __init__(self, d: "LongSparkDraft", B: int, with_logits: bool = False):
        self.d, self.B, self.with_logits = d, B, with_logits
        if with_logits:
            d._logits_buffer()
        slot_t, lens_t, cnt_t, off_t, anc_t = (v[:B] for v in d._meta_views(d._meta_dev))
        self.args = (slot_t, lens_t, cnt_t, off_t, anc_t)
        self.table = torch.zeros(B, d.pools.page_table.shape[1], dtype=torch.int32, device=d.device)
        s = torch.cuda.Stream(device=d.device)
        s.wait_stream(torch.cuda.current_stream(d.device))
        with torch.cuda.stream(s):
            # warm-up (kernel attributes, module loading) without the refresh:
            # the scatter is idempotent, the refresh would fold the rows twice
            torch.index_select(d.pools.page_table, 0, self.args[0], out=self.table)
            d.engine.draft(slots=self.args[0], seq_lens=self.args[1], anchors=self.args[4], page_table=self.table,
                           batch=B)
            if with_logits:
                d.engine.corrected_logits(self.args[4], d._logits, batch=B)
        torch.cuda.current_stream(d.device).wait_stream(s)
        torch.cuda.synchronize(d.device)
        self.graph = torch.cuda.CUDAGraph()
        with capture_guard(), torch.cuda.graph(self.graph, stream=s):
            self._run()
        torch.cuda.current_stream(d.device).wait_stream(s)

    def _run(self):
        d, B = self.d, self.B
        slot_t, lens_t, cnt_t, off_t, anc_t = self.args
        torch.index_select(d.pools.page_table, 0, slot_t, out=self.table)
        ops.window_scatter(keys=d._stage_k, values=d._stage_v, row_offsets=off_t, counts=cnt_t, seq_lens=lens_t,
                           kv_k=d.pools.kv_k, kv_v=d.pools.kv_v, page_table=self.table,
                           ring_pages=d.pools.ring_pages, last_hidden=d._stage_h, hidden_pool=d.pools.hidden,
                           slots=slot_t, status=d.engine.buf["status"], batch=B)
        d.engine.draft(slots=slot_t, seq_lens=lens_t, anchors=anc_t, page_table=self.table, batch=B,
                       commit_lens=cnt_t)
        if self.with_logits:
            d.engine.corrected_logits(anc_t, d._logits, batch=B)

    def replay(self):
        self.graph.replay()
