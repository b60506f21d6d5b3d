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

import torch

from . import ops
from .config import DraftShape
from .engine import DraftEngine, DraftWeights, GraphedDraft, ViewPools
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

    # ------------------------------------------------------------------ state
    @property
    def requests(self):
        return self.table.requests

    @property
    def free_slots(self):
        return self.table.free_slots

    @torch.inference_mode()
    def update(self, packets, *, prefill=False):
        meta, counts, keys, values, hidden, extra = unpack_packets(packets)
        if not meta:
            return
        dev = self.device
        if prefill:
            if "global_output" not in extra:
                raise ValueError("prefill packets must carry global_output / global_lse")
            commit = self.table.prefill(meta, counts)
        else:
            commit = self.table.decode(meta, counts)
        B = len(meta)
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
        if prefill:
            self.pools.summary_out.index_copy_(0, slot_t.long(), extra["global_output"].to(dev, torch.float32))
            self.pools.summary_lse.index_copy_(0, slot_t.long(), extra["global_lse"].to(dev, torch.float32))
            self.pools.sync_summary_bf16(slot_t)
        else:
            self.engine.refresh(slots=slot_t, seq_lens=lens_t, commit_lens=cnt_t, page_table=table, batch=B)

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
    def propose(self, ids, anchors, temperature):
        if temperature != 0:
            raise NotImplementedError("sampled (T > 0) proposals are not implemented by the B200 drafter")
        dev = self.device
        B = len(ids)
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
        tokens = self.engine.buf["tokens"][:B].clone()
        logits = None
        if self.materialize_logits:
            s = self.shape
            if self._logits is None:
                self._logits = torch.empty(self.capacity * s.block, s.vocab, dtype=torch.bfloat16, device=dev)
            self.engine.corrected_logits(run_anchors, self._logits, batch=run_batch)
            logits = self._logits[:B * s.block].view(B, s.block, s.vocab).clone()
        return tokens, logits, None

    def release(self, ids):
        self.table.release(ids)

    def graph_stats(self):
        return dict(replays=self.engine.graph_replays, captured_batch_sizes=sorted(self.graphs),
                    fallbacks=self.fallbacks)

    def device_status(self):
        """Device status word of the kernels (0 = ok); synchronises."""
        return self.engine.device_status()
