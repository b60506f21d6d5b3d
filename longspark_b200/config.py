"""Shapes of the drafting round and the benchmark presets.

``DraftShape`` gathers every dimension the drafting kernels need.  The
reference hard-codes several of them (16 summary slots, a 256-row window,
7 drafter rows, at most 8 committed rows: ``vendor/specforge/modeling/draft/
global16_raw256.py:62-69``); here they are parameters so the benchmark shapes
(S=64/256, W=512..2048, a 16-token verify block) run on the same kernels.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

QWEN3_VOCAB = 151936


@dataclass(frozen=True)
class DraftShape:
    hidden: int = 4096            # H
    q_heads: int = 32             # Hq
    kv_heads: int = 8             # Hkv
    head_dim: int = 128           # D (the kernels require 128)
    inter: int = 12288            # I, SwiGLU width
    vocab: int = QWEN3_VOCAB      # V
    tap_layers: int = 5           # L_tap: target layers whose views the drafter keeps
    draft_layers: int = 1         # L_draft: drafter decoder layers
    slots: int = 256              # S: learned summary queries per (layer, q-head)
    window: int = 1024            # W: recent target K/V rows
    block: int = 15               # P: drafter rows (proposals) per round
    max_commit: int = 16          # most K/V rows committed per round (anchor + accepted)
    page_size: int = 16           # rows per KV-cache page
    markov_rank: int = 256        # rank of the Markov previous-token bias (0 = none)
    mask_token_id: int = 151643
    rms_eps: float = 1e-6
    final_eps: float = 1e-6
    rope_theta: float = 1_000_000.0

    def __post_init__(self):
        if self.head_dim != 128:
            raise ValueError("the drafting kernels are written for head_dim 128")
        if self.q_heads % self.kv_heads:
            raise ValueError("q_heads must be a multiple of kv_heads")
        if self.hidden % 128 or self.inter % 64 or self.vocab % 128:
            raise ValueError("hidden must be a multiple of 128, inter of 64, vocab of 128")
        if not 1 <= self.block <= 16:
            raise ValueError("block (drafter rows) must be in [1, 16]")
        if not 1 <= self.max_commit <= 32:
            raise ValueError("max_commit must be in [1, 32]")
        if self.window % self.page_size or self.page_size != 16:
            raise ValueError("page_size must be 16 and divide the window")
        if self.slots % 16 or self.slots > 512:
            raise ValueError("slots must be a multiple of 16, at most 512")
        if not 1 <= self.draft_layers <= self.tap_layers:
            raise ValueError("draft_layers must be in [1, tap_layers]")
        if self.markov_rank % 64 and self.markov_rank != 0:
            raise ValueError("markov_rank must be 0 or a multiple of 64")
        if not 0 <= self.mask_token_id < self.vocab:
            raise ValueError("mask_token_id out of range")

    @property
    def group(self) -> int:
        return self.q_heads // self.kv_heads

    def view_layer(self, draft_layer: int) -> int:
        """Tapped layer whose views drafter layer ``draft_layer`` attends to.

        The reference pairs drafter layer j with tapped layer j and requires
        equal counts (``vendor/specforge/modeling/draft/draftfreekv.py:3275-3280``);
        with fewer drafter layers than taps, drafter layer j reads tap j."""
        return draft_layer

    def with_(self, **kw) -> "DraftShape":
        return replace(self, **kw)


# The reference contract (Global16 / Raw256 / Local7, at most 8 committed rows).
REFERENCE_CONTRACT = dict(slots=16, window=256, block=7, max_commit=8)

QWEN3_4B = dict(hidden=2560, q_heads=32, kv_heads=8, inter=9728)
QWEN3_8B = dict(hidden=4096, q_heads=32, kv_heads=8, inter=12288)
QWEN3_14B = dict(hidden=5120, q_heads=40, kv_heads=8, inter=17408)


@dataclass(frozen=True)
class Workload:
    """One benchmark configuration (BASELINE.json ``configs``)."""
    name: str
    shape: DraftShape
    batch: int
    contexts: tuple = (4096,)
    rounds: int = 1
    notes: str = ""
    extra: dict = field(default_factory=dict)


# Verify block B=16 of the benchmark configs = anchor + 15 proposals, so the
# drafter runs P=15 rows and up to 16 rows are committed per round.
CFG1 = Workload("cfg1-qwen3-4b-ctx4k", DraftShape(**QWEN3_4B, tap_layers=1, draft_layers=1,
                                                  slots=64, window=512, block=15, max_commit=16),
                batch=1, contexts=(4096,))
CFG2 = Workload("cfg2-qwen3-8b", DraftShape(**QWEN3_8B, tap_layers=5, draft_layers=1,
                                            slots=256, window=1024, block=15, max_commit=16),
                batch=1, contexts=(1024, 8192, 32768, 65536, 131072))
CFG3 = Workload("cfg3-qwen3-14b-ctx128k", DraftShape(**QWEN3_14B, tap_layers=5, draft_layers=1,
                                                     slots=256, window=2048, block=15, max_commit=16),
                batch=1, contexts=(131072,), rounds=200)
CFG4 = Workload("cfg4-qwen3-8b-concurrency", CFG2.shape, batch=64, contexts=(2048, 32768),
                notes="per-request context uniform in [2K, 32K]")
CFG5 = Workload("cfg5-qwen3-14b-tp", CFG3.shape, batch=32, contexts=(65536,))

WORKLOADS = {w.name: w for w in (CFG1, CFG2, CFG3, CFG4, CFG5)}
