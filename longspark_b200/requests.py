"""Host-side request bookkeeping of the drafter (no device work): pool slots,
committed lengths, packet validation, and request sharding across GPUs.

The validation rules are the reference's (``src/longspark/engine/draft.py``):
a prefill needs a free slot and an id not already owned (:190-191); a decode
commit must satisfy ``previous + commit_len == length`` and
``1 <= commit_len <= max_commit`` (:226-229, ``RuntimeError("out-of-order
LongSpark state commit")``); a batch message must carry exactly the committed
rows (:238-239, ``ValueError``).  The batch message format is
``longspark_state_batch_v1`` (``src/longspark/engine/state_export.py:50-66``).
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass, field

BATCH_FORMAT = "longspark_state_batch_v1"


@dataclass
class Commit:
    slots: list
    lengths: list
    counts: list
    offsets: list


class RequestTable:
    """Slot allocation and commit validation for ``capacity`` pool slots."""

    def __init__(self, capacity: int, max_commit: int, window: int):
        if capacity < 1:
            raise ValueError("draft state budget cannot fit one LongSpark request")
        self.capacity = capacity
        self.max_commit = max_commit
        self.window = window
        self.free_slots = list(range(capacity))
        self.requests = {}  # id -> [slot, committed length]

    def prefill(self, meta, counts):
        """Claim slots for new requests; returns the commit description."""
        for m in meta:
            if m["id"] in self.requests:
                raise RuntimeError("LongSpark request slot unavailable or already owned")
        if len(meta) > len(self.free_slots) or len({m["id"] for m in meta}) != len(meta):
            raise RuntimeError("LongSpark request slot unavailable or already owned")
        for m, c in zip(meta, counts):
            if c != min(m["length"], self.window):
                raise ValueError("prefill must export the last min(length, window) K/V rows")
        slots = []
        for m in meta:
            slot = self.free_slots.pop()
            self.requests[m["id"]] = [slot, m["length"]]
            slots.append(slot)
        return Commit(slots, [m["length"] for m in meta], list(counts), _offsets(counts))

    def check_decode(self, meta, counts):
        """Validate a decode commit for every request without applying it;
        returns the requests' slots."""
        slots = []
        for m, c in zip(meta, counts):
            if m["id"] not in self.requests:
                raise RuntimeError("unknown LongSpark request")
            slot, previous = self.requests[m["id"]]
            if previous + m["commit_len"] != m["length"] or not 1 <= m["commit_len"] <= self.max_commit:
                raise RuntimeError("out-of-order LongSpark state commit")
            if c != m["commit_len"]:
                raise ValueError("decode batch must contain exactly the committed KV rows")
            slots.append(slot)
        return slots

    def decode(self, meta, counts):
        """Validate a decode commit for every request first, then apply it."""
        slots = self.check_decode(meta, counts)
        for m in meta:
            self.requests[m["id"]][1] = m["length"]
        return Commit(slots, [m["length"] for m in meta], list(counts), _offsets(counts))

    def lookup(self, ids):
        try:
            return [self.requests[i][0] for i in ids], [self.requests[i][1] for i in ids]
        except KeyError as e:
            raise RuntimeError(f"unknown LongSpark request {e.args[0]!r}") from None

    def release(self, ids):
        for rid in ids:
            slot, _ = self.requests.pop(rid)
            self.free_slots.append(slot)


def _offsets(counts):
    out, acc = [], 0
    for c in counts:
        out.append(acc)
        acc += c
    return out


def unpack_packets(packets):
    """(meta, counts, keys, values, last_hidden, extra) from a batch message or
    a list of per-request packets (``unpack_longspark_states`` semantics)."""
    import torch

    if isinstance(packets, dict):
        if packets.get("format") != BATCH_FORMAT:
            raise ValueError("unknown batched LongSpark state format")
        meta = [dict(id=i, length=l, commit_len=c) for i, l, c in
                zip(packets["ids"], packets["lengths"], packets["commit_lens"], strict=True)]
        counts = list(packets["export_counts"])
        if len(counts) != len(meta):
            raise ValueError("batched export counts disagree with request metadata")
        keys, values = packets.get("keys"), packets.get("values")
        extra = {k: packets[k] for k in ("global_output", "global_lse") if k in packets}
        if keys is None:  # rows and hidden states already stored in place (export.export_rows)
            if values is not None or packets.get("last_hidden") is not None:
                raise ValueError("a message without keys carries no values or hidden states either")
            return meta, counts, None, None, None, extra
        if keys.shape != values.shape or keys.shape[1] != sum(counts):
            raise ValueError("batched tensor extent disagrees with export counts")
        return meta, counts, keys, values, packets["last_hidden"], extra
    meta = [dict(id=p["id"], length=p["length"], commit_len=p.get("commit_len", p["keys"].shape[1]))
            for p in packets]
    counts = [p["keys"].shape[1] for p in packets]
    if not packets:
        return meta, counts, None, None, None, {}
    keys = torch.cat([p["keys"] for p in packets], dim=1)
    values = torch.cat([p["values"] for p in packets], dim=1)
    hidden = torch.stack([p["last_hidden"] for p in packets])
    extra = {}
    if "global_output" in packets[0]:
        extra = dict(global_output=torch.stack([p["global_output"] for p in packets]),
                     global_lse=torch.stack([p["global_lse"] for p in packets]))
    return meta, counts, keys, values, hidden, extra


def owner_rank(request_id, world_size: int) -> int:
    """Rank that owns a request under request sharding (stable across processes:
    CRC32 of the id's text, not Python's salted ``hash``)."""
    return zlib.crc32(str(request_id).encode()) % world_size


def shard(ids, world_size: int, rank: int):
    """The ids (in order) this rank drafts for."""
    return [i for i in ids if owner_rank(i, world_size) == rank]


def split_batch_message(payload, world_size: int, rank: int):
    """The part of a ``longspark_state_batch_v1`` message owned by ``rank`` (no
    cross-GPU traffic: each rank keeps only its requests' rows)."""
    import torch

    meta = list(zip(payload["ids"], payload["lengths"], payload["commit_lens"], payload["export_counts"]))
    offs = _offsets(payload["export_counts"])
    keep = [k for k, m in enumerate(meta) if owner_rank(m[0], world_size) == rank]
    rows = [r for k in keep for r in range(offs[k], offs[k] + meta[k][3])]
    idx = torch.tensor(rows, dtype=torch.long)
    out = dict(format=BATCH_FORMAT, ids=[meta[k][0] for k in keep], lengths=[meta[k][1] for k in keep],
               commit_lens=[meta[k][2] for k in keep], export_counts=[meta[k][3] for k in keep],
               keys=payload["keys"].index_select(1, idx.to(payload["keys"].device)),
               values=payload["values"].index_select(1, idx.to(payload["values"].device)),
               last_hidden=payload["last_hidden"][torch.tensor(keep, dtype=torch.long)])
    for k in ("global_output", "global_lse"):
        if k in payload:
            out[k] = payload[k][torch.tensor(keep, dtype=torch.long)]
    return out
