"""Target-side export of the accepted rows straight into a drafter's pool.

The reference's target gathers the accepted K/V rows of every tapped layer
(``TargetModel._kv_rows``, src/longspark/engine/target.py:213-228, and
``gather_selected_kv``, src/longspark/engine/state_export.py:14-47, which
``dist.gather``s the head shards to rank 0 under target TP), packs them with the
boundary hidden states into a ``longspark_state_batch_v1`` message, ships it to
the drafter process (engine/transport.py), and the drafter scatters the rows
into its ring window (``LongSparkDraft.update``, engine/draft.py:207-212).

Here the target calls :func:`export_rows` after its verify pass: one kernel
(``ls_export_rows``) on the target's GPU gathers the rows from the target's
pool and stores them into the drafter's paged pool, on the same GPU or a peer
GPU over NVLink, and every target TP rank stores its own KV-head slice.  The
drafter is then told with a metadata-only message (``keys`` None, see
``LongSparkDraft.update``) and only folds the rows into its summary.

:class:`ExportDestination` says where the drafter's pool is, as seen from the
exporting GPU: ``LongSparkDraft.export_destination`` builds one in the same
process; across processes build it from an IPC mapping of the drafter's pool
(``ls_ipc_open``) and the drafter's page-table rows, slots and lengths.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _native as N
from .ops import _p, _stream


@dataclass
class ExportDestination:
    """A drafter pool as seen from the exporting GPU.

    kv_k, kv_v: device addresses of ``[tap_layers, pool_pages, 16, heads, 128]``
    bf16 pools; page_table ``[batch, stride]`` int32 (the requests' rows),
    seq_lens ``[batch]`` int32 (lengths after the commit) and slots ``[batch]``
    int32, in memory the exporting GPU can read; hidden_pool: address of the
    ``[capacity, tap_layers * hidden]`` bf16 boundary-hidden pool (0: none).
    ``keepalive`` holds whatever owns the addresses."""

    kv_k: int
    kv_v: int
    pool_pages: int
    heads: int
    tap_layers: int
    ring_pages: int
    page_table: torch.Tensor
    seq_lens: torch.Tensor
    slots: torch.Tensor
    hidden_pool: int = 0
    capacity: int = 0
    hidden: int = 0
    keepalive: object = None

    def to(self, device):
        """The same destination with its index arrays copied to ``device``."""
        dev = torch.device(device)
        return ExportDestination(self.kv_k, self.kv_v, self.pool_pages, self.heads, self.tap_layers,
                                 self.ring_pages, self.page_table.to(dev), self.seq_lens.to(dev),
                                 self.slots.to(dev), self.hidden_pool, self.capacity, self.hidden, self.keepalive)


class PreparedExport:
    """The argument block of one ``ls_export_rows`` launch with the device
    arrays it points to; ``launch()`` only enqueues the kernel (repeat
    launches re-store the same rows)."""

    def __init__(self, args, device, keep):
        self.args, self.device, self._keep = args, device, keep

    def launch(self):
        N.call("ls_export_rows", _stream(self.device), C.byref(self.args))


def prepare_export(dest: ExportDestination, *, src_k, src_v, locations, counts, head_offset=0, last_hidden=None,
                   status=None):
    """Check the arguments of :func:`export_rows` and stage its device arrays
    (row offsets, counts, locations) without launching."""
    L = len(src_k)
    if L != len(src_v) or L != dest.tap_layers or L > N.EXPORT_MAX_LAYERS:
        raise ValueError(f"export needs {dest.tap_layers} tapped layers of K and V (at most {N.EXPORT_MAX_LAYERS})")
    dev = src_k[0].device
    if dev.type != "cuda":
        raise ValueError("the export runs on the target's GPU: the source pools must be CUDA tensors")
    for t in list(src_k) + list(src_v):
        if t.device != dev or t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[-1] != 128 or \
                not t.is_contiguous() or t.shape != src_k[0].shape:
            raise ValueError("target pools must be contiguous bf16 [rows, heads, 128] on one device")
    if dest.page_table.device != dev:
        dest = dest.to(dev)
    counts_t = torch.as_tensor(counts, dtype=torch.int32).to(dev)
    B = counts_t.shape[0]
    if dest.seq_lens.shape[0] < B or dest.page_table.shape[0] < B:
        raise ValueError("destination describes fewer requests than counts")
    offsets = torch.zeros(B, dtype=torch.int32, device=dev)
    if B > 1:
        offsets[1:] = torch.cumsum(counts_t[:-1], 0)
    loc = torch.as_tensor(locations, dtype=torch.int64).to(dev).contiguous()
    if last_hidden is not None:
        if not dest.hidden_pool:
            raise ValueError("destination has no hidden pool")
        last_hidden = last_hidden.to(dev, torch.bfloat16).contiguous()
    a = N.ExportArgs()
    for l in range(L):
        a.src_k[l] = src_k[l].data_ptr()
        a.src_v[l] = src_v[l].data_ptr()
    a.src_rows, a.src_heads = src_k[0].shape[0], src_k[0].shape[1]
    a.locations, a.total_rows = _p(loc), loc.numel()
    a.row_offsets, a.counts, a.seq_lens = _p(offsets), _p(counts_t), _p(dest.seq_lens)
    a.dst_k, a.dst_v, a.pool_pages, a.dst_heads = dest.kv_k, dest.kv_v, dest.pool_pages, dest.heads
    a.head_offset = head_offset
    a.page_table, a.table_stride, a.ring_pages = _p(dest.page_table), dest.page_table.stride(0), dest.ring_pages
    a.last_hidden, a.hidden_pool, a.slots = _p(last_hidden), dest.hidden_pool or None, _p(dest.slots)
    a.capacity, a.hidden, a.batch, a.tap_layers = dest.capacity, dest.hidden, B, L
    a.status = _p(status)
    return PreparedExport(a, dev, (src_k, src_v, loc, offsets, counts_t, last_hidden, dest, status))


def export_rows(dest: ExportDestination, *, src_k, src_v, locations, counts, head_offset=0, last_hidden=None,
                status=None):
    """Store each request's exported rows into the drafter pool ``dest``.

    src_k, src_v: one tensor per tapped layer, the target's K/V pool
    ``[rows, heads_local, 128]`` bf16 on the exporting GPU; locations: int64
    ``[total]`` source rows, request-major (request b owns ``counts[b]``
    consecutive entries); row i of request b lands at drafter position
    ``dest.seq_lens[b] - counts[b] + i``, heads ``[head_offset, head_offset +
    heads_local)``.  last_hidden ``[batch, tap_layers, hidden]`` bf16 (one
    rank under target TP) goes to ``hidden_pool[dest.slots[b]]``.  Launches on
    the exporting GPU's current stream; nothing is waited for."""
    prepare_export(dest, src_k=src_k, src_v=src_v, locations=locations, counts=counts, head_offset=head_offset,
                   last_hidden=last_hidden, status=status).launch()


def enable_peer_access(device, peer):
    """Let kernels on ``device`` store into ``peer``'s memory (same process)."""
    with torch.cuda.device(torch.device(device)):
        N.call("ls_enable_peer_access", torch.device(peer).index)
