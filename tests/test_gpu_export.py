"""Target-side export into the drafter's pool (ls_export_rows): the rows and
hidden states against the oracle's gather + window store (full heads, two head
slices as two target TP ranks would store them, ring pages, a prefill-sized
request, a bad location), the drop-in API path (export_destination, export,
metadata-only update) against the packet path, and two GPUs where each rank
stores its head slice into rank 0's pool over NVLink."""

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
import tp_workers
from longspark_b200.draft import LongSparkDraft
from longspark_b200.export import ExportDestination, export_rows, prepare_export
from longspark_b200.synthetic import make_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _bits(t):
    """bf16 bit patterns as a fresh int16 array (never a view of a CPU tensor:
    the oracle writes into the pools it is given)."""
    return t.detach().cpu().view(torch.int16).numpy().copy()


def _case(seed, ring_pages, counts, L=3, H=8, R=5000, hidden=256):
    """Target pools, locations, a drafter page table (ring_pages columns, or
    enough pages for every position) over a shuffled pool, post-commit lengths,
    boundary hidden states and slots."""
    g = torch.Generator().manual_seed(seed)
    B = len(counts)
    src_k = torch.randn(L, R, H, 128, generator=g).to(torch.bfloat16)
    src_v = torch.randn(L, R, H, 128, generator=g).to(torch.bfloat16)
    locations = torch.randperm(R, generator=g)[:sum(counts)].to(torch.int64)
    lens = torch.tensor([c + int(torch.randint(0, 200, (1,), generator=g)) for c in counts], dtype=torch.int32)
    stride = ring_pages if ring_pages else (int(lens.max()) + 15) // 16
    pages = B * stride + 8
    table = torch.randperm(pages, generator=g)[:B * stride].view(B, stride).to(torch.int32)
    last_hidden = torch.randn(B, L, hidden, generator=g).to(torch.bfloat16)
    slots = torch.randperm(B + 2, generator=g)[:B].to(torch.int32)
    return src_k, src_v, locations, table, lens, last_hidden, slots, pages


@pytest.mark.parametrize("ring_pages,counts,heads_split", [
    (0, [1, 16, 7, 3, 12], 1),
    (8, [5, 16, 128, 2], 1),       # ring pages; a prefill-sized request (the whole 128-row ring)
    (2, [50, 5, 33, 32], 1),        # counts above the 32-row ring: only the last 32 rows of a request land
    (0, [9, 16, 1, 300], 2),        # two head slices, as two target TP ranks store them
])
def test_export_rows_matches_oracle(ring_pages, counts, heads_split):
    dev = torch.device("cuda")
    src_k, src_v, loc, table, lens, last_hidden, slots, pages = _case(7 + len(counts), ring_pages, counts)
    L, R, H, D = src_k.shape
    B = len(counts)
    fill = torch.full((L, pages, 16, H, D), -3.0).to(torch.bfloat16)
    pool_k, pool_v = fill.clone().to(dev), fill.clone().to(dev)
    hid_pool = torch.zeros(B + 2, L * 256, dtype=torch.bfloat16, device=dev)
    dest = ExportDestination(kv_k=pool_k.data_ptr(), kv_v=pool_v.data_ptr(), pool_pages=pages, heads=H, tap_layers=L,
                             ring_pages=ring_pages, page_table=table.to(dev), seq_lens=lens.to(dev),
                             slots=slots.to(dev), hidden_pool=hid_pool.data_ptr(), capacity=B + 2, hidden=256)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    h = H // heads_split
    for r in range(heads_split):
        sk = [src_k[l, :, r * h:(r + 1) * h].contiguous().to(dev) for l in range(L)]
        sv = [src_v[l, :, r * h:(r + 1) * h].contiguous().to(dev) for l in range(L)]
        export_rows(dest, src_k=sk, src_v=sv, locations=loc, counts=counts, head_offset=r * h,
                    last_hidden=last_hidden if r == 0 else None, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref_k, ref_v = O.export_rows(_bits(fill), _bits(fill), _bits(src_k), _bits(src_v), loc.numpy(), counts,
                                 lens.numpy(), table.numpy(), ring_pages)
    np.testing.assert_array_equal(_bits(pool_k), ref_k)
    np.testing.assert_array_equal(_bits(pool_v), ref_v)
    hp = _bits(hid_pool)
    for b in range(B):
        np.testing.assert_array_equal(hp[slots[b]], _bits(last_hidden[b]).reshape(-1))


def test_export_rows_bad_location_skips_the_row():
    dev = torch.device("cuda")
    counts = [4, 6]
    src_k, src_v, loc, table, lens, _, slots, pages = _case(3, 0, counts)
    L, R, H, D = src_k.shape
    good = loc.clone()
    loc = loc.clone()
    loc[5] = R  # one past the target pool: request 1, row 1
    fill = torch.full((L, pages, 16, H, D), -3.0).to(torch.bfloat16)
    pool_k, pool_v = fill.clone().to(dev), fill.clone().to(dev)
    dest = ExportDestination(kv_k=pool_k.data_ptr(), kv_v=pool_v.data_ptr(), pool_pages=pages, heads=H, tap_layers=L,
                             ring_pages=0, page_table=table.to(dev), seq_lens=lens.to(dev), slots=slots.to(dev))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    export_rows(dest, src_k=[src_k[l].to(dev) for l in range(L)], src_v=[src_v[l].to(dev) for l in range(L)],
                locations=loc, counts=counts, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 110
    ref_k, _ = O.export_rows(_bits(fill), _bits(fill), _bits(src_k), _bits(src_v), good.numpy(), counts,
                             lens.numpy(), table.numpy())
    # the bad row's destination keeps its old contents, every other row landed
    pos = int(lens[1]) - counts[1] + 1
    page, r = int(table[1, pos // 16]), pos % 16
    gk = _bits(pool_k)
    assert (gk[:, page, r] == _bits(fill)[:, page, r]).all()
    ref_k[:, page, r] = _bits(fill)[:, page, r]
    np.testing.assert_array_equal(gk, ref_k)


def test_export_rows_bad_count_skips_the_request():
    """A count that runs past the end of the locations: that request is
    skipped whole (status LS_DEV_BAD_INDEX), the other request lands."""
    dev = torch.device("cuda")
    counts = [4, 6]
    src_k, src_v, loc, table, lens, _, slots, pages = _case(5, 0, counts)
    L, R, H, D = src_k.shape
    fill = torch.full((L, pages, 16, H, D), -3.0).to(torch.bfloat16)
    pool_k, pool_v = fill.clone().to(dev), fill.clone().to(dev)
    dest = ExportDestination(kv_k=pool_k.data_ptr(), kv_v=pool_v.data_ptr(), pool_pages=pages, heads=H, tap_layers=L,
                             ring_pages=0, page_table=table.to(dev), seq_lens=lens.to(dev), slots=slots.to(dev))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    prep = prepare_export(dest, src_k=[src_k[l].to(dev) for l in range(L)], src_v=[src_v[l].to(dev) for l in range(L)],
                          locations=loc, counts=counts, status=status)
    bad = torch.tensor([4, 1 << 30], dtype=torch.int32, device=dev)  # request 1 claims far more rows than exist
    prep.args.counts = bad.data_ptr()
    prep.launch()
    torch.cuda.synchronize()
    assert int(status.item()) == 110
    ref_k, _ = O.export_rows(_bits(fill), _bits(fill), _bits(src_k), _bits(src_v), loc.numpy()[:4], [4],
                             lens.numpy()[:1], table.numpy()[:1])
    np.testing.assert_array_equal(_bits(pool_k), ref_k)


def test_longspark_draft_in_place_export_matches_packets():
    """Two drafters with the same weights and prefill; one decode step reaches
    the first through the batch message, the second through the fused export
    and a metadata-only update: identical tokens, pools and summary state."""
    from longspark_b200.config import DraftShape
    shape = DraftShape(hidden=512, q_heads=8, kv_heads=2, inter=1024, vocab=4096, tap_layers=2, draft_layers=2,
                       slots=64, window=256, block=7, max_commit=16, markov_rank=64, mask_token_id=4000)
    W = make_weights(shape, seed=41, norm_jitter=0.05)
    cfg = dict(draft_device=0, max_running_requests=4, draft_state_gib=1.0, cuda_graph=True, graph_batch_sizes=(2,))
    d1, d2 = LongSparkDraft(cfg, weights=W, shape=shape), LongSparkDraft(cfg, weights=W, shape=shape)
    g = torch.Generator().manual_seed(42)
    L, Hkv, Hq, S = shape.tap_layers, shape.kv_heads, shape.q_heads, shape.slots
    ids, lengths = ["x", "y"], [300, 40]
    hist = {i: (torch.randn(L, n + 32, Hkv, 128, generator=g).to(torch.bfloat16),
                torch.randn(L, n + 32, Hkv, 128, generator=g).to(torch.bfloat16)) for i, n in zip(ids, lengths)}
    cnt = [min(n, shape.window) for n in lengths]
    pre = dict(format="longspark_state_batch_v1", ids=ids, lengths=lengths, commit_lens=cnt, export_counts=cnt,
               keys=torch.cat([hist[i][0][:, n - c:n] for i, n, c in zip(ids, lengths, cnt)], dim=1),
               values=torch.cat([hist[i][1][:, n - c:n] for i, n, c in zip(ids, lengths, cnt)], dim=1),
               last_hidden=torch.randn(2, L, shape.hidden, generator=g).to(torch.bfloat16),
               global_output=0.1 * torch.randn(2, L, Hq, S, 128, generator=g),
               global_lse=torch.randn(2, L, Hq, S, generator=g) + 5.0)
    d1.update(pre, prefill=True)
    d2.update(pre, prefill=True)
    commit = [6, 16]
    new_len = [n + c for n, c in zip(lengths, commit)]
    keys = torch.cat([hist[i][0][:, n:n + c] for i, n, c in zip(ids, lengths, commit)], dim=1)
    vals = torch.cat([hist[i][1][:, n:n + c] for i, n, c in zip(ids, lengths, commit)], dim=1)
    hidden = torch.randn(2, L, shape.hidden, generator=g).to(torch.bfloat16)
    d1.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=new_len, commit_lens=commit,
                   export_counts=commit, keys=keys, values=vals, last_hidden=hidden))
    # the target's pool: the committed rows at scattered locations
    dev = torch.device("cuda")
    R = 4000
    loc = torch.randperm(R, generator=g)[:sum(commit)]
    tk = torch.zeros(L, R, Hkv, 128, dtype=torch.bfloat16)
    tv = torch.zeros_like(tk)
    tk[:, loc], tv[:, loc] = keys, vals
    with pytest.raises(RuntimeError, match="out-of-order"):
        d2.export_destination(ids, [n + 1 for n in new_len], commit)
    dest = d2.export_destination(ids, new_len, commit)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    export_rows(dest, src_k=[tk[l].to(dev) for l in range(L)], src_v=[tv[l].to(dev) for l in range(L)],
                locations=loc, counts=commit, last_hidden=hidden, status=status)
    d2.update(dict(format="longspark_state_batch_v1", ids=ids, lengths=new_len, commit_lens=commit,
                   export_counts=commit, keys=None, values=None, last_hidden=None))
    anchors = [11, 4000]
    t1, l1, _ = d1.propose(ids, anchors, 0.0)
    t2, l2, _ = d2.propose(ids, anchors, 0.0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and d1.device_status() == 0 and d2.device_status() == 0
    assert torch.equal(t1, t2)
    assert torch.equal(l1.view(torch.int16), l2.view(torch.int16))
    for name in ("kv_k", "kv_v", "hidden", "summary_out", "summary_lse"):
        a, b = getattr(d1.pools, name), getattr(d2.pools, name)
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), name


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_export_rows_two_gpus_head_slices_over_nvlink():
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 CUDA devices")
    mp.start_processes(tp_workers.export_worker, args=(world, _port()), nprocs=world, join=True, start_method="spawn")
