"""Host-side logic on the CPU: request bookkeeping and the reference's error
contract, batch-message handling, request sharding, synthetic inputs."""

import pytest
import torch

from longspark_b200.config import CFG1, CFG2, CFG3, DraftShape
from longspark_b200.requests import (BATCH_FORMAT, RequestTable, owner_rank, shard, split_batch_message,
                                     unpack_packets)
from longspark_b200.synthetic import geometric_accept, make_views, target_from_draft


def _meta(ids, lengths, commits):
    return [dict(id=i, length=l, commit_len=c) for i, l, c in zip(ids, lengths, commits)]


def test_prefill_decode_release_cycle():
    t = RequestTable(capacity=2, max_commit=16, window=1024)
    c = t.prefill(_meta(["a", "b"], [3000, 100], [1024, 100]), [1024, 100])
    assert sorted(c.slots) == [0, 1] and c.offsets == [0, 1024]
    with pytest.raises(RuntimeError, match="unavailable or already owned"):
        t.prefill(_meta(["c"], [10], [10]), [10])          # no free slot
    with pytest.raises(RuntimeError, match="unavailable or already owned"):
        t.prefill(_meta(["a"], [10], [10]), [10])          # already owned
    d = t.decode(_meta(["a", "b"], [3016, 101], [16, 1]), [16, 1])
    assert d.lengths == [3016, 101] and d.offsets == [0, 16]
    t.release(["a"])
    assert len(t.free_slots) == 1 and "a" not in t.requests


@pytest.mark.parametrize("lengths,commits,counts,exc", [
    ([3005], [4], [4], RuntimeError),    # previous + commit != length
    ([3017], [17], [17], RuntimeError),  # commit beyond max_commit
    ([3000], [0], [0], RuntimeError),    # empty commit
    ([3004], [4], [3], ValueError),      # rows disagree with commit_len
])
def test_decode_errors_follow_reference_contract(lengths, commits, counts, exc):
    t = RequestTable(capacity=1, max_commit=16, window=1024)
    t.prefill(_meta(["a"], [3000], [1024]), [1024])
    with pytest.raises(exc):
        t.decode(_meta(["a"], lengths, commits), counts)
    assert t.requests["a"][1] == 3000  # state untouched by a rejected commit


def test_decode_batch_is_all_or_nothing():
    t = RequestTable(capacity=2, max_commit=8, window=256)
    t.prefill(_meta(["a", "b"], [50, 60], [50, 60]), [50, 60])
    with pytest.raises(RuntimeError):
        t.decode(_meta(["a", "b"], [52, 99], [2, 3]), [2, 3])
    assert t.requests["a"][1] == 50 and t.requests["b"][1] == 60


def test_unpack_batch_message_checks_extents():
    keys = torch.zeros(5, 7, 8, 128)
    msg = dict(format=BATCH_FORMAT, ids=["a", "b"], lengths=[10, 20], commit_lens=[3, 4], export_counts=[3, 4],
               keys=keys, values=keys.clone(), last_hidden=torch.zeros(2, 5, 64))
    meta, counts, k, v, h, extra = unpack_packets(msg)
    assert counts == [3, 4] and [m["id"] for m in meta] == ["a", "b"] and extra == {}
    with pytest.raises(ValueError, match="extent"):
        unpack_packets(dict(msg, export_counts=[3, 5]))
    with pytest.raises(ValueError, match="unknown"):
        unpack_packets(dict(msg, format="v0"))


def test_metadata_only_message_for_rows_exported_in_place():
    """A batch message whose keys are None (the rows were stored in the
    drafter's pool by the target's export) carries metadata only."""
    msg = dict(format=BATCH_FORMAT, ids=["a"], lengths=[10], commit_lens=[3], export_counts=[3], keys=None,
               values=None, last_hidden=None)
    meta, counts, k, v, h, extra = unpack_packets(msg)
    assert counts == [3] and k is None and v is None and h is None
    with pytest.raises(ValueError, match="no values"):
        unpack_packets(dict(msg, values=torch.zeros(1, 3, 8, 128)))


def test_check_decode_validates_without_applying():
    t = RequestTable(capacity=2, max_commit=8, window=256)
    t.prefill(_meta(["a", "b"], [50, 60], [50, 60]), [50, 60])
    slots = t.check_decode(_meta(["a", "b"], [52, 63], [2, 3]), [2, 3])
    assert slots == [t.requests["a"][0], t.requests["b"][0]]
    assert t.requests["a"][1] == 50 and t.requests["b"][1] == 60
    with pytest.raises(RuntimeError, match="out-of-order"):
        t.check_decode(_meta(["a"], [53], [2]), [2])


def test_request_sharding_partitions_ids():
    ids = [f"req{i}" for i in range(100)]
    for world in (1, 2, 4, 8):
        parts = [shard(ids, world, r) for r in range(world)]
        assert sorted(sum(parts, [])) == sorted(ids)
        assert all(owner_rank(i, world) == r for r, p in enumerate(parts) for i in p)
    assert owner_rank("req7", 8) == owner_rank("req7", 8)


def test_split_batch_message_keeps_owned_rows():
    keys = torch.arange(2 * 6).float().view(1, 6, 1, 2).expand(5, 6, 1, 2).contiguous()
    msg = dict(format=BATCH_FORMAT, ids=["x", "y", "z"], lengths=[5, 6, 7], commit_lens=[1, 2, 3],
               export_counts=[1, 2, 3], keys=keys, values=keys.clone(), last_hidden=torch.arange(3).float()[:, None])
    world = 2
    parts = [split_batch_message(msg, world, r) for r in range(world)]
    assert sorted(parts[0]["ids"] + parts[1]["ids"]) == ["x", "y", "z"]
    for p in parts:
        assert p["keys"].shape[1] == sum(p["export_counts"])
        off = 0
        for i, c in zip(p["ids"], p["export_counts"]):
            src = {"x": 0, "y": 1, "z": 3}[i]
            assert torch.equal(p["keys"][:, off:off + c], keys[:, src:src + c])
            off += c


def test_workload_shapes():
    assert CFG1.shape.hidden == 2560 and CFG1.shape.slots == 64 and CFG1.shape.window == 512
    assert CFG2.shape.block + 1 == 16 and CFG2.shape.tap_layers == 5 and CFG2.shape.window == 1024
    assert CFG3.shape.q_heads // CFG3.shape.kv_heads == 5 and CFG3.rounds == 200
    with pytest.raises(ValueError):
        DraftShape(head_dim=64)
    with pytest.raises(ValueError):
        DraftShape(block=17)


def test_synthetic_views_page_table_is_a_permutation():
    shape = DraftShape(hidden=256, q_heads=8, kv_heads=2, inter=256, vocab=1024, tap_layers=1, slots=16,
                       window=256, block=7, max_commit=8, markov_rank=0, mask_token_id=0)
    v = make_views(shape, 3, [100, 4096, 17], seed=0, pool_pages=400)
    used = torch.cat([v["page_table"][0, :7], v["page_table"][1, :256], v["page_table"][2, :2]])
    assert used.unique().numel() == used.numel() and int(used.max()) < 400


def test_target_from_draft_gives_requested_accept_length():
    g = torch.Generator().manual_seed(0)
    draft = torch.randint(0, 1000, (64, 15), generator=g)
    k = geometric_accept(g, 64, 15)
    tgt = target_from_draft(draft, k, 1000)
    acc = (tgt[:, :15] == draft).long().cumprod(1).sum(1)
    assert torch.equal(acc, k)
    assert 1.5 < k.float().mean() < 4.5  # geometric with mean 3


def test_sampling_hash_is_uniform_and_counter_based():
    """The T > 0 noise source: deterministic in (seed, request, step, token),
    different across each counter, and uniform on (0, 1)."""
    import numpy as np
    import oracle as O
    v = np.arange(1 << 18)
    u = O.gumbel_hash_uniform(7, 0, 0, v)
    assert np.array_equal(u, O.gumbel_hash_uniform(7, 0, 0, v))
    assert 0.0 < u.min() and u.max() < 1.0
    hist = np.histogram(u, bins=16, range=(0, 1))[0]
    assert np.abs(hist / len(v) * 16 - 1).max() < 0.02
    for other in (O.gumbel_hash_uniform(8, 0, 0, v), O.gumbel_hash_uniform(7, 1, 0, v),
                  O.gumbel_hash_uniform(7, 0, 1, v), O.gumbel_hash_uniform(7 << 32, 0, 0, v)):
        assert np.mean(other == u) < 1e-3
        assert abs(np.corrcoef(other, u)[0, 1]) < 0.01


def test_export_arguments_are_checked_on_the_host():
    """export.prepare_export rejects mismatched tapped layers and pools that are
    not on a CUDA device before any native call."""
    from longspark_b200.export import ExportDestination, prepare_export
    dest = ExportDestination(kv_k=256, kv_v=512, pool_pages=4, heads=8, tap_layers=2, ring_pages=0,
                             page_table=torch.zeros(1, 4, dtype=torch.int32), seq_lens=torch.ones(1, dtype=torch.int32),
                             slots=torch.zeros(1, dtype=torch.int32))
    pool = torch.zeros(10, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="tapped layers"):
        prepare_export(dest, src_k=[pool], src_v=[pool], locations=[0], counts=[1])
    with pytest.raises(ValueError, match="CUDA tensors"):
        prepare_export(dest, src_k=[pool, pool], src_v=[pool, pool], locations=[0], counts=[1])


def test_capture_guard_pauses_and_restores_the_collector():
    import gc
    from longspark_b200.engine import capture_guard
    assert gc.isenabled()
    with capture_guard():
        assert not gc.isenabled()
        assert gc.collect() >= 0  # an explicit collection still runs
    assert gc.isenabled()
    gc.disable()
    try:
        with capture_guard():
            pass
        assert not gc.isenabled()  # a collector that was off stays off
    finally:
        gc.enable()
    with pytest.raises(RuntimeError):
        with capture_guard():
            raise RuntimeError("capture failed")
    assert gc.isenabled()
