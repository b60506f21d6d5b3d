"""ls_markov_argmax_static (scratch in a static device array, no allocation)
against ls_markov_argmax (caller workspace), called through the C ABI.

Two calls of the static entry point in a row, on different inputs, so the
second call runs on the scratch the first one left behind.  Token ids and
accept lengths are integers: the two entry points must agree exactly.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from longspark_b200 import _native as N
from longspark_b200 import ops

pytestmark = pytest.mark.gpu

MAX_ROWS = 1024  # LS_MARKOV_STATIC_MAX_ROWS


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _case(seed, batch, block, vocab, rank, wstd=0.02):
    g = torch.Generator().manual_seed(seed)
    dev = "cuda"
    base = (1.3 * torch.randn(batch * block, vocab, generator=g)).to(torch.bfloat16)
    lv = base.float().numpy().reshape(batch * block, vocab // 128, 128)
    c = {
        "base": base.to(dev),
        "tile_max": torch.from_numpy(lv.max(-1)).to(dev),
        "tile_arg": torch.from_numpy((lv.argmax(-1) + np.arange(vocab // 128)[None] * 128).astype(np.int32)).to(dev),
        "anchors": torch.randint(0, vocab, (batch,), generator=g).to(dev),
        "target": torch.randint(0, vocab, (batch, block + 1), generator=g).to(dev),
        "w1": None, "w2": None, "b1": None, "b2": None,
        "batch": batch, "block": block, "vocab": vocab, "rank": rank,
    }
    if rank:
        c["w1"] = (wstd * torch.randn(vocab, rank, generator=g)).to(torch.bfloat16).to(dev)
        c["w2"] = (wstd * torch.randn(vocab, rank, generator=g)).to(torch.bfloat16).to(dev)
        c["b1"], c["b2"] = torch.zeros(1, device=dev), torch.zeros(1, device=dev)
        ops.row_norm_bound(c["w1"], c["b1"])
        ops.row_norm_bound(c["w2"], c["b2"])
    return c


def _args(c, tokens, accept, status):
    p = lambda t: None if t is None else C.c_void_p(t.data_ptr())  # noqa: E731
    return N.MarkovArgs(base=p(c["base"]), tile_max=p(c["tile_max"]), tile_arg=p(c["tile_arg"]), w1=p(c["w1"]),
                        w2=p(c["w2"]), w1_row_bound=p(c["b1"]), w2_row_bound=p(c["b2"]), rank=c["rank"],
                        anchors=p(c["anchors"]), tokens=p(tokens), target=p(c["target"]),
                        target_ld=c["target"].stride(0), accept_out=p(accept), batch=c["batch"], block=c["block"],
                        vocab=c["vocab"], status=p(status))


def _outputs(c):
    tokens = torch.full((c["batch"], c["block"]), -1, dtype=torch.int64, device="cuda")
    accept = torch.full((c["batch"],), -1, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    return tokens, accept, status


def _run_static(c):
    tokens, accept, status = _outputs(c)
    a = _args(c, tokens, accept, status)
    N.call("ls_markov_argmax_static", C.c_void_p(torch.cuda.current_stream().cuda_stream), C.byref(a))
    return tokens, accept, status


def _run_workspace(c):
    tokens, accept, status = _outputs(c)
    a = _args(c, tokens, accept, status)
    ws = torch.zeros(ops.markov_workspace_bytes(c["batch"], c["block"]), dtype=torch.uint8, device="cuda")
    N.call("ls_markov_argmax", C.c_void_p(torch.cuda.current_stream().cuda_stream), C.byref(a),
           C.c_void_p(ws.data_ptr()), ws.numel())
    return tokens, accept, status


def test_static_scratch_matches_workspace_entry_point_twice():
    first = _case(seed=5, batch=3, block=15, vocab=151936, rank=64)
    second = _case(seed=6, batch=MAX_ROWS // 16, block=16, vocab=151936, rank=256)  # the maximum rows
    got = [_run_static(first), _run_static(second)]  # back to back on the shared scratch
    want = [_run_workspace(first), _run_workspace(second)]
    torch.cuda.synchronize()
    for (gt, ga, gs), (wt, wa, ws), c in zip(got, want, (first, second)):
        assert int(gs.item()) == 0 and int(ws.item()) == 0
        assert (gt >= 0).all() and (gt < c["vocab"]).all()
        np.testing.assert_array_equal(gt.cpu().numpy(), wt.cpu().numpy())
        np.testing.assert_array_equal(ga.cpu().numpy(), wa.cpu().numpy())


def test_static_scratch_rejects_more_rows_than_its_maximum():
    c = _case(seed=7, batch=MAX_ROWS // 16 + 1, block=16, vocab=1024, rank=0)
    tokens, accept, status = _outputs(c)
    a = _args(c, tokens, accept, status)
    with pytest.raises(N.NativeError, match="static scratch maximum of 1024 rows"):
        N.call("ls_markov_argmax_static", C.c_void_p(torch.cuda.current_stream().cuda_stream), C.byref(a))
    torch.cuda.synchronize()
    assert (tokens == -1).all()  # nothing launched
    assert int(status.item()) == 0  # and no device status recorded


def test_static_scratch_empty_batch_and_bad_block():
    """An empty batch returns LS_OK with nothing launched; a block of 0 is
    rejected with LS_ERR_UNSUPPORTED like the workspace entry point does,
    before anything is enqueued."""
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = N.lib()
    c = _case(seed=8, batch=2, block=4, vocab=1024, rank=0)
    tokens, accept, status = _outputs(c)
    a = _args(c, tokens, accept, status)
    a.batch = 0
    assert lib.ls_markov_argmax_static(stream, C.byref(a)) == N.LS_OK
    a.batch, a.block = 2, 0
    assert lib.ls_markov_argmax_static(stream, C.byref(a)) == 3  # LS_ERR_UNSUPPORTED
    assert b"block <= 16" in lib.ls_last_error()
    torch.cuda.synchronize()
    assert (tokens == -1).all() and (accept == -1).all()
    assert int(status.item()) == 0
