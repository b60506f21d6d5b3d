"""The bounded peer waits of the tensor-parallel kernels, on one GPU: a group
of two "ranks" whose second heap is a plain local buffer that no process
drives, so the flags the kernels wait for are never set.  Each wait gives up
after its limit, the kernel records LS_DEV_TIMEOUT_PEER and returns, and the
context stays usable (a plain GEMM runs correctly afterwards)."""

import ctypes as C
import types

import pytest
import torch

from longspark_b200 import _native as N
from longspark_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _fake_group(nbytes):
    dev = torch.device("cuda")
    heaps = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    st = N.TpGroup(world=2, rank=0, heap=(C.c_void_p * N.TP_MAX_RANKS)(heaps[0].data_ptr(), heaps[1].data_ptr()),
                   heap_bytes=nbytes, sync_offset=0)
    return types.SimpleNamespace(struct=st, device=dev, heaps=heaps)


def test_barrier_without_peer_reports_timeout():
    g = _fake_group(1 << 20)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.tp_barrier(g, slot=0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == N.DEV_TIMEOUT_PEER


def test_gemm_allreduce_without_peer_reports_timeout_and_context_survives():
    rows, k, n = 32, 512, 512
    sync = N.lib().ls_tp_sync_bytes(2, rows, n, N.TP_WIRE_F32)
    g = _fake_group(sync + (1 << 20))
    dev = torch.device("cuda")
    out = g.heaps[0][sync:sync + rows * n * 2].view(torch.bfloat16).view(rows, n)
    x = torch.randn(rows, k, device=dev).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev) * 0.05).to(torch.bfloat16)
    ws = torch.zeros(max(1, ops.gemm_workspace_bytes(rows, k, n)), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.gemm_allreduce(x, ops.TiledWeight(w), out, group=g, workspace=ws, rows=rows, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == N.DEV_TIMEOUT_PEER
    # the context is intact: an ordinary GEMM still computes the right product
    y = torch.empty(rows, n, dtype=torch.bfloat16, device=dev)
    ws.zero_()
    status.zero_()
    ops.gemm(x, ops.TiledWeight(w), y, workspace=ws, rows=rows, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = (x.float() @ w.float().T)
    assert torch.allclose(y.float(), ref, atol=2e-2, rtol=2e-2)
