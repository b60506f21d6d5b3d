"""tcgen05 stream-K GEMM and its fused epilogues against fp32 references."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_util import assert_bf16_close, gemm_ws, to_np
from longspark_b200 import _native as N
from longspark_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.manual_seed(0)


def _rand(*shape, std=1.0):
    return (torch.randn(*shape, device="cuda") * std).to(torch.bfloat16)


@pytest.mark.parametrize("rows,k,n", [
    (16, 4096, 4096),      # stream-K: 32 tiles x 64 k-blocks over every SM
    (1, 64, 128),          # single unit
    (7, 256, 384),
    (15, 2560, 9728),
    (30, 1024, 512),
    (100, 512, 256),       # token tile 112
    (300, 256, 384),       # two token tiles of 256
    (16, 20480, 4096),     # state-encoder shape (5 taps x 4096)
    (16, 4096, 151936),    # vocabulary projection
    (480, 256, 65664),     # many tokens over an odd count (513) of 128-row blocks
    (480, 2560, 5120),     # narrowed token tile (128)
    (480, 640, 5120),      # narrowed token tile (64), short k
    (480, 4096, 24576),    # gate/up shape at 32 requests, stream-K partial tiles
    (1920, 1024, 8192),    # eight token tiles
])
def test_gemm_store_matches_fp32(rows, k, n):
    x = _rand(rows, k)
    w = _rand(n, k, std=0.02)
    out = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.gemm(x, w, out, workspace=gemm_ws(rows, k, n), status=st)
    ref = (x.float() @ w.float().T).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert_bf16_close(to_np(out), to_np(ref), steps=1.0, exact_frac=0.97, what=f"gemm {rows}x{k}x{n}")


def test_gemm_repeated_launches_are_deterministic():
    x = _rand(16, 4096)
    w = _rand(4096, 4096, std=0.02)
    ws = gemm_ws(16, 4096, 4096)
    a = torch.empty(16, 4096, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    ops.gemm(x, w, a, workspace=ws)
    for _ in range(3):
        ops.gemm(x, w, b, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    assert int(ws[:65536].view(torch.int32).abs().sum().item()) == 0  # tile counters self-clean


def test_gemm_silu_and_residual():
    rows, k, n = 15, 1024, 768
    x, w = _rand(rows, k), _rand(n, k, std=0.02)
    ws = gemm_ws(rows, k, n)
    ref = to_np((x.float() @ w.float().T))
    out = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, w, out, workspace=ws, epilogue=N.EPI_SILU)
    assert_bf16_close(to_np(out), O.silu(O.bf16_round(ref), "bf16"), steps=1.0, exact_frac=0.97, what="silu")
    res = _rand(rows, n)
    out2 = res.clone()
    ops.gemm(x, w, out2, workspace=ws, epilogue=N.EPI_RESIDUAL, residual=out2)
    assert_bf16_close(to_np(out2), O.bf16_round(O.bf16_round(ref) + to_np(res)), steps=1.0, exact_frac=0.97,
                      what="residual")


def test_gemm_gate_up_interleaved():
    from longspark_b200.engine import _interleave_gate_up
    rows, k, inter = 15, 512, 384
    x = _rand(rows, k)
    g, u = _rand(inter, k, std=0.05), _rand(inter, k, std=0.05)
    w = _interleave_gate_up(g, u)
    out = torch.empty(rows, inter, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, w, out, workspace=gemm_ws(rows, k, 2 * inter), epilogue=N.EPI_GATEUP)
    gr = O.bf16_round(to_np(x.float() @ g.float().T))
    ur = O.bf16_round(to_np(x.float() @ u.float().T))
    ref = O.bf16_round(O.silu(gr, "bf16") * ur)
    assert_bf16_close(to_np(out), ref, steps=1.0, exact_frac=0.95, what="gate_up")


@pytest.mark.parametrize("rows", [15, 300])
def test_gemm_qkv_norm_rope(rows):
    hidden, hq, hkv = 512, 4, 2
    x = _rand(rows, hidden)
    w = _rand((hq + 2 * hkv) * 128, hidden, std=0.05)
    qn = (1 + 0.1 * torch.randn(128, device="cuda")).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(128, device="cuda")).to(torch.bfloat16)
    pos = torch.arange(rows, dtype=torch.int32, device="cuda") + 131000
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    out = torch.empty(rows, (hq + 2 * hkv) * 128, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, w, out, workspace=gemm_ws(rows, hidden, w.shape[0]), epilogue=N.EPI_QKV, q_heads=hq,
             kv_heads=hkv, q_norm_w=qn, k_norm_w=kn, norm_eps=1e-6, positions=pos, inv_freq=inv.cuda())
    y = O.bf16_round(to_np(x.float() @ w.float().T)).reshape(rows, hq + 2 * hkv, 128)
    q = O.rmsnorm_hf(y[:, :hq], to_np(qn), 1e-6, "bf16")
    k = O.rmsnorm_hf(y[:, hq:hq + hkv], to_np(kn), 1e-6, "bf16")
    cos, sin = O.rope_tables(pos.cpu().numpy()[None].astype(np.int64), inv.numpy(), "bf16")
    q = O.apply_rotary(q.transpose(1, 0, 2)[None], cos, sin, "bf16")[0].transpose(1, 0, 2)
    k = O.apply_rotary(k.transpose(1, 0, 2)[None], cos, sin, "bf16")[0].transpose(1, 0, 2)
    ref = np.concatenate([q, k, y[:, hq + hkv:]], axis=1).reshape(rows, -1)
    assert_bf16_close(to_np(out), ref, steps=1.0, exact_frac=0.95, what="qkv")


@pytest.mark.parametrize("rows,k,v", [(15, 512, 1024 * 8), (300, 512, 151936)])
def test_gemm_lm_head_tile_argmax(rows, k, v):
    """Per-128-token tile maxima; (300, 512, 151936) covers two token tiles
    over the full 1187-tile vocabulary."""
    x = _rand(rows, k)
    w = _rand(v, k, std=0.05)
    out = torch.empty(rows, v, dtype=torch.bfloat16, device="cuda")
    tmax = torch.empty(rows, v // 128, dtype=torch.float32, device="cuda")
    targ = torch.empty(rows, v // 128, dtype=torch.int32, device="cuda")
    ops.gemm(x, w, out, workspace=gemm_ws(rows, k, v), epilogue=N.EPI_LMHEAD, tile_max=tmax, tile_arg=targ)
    lg = to_np(out).reshape(rows, v // 128, 128)
    np.testing.assert_array_equal(to_np(tmax), lg.max(-1))
    np.testing.assert_array_equal(targ.cpu().numpy(), lg.argmax(-1) + np.arange(v // 128)[None] * 128)
    assert_bf16_close(to_np(out), to_np((x.float() @ w.float().T).to(torch.bfloat16)), steps=1.0,
                      exact_frac=0.97, what="lm head")


def test_gemm_markov_add():
    rows, r, v = 15, 256, 2048
    x, w = _rand(rows, r, std=0.02), _rand(v, r, std=0.02)
    base = _rand(rows, v)
    out = torch.empty(rows, v, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, w, out, workspace=gemm_ws(rows, r, v), epilogue=N.EPI_MARKOV_ADD, base=base)
    ref = O.bf16_round(to_np(base) + O.bf16_round(to_np(x.float() @ w.float().T)))
    assert_bf16_close(to_np(out), ref, steps=1.0, exact_frac=0.97, what="markov add")


def test_gemm_rejects_bad_shapes():
    x = _rand(16, 100)
    w = _rand(128, 100)
    out = torch.empty(16, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(N.NativeError, match="k%64"):
        ops.gemm(x, w, out, workspace=gemm_ws(16, 128, 128))


def test_gemms_of_different_shapes_share_one_workspace():
    """A small-tile-count GEMM leaves partial tiles in the shared workspace; a
    following GEMM with many tiles must still find zeroed arrival counters."""
    shapes = [(15, 2560, 6144), (15, 2560, 19456), (1, 2560, 2560), (15, 2560, 151936), (15, 9728, 2560)]
    ws = torch.zeros(max(ops.gemm_workspace_bytes(*s) for s in shapes), dtype=torch.uint8, device="cuda")
    for rows, k, n in shapes * 2:
        x = _rand(rows, k)
        w = _rand(n, k, std=0.02)
        out = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
        ops.gemm(x, w, out, workspace=ws)
        ref = (x.float() @ w.float().T).to(torch.bfloat16)
        assert_bf16_close(to_np(out), to_np(ref), steps=1.0, exact_frac=0.97, what=f"shared ws {rows}x{k}x{n}")


@pytest.mark.parametrize("rows,k,n", [(15, 4096, 4096), (1, 20480, 4096), (16, 4096, 151936), (300, 256, 384),
                                      (480, 256, 65664)])
def test_tiled_weights_match_row_major(rows, k, n):
    """The tensor-core tile layout streams the same weights: results are bit-identical."""
    x = _rand(rows, k)
    w = _rand(n, k, std=0.02)
    wt = ops.TiledWeight(w)
    a = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    ws = gemm_ws(rows, k, n)
    ops.gemm(x, w, a, workspace=ws)
    ops.gemm(x, wt, b, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(a, b)

