"""GEMM planner invariants, checked without a GPU through ``ls_gemm_plan_info``
(148 SMs assumed).  Every plan the library can pick must fit the hardware
(shared memory per CTA, 512 TMEM columns, 16-aligned token tiles), divide k
into its stages, stay within the workspace ``ls_gemm_workspace_bytes``
reports for the shape whatever the epilogue, and -- for the fused-allreduce
GEMMs -- within the exchange region ``ls_tp_sync_bytes`` reports for that
world and wire format (the GEMM writes its partials there, so a plan that
outgrew it would write past the region)."""

import ctypes as C

import pytest

from longspark_b200 import _native as N

SHAPES = [(r, k, n) for r in (1, 7, 15, 16, 33, 64, 65, 100, 120, 128, 129, 240, 300, 480, 960, 1920)
          for (k, n) in ((64, 128), (256, 384), (4096, 6144), (4096, 4096), (8192, 4096), (12288, 4096),
                         (4096, 24576), (5120, 10240), (4096, 151936))]
EPILOGUES = [N.EPI_STORE, N.EPI_SILU, N.EPI_RESIDUAL, N.EPI_QKV, N.EPI_GATEUP, N.EPI_LMHEAD, N.EPI_MARKOV_ADD]


def _plan(rows, k, n, epi, fused=0, world=1, wire=0):
    p = N.GemmPlan()
    rc = N.lib().ls_gemm_plan_info(rows, k, n, epi, fused, world, wire, C.byref(p))
    assert rc == 0, N.lib().ls_last_error()
    return p


def _check_fits(p, rows, k, n):
    assert p.bn % 16 == 0 and 16 <= p.bn <= 256
    assert p.mw in (1, 2) and p.kg in (1, 2, 4) and k % (64 * p.kg) == 0
    assert p.stages >= 2
    assert p.smem_bytes <= 227 * 1024
    assert p.tmem_cols <= 512
    assert 1 <= p.grid <= 148 and p.grid <= p.units
    assert p.n_tiles == -(-rows // p.bn) and p.m_tiles == n // 128
    work_tiles = -(-p.m_tiles // p.mw) * p.n_tiles
    assert p.units == work_tiles * (k // (64 * p.kg))


@pytest.mark.parametrize("rows,k,n", SHAPES)
def test_single_gpu_plans_fit_the_hardware_and_the_workspace(rows, k, n):
    ws = N.lib().ls_gemm_workspace_bytes(rows, k, n)
    for epi in EPILOGUES:
        p = _plan(rows, k, n, epi)
        _check_fits(p, rows, k, n)
        assert p.workspace_bytes <= ws, (rows, k, n, epi)
        if epi in (N.EPI_QKV, N.EPI_GATEUP):
            assert p.mw == 1  # these epilogues are planned with one feature tile per work tile
        if rows <= 64:
            assert p.mw == 1  # weight streaming keeps the token-tile rule


@pytest.mark.parametrize("rows,k,n", [s for s in SHAPES if s[2] <= 24576])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_plans_fit_the_exchange_region(rows, k, n, world):
    ws = N.lib().ls_gemm_workspace_bytes(rows, k, n)
    for epi in (N.EPI_STORE, N.EPI_RESIDUAL):
        for wire in (N.TP_WIRE_F32, N.TP_WIRE_BF16):
            p = _plan(rows, k, n, epi, fused=1, world=world, wire=wire)
            _check_fits(p, rows, k, n)
            assert p.mw == 1 and p.kernel_weight_streaming == 0
            assert p.m_tiles * p.n_tiles <= 4096  # the exchange's per-tile flags
            assert p.workspace_bytes <= ws
            assert p.tp_sync_bytes <= N.lib().ls_tp_sync_bytes(world, rows, n, wire), (rows, k, n, world, wire)


def test_plan_info_rejects_bad_arguments():
    p = N.GemmPlan()
    lib = N.lib()
    assert lib.ls_gemm_plan_info(0, 64, 128, 0, 0, 1, 0, C.byref(p)) == 1
    assert lib.ls_gemm_plan_info(16, 65, 128, 0, 0, 1, 0, C.byref(p)) == 1
    assert lib.ls_gemm_plan_info(16, 64, 100, 0, 0, 1, 0, C.byref(p)) == 1
    assert lib.ls_gemm_plan_info(16, 64, 128, 9, 0, 1, 0, C.byref(p)) == 1
    assert lib.ls_gemm_plan_info(16, 64, 128, 0, 1, 9, 0, C.byref(p)) == 1
    assert lib.ls_gemm_plan_info(16, 64, 128, 0, 0, 1, 0, None) == 1


def test_many_token_plans_of_the_measured_shapes():
    """A few picks measured on a B200 (see the planner's comment in gemm.cu):
    480 tokens of the QKV projection run one 160-token tile per CTA, the
    vocabulary projection at 480 tokens two feature tiles per work tile."""
    q = _plan(480, 4096, 6144, N.EPI_QKV)
    assert (q.bn, q.mw, q.grid) == (160, 1, 144)
    lm = _plan(480, 4096, 151936, N.EPI_LMHEAD)
    assert (lm.bn, lm.mw) == (240, 2)
