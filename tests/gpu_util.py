"""Helpers shared by the GPU tests (imported by test modules, not collected)."""

import numpy as np
import torch

import oracle as O
from longspark_b200 import ops


def bf16_step(ref):
    """One bf16 step at the largest magnitude of ``ref`` (2^(floor(log2 max|ref|) - 7))."""
    m = float(np.abs(np.asarray(ref, dtype=np.float32)).max())
    if m == 0.0:
        return 0.0
    return 2.0 ** (np.floor(np.log2(m)) - 7)


def to_np(t):
    return t.detach().float().cpu().numpy()


def gemm_ws(rows, k, n, device="cuda"):
    return torch.zeros(max(1, ops.gemm_workspace_bytes(rows, k, n)), dtype=torch.uint8, device=device)


def assert_bf16_close(actual, ref, *, steps=1.0, exact_frac=None, what=""):
    """|actual - ref| <= steps * (one bf16 step at the largest |ref|), and
    optionally a minimum fraction of bit-identical values."""
    a = np.asarray(actual, dtype=np.float32)
    r = np.asarray(ref, dtype=np.float32)
    tol = steps * bf16_step(r)
    err = float(np.abs(a - r).max()) if a.size else 0.0
    assert err <= tol, f"{what}: max |diff| {err:.3g} > {tol:.3g}"
    if exact_frac is not None:
        frac = float((a == r).mean())
        assert frac >= exact_frac, f"{what}: only {frac:.4f} bit-identical (< {exact_frac})"


def tokens_exact_or_tied(gpu_tokens, step_logits, what=""):
    """Every GPU token is the oracle's argmax, or its oracle logit equals the
    oracle maximum (a tie broken differently cannot happen for the first-max
    rule, so equality means identical) or lies within one bf16 step of it
    (a near-tie flipped by fp32 accumulation order).  Returns the tie count."""
    gt = np.asarray(gpu_tokens)
    lg = np.asarray(step_logits, dtype=np.float32)
    ref = O.greedy_argmax(lg)
    mism = gt != ref
    ties = 0
    if mism.any():
        best = lg.max(axis=-1)
        got = np.take_along_axis(lg, gt[..., None], axis=-1)[..., 0]
        step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(best), 1e-30))) - 7)
        near = (best - got) <= step
        bad = mism & ~near
        assert not bad.any(), f"{what}: {int(bad.sum())} tokens differ beyond a near-tie"
        ties = int(mism.sum())
    return ties
