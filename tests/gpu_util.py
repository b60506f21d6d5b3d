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


def bf16_ulp(v):
    """One bf16 step at |v| (elementwise): 2^(floor(log2 |v|) - 7)."""
    a = np.maximum(np.abs(np.asarray(v, dtype=np.float32)), np.float32(1e-30))
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def compare_chain_with_reference(gpu_tokens, ref_tokens, ref_top_vals, ref_top_ids, what="", max_steps=1.0):
    """GPU greedy tokens ``[B, P]`` against the reference's own tokens.

    Rows must agree token for token.  The one difference accepted is a tie in
    the reference's own bf16 logits: at the first step where a row differs,
    the GPU's token must be among the reference's top-k at that step with a
    value at most ``max_steps`` bf16 steps below the reference's maximum (0
    steps is an exact tie).  From that step on the row conditions on a different previous
    token, so its later steps are not compared with the reference.
    ``ref_top_vals`` / ``ref_top_ids``: ``[B, P, k]`` of the reference's
    corrected step logits, largest first.  Returns a list of (row, step, gap
    in bf16 steps) for those ties; raises on any other difference."""
    gt = np.asarray(gpu_tokens)
    rt = np.asarray(ref_tokens)
    ties = []
    for b in range(gt.shape[0]):
        diff = np.nonzero(gt[b] != rt[b])[0]
        if diff.size == 0:
            continue
        t = int(diff[0])
        ids = list(np.asarray(ref_top_ids[b, t]))
        vals = np.asarray(ref_top_vals[b, t], dtype=np.float32)
        assert gt[b, t] in ids, (f"{what}: row {b} step {t}: token {gt[b, t]} is not in the reference's top "
                                 f"{len(ids)} ({ids}, reference token {rt[b, t]})")
        gap = float(vals[0] - vals[ids.index(gt[b, t])])
        steps = gap / float(bf16_ulp(vals[0]))
        assert steps <= max_steps, (f"{what}: row {b} step {t}: token {gt[b, t]} is {steps:.2f} bf16 steps below the "
                              f"reference maximum (token {rt[b, t]}); not a tie")
        ties.append((b, t, steps))
    return ties
