"""Seeded inputs of the T > 0 rejection-sampling fixtures, shared by the
fixture generator (``make_golden.py``, which runs the reference's
``decide_acceptance`` / ``finish_sampling`` on them) and the tests (which
rebuild them from the stored seeds and compare with the stored outputs).

The drafter's corrected logits are N(0, sigma_draft); the target's logits
are the drafter's plus N(0, sigma_noise), so the two distributions overlap and
acceptance runs a few tokens deep; the first ``same_rows`` requests get target
rows equal to the drafter's, and the generator gives them q = 1, so they
reject where the uniform exceeds p and meet a residual of zero mass there (the
reference's fallback to the target row).  Both are rounded to bf16, the dtype the logits have on
the device.  Candidates are drawn from softmax(draft / T) by inverse CDF.
"""

from __future__ import annotations

import numpy as np
import torch


def sampling_logits(batch, block, vocab, seed, sigma_draft, sigma_noise, same_rows):
    """(target [B, P + 1, V], draft [B, P, V]) as bf16 torch tensors."""
    rng = np.random.default_rng(seed)
    draft = rng.standard_normal((batch, block + 1, vocab), dtype=np.float32) * np.float32(sigma_draft)
    target = draft + rng.standard_normal((batch, block + 1, vocab), dtype=np.float32) * np.float32(sigma_noise)
    target[:same_rows] = draft[:same_rows]
    t = torch.from_numpy(target).to(torch.bfloat16)
    d = torch.from_numpy(np.ascontiguousarray(draft[:, :block])).to(torch.bfloat16)
    return t, d


def sampling_draws(draft, temperature, seed):
    """Candidates [B, P] int64 drawn from softmax(draft / T), the acceptance
    uniforms [B, P] and the final uniforms [B] (float32)."""
    rng = np.random.default_rng(seed + 1)
    probs = torch.softmax(draft.float() / temperature, -1).numpy()
    b, p, v = probs.shape
    u = rng.random((b, p), dtype=np.float32)
    cdf = np.cumsum(probs.astype(np.float64), axis=-1)
    cand = np.minimum((cdf < u[..., None]).sum(-1), v - 1).astype(np.int64)
    uniforms = rng.random((b, p), dtype=np.float32)
    final = rng.random(b, dtype=np.float32)
    return cand, uniforms, final


# name -> (batch, block, vocab, temperature, seed, sigma_draft, sigma_noise, same_rows)
CASES = {
    "v4096_p7": (64, 7, 4096, 0.8, 401, 2.0, 0.5, 6),
    "v151936_p15": (8, 15, 151936, 1.0, 402, 3.0, 0.3, 1),
    "v151936_p7": (8, 7, 151936, 0.6, 403, 2.0, 0.2, 1),
}
