"""Shared helpers for the parity tests (test infrastructure only)."""
from __future__ import annotations

import numpy as np

import oracle
from oracle import XorShift32

# Tolerances of the north-star contract, on the normalised error below.
TOL_FFMA = 1e-5
TOL_TF32 = 5e-3
# Transcendental activations: CUDA's expf/tanhf and glibc's may differ by
# an ulp or two, so "strict" math is compared bit for bit only without them.
EXACT_ACTS = {"none", "relu", "hardswish", "hardsigmoid", "clamp01", "relu6", "neg"}


def normalised_error(got, want, scale) -> float:
    """max |got - want| / max(|want|, scale).  `scale` is |bias| + sum_k |x_k w_k|
    (+ |res|): the magnitude the reordered sum's rounding is relative to.
    This keeps "relative error" meaningful at outputs that cancel to ~0
    and at activation kinks."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.maximum(np.maximum(np.abs(want), np.asarray(scale, np.float64)), 1e-30)
    return float(np.max(np.abs(got - want) / den)) if got.size else 0.0


def case_tensors(op, n, ih, iw, seed, with_res):
    """Inputs in ai-gpu testsuite draw order: input, weights, bias, residual
    (crates/ai-gpu/src/testsuite.rs:337-341)."""
    rng = XorShift32(seed)
    x = rng.vec_f32(n * ih * iw * op.cin).reshape(n, ih, iw, op.cin)
    w = rng.vec_f32(op.cout * (op.cin // op.groups) * op.kh * op.kw)
    b = rng.vec_f32(op.cout)
    oh, ow = op.out_hw(ih, iw)
    res = rng.vec_f32(n * oh * ow * op.cout).reshape(n, oh, ow, op.cout) if with_res else None
    return x, w, b, res


def oracle_conv(op, x, w, b, res):
    want = oracle.conv_aicpu(op, x, w, b, res)
    scale = oracle.dot_scale(op, x, w, b)
    if res is not None:
        scale = scale + np.abs(res)
    return want, scale
