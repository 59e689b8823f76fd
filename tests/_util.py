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


def plain_rel_error(got, want, floor: float = 1e-3) -> float:
    """The north-star's plain max relative error max |got - want| / |want|,
    over the outputs with |want| >= floor * max|want| (below that a
    relative error measures cancellation, not the kernel).  Reported beside
    the normalised error so the contract's own figure is visible."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if not want.size:
        return 0.0
    m = np.abs(want) >= floor * np.max(np.abs(want))
    if not m.any():
        return 0.0
    return float(np.max(np.abs(got[m] - want[m]) / np.abs(want[m])))


def errors(got, want, scale) -> str:
    """Both error figures, for assertion messages."""
    return (f"normalised {normalised_error(got, want, scale):.3e}, plain relative "
            f"{plain_rel_error(got, want):.3e} (|want| >= 1e-3 max)")


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


def check_net_ops(model, onet, weights, label=""):
    """Re-run every node of the step `model` (a NetModel) just recorded on
    the oracle net, from the GPU's own inputs to that node, and hold each op
    to its own bar: convs to the normalised tolerance of their math, glue
    ops bit-exact (4 ulp where they apply sigmoid or tanh).  Returns the set of (kernel, math) the convs used."""
    kinds = set()
    for rec in model.recs:
        nd = rec.node
        if nd.kind in ("split", "view"):
            continue
        ins = {i: model.tensor(i).cpu().numpy() for i in (*nd.ins, nd.res) if i is not None and i in model.shapes}
        want = onet.run_node(nd, ins)[nd.out]
        got = model.tensor(nd.out).cpu().numpy()
        assert got.shape == want.shape, nd.out
        if nd.kind == "conv":
            wt, b = weights[nd.out]
            scale = oracle.dot_scale(nd.conv, ins[nd.ins[0]], wt, b)
            if nd.res is not None:
                scale = scale + np.abs(ins[nd.res])
            tol = TOL_TF32 if rec.plan.math == "tf32" else TOL_FFMA
            err = normalised_error(got, want, scale)
            assert err <= tol, f"{label} {nd.out} ({rec.plan.kernel}/{rec.plan.math}): {err:.2e} > {tol}"
            kinds.add((rec.plan.kernel, rec.plan.math))
        elif nd.act in ("sigmoid", "tanh"):
            # CUDA's expf / tanhf against glibc's: within 4 ulp
            ulp = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
            assert np.all(np.abs(got.astype(np.float64) - want) <= 4 * ulp), f"{label} {nd.out} ({nd.kind}/{nd.act})"
        else:
            assert np.array_equal(got, want), \
                f"{label} {nd.out} ({nd.kind}): {float(np.max(np.abs(got - want))):.3e}"
    return kinds
