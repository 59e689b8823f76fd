"""Golden vectors (tests/golden/conv_cases.npz, made by make_golden.py from
the reference's own kernel-test cases and seeds).

CPU: the oracle reproduces the committed bytes exactly, and agrees with the
naive reference conv within the reference's own test tolerance
(|a-b| <= 1e-4 * max(|a|, 1), crates/ai-cpu/src/kernels/conv.rs:503-508).
GPU: the CUDA path through the C ABI matches the golden outputs --
bit-exact in fp32_strict mode (transcendental activations within FFMA
tolerance), <= 1e-5 normalised in FFMA mode, <= 5e-3 in TF32 mode.
"""
import os

import numpy as np
import pytest

import oracle
from tests._util import EXACT_ACTS, TOL_FFMA, TOL_TF32, normalised_error

HERE = os.path.dirname(os.path.abspath(__file__))
from tests.golden.make_golden import CASES, Op  # noqa: E402

G = np.load(os.path.join(HERE, "golden", "conv_cases.npz"))


def conv_of(name):
    return Op(CASES[name])


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_reproduces_golden_bytes(name):
    op = conv_of(name)
    x, w, b = G[f"{name}/x"], G[f"{name}/w"], G[f"{name}/b"]
    res = G[f"{name}/res"] if f"{name}/res" in G else None
    _, ih, iw, _ = x.shape
    plan = oracle.Plan(op, ih, iw, w, b, True, res is not None)
    y = np.empty(G[f"{name}/y"].size, np.float32)
    plan.run_frame(np.ascontiguousarray(x.reshape(-1)), y, None if res is None else np.ascontiguousarray(res.reshape(-1)))
    assert np.array_equal(y, G[f"{name}/y"].reshape(-1))
    ref = G[f"{name}/ref"].reshape(-1)
    assert np.all(np.abs(ref - y) <= 1e-4 * np.maximum(np.abs(ref), 1.0))


def test_resize_golden():
    x = G["resize/x"]
    assert np.array_equal(oracle.resize_bilinear(x, 10, 14, "half_pixel"), G["resize/half_pixel"])
    assert np.array_equal(oracle.resize_bilinear(x, 10, 14, "asymmetric"), G["resize/asymmetric"])


@pytest.mark.gpu
@pytest.mark.parametrize("math", ["fp32_strict", "ffma", "tf32"])
@pytest.mark.parametrize("name", sorted(CASES))
def test_cuda_matches_golden(cuda_ok, name, math):
    import torch
    from ai_engine_b200 import Conv2d
    from ai_engine_b200._lib import AieError
    from ai_engine_b200.conv import ConvPlan
    o = conv_of(name)
    op = Conv2d(o.cin, o.cout, o.kh, o.kw, o.sh, o.sw, tuple(o.pad), o.dil, o.groups, o.act)
    x, w, b, want = G[f"{name}/x"], G[f"{name}/w"], G[f"{name}/b"], G[f"{name}/y"]
    res = G[f"{name}/res"] if f"{name}/res" in G else None
    try:
        plan = ConvPlan(op, 1, x.shape[1], x.shape[2], has_res=res is not None, math=math).load_weights(w, b)
    except AieError as e:
        assert math == "tf32" and e.status == -3  # memory-bound families / cin % 4 != 0 have no TF32 form
        return
    got = plan(torch.from_numpy(x).cuda(), None if res is None else torch.from_numpy(res).cuda()).cpu().numpy()
    if math == "fp32_strict" and op.act in EXACT_ACTS:
        assert np.array_equal(got, want)
    else:
        scale = oracle.dot_scale(o, x, w, b) + (0 if res is None else np.abs(res))
        tol = TOL_TF32 if plan.math == "tf32" else TOL_FFMA
        assert normalised_error(got, want, scale) <= tol


@pytest.mark.gpu
def test_cuda_resize_golden(cuda_ok):
    import torch
    from ai_engine_b200 import resize_bilinear
    x = torch.from_numpy(G["resize/x"]).cuda()
    assert np.array_equal(resize_bilinear(x, 10, 14, "half_pixel").cpu().numpy(), G["resize/half_pixel"])
    assert np.array_equal(resize_bilinear(x, 10, 14, "asymmetric").cpu().numpy(), G["resize/asymmetric"])
