"""BASELINE configs 2 and 3 at their largest batch (256 frames), against
the CPU oracle on sampled frames.

The GPU runs the whole batch in one launch, exactly as bench.py's
``--workload cfg2`` / ``cfg3`` lines time it; the oracle (the C
restatement of ai-cpu's conv_std) recomputes a few frames spread over the
batch -- the first, one in the middle and the last -- so that every part of
the persistent schedule (first wave, middle, ragged last tile) is covered.
Each conv is held to its math's bar on the normalised error (TF32 5e-3,
FFMA 1e-5); messages carry the plain max relative error as well.

Config 2: 3x3 pad 1 at 160x288, bias + HardSwish, (Cin, Cout) in
(16,16) ... (128,256), stride 1 and 2.  Config 3: 1x1 at 10x18 with deep K,
split-K on the tensor cores (auto and the sweep's explicit factors).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200 import Conv2d
from ai_engine_b200.conv import ConvPlan
from tests._util import TOL_FFMA, TOL_TF32, errors, normalised_error

pytestmark = pytest.mark.gpu

B = 256
FRAMES = [0, 131, 255]
THREADS = os.cpu_count() or 1


def _uniform_frames(shape, seed):
    """U(-1, 1) frames made on the GPU (a 256-frame batch is up to 6 GB) and
    the sampled frames' host copy for the oracle."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    xd = torch.rand(shape, device="cuda", generator=g).mul_(2).sub_(1)
    return xd, xd.index_select(0, torch.tensor(FRAMES, device="cuda")).cpu().numpy()


def _check_sampled(op, plan, xs, w, b, got, tol):
    """xs, got: the sampled frames' input and GPU output."""
    p = oracle.Plan(op, xs.shape[1], xs.shape[2], w, b)
    for i, f in enumerate(FRAMES):
        ref = np.empty((p.oh, p.ow, op.cout), np.float32)
        p.run_frame(xs[i], ref, threads=THREADS)
        scale = oracle.dot_scale(op, xs[i:i + 1], w, b)[0]
        err = normalised_error(got[i], ref, scale)
        assert err <= tol, f"{plan.kernel}/{plan.math} frame {f}: {errors(got[i], ref, scale)} > {tol}"


@pytest.mark.parametrize("cin,cout,s", [(128, 256, 1), (16, 16, 1), (128, 256, 2), (64, 128, 1)])
def test_config2_b256_sampled_frames(cuda_ok, cin, cout, s):
    op = Conv2d.same(cin, cout, 3, s, "hardswish")
    rng = np.random.default_rng(7000 + cin + s)
    w = (rng.standard_normal(cout * cin * 9) * np.sqrt(2.0 / (9 * cin))).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    xd, xs = _uniform_frames((B, 160, 288, cin), 7000 + cin + s)
    idx = torch.tensor(FRAMES, device="cuda")
    for math, tol in (("auto", TOL_TF32), ("ffma", TOL_FFMA)):
        plan = ConvPlan(op, B, 160, 288, math=math).load_weights(w, b)
        if math == "auto":
            assert plan.math == "tf32" and plan.kernel == "igemm"
        got = plan(xd).index_select(0, idx).cpu().numpy()
        _check_sampled(op, plan, xs, w, b, got, tol)
        del plan
        torch.cuda.empty_cache()


@pytest.mark.parametrize("k,n", [(960, 1280), (1280, 960), (512, 2048)])
@pytest.mark.parametrize("split", [0, 8])
def test_config3_b256_sampled_frames(cuda_ok, k, n, split):
    rng = np.random.default_rng(k + 3 * n + split)
    op = Conv2d.pointwise(k, n, "none")
    w = (rng.standard_normal(n * k) / np.sqrt(k)).astype(np.float32)
    b = np.zeros(n, np.float32)
    xd, xs = _uniform_frames((B, 10, 18, k), k + 3 * n + split)
    plan = ConvPlan(op, B, 10, 18, math="tf32", split_k=split).load_weights(w, b)
    assert plan.math == "tf32"
    if split:
        assert plan.info.split_k > 1
    idx = torch.tensor(FRAMES, device="cuda")
    got = plan(xd).index_select(0, idx).cpu().numpy()
    _check_sampled(op, plan, xs, w, b, got, TOL_TF32)
