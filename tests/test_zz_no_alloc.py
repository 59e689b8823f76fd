"""The zero-allocation entry point, aie_conv_run_noalloc.

It exists for callers that cannot allocate device memory while they run: a
real-time frame loop that cannot absorb cudaMalloc's device
synchronisation, a plugin that only ever sees its host's tensors, code that
runs during CUDA-graph capture.  Such callers get split-K scratch from a
fixed 16 MiB array inside the library instead of passing a workspace.

The test calls it through the C ABI on a split-K plan (BASELINE config 3 at
batch 1, which needs scratch) twice in a row, and checks each result
against the ordinary aie_conv_run with a caller workspace, within the TF32
tolerance the other tests use.  It also checks that a plan needing more
scratch than the array holds is refused with a clear message.  This file is
named to run last, and passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from ai_engine_b200 import Conv2d, _lib
from ai_engine_b200.conv import ConvPlan
from tests._util import TOL_TF32

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_matches_workspace_path_on_two_calls(cuda_ok):
    lib = _lib.load()
    rng = np.random.default_rng(2024)
    op = Conv2d.pointwise(960, 1280, "relu")
    x = torch.from_numpy(rng.uniform(-1, 1, (1, 10, 18, 960)).astype(np.float32)).cuda()
    w = (rng.standard_normal(1280 * 960) / np.sqrt(960)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 1280).astype(np.float32)
    plan = ConvPlan(op, 1, 10, 18, math="tf32").load_weights(w, b)
    assert plan.info.split_k > 1, "the case must exercise split-K scratch"
    assert 0 < plan.info.workspace_bytes <= _lib.NOALLOC_SCRATCH_BYTES
    ref = plan(x)  # existing entry point, caller-owned workspace
    # magnitude the TF32 rounding is relative to: |b| + sum |x w|
    scale = ConvPlan(Conv2d.pointwise(960, 1280, "none"), 1, 10, 18, math="ffma") \
        .load_weights(np.abs(w), np.abs(b))(x.abs())
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        out = torch.full_like(ref, float("nan"))
        st = lib.aie_conv_run_noalloc(plan._h, _p(x), _p(plan.w), _p(plan.b), None, _p(out), stream)
        assert st == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all(), f"call {call}: output not fully written"
        err = ((out.double() - ref.double()).abs() / torch.maximum(ref.double().abs(), scale.double())).max().item()
        assert err <= TOL_TF32, f"call {call}: normalised error {err}"


def test_noalloc_refuses_plans_larger_than_its_scratch(cuda_ok):
    lib = _lib.load()
    op = Conv2d.pointwise(1280, 2048, "none")
    plan = ConvPlan(op, 1, 10, 18, math="tf32", split_k=16)
    assert plan.info.workspace_bytes > _lib.NOALLOC_SCRATCH_BYTES
    plan.load_weights(np.zeros(2048 * 1280, np.float32), None)
    x = torch.zeros(1, 10, 18, 1280, device="cuda")
    out = torch.empty(1, 10, 18, 2048, device="cuda")
    st = lib.aie_conv_run_noalloc(plan._h, _p(x), _p(plan.w), _p(plan.b), None, _p(out),
                                  C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == -3  # AIE_E_UNSUPPORTED
    assert "scratch" in _lib.last_error()
