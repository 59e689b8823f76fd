"""The zero-allocation entry point, aie_conv_run_noalloc.

Some callers cannot allocate device memory while they run: a real-time
frame loop that cannot absorb cudaMalloc's implicit device
synchronisation, or a plugin whose host application owns the device
allocator and hands it only tensors.  Such callers get split-K scratch
from a fixed 16 MiB array inside the library instead of passing a
workspace.

The test calls it through the C ABI on split-K plans (BASELINE config 3 at
batch 1, which needs scratch) two calls in a row, and checks each result
bit for bit against the ordinary aie_conv_run with a caller workspace (the
same kernel and the same fixed-order split-K reduction, so the results must
be identical) and against the CPU oracle within the TF32 tolerance the
other tests use.  A second, smaller split-K plan then runs through the same
array after the larger one has left its partials there.  A plan needing
more scratch than the array holds is refused with a clear message.  This
file is named to run last, and passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200 import Conv2d, _lib
from ai_engine_b200.conv import ConvPlan
from tests._util import TOL_TF32, normalised_error

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def _case(k, n, split, seed):
    rng = np.random.default_rng(seed)
    op = Conv2d.pointwise(k, n, "relu")
    x = rng.uniform(-1, 1, (1, 10, 18, k)).astype(np.float32)
    w = (rng.standard_normal(n * k) / np.sqrt(k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    plan = ConvPlan(op, 1, 10, 18, math="tf32", split_k=split).load_weights(w, b)
    assert plan.info.split_k > 1, "the case must exercise split-K scratch"
    assert 0 < plan.info.workspace_bytes <= _lib.NOALLOC_SCRATCH_BYTES
    want = oracle.conv_aicpu(op, x, w, b)
    scale = oracle.dot_scale(op, x, w, b)
    return plan, torch.from_numpy(x).cuda(), want, scale


def _run_noalloc(lib, plan, x, like):
    out = torch.full_like(like, float("nan"))
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = lib.aie_conv_run_noalloc(plan._h, _p(x), _p(plan.w), _p(plan.b), None, _p(out), stream)
    assert st == 0, _lib.last_error()
    torch.cuda.synchronize()
    return out


def test_noalloc_matches_workspace_path_on_two_calls(cuda_ok):
    lib = _lib.load()
    big, xb, want_b, scale_b = _case(960, 1280, 0, 2024)
    ref = big(xb).clone()  # the existing entry point, with a caller-owned workspace
    for call in range(2):
        out = _run_noalloc(lib, big, xb, ref)
        assert torch.isfinite(out).all(), f"call {call}: output not fully written"
        assert torch.equal(out, ref), f"call {call}: differs from aie_conv_run"
        err = normalised_error(out.cpu().numpy(), want_b, scale_b)
        assert err <= TOL_TF32, f"call {call}: normalised error against the oracle {err:.2e}"
    # a smaller split-K plan through the same array, which still holds the
    # larger plan's partials and tickets
    small, xs, want_s, scale_s = _case(512, 256, 4, 2025)
    assert small.info.workspace_bytes < big.info.workspace_bytes
    ref_s = small(xs).clone()
    for call in range(2):
        out = _run_noalloc(lib, small, xs, ref_s)
        assert torch.equal(out, ref_s), f"smaller plan, call {call}: differs from aie_conv_run"
        assert normalised_error(out.cpu().numpy(), want_s, scale_s) <= TOL_TF32


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
