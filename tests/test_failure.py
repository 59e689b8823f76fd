"""Failure detection without a GPU fault.

Host side (no GPU): every ABI entry returns a status for bad input instead
of aborting, with a detail message -- the reference's FFI contract
(ai-ffi catch_unwind -> VbResult::Failure, crates/ai-ffi/src/lib.rs:179).
Device side: a bounded wait that runs out sets the device error word, the
host reads AIE_E_DEVICE_TIMEOUT, and the context stays usable (the
reference's device-loss test, crates/ai-gpu/tests/device_lost.rs, is the
counterpart).  Nothing here traps, faults or hangs a GPU.
"""
import ctypes as C

import numpy as np
import pytest

from ai_engine_b200 import _lib
from ai_engine_b200.build import build


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def _desc(**kw):
    d = _lib.ConvDesc()
    base = dict(n=1, ih=8, iw=8, cin=16, cout=16, kh=1, kw=1, sh=1, sw=1, dil=1, groups=1)
    base.update(kw)
    for k, v in base.items():
        setattr(d, k, v)
    return d


def test_run_rejects_missing_buffers(lib):
    d = _desc(has_res=1)
    h = C.c_void_p()
    assert lib.aie_conv_plan(C.byref(d), C.byref(h)) == 0
    fake = C.c_void_p(0x1000)
    # residual plan without a residual pointer: refused before any launch
    assert lib.aie_conv_run(h, fake, fake, fake, None, fake, None, None) == -2
    assert "residual" in _lib.last_error()
    # unaligned weights: refused before any launch
    odd = C.c_void_p(0x1004)
    assert lib.aie_conv_run(h, fake, odd, fake, fake, fake, None, None) == -5
    lib.aie_plan_free(h)


def test_split_k_plan_requires_workspace(lib):
    d = _desc(ih=10, iw=18, cin=960, cout=1280, math=_lib.MATH_TF32, split_k=8)
    h = C.c_void_p()
    assert lib.aie_conv_plan(C.byref(d), C.byref(h)) == 0
    fake = C.c_void_p(0x1000)
    assert lib.aie_conv_run(h, fake, fake, fake, None, fake, None, None) == -2
    assert "workspace" in _lib.last_error()
    lib.aie_plan_free(h)


def test_pack_rejects_bad_format(lib):
    d = _desc()
    h = C.c_void_p()
    assert lib.aie_conv_plan(C.byref(d), C.byref(h)) == 0
    w = np.zeros(256, np.float32)
    fp = C.POINTER(C.c_float)
    assert lib.aie_conv_pack_weights(h, 7, w.ctypes.data_as(fp), None, C.c_void_p(1), C.c_void_p(1), None) == -2
    lib.aie_plan_free(h)


def test_selftest_rejects_bad_timeout(lib):
    assert lib.aie_selftest_wait_timeout(0, None) == -2
    assert lib.aie_selftest_wait_timeout(10_000_000, None) == -2


@pytest.mark.gpu
def test_bounded_wait_expiry_is_reported_and_context_survives(lib, cuda_ok):
    import torch
    from ai_engine_b200 import Conv2d
    from ai_engine_b200.conv import ConvPlan
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    code = C.c_uint32(0)
    assert lib.aie_device_status(stream, C.byref(code)) == 0 and code.value == 0
    assert lib.aie_selftest_wait_timeout(20_000, stream) == 0  # 20 ms limit
    assert lib.aie_device_status(stream, C.byref(code)) == -6  # AIE_E_DEVICE_TIMEOUT
    assert code.value == 0x7F000001
    assert lib.aie_device_status(stream, C.byref(code)) == 0  # the word was cleared
    # the context is still usable: a conv runs and is correct
    op = Conv2d.pointwise(16, 16, "none")
    p = ConvPlan(op, 1, 4, 4, math="tf32").load_weights(np.eye(16, dtype=np.float32).reshape(-1), None)
    x = torch.rand(1, 4, 4, 16, device="cuda")
    assert torch.allclose(p(x), x, rtol=2e-3, atol=2e-3)
