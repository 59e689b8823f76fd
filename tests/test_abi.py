"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/aie_conv.h declares, and plans convs the way ai-gpu-runtime's
lower_op picks kernels (crates/ai-gpu-runtime/src/lowering.rs:130-168).
aie_conv_plan is host-only, so no CUDA call is made here."""
import ctypes as C
import os
import re

import pytest

from ai_engine_b200 import _lib
from ai_engine_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def header_symbols():
    src = open(os.path.join(ROOT, "include", "aie_conv.h")).read()
    return sorted(set(re.findall(r"AIE_API\s+[\w\s\*]*?\b(aie_\w+)\s*\(", src)))


def test_header_declares_the_binding(lib):
    names = header_symbols()
    assert len(names) >= 11
    assert sorted(_lib.SIGNATURES) == names


def test_every_declared_symbol_is_exported(lib):
    for name in header_symbols():
        assert hasattr(lib, name), name
    assert lib.aie_abi_version() == 2
    assert b"sm_100a" in lib.aie_build_info()


def test_struct_sizes_match_header(lib):
    # 11 u32 + pad[4] + 4 i32 + 7 u32 = 26 * 4 bytes
    assert C.sizeof(_lib.ConvDesc) == 29 * 4
    assert C.sizeof(_lib.PlanInfo) == 8 * 4 + 6 * 8


def plan(lib, **kw):
    d = _lib.ConvDesc()
    base = dict(n=1, ih=8, iw=8, cin=16, cout=16, kh=3, kw=3, sh=1, sw=1, dil=1, groups=1, act=0, layout=0,
                math=0)
    base.update(kw)
    pad = base.pop("pad", (1, 1, 1, 1))
    for k, v in base.items():
        setattr(d, k, v)
    for i in range(4):
        d.pad[i] = pad[i]
    h = C.c_void_p()
    st = lib.aie_conv_plan(C.byref(d), C.byref(h))
    info = _lib.PlanInfo()
    if st == 0:
        assert lib.aie_conv_plan_info(h, C.byref(info)) == 0
        lib.aie_plan_free(h)
    return st, info


def test_kernel_choice_mirrors_lower_op(lib):
    st, i = plan(lib, groups=16)
    assert st == 0 and i.kernel == _lib.KERNEL_DW
    st, i = plan(lib, kh=1, kw=1, pad=(0, 0, 0, 0), cout=64)
    assert st == 0 and i.kernel == _lib.KERNEL_PW
    st, i = plan(lib, kh=1, kw=1, pad=(0, 0, 0, 0), cout=2)
    assert st == 0 and i.kernel == _lib.KERNEL_PW_DOT
    st, i = plan(lib)
    assert st == 0 and i.kernel == _lib.KERNEL_IGEMM and (i.oh, i.ow) == (8, 8)
    # 1x1 with stride: the reference GPU rejects it; ai-cpu runs it as conv_std
    st, i = plan(lib, kh=1, kw=1, sh=2, sw=2, pad=(0, 0, 0, 0))
    assert st == 0 and i.kernel == _lib.KERNEL_IGEMM and (i.oh, i.ow) == (4, 4)


def test_stem_variant_is_reported(lib):
    # auto / tf32: the tensor-core stem (cin <= 3, cout = 32, no residual)
    for math in (_lib.MATH_AUTO, _lib.MATH_TF32):
        st, i = plan(lib, ih=160, iw=288, cin=3, cout=32, sh=2, sw=2, math=math)
        assert st == 0 and i.kernel == _lib.KERNEL_IGEMM and i.variant == 2 and i.math == _lib.MATH_TF32
        assert i.weight_bytes == 9 * 3 * 32 * 4 and i.workspace_bytes == 0
    # explicit FFMA, 4 input channels or another cout: the FFMA direct conv
    st, i = plan(lib, ih=160, iw=288, cin=3, cout=32, sh=2, sw=2, math=_lib.MATH_FFMA)
    assert st == 0 and i.variant == 1
    st, i = plan(lib, cin=4, cout=32, math=_lib.MATH_FFMA)
    assert st == 0 and i.variant == 1
    # cin = 4 under auto is TMA-compatible: the general tensor-core GEMM
    st, i = plan(lib, cin=4, cout=32)
    assert st == 0 and i.variant == 0 and i.math == _lib.MATH_TF32
    st, i = plan(lib, cin=3, cout=16)
    assert st == 0 and i.variant == 1
    st, i = plan(lib, cin=6, cout=32)
    assert st == 0 and i.variant == 0


def test_out_hw_and_work_accounting(lib):
    st, i = plan(lib, ih=160, iw=288, cin=16, cout=16, sh=2, sw=2, n=2)
    assert st == 0 and (i.oh, i.ow) == (80, 144)
    assert i.flops == 2 * 2 * 80 * 144 * 16 * 16 * 9
    assert i.min_bytes == 4 * (2 * 160 * 288 * 16 + 16 * 16 * 9 + 16 + 2 * 80 * 144 * 16)


@pytest.mark.parametrize("kw,status", [
    (dict(n=0), _lib.STATUS and -2), (dict(cin=0), -2), (dict(act=11), -2), (dict(layout=5), -2),
    (dict(math=9), -2), (dict(groups=4, cin=16, cout=16), -3), (dict(ih=1, iw=1, pad=(0, 0, 0, 0)), -2),
    (dict(in_stride=8), -2), (dict(kh=17, kw=17), -3)])
def test_invalid_descriptors_are_rejected(lib, kw, status):
    st, _ = plan(lib, **kw)
    assert st == status
    msg = _lib.last_error()
    assert msg, "a failure must leave a detail message"


def test_tf32_request_on_depthwise_is_unsupported(lib):
    st, _ = plan(lib, groups=16, math=_lib.MATH_TF32)
    assert st == -3


def test_status_strings(lib):
    for s in (0, -1, -2, -3, -4, -5, -6, -7):
        assert lib.aie_status_string(s)
    assert lib.aie_status_string(-99) == b"unknown status"


def test_null_arguments(lib):
    assert lib.aie_conv_plan(None, None) == -2
    assert lib.aie_conv_plan_info(None, None) == -2
    assert lib.aie_conv_run(None, None, None, None, None, None, None, None) == -2
    assert lib.aie_conv_pack_weights(None, 0, None, None, None, None, None) == -2
    assert lib.aie_resize_bilinear(1, 1, 1, 1, None, 1, 1, 0, None, 0, None, None) == -2
    lib.aie_plan_free(None)


def test_views_and_c4_layout_strides(lib):
    st, i = plan(lib, cin=6, cout=10, layout=_lib.LAYOUT_NHWC_C4)
    assert st == 0
    st, _ = plan(lib, cin=6, in_stride=10, in_coff=4)
    assert st == 0
    st, _ = plan(lib, cin=6, in_stride=10, in_coff=5)
    assert st == -2


def test_fused_head_rejects_plans_that_do_not_qualify(lib):
    """aie_conv_run_dw_pw checks both plans before any device call."""
    def mk(**kw):
        d = _lib.ConvDesc()
        base = dict(n=1, ih=8, iw=8, cin=16, cout=16, kh=3, kw=3, sh=1, sw=1, dil=1, groups=1, act=0, layout=0, math=0)
        base.update(kw)
        pad = base.pop("pad", (1, 1, 1, 1))
        for k, v in base.items():
            setattr(d, k, v)
        for i in range(4):
            d.pad[i] = pad[i]
        h = C.c_void_p()
        assert lib.aie_conv_plan(C.byref(d), C.byref(h)) == 0
        return h
    dw = mk(groups=16)
    pw = mk(kh=1, kw=1, pad=(0, 0, 0, 0), cout=2)
    conv = mk()
    strict_dw = mk(groups=16, math=_lib.MATH_FP32_STRICT)
    big_pw = mk(kh=1, kw=1, pad=(0, 0, 0, 0), cout=8)
    other_shape = mk(kh=1, kw=1, pad=(0, 0, 0, 0), cout=2, ih=4)
    p = C.c_void_p(16)
    for a, b in [(conv, pw), (strict_dw, pw), (dw, big_pw), (dw, other_shape), (dw, conv)]:
        assert lib.aie_conv_run_dw_pw(a, b, p, p, p, p, p, p, None) == -3
        assert _lib.last_error()
    assert lib.aie_conv_run_dw_pw(None, pw, p, p, p, p, p, p, None) == -2
    for h in (dw, pw, conv, strict_dw, big_pw, other_shape):
        lib.aie_plan_free(h)


def test_input_u8_argument_checks(lib):
    p = C.c_void_p(16)
    assert lib.aie_input_u8(1, 2, 2, 2, p, 0, p, None) == -2    # not RGB/RGBA
    assert lib.aie_input_u8(1, 2, 2, 3, p, 7, p, None) == -2    # bad layout
    assert lib.aie_input_u8(0, 2, 2, 3, p, 0, p, None) == -2    # empty batch
    assert lib.aie_input_u8(1, 2, 2, 3, None, 0, p, None) == -2
    assert lib.aie_input_u8(1, 2, 2, 3, p, 1, C.c_void_p(20), None) == -5  # C4 output must be 16-byte aligned


def test_concat_parts_plan_checks(lib):
    """aie_conv_plan_parts validates on the host: 1-3 parts summing to cin,
    a dense non-grouped conv on the tensor cores; a parts plan is refused by
    aie_conv_run and an ordinary plan by aie_conv_run_parts (both before any
    CUDA call)."""
    def desc(cin, cout, k, groups=1, math=0):
        d = _lib.ConvDesc()
        d.n, d.ih, d.iw, d.cin, d.cout, d.kh, d.kw, d.sh, d.sw = 2, 12, 20, cin, cout, k, k, 1, 1
        for i in range(4):
            d.pad[i] = k // 2
        d.dil, d.groups, d.act, d.math = 1, groups, 1, math
        return d
    h = C.c_void_p()
    pc = (C.c_uint32 * 3)(40, 24, 3)
    assert lib.aie_conv_plan_parts(C.byref(desc(67, 32, 3)), 3, pc, C.byref(h)) == 0
    info = _lib.PlanInfo()
    assert lib.aie_conv_plan_info(h, C.byref(info)) == 0
    assert info.math == _lib.MATH_TF32 and info.kernel == _lib.KERNEL_IGEMM
    # weights: [9 taps][32 cout][(2 + 1 + 1) K blocks x 32]
    assert info.weight_bytes == 9 * 32 * 4 * 32 * 4
    p = C.c_void_p(16)
    tv = (_lib.TView * 3)()
    assert lib.aie_conv_run(h, p, p, p, None, p, None, None) == -2
    lib.aie_plan_free(h)
    bad = [(desc(66, 32, 3), 3, (40, 24, 3), -2),       # parts sum to 67, not 66
           (desc(67, 32, 3), 0, (40, 24, 3), -2),       # no parts
           (desc(67, 32, 3), 4, (40, 24, 3), -2),       # more than 3
           (desc(64, 64, 3, groups=64), 2, (32, 32, 0), -3),  # depthwise
           (desc(64, 2, 1), 2, (32, 32, 0), -3),        # 1x1 with cout <= 4: the dot kernel
           (desc(64, 32, 3, math=1), 2, (32, 32, 0), -3)]     # FFMA
    for d, n, parts, want in bad:
        pcs = (C.c_uint32 * 4)(*parts, 0)
        assert lib.aie_conv_plan_parts(C.byref(d), n, pcs, C.byref(h)) == want, (n, parts, want)
        assert _lib.last_error()
    assert lib.aie_conv_plan(C.byref(desc(64, 32, 3)), C.byref(h)) == 0
    assert lib.aie_conv_run_parts(h, tv, p, p, None, p, None, None) == -2
    lib.aie_plan_free(h)


def test_input_yuv420_argument_checks(lib):
    p = 16
    def desc(**kw):
        d = _lib.Yuv420(p, p, p, 8, 4, 4, 1, 0, 0, 0)
        for k, v in kw.items():
            setattr(d, k, v)
        return C.byref(d)
    out = C.c_void_p(16)
    assert lib.aie_input_yuv420(1, 4, 8, None, 0, out, None) == -2                 # no planes
    assert lib.aie_input_yuv420(1, 4, 8, desc(y=None), 0, out, None) == -2
    assert lib.aie_input_yuv420(0, 4, 8, desc(), 0, out, None) == -2              # empty batch
    assert lib.aie_input_yuv420(1, 4, 8, desc(), 7, out, None) == -2               # bad layout
    assert lib.aie_input_yuv420(1, 4, 8, desc(uv_step=3), 0, out, None) == -2      # neither planar nor interleaved
    assert lib.aie_input_yuv420(1, 4, 8, desc(stride_y=7), 0, out, None) == -2     # luma row shorter than w
    assert lib.aie_input_yuv420(1, 4, 8, desc(stride_u=3), 0, out, None) == -2     # chroma row shorter than w/2
    assert lib.aie_input_yuv420(1, 4, 8, desc(uv_step=2), 0, out, None) == -2      # interleaved row spans 7 bytes
    assert lib.aie_input_yuv420(2, 4, 8, desc(frame_y=16), 0, out, None) == -2     # frames overlap
    assert lib.aie_input_yuv420(1, 4, 8, desc(), 1, C.c_void_p(20), None) == -5    # C4 output alignment
    assert "stride" in _lib.last_error() or "align" in _lib.last_error()


def test_glue_entry_points_reject_bad_arguments(lib):
    """The graph-glue entry points validate on the host and return a status
    (no launch, no CUDA call) for null pointers, zero sizes, out-of-range
    enums and views whose channels run past their pixel stride."""
    TV = _lib.TView
    buf = (C.c_float * 64)()
    good = TV(C.cast(buf, C.c_void_p), 0, 0)
    null = TV(None, 0, 0)
    inv = -2
    # aie_binary(n, px, c, a, op, kind, b, scalar, act, out, stream)
    assert lib.aie_binary(1, 4, 4, null, 0, 0, good, 0.0, 0, good, None) == inv
    assert lib.aie_binary(0, 4, 4, good, 0, 0, good, 0.0, 0, good, None) == inv
    assert lib.aie_binary(1, 4, 4, good, 9, 0, good, 0.0, 0, good, None) == inv
    assert lib.aie_binary(1, 4, 4, good, 0, 9, good, 0.0, 0, good, None) == inv
    assert lib.aie_binary(1, 4, 4, good, 0, 0, good, 0.0, 42, good, None) == inv
    assert lib.aie_binary(1, 4, 4, TV(C.cast(buf, C.c_void_p), 6, 3), 0, 0, good, 0.0, 0, good, None) == inv
    assert "pixel stride" in _lib.last_error()
    assert lib.aie_binary(1, 4, 4, good, 0, _lib.OPND_CVEC, null, 0.0, 0, good, None) == inv
    assert lib.aie_mix(1, 4, 4, good, null, good, good, None) == inv
    assert lib.aie_gpool(1, 4, 4, good, None, None) == inv
    assert lib.aie_gpool(1, 0, 4, good, C.cast(buf, C.c_void_p), None) == inv
    pad = (C.c_uint32 * 4)(0, 0, 0, 0)
    assert lib.aie_avgpool(1, 2, 2, 1, 3, 3, 1, 1, pad, C.cast(buf, C.c_void_p), C.cast(buf, C.c_void_p), None) == inv
    assert lib.aie_avgpool(1, 2, 2, 1, 2, 2, 0, 1, pad, C.cast(buf, C.c_void_p), C.cast(buf, C.c_void_p), None) == inv
    assert lib.aie_channel_copy(1, 4, 4, good, 11, good, None) == inv
    assert lib.aie_channel_copy(1, 4, 4, good, 0, TV(C.cast(buf, C.c_void_p), 4, 1), None) == inv
    assert "pixel stride" in _lib.last_error()


def test_concat_rejects_bad_arguments(lib):
    TV = _lib.TView
    buf = (C.c_float * 64)()
    good = TV(C.cast(buf, C.c_void_p), 0, 0)
    parts = (TV * 2)(good, good)
    cs = (C.c_uint32 * 2)(2, 2)
    assert lib.aie_concat(1, 4, 0, parts, cs, 4, good, None) == -2
    assert lib.aie_concat(1, 4, 9, parts, cs, 4, good, None) == -2
    assert lib.aie_concat(1, 4, 2, parts, cs, 3, good, None) == -2      # parts wider than the output
    assert "out_c" in _lib.last_error()
    cs0 = (C.c_uint32 * 2)(2, 0)
    assert lib.aie_concat(1, 4, 2, parts, cs0, 4, good, None) == -2
    assert lib.aie_concat(1, 4, 2, None, cs, 4, good, None) == -2
