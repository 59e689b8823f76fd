"""ctypes binding of ``libaie_conv.so`` (the C ABI in ``include/aie_conv.h``).

The product path has no CPU fallback: importing this module on a machine
without the built library raises, and every ABI call that returns a
non-zero status raises ``AieError`` with the library's detail message.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaie_conv.so")

AIE_OK = 0
STATUS = {0: "AIE_OK", -1: "AIE_E_FAILURE", -2: "AIE_E_INVALID", -3: "AIE_E_UNSUPPORTED", -4: "AIE_E_CUDA",
          -5: "AIE_E_ALIGN", -6: "AIE_E_DEVICE_TIMEOUT", -7: "AIE_E_NOMEM"}

LAYOUT_NHWC, LAYOUT_NHWC_C4 = 0, 1
MATH_AUTO, MATH_FFMA, MATH_TF32, MATH_FP32_STRICT = 0, 1, 2, 3
KERNEL_DW, KERNEL_PW, KERNEL_IGEMM, KERNEL_PW_DOT = 1, 2, 3, 4
WFMT_OIHW, WFMT_SW_PACKED = 0, 1
RES_TENSOR, RES_BILINEAR_HALF_PIXEL, RES_BILINEAR_ASYMMETRIC = 0, 1, 2
NOALLOC_SCRATCH_BYTES = 16 << 20  # AIE_NOALLOC_SCRATCH_BYTES


class AieError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        self.status = status
        super().__init__(f"{where}: {STATUS.get(status, status)}: {detail}")


class ConvDesc(C.Structure):
    _fields_ = [("n", C.c_uint32), ("ih", C.c_uint32), ("iw", C.c_uint32), ("cin", C.c_uint32),
                ("cout", C.c_uint32), ("kh", C.c_uint32), ("kw", C.c_uint32), ("sh", C.c_uint32),
                ("sw", C.c_uint32), ("pad", C.c_uint32 * 4), ("dil", C.c_uint32), ("groups", C.c_uint32),
                ("act", C.c_int32), ("has_res", C.c_int32), ("layout", C.c_int32), ("math", C.c_int32),
                ("split_k", C.c_uint32), ("in_stride", C.c_uint32), ("in_coff", C.c_uint32),
                ("res_stride", C.c_uint32), ("res_coff", C.c_uint32), ("out_stride", C.c_uint32),
                ("out_coff", C.c_uint32), ("res_mode", C.c_int32), ("res_h", C.c_uint32), ("res_w", C.c_uint32)]


class PlanInfo(C.Structure):
    _fields_ = [("kernel", C.c_int32), ("math", C.c_int32), ("oh", C.c_uint32), ("ow", C.c_uint32),
                ("split_k", C.c_uint32), ("tile_m", C.c_uint32), ("tile_n", C.c_uint32),
                ("variant", C.c_uint32), ("weight_bytes", C.c_uint64), ("bias_bytes", C.c_uint64),
                ("workspace_bytes", C.c_uint64), ("flops", C.c_uint64), ("min_bytes", C.c_uint64),
                ("grid_ctas", C.c_uint64)]


class TView(C.Structure):
    """aie_tview: a channel view of an NHWC buffer (data, pixel stride, first channel)."""
    _fields_ = [("data", C.c_void_p), ("stride", C.c_uint32), ("coff", C.c_uint32)]


class Yuv420(C.Structure):
    """aie_yuv420: the planes of a batch of YUV 4:2:0 frames."""
    _fields_ = [("y", C.c_void_p), ("u", C.c_void_p), ("v", C.c_void_p), ("stride_y", C.c_uint32),
                ("stride_u", C.c_uint32), ("stride_v", C.c_uint32), ("uv_step", C.c_uint32),
                ("frame_y", C.c_uint64), ("frame_u", C.c_uint64), ("frame_v", C.c_uint64)]


BIN_OPS = {"add": 0, "sub": 1, "mul": 2, "prelu": 3}          # aie_binop
OPND_TENSOR, OPND_SCALAR, OPND_SCALAR_FIRST, OPND_CVEC, OPND_CVEC_TENSOR, OPND_PVEC_TENSOR = range(6)

# Every symbol include/aie_conv.h declares, with its ctypes signature.
_vp, _fp = C.c_void_p, C.POINTER(C.c_float)
SIGNATURES = {
    "aie_abi_version": (C.c_int32, []),
    "aie_build_info": (C.c_char_p, []),
    "aie_conv_plan": (C.c_int, [C.POINTER(ConvDesc), C.POINTER(_vp)]),
    "aie_conv_plan_info": (C.c_int, [_vp, C.POINTER(PlanInfo)]),
    "aie_plan_free": (None, [_vp]),
    "aie_conv_pack_weights": (C.c_int, [_vp, C.c_int32, _fp, _fp, _vp, _vp, _vp]),
    "aie_conv_run": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "aie_conv_run_noalloc": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "aie_conv_plan_parts": (C.c_int, [C.POINTER(ConvDesc), C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(_vp)]),
    "aie_resize_bilinear": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, _vp, C.c_uint32,
                                      C.c_uint32, C.c_int32, _vp, C.c_int32, _vp, _vp]),
    "aie_status_string": (C.c_char_p, [C.c_int]),
    "aie_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "aie_device_status": (C.c_int, [_vp, C.POINTER(C.c_uint32)]),
    "aie_conv_run_dw_pw": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "aie_conv_run_dw_pw_up2": (C.c_int, [_vp, _vp, _vp, _vp, C.c_uint32, C.c_uint32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "aie_conv_run_mbconv": (C.c_int, [_vp] * 13),
    "aie_conv_run_stem_pw": (C.c_int, [_vp] * 10),
    "aie_input_u8": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, _vp, C.c_int32, _vp, _vp]),
    "aie_input_yuv420": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(Yuv420), C.c_int32, _vp, _vp]),
    "aie_selftest_wait_timeout": (C.c_int, [C.c_uint32, _vp]),
    "aie_binary": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, TView, C.c_int32, C.c_int32, TView, C.c_float,
                             C.c_int32, TView, _vp]),
    "aie_mix": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, TView, TView, TView, TView, _vp]),
    "aie_gpool": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, TView, _vp, _vp]),
    "aie_avgpool": (C.c_int, [C.c_uint32] * 8 + [C.POINTER(C.c_uint32), _vp, _vp, _vp]),
    "aie_channel_copy": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, TView, C.c_int32, TView, _vp]),
    "aie_concat": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(TView), C.POINTER(C.c_uint32), C.c_uint32,
                             TView, _vp]),
    "aie_conv_run_parts": (C.c_int, [_vp, C.POINTER(TView), _vp, _vp, _vp, _vp, _vp, _vp]),
}

_LIB = None


def load(path: str = LIB_PATH):
    """Load the library (once).  Raises if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m ai_engine_b200.build` "
                          "(the conv path has no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def last_error() -> str:
    buf = C.create_string_buffer(512)
    load().aie_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, where: str):
    if status != AIE_OK:
        raise AieError(status, where, last_error())
