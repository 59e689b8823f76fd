"""Host-side mirror of ai_engine's conv operator surface over the C ABI.

``Conv2d`` restates crates/ai-core/src/ops/conv.rs:6-56; ``lower_conv``
plays the part of the ``SwOp::Conv`` arm of ai-gpu-runtime's ``lower_op``
(crates/ai-gpu-runtime/src/lowering.rs:99-187) and returns a ``ConvPlan``
that owns the packed device weights; calling the plan records one dispatch
on the current CUDA stream (kernel::record, crates/ai-gpu/src/kernel.rs:181).

PyTorch supplies device memory and streams only; all arithmetic runs in
``libaie_conv.so``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Sequence, Optional, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import check

# crates/ai-core/src/activation.rs:7-24, in enum order
ACTIVATIONS = ["none", "relu", "sigmoid", "tanh", "hardswish", "hardsigmoid", "clamp01", "relu6", "sqrt",
               "neg", "recip"]
ACT_ID = {a: i for i, a in enumerate(ACTIVATIONS)}
MATH = {"auto": _lib.MATH_AUTO, "ffma": _lib.MATH_FFMA, "tf32": _lib.MATH_TF32,
        "fp32_strict": _lib.MATH_FP32_STRICT}
MATH_NAME = {v: k for k, v in MATH.items()}
KERNEL_NAME = {_lib.KERNEL_DW: "dw", _lib.KERNEL_PW: "pw", _lib.KERNEL_IGEMM: "igemm",
               _lib.KERNEL_PW_DOT: "pw_dot"}
LAYOUT = {"nhwc": _lib.LAYOUT_NHWC, "nhwc_c4": _lib.LAYOUT_NHWC_C4}


@dataclass(frozen=True)
class Conv2d:
    """Conv attributes (crates/ai-core/src/ops/conv.rs:6-21)."""
    cin: int
    cout: int
    kh: int
    kw: int
    sh: int = 1
    sw: int = 1
    pad: Tuple[int, int, int, int] = (0, 0, 0, 0)  # top, left, bottom, right
    dil: int = 1
    groups: int = 1
    act: str = "none"

    @staticmethod
    def pointwise(cin: int, cout: int, act: str = "none") -> "Conv2d":
        return Conv2d(cin, cout, 1, 1, act=act)

    @staticmethod
    def depthwise(c: int, k: int, stride: int, act: str = "none") -> "Conv2d":
        p = (k - 1) // 2
        return Conv2d(c, c, k, k, stride, stride, (p, p, p, p), 1, c, act)

    @staticmethod
    def same(cin: int, cout: int, k: int, stride: int = 1, act: str = "none") -> "Conv2d":
        p = (k - 1) // 2
        return Conv2d(cin, cout, k, k, stride, stride, (p, p, p, p), 1, 1, act)

    def is_depthwise(self) -> bool:
        return self.groups == self.cin and self.cin == self.cout and self.groups > 1

    def out_hw(self, ih: int, iw: int) -> Tuple[int, int]:
        ekh = self.dil * (self.kh - 1) + 1
        ekw = self.dil * (self.kw - 1) + 1
        return ((ih + self.pad[0] + self.pad[2] - ekh) // self.sh + 1,
                (iw + self.pad[1] + self.pad[3] - ekw) // self.sw + 1)


@dataclass
class View:
    """Channel view of an NHWC buffer (SrcView, crates/ai-gpu/src/kernels/common/source.rs:17):
    pixel stride and first channel, in floats."""
    stride: int = 0
    coff: int = 0


def _stream_handle(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _dptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda or t.dtype != torch.float32:
        raise TypeError("conv tensors must be float32 CUDA tensors")
    return C.c_void_p(t.data_ptr())


class ConvPlan:
    """One lowered convolution with its packed device weights."""

    def __init__(self, op: Conv2d, n: int, ih: int, iw: int, *, has_res: bool = False, layout: str = "nhwc",
                 math: str = "auto", split_k: int = 0, in_view: Optional[View] = None,
                 res_view: Optional[View] = None, out_view: Optional[View] = None,
                 res_resize: Optional[Tuple[int, int, str]] = None, parts: Optional[Sequence[int]] = None,
                 device=None):
        self.lib = _lib.load()
        self.op, self.n, self.ih, self.iw = op, n, ih, iw
        self.layout = layout
        self.has_res = has_res
        d = _lib.ConvDesc()
        d.n, d.ih, d.iw, d.cin, d.cout = n, ih, iw, op.cin, op.cout
        d.kh, d.kw, d.sh, d.sw = op.kh, op.kw, op.sh, op.sw
        for i in range(4):
            d.pad[i] = op.pad[i]
        d.dil, d.groups, d.act = op.dil, op.groups, ACT_ID[op.act]
        d.has_res, d.layout, d.math, d.split_k = int(has_res), LAYOUT[layout], MATH[math], split_k
        for v, s, c in ((in_view, "in_stride", "in_coff"), (res_view, "res_stride", "res_coff"),
                        (out_view, "out_stride", "out_coff")):
            if v is not None:
                setattr(d, s, v.stride)
                setattr(d, c, v.coff)
        if res_resize is not None:
            # residual = bilinear sample of a [n, rh, rw, cout] tensor (fused Resize -> Conv(res))
            rh, rw, mode = res_resize
            d.res_mode = _lib.RES_BILINEAR_HALF_PIXEL if mode == "half_pixel" else _lib.RES_BILINEAR_ASYMMETRIC
            d.res_h, d.res_w = rh, rw
        self.res_resize = res_resize
        self.desc = d
        h = C.c_void_p()
        self.parts = tuple(int(c) for c in parts) if parts else None
        if self.parts:
            # concat-into-conv: the input is the channel concat of these
            # parts, read in place (aie_conv_plan_parts)
            pc = (C.c_uint32 * len(self.parts))(*self.parts)
            check(self.lib.aie_conv_plan_parts(C.byref(d), len(self.parts), pc, C.byref(h)), "aie_conv_plan_parts")
        else:
            check(self.lib.aie_conv_plan(C.byref(d), C.byref(h)), "aie_conv_plan")
        self._h = h
        info = _lib.PlanInfo()
        check(self.lib.aie_conv_plan_info(h, C.byref(info)), "aie_conv_plan_info")
        self.info = info
        self.kernel = "stem" if info.variant in (1, 2) else "pw_simt" if info.variant == 3 else KERNEL_NAME[info.kernel]
        self.math = MATH_NAME[info.math]
        self.oh, self.ow = info.oh, info.ow
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.w = None
        self.b = None
        self.workspace = None
        if info.workspace_bytes:
            self.workspace = torch.empty(int(info.workspace_bytes), dtype=torch.uint8, device=self.device)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self.lib.aie_plan_free(h)
            self._h = None

    # -- shapes ---------------------------------------------------------
    def cpad(self, c: int) -> int:
        return (c + 3) // 4 * 4 if self.layout == "nhwc_c4" else c

    def out_shape(self):
        return (self.n, self.oh, self.ow, self.cpad(self.op.cout))

    @property
    def flops(self) -> int:
        return int(self.info.flops)

    @property
    def min_bytes(self) -> int:
        return int(self.info.min_bytes)

    # -- weights ----------------------------------------------------------
    def load_weights(self, w: np.ndarray, bias: Optional[np.ndarray] = None, fmt: str = "oihw", stream=None):
        """Pack host weights (logical OIHW, or the .sw blob's packed form) into device memory."""
        w = np.ascontiguousarray(w, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.w = torch.empty(int(self.info.weight_bytes) // 4, dtype=torch.float32, device=self.device)
        self.b = torch.empty(int(self.info.bias_bytes) // 4, dtype=torch.float32, device=self.device)
        wf = _lib.WFMT_OIHW if fmt == "oihw" else _lib.WFMT_SW_PACKED
        fp = C.POINTER(C.c_float)
        check(self.lib.aie_conv_pack_weights(
            self._h, wf, w.ctypes.data_as(fp), None if b is None else b.ctypes.data_as(fp),
            C.c_void_p(self.w.data_ptr()), C.c_void_p(self.b.data_ptr()), C.c_void_p(_stream_handle(stream))),
            "aie_conv_pack_weights")
        return self

    # -- run ----------------------------------------------------------------
    def __call__(self, x: torch.Tensor, res: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                 stream=None) -> torch.Tensor:
        if self.w is None:
            raise RuntimeError("load_weights() first")
        if out is None:
            out = torch.empty(self.out_shape(), dtype=torch.float32, device=x.device)
        ws = None if self.workspace is None else C.c_void_p(self.workspace.data_ptr())
        check(self.lib.aie_conv_run(self._h, _dptr(x), C.c_void_p(self.w.data_ptr()), C.c_void_p(self.b.data_ptr()),
                                    _dptr(res), _dptr(out), ws, C.c_void_p(_stream_handle(stream))), "aie_conv_run")
        return out


def run_parts(plan: "ConvPlan", parts: Sequence, res: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
              stream=None) -> torch.Tensor:
    """Run a concat-into-conv plan (ConvPlan(..., parts=...)) over its parts,
    read in place (aie_conv_run_parts).  Each part is a dense [n, h, w, c_i]
    tensor or a (tensor, coff) channel view of a wider buffer [n, h, w,
    stride] holding the part at channels coff .. coff + c_i."""
    if not plan.parts or len(parts) != len(plan.parts):
        raise ValueError("plan and parts disagree")
    if plan.w is None:
        raise RuntimeError("load_weights() first")
    tv = (_lib.TView * len(parts))()
    for i, pt in enumerate(parts):
        t, coff = (pt, 0) if isinstance(pt, torch.Tensor) else pt
        tv[i] = _lib.TView(C.c_void_p(t.data_ptr()), t.shape[-1], coff)
    if out is None:
        out = torch.empty(plan.out_shape(), dtype=torch.float32, device=plan.device)
    ws = None if plan.workspace is None else C.c_void_p(plan.workspace.data_ptr())
    check(plan.lib.aie_conv_run_parts(plan._h, tv, C.c_void_p(plan.w.data_ptr()), C.c_void_p(plan.b.data_ptr()),
                                      _dptr(res), _dptr(out), ws, C.c_void_p(_stream_handle(stream))),
          "aie_conv_run_parts")
    return out


def run_dw_pw(dw: "ConvPlan", pw: "ConvPlan", x: torch.Tensor, out: Optional[torch.Tensor] = None,
              stream=None, up: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Depthwise conv `dw` and the 1x1 conv `pw` (cout <= 4) that consumes its
    output, in one launch (aie_conv_run_dw_pw): the depthwise result never
    reaches memory.  With `up` (a dense [n, h/2, w/2, C] tensor) the
    depthwise input is x + the exact-2x half_pixel resize of `up`
    (aie_conv_run_dw_pw_up2).  Raises AieError(AIE_E_UNSUPPORTED) for shapes
    the fused kernel does not cover."""
    if dw.w is None or pw.w is None:
        raise RuntimeError("load_weights() first")
    if out is None:
        out = torch.empty(pw.out_shape(), dtype=torch.float32, device=x.device)
    weights = (C.c_void_p(dw.w.data_ptr()), C.c_void_p(dw.b.data_ptr()), C.c_void_p(pw.w.data_ptr()),
               C.c_void_p(pw.b.data_ptr()))
    if up is None:
        check(dw.lib.aie_conv_run_dw_pw(dw._h, pw._h, _dptr(x), *weights, _dptr(out),
                                        C.c_void_p(_stream_handle(stream))), "aie_conv_run_dw_pw")
    else:
        if up.dim() != 4 or not up.is_contiguous():
            raise ValueError("up must be a dense [n, h, w, c] tensor")
        check(dw.lib.aie_conv_run_dw_pw_up2(dw._h, pw._h, _dptr(x), _dptr(up), up.shape[1], up.shape[2], *weights,
                                            _dptr(out), C.c_void_p(_stream_handle(stream))),
              "aie_conv_run_dw_pw_up2")
    return out


def run_mbconv(ex: "ConvPlan", dw: Optional["ConvPlan"], pj: "ConvPlan", x: torch.Tensor,
               res: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """An inverted-bottleneck block -- 1x1 expand `ex`, depthwise 3x3 `dw`,
    1x1 project `pj` (+ `res`) -- in one launch (aie_conv_run_mbconv) for
    frames up to 10 x 18: the expanded tensor never reaches memory.  `dw`
    None: the expand feeds the project directly.  Raises
    AieError(AIE_E_UNSUPPORTED) for blocks the fused kernel does not cover."""
    for p in (ex, dw, pj):
        if p is not None and p.w is None:
            raise RuntimeError("load_weights() first")
    if out is None:
        out = torch.empty(pj.out_shape(), dtype=torch.float32, device=x.device)
    check(ex.lib.aie_conv_run_mbconv(ex._h, dw._h if dw is not None else None, pj._h, _dptr(x),
                                     C.c_void_p(ex.w.data_ptr()), C.c_void_p(ex.b.data_ptr()),
                                     C.c_void_p(dw.w.data_ptr() if dw is not None else None),
                                     C.c_void_p(dw.b.data_ptr() if dw is not None else None),
                                     C.c_void_p(pj.w.data_ptr()),
                                     C.c_void_p(pj.b.data_ptr()), _dptr(res), _dptr(out),
                                     C.c_void_p(_stream_handle(stream))), "aie_conv_run_mbconv")
    return out


def run_stem_pw(stem: "ConvPlan", pw: "ConvPlan", x: torch.Tensor, stem_out: Optional[torch.Tensor] = None,
                pw_out: Optional[torch.Tensor] = None, stream=None):
    """The tensor-core stem and a 1x1 conv over its output (cin 32,
    cout <= 32) in one launch (aie_conv_run_stem_pw): both outputs are
    written, the 1x1 reads the stem's tile from shared memory.  Raises
    AieError(AIE_E_UNSUPPORTED) for plans outside that shape."""
    if stem.w is None or pw.w is None:
        raise RuntimeError("load_weights() first")
    if stem_out is None:
        stem_out = torch.empty(stem.out_shape(), dtype=torch.float32, device=x.device)
    if pw_out is None:
        pw_out = torch.empty(pw.out_shape(), dtype=torch.float32, device=x.device)
    check(stem.lib.aie_conv_run_stem_pw(stem._h, pw._h, _dptr(x), C.c_void_p(stem.w.data_ptr()),
                                        C.c_void_p(stem.b.data_ptr()), C.c_void_p(pw.w.data_ptr()),
                                        C.c_void_p(pw.b.data_ptr()), _dptr(stem_out), _dptr(pw_out),
                                        C.c_void_p(_stream_handle(stream))), "aie_conv_run_stem_pw")
    return stem_out, pw_out


def input_u8(frames: torch.Tensor, layout: str = "nhwc", out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """u8 RGB / RGBA frames [n, h, w, 3|4] on the GPU -> the network's f32
    input [n, h, w, 3] (NHWC) or [n, h, w, 4] (NHWC-C4), value / 255
    (aie_input_u8)."""
    if not frames.is_cuda or frames.dtype != torch.uint8 or frames.dim() != 4:
        raise TypeError("frames must be a uint8 CUDA tensor [n, h, w, c]")
    n, h, w, c = frames.shape
    if out is None:
        out = torch.empty((n, h, w, 4 if layout == "nhwc_c4" else 3), dtype=torch.float32, device=frames.device)
    check(_lib.load().aie_input_u8(n, h, w, c, C.c_void_p(frames.data_ptr()), LAYOUT[layout], _dptr(out),
                                   C.c_void_p(_stream_handle(stream))), "aie_input_u8")
    return out


def input_yuv420(y: torch.Tensor, u: torch.Tensor, v: Optional[torch.Tensor] = None, *, h: Optional[int] = None,
                 w: Optional[int] = None, nv21: bool = False, layout: str = "nhwc", out: Optional[torch.Tensor] = None,
                 stream=None) -> torch.Tensor:
    """YUV 4:2:0 frames on the GPU -> the network's f32 RGB input
    (aie_input_yuv420; ai-ffi's i420_to_rgba, then v / 255).

    I420: y [n, h, stride_y], u and v [n, ceil(h/2), stride_uv] uint8 planes.
    NV12 (v None): u is the interleaved chroma plane [n, ceil(h/2), stride]
    (U first; V first with nv21=True).  h, w default to y's rows and row
    length."""
    planes = [y, u] + ([v] if v is not None else [])
    if any((not p.is_cuda) or p.dtype != torch.uint8 or p.dim() != 3 or not p.is_contiguous() for p in planes):
        raise TypeError("planes must be contiguous uint8 CUDA tensors [n, rows, stride]")
    n = y.shape[0]
    h = y.shape[1] if h is None else h
    w = y.shape[2] if w is None else w
    d = _lib.Yuv420()
    d.y, d.stride_y, d.frame_y = y.data_ptr(), y.shape[2], y.shape[1] * y.shape[2]
    if v is not None:
        d.u, d.v, d.uv_step = u.data_ptr(), v.data_ptr(), 1
        d.stride_u, d.stride_v = u.shape[2], v.shape[2]
        d.frame_u, d.frame_v = u.shape[1] * u.shape[2], v.shape[1] * v.shape[2]
    else:
        base = u.data_ptr()
        d.u, d.v, d.uv_step = (base + 1, base, 2) if nv21 else (base, base + 1, 2)
        d.stride_u = d.stride_v = u.shape[2]
        d.frame_u = d.frame_v = u.shape[1] * u.shape[2]
    if out is None:
        out = torch.empty((n, h, w, 4 if layout == "nhwc_c4" else 3), dtype=torch.float32, device=y.device)
    check(_lib.load().aie_input_yuv420(n, h, w, C.byref(d), LAYOUT[layout], _dptr(out),
                                       C.c_void_p(_stream_handle(stream))), "aie_input_yuv420")
    return out


def lower_conv(op: Conv2d, n: int, ih: int, iw: int, w: np.ndarray, bias: Optional[np.ndarray] = None, *,
               has_res: bool = False, layout: str = "nhwc", math: str = "auto", wfmt: str = "oihw",
               **kw) -> ConvPlan:
    """Lower one conv and upload its weights (lowering.rs:99-187 + the
    weight upload of Model::load, crates/ai-gpu-runtime/src/model.rs:62-69)."""
    return ConvPlan(op, n, ih, iw, has_res=has_res, layout=layout, math=math, **kw).load_weights(w, bias, wfmt)


def resize_bilinear(x: torch.Tensor, oh: int, ow: int, mode: str = "half_pixel", add: Optional[torch.Tensor] = None,
                    act: str = "none", out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Bilinear resize of [n, ih, iw, c] (crates/ai-core/src/reference/resize.rs:5-42),
    optionally fused with an add of a tensor of the output's shape."""
    lib = _lib.load()
    n, ih, iw, c = x.shape
    if out is None:
        out = torch.empty((n, oh, ow, c), dtype=torch.float32, device=x.device)
    check(lib.aie_resize_bilinear(n, ih, iw, c, _dptr(x), oh, ow, 0 if mode == "half_pixel" else 1, _dptr(add),
                                  ACT_ID[act], _dptr(out), C.c_void_p(_stream_handle(stream))),
          "aie_resize_bilinear")
    return out


def device_status(stream=None) -> int:
    """Read and clear the device error word (aie_device_status)."""
    code = C.c_uint32(0)
    lib = _lib.load()
    st = lib.aie_device_status(C.c_void_p(_stream_handle(stream)), C.byref(code))
    if st not in (0, -6):
        check(st, "aie_device_status")
    return code.value
