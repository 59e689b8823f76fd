"""CPU oracle for ai_engine's convolution path -- TEST INFRASTRUCTURE ONLY.

This package is the checker that the CUDA library is compared against, and
the timed CPU baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import it.  The product package
``ai_engine_b200`` never imports it and has no CPU fallback.

It wraps ``aie_oracle.c`` (a C restatement of ai_engine's ``ai-core``
reference conv and ``ai-cpu`` kernels; see that file's header for the
file:line map) through ctypes.  Parity is pinned by the reference's own
known-answer tests (crates/ai-core/src/reference/conv.rs:66-162,
activation.rs:62-77, reference/resize.rs:46-73), restated in
``tests/test_oracle.py``.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

from . import build as _build

_LIB = None

# Activation enum order of crates/ai-core/src/activation.rs:7-24
ACTS = ["none", "relu", "sigmoid", "tanh", "hardswish", "hardsigmoid", "clamp01", "relu6",
        "sqrt", "neg", "recip"]
ACT_ID = {n: i for i, n in enumerate(ACTS)}

K_STD, K_DW, K_STEM, K_PWDOT = 1, 2, 3, 4


class OrcConv(C.Structure):
    _fields_ = [("cin", C.c_uint32), ("cout", C.c_uint32), ("kh", C.c_uint32), ("kw", C.c_uint32),
                ("sh", C.c_uint32), ("sw", C.c_uint32), ("pad", C.c_uint32 * 4), ("dil", C.c_uint32),
                ("groups", C.c_uint32), ("act", C.c_int32)]


_fp = C.POINTER(C.c_float)


def lib():
    global _LIB
    if _LIB is None:
        path = _build.build()
        L = C.CDLL(path)
        L.orc_xorshift32_seed.restype = C.c_uint32
        L.orc_xorshift32_seed.argtypes = [C.c_uint32]
        L.orc_fill_uniform.argtypes = [C.POINTER(C.c_uint32), _fp, C.c_size_t]
        L.orc_act_apply.restype = C.c_float
        L.orc_act_apply.argtypes = [C.c_int, C.c_float]
        L.orc_act_apply4_lane.restype = C.c_float
        L.orc_act_apply4_lane.argtypes = [C.c_int, C.c_float]
        L.orc_out_hw.argtypes = [C.POINTER(OrcConv), C.c_uint32, C.c_uint32, C.POINTER(C.c_uint32),
                                 C.POINTER(C.c_uint32)]
        L.orc_conv2d_ref.argtypes = [C.POINTER(OrcConv), C.c_uint32, C.c_uint32, _fp, _fp, _fp, _fp, _fp]
        L.orc_plan_create.restype = C.c_void_p
        L.orc_plan_create.argtypes = [C.POINTER(OrcConv), C.c_uint32, C.c_uint32, _fp, _fp, C.c_int, C.c_int]
        L.orc_plan_free.argtypes = [C.c_void_p]
        L.orc_plan_kind.argtypes = [C.c_void_p]
        L.orc_plan_run.argtypes = [C.c_void_p, _fp, C.c_size_t, C.c_size_t, _fp, C.c_size_t, C.c_size_t,
                                   _fp, C.c_int]
        L.orc_resize_bilinear.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, _fp, C.c_uint32, C.c_uint32,
                                          C.c_int, _fp]
        L.orc_add.argtypes = [_fp, _fp, C.c_size_t, C.c_size_t, C.c_int, _fp]
        sz = C.c_size_t
        L.orc_binary.argtypes = [sz, sz, sz, _fp, sz, sz, C.c_int, C.c_int, _fp, sz, sz, C.c_float, C.c_int,
                                 _fp, sz, sz]
        L.orc_mix.argtypes = [sz, sz, sz] + [_fp, sz, sz] * 4
        L.orc_gpool.argtypes = [sz, sz, sz, _fp, sz, sz, _fp]
        L.orc_avgpool.argtypes = [C.c_uint32] * 11 + [_fp, _fp]
        L.orc_channel_copy.argtypes = [sz, sz, sz, _fp, sz, sz, C.c_int, _fp, sz, sz]
        _u8 = C.POINTER(C.c_uint8)
        L.orc_i420_to_rgba.argtypes = [_u8, _u8, _u8, sz, sz, sz, sz, sz, _u8]
        L.orc_rgba_to_i420.argtypes = [_u8, sz, sz, _u8, _u8, _u8, sz, sz, sz]
        _LIB = L
    return _LIB


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], "oracle wants contiguous float32"
    return a.ctypes.data_as(_fp)


def _act(a) -> int:
    return a if isinstance(a, int) else ACT_ID[a]


def make_conv(op) -> OrcConv:
    """Accept any object with the Conv2d attribute names of
    crates/ai-core/src/ops/conv.rs:6-21."""
    c = OrcConv()
    c.cin, c.cout, c.kh, c.kw, c.sh, c.sw = op.cin, op.cout, op.kh, op.kw, op.sh, op.sw
    for i in range(4):
        c.pad[i] = op.pad[i]
    c.dil, c.groups, c.act = op.dil, op.groups, _act(op.act)
    return c


# ------------------------------------------------------------------ rng ---

class XorShift32:
    """crates/ai-core/src/rng.rs:3-27, via the C restatement."""

    def __init__(self, seed: int):
        self.state = C.c_uint32(lib().orc_xorshift32_seed(seed & 0xFFFFFFFF))

    def vec_f32(self, n: int) -> np.ndarray:
        out = np.empty(int(n), np.float32)
        if n:
            lib().orc_fill_uniform(C.byref(self.state), _ptr(out), int(n))
        return out


# ----------------------------------------------------------- activation ---

def act_apply(act, x: float) -> float:
    return float(lib().orc_act_apply(_act(act), float(x)))


def act_apply4_lane(act, x: float) -> float:
    return float(lib().orc_act_apply4_lane(_act(act), float(x)))


def out_hw(op, ih: int, iw: int):
    oh, ow = C.c_uint32(), C.c_uint32()
    c = make_conv(op)
    if lib().orc_out_hw(C.byref(c), ih, iw, C.byref(oh), C.byref(ow)):
        raise ValueError("invalid conv geometry")
    return oh.value, ow.value


# ----------------------------------------------------------------- conv ---

def conv2d_ref(op, ih: int, iw: int, x: np.ndarray, w: np.ndarray, bias=None, res=None) -> np.ndarray:
    """Naive reference conv (reference/conv.rs:9-62) for one frame.
    x: [ih*iw*cin] NHWC, w: OIHW, returns [oh*ow*cout]."""
    oh, ow = out_hw(op, ih, iw)
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    w = np.ascontiguousarray(w, np.float32).reshape(-1)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    r = None if res is None else np.ascontiguousarray(res, np.float32).reshape(-1)
    out = np.empty(oh * ow * op.cout, np.float32)
    c = make_conv(op)
    if lib().orc_conv2d_ref(C.byref(c), ih, iw, _ptr(x), _ptr(w), _ptr(b), _ptr(r), _ptr(out)):
        raise ValueError("orc_conv2d_ref rejected the geometry")
    return out


class Plan:
    """ai-cpu load-time lowering (plan.rs:462-619) plus its per-frame kernels."""

    def __init__(self, op, ih: int, iw: int, w: np.ndarray, bias=None, dense_input=True, has_res=False):
        self.op, self.ih, self.iw = op, ih, iw
        self.oh, self.ow = out_hw(op, ih, iw)
        self._c = make_conv(op)
        w = np.ascontiguousarray(w, np.float32).reshape(-1)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self._h = lib().orc_plan_create(C.byref(self._c), ih, iw, _ptr(w), _ptr(b), int(dense_input),
                                        int(has_res))
        if not self._h:
            raise ValueError("oracle plan rejected the conv")
        self.kind = lib().orc_plan_kind(self._h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _LIB is not None:
            _LIB.orc_plan_free(h)
            self._h = None

    def run_frame(self, x: np.ndarray, out: np.ndarray, res=None, x_stride=0, x_coff=0, res_stride=0,
                  res_coff=0, threads: int = 1):
        rc = lib().orc_plan_run(self._h, _ptr(x), x_stride, x_coff, _ptr(res), res_stride, res_coff,
                                _ptr(out), int(threads))
        if rc:
            raise MemoryError("orc_plan_run failed")
        return out

    def run(self, x: np.ndarray, res=None, threads: int = 1) -> np.ndarray:
        """x: [N, ih, iw, cin] dense; returns [N, oh, ow, cout]."""
        x = np.ascontiguousarray(x, np.float32)
        n = x.shape[0]
        out = np.empty((n, self.oh, self.ow, self.op.cout), np.float32)
        if res is not None:
            res = np.ascontiguousarray(res, np.float32)
        for f in range(n):
            self.run_frame(x[f], out[f], None if res is None else res[f], threads=threads)
        return out


def conv_aicpu(op, x: np.ndarray, w: np.ndarray, bias=None, res=None, threads: int = 1) -> np.ndarray:
    """Batched convenience wrapper: x [N,H,W,C] -> [N,oh,ow,cout] via ai-cpu order."""
    x = np.ascontiguousarray(x, np.float32)
    p = Plan(op, x.shape[1], x.shape[2], w, bias, True, res is not None)
    return p.run(x, res, threads)


def resize_bilinear(x: np.ndarray, oh: int, ow: int, mode: str = "half_pixel") -> np.ndarray:
    """reference/resize.rs:5-42 over [N,H,W,C]."""
    x = np.ascontiguousarray(x, np.float32)
    n, ih, iw, c = x.shape
    out = np.empty((n, oh, ow, c), np.float32)
    m = 0 if mode == "half_pixel" else 1
    for f in range(n):
        lib().orc_resize_bilinear(ih, iw, c, _ptr(x[f]), oh, ow, m, _ptr(out[f]))
    return out


def add(a: np.ndarray, b: np.ndarray, act="none") -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    out = np.empty_like(a)
    lib().orc_add(_ptr(a), _ptr(b), a.size, a.shape[-1], _act(act), _ptr(out))
    return out


def dot_scale(op, x: np.ndarray, w: np.ndarray, bias=None) -> np.ndarray:
    """Per-output condition scale |b| + sum_k |x_k * w_k| in float64, used to
    normalise errors of reordered sums (the oracle conv of |x|, |w|, |b|)."""
    x = np.abs(np.asarray(x, np.float64))
    w = np.abs(np.asarray(w, np.float64))
    n, ih, iw, cin = x.shape
    oh, ow = out_hw(op, ih, iw)
    kh, kw, sh, sw, d = op.kh, op.kw, op.sh, op.sw, op.dil
    pt, pl = op.pad[0], op.pad[1]
    g = op.groups
    cout = op.cout
    out = np.zeros((n, oh, ow, cout), np.float64)
    if bias is not None:
        out += np.abs(np.asarray(bias, np.float64))
    wv = w.reshape(cout, cin // g, kh, kw)
    for ky in range(kh):
        for kx in range(kw):
            iy = np.arange(oh) * sh + ky * d - pt
            ix = np.arange(ow) * sw + kx * d - pl
            ys = np.nonzero((iy >= 0) & (iy < ih))[0]
            xs = np.nonzero((ix >= 0) & (ix < iw))[0]
            if ys.size == 0 or xs.size == 0:
                continue
            patch = x[:, iy[ys]][:, :, ix[xs]]  # [n, oh', ow', cin]
            if g == 1:
                contrib = patch @ wv[:, :, ky, kx].T
            else:
                contrib = patch * wv[:, 0, ky, kx]
            out[:, ys[:, None], xs[None, :], :] += contrib
    return out


# ----------------------------------------------------------- graph glue ---
# Views: (array, coff, c) selects channels [coff, coff + c) of a dense
# [..., C] float32 array; a bare array is the whole channel range.

def _view(v):
    if isinstance(v, tuple):
        arr, coff, c = v
    else:
        arr, coff, c = v, 0, v.shape[-1]
    if arr.dtype != np.float32 or not arr.flags.c_contiguous:
        raise TypeError("oracle views need contiguous float32 arrays")
    return arr, arr.shape[-1], coff, c


def _npx(arr):
    return arr.shape[0], arr.size // (arr.shape[0] * arr.shape[-1])


BIN_OPS = {"add": 0, "sub": 1, "mul": 2, "prelu": 3}
OPND_KINDS = {"tensor": 0, "scalar": 1, "scalar_first": 2, "cvec": 3, "cvec_tensor": 4, "pvec_tensor": 5}


def binary(op: str, a, b, out, act="none", kind: str = "tensor") -> None:
    """SwOp::Binary into `out` (a view), ai-cpu rounding (elementwise.rs)."""
    aa, as_, ao, c = _view(a)
    oa, os_, oo, _ = _view(out)
    n, px = _npx(aa)
    bs = bo = 0
    scalar = 0.0
    if kind == "tensor":
        ba, bs, bo, _ = _view(b)
    elif kind in ("scalar", "scalar_first"):
        ba, scalar = None, float(b)
    else:
        ba = np.ascontiguousarray(b, np.float32)
    lib().orc_binary(n, px, c, _ptr(aa), as_, ao, BIN_OPS[op], OPND_KINDS[kind], _ptr(ba), bs, bo,
                     C.c_float(scalar), _act(act), _ptr(oa), os_, oo)


def mix(z, a, b, out) -> None:
    """SwOp::Mix out = a + z (b - a) in ai-cpu's order (elementwise.rs:128-150)."""
    za, zs, zo, c = _view(z)
    aa, as_, ao, _ = _view(a)
    ba, bs, bo, _ = _view(b)
    oa, os_, oo, _ = _view(out)
    n, px = _npx(za)
    lib().orc_mix(n, px, c, _ptr(za), zs, zo, _ptr(aa), as_, ao, _ptr(ba), bs, bo, _ptr(oa), os_, oo)


def gpool(x) -> np.ndarray:
    """SwOp::Gpool: [n, ..., C] view -> [n, c] channel means (segate.rs:46-57)."""
    xa, xs, xo, c = _view(x)
    n, px = _npx(xa)
    out = np.empty((n, c), np.float32)
    lib().orc_gpool(n, px, c, _ptr(xa), xs, xo, _ptr(out))
    return out


def avgpool(x: np.ndarray, k, s, pad=(0, 0, 0, 0)) -> np.ndarray:
    """SwOp::Avgpool over [n, h, w, c] (reference/pool.rs:22-46)."""
    x = np.ascontiguousarray(x, np.float32)
    n, ih, iw, c = x.shape
    oh = (ih + pad[0] + pad[2] - k[0]) // s[0] + 1
    ow = (iw + pad[1] + pad[3] - k[1]) // s[1] + 1
    out = np.empty((n, oh, ow, c), np.float32)
    for f in range(n):
        lib().orc_avgpool(ih, iw, c, k[0], k[1], s[0], s[1], pad[0], pad[1], oh, ow, _ptr(x[f]), _ptr(out[f]))
    return out


def channel_copy(x, out, act="none") -> None:
    """Concat part / Chcopy / Act: out view = act(x view)."""
    xa, xs, xo, c = _view(x)
    oa, os_, oo, _ = _view(out)
    n, px = _npx(xa)
    lib().orc_channel_copy(n, px, c, _ptr(xa), xs, xo, _act(act), _ptr(oa), os_, oo)


# ----------------------------------------------------------- frame formats ---

def _u8p(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags["C_CONTIGUOUS"], "oracle wants contiguous uint8"
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def i420_to_rgba(y: np.ndarray, u: np.ndarray, v: np.ndarray, w: int, h: int) -> np.ndarray:
    """One I420 frame (planes [h][stride_y], [ceil(h/2)][stride_u], ...) ->
    RGBA8 [h, w, 4] (crates/ai-ffi/src/yuv.rs:7-31)."""
    out = np.empty((h, w, 4), np.uint8)
    lib().orc_i420_to_rgba(_u8p(y), _u8p(u), _u8p(v), w, h, y.shape[-1], u.shape[-1], v.shape[-1], _u8p(out))
    return out


def rgba_to_i420(rgba: np.ndarray):
    """RGBA8 [h, w, 4] -> I420 planes, tightly packed (yuv.rs:33-58)."""
    h, w, _ = rgba.shape
    y = np.zeros((h, w), np.uint8)
    u = np.zeros(((h + 1) // 2, (w + 1) // 2), np.uint8)
    v = np.zeros_like(u)
    lib().orc_rgba_to_i420(_u8p(np.ascontiguousarray(rgba)), w, h, _u8p(y), _u8p(u), _u8p(v), w, u.shape[1],
                           v.shape[1])
    return y, u, v
