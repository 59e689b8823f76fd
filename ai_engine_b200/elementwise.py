"""Host mirror of ai_engine's non-conv graph ops over the C ABI.

The ops a recurrent matting graph (RVM) and the segmentation heads place
between their convs: ``SwOp::Binary`` / ``Mix`` / ``Gpool`` / ``Avgpool`` /
``Concat`` / ``Chcopy`` / ``Act`` (crates/ai-core/src/format/model.rs:
111-214), each one launch of ``libaie_conv.so`` on the current (or given)
CUDA stream.  Results round like ai-cpu's kernels
(crates/ai-cpu/src/kernels/elementwise.rs, segate.rs; crates/ai-core/src/
reference/pool.rs).

Tensors are dense NHWC float32 CUDA tensors ``[n, h, w, C]``; a
``ChView`` selects ``c`` channels starting at ``coff`` of one (ai-cpu's
``View``, crates/ai-cpu/src/view.rs:8-16), so split outputs and concat parts
need no copies of their own.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence, Union

import torch

from . import _lib
from ._lib import check
from .conv import ACT_ID, _stream_handle


@dataclass
class ChView:
    """Channels [coff, coff + c) of a dense NHWC tensor."""
    t: torch.Tensor
    coff: int = 0
    c: Optional[int] = None

    def __post_init__(self):
        if not self.t.is_cuda or self.t.dtype != torch.float32 or not self.t.is_contiguous():
            raise TypeError("views need a contiguous float32 CUDA tensor")
        if self.c is None:
            self.c = self.t.shape[-1] - self.coff
        if self.coff < 0 or self.c <= 0 or self.coff + self.c > self.t.shape[-1]:
            raise ValueError(f"channels [{self.coff}, {self.coff + self.c}) outside a {self.t.shape[-1]}-channel tensor")

    @property
    def frames(self) -> int:
        return self.t.shape[0]

    @property
    def px(self) -> int:
        return self.t.numel() // (self.t.shape[0] * self.t.shape[-1])

    def tview(self) -> _lib.TView:
        return _lib.TView(self.t.data_ptr(), self.t.shape[-1], self.coff)


ViewLike = Union[ChView, torch.Tensor]


def _v(x: ViewLike) -> ChView:
    return x if isinstance(x, ChView) else ChView(x)


def _same(*vs: ChView):
    n, px, c = vs[0].frames, vs[0].px, vs[0].c
    for v in vs[1:]:
        if (v.frames, v.px, v.c) != (n, px, c):
            raise ValueError(f"view shapes differ: {(n, px, c)} vs {(v.frames, v.px, v.c)}")
    return n, px, c


def _stream(stream):
    return C.c_void_p(_stream_handle(stream))


def binary(op: str, a: ViewLike, b, out: ViewLike, act: str = "none", *, kind: str = "tensor",
           scalar_first: bool = False, stream=None) -> None:
    """out = act(a o b) (SwOp::Binary).  kind: "tensor" (b a view of a's
    shape), "scalar" (b a float; scalar_first gives b o a), "cvec" (b a [c]
    CUDA tensor for every frame), "cvec_tensor" (b [n, c] or [n, 1, 1, c]:
    one channel vector per frame, an SE gate), "pvec_tensor" (b [n * px]:
    one scalar per pixel)."""
    a, out = _v(a), _v(out)
    n, px, c = _same(a, out)
    bt = _lib.TView(None, 0, 0)
    s = 0.0
    if kind == "tensor":
        bv = _v(b)
        _same(a, bv)
        bt, k = bv.tview(), _lib.OPND_TENSOR
    elif kind == "scalar":
        s, k = float(b), (_lib.OPND_SCALAR_FIRST if scalar_first else _lib.OPND_SCALAR)
    else:
        k = {"cvec": _lib.OPND_CVEC, "cvec_tensor": _lib.OPND_CVEC_TENSOR, "pvec_tensor": _lib.OPND_PVEC_TENSOR}[kind]
        want = {"cvec": c, "cvec_tensor": n * c, "pvec_tensor": n * px}[kind]
        if not b.is_cuda or b.dtype != torch.float32 or not b.is_contiguous() or b.numel() != want:
            raise ValueError(f"{kind} operand must be a contiguous float32 CUDA tensor of {want} values")
        bt = _lib.TView(b.data_ptr(), 0, 0)
    check(_lib.load().aie_binary(n, px, c, a.tview(), _lib.BIN_OPS[op], k, bt, C.c_float(s), ACT_ID[act],
                                 out.tview(), _stream(stream)), "aie_binary")


def mix(z: ViewLike, a: ViewLike, b: ViewLike, out: ViewLike, stream=None) -> None:
    """out = a + z (b - a), the ConvGRU state update (SwOp::Mix)."""
    z, a, b, out = _v(z), _v(a), _v(b), _v(out)
    n, px, c = _same(z, a, b, out)
    check(_lib.load().aie_mix(n, px, c, z.tview(), a.tview(), b.tview(), out.tview(), _stream(stream)), "aie_mix")


def gpool(x: ViewLike, out: torch.Tensor, stream=None) -> None:
    """out[f, c] = mean over frame f's pixels (SwOp::Gpool); out holds n * c floats."""
    x = _v(x)
    if out.numel() != x.frames * x.c or not out.is_contiguous():
        raise ValueError("gpool output must be a contiguous [n, c] tensor")
    check(_lib.load().aie_gpool(x.frames, x.px, x.c, x.tview(), C.c_void_p(out.data_ptr()), _stream(stream)),
          "aie_gpool")


def avgpool(x: torch.Tensor, out: torch.Tensor, k: Sequence[int], s: Sequence[int],
            pad: Sequence[int] = (0, 0, 0, 0), stream=None) -> None:
    """Average pool with the fixed kh*kw divisor (SwOp::Avgpool)."""
    n, ih, iw, c = x.shape
    pads = (C.c_uint32 * 4)(*pad)
    check(_lib.load().aie_avgpool(n, ih, iw, c, k[0], k[1], s[0], s[1], pads, C.c_void_p(x.data_ptr()),
                                  C.c_void_p(out.data_ptr()), _stream(stream)), "aie_avgpool")


def channel_copy(x: ViewLike, out: ViewLike, act: str = "none", stream=None) -> None:
    """out = act(x) between channel views (SwOp::Concat part / Chcopy / Act)."""
    x, out = _v(x), _v(out)
    n, px, c = _same(x, out)
    check(_lib.load().aie_channel_copy(n, px, c, x.tview(), ACT_ID[act], out.tview(), _stream(stream)),
          "aie_channel_copy")


def concat(parts: Sequence[ViewLike], out: ViewLike, stream=None) -> None:
    """Channel concat of `parts` into `out` in one pass (SwOp::Concat); `out`
    may be wider than the parts' total, its trailing lanes are zeroed."""
    ps = [_v(p) for p in parts]
    out = _v(out)
    for p in ps:
        if (p.frames, p.px) != (out.frames, out.px):
            raise ValueError("concat parts differ in frames or pixels from the output")
    arr = (_lib.TView * len(ps))(*[p.tview() for p in ps])
    cs = (C.c_uint32 * len(ps))(*[p.c for p in ps])
    check(_lib.load().aie_concat(out.frames, out.px, len(ps), arr, cs, out.c, out.tview(), _stream(stream)),
          "aie_concat")
