"""The benchmark workload: a MobileNetV4-small-style segmentation network
at 160x288, built from the conv path's ops.

Neither of ai_engine's shipped segmentation nets has the widths the
benchmark names (32/64/96/128/960, 1-channel sigmoid), so the network is
defined here synthetically with random-init weights (there is no
checkpoint): a stride-2 stem, three implicit-GEMM downsamplers, universal
inverted bottlenecks (depthwise 3x3/5x5 plus pointwise expand/project) and
an FPN-style decoder of 1x1 laterals merged with bilinear x2 upsamples,
one 3x3 smoothing conv and a depthwise + 1x1 sigmoid head, resized to the
input resolution.  It costs 534.8 MFLOP of conv per frame.

Weights follow the benchmark's init: Kaiming-normal N(0, 2/fan_in) and
bias U(-0.1, 0.1), from a fixed seed.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np

from .conv import Conv2d

H, W = 160, 288


def _pw(cin, cout, act="relu"):
    return Conv2d.pointwise(cin, cout, act)


def _cv(cin, cout, k, s, act="relu"):
    return Conv2d.same(cin, cout, k, s, act)


def _dw(c, k, s=1, act="relu"):
    return Conv2d.depthwise(c, k, s, act)


def build_graph() -> List[tuple]:
    g: List[tuple] = []

    def conv(out, src, op, res=None):
        g.append(("conv", out, src, op, res))
        return out

    s0 = conv("stem", "input", _cv(3, 32, 3, 2))               # 80x144x32
    t = conv("e1.conv", s0, _cv(32, 32, 3, 2))                 # 40x72x32
    f4 = conv("e1.pw", t, _pw(32, 32))
    t = conv("e2.conv", f4, _cv(32, 96, 3, 2))                 # 20x36x96
    f8 = conv("e2.pw", t, _pw(96, 64, "none"))                 # 20x36x64
    t = conv("e3.dw5", f8, _dw(64, 5))
    t = conv("e3.exp", t, _pw(64, 192))
    t = conv("e3.dw5s2", t, _dw(192, 5, 2))                    # 10x18x192
    t = conv("e3.proj", t, _pw(192, 96, "none"))
    for i in range(2):
        blk = t
        t = conv(f"e4.{i}.exp", blk, _pw(96, 192))
        t = conv(f"e4.{i}.dw3", t, _dw(192, 3))
        t = conv(f"e4.{i}.proj", t, _pw(192, 96, "none"), res=blk)
    t = conv("e5.exp", t, _pw(96, 384))
    t = conv("e5.dw3", t, _dw(384, 3))
    t = conv("e5.proj", t, _pw(384, 128, "none"))
    for i in range(2):
        blk = t
        t = conv(f"e5.{i}.exp", blk, _pw(128, 512))
        t = conv(f"e5.{i}.dw3", t, _dw(512, 3))
        t = conv(f"e5.{i}.proj", t, _pw(512, 128, "none"), res=blk)
    f16 = conv("head960", t, _pw(128, 960))                    # 10x18x960
    # FPN decoder: lateral 1x1 convs whose epilogue adds the upsampled
    # coarser level (residual added after the activation)
    p16 = conv("fpn.lat16", f16, _pw(960, 64, "none"))
    g.append(("resize", "fpn.up16", p16, (20, 36), None))
    p8 = conv("fpn.lat8", f8, _pw(64, 64, "none"), res="fpn.up16")
    g.append(("resize", "fpn.up8", p8, (40, 72), None))
    p4 = conv("fpn.lat4", f4, _pw(32, 64, "none"), res="fpn.up8")
    q4 = conv("fpn.smooth4", p4, _cv(64, 32, 3, 1))
    g.append(("resize", "fpn.up4", q4, (80, 144), None))
    p2 = conv("fpn.lat2", s0, _pw(32, 32, "none"), res="fpn.up4")
    t = conv("head.dw3", p2, _dw(32, 3))
    t = conv("head.pw", t, _pw(32, 1, "sigmoid"))
    g.append(("resize", "mask", t, (H, W), None))
    return g


def init_weights(graph, seed: int = 4) -> Dict[str, Tuple[np.ndarray, np.ndarray]]:
    """Kaiming-normal weights N(0, 2/fan_in) (OIHW) and U(-0.1, 0.1) bias per conv."""
    rng = np.random.default_rng(seed)
    out = {}
    for op in graph:
        if op[0] != "conv":
            continue
        cv: Conv2d = op[3]
        fan_in = (cv.cin // cv.groups) * cv.kh * cv.kw
        w = rng.standard_normal(cv.cout * (cv.cin // cv.groups) * cv.kh * cv.kw) * np.sqrt(2.0 / fan_in)
        b = rng.uniform(-0.1, 0.1, cv.cout)
        out[op[1]] = (w.astype(np.float32), b.astype(np.float32))
    return out


def synthetic_input(n: int, seed: int = 0) -> np.ndarray:
    """Frames [n, 160, 288, 3] with values U(0, 1)."""
    return np.random.default_rng(seed).random((n, H, W, 3), dtype=np.float32)


def conv_flops_per_frame(graph=None) -> int:
    graph = graph or build_graph()
    from .graph import infer_shapes
    shapes = infer_shapes(graph, (H, W, 3))
    total = 0
    for op in graph:
        if op[0] == "conv":
            cv = op[3]
            oh, ow, _ = shapes[op[1]]
            total += 2 * oh * ow * cv.cout * (cv.cin // cv.groups) * cv.kh * cv.kw
    return total
