"""The recurrent video-matting network of BASELINE config 5, built from the
conv path and its glue ops.

An RVM-style net (Robust Video Matting: MobileNetV3-Large encoder with SE
blocks and hardswish, LR-ASPP, and a ConvGRU recurrent decoder at 1/2, 1/4,
1/8 and 1/16 scale carrying hidden state across frames, with foreground
(3 ch) and alpha (1 ch) outputs).  ai_engine ships this graph only as the
layer list ``web/compare/assets/rvm_144x256.plan.json`` (its weights are
absent); the node list below follows that layer list op for op at any
input size divisible by 16, with two rewrites ai_engine's converter makes
too: the ConvGRU's ``(1 - z) h + z c`` chain is one ``Mix`` node
(``fuse_mix``, SwOp::Mix, crates/ai-core/src/format/model.rs:193-199), and
each residual ``Add`` after a project conv is that conv's residual epilogue
(the conv-tail rule, ``Conv.res``, model.rs:87-89).  The crop ``Slice``
aliases of the plan are identities at sizes divisible by 16 and are left
out.  Weights are random-init (Kaiming-normal N(0, 2/fan_in), bias
U(-0.1, 0.1)); inputs are U(0, 1) frames; 2.25 GFLOP of conv per 144x256
frame.

State: ``r1..r4`` (16 / 20 / 40 / 64 channels at 1/2 .. 1/16) feed step t,
``r1o..r4o`` are step t's new state; they start at zero.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np

from .conv import Conv2d
from .net import Node

H, W = 144, 256
STATES = {"r1": "r1o", "r2": "r2o", "r3": "r3o", "r4": "r4o"}
STATE_CH = {"r1": 16, "r2": 20, "r3": 40, "r4": 64}
OUTPUTS = ["fgr", "pha", "r1o", "r2o", "r3o", "r4o"]
# torchvision's ImageNet normalisation, the plan's __const_0 / __const_1
MEAN = np.array([0.485, 0.456, 0.406], np.float32)
INV_STD = np.float32(1) / np.array([0.229, 0.224, 0.225], np.float32)  # 1 / std, divided in f32

# MobileNetV3-Large inverted residuals (Howard et al. 2019, table 2):
# kernel, expanded width, output width, SE, activation, stride; the last
# three run at stride 1 with dilation 2 (the segmentation form RVM uses).
_BNECK = [
    (3, 16, 16, False, "relu", 1, 1),
    (3, 64, 24, False, "relu", 2, 1),
    (3, 72, 24, False, "relu", 1, 1),
    (5, 72, 40, True, "relu", 2, 1),
    (5, 120, 40, True, "relu", 1, 1),
    (5, 120, 40, True, "relu", 1, 1),
    (3, 240, 80, False, "hardswish", 2, 1),
    (3, 200, 80, False, "hardswish", 1, 1),
    (3, 184, 80, False, "hardswish", 1, 1),
    (3, 184, 80, False, "hardswish", 1, 1),
    (3, 480, 112, True, "hardswish", 1, 1),
    (3, 672, 112, True, "hardswish", 1, 1),
    (5, 672, 160, True, "hardswish", 1, 2),
    (5, 960, 160, True, "hardswish", 1, 2),
    (5, 960, 160, True, "hardswish", 1, 2),
]


def _squeeze(c: int) -> int:
    """SE bottleneck width: c / 4 rounded to a multiple of 8 (never below 90%)."""
    v = max(8, int(c / 4 + 4) // 8 * 8)
    return v + 8 if v < 0.9 * c / 4 else v


def build_graph(h: int = H, w: int = W) -> List[Node]:
    if h % 16 or w % 16:
        raise ValueError("RVM frames need sizes divisible by 16")
    g: List[Node] = []

    def conv(out, src, op: Conv2d, res=None):
        g.append(Node("conv", out, (src,), conv=op, res=res))
        return out

    def binary(out, a, b, op, act="none", bkind="tensor", scalar=0.0):
        g.append(Node("binary", out, (a,) if b is None else (a, b), op=op, act=act, bkind=bkind, scalar=scalar))
        return out

    # input normalisation (plan ops 0-1): (src - mean) * (1 / std)
    t = binary("norm.sub", "src", "mean", "sub", bkind="cvec")
    t = binary("norm", t, "inv_std", "mul", bkind="cvec")
    t = conv("f0", t, Conv2d.same(3, 16, 3, 2, "hardswish"))
    feats = {}
    cin = 16
    for i, (k, exp, cout, se, act, s, d) in enumerate(_BNECK, start=1):
        name = f"f{i}"
        x = t
        if exp != cin:
            t = conv(f"{name}.exp", t, Conv2d.pointwise(cin, exp, act))
        p = d * (k - 1) // 2
        t = conv(f"{name}.dw", t, Conv2d(exp, exp, k, k, s, s, (p, p, p, p), d, exp, act))
        if se:
            sq = _squeeze(exp)
            g.append(Node("gpool", f"{name}.se.pool", (t,)))
            conv(f"{name}.se.fc1", f"{name}.se.pool", Conv2d.pointwise(exp, sq, "relu"))
            conv(f"{name}.se.fc2", f"{name}.se.fc1", Conv2d.pointwise(sq, exp, "hardsigmoid"))
            t = binary(f"{name}.se", t, f"{name}.se.fc2", "mul", bkind="cvec_tensor")
        res = x if (s == 1 and cin == cout) else None
        t = conv(name, t, Conv2d.pointwise(exp, cout, "none"), res=res)
        cin = cout
        feats[i] = t
    f16 = conv("f16", t, Conv2d.pointwise(160, 960, "hardswish"))
    f1, f2, f3 = feats[1], feats[3], feats[6]

    # LR-ASPP (plan ops 90-93)
    a1 = conv("aspp1", f16, Conv2d.pointwise(960, 128, "relu"))
    g.append(Node("gpool", "aspp2.pool", (f16,)))
    conv("aspp2", "aspp2.pool", Conv2d.pointwise(960, 128, "sigmoid"))
    f4 = binary("aspp", a1, "aspp2", "mul", bkind="cvec_tensor")

    # decoder input pyramid: 2x2 average pools of the raw frame (ops 94-96)
    g.append(Node("avgpool", "s1", ("src",), size=(2, 2, 2, 2)))
    g.append(Node("avgpool", "s2", ("s1",), size=(2, 2, 2, 2)))
    g.append(Node("avgpool", "s3", ("s2",), size=(2, 2, 2, 2)))

    def gru(tag, x, r, c):
        """ConvGRU: [r | z] = sigmoid(conv([x, h])); c~ = tanh(conv([x, r h]));
        h' = h + z (c~ - h) = (1 - z) h + z c~."""
        g.append(Node("concat", f"{tag}.xh", (x, r)))
        conv(f"{tag}.ih", f"{tag}.xh", Conv2d.same(2 * c, 2 * c, 3, 1, "sigmoid"))
        g.append(Node("split", (f"{tag}.r", f"{tag}.z"), (f"{tag}.ih",), parts=(c, c)))
        binary(f"{tag}.rh", f"{tag}.r", r, "mul")
        g.append(Node("concat", f"{tag}.xrh", (x, f"{tag}.rh")))
        conv(f"{tag}.hh", f"{tag}.xrh", Conv2d.same(2 * c, c, 3, 1, "tanh"))
        g.append(Node("mix", STATES[r], (f"{tag}.z", r, f"{tag}.hh")))
        return STATES[r]

    # decode4: bottleneck block at 1/16 (ops 97-108)
    g.append(Node("split", ("d4.a", "d4.b"), (f4,), parts=(64, 64)))
    r4o = gru("d4.gru", "d4.b", "r4", 64)
    g.append(Node("concat", "d4", ("d4.a", r4o)))
    x = "d4"
    # decode3..decode1: upsample, concat skip + pooled frame, conv, half-GRU
    for lvl, (skip, s_img, cin_x, cout, rname, hs) in zip(
            (3, 2, 1), ((f3, "s3", 128, 80, "r3", 8), (f2, "s2", 80, 40, "r2", 4), (f1, "s1", 40, 32, "r1", 2))):
        tag = f"d{lvl}"
        g.append(Node("resize", f"{tag}.up", (x,), size=(h // hs, w // hs)))
        g.append(Node("concat", f"{tag}.cat", (f"{tag}.up", skip, s_img)))
        ccat = cin_x + {3: 40, 2: 24, 1: 16}[lvl] + 3
        conv(f"{tag}.conv", f"{tag}.cat", Conv2d.same(ccat, cout, 3, 1, "relu"))
        half = cout // 2
        g.append(Node("split", (f"{tag}.a", f"{tag}.b"), (f"{tag}.conv",), parts=(half, half)))
        ro = gru(f"{tag}.gru", f"{tag}.b", rname, half)
        g.append(Node("concat", tag, (f"{tag}.a", ro)))
        x = tag
    # decode0: output block at full resolution (ops 160-165)
    g.append(Node("resize", "d0.up", (x,), size=(h, w)))
    g.append(Node("concat", "d0.cat", ("d0.up", "src")))
    conv("d0.conv1", "d0.cat", Conv2d.same(35, 16, 3, 1, "relu"))
    conv("d0.conv2", "d0.conv1", Conv2d.same(16, 16, 3, 1, "relu"))
    # projection and outputs (ops 166-171): fgr = clamp01(residual + src)
    conv("project", "d0.conv2", Conv2d.pointwise(16, 4, "none"))
    g.append(Node("split", ("project.fgr", "project.pha"), ("project",), parts=(3, 1)))
    binary("fgr", "project.fgr", "src", "add", act="clamp01")
    g.append(Node("chcopy", "pha", ("project",), act="clamp01", parts=(3, 1)))
    return g


def inputs(h: int = H, w: int = W) -> Dict[str, Tuple[int, int, int]]:
    d = {"src": (h, w, 3)}
    for r, c in STATE_CH.items():
        s = {"r1": 2, "r2": 4, "r3": 8, "r4": 16}[r]
        d[r] = (h // s, w // s, c)
    return d


def consts() -> Dict[str, np.ndarray]:
    return {"mean": MEAN, "inv_std": INV_STD}


def init_weights(graph: List[Node], seed: int = 5) -> Dict[str, Tuple[np.ndarray, np.ndarray]]:
    """Kaiming-normal N(0, 2/fan_in) (OIHW) and U(-0.1, 0.1) bias per conv."""
    rng = np.random.default_rng(seed)
    out = {}
    for nd in graph:
        if nd.kind != "conv":
            continue
        cv = nd.conv
        fan_in = (cv.cin // cv.groups) * cv.kh * cv.kw
        w = rng.standard_normal(cv.cout * (cv.cin // cv.groups) * cv.kh * cv.kw) * np.sqrt(2.0 / fan_in)
        b = rng.uniform(-0.1, 0.1, cv.cout)
        out[nd.out] = (w.astype(np.float32), b.astype(np.float32))
    return out


def synthetic_frames(streams: int, frames: int, h: int = H, w: int = W, seed: int = 0) -> np.ndarray:
    """[frames, streams, h, w, 3] U(0, 1): frame t of every stream is one step's batch."""
    return np.random.default_rng(seed).random((frames, streams, h, w, 3), dtype=np.float32)


def conv_flops_per_frame(h: int = H, w: int = W) -> int:
    from .net import infer_shapes
    g = build_graph(h, w)
    sh = infer_shapes(g, inputs(h, w))
    total = 0
    for nd in g:
        if nd.kind == "conv":
            cv = nd.conv
            oh, ow, _ = sh[nd.out]
            total += 2 * oh * ow * cv.cout * (cv.cin // cv.groups) * cv.kh * cv.kw
    return total
