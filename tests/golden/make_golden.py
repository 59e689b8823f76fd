"""Generate tests/golden/conv_cases.npz -- golden vectors for the conv path.

The cases are ai_engine's own kernel-vs-reference tests (file:line per case
below), with their seeds and their draw order (input, weights, bias,
residual from XorShift32).  Outputs come from the CPU oracle's ai-cpu
restatement; tests/test_golden.py pins the oracle to these bytes on CPU and
checks the CUDA path against them on the GPU.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from oracle import XorShift32  # noqa: E402

# name: (cin, cout, kh, kw, sh, sw, pad, dil, groups, act, ih, iw, with_res, seed, source)
CASES = {
    "pw_3_5_relu": (3, 5, 1, 1, 1, 1, (0, 0, 0, 0), 1, 1, "relu", 6, 7, False, 1, "crates/ai-cpu/src/kernels/conv.rs:514"),
    "pw_8_16_hswish_res": (8, 16, 1, 1, 1, 1, (0, 0, 0, 0), 1, 1, "hardswish", 5, 9, True, 2, "crates/ai-cpu/src/kernels/conv.rs:516"),
    "k3_6_10": (6, 10, 3, 3, 1, 1, (1, 1, 1, 1), 1, 1, "none", 8, 8, False, 3, "crates/ai-cpu/src/kernels/conv.rs:521-533"),
    "k3s2_6_10_relu_res": (6, 10, 3, 3, 2, 2, (1, 1, 1, 1), 1, 1, "relu", 9, 11, True, 4, "crates/ai-cpu/src/kernels/conv.rs:535-536"),
    "k2s2_asym_4_8": (4, 8, 2, 2, 2, 2, (1, 0, 0, 1), 1, 1, "none", 6, 6, False, 5, "crates/ai-cpu/src/kernels/conv.rs:541-553"),
    "k3d2_3_5_sigmoid": (3, 5, 3, 3, 1, 1, (2, 2, 2, 2), 2, 1, "sigmoid", 7, 7, False, 6, "crates/ai-cpu/src/kernels/conv.rs:555-569"),
    "dw_c8_k3_relu": (8, 8, 3, 3, 1, 1, (1, 1, 1, 1), 1, 8, "relu", 7, 9, True, 1, "crates/ai-cpu/src/kernels/dw.rs:306"),
    "dw_c7_k3s2_hswish": (7, 7, 3, 3, 2, 2, (1, 1, 1, 1), 1, 7, "hardswish", 8, 8, True, 2, "crates/ai-cpu/src/kernels/dw.rs:307"),
    "dw_c3_k5_pad2": (3, 3, 5, 5, 1, 1, (2, 2, 2, 2), 1, 3, "none", 9, 6, True, 3, "crates/ai-cpu/src/kernels/dw.rs:308"),
    "stem_3_8_k3s2_relu": (3, 8, 3, 3, 2, 2, (1, 1, 1, 1), 1, 1, "relu", 10, 12, False, 9, "crates/ai-cpu/src/kernels/im2row.rs:116-133"),
    "pwdot_24_2": (24, 2, 1, 1, 1, 1, (0, 0, 0, 0), 1, 1, "none", 5, 6, False, 26, "crates/ai-cpu/src/kernels/pw_dot.rs:76-79"),
    "pwdot_7_3_relu": (7, 3, 1, 1, 1, 1, (0, 0, 0, 0), 1, 1, "relu", 5, 6, False, 10, "crates/ai-cpu/src/kernels/pw_dot.rs:76-79"),
    "pwdot_16_4_sigmoid": (16, 4, 1, 1, 1, 1, (0, 0, 0, 0), 1, 1, "sigmoid", 5, 6, False, 20, "crates/ai-cpu/src/kernels/pw_dot.rs:76-79"),
}


class Op:
    def __init__(self, t):
        (self.cin, self.cout, self.kh, self.kw, self.sh, self.sw, self.pad, self.dil, self.groups, self.act) = t[:10]


def make():
    out = {}
    for name, t in CASES.items():
        op = Op(t)
        ih, iw, with_res, seed = t[10], t[11], t[12], t[13]
        rng = XorShift32(seed)
        x = rng.vec_f32(ih * iw * op.cin)
        w = rng.vec_f32(op.cout * (op.cin // op.groups) * op.kh * op.kw)
        b = rng.vec_f32(op.cout)
        oh, ow = oracle.out_hw(op, ih, iw)
        res = rng.vec_f32(oh * ow * op.cout) if with_res else None
        plan = oracle.Plan(op, ih, iw, w, b, True, with_res)
        y = np.empty(oh * ow * op.cout, np.float32)
        plan.run_frame(x, y, res)
        out[f"{name}/x"] = x.reshape(1, ih, iw, op.cin)
        out[f"{name}/w"] = w
        out[f"{name}/b"] = b
        if res is not None:
            out[f"{name}/res"] = res.reshape(1, oh, ow, op.cout)
        out[f"{name}/y"] = y.reshape(1, oh, ow, op.cout)
        out[f"{name}/ref"] = oracle.conv2d_ref(op, ih, iw, x, w, b, res).reshape(1, oh, ow, op.cout)
    # resize (reference/resize.rs:79-92 single-part case, seed 1)
    x = XorShift32(1).vec_f32(5 * 7 * 3).reshape(1, 5, 7, 3)
    out["resize/x"] = x
    out["resize/half_pixel"] = oracle.resize_bilinear(x, 10, 14, "half_pixel")
    out["resize/asymmetric"] = oracle.resize_bilinear(x, 10, 14, "asymmetric")
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "conv_cases.npz")
    np.savez_compressed(path, **out)
    return path


if __name__ == "__main__":
    print(make())
