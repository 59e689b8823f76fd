"""Pin the CPU oracle to the reference's own known answers.

Each test restates a known-answer or kernel-vs-reference test from
ai_engine; the file:line of the original is in the docstring.  These run
without a GPU.
"""
from types import SimpleNamespace

import numpy as np
import pytest

import oracle
from oracle import XorShift32


def conv(cin, cout, kh, kw, sh=1, sw=1, pad=(0, 0, 0, 0), dil=1, groups=1, act="none"):
    return SimpleNamespace(cin=cin, cout=cout, kh=kh, kw=kw, sh=sh, sw=sw, pad=tuple(pad), dil=dil,
                           groups=groups, act=act)


def pointwise(cin, cout, act="none"):
    return conv(cin, cout, 1, 1, act=act)


def depthwise(c, k, s, act="none"):
    p = (k - 1) // 2
    return conv(c, c, k, k, s, s, (p, p, p, p), 1, c, act)


# ------------------------------------------------------------------ rng ---

def _py_xorshift(seed, n):
    x = seed if seed else 0x9E3779B9
    out = []
    for _ in range(n):
        x ^= (x << 13) & 0xFFFFFFFF
        x ^= x >> 17
        x ^= (x << 5) & 0xFFFFFFFF
        out.append(np.float32(np.float32(x >> 8) / np.float32(1 << 24) * np.float32(2.0) - np.float32(1.0)))
    return np.array(out, np.float32)


def test_rng_deterministic_and_in_range():
    """crates/ai-core/src/rng.rs:40-51"""
    a = XorShift32(42).vec_f32(1000)
    b = XorShift32(42).vec_f32(1000)
    assert np.array_equal(a, b)
    assert (a >= -1).all() and (a < 1).all()


@pytest.mark.parametrize("seed", [0, 1, 42, 2001, 0xFFFFFFFF])
def test_rng_matches_python_restatement(seed):
    """rng.rs:13-24 restated a second time in pure Python: bit-identical."""
    assert np.array_equal(XorShift32(seed).vec_f32(257), _py_xorshift(seed, 257))


# ----------------------------------------------------------- activation ---

def test_hard_activations_match_mnv3_convention():
    """crates/ai-core/src/activation.rs:62-77"""
    assert oracle.act_apply("hardsigmoid", 3.0) == 1.0
    assert oracle.act_apply("hardsigmoid", -3.0) == 0.0
    assert oracle.act_apply("hardsigmoid", 0.0) == 0.5
    assert oracle.act_apply("hardswish", 3.0) == 3.0
    assert oracle.act_apply("hardswish", -3.0) == 0.0
    assert abs(oracle.act_apply("hardswish", 1.0) - 2.0 / 3.0) < 1e-6


def test_apply4_lane_vs_scalar():
    """apply4 (crates/ai-cpu/src/kernels/mod.rs:21-50) agrees with the scalar
    form within one rounding for every activation."""
    xs = XorShift32(5).vec_f32(200) * 8
    for act in oracle.ACTS:
        for x in xs:
            if act in ("recip",) and abs(x) < 1e-3:
                continue
            a, b = oracle.act_apply(act, x), oracle.act_apply4_lane(act, x)
            assert abs(a - b) <= 2e-7 * max(1.0, abs(a)), (act, x, a, b)


# ------------------------------------------------- reference conv2d KATs ---

def test_hand_computed_box_sum():
    """crates/ai-core/src/reference/conv.rs:71-90"""
    x = np.arange(1, 10, dtype=np.float32)
    out = oracle.conv2d_ref(conv(1, 1, 3, 3, pad=(1, 1, 1, 1)), 3, 3, x, np.ones(9, np.float32))
    assert (out[4], out[0], out[8]) == (45.0, 12.0, 28.0)


def test_pointwise_identity():
    """reference/conv.rs:93-102"""
    x = (np.arange(12, dtype=np.float32) * 0.5)
    w = np.eye(3, dtype=np.float32).reshape(-1)
    assert np.array_equal(oracle.conv2d_ref(pointwise(3, 3), 2, 2, x, w), x)


def test_hand_computed_pointwise_bias_act():
    """reference/conv.rs:105-113"""
    out = oracle.conv2d_ref(pointwise(2, 1, "relu"), 1, 2, np.array([1, -1, 0.5, 2], np.float32),
                            np.array([2, 3], np.float32), np.array([1], np.float32))
    assert out.tolist() == [0.0, 8.0]


def test_hand_computed_depthwise():
    """reference/conv.rs:116-129"""
    x = np.array([1, 10, 2, 20, 3, 30, 4, 40], np.float32)
    w = np.concatenate([np.ones(9), np.full(9, 2.0)]).astype(np.float32)
    out = oracle.conv2d_ref(depthwise(2, 3, 1), 2, 2, x, w)
    assert out[0] == 10.0 and out[1] == 200.0


def test_residual_applied_after_activation():
    """reference/conv.rs:132-139"""
    out = oracle.conv2d_ref(pointwise(1, 1, "relu"), 1, 1, np.array([-1], np.float32),
                            np.array([1], np.float32), None, np.array([5], np.float32))
    assert out.tolist() == [5.0]


def test_stride2_asymmetric_pad():
    """reference/conv.rs:142-165"""
    op = conv(1, 1, 2, 2, 2, 2, (1, 0, 0, 1))
    assert oracle.out_hw(op, 4, 4) == (2, 2)
    out = oracle.conv2d_ref(op, 4, 4, np.arange(1, 17, dtype=np.float32), np.ones(4, np.float32))
    assert out[0] == 3.0 and out[3] == 38.0


# ------------------------------------------------------ resize KATs ---

def test_resize_half_pixel_1d():
    """crates/ai-core/src/reference/resize.rs:50-55"""
    out = oracle.resize_bilinear(np.array([0, 1], np.float32).reshape(1, 1, 2, 1), 1, 4, "half_pixel")
    assert out.reshape(-1).tolist() == [0.0, 0.25, 0.75, 1.0]


def test_resize_asymmetric_1d():
    """reference/resize.rs:58-63"""
    out = oracle.resize_bilinear(np.array([0, 1], np.float32).reshape(1, 1, 2, 1), 1, 4, "asymmetric")
    assert out.reshape(-1).tolist() == [0.0, 0.5, 1.0, 1.0]


def test_resize_identity_and_constant():
    """reference/resize.rs:66-73"""
    x = np.full((1, 5, 7, 2), 3.0, np.float32)
    assert np.array_equal(oracle.resize_bilinear(x, 5, 7), x)
    assert np.all(np.abs(oracle.resize_bilinear(x, 10, 14) - 3.0) < 1e-6)


# ----------------------------------------- ai-cpu kernels vs reference ---

def _close(want, got):
    """ai-cpu test tolerance: |a-b| <= 1e-4 * max(|a|, 1) (conv.rs:503-508)."""
    want, got = np.asarray(want).reshape(-1), np.asarray(got).reshape(-1)
    assert want.shape == got.shape
    bad = np.abs(want - got) > 1e-4 * np.maximum(np.abs(want), 1.0)
    assert not bad.any(), f"{bad.sum()} mismatches, first at {np.argmax(bad)}"


def _run_case(op, ih, iw, with_res, seed, threads=1):
    """crates/ai-cpu/src/kernels/conv.rs:476-509 (same rng draw order)."""
    rng = XorShift32(seed)
    x = rng.vec_f32(ih * iw * op.cin)
    w = rng.vec_f32(op.cout * (op.cin // op.groups) * op.kh * op.kw)
    b = rng.vec_f32(op.cout)
    oh, ow = oracle.out_hw(op, ih, iw)
    res = rng.vec_f32(oh * ow * op.cout) if with_res else None
    want = oracle.conv2d_ref(op, ih, iw, x, w, b, res)
    p = oracle.Plan(op, ih, iw, w, b, True, with_res)
    got = np.empty(oh * ow * op.cout, np.float32)
    p.run_frame(x, got, res, threads=threads)
    _close(want, got)
    return p.kind, want, got


def test_pointwise_matches_reference():
    """conv.rs:511-517; cout 5 (< NR) and cin 3, then residual"""
    _run_case(pointwise(3, 5, "relu"), 6, 7, False, 1)
    _run_case(pointwise(8, 16, "hardswish"), 5, 9, True, 2)


def test_k3_stride_pad_matches_reference():
    """conv.rs:520-537"""
    op = conv(6, 10, 3, 3, pad=(1, 1, 1, 1))
    kind, _, _ = _run_case(op, 8, 8, False, 3)
    assert kind == oracle.K_STD
    _run_case(conv(6, 10, 3, 3, 2, 2, (1, 1, 1, 1), act="relu"), 9, 11, True, 4)


def test_asymmetric_pad_and_dilation():
    """conv.rs:540-570"""
    _run_case(conv(4, 8, 2, 2, 2, 2, (1, 0, 0, 1)), 6, 6, False, 5)
    _run_case(conv(3, 5, 3, 3, 1, 1, (2, 2, 2, 2), 2, act="sigmoid"), 7, 7, False, 6)


def test_row_split_equals_full():
    """conv.rs:641-667: banded threading is bit-identical to one thread"""
    op = conv(5, 9, 3, 3, 2, 2, (1, 1, 1, 1), act="relu")
    rng = XorShift32(8)
    x = rng.vec_f32(11 * 13 * 5)
    w = rng.vec_f32(9 * 5 * 9)
    b = rng.vec_f32(9)
    p = oracle.Plan(op, 11, 13, w, b)
    full = np.empty(p.oh * p.ow * 9, np.float32)
    split = np.empty_like(full)
    p.run_frame(x, full, threads=1)
    p.run_frame(x, split, threads=2)
    assert np.array_equal(full, split)


@pytest.mark.parametrize("c,k,s,pad,act,ih,iw,seed", [
    (8, 3, 1, 1, "relu", 7, 9, 1), (7, 3, 2, 1, "hardswish", 8, 8, 2), (3, 5, 1, 2, "none", 9, 6, 3)])
def test_dw_matches_reference(c, k, s, pad, act, ih, iw, seed):
    """crates/ai-cpu/src/kernels/dw.rs:280-309 (with residual)"""
    op = conv(c, c, k, k, s, s, (pad,) * 4, 1, c, act)
    kind, _, _ = _run_case(op, ih, iw, True, seed)
    assert kind == oracle.K_DW


def test_dw_strided_view_input():
    """dw.rs:313-347: a channel slice of a wider tensor"""
    ih, iw, big_c, c, c_off = 6, 5, 10, 6, 3
    rng = XorShift32(4)
    big = rng.vec_f32(ih * iw * big_c)
    w = rng.vec_f32(c * 9)
    b = rng.vec_f32(c)
    xm = big.reshape(-1, big_c)[:, c_off:c_off + c].copy()
    op = depthwise(c, 3, 1, "relu")
    want = oracle.conv2d_ref(op, ih, iw, xm, w, b)
    p = oracle.Plan(op, ih, iw, w, b, dense_input=False)
    got = np.empty(ih * iw * c, np.float32)
    p.run_frame(big, got, x_stride=big_c, x_coff=c_off)
    _close(want, got)


@pytest.mark.parametrize("cin,cout,act", [(24, 2, "none"), (7, 3, "relu"), (16, 4, "sigmoid")])
def test_pw_dot_matches_reference(cin, cout, act):
    """crates/ai-cpu/src/kernels/pw_dot.rs:69-98"""
    op = pointwise(cin, cout, act)
    rng = XorShift32(cin + cout)
    x = rng.vec_f32(5 * 6 * cin)
    w = rng.vec_f32(cout * cin)
    b = rng.vec_f32(cout)
    want = oracle.conv2d_ref(op, 5, 6, x, w, b)
    p = oracle.Plan(op, 5, 6, w, b)
    assert p.kind == oracle.K_PWDOT
    got = np.empty_like(want)
    p.run_frame(x, got)
    _close(want, got)


def test_stem_via_im2row_matches_reference():
    """crates/ai-cpu/src/kernels/im2row.rs:111-154"""
    op = conv(3, 8, 3, 3, 2, 2, (1, 1, 1, 1), act="relu")
    kind, _, _ = _run_case(op, 10, 12, False, 9)
    assert kind == oracle.K_STEM


def test_aicpu_order_equals_reference_order():
    """Both accumulate bias, then (ky, kx, ic) in order with unfused
    multiply-add, so for full 4-lane channel blocks and activations whose
    4-lane form is exact they agree bit for bit."""
    for op, ih, iw, seed in [(conv(8, 16, 3, 3, 1, 1, (1, 1, 1, 1), act="relu"), 9, 10, 11),
                             (depthwise(16, 5, 2, "none"), 11, 9, 12),
                             (pointwise(32, 8), 4, 5, 13)]:
        _, want, got = _run_case(op, ih, iw, False, seed)
        assert np.array_equal(want, got)


def test_dot_scale_bounds_error():
    op = conv(6, 10, 3, 3, 2, 2, (1, 1, 1, 1))
    rng = XorShift32(21)
    x = rng.vec_f32(9 * 11 * 6).reshape(1, 9, 11, 6)
    w = rng.vec_f32(10 * 6 * 9)
    b = rng.vec_f32(10)
    s = oracle.dot_scale(op, x, w, b)
    y = oracle.conv_aicpu(op, x, w, b)
    assert s.shape == y.shape and (s + 1e-6 >= np.abs(y)).all()


# ---- graph glue: the reference's own known answers -----------------------

def test_binary_known_answers():
    """crates/ai-core/src/reference/elementwise.rs:32-43."""
    a = np.array([1.0, -2.0, 3.0], np.float32).reshape(1, 1, 3, 1)
    b = np.array([0.5, 1.0, -1.0], np.float32).reshape(1, 1, 3, 1)
    o = np.empty_like(a)
    oracle.binary("add", a, b, o)
    assert o.ravel().tolist() == [1.5, -1.0, 2.0]
    oracle.binary("mul", a, b, o, act="relu")
    assert o.ravel().tolist() == [0.5, 0.0, 0.0]
    oracle.binary("sub", a, 1.0, o, kind="scalar_first")
    assert o.ravel().tolist() == [0.0, 3.0, -2.0]


def test_cvec_and_mix_known_answers():
    """crates/ai-cpu/src/kernels/elementwise.rs:258-275 (cvec mul, GRU mix)."""
    a = np.array([1, 4, 3, 8], np.float32).reshape(1, 1, 2, 2)
    o = np.empty_like(a)
    oracle.binary("mul", a, np.array([2.0, 0.5], np.float32), o, kind="cvec")
    assert o.ravel().tolist() == [2.0, 2.0, 6.0, 4.0]
    z = np.array([0, 1, 0.5, 0.5], np.float32).reshape(1, 1, 2, 2)
    av = np.array([1, 1, 2, 4], np.float32).reshape(1, 1, 2, 2)
    bv = np.array([3, 3, 4, 8], np.float32).reshape(1, 1, 2, 2)
    oracle.mix(z, av, bv, o)
    assert o.ravel().tolist() == [1.0, 3.0, 3.0, 6.0]


def test_strided_view_binary_matches_dense():
    """crates/ai-cpu/src/kernels/elementwise.rs:278-300: a channel-slice view
    gives the same result as the materialised slice."""
    rng = oracle.XorShift32(2)
    px, big_c, c, off = 6, 7, 3, 2
    big = rng.vec_f32(px * big_c).reshape(1, 1, px, big_c)
    b = rng.vec_f32(px * c).reshape(1, 1, px, c)
    dense = np.ascontiguousarray(big[..., off:off + c])
    want = np.empty_like(b)
    oracle.binary("add", dense, b, want, act="sigmoid")
    got = np.empty_like(b)
    oracle.binary("add", (big, off, c), b, got, act="sigmoid")
    assert np.array_equal(want, got)
    ref = 1.0 / (1.0 + np.exp(-(dense.astype(np.float64) + b)))
    assert np.allclose(got, ref, rtol=1e-6)


def test_pool_known_answers():
    """crates/ai-core/src/reference/pool.rs:84-101 (gpool, 2x2 average pool)."""
    x = np.array([1.0, 4.0, 2.0, 8.0, 3.0, 12.0, 4.0, 16.0], np.float32).reshape(1, 2, 2, 2)
    assert oracle.gpool(x).ravel().tolist() == [2.5, 10.0]
    ramp = np.arange(1, 17, dtype=np.float32).reshape(1, 4, 4, 1)
    assert oracle.avgpool(ramp, (2, 2), (2, 2)).ravel().tolist() == [3.5, 5.5, 11.5, 13.5]


def test_se_gate_known_answers():
    """crates/ai-cpu/src/kernels/segate.rs:84-121: gpool then FC1 (ReLU), and
    gpool -> FC1 (identity) -> FC2, with the FCs as 1x1 convs over a 1x1 frame."""
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32).reshape(1, 1, 2, 2)
    mean = oracle.gpool(x).reshape(1, 1, 1, 2)
    assert mean.ravel().tolist() == [2.0, 3.0]
    fc1 = conv(2, 2, 1, 1, act="relu")
    got = oracle.conv_aicpu(fc1, mean, np.array([1, 1, 1, -2], np.float32), np.zeros(2, np.float32))
    assert got.ravel().tolist() == [5.0, 0.0]
    ident = oracle.conv_aicpu(conv(2, 2, 1, 1), mean, np.array([1, 0, 0, 1], np.float32), np.zeros(2, np.float32))
    got = oracle.conv_aicpu(conv(2, 2, 1, 1), ident, np.array([2, 0, 0, 2], np.float32), np.ones(2, np.float32))
    assert got.ravel().tolist() == [5.0, 7.0]


# ---- YUV 4:2:0 frames (crates/ai-ffi/src/yuv.rs) ---------------------------

def test_yuv_roundtrip_flat_colors():
    """yuv.rs:106-124 (roundtrip_flat_colors): flat 4 x 2 frames of red,
    green, blue and grey survive RGBA -> I420 -> RGBA within 3 per channel."""
    w, h = 4, 2
    for color in ([255, 0, 0], [0, 255, 0], [0, 0, 255], [128, 128, 128]):
        rgba = np.empty((h, w, 4), np.uint8)
        rgba[..., :3] = color
        rgba[..., 3] = 255
        y, u, v = oracle.rgba_to_i420(rgba)
        back = oracle.i420_to_rgba(y, u, v, w, h)
        d = np.abs(back[..., :3].astype(int) - np.array(color))
        assert d.max() <= 3, (color, d.max())
        assert (back[..., 3] == 255).all()


def test_yuv_known_values():
    """Hand-computed BT.601 full-range values of yuv.rs:24-27: neutral
    chroma gives grey; U = V = 255 saturates R and B, G = floor of the sum."""
    y = np.array([[0, 128], [255, 77]], np.uint8)
    u = np.array([[128]], np.uint8)
    v = np.array([[128]], np.uint8)
    out = oracle.i420_to_rgba(y, u, v, 2, 2)
    assert out[..., 0].tolist() == [[0, 128], [255, 77]] and (out[..., 1] == out[..., 0]).all()
    out = oracle.i420_to_rgba(np.array([[200, 100]], np.uint8), np.array([[255]], np.uint8),
                              np.array([[255]], np.uint8), 2, 1)
    g = np.float32(200) - np.float32(0.344136) * np.float32(127) - np.float32(0.714136) * np.float32(127)
    assert out[0, 0].tolist() == [255, int(g), 255, 255] and int(g) == 65
    assert out[0, 1].tolist() == [255, 0, 255, 255]  # G below zero clamps to 0
