"""GPU parity of the conv kernels against the CPU oracle, through the C ABI.

The shape grids, seeds and draw order restate ai_engine's GPU-vs-CPU
accuracy suite (crates/ai-gpu/src/testsuite.rs:373-411 pointwise,
:466-495 depthwise, :722-785 implicit GEMM).  Tolerances
(normalised error of tests/_util.py):
  fp32_strict  bit-exact with the ai-cpu restatement (non-transcendental acts)
  ffma         <= 1e-5
  tf32         <= 5e-3
"""
import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200 import Conv2d, View, pack
from ai_engine_b200.conv import ConvPlan
from tests._util import EXACT_ACTS, TOL_FFMA, TOL_TF32, case_tensors, normalised_error, oracle_conv

pytestmark = pytest.mark.gpu

MATHS = ["fp32_strict", "ffma"]


def run_gpu(op, x, w, b, res=None, *, layout="nhwc", math="ffma", wfmt="oihw", **kw):
    n, ih, iw, cin = x.shape
    plan = ConvPlan(op, n, ih, iw, has_res=res is not None, layout=layout, math=math, **kw)
    if wfmt == "sw":
        if op.groups > 1:
            wp = pack.pack_weights_dw(w, op.cout, op.kh, op.kw)
        else:
            wp, _ = pack.pack_weights_conv(w, op.cout, op.cin, op.kh, op.kw, 4)
        plan.load_weights(wp, pack.pack_bias(b, op.cout), fmt="sw")
    else:
        plan.load_weights(w, b)
    if layout == "nhwc_c4":
        xd = torch.from_numpy(pack.pack_nhwc(x)).cuda()
        rd = None if res is None else torch.from_numpy(pack.pack_nhwc(res)).cuda()
    else:
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        rd = None if res is None else torch.from_numpy(np.ascontiguousarray(res)).cuda()
    out = plan(xd, rd)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    if layout == "nhwc_c4":
        # bit-exact layout: padding lanes are zero, i.e. out == pack_nhwc(logical)
        assert got.shape[-1] == pack.cg(op.cout) * 4
        assert not got[..., op.cout:].any(), "C4 padding lanes must be zero"
        got = got[..., :op.cout]
    return plan, got


def check(op, x, w, b, res, math, **kw):
    want, scale = oracle_conv(op, x, w, b, res)
    plan, got = run_gpu(op, x, w, b, res, math=math, **kw)
    assert got.shape == want.shape
    assert plan.math == math or (math == "auto")
    if math == "fp32_strict" and op.act in EXACT_ACTS:
        diff = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
        assert diff.size == 0, f"{diff.size} outputs differ from ai-cpu, first {diff[:5]}"
    else:
        tol = TOL_TF32 if plan.math == "tf32" else TOL_FFMA
        err = normalised_error(got, want, scale)
        assert err <= tol, f"normalised error {err:.3g} > {tol} ({plan.kernel}/{plan.math})"
    return plan, got


# ---------------------------------------------------------------- pointwise ---

PW_SHAPES = [(1, 1, 64, 16), (9, 16, 128, 24), (3, 5, 6, 10), (72, 128, 16, 64), (24, 32, 6, 10),
             (23, 33, 8, 20), (9, 16, 960, 160), (9, 16, 240, 68), (11, 13, 72, 68)]
PW_ACTS = ["none", "relu", "hardswish", "sigmoid"]


def pw_cases():
    seed = 2000
    for (h, w, cin, cout) in PW_SHAPES:
        for act in PW_ACTS:
            seed += 1
            yield pytest.param(h, w, cin, cout, act, seed, id=f"{h}x{w}-{cin}-{cout}-{act}")


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("h,w,cin,cout,act,seed", list(pw_cases()))
def test_pointwise_grid(cuda_ok, math, h, w, cin, cout, act, seed):
    """testsuite.rs:373-391 (pw_case grid)"""
    op = Conv2d.pointwise(cin, cout, act)
    x, wt, b, _ = case_tensors(op, 1, h, w, seed, False)
    check(op, x, wt, b, None, math)


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("h,w,cin,cout,act,seed", [(9, 16, 32, 32, "relu", 3001), (9, 16, 960, 160, "relu", 3003),
                                                   (72, 128, 16, 16, "hardswish", 3002)])
def test_pointwise_residual(cuda_ok, math, h, w, cin, cout, act, seed):
    """testsuite.rs:393-398: residual added after the activation"""
    op = Conv2d.pointwise(cin, cout, act)
    x, wt, b, res = case_tensors(op, 1, h, w, seed, True)
    check(op, x, wt, b, res, math)


# ---------------------------------------------------------------- depthwise ---

DW_SHAPES = [(72, 128, 64, 3, 1), (36, 64, 96, 5, 2), (33, 17, 6, 3, 2), (16, 16, 10, 5, 1),
             # beyond the reference grid: the register-blocked variants (C % 4 == 0)
             (20, 37, 64, 5, 1), (41, 72, 32, 3, 2), (10, 18, 512, 3, 1), (9, 7, 8, 5, 2),
             # the shared-memory halo-tile variants (frames >= 40 x 64): ragged
             # tiles, partial 32-channel slices, both strides and kernel sizes
             (100, 150, 32, 3, 2), (44, 70, 36, 5, 1), (96, 130, 8, 5, 2), (41, 67, 48, 3, 1)]


def dw_cases():
    seed = 4000
    for (ih, iw, c, k, s) in DW_SHAPES:
        for act in ["none", "relu", "hardswish"]:
            seed += 1
            yield pytest.param(ih, iw, c, k, s, act, seed, id=f"{ih}x{iw}-c{c}-k{k}s{s}-{act}")


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("ih,iw,c,k,s,act,seed", list(dw_cases()))
def test_depthwise_grid(cuda_ok, math, ih, iw, c, k, s, act, seed):
    """testsuite.rs:469-484 (dw_case grid)"""
    op = Conv2d.depthwise(c, k, s, act)
    x, wt, b, _ = case_tensors(op, 1, ih, iw, seed, False)
    check(op, x, wt, b, None, math)


@pytest.mark.parametrize("math", MATHS)
def test_depthwise_residual_and_dilation(cuda_ok, math):
    """testsuite.rs:485-488 (residual 5001, dilated dw 5201, dilated igemm 5202)"""
    op = Conv2d.depthwise(32, 3, 1, "relu")
    x, wt, b, res = case_tensors(op, 1, 36, 64, 5001, True)
    check(op, x, wt, b, res, math)
    op = Conv2d(40, 40, 3, 3, 1, 1, (2, 2, 2, 2), 2, 40, "relu")
    x, wt, b, _ = case_tensors(op, 1, 18, 32, 5201, False)
    check(op, x, wt, b, None, math)
    op = Conv2d(8, 12, 3, 3, 1, 1, (2, 2, 2, 2), 2, 1, "hardswish")
    x, wt, b, _ = case_tensors(op, 1, 24, 32, 5202, False)
    check(op, x, wt, b, None, math)


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("ih,iw,c,k,act,seed", [(9, 16, 672, 5, "hardswish", 5211), (9, 16, 960, 5, "hardswish", 5212),
                                               (18, 32, 40, 3, "relu", 5213), (11, 13, 24, 5, "none", 5214),
                                               (7, 6, 8, 3, "relu", 5215)])
def test_depthwise_dilated_blocked(cuda_ok, math, ih, iw, c, k, act, seed):
    """Dilation-2 depthwise on the register-blocked kernel (C % 4 == 0,
    stride 1): RVM's dilated last stage (k5 d2 pad 4 at 9x16, 672 / 960
    channels) and ragged frames smaller than the dilated window."""
    p = 2 * (k - 1) // 2
    op = Conv2d(c, c, k, k, 1, 1, (p, p, p, p), 2, c, act)
    x, wt, b, res = case_tensors(op, 2, ih, iw, seed, seed % 2 == 0)
    check(op, x, wt, b, res, math)


# ------------------------------------------------------------ implicit GEMM ---

IG_SHAPES = [(36, 64, 3, 16, 3, 2), (24, 32, 16, 24, 3, 1), (40, 64, 20, 32, 3, 1), (17, 23, 6, 8, 3, 2),
             (33, 45, 8, 12, 5, 2), (9, 16, 128, 128, 3, 1), (18, 32, 171, 80, 3, 1)]


def ig_cases():
    seed = 6000
    for (ih, iw, cin, cout, k, s) in IG_SHAPES:
        for act in ["none", "relu", "hardswish"]:
            seed += 1
            yield pytest.param(ih, iw, cin, cout, k, s, act, seed, id=f"{ih}x{iw}-{cin}-{cout}-k{k}s{s}-{act}")


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("ih,iw,cin,cout,k,s,act,seed", list(ig_cases()))
def test_igemm_grid(cuda_ok, math, ih, iw, cin, cout, k, s, act, seed):
    """testsuite.rs:725-743 (igemm_case grid)"""
    op = Conv2d.same(cin, cout, k, s, act)
    x, wt, b, _ = case_tensors(op, 1, ih, iw, seed, False)
    check(op, x, wt, b, None, math)


IG_SPECIAL = [  # testsuite.rs:745-773: asymmetric SAME pads, real stem size, residuals
    (16, 16, 4, 8, 3, 1, (1, 0, 0, 1), "relu", False, 7001),
    (128, 128, 3, 16, 3, 2, (0, 0, 1, 1), "none", False, 7008),
    (32, 32, 3, 16, 3, 2, (0, 0, 1, 1), "none", False, 7005),
    (32, 32, 3, 24, 5, 2, (1, 1, 2, 2), "none", False, 7006),
    (24, 24, 16, 16, 3, 2, (0, 0, 1, 1), "relu", False, 7007),
    (24, 32, 16, 16, 3, 1, (1, 1, 1, 1), "hardswish", True, 7002),
    (9, 16, 8, 8, 3, 1, (1, 1, 1, 1), "none", True, 7003),
    (9, 16, 128, 128, 3, 1, (1, 1, 1, 1), "relu", True, 7004),
]


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("ih,iw,cin,cout,k,s,pad,act,res,seed", IG_SPECIAL, ids=[str(c[-1]) for c in IG_SPECIAL])
def test_igemm_special(cuda_ok, math, ih, iw, cin, cout, k, s, pad, act, res, seed):
    op = Conv2d(cin, cout, k, k, s, s, pad, 1, 1, act)
    x, wt, b, r = case_tensors(op, 1, ih, iw, seed, res)
    check(op, x, wt, b, r, math)


# ------------------------------------------------- layouts, formats, views ---

@pytest.mark.parametrize("kind", ["pw", "dw", "igemm", "pw_dot"])
def test_c4_layout_and_sw_packed_weights(cuda_ok, kind):
    """The reference GPU layout: NHWC-C4 activations and .sw-packed weights
    (crates/ai-core/src/pack.rs:34-184).  Output padding lanes must be zero."""
    op = {"pw": Conv2d.pointwise(6, 10, "relu"), "dw": Conv2d.depthwise(7, 3, 2, "hardswish"),
          "igemm": Conv2d.same(6, 10, 3, 1, "none"), "pw_dot": Conv2d.pointwise(7, 3, "sigmoid")}[kind]
    x, wt, b, res = case_tensors(op, 2, 9, 11, 77, kind != "pw_dot")
    plan, _ = check(op, x, wt, b, res, "ffma", layout="nhwc_c4", wfmt="sw")
    assert plan.kernel == kind


def test_strided_view_input(cuda_ok):
    """dw.rs:313-347 on the GPU: the input is a channel slice of a wider tensor."""
    ih, iw, big_c, c, c_off = 6, 5, 10, 6, 3
    from oracle import XorShift32
    rng = XorShift32(4)
    big = rng.vec_f32(ih * iw * big_c).reshape(1, ih, iw, big_c)
    wt = rng.vec_f32(c * 9)
    b = rng.vec_f32(c)
    op = Conv2d.depthwise(c, 3, 1, "relu")
    xm = np.ascontiguousarray(big[..., c_off:c_off + c])
    want, scale = oracle_conv(op, xm, wt, b, None)
    plan = ConvPlan(op, 1, ih, iw, in_view=View(big_c, c_off), math="fp32_strict").load_weights(wt, b)
    got = plan(torch.from_numpy(big).cuda()).cpu().numpy()
    assert np.array_equal(got, want)


def test_output_view_writes_only_its_channels(cuda_ok):
    """An output view (concat slot) leaves the other channels untouched."""
    op = Conv2d.pointwise(16, 8, "relu")
    x, wt, b, _ = case_tensors(op, 2, 5, 7, 91, False)
    want, _ = oracle_conv(op, x, wt, b, None)
    big = torch.full((2, 5, 7, 20), 7.0, device="cuda")
    plan = ConvPlan(op, 2, 5, 7, out_view=View(20, 4), math="fp32_strict").load_weights(wt, b)
    plan(torch.from_numpy(x).cuda(), out=big)
    got = big.cpu().numpy()
    assert np.array_equal(got[..., 4:12], want)
    assert (got[..., :4] == 7).all() and (got[..., 12:] == 7).all()


@pytest.mark.parametrize("math", MATHS)
def test_batch_matches_per_frame(cuda_ok, math):
    """Frames are independent: a batch of 5 equals 5 single-frame runs."""
    op = Conv2d.same(16, 24, 3, 2, "relu")
    x, wt, b, _ = case_tensors(op, 5, 17, 19, 123, False)
    _, batched = run_gpu(op, x, wt, b, math=math)
    for f in range(5):
        _, single = run_gpu(op, x[f:f + 1], wt, b, math=math)
        assert np.array_equal(single[0], batched[f])


def test_canary_no_write_outside_output(cuda_ok):
    """Layout check: nothing is written past the output tensor."""
    op = Conv2d.same(8, 12, 3, 1, "none")
    x, wt, b, _ = case_tensors(op, 1, 7, 9, 5, False)
    plan = ConvPlan(op, 1, 7, 9).load_weights(wt, b)
    n_out = 7 * 9 * 12
    buf = torch.full((n_out + 4096,), 1234.5, device="cuda")
    plan(torch.from_numpy(x).cuda(), out=buf[:n_out].view(1, 7, 9, 12))
    assert (buf[n_out:] == 1234.5).all()


@pytest.mark.parametrize("c,ih,iw,oh,ow", [
    (6, 5, 9, 10, 18), (4, 5, 9, 10, 18), (3, 7, 5, 14, 10), (1, 5, 9, 20, 36), (1, 5, 9, 13, 23),
    (1, 40, 72, 160, 288), (8, 9, 7, 4, 3),
    # exact 2x (the dedicated source-pixel kernel): C4, one channel, the
    # benchmark's mask and lateral shapes, and 2x shapes it must leave to the
    # general kernel (width not a multiple of 4 with one channel)
    (32, 9, 13, 18, 26), (1, 5, 8, 10, 16), (1, 80, 144, 160, 288), (32, 40, 72, 80, 144), (1, 5, 9, 10, 18),
    # two channels (the shipped model's logits): even widths take the
    # two-pixel kernel, an odd width the general one
    (2, 5, 8, 10, 16), (2, 1, 2, 2, 4), (2, 80, 144, 160, 288), (2, 5, 9, 10, 18)])
def test_resize_bilinear_bit_exact(cuda_ok, c, ih, iw, oh, ow):
    """GPU resize (+ fused add) equals the CPU restatement bit for bit:
    vector channel groups, ragged channel tails, the 4-pixel single-channel
    path with aligned and ragged widths, and downsampling."""
    from ai_engine_b200 import resize_bilinear
    from oracle import XorShift32
    rng = XorShift32(31 + c + ow)
    x = rng.vec_f32(2 * ih * iw * c).reshape(2, ih, iw, c)
    add = rng.vec_f32(2 * oh * ow * c).reshape(2, oh, ow, c)
    for mode in ["half_pixel", "asymmetric"]:
        want = oracle.resize_bilinear(x, oh, ow, mode)
        got = resize_bilinear(torch.from_numpy(x).cuda(), oh, ow, mode).cpu().numpy()
        assert np.array_equal(got, want)
    want = oracle.add(oracle.resize_bilinear(x, oh, ow), add)
    got = resize_bilinear(torch.from_numpy(x).cuda(), oh, ow, add=torch.from_numpy(add).cuda()).cpu().numpy()
    assert np.array_equal(got, want)


HEADS = [  # n, ih, iw, c, k, s, dw act, pw cout, pw act, layout
    (2, 40, 72, 32, 3, 1, "relu", 1, "sigmoid", "nhwc"),      # the benchmark head's shape
    (3, 33, 50, 16, 5, 2, "hardswish", 3, "none", "nhwc"),    # ragged tiles, k5 s2, 3 outputs
    (1, 17, 9, 8, 3, 2, "relu6", 2, "sigmoid", "nhwc_c4"),    # narrow frame, C4 output padding
    (2, 21, 30, 32, 5, 1, "none", 4, "relu", "nhwc"),
]


@pytest.mark.parametrize("n,ih,iw,c,k,s,act,cout,act2,layout", HEADS, ids=[f"{h[1]}x{h[2]}c{h[3]}k{h[4]}s{h[5]}" for h in HEADS])
def test_fused_dw_pw_head(cuda_ok, n, ih, iw, c, k, s, act, cout, act2, layout):
    """Depthwise + 1x1 (cout <= 4) in one launch equals the two convs run in
    turn on the GPU (FFMA tolerance) and the ai-cpu restatement of the chain."""
    from ai_engine_b200.conv import run_dw_pw
    from oracle import XorShift32
    dw_op = Conv2d.depthwise(c, k, s, act)
    pw_op = Conv2d.pointwise(c, cout, act2)
    x, wd, bd, _ = case_tensors(dw_op, n, ih, iw, 8300 + c + k, False)
    dwp = ConvPlan(dw_op, n, ih, iw, math="ffma").load_weights(wd, bd)
    rng = XorShift32(8400 + cout)
    wp = rng.vec_f32(cout * c)
    bp = (rng.vec_f32(cout) * 0.1).astype(np.float32)
    pwp = ConvPlan(pw_op, n, dwp.oh, dwp.ow, math="ffma", layout=layout).load_weights(wp, bp)
    assert dwp.kernel == "dw" and pwp.kernel == "pw_dot"
    xd = torch.from_numpy(x).cuda()
    fused = run_dw_pw(dwp, pwp, xd)
    inter = dwp(xd)
    pw_in = torch.from_numpy(pack.pack_nhwc(inter.cpu().numpy())).cuda() if layout == "nhwc_c4" else inter
    ref = pwp(pw_in)
    torch.cuda.synchronize()
    got, want = fused.cpu().numpy(), ref.cpu().numpy()
    if layout == "nhwc_c4":
        assert not got[..., cout:].any(), "C4 padding lanes must be zero"
        got, want = got[..., :cout], want[..., :cout]
    scale = oracle.dot_scale(pw_op, inter.cpu().numpy(), wp, bp)
    assert normalised_error(got, want, scale) <= TOL_FFMA
    # against the CPU restatement of the two convs, normalised by the
    # chain's magnitude (the pair run on |x|, |w|, |b|): the depthwise's
    # rounding reaches the output through the 1x1 weights
    want_dw, _ = oracle_conv(dw_op, x, wd, bd, None)
    want_pw, _ = oracle_conv(pw_op, want_dw, wp, bp, None)
    chain = oracle.dot_scale(pw_op, oracle.dot_scale(dw_op, x, wd, bd), wp, bp)
    assert normalised_error(got, want_pw, chain) <= TOL_FFMA


@pytest.mark.parametrize("n,h,w,c,k,s,cout", [(2, 80, 144, 32, 3, 1, 1), (3, 18, 26, 16, 3, 1, 2),
                                                (1, 20, 36, 32, 5, 1, 1), (2, 12, 16, 8, 3, 2, 4),
                                                (1, 6, 10, 24, 5, 2, 3)])
def test_fused_head_up2_input(cuda_ok, n, h, w, c, k, s, cout):
    """aie_conv_run_dw_pw_up2: the depthwise input is x + the exact-2x
    half_pixel resize of a half-size tensor, mixed in the staged tile with
    fused multiply-adds.  Equals the fused head run on x + resize(q) formed
    by the resize kernel, and the ai-cpu restatement, within the FFMA bar."""
    from ai_engine_b200 import resize_bilinear
    from ai_engine_b200.conv import run_dw_pw
    from oracle import XorShift32
    dw_op = Conv2d.depthwise(c, k, s, "relu")
    pw_op = Conv2d.pointwise(c, cout, "sigmoid")
    rng = XorShift32(7100 + h + c)
    x = rng.vec_f32(n * h * w * c).reshape(n, h, w, c)
    q = rng.vec_f32(n * (h // 2) * (w // 2) * c).reshape(n, h // 2, w // 2, c)
    wd, bd = rng.vec_f32(c * k * k), rng.vec_f32(c)
    wp, bp = rng.vec_f32(cout * c), rng.vec_f32(cout)
    dwp = ConvPlan(dw_op, n, h, w, math="ffma").load_weights(wd, bd)
    pwp = ConvPlan(pw_op, n, dwp.oh, dwp.ow, math="ffma").load_weights(wp, bp)
    xd, qd = torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda()
    got = run_dw_pw(dwp, pwp, xd, up=qd).cpu().numpy()
    summed = resize_bilinear(qd, h, w, add=xd)
    same = run_dw_pw(dwp, pwp, summed).cpu().numpy()
    p2 = oracle.add(oracle.resize_bilinear(q, h, w), x)
    want_dw, _ = oracle_conv(dw_op, p2, wd, bd, None)
    want, _ = oracle_conv(pw_op, want_dw, wp, bp, None)
    scale = oracle.dot_scale(pw_op, want_dw, wp, bp)
    assert normalised_error(got, same, scale) <= TOL_FFMA
    # the chain's magnitude: resize + add, depthwise and 1x1 run on |.|
    mag_in = oracle.add(oracle.resize_bilinear(np.abs(q), h, w), np.abs(x))
    chain = oracle.dot_scale(pw_op, oracle.dot_scale(dw_op, mag_in, wd, bd), wp, bp)
    assert normalised_error(got, want, chain) <= TOL_FFMA


def test_fused_head_up2_rejects_bad_source(cuda_ok):
    """The up-sampled source must be half the depthwise input and aligned."""
    from ai_engine_b200._lib import AieError
    from ai_engine_b200.conv import run_dw_pw
    dwp = ConvPlan(Conv2d.depthwise(32, 3, 1, "relu"), 1, 8, 12, math="ffma")
    pwp = ConvPlan(Conv2d.pointwise(32, 1, "sigmoid"), 1, 8, 12, math="ffma")
    dwp.load_weights(np.zeros(32 * 9, np.float32), np.zeros(32, np.float32))
    pwp.load_weights(np.zeros(32, np.float32), np.zeros(1, np.float32))
    x = torch.zeros(1, 8, 12, 32, device="cuda")
    with pytest.raises(AieError):
        run_dw_pw(dwp, pwp, x, up=torch.zeros(1, 5, 6, 32, device="cuda"))


@pytest.mark.parametrize("math", ["auto", "ffma"])
def test_model_fpn_tail_fusion_matches(cuda_ok, math):
    """The benchmark network with its FPN tail folded into the head (the
    last lateral conv without its residual, the resize dropped, the head
    adding the up-sampled coarser level) equals the network run op by op
    within the FFMA bar on the mask (sigmoid, in (0, 1)): the fused head
    mixes the up-sampling with fused multiply-adds where the resize kernel
    rounds each product and sum."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    x = torch.from_numpy(segnet.synthetic_input(2, seed=15)).cuda()
    # the stem + lateral fusion is kept out of both so that fpn.lat2 runs on
    # its own in each (its exactness is tested in test_stem_pw_gpu.py)
    a = Model(g, wts, 2, (segnet.H, segnet.W, 3), math=math, fuse_stem=False)
    b = Model(g, wts, 2, (segnet.H, segnet.W, 3), math=math, fuse_tail=False, fuse_stem=False)
    assert any(r.out == "fpn.up4" for r in b.ops) and next(r for r in b.ops if r.kind == "dwpw").up is None
    heads = [r for r in a.ops if r.kind == "dwpw"]
    assert len(heads) == 1 and heads[0].up == "fpn.smooth4"
    assert not any(r.out == "fpn.up4" for r in a.ops)
    lat2 = next(r for r in a.ops if r.out == "fpn.lat2")
    assert lat2.res is None
    assert (a.infer(x) - b.infer(x)).abs().max().item() <= TOL_FFMA


def test_model_head_fusion(cuda_ok):
    """The benchmark network with its dw3 -> 1x1 sigmoid head fused equals
    the same network run op by op (FFMA path)."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    x = torch.from_numpy(segnet.synthetic_input(2, seed=5)).cuda()
    a = Model(g, wts, 2, (segnet.H, segnet.W, 3), math="ffma", fuse_heads=True)
    b = Model(g, wts, 2, (segnet.H, segnet.W, 3), math="ffma", fuse_heads=False)
    assert any(r.kind == "dwpw" for r in a.ops) and not any(r.kind == "dwpw" for r in b.ops)
    d = (a.infer(x) - b.infer(x)).abs().max().item()
    assert d <= 1e-5, d


@pytest.mark.parametrize("cin,layout,n,h,w", [(3, "nhwc", 2, 17, 23), (4, "nhwc", 3, 8, 8), (3, "nhwc_c4", 1, 5, 7),
                                              (4, "nhwc_c4", 2, 160, 288), (3, "nhwc", 4, 160, 288)])
def test_input_u8_staging_bit_exact(cuda_ok, cin, layout, n, h, w):
    """u8 RGB/RGBA frames -> f32 network input equals u8 / 255 in IEEE f32
    (ragged pixel counts, alpha dropped, C4 padding lane zero)."""
    from ai_engine_b200.conv import input_u8
    rng = np.random.default_rng(cin * 100 + h)
    fr = rng.integers(0, 256, (n, h, w, cin), dtype=np.uint8)
    got = input_u8(torch.from_numpy(fr).cuda(), layout=layout).cpu().numpy()
    want = fr[..., :3].astype(np.float32) / np.float32(255.0)
    assert np.array_equal(got[..., :3], want)
    if layout == "nhwc_c4":
        assert got.shape[-1] == 4 and not got[..., 3].any()


def test_model_u8_input_equals_normalised_f32(cuda_ok):
    """A model fed u8 frames (normalised by its first op) equals the same
    model fed the f32 frames u8 / 255, also through the pipelined path."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    rng = np.random.default_rng(9)
    fr = [rng.integers(0, 256, (2, segnet.H, segnet.W, 3), dtype=np.uint8) for _ in range(3)]
    a = Model(g, wts, 2, (segnet.H, segnet.W, 3), input_u8=True)
    b = Model(g, wts, 2, (segnet.H, segnet.W, 3))
    for f in fr:
        ya = a.infer(torch.from_numpy(f).cuda()).clone()
        yb = b.infer(torch.from_numpy(f.astype(np.float32) / np.float32(255.0)).cuda()).clone()
        assert torch.equal(ya, yb)
    hin = [torch.from_numpy(f).pin_memory() for f in fr]
    outs = [torch.empty(ya.shape, dtype=torch.float32).pin_memory() for _ in fr]
    a.run_pipelined(hin, outs)
    torch.cuda.synchronize()
    for f, o in zip(fr, outs):
        yb = b.infer(torch.from_numpy(f.astype(np.float32) / np.float32(255.0)).cuda()).cpu()
        assert torch.equal(o, yb)
    a.release()


def _yuv_oracle(yp, up, vp, h, w):
    """Oracle: ai-ffi's i420_to_rgba per frame, then the model's v / 255."""
    import oracle
    out = np.empty((yp.shape[0], h, w, 3), np.float32)
    for f in range(yp.shape[0]):
        rgba = oracle.i420_to_rgba(np.ascontiguousarray(yp[f]), np.ascontiguousarray(up[f]),
                                   np.ascontiguousarray(vp[f]), w, h)
        out[f] = rgba[..., :3].astype(np.float32) / np.float32(255.0)
    return out


@pytest.mark.parametrize("n,h,w,pad", [(2, 160, 288, 0), (3, 37, 51, 5), (1, 1, 1, 0), (2, 6, 9, 3)])
@pytest.mark.parametrize("fmt", ["i420", "nv12", "nv21"])
@pytest.mark.parametrize("layout", ["nhwc", "nhwc_c4"])
def test_input_yuv420_bit_exact(cuda_ok, n, h, w, pad, fmt, layout):
    """YUV 4:2:0 staging (aie_input_yuv420) equals ai-ffi's i420_to_rgba
    followed by v / 255, bit for bit: I420 planes and NV12 / NV21
    interleaved chroma, odd sizes (the last chroma row / column serves one
    pixel), padded row strides, both output layouts."""
    from ai_engine_b200.conv import input_yuv420
    rng = np.random.default_rng(h * w + pad)
    ch, cw = (h + 1) // 2, (w + 1) // 2
    y = rng.integers(0, 256, (n, h, w + pad), dtype=np.uint8)
    u = rng.integers(0, 256, (n, ch, cw + pad), dtype=np.uint8)
    v = rng.integers(0, 256, (n, ch, cw + pad), dtype=np.uint8)
    want = _yuv_oracle(y, u, v, h, w)
    yd = torch.from_numpy(y).cuda()
    if fmt == "i420":
        got = input_yuv420(yd, torch.from_numpy(u).cuda(), torch.from_numpy(v).cuda(), w=w, layout=layout)
    else:
        first, second = (u, v) if fmt == "nv12" else (v, u)
        uv = np.zeros((n, ch, 2 * cw + pad), np.uint8)
        uv[..., 0:2 * cw:2], uv[..., 1:2 * cw:2] = first[..., :cw], second[..., :cw]
        got = input_yuv420(yd, torch.from_numpy(uv).cuda(), w=w, nv21=fmt == "nv21", layout=layout)
    got = got.cpu().numpy()
    assert np.array_equal(got[..., :3], want)
    if layout == "nhwc_c4":
        assert (got[..., 3] == 0).all()
