"""GPU parity of the tcgen05 TF32 path (tolerance 5e-3 normalised, the
north-star's TF32 bound) and the BASELINE configs 1-3 on every path.

Small sizes are checked against the CPU oracle; full BASELINE sizes that
the oracle cannot finish in seconds are checked through properties: the
TF32 result agrees with the FFMA result (itself pinned to the oracle), and
split-K factors agree with each other."""
import numpy as np
import pytest
import torch

from ai_engine_b200 import Conv2d
from ai_engine_b200._lib import AieError
from ai_engine_b200.conv import ConvPlan
from tests._util import TOL_FFMA, TOL_TF32, case_tensors, normalised_error, oracle_conv
from tests.test_conv_gpu import IG_SHAPES, IG_SPECIAL, PW_SHAPES, check, run_gpu

pytestmark = pytest.mark.gpu


def stem_tc_shape(op, res=False):
    """The tensor-core stem's domain: 3x3, cin <= 3, cout = 32, stride 1 or 2,
    dilation 1, no residual."""
    return (op.groups == 1 and op.cin <= 3 and op.cout == 32 and op.kh == 3 and op.kw == 3 and op.dil == 1
            and op.sh == op.sw and op.sh in (1, 2) and not res)


def tf32_eligible(op, res=False):
    return (op.groups == 1 and op.cin % 4 == 0 and op.sh <= 2 and op.sw <= 2) or stem_tc_shape(op, res)


def check_tf32(op, x, w, b, res=None, **kw):
    if not tf32_eligible(op, res is not None):
        with pytest.raises(AieError) as e:
            run_gpu(op, x, w, b, res, math="tf32", **kw)
        assert e.value.status == -3
        return None
    plan, got = check(op, x, w, b, res, "tf32", **kw)
    assert plan.math == "tf32"
    return plan


@pytest.mark.parametrize("h,w,cin,cout", PW_SHAPES)
@pytest.mark.parametrize("act", ["none", "relu", "hardswish", "sigmoid"])
def test_tf32_pointwise_grid(cuda_ok, h, w, cin, cout, act):
    op = Conv2d.pointwise(cin, cout, act)
    x, wt, b, _ = case_tensors(op, 1, h, w, 2001 + h + cin, False)
    check_tf32(op, x, wt, b)


@pytest.mark.parametrize("ih,iw,cin,cout,k,s", IG_SHAPES)
@pytest.mark.parametrize("act", ["none", "relu", "hardswish"])
def test_tf32_igemm_grid(cuda_ok, ih, iw, cin, cout, k, s, act):
    op = Conv2d.same(cin, cout, k, s, act)
    x, wt, b, _ = case_tensors(op, 1, ih, iw, 6001 + ih + cin, False)
    check_tf32(op, x, wt, b)


@pytest.mark.parametrize("ih,iw,cin,cout,k,s,pad,act,res,seed", IG_SPECIAL, ids=[str(c[-1]) for c in IG_SPECIAL])
def test_tf32_igemm_special(cuda_ok, ih, iw, cin, cout, k, s, pad, act, res, seed):
    op = Conv2d(cin, cout, k, k, s, s, pad, 1, 1, act)
    x, wt, b, r = case_tensors(op, 1, ih, iw, seed, res)
    check_tf32(op, x, wt, b, r)


def test_tf32_dilation_batch_and_c4(cuda_ok):
    op = Conv2d(8, 12, 3, 3, 1, 1, (2, 2, 2, 2), 2, 1, "hardswish")
    x, wt, b, _ = case_tensors(op, 3, 24, 32, 5202, False)
    check_tf32(op, x, wt, b)
    op = Conv2d.same(16, 40, 3, 2, "relu")
    x, wt, b, r = case_tensors(op, 3, 21, 37, 5203, True)
    check_tf32(op, x, wt, b, r, layout="nhwc_c4", wfmt="sw")


# ------------------------------------------------------------- BASELINE cfg ---

def kaiming(rng, cout, fan_in, n):
    return (rng.standard_normal(n) * np.sqrt(2.0 / fan_in)).astype(np.float32)


@pytest.mark.parametrize("math", ["fp32_strict", "ffma", "tf32"])
def test_config1_pointwise_full_size(cuda_ok, math):
    """[1,80,144,32] -> [1,80,144,64], Kaiming W, U(-0.1,0.1) bias, ReLU."""
    rng = np.random.default_rng(1)
    op = Conv2d.pointwise(32, 64, "relu")
    x = rng.uniform(-1, 1, (1, 80, 144, 32)).astype(np.float32)
    w = kaiming(rng, 64, 32, 64 * 32)
    b = rng.uniform(-0.1, 0.1, 64).astype(np.float32)
    plan, got = check(op, x, w, b, None, math)
    assert got.shape == (1, 80, 144, 64)


CFG2 = [(16, 16), (32, 64), (64, 128), (128, 256)]


@pytest.mark.parametrize("cin,cout", CFG2)
@pytest.mark.parametrize("s", [1, 2])
def test_config2_igemm_sweep_b1(cuda_ok, cin, cout, s):
    """BASELINE config 2 at batch 1: 3x3 p1 at 160x288, bias + HardSwish,
    TF32 and FFMA against the oracle."""
    rng = np.random.default_rng(200 + cin + s)
    op = Conv2d.same(cin, cout, 3, s, "hardswish")
    x = rng.uniform(-1, 1, (1, 160, 288, cin)).astype(np.float32)
    w = kaiming(rng, cout, 9 * cin, cout * cin * 9)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    import os
    import oracle
    want = oracle.Plan(op, 160, 288, w, b)
    oh, ow = op.out_hw(160, 288)
    ref = np.empty((oh, ow, cout), np.float32)
    want.run_frame(x[0], ref, threads=os.cpu_count() or 1)
    scale = oracle.dot_scale(op, x, w, b)[0]
    for math, tol in (("tf32", TOL_TF32), ("ffma", TOL_FFMA)):
        _, got = run_gpu(op, x, w, b, math=math)
        assert normalised_error(got[0], ref, scale) <= tol, math


@pytest.mark.parametrize("cin,cout", CFG2)
@pytest.mark.parametrize("s", [1, 2])
def test_config2_igemm_sweep_b16(cuda_ok, cin, cout, s):
    """Config 2 at batch 16: TF32 agrees with FFMA (property check at full size)."""
    rng = np.random.default_rng(300 + cin + s)
    op = Conv2d.same(cin, cout, 3, s, "hardswish")
    x = rng.uniform(-1, 1, (16, 160, 288, cin)).astype(np.float32)
    w = kaiming(rng, cout, 9 * cin, cout * cin * 9)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    outs = {}
    for math in ("ffma", "tf32"):
        p = ConvPlan(op, 16, 160, 288, math=math).load_weights(w, b)
        outs[math] = p(xd)
    ref = outs["ffma"].double()
    # scale: |b| + sum |x w| <= |b| + 9*cin*max|w| bound is loose; use the
    # FFMA conv of |x|, |w| instead
    pa = ConvPlan(Conv2d.same(cin, cout, 3, s, "none"), 16, 160, 288, math="ffma").load_weights(np.abs(w), np.abs(b))
    scale = pa(xd.abs()).double()
    err = ((outs["tf32"].double() - ref).abs() / torch.maximum(ref.abs(), scale)).max().item()
    assert err <= TOL_TF32


CFG3 = [(960, 1280), (1280, 960), (512, 2048)]


@pytest.mark.parametrize("k,n", CFG3)
@pytest.mark.parametrize("split", [0, 1, 4, 8, 16])
def test_config3_splitk_b1(cuda_ok, k, n, split):
    """BASELINE config 3 at batch 1 (M=180): every split factor, and the
    automatic choice (split 0: narrower N tiles and a K split), against the
    oracle."""
    rng = np.random.default_rng(k + n + split)
    op = Conv2d.pointwise(k, n, "none")
    x = rng.uniform(-1, 1, (1, 10, 18, k)).astype(np.float32)
    w = (rng.standard_normal(n * k) / np.sqrt(k)).astype(np.float32)
    b = np.zeros(n, np.float32)
    want, scale = oracle_conv(op, x, w, b, None)
    plan, got = run_gpu(op, x, w, b, math="tf32", split_k=split)
    assert plan.info.split_k >= 1 and (split == 0 or plan.info.split_k <= split)
    if split != 1:
        assert plan.info.split_k > 1 and plan.info.workspace_bytes > 0
    assert normalised_error(got, want, scale) <= TOL_TF32


@pytest.mark.parametrize("k,n", CFG3)
@pytest.mark.parametrize("batch", [64, 256])
def test_config3_splitk_large_batch(cuda_ok, k, n, batch):
    """Config 3 at batch 64/256: split 1 vs 4 vs 16 agree, and TF32 agrees with FFMA."""
    rng = np.random.default_rng(k * n + batch)
    op = Conv2d.pointwise(k, n, "none")
    x = torch.from_numpy(rng.uniform(-1, 1, (batch, 10, 18, k)).astype(np.float32)).cuda()
    w = (rng.standard_normal(n * k) / np.sqrt(k)).astype(np.float32)
    b = np.zeros(n, np.float32)
    ref = ConvPlan(op, batch, 10, 18, math="ffma").load_weights(w, b)(x).double()
    scale = ConvPlan(op, batch, 10, 18, math="ffma").load_weights(np.abs(w), b)(x.abs()).double()
    for split in (1, 4, 16):
        got = ConvPlan(op, batch, 10, 18, math="tf32", split_k=split).load_weights(w, b)(x).double()
        err = ((got - ref).abs() / torch.maximum(ref.abs(), scale)).max().item()
        assert err <= TOL_TF32, (split, err)


def test_splitk_is_deterministic_and_reusable(cuda_ok):
    """Same inputs, same split: bitwise-identical results on repeated runs
    (fixed-order reduction; tickets reset between launches)."""
    op = Conv2d.pointwise(960, 160, "relu")
    x, wt, b, _ = case_tensors(op, 1, 9, 16, 3003, False)
    plan = ConvPlan(op, 1, 9, 16, math="tf32", split_k=8).load_weights(wt, b)
    xd = torch.from_numpy(x).cuda()
    first = plan(xd).clone()
    for _ in range(3):
        assert torch.equal(plan(xd), first)
    from ai_engine_b200 import device_status
    assert device_status() == 0


@pytest.mark.parametrize("coff", [4, 2])
def test_tf32_output_view(cuda_ok, coff):
    """Output written into a channel slice of a wider buffer: 16-byte aligned
    slices take the TMA-store epilogue, unaligned ones the direct-store one;
    both leave the other channels untouched."""
    from ai_engine_b200 import View
    op = Conv2d.same(16, 24, 3, 1, "relu")
    x, wt, b, res = case_tensors(op, 2, 13, 21, 92, True)
    want, scale = oracle_conv(op, x, wt, b, res)
    big = torch.full((2, 13, 21, 32), 7.0, device="cuda")
    plan = ConvPlan(op, 2, 13, 21, has_res=True, out_view=View(32, coff), math="tf32").load_weights(wt, b)
    plan(torch.from_numpy(x).cuda(), torch.from_numpy(res).cuda(), out=big)
    got = big.cpu().numpy()
    assert normalised_error(got[..., coff:coff + 24], want, scale) <= TOL_TF32
    assert (got[..., :coff] == 7).all() and (got[..., coff + 24:] == 7).all()


@pytest.mark.parametrize("n,h,w,cin,cout", [(3, 10, 18, 64, 96), (2, 7, 9, 32, 200), (1, 40, 72, 128, 48)])
def test_tf32_partial_tiles_residual(cuda_ok, n, h, w, cin, cout):
    """Ragged M (pixels not a multiple of 128), ragged N tiles, residual."""
    op = Conv2d.pointwise(cin, cout, "hardswish")
    x, wt, b, res = case_tensors(op, n, h, w, 93 + cout, True)
    check_tf32(op, x, wt, b, res)
    op3 = Conv2d.same(cin, cout, 3, 2, "relu")
    x, wt, b, res = case_tensors(op3, n, h, w, 94 + cout, True)
    check_tf32(op3, x, wt, b, res)


@pytest.mark.parametrize("math", ["fp32_strict", "ffma", "tf32"])
@pytest.mark.parametrize("kind", ["pw", "igemm"])
@pytest.mark.parametrize("mode", ["half_pixel", "asymmetric"])
@pytest.mark.parametrize("rh,rw", [(9, 13), (7, 10)])
def test_fused_bilinear_residual(cuda_ok, math, kind, mode, rh, rw):
    """Resize -> Conv(res) fused into the conv epilogue equals the unfused
    pair (oracle resize, then oracle conv with that residual): bit for bit
    in fp32_strict mode.  9x13 -> 18x26 is an exact 2x (the integer
    half_pixel path), 7x10 the general one."""
    import oracle
    from oracle import XorShift32
    op = Conv2d.pointwise(32, 40, "relu") if kind == "pw" else Conv2d.same(32, 40, 3, 1, "hardswish")
    n, h, w = 2, 18, 26
    rng = XorShift32(777)
    x = rng.vec_f32(n * h * w * 32).reshape(n, h, w, 32)
    wt = rng.vec_f32(op.cout * op.cin * op.kh * op.kw)
    b = rng.vec_f32(op.cout)
    lo = rng.vec_f32(n * rh * rw * op.cout).reshape(n, rh, rw, op.cout)
    up = oracle.resize_bilinear(lo, h, w, mode)
    want, scale = oracle_conv(op, x, wt, b, up)
    plan = ConvPlan(op, n, h, w, has_res=True, math=math, res_resize=(rh, rw, mode)).load_weights(wt, b)
    got = plan(torch.from_numpy(x).cuda(), torch.from_numpy(lo).cuda()).cpu().numpy()
    if math == "fp32_strict":
        assert np.array_equal(got, want)
    else:
        assert normalised_error(got, want, scale) <= (TOL_TF32 if math == "tf32" else TOL_FFMA)


@pytest.mark.parametrize("math", ["fp32_strict", "tf32"])
@pytest.mark.parametrize("n,h,w,cin,cout,split", [
    (2, 10, 76, 32, 40, 0),     # rows of 76: a warp's 32 pixels wrap rows and frames; ragged last tile; 2 chunks
    (3, 12, 36, 64, 64, 0),     # 36-wide rows (the FPN's 20x36 lateral)
    (1, 20, 144, 32, 32, 0),    # 144-wide rows (the FPN's 80x144 lateral)
    (2, 8, 64, 256, 48, 4),     # split-K: the patch is fetched while the partials are summed
])
def test_fused_up2_residual_patch(cuda_ok, math, n, h, w, cin, cout, split):
    """Exact-2x half_pixel residual on 1x1 tensor-core tiles with ow >= 32:
    the epilogue reads each warp's source patch from shared memory.  Equals
    the unfused pair bit for bit in fp32_strict mode (which runs the FFMA
    kernels) and within the TF32 bar on the tensor-core path."""
    import oracle
    from oracle import XorShift32
    op = Conv2d.pointwise(cin, cout, "none")
    rng = XorShift32(900 + w + cout)
    x = rng.vec_f32(n * h * w * cin).reshape(n, h, w, cin)
    wt = rng.vec_f32(op.cout * op.cin)
    b = rng.vec_f32(op.cout)
    lo = rng.vec_f32(n * (h // 2) * (w // 2) * cout).reshape(n, h // 2, w // 2, cout)
    up = oracle.resize_bilinear(lo, h, w, "half_pixel")
    want, scale = oracle_conv(op, x, wt, b, up)
    plan = ConvPlan(op, n, h, w, has_res=True, math=math, split_k=split,
                    res_resize=(h // 2, w // 2, "half_pixel")).load_weights(wt, b)
    got = plan(torch.from_numpy(x).cuda(), torch.from_numpy(lo).cuda()).cpu().numpy()
    if math == "fp32_strict":
        assert np.array_equal(got, want)
    else:
        assert plan.kernel == "pw" and plan.math == "tf32"
        assert normalised_error(got, want, scale) <= TOL_TF32
        # the same GEMM with the upsampled residual as a plain tensor: only
        # the residual's source differs, so the outputs agree bit for bit
        ref = ConvPlan(op, n, h, w, has_res=True, math=math, split_k=split).load_weights(wt, b)
        same = ref(torch.from_numpy(x).cuda(), torch.from_numpy(up).cuda()).cpu().numpy()
        assert np.array_equal(got, same)


def test_graph_fusion_matches_unfused(cuda_ok):
    """The whole benchmark network with Resize->Conv fusion equals the same
    network run op by op (FFMA path, so the only difference is the fusion)."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    x = torch.from_numpy(segnet.synthetic_input(2, seed=3)).cuda()
    a = Model(g, wts, 2, (segnet.H, segnet.W, 3), math="fp32_strict", fuse=True)
    b = Model(g, wts, 2, (segnet.H, segnet.W, 3), math="fp32_strict", fuse=False)
    assert len(a.ops) < len(b.ops)
    assert torch.equal(a.infer(x), b.infer(x))


def test_pipelined_run_matches_per_batch(cuda_ok):
    """Model.run_pipelined (double-buffered upload / graph replay / read-back
    on three streams) gives, for every batch, exactly what a plain
    upload + infer + read-back of that batch gives."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    m = Model(g, wts, 2, (segnet.H, segnet.W, 3), math="auto")
    xs = [torch.from_numpy(segnet.synthetic_input(2, seed=50 + k)).pin_memory() for k in range(5)]
    want = [m.infer(x.cuda()).cpu() for x in xs]
    outs = [torch.empty(want[0].shape, dtype=torch.float32).pin_memory() for _ in range(5)]
    m.run_pipelined(xs, outs)
    torch.cuda.synchronize()
    for k in range(5):
        assert torch.equal(outs[k], want[k]), k
    # a second pass reuses the captured slot graphs
    outs2 = [torch.empty_like(o).pin_memory() for o in outs]
    m.run_pipelined(xs[::-1], outs2)
    torch.cuda.synchronize()
    for k in range(5):
        assert torch.equal(outs2[k], want[4 - k]), k
    m.release()


STEM_TC = [  # n, ih, iw, cin, stride, pad (t, l, b, r), act
    (2, 160, 288, 3, 2, (1, 1, 1, 1), "relu"),       # the benchmark stem
    (1, 37, 51, 3, 2, (0, 0, 1, 1), "hardswish"),   # ragged tiles, asymmetric SAME pad
    (3, 20, 33, 1, 1, (1, 1, 1, 1), "none"),
    (1, 17, 16, 2, 1, (1, 1, 1, 1), "sigmoid"),
    (2, 64, 64, 3, 1, (1, 1, 1, 1), "relu6"),
    (1, 5, 7, 3, 2, (1, 1, 1, 1), "none"),          # smaller than one tile
    (12, 160, 288, 3, 2, (1, 1, 1, 1), "relu"),      # 540 tiles: more than the resident CTAs,
                                                     # so each CTA cycles both halo buffers
]


@pytest.mark.parametrize("math", ["tf32", "auto"])
@pytest.mark.parametrize("n,ih,iw,cin,s,pad,act", STEM_TC, ids=[f"{c[1]}x{c[2]}c{c[3]}s{c[4]}" for c in STEM_TC])
def test_tc_stem(cuda_ok, math, n, ih, iw, cin, s, pad, act):
    """The tensor-core stem (im2col GEMM, K = 9*cin padded to 32) against
    the ai-cpu restatement; auto picks it for the stem shape."""
    op = Conv2d(cin, 32, 3, 3, s, s, pad, 1, 1, act)
    x, wt, b, _ = case_tensors(op, n, ih, iw, 9100 + ih + cin, False)
    plan, _ = check(op, x, wt, b, None, math)
    assert plan.math == "tf32" and plan.kernel == "stem" and plan.info.variant == 2


def test_tc_stem_views_and_fallback(cuda_ok):
    """C4 input (pixel stride 4); an aligned output view takes the tensor-core
    stem, a misaligned one (coff 2: 8-byte offset) falls back to the FFMA
    implicit GEMM with the same packed weights."""
    from tests.test_conv_gpu import case_tensors as ct
    op = Conv2d(3, 32, 3, 3, 2, 2, (1, 1, 1, 1), 1, 1, "relu")
    x, wt, b, _ = ct(op, 2, 30, 46, 9201, False)
    want, scale = oracle_conv(op, x, wt, b, None)
    plan, got = run_gpu(op, x, wt, b, None, layout="nhwc_c4", math="tf32")
    assert normalised_error(got, want, scale) <= TOL_TF32
    from ai_engine_b200 import View
    for coff in (4, 2):
        stride = 40
        plan = ConvPlan(op, 2, 30, 46, math="tf32", out_view=View(stride, coff)).load_weights(wt, b)
        buf = torch.full((2, plan.oh, plan.ow, stride), 7.0, device="cuda")
        plan(torch.from_numpy(x).cuda(), out=buf)
        torch.cuda.synchronize()
        g = buf.cpu().numpy()
        assert normalised_error(g[..., coff:coff + 32], want, scale) <= TOL_TF32
        assert (g[..., :coff] == 7.0).all() and (g[..., coff + 32:] == 7.0).all()


@pytest.mark.parametrize("case", ["3x3 128->250", "3x3 128->256 res", "1x1 512->256 res", "1x1 512->256 bilinear res"])
def test_wide_tiles_read_bias_from_global(cuda_ok, case):
    """Wide (N = 256) tiles whose 48 KB stages leave room for only three
    ring stages drop the epilogue's shared bias copies for a fourth stage
    and read the bias from global memory: a partial last 32-column chunk
    (cout 250), a 1x1 with a long K, and a resized (bilinear, not exact-2x)
    residual read by the epilogue; with a tensor residual the prefetch
    buffers keep the ring at three stages either way, so that case keeps
    the copies.  Against the oracle at the TF32 bar."""
    import oracle
    from oracle import XorShift32
    rng = XorShift32(1700 + len(case))
    if case.startswith("3x3"):
        n, h, w = 2, 9, 16  # few tiles: split-K, the N tile stays 256
        cout = 250 if "250" in case else 256
        op = Conv2d.same(128, cout, 3, 1, "hardswish")
    else:
        n, h, w = 1, 100, 192  # 150 M tiles: no split, so the 1x1 keeps its 256-wide N tile
        cout = 256
        op = Conv2d.pointwise(512, cout, "relu")
    x = rng.vec_f32(n * h * w * op.cin).reshape(n, h, w, op.cin)
    wt = rng.vec_f32(op.cout * op.cin * op.kh * op.kw)
    b = rng.vec_f32(op.cout)
    if "bilinear" in case:
        lh, lw = 37, 71
        lo = rng.vec_f32(n * lh * lw * cout).reshape(n, lh, lw, cout)
        res = oracle.resize_bilinear(lo, h, w, "half_pixel")
        plan = ConvPlan(op, n, h, w, has_res=True, math="tf32", res_resize=(lh, lw, "half_pixel")).load_weights(wt, b)
        got = plan(torch.from_numpy(x).cuda(), torch.from_numpy(lo).cuda()).cpu().numpy()
    else:
        res = rng.vec_f32(n * h * w * cout).reshape(n, h, w, cout) if "res" in case else None
        plan = ConvPlan(op, n, h, w, has_res=res is not None, math="tf32").load_weights(wt, b)
        got = plan(torch.from_numpy(x).cuda(), None if res is None else torch.from_numpy(res).cuda()).cpu().numpy()
    assert plan.math == "tf32" and plan.info.tile_n == 256
    want, scale = oracle_conv(op, x, wt, b, res)
    assert normalised_error(got, want, scale) <= TOL_TF32
