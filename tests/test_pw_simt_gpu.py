"""GPU parity of pw_simt_kernel: the 1x1 conv on the FP32 pipes for cin and
cout in {32, 64}, with no residual, a residual tensor, or the exact-2x
half_pixel bilinear sample of a half-size tensor (the FPN's Resize ->
Conv(res) pair in one pass).  FFMA tolerance (1e-5 normalised) against the
CPU oracle; the fused bilinear residual equals the unfused pair bit for bit."""
import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200 import Conv2d
from ai_engine_b200.conv import ConvPlan, View
from oracle import XorShift32
from tests._util import TOL_FFMA, normalised_error, oracle_conv

pytestmark = pytest.mark.gpu

CHANNELS = [(32, 32), (32, 64), (64, 32), (64, 64)]
# (n, h, w): ragged last tile with rows wrapping across frames; a batch
# smaller than one tile; several full tiles
SIZES = [(2, 10, 38), (1, 4, 6), (3, 16, 64)]
ACTS = ["none", "relu", "hardswish", "sigmoid"]


def _tensors(cin, cout, n, h, w, seed):
    rng = XorShift32(seed)
    x = rng.vec_f32(n * h * w * cin).reshape(n, h, w, cin)
    wt = rng.vec_f32(cout * cin)
    b = rng.vec_f32(cout)
    lo = rng.vec_f32(n * (h // 2) * (w // 2) * cout).reshape(n, h // 2, w // 2, cout)
    return x, wt, b, lo


@pytest.mark.parametrize("cin,cout", CHANNELS)
@pytest.mark.parametrize("res", ["none", "tensor", "up2"])
@pytest.mark.parametrize("size", SIZES)
def test_pw_simt_matches_oracle(cuda_ok, cin, cout, res, size):
    n, h, w = size
    act = ACTS[(cin + cout + len(res) + h) % len(ACTS)]
    op = Conv2d.pointwise(cin, cout, act)
    x, wt, b, lo = _tensors(cin, cout, n, h, w, 31 * cin + cout + h)
    up = oracle.resize_bilinear(lo, h, w, "half_pixel")
    want, scale = oracle_conv(op, x, wt, b, None if res == "none" else up)
    kw = {"res_resize": (h // 2, w // 2, "half_pixel")} if res == "up2" else {}
    plan = ConvPlan(op, n, h, w, has_res=res != "none", math="ffma", **kw).load_weights(wt, b)
    assert plan.kernel == "pw_simt" and plan.math == "ffma"
    rd = None if res == "none" else torch.from_numpy(lo if res == "up2" else up).cuda()
    got = plan(torch.from_numpy(x).cuda(), rd).cpu().numpy()
    err = normalised_error(got, want, scale)
    assert err <= TOL_FFMA, f"normalised error {err:.3g}"


@pytest.mark.parametrize("cin,cout", CHANNELS)
def test_pw_simt_up2_equals_unfused(cuda_ok, cin, cout):
    """AUTO picks the FP32-pipe kernel for an exact-2x residual; the fused
    sample is the resize kernel's value bit for bit, so the output equals
    the same kernel run with the upsampled tensor as a plain residual."""
    from ai_engine_b200 import resize_bilinear
    n, h, w = 2, 20, 36
    op = Conv2d.pointwise(cin, cout, "none")
    x, wt, b, lo = _tensors(cin, cout, n, h, w, 500 + cin + cout)
    fused = ConvPlan(op, n, h, w, has_res=True, math="auto",
                     res_resize=(h // 2, w // 2, "half_pixel")).load_weights(wt, b)
    assert fused.kernel == "pw_simt" and fused.math == "ffma"
    lo_d = torch.from_numpy(lo).cuda()
    got = fused(torch.from_numpy(x).cuda(), lo_d).cpu().numpy()
    up = resize_bilinear(lo_d, h, w)
    plain = ConvPlan(op, n, h, w, has_res=True, math="ffma").load_weights(wt, b)
    same = plain(torch.from_numpy(x).cuda(), up).cpu().numpy()
    assert np.array_equal(got, same)


@pytest.mark.parametrize("coff", [0, 4, 2])
def test_pw_simt_channel_views(cuda_ok, coff):
    """Input, residual and output as channel slices of wider tensors; an
    offset that breaks 16-byte alignment (coff 2) still gives the right
    result (the FFMA implicit GEMM runs it)."""
    n, h, w, cin, cout = 2, 6, 40, 32, 32
    op = Conv2d.pointwise(cin, cout, "relu")
    x, wt, b, lo = _tensors(cin, cout, n, h, w, 77 + coff)
    res = oracle.resize_bilinear(lo, h, w, "half_pixel")
    want, scale = oracle_conv(op, x, wt, b, res)
    big_x = np.zeros((n, h, w, cin + 8), np.float32)
    big_x[..., coff:coff + cin] = x
    big_r = np.zeros((n, h, w, cout + 8), np.float32)
    big_r[..., coff:coff + cout] = res
    big_y = torch.full((n, h, w, cout + 8), 7.0, device="cuda")
    plan = ConvPlan(op, n, h, w, has_res=True, math="ffma", in_view=View(cin + 8, coff),
                    res_view=View(cout + 8, coff), out_view=View(cout + 8, coff)).load_weights(wt, b)
    plan(torch.from_numpy(big_x).cuda(), torch.from_numpy(big_r).cuda(), out=big_y)
    got = big_y.cpu().numpy()
    assert normalised_error(got[..., coff:coff + cout], want, scale) <= TOL_FFMA
    assert (got[..., :coff] == 7).all() and (got[..., coff + cout:] == 7).all()


def test_pw_simt_large_batch_tiles(cuda_ok):
    """Many tiles per CTA (persistent loop, both input buffers cycling):
    the FPN lateral at 80x144 against the tensor-core GEMM of the same conv
    (itself pinned to the oracle), within the TF32 bar."""
    from tests._util import TOL_TF32
    n, h, w, cin, cout = 24, 80, 144, 32, 32
    op = Conv2d.pointwise(cin, cout, "none")
    x, wt, b, lo = _tensors(cin, cout, n, h, w, 9)
    xd = torch.from_numpy(x).cuda()
    up = torch.from_numpy(oracle.resize_bilinear(lo, h, w, "half_pixel")).cuda()
    a = ConvPlan(op, n, h, w, has_res=True, math="ffma").load_weights(wt, b)
    t = ConvPlan(op, n, h, w, has_res=True, math="tf32").load_weights(wt, b)
    assert a.kernel == "pw_simt" and t.kernel == "pw"
    ga, gt = a(xd, up).cpu().numpy(), t(xd, up).cpu().numpy()
    scale = oracle.dot_scale(op, x, wt, b) + np.abs(up.cpu().numpy())
    assert normalised_error(ga, gt, scale) <= TOL_TF32
