"""Concat-into-conv on the tensor cores (aie_conv_plan_parts /
aie_conv_run_parts): the conv reads up to three channel views in place, as
ai-gpu's implicit-GEMM conv reads its concat parts (ConvIgemmSpec srcs,
crates/ai-gpu/src/kernels/conv_igemm.rs:49-76), against the oracle conv of
the concatenated input (TF32 bar, normalised error) and against concat +
ordinary conv on the GPU."""
import numpy as np
import pytest
import torch

from ai_engine_b200 import Conv2d
from ai_engine_b200.conv import ConvPlan, run_parts
from oracle import XorShift32
from tests._util import TOL_TF32, errors, normalised_error, oracle_conv

pytestmark = pytest.mark.gpu

CASES = [  # n, h, w, parts, cout, k, stride, residual
    (2, 18, 32, (40, 24, 20), 32, 3, 1, False),   # flat mode (narrow N), three parts, ragged K blocks
    (3, 20, 36, (16, 16), 16, 3, 1, True),        # ConvGRU-style (x, h) pair, residual
    (2, 40, 72, (32, 4), 16, 3, 1, False),        # a 4-channel part (one K block of zero fill)
    (2, 21, 37, (64, 36), 96, 3, 2, False),       # stride 2 (general mode), ragged frame
    (2, 10, 18, (96, 64, 128), 128, 1, 1, True),  # 1x1 GEMM, residual
    (4, 9, 16, (128, 40), 200, 3, 1, False),      # wide N (per-tap boxes), two N tiles
    (2, 18, 30, (8, 16, 12), 24, 3, 1, False),    # three parts of <= 16 channels: 16-channel K blocks
    (2, 10, 18, (16, 16), 48, 1, 1, True),        # 1x1 over two 16-channel parts
]


def _case(n, h, w, parts, cout, k, s, res, seed):
    cin = sum(parts)
    op = Conv2d.same(cin, cout, k, s, "relu")
    rng = XorShift32(seed)
    xs = [rng.vec_f32(n * h * w * c).reshape(n, h, w, c) for c in parts]
    wt = rng.vec_f32(cout * cin * k * k)
    b = rng.vec_f32(cout)
    oh, ow = op.out_hw(h, w)
    r = rng.vec_f32(n * oh * ow * cout).reshape(n, oh, ow, cout) if res else None
    return op, xs, wt, b, r


@pytest.mark.parametrize("n,h,w,parts,cout,k,s,res", CASES, ids=[str(c[3]) + f"k{c[5]}s{c[6]}" for c in CASES])
def test_parts_match_oracle_and_concat(cuda_ok, n, h, w, parts, cout, k, s, res):
    op, xs, wt, b, r = _case(n, h, w, parts, cout, k, s, res, 4100 + sum(parts) + k)
    x = np.concatenate(xs, axis=-1)
    want, scale = oracle_conv(op, x, wt, b, r)
    plan = ConvPlan(op, n, h, w, has_res=res, parts=parts).load_weights(wt, b)
    assert plan.math == "tf32"
    rd = torch.from_numpy(r).cuda() if res else None
    got = run_parts(plan, [torch.from_numpy(a).cuda() for a in xs], rd).cpu().numpy()
    err = normalised_error(got, want, scale)
    assert err <= TOL_TF32, errors(got, want, scale)
    ref = ConvPlan(op, n, h, w, has_res=res, math="tf32").load_weights(wt, b)
    same = ref(torch.from_numpy(x).cuda(), rd).cpu().numpy()
    assert normalised_error(got, same, scale) <= TOL_TF32
    # twice in a row: same result (deterministic)
    again = run_parts(plan, [torch.from_numpy(a).cuda() for a in xs], rd).cpu().numpy()
    assert np.array_equal(got, again)


def test_parts_read_channel_views(cuda_ok):
    """Parts given as channel slices of wider buffers (a split's outputs, a
    state buffer), the other channels of those buffers ignored."""
    n, h, w = 2, 16, 24
    op, xs, wt, b, _ = _case(n, h, w, (24, 16), 32, 3, 1, False, 4200)
    big0 = torch.full((n, h, w, 40), 9.0, device="cuda")
    big0[..., 8:32] = torch.from_numpy(xs[0]).cuda()
    big1 = torch.full((n, h, w, 16), 0.0, device="cuda")
    big1.copy_(torch.from_numpy(xs[1]))
    want, scale = oracle_conv(op, np.concatenate(xs, -1), wt, b, None)
    plan = ConvPlan(op, n, h, w, parts=(24, 16)).load_weights(wt, b)
    got = run_parts(plan, [(big0, 8), big1]).cpu().numpy()
    assert normalised_error(got, want, scale) <= TOL_TF32, errors(got, want, scale)


def test_parts_reject_unaligned_views(cuda_ok):
    """A part whose pixel stride is not a multiple of 4 channels cannot be a
    TMA source: AIE_E_ALIGN, nothing launched."""
    from ai_engine_b200._lib import AieError
    n, h, w = 1, 8, 8
    op = Conv2d.same(35, 16, 3, 1, "relu")
    plan = ConvPlan(op, n, h, w, parts=(32, 3)).load_weights(np.zeros(16 * 35 * 9, np.float32))
    a = torch.zeros(n, h, w, 32, device="cuda")
    bad = torch.zeros(n, h, w, 3, device="cuda")  # 12-byte pixel stride
    with pytest.raises(AieError) as e:
        run_parts(plan, [a, bad])
    assert e.value.status == -5
