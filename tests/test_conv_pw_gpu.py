"""GPU parity of the conv + 1x1 chain (aie_conv_run_conv_pw): a TF32
tensor-core conv with 32 output channels and a TF32 1x1 over its output in
one launch.  The first conv's output (when stored) equals the conv run alone
bit for bit, the 1x1's output matches the 1x1 plan run on that output (same
MMA sequence on the same values) and the oracle within the TF32 bar."""
import numpy as np
import pytest
import torch

from ai_engine_b200 import Conv2d
from ai_engine_b200._lib import AieError
from ai_engine_b200.conv import ConvPlan, run_conv_pw
from tests._util import TOL_TF32, case_tensors, normalised_error, oracle_conv

pytestmark = pytest.mark.gpu

CASES = [  # (n, ih, iw, first conv, 1x1 cout, 1x1 act)
    (2, 80, 144, Conv2d.same(32, 32, 3, 2, "relu"), 32, "relu"),      # the benchmark's e1.conv -> e1.pw
    (3, 13, 29, Conv2d.pointwise(64, 32, "hardswish"), 16, "hardswish"),
    (1, 37, 53, Conv2d.same(16, 32, 3, 1, "none"), 8, "sigmoid"),
    (2, 20, 36, Conv2d.same(64, 32, 3, 1, "relu"), 32, "none"),
]


@pytest.mark.parametrize("n,ih,iw,op1,cout2,act2", CASES, ids=[f"{c[3].kh}x{c[3].kw}s{c[3].sh}-{c[3].cin}-{c[4]}"
                                                                for c in CASES])
def test_conv_pw_matches_the_two_launches(cuda_ok, n, ih, iw, op1, cout2, act2):
    x, w1, b1, _ = case_tensors(op1, n, ih, iw, 8300 + ih + cout2, False)
    oh, ow = op1.out_hw(ih, iw)
    op2 = Conv2d.pointwise(32, cout2, act2)
    rng = np.random.default_rng(8400 + cout2)
    w2 = (rng.standard_normal(cout2 * 32) * 0.25).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, cout2).astype(np.float32)
    p1 = ConvPlan(op1, n, ih, iw).load_weights(w1, b1)
    p2 = ConvPlan(op2, n, oh, ow).load_weights(w2, b2)
    assert p1.math == "tf32" and p2.kernel == "pw" and p2.math == "tf32"
    gx = torch.from_numpy(x).cuda()
    y1 = p1(gx)
    y2 = p2(y1)
    f1 = torch.full_like(y1, 7.0)
    f2 = run_conv_pw(p1, p2, gx, out1=f1)
    g2 = run_conv_pw(p1, p2, gx)  # without the first output
    torch.cuda.synchronize()
    assert torch.equal(f1, y1)
    a, f, g = y2.cpu().numpy(), f2.cpu().numpy(), g2.cpu().numpy()
    assert np.array_equal(f, g)
    assert np.max(np.abs(a - f) / np.maximum(np.abs(a), 1e-3)) <= 1e-6
    want, scale = oracle_conv(op2, y1.cpu().numpy(), w2, b2, None)
    assert normalised_error(f, want, scale) <= TOL_TF32


def test_conv_pw_rejects_other_shapes(cuda_ok):
    op2 = Conv2d.pointwise(32, 16)
    w2, b2 = np.zeros(16 * 32, np.float32), np.zeros(16, np.float32)
    gx = torch.zeros((1, 16, 16, 32), device="cuda")
    wide = Conv2d.pointwise(32, 64)
    p1 = ConvPlan(wide, 1, 16, 16).load_weights(np.zeros(64 * 32, np.float32), np.zeros(64, np.float32))
    p2 = ConvPlan(Conv2d.pointwise(64, 16), 1, 16, 16).load_weights(np.zeros(16 * 64, np.float32), b2)
    with pytest.raises(AieError) as e:
        run_conv_pw(p1, p2, gx)
    assert e.value.status == -3
    p1 = ConvPlan(Conv2d.pointwise(32, 32), 1, 16, 16, has_res=True).load_weights(np.zeros(1024, np.float32),
                                                                                   np.zeros(32, np.float32))
    p2 = ConvPlan(op2, 1, 16, 16).load_weights(w2, b2)
    with pytest.raises(AieError) as e:
        run_conv_pw(p1, p2, gx)
    assert e.value.status == -3


def test_segnet_with_and_without_the_chain(cuda_ok):
    """The benchmark network with e1.conv -> e1.pw chained equals the network
    without the chain."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    x = torch.from_numpy(segnet.synthetic_input(2, seed=4)).cuda()
    a = Model(g, wts, 2, (segnet.H, segnet.W, 3), fuse_chain=True)
    b = Model(g, wts, 2, (segnet.H, segnet.W, 3), fuse_chain=False)
    chained = [r for r in a.ops if r.kind == "convpw"]
    assert [(r.out, r.out2) for r in chained] == [("e1.conv", "e1.pw")]
    ya, yb = a.infer(x).cpu().numpy(), b.infer(x).cpu().numpy()
    assert np.max(np.abs(ya - yb)) <= 1e-5
