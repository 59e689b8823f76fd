"""GPU parity of the stem + 1x1 fusion (aie_conv_run_stem_pw): the tensor-
core stem and a TF32 1x1 conv over its output in one launch.  The stem
output must equal the stem run alone bit for bit (same kernel arithmetic),
the 1x1 output must match the 1x1 plan run on that stem output (same MMA
sequence over the same operand values) and the oracle within the TF32 bar."""
import numpy as np
import pytest
import torch

from ai_engine_b200 import Conv2d
from ai_engine_b200._lib import AieError
from ai_engine_b200.conv import ConvPlan, run_stem_pw
from tests._util import TOL_TF32, case_tensors, normalised_error, oracle_conv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,ih,iw,cin,s,cout2,act2", [(2, 160, 288, 3, 2, 32, "none"), (1, 37, 53, 3, 1, 32, "relu"),
                                                       (3, 30, 46, 3, 2, 8, "hardswish"), (1, 19, 33, 1, 2, 16, "none"),
                                                       (1, 64, 64, 2, 1, 12, "sigmoid")])
def test_stem_pw_matches_the_two_launches(cuda_ok, n, ih, iw, cin, s, cout2, act2):
    st = Conv2d.same(cin, 32, 3, s, "relu")
    x, w1, b1, _ = case_tensors(st, n, ih, iw, 8100 + ih + cout2, False)
    pw = Conv2d.pointwise(32, cout2, act2)
    oh, ow = st.out_hw(ih, iw)
    rng = np.random.default_rng(8200 + cout2)
    w2 = (rng.standard_normal(cout2 * 32) * 0.25).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, cout2).astype(np.float32)
    sp = ConvPlan(st, n, ih, iw).load_weights(w1, b1)
    pp = ConvPlan(pw, n, oh, ow).load_weights(w2, b2)
    assert sp.info.variant == 2 and pp.kernel == "pw" and pp.math == "tf32"
    gx = torch.from_numpy(x).cuda()
    s_alone = sp(gx)
    p_alone = pp(s_alone)
    s_fused, p_fused = run_stem_pw(sp, pp, gx)
    torch.cuda.synchronize()
    assert torch.equal(s_fused, s_alone)
    a, f = p_alone.cpu().numpy(), p_fused.cpu().numpy()
    assert np.max(np.abs(a - f) / np.maximum(np.abs(a), 1e-3)) <= 1e-6
    want, scale = oracle_conv(pw, s_alone.cpu().numpy(), w2, b2, None)
    assert normalised_error(f, want, scale) <= TOL_TF32


def test_stem_pw_rejects_other_shapes(cuda_ok):
    st = Conv2d.same(3, 32, 3, 2, "relu")
    sp = ConvPlan(st, 1, 32, 32).load_weights(np.zeros(32 * 27, np.float32), np.zeros(32, np.float32))
    gx = torch.zeros((1, 32, 32, 3), device="cuda")
    for pw in (Conv2d.pointwise(32, 64), Conv2d.pointwise(32, 6)):
        pp = ConvPlan(pw, 1, 16, 16).load_weights(np.zeros(pw.cout * 32, np.float32), np.zeros(pw.cout, np.float32))
        with pytest.raises(AieError) as e:
            run_stem_pw(sp, pp, gx)
        assert e.value.status == -3


def test_segnet_with_and_without_the_stem_fusion(cuda_ok):
    """The benchmark network with the stem + lateral fusion equals the
    network without it (same kernels' arithmetic on the same values)."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    x = torch.from_numpy(segnet.synthetic_input(2, seed=3)).cuda()
    a = Model(g, wts, 2, (segnet.H, segnet.W, 3), fuse_stem=True)
    b = Model(g, wts, 2, (segnet.H, segnet.W, 3), fuse_stem=False)
    assert any(r.kind == "stempw" for r in a.ops) and not any(r.kind == "stempw" for r in b.ops)
    ya, yb = a.infer(x).cpu().numpy(), b.infer(x).cpu().numpy()
    assert np.max(np.abs(ya - yb)) <= 1e-5
