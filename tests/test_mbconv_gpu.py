"""GPU parity of the fused inverted-bottleneck block (aie_conv_run_mbconv):
1x1 expand -> depthwise 3x3 -> 1x1 project (+ residual) in one launch,
against the same three plans run one after another on the GPU and against
the CPU oracle's chain (TF32 bar, 5e-3 normalised)."""
import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200 import Conv2d
from ai_engine_b200._lib import AieError
from ai_engine_b200.conv import ConvPlan, run_mbconv
from oracle import XorShift32
from tests._util import TOL_TF32, normalised_error, oracle_conv

pytestmark = pytest.mark.gpu

# (n, h, w, cin, cexp, cout, residual, expand / depthwise / project activations)
BLOCKS = [
    (3, 10, 18, 96, 192, 96, True, ("relu", "relu", "none")),      # e4: the second chunk is half padding
    (2, 10, 18, 128, 512, 128, True, ("relu", "relu", "none")),    # e5.0 / e5.1
    (2, 10, 18, 96, 384, 128, False, ("relu", "relu", "none")),    # e5
    (5, 7, 11, 64, 160, 64, True, ("hardswish", "hardswish", "none")),
    (1, 10, 18, 32, 128, 32, False, ("relu6", "relu", "sigmoid")),  # the largest frame
    (4, 3, 5, 32, 256, 32, True, ("relu", "none", "relu")),        # a frame smaller than every tile
    (149, 10, 18, 32, 128, 32, True, ("relu", "relu", "none")),    # more frames than SMs
]


def _block(n, h, w, cin, cexp, cout, res, acts, seed):
    rng = XorShift32(seed)
    x = rng.vec_f32(n * h * w * cin).reshape(n, h, w, cin)
    we, be = rng.vec_f32(cexp * cin), rng.vec_f32(cexp)
    wd, bd = rng.vec_f32(cexp * 9), rng.vec_f32(cexp)
    wp, bp = rng.vec_f32(cout * cexp), rng.vec_f32(cout)
    ops = (Conv2d.pointwise(cin, cexp, acts[0]), Conv2d.depthwise(cexp, 3, 1, acts[1]),
           Conv2d.pointwise(cexp, cout, acts[2]))
    return x, (we, be), (wd, bd), (wp, bp), ops


@pytest.mark.parametrize("n,h,w,cin,cexp,cout,res,acts", BLOCKS)
def test_fused_block_matches_chain(cuda_ok, n, h, w, cin, cexp, cout, res, acts):
    x, (we, be), (wd, bd), (wp, bp), (eop, dop, pop) = _block(n, h, w, cin, cexp, cout, res, acts, 300 + cexp + h)
    ex = ConvPlan(eop, n, h, w, math="tf32").load_weights(we, be)
    dw = ConvPlan(dop, n, h, w, math="ffma").load_weights(wd, bd)
    pj = ConvPlan(pop, n, h, w, has_res=res, math="tf32").load_weights(wp, bp)
    xd = torch.from_numpy(x).cuda()
    rd = xd if res else None
    got = run_mbconv(ex, dw, pj, xd, res=rd).cpu().numpy()
    # the three plans one after another
    chain = pj(dw(ex(xd)), rd).cpu().numpy()
    # the oracle's chain (ai-cpu arithmetic) and the magnitude the last sum's rounding is relative to
    e_o, _ = oracle_conv(eop, x, we, be, None)
    d_o, _ = oracle_conv(dop, e_o, wd, bd, None)
    want, scale = oracle_conv(pop, d_o, wp, bp, x if res else None)
    assert normalised_error(got, chain, scale) <= TOL_TF32
    assert normalised_error(got, want, scale) <= TOL_TF32
    assert np.isfinite(got).all()


# (n, h, w, cin, cexp, cout, residual, expand / project activations)
PAIRS = [
    (3, 10, 18, 128, 960, 64, False, ("relu", "none")),    # head960 -> fpn.lat16: 7.5 chunks
    (2, 10, 18, 64, 256, 128, True, ("hardswish", "relu")),
    (149, 7, 11, 32, 96, 16, False, ("relu", "sigmoid")),  # more frames than SMs, a partial chunk
]


@pytest.mark.parametrize("n,h,w,cin,cexp,cout,res,acts", PAIRS)
def test_fused_expand_project_matches_chain(cuda_ok, n, h, w, cin, cexp, cout, res, acts):
    """No depthwise (dw = None): a 1x1 expand read only by a 1x1 project in
    one launch, the expanded tensor kept on chip."""
    rng = XorShift32(500 + cexp + h)
    x = rng.vec_f32(n * h * w * cin).reshape(n, h, w, cin)
    we, be = rng.vec_f32(cexp * cin), rng.vec_f32(cexp)
    wp, bp = rng.vec_f32(cout * cexp), rng.vec_f32(cout)
    eop, pop = Conv2d.pointwise(cin, cexp, acts[0]), Conv2d.pointwise(cexp, cout, acts[1])
    ex = ConvPlan(eop, n, h, w, math="tf32").load_weights(we, be)
    pj = ConvPlan(pop, n, h, w, has_res=res, math="tf32").load_weights(wp, bp)
    r = rng.vec_f32(n * h * w * cout).reshape(n, h, w, cout) if res else None
    xd = torch.from_numpy(x).cuda()
    rd = torch.from_numpy(r).cuda() if res else None
    got = run_mbconv(ex, None, pj, xd, res=rd).cpu().numpy()
    chain = pj(ex(xd), rd).cpu().numpy()
    e_o, _ = oracle_conv(eop, x, we, be, None)
    want, scale = oracle_conv(pop, e_o, wp, bp, r)
    assert normalised_error(got, chain, scale) <= TOL_TF32
    assert normalised_error(got, want, scale) <= TOL_TF32
    assert np.isfinite(got).all()


def test_fused_block_rejects_unsupported(cuda_ok):
    """Frames above 10 x 18, cin not a multiple of 32, an FP32_STRICT
    depthwise plan and a missing residual are refused, not run."""
    def plans(n, h, w, cin, cexp, cout, dw_math="ffma", res=False):
        ex = ConvPlan(Conv2d.pointwise(cin, cexp, "relu"), n, h, w, math="tf32")
        dw = ConvPlan(Conv2d.depthwise(cexp, 3, 1, "relu"), n, h, w, math=dw_math)
        pj = ConvPlan(Conv2d.pointwise(cexp, cout, "none"), n, h, w, has_res=res, math="tf32")
        ex.load_weights(np.zeros(cexp * cin, np.float32), np.zeros(cexp, np.float32))
        dw.load_weights(np.zeros(cexp * 9, np.float32), np.zeros(cexp, np.float32))
        pj.load_weights(np.zeros(cout * cexp, np.float32), np.zeros(cout, np.float32))
        return ex, dw, pj
    for args, kw in [((1, 11, 18, 32, 64, 32), {}), ((1, 10, 19, 32, 64, 32), {}), ((1, 10, 18, 48, 96, 32), {}),
                     ((1, 10, 18, 32, 64, 32), {"dw_math": "fp32_strict"})]:
        ex, dw, pj = plans(*args, **kw)
        x = torch.zeros(1, args[1], args[2], args[3], device="cuda")
        with pytest.raises(AieError):
            run_mbconv(ex, dw, pj, x)
    ex, dw, pj = plans(1, 10, 18, 32, 64, 32, res=True)
    with pytest.raises(AieError):
        run_mbconv(ex, dw, pj, torch.zeros(1, 10, 18, 32, device="cuda"))  # residual plan without a residual


def test_model_fuses_the_small_frame_blocks(cuda_ok):
    """The benchmark network runs its five 10x18 inverted-bottleneck blocks
    (e4.0, e4.1, e5, e5.0, e5.1) and the 960-channel head conv with the
    pyramid lateral on it (head960 -> fpn.lat16) as fused launches; the mask
    equals the network run op by op within the TF32 bar."""
    from ai_engine_b200 import segnet
    from ai_engine_b200.graph import Model
    g = segnet.build_graph()
    wts = segnet.init_weights(g)
    x = torch.from_numpy(segnet.synthetic_input(2, seed=21)).cuda()
    a = Model(g, wts, 2, (segnet.H, segnet.W, 3), fuse_blocks=True)
    b = Model(g, wts, 2, (segnet.H, segnet.W, 3), fuse_blocks=False)
    blocks = [r.out for r in a.ops if r.kind == "mb"]
    assert blocks == ["e4.0.proj", "e4.1.proj", "e5.proj", "e5.0.proj", "e5.1.proj", "fpn.lat16"]
    assert len(a.ops) == len(b.ops) - 11
    ya, yb = a.infer(x), b.infer(x)
    assert torch.isfinite(ya).all()
    assert (ya - yb).abs().max().item() <= 5e-3
