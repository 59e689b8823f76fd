"""Parity of the benchmarked network exactly as bench.py builds it.

bench.py times BASELINE config 4: ``graph.Model`` over the synthetic
MNv4-style segmentation net at 160x288, 256 frames, math "auto" (TF32
tensor cores where the operands allow TMA), every default fusion on (stem +
lateral, the five small-frame inverted-bottleneck blocks, the 960-channel
head conv with the pyramid lateral on it, the depthwise + 1x1 head with the
feature-pyramid tail folded in).  This file builds that
same model with bench.py's own weights and rank-0 input, runs one step on
the GPU, and checks sampled frames of it against the CPU oracle (the C
restatement of ai-cpu):

* op by op: every launch is re-run on the oracle from the GPU's own inputs
  to that launch.  A plain conv is held to its math's bar (TF32 5e-3, FFMA
  1e-5) on the normalised error; a fused launch is compared with the
  oracle's chain of its member ops, normalised by the chain's magnitude
  (the same chain run on |x|, |w|, |b|), at the bar of its least precise
  member; resizes bit for bit.
* end to end: the mask against the oracle chain with the TF32 convs'
  operands truncated to TF32 as the tensor cores read them
  (``OracleModel(tf32=...)``), at a bound derived from that emulation; and
  against the plain fp32 oracle, at a bound derived from the TF32 operand
  format.

Each assertion message carries the plain max relative error too (outputs
with |want| >= 1e-3 max|want|), the north-star contract's own figure.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200 import segnet
from ai_engine_b200.graph import Model
from oracle.graph import OracleModel
from tests._util import TOL_FFMA, TOL_TF32, errors, normalised_error, plain_rel_error

pytestmark = pytest.mark.gpu

N = 256                      # bench.py's frames per GPU
FRAMES = [0, 101, 255]       # sampled frames checked on the CPU
THREADS = os.cpu_count() or 1

# End-to-end bounds on the mask (sigmoid output in (0, 1), then a bilinear
# resize), max abs over the sampled frames.
# * Against the TF32-emulating oracle the two chains differ in the order of
#   fp32 sums (tensor-core accumulation, fused launches), and an activation
#   one fp32 ulp apart can truncate to TF32 values one TF32 ulp (2^-10
#   relative) apart, so the emulation tracks the GPU only approximately:
#   measured 2.9e-3 on frame 0 of bench.py's input; bound 2x that.
E2E_EMULATED = 6e-3
# * Against the plain fp32 oracle the TF32 operand format itself moves the
#   mask (10 mantissa bits per operand, truncated): measured 9.7e-3 on frame
#   0; bound 3x that.
E2E_FP32 = 3e-2


@pytest.fixture(scope="module")
def bench_step():
    g = segnet.build_graph()
    wts = segnet.init_weights(g)             # bench.py: segnet.init_weights(g)
    x = segnet.synthetic_input(N, seed=100)  # bench.py rank 0: seed 100 + rank
    m = Model(g, wts, N, (segnet.H, segnet.W, 3), math="auto")  # bench.py's defaults
    m.bufs["input"].copy_(torch.from_numpy(x))
    m.record()
    torch.cuda.synchronize()
    idx = torch.tensor(FRAMES, device=m.device)
    host = {k: v.index_select(0, idx).cpu().numpy() for k, v in m.bufs.items()}
    yield g, wts, m, x, host
    m.release()


def _conv(g, name):
    return next(op[3] for op in g if op[0] == "conv" and op[1] == name)


def _chain(g, wts, names, x, res=None, add=None):
    """The oracle's chain of convs `names` from x (and |.| magnitude chain);
    `add` is added to x first, `res` is the last conv's residual."""
    if add is not None:
        x = (x + add).astype(np.float32)
    val, mag = x, np.abs(x.astype(np.float64))
    for i, nm in enumerate(names):
        op = _conv(g, nm)
        w, b = wts[nm]
        last = i == len(names) - 1
        r = res if last else None
        val = oracle.conv_aicpu(op, val, w, b, r)
        mag = oracle.dot_scale(op, mag, w, b) + (np.abs(r) if r is not None else 0.0)
    return val, mag


def test_bench_model_is_the_fused_config4_net(cuda_ok, bench_step):
    """The model under test has the launches bench.py times."""
    g, wts, m, x, host = bench_step
    kinds = [r.kind for r in m.ops]
    assert kinds.count("mb") == 6 and kinds.count("stempw") == 1 and kinds.count("dwpw") == 1
    dwpw = next(r for r in m.ops if r.kind == "dwpw")
    assert dwpw.up is not None, "the feature-pyramid tail is folded into the head"
    assert all(r.plan.math == "tf32" for r in m.ops if r.kind == "conv" and r.plan.kernel in ("pw", "igemm"))
    assert m.n == N and m.bufs["mask"].shape == (N, segnet.H, segnet.W, 1)


def test_bench_model_op_by_op(cuda_ok, bench_step):
    g, wts, m, x, host = bench_step
    report = []
    checked = set()
    for r in m.ops:
        src = host[r.src]
        if r.kind == "conv":
            res = host[r.res] if r.res else None
            w, b = wts[r.out]
            want = oracle.conv_aicpu(r.conv, src, w, b, res)
            scale = oracle.dot_scale(r.conv, src, w, b) + (np.abs(res) if res is not None else 0.0)
            pairs = [(r.out, host[r.out], want, scale, TOL_TF32 if r.plan.math == "tf32" else TOL_FFMA)]
        elif r.kind == "stempw":
            stem, lat = r.members
            want_s, scale_s = _chain(g, wts, [stem], src)
            # the fused 1x1 reads the stem's staged tile: the stem output the GPU wrote
            want_l, scale_l = _chain(g, wts, [lat], host[stem])
            pairs = [(stem, host[stem], want_s, scale_s, TOL_TF32), (lat, host[lat], want_l, scale_l, TOL_TF32)]
        elif r.kind == "mb":
            want, scale = _chain(g, wts, list(r.members), src, res=host[r.res] if r.res else None)
            pairs = [(r.out, host[r.out], want, scale, TOL_TF32)]
        elif r.kind == "dwpw":
            add = None
            if r.up:  # the head adds the exact-2x resize of `up` to its input
                h, w_, _ = m.shapes[r.src]
                add = oracle.resize_bilinear(host[r.up], h, w_)
            want, scale = _chain(g, wts, list(r.members), src, add=add)
            tol = TOL_TF32 if "tf32" in (r.plan.math, r.head.math) else TOL_FFMA
            pairs = [(r.out, host[r.out], want, scale, tol)]
        elif r.kind == "resize":
            oh, ow = r.size
            want = oracle.resize_bilinear(src, oh, ow)
            if r.res:
                want = (want + host[r.res]).astype(np.float32)
            assert np.array_equal(host[r.out], want), f"{r.out} (resize): not bit-exact"
            checked.add(r.out)
            continue
        else:
            raise AssertionError(f"unexpected launch kind {r.kind}")
        for name, got, want, scale, tol in pairs:
            assert got.shape == want.shape, name
            err = normalised_error(got, want, scale)
            report.append(f"{name:12s} {r.kind:7s} normalised {err:.2e} plain {plain_rel_error(got, want):.2e}")
            assert err <= tol, f"{name} ({r.kind}): {errors(got, want, scale)} > {tol}"
            checked.add(name)
    print("\n".join(report))
    # every conv and every resize of the graph was checked, alone or inside its fused launch
    graph_names = {op[1] for op in g}
    covered = checked | {mb for r in m.ops for mb in r.members}
    assert graph_names - covered == {"fpn.up4"}, graph_names - covered  # fpn.up4 lives inside the head


def test_bench_model_end_to_end(cuda_ok, bench_step):
    g, wts, m, x, host = bench_step
    emu = OracleModel(g, wts, (segnet.H, segnet.W, 3), tf32=m.tf32_convs())
    fp32 = OracleModel(g, wts, (segnet.H, segnet.W, 3))
    got = host["mask"]
    rows = []
    for i, f in enumerate(FRAMES):
        want_e = emu.infer_frame(x[f], threads=THREADS)
        want_f = fp32.infer_frame(x[f], threads=THREADS)
        rows.append((f, float(np.max(np.abs(got[i] - want_e))), plain_rel_error(got[i], want_e),
                     float(np.max(np.abs(got[i] - want_f))), plain_rel_error(got[i], want_f)))
        print("frame %d: max abs vs TF32-emulated %.3e (plain rel %.3e), vs fp32 %.3e (plain rel %.3e)" % rows[-1])
    for f, e_emu, p_emu, e_fp32, p_fp32 in rows:
        assert e_emu <= E2E_EMULATED, f"frame {f}: mask vs the TF32-emulating oracle: max abs {e_emu:.3e}, " \
            f"plain relative {p_emu:.3e}"
        assert e_fp32 <= E2E_FP32, f"frame {f}: mask vs the fp32 oracle: max abs {e_fp32:.3e}, " \
            f"plain relative {p_fp32:.3e}"
    assert np.all((got >= 0) & (got <= 1))


def test_bench_model_graph_replay_matches_eager(cuda_ok, bench_step):
    """bench.py times the captured CUDA graph: its replay writes the same
    mask as the eager step checked above, bit for bit."""
    g, wts, m, x, host = bench_step
    m.capture()
    m.bufs["mask"].zero_()
    m.infer()
    torch.cuda.synchronize()
    idx = torch.tensor(FRAMES, device=m.device)
    assert np.array_equal(m.bufs["mask"].index_select(0, idx).cpu().numpy(), host["mask"])
