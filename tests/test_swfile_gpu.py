"""ai_engine's shipped segmentation model (segm_r11_160x288.sw, real
weights) on the GPU through the .sw reader and the node executor, against
the ai-cpu restatement -- the counterpart of ai-gpu-runtime's graph-exec
gate (crates/ai-gpu-runtime/tests/graph_exec.rs:12-72: seeded input
XorShift32(77), every output within max abs error 2e-3 of the CPU
reference)."""
import os

import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200.net import NetModel
from ai_engine_b200.swfile import load_sw
from oracle.net import OracleNet
from tests._util import check_net_ops

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def model():
    fx = np.load(os.path.join(HERE, "golden", "segm_r11.npz"))
    return load_sw(fx["sw"].tobytes()), fx


def _input(sw, seeds):
    (inp, (h, w, c)), = sw.inputs.items()
    return inp, np.stack([oracle.XorShift32(s).vec_f32(h * w * c).reshape(h, w, c) for s in seeds])


def test_segm_r11_graph_exec_gate(cuda_ok, model):
    """The reference's bar, 2e-3 max abs error on the logits, on the FP32
    (FFMA) path -- the precision of the reference's own GPU path -- for the
    seed-77 frame (against the committed golden output) and a second frame
    (against the oracle run here), batched."""
    sw, fx = model
    inp, x = _input(sw, [int(fx["seed"]), 78])
    m = NetModel(sw.nodes, sw.weights, 2, sw.inputs, sw.outputs, sw.states, sw.consts, math="ffma")
    out = m.step({inp: torch.from_numpy(x).cuda()})[sw.outputs[0]].cpu().numpy()
    err0 = float(np.max(np.abs(out[0] - fx["output"])))
    o = OracleNet(sw.nodes, sw.weights, sw.inputs, sw.states, sw.consts)
    want1 = o.step({inp: x[1:]}, {})[sw.outputs[0]][0]
    err1 = float(np.max(np.abs(out[1] - want1)))
    assert err0 < 2e-3 and err1 < 2e-3, (err0, err1)


def test_segm_r11_tf32_end_to_end(cuda_ok, model):
    """The default path (TF32 tensor cores for the dense convs).  Against the
    oracle with those convs' operands truncated to TF32: within 2e-2.
    Against the plain fp32 golden: the TF32 format itself moves the logits
    (range about +-8) by up to ~0.12 -- a CPU emulation of the truncation
    gives 0.122 max, 0.016 mean -- and the per-pixel class (argmax of the two
    logits) agrees on >= 99.5% of pixels."""
    sw, fx = model
    inp, x = _input(sw, [int(fx["seed"])])
    m = NetModel(sw.nodes, sw.weights, 1, sw.inputs, sw.outputs, sw.states, sw.consts)
    out = m.step({inp: torch.from_numpy(x).cuda()})[sw.outputs[0]].cpu().numpy()[0]
    o = OracleNet(sw.nodes, sw.weights, sw.inputs, sw.states, sw.consts, tf32=m.tf32_convs())
    emu = o.step({inp: x}, {})[sw.outputs[0]][0]
    err_emu = float(np.max(np.abs(out - emu)))
    d = np.abs(out - fx["output"])
    agree = float(np.mean(np.argmax(out, -1) == np.argmax(fx["output"], -1)))
    assert err_emu <= 2e-2, err_emu
    assert float(d.max()) <= 0.3 and float(d.mean()) <= 0.03 and agree >= 0.995, (float(d.max()), float(d.mean()), agree)


def test_segm_r11_op_by_op(cuda_ok, model):
    """Every op of the shipped model on the default (TF32 tensor-core) path
    within its own bar, from the GPU's inputs to it."""
    sw, fx = model
    inp, x = _input(sw, [int(fx["seed"])])
    m = NetModel(sw.nodes, sw.weights, 1, sw.inputs, sw.outputs, sw.states, sw.consts)
    m.bufs[inp].copy_(torch.from_numpy(x))
    m.record()
    torch.cuda.synchronize()
    o = OracleNet(m.nodes, sw.weights, sw.inputs, sw.states, sw.consts)
    kinds = check_net_ops(m, o, sw.weights, "segm_r11")
    assert ("pw", "tf32") in kinds and ("dw", "ffma") in kinds, kinds


def test_segm_r11_pipelined_io(cuda_ok, model):
    """The shipped model through run_pipelined (its output is a channel alias
    of the last resize, resolved to that tensor) equals eager steps."""
    sw, fx = model
    inp, x = _input(sw, [5, 6, 7])
    out = sw.outputs[0]
    eager = NetModel(sw.nodes, sw.weights, 1, sw.inputs, sw.outputs, sw.states, sw.consts)
    want = [eager.step({inp: torch.from_numpy(x[k:k + 1]).cuda()})[out].cpu().numpy() for k in range(3)]
    pm = NetModel(sw.nodes, sw.weights, 1, sw.inputs, sw.outputs, sw.states, sw.consts)
    host_in = [{inp: torch.from_numpy(x[k:k + 1]).pin_memory()} for k in range(3)]
    host_out = [{out: torch.empty(want[0].shape).pin_memory()} for _ in range(3)]
    pm.run_pipelined(host_in, host_out)
    torch.cuda.synchronize()
    for k in range(3):
        assert np.array_equal(host_out[k][out].numpy(), want[k]), k


def test_synthetic_sw_graph_op_by_op(cuda_ok):
    """The synthetic .sw graph (SE gate FCs over n frames of 1x1, scalar /
    channel-vector operands, Mix with carried state, Avgpool, Chcopy, Act)
    on the GPU, every op of two steps within its own bar."""
    from tests.test_swfile import synthetic_sw
    sw = synthetic_sw()
    m = NetModel(sw.nodes, sw.weights, 3, sw.inputs, sw.outputs, sw.states, sw.consts)
    o = OracleNet(m.nodes, sw.weights, sw.inputs, sw.states, sw.consts)
    x = np.random.default_rng(2).uniform(-1, 1, (3, 8, 8, 8)).astype(np.float32)
    for t in range(2):
        m.bufs["t0"].copy_(torch.from_numpy(x))
        m.record()
        torch.cuda.synchronize()
        check_net_ops(m, o, sw.weights, f"synthetic step {t}")
        m.advance()
