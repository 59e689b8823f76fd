"""The recurrent matting network on CPU: its node list
against ai_engine's own layer list of the graph, and the oracle's
execution of it.  The GPU parity tests are in test_rvm_gpu.py."""
import json
import os

import numpy as np
import pytest

from ai_engine_b200 import rvm
from ai_engine_b200.net import infer_shapes

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def plan():
    return json.load(open(os.path.join(HERE, "golden", "rvm_plan_layers.json")))


def test_convs_match_the_reference_layer_list(plan):
    """Every conv of ai_engine's RVM graph (rvm_144x256.plan.json), in order:
    channels, kernel, stride, dilation, padding, depthwise, activation and
    output shape at 144x256."""
    want = [o for o in plan["ops"] if o["type"] == "Conv"]
    g = rvm.build_graph()
    sh = infer_shapes(g, rvm.inputs())
    got = [nd for nd in g if nd.kind == "conv"]
    assert len(got) == len(want) == 78
    for nd, o in zip(got, want):
        cv = nd.conv
        assert (cv.cin, cv.cout) == (o["cin"], o["cout"]), nd.out
        assert (cv.kh, cv.kw, cv.sh, cv.sw, cv.dil) == (*o["k"], *o["s"], o["dil"][0]), nd.out
        assert list(cv.pad) == o["pad"] and (cv.groups > 1) == o["dw"] and cv.act == o["act"], nd.out
        n_, c_, h_, w_ = o["out"][0]
        assert sh[nd.out] == (h_, w_, c_), nd.out


def test_glue_ops_match_the_reference_layer_list(plan):
    """Non-conv ops: the SE / LR-ASPP gates, pools, resizes and the ConvGRU
    updates appear with the reference's shapes.  The plan's Sub/Mul/Mul/Add
    chain per GRU is one Mix node here (ai_engine's fuse_mix rewrite), each
    residual Add is the project conv's epilogue, and Slice aliases are
    identities."""
    g = rvm.build_graph()
    sh = infer_shapes(g, rvm.inputs())
    ops = plan["ops"]
    kinds = [o["type"] for o in ops]
    assert kinds.count("gpool") == sum(nd.kind == "gpool" for nd in g) == 9
    assert kinds.count("AveragePool") == sum(nd.kind == "avgpool" for nd in g) == 3
    assert kinds.count("Resize") == sum(nd.kind == "resize" for nd in g) == 4
    assert kinds.count("Concat") == sum(nd.kind == "concat" for nd in g) == 16
    assert kinds.count("Split") + kinds.count("chcopy") // 2 == sum(nd.kind == "split" for nd in g) == 9
    # cvec-tensor multiplies: 8 SE gates + LR-ASPP
    gates = [o for o in ops if o["type"] == "binary" and o["mode"] == "mul" and len(o["in"]) == 2
             and isinstance(o["in"][0], list) and isinstance(o["in"][1], list)
             and (o["in"][0][2:] == [1, 1] or o["in"][1][2:] == [1, 1])]
    assert len(gates) == sum(nd.kind == "binary" and nd.bkind == "cvec_tensor" for nd in g) == 9
    # one Mix per GRU replaces `1 - z`, two multiplies and an add
    subs = [o for o in ops if o["type"] == "binary" and o["mode"] == "sub" and o.get("scalar") == 1.0]
    assert len(subs) == sum(nd.kind == "mix" for nd in g) == 4
    # residual adds between same-shape tensors, other than the GRU / output adds
    adds = [o for o in ops if o["type"] == "binary" and o["mode"] == "add"]
    assert len(adds) == 10 + 4 + 1
    assert sum(nd.kind == "conv" and nd.res is not None for nd in g) == 10
    # resize / concat / state shapes
    want_rs = [o["out"][0] for o in ops if o["type"] == "Resize"]
    got_rs = [sh[nd.out] for nd in g if nd.kind == "resize"]
    assert [(s[2], s[3], s[1]) for s in want_rs] == got_rs
    want_cat = [o["out"][0][1] for o in ops if o["type"] == "Concat"]
    got_cat = [sh[nd.out][2] for nd in g if nd.kind == "concat"]
    assert want_cat == got_cat
    ins = {i["name"]: i["shape"] for i in plan["inputs"]}
    for r in rvm.STATES:
        n_, c_, h_, w_ = ins[r]
        assert rvm.inputs()[r] == (h_, w_, c_)
    # input normalisation constants (plan __const_0 / __const_1)
    assert np.array_equal(rvm.consts()["mean"], np.array(plan["consts"]["__const_0"]["values"], np.float32))
    assert np.array_equal(rvm.consts()["inv_std"], np.array(plan["consts"]["__const_1"]["values"], np.float32))


def test_conv_flops_per_frame():
    assert rvm.conv_flops_per_frame() == 2250390528  # 2.25 GFLOP at 144x256


def test_oracle_net_batch_equals_streams():
    """Streams are independent: a 2-stream batch over two steps equals each
    stream run on its own (same oracle, recurrent state carried)."""
    from oracle.net import OracleNet
    h, w = 32, 48
    g = rvm.build_graph(h, w)
    o = OracleNet(g, rvm.init_weights(g), rvm.inputs(h, w), rvm.STATES, rvm.consts())
    x = rvm.synthetic_frames(2, 2, h, w, seed=3)
    st = o.zero_state(2)
    singles = [o.zero_state(1) for _ in range(2)]
    for t in range(2):
        out = o.step({"src": x[t]}, st)
        st = {k: out[v] for k, v in rvm.STATES.items()}
        for s in range(2):
            o1 = o.step({"src": x[t, s:s + 1]}, singles[s])
            singles[s] = {k: o1[v] for k, v in rvm.STATES.items()}
            for k in ("fgr", "pha", *rvm.STATES.values()):
                assert np.array_equal(out[k][s:s + 1], o1[k]), (t, s, k)
    assert 0.0 <= out["pha"].min() and out["pha"].max() <= 1.0
