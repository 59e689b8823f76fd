"""The .sw container reader on ai_engine's shipped segmentation model
(web/models/segm_r11_160x288.sw, committed as tests/golden/segm_r11.npz by
tests/golden/make_segm_r11.py), on CPU."""
import collections
import os
import struct

import numpy as np
import pytest

import oracle
from ai_engine_b200 import pack
from ai_engine_b200.swfile import SwFormatError, load_sw, parse_container
from oracle.net import OracleNet

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def fixture():
    return np.load(os.path.join(HERE, "golden", "segm_r11.npz"))


def test_container_header(fixture):
    data = fixture["sw"].tobytes()
    g, blob = parse_container(data)
    assert g["name"] == "segm-r11" and len(g["ops"]) == 44 and len(g["tensors"]) == 46
    # header.rs:1-14: magic, version 1, blob aligned to 256 after the JSON
    magic, version, flags, align, json_off, json_len = struct.unpack_from("<4sIIIQQ", data, 0)
    assert (magic, version, flags, align, json_off) == (b"SW1\x00", 1, 0, 256, 32)
    assert len(blob) == len(data) - (-(-(json_off + json_len) // align) * align)
    with pytest.raises(SwFormatError):
        parse_container(b"XX1\x00" + data[4:])
    with pytest.raises(SwFormatError):
        parse_container(data[:16])
    with pytest.raises(SwFormatError):
        parse_container(data[:4] + struct.pack("<I", 2) + data[8:])


def test_graph_lowering(fixture):
    sw = load_sw(fixture["sw"].tobytes())
    kinds = collections.Counter(nd.kind for nd in sw.nodes)
    # 36 convs (one with concat-into-conv parts), 4 resizes, 2 binaries,
    # a gpool, a concat, and the 2-channel output alias
    assert kinds == {"conv": 36, "resize": 4, "binary": 2, "gpool": 1, "concat": 2, "view": 1}
    assert sw.inputs == {"t0": (160, 288, 3)} and sw.outputs == ["t45"] and not sw.states
    assert sw.tensor_names["t0"] == "input_1" and sw.tensor_names["t45"] == "segment"
    gate = next(nd for nd in sw.nodes if nd.kind == "binary" and nd.bkind == "cvec_tensor")
    assert gate.op == "mul"


def test_weights_repack_to_the_blob(fixture):
    """Unpacking the blob's packed weights and packing them again with the
    converter's layouts (pack.rs:68-122, kg_align 4) gives the same bytes."""
    data = fixture["sw"].tobytes()
    g, blob = parse_container(data)
    sw = load_sw(data)
    convs = [o for o in g["ops"] if o["kind"] == "conv"]
    assert len(convs) == 36
    for op in convs:
        w, b = sw.weights[f"t{op['out']}"]
        raw = np.frombuffer(blob[op["w"]["off"]:op["w"]["off"] + op["w"]["len"]], np.float32)
        if op["groups"] == 1:
            packed, kg = pack.pack_weights_conv(w, op["cout"], op["cin"], op["kh"], op["kw"], 4)
            assert kg == op["kg_pad"]
        else:
            packed = pack.pack_weights_dw(w, op["cout"], op["kh"], op["kw"])
        assert np.array_equal(packed, raw), op["out"]
        rb = np.frombuffer(blob[op["b"]["off"]:op["b"]["off"] + op["b"]["len"]], np.float32)
        assert np.array_equal(pack.pack_bias(b, op["cout"]), rb)


def test_oracle_matches_golden(fixture):
    """The ai-cpu restatement on the graph-exec test input XorShift32(77)
    (crates/ai-gpu-runtime/tests/graph_exec.rs:36-39) reproduces the
    committed output bit for bit."""
    sw = load_sw(fixture["sw"].tobytes())
    (inp, (h, w, c)), = sw.inputs.items()
    x = oracle.XorShift32(int(fixture["seed"])).vec_f32(h * w * c).reshape(1, h, w, c)
    t = OracleNet(sw.nodes, sw.weights, sw.inputs, sw.states, sw.consts).step({inp: x}, {})
    assert np.array_equal(t[sw.outputs[0]][0], fixture["output"])


def _container(graph: dict, blob: bytes) -> bytes:
    """A .sw container (crates/ai-core/src/format/header.rs:1-14 layout)."""
    import json as _json
    js = _json.dumps(graph).encode()
    off = 32
    blob_off = -(-(off + len(js)) // 256) * 256
    hdr = b"SW1\x00" + struct.pack("<IIIQQ", 1, 0, 256, off, len(js))
    return hdr + js + b"\x00" * (blob_off - off - len(js)) + blob


def synthetic_sw():
    """A small recurrent .sw graph with the op kinds segm_r11 does not use:
    SE gate (two FCs), scalar-first and channel-vector Binary operands, Act,
    Chcopy, Mix, Avgpool and a state pair."""
    rng = np.random.default_rng(0)
    parts, offs = [], {}

    def put(name, arr):
        a = np.ascontiguousarray(arr, np.float32).reshape(-1)
        offs[name] = {"off": sum(len(p) for p in parts), "len": a.nbytes}
        parts.append(a.tobytes())

    c = 8
    w_pw, kg = pack.pack_weights_conv(rng.standard_normal(c * c).astype(np.float32), c, c, 1, 1, 4)
    put("w", w_pw); put("b", pack.pack_bias(rng.uniform(-0.1, 0.1, c), c))
    w1, _ = pack.pack_weights_conv(rng.standard_normal(4 * c).astype(np.float32), 4, c, 1, 1, 4)
    put("w1", w1); put("b1", pack.pack_bias(np.zeros(4), 4))
    w2, _ = pack.pack_weights_conv(rng.standard_normal(4 * c).astype(np.float32), c, 4, 1, 1, 4)
    put("w2", w2); put("b2", pack.pack_bias(np.zeros(c), c))
    put("cv", pack.pack_nhwc(rng.uniform(0.5, 1.5, c)))
    T = lambda name, h, w, ch: {"name": name, "h": h, "w": w, "c": ch, "dt": "f32", "alias": None, "last_use": 0}
    tensors = [T("x", 8, 8, c), T("h", 8, 8, c), T("y", 8, 8, c), T("g", 1, 1, c), T("ys", 8, 8, c),
               T("z", 8, 8, c), T("zz", 8, 8, c), T("h_out", 8, 8, c), T("p", 4, 4, c), T("q", 4, 4, 4),
               T("r", 4, 4, 4)]
    ops = [
        {"kind": "conv", "in": 0, "out": 2, "res": None, "cin": c, "cout": c, "kh": 1, "kw": 1, "sh": 1, "sw": 1,
         "pad": [0, 0, 0, 0], "d": 1, "groups": 1, "act": "relu", "w": offs["w"], "b": offs["b"], "kg_pad": kg},
        {"kind": "se_gate", "in": 2, "out": 3, "c_mid": 4, "act1": "relu", "w1": offs["w1"], "b1": offs["b1"],
         "fc2": {"c_out": c, "act": "hardsigmoid", "w": offs["w2"], "b": offs["b2"]}},
        {"kind": "binary", "a": 2, "b": {"cvectensor": {"tid": 3}}, "out": 4, "op": "mul", "act": "none"},
        {"kind": "binary", "a": 4, "b": {"scalar": {"v": 1.0, "first": True}}, "out": 5, "op": "sub", "act": "none"},
        {"kind": "binary", "a": 5, "b": {"cvec": {"w": offs["cv"], "c": c}}, "out": 6, "op": "mul",
         "act": "sigmoid"},
        {"kind": "mix", "z": 6, "a": 1, "b": 4, "out": 7},
        {"kind": "avgpool", "in": 7, "out": 8, "kh": 2, "kw": 2, "sh": 2, "sw": 2, "pad": [0, 0, 0, 0]},
        {"kind": "chcopy", "in": 8, "out": 9, "src_c": 2, "n": 4},
        {"kind": "act", "in": 9, "out": 10, "act": "tanh"},
    ]
    graph = {"name": "synthetic", "size": {"h": 8, "w": 8}, "dt_default": "f32", "tensors": tensors,
             "inputs": [0, 1], "outputs": [10, 7], "states": [{"input": 1, "output": 7}], "ops": ops}
    return load_sw(_container(graph, b"".join(parts)))


def test_synthetic_container_every_op_kind():
    """The reader lowers every op kind of synthetic_sw() and the oracle runs
    two steps, the state feeding back."""
    rng = np.random.default_rng(1)
    c = 8
    sw = synthetic_sw()
    kinds = collections.Counter(nd.kind for nd in sw.nodes)
    assert kinds == {"conv": 3, "gpool": 1, "binary": 3, "mix": 1, "avgpool": 1, "chcopy": 2}
    assert sw.states == {"t1": "t7"} and sw.inputs == {"t0": (8, 8, c), "t1": (8, 8, c)}
    assert sw.outputs == ["t10", "t7"]
    o = OracleNet(sw.nodes, sw.weights, sw.inputs, sw.states, sw.consts)
    x = rng.uniform(-1, 1, (2, 8, 8, c)).astype(np.float32)
    st = o.zero_state(2)
    out1 = o.step({"t0": x}, st)
    out2 = o.step({"t0": x}, {"t1": out1["t7"]})
    # step 1 from zero state: h' = 0 + z (y_se - 0) = z * y_se
    assert np.allclose(out1["t7"], out1["t6"] * out1["t4"], rtol=1e-6, atol=1e-7)
    # step 2 mixes the carried state: h' = h + z (y_se - h)
    h = out1["t7"]
    assert np.allclose(out2["t7"], h + out2["t6"] * (out2["t4"] - h), rtol=1e-5, atol=1e-6)
    assert out2["t10"].shape == (2, 4, 4, 4) and np.all(np.abs(out2["t10"]) <= 1.0)
