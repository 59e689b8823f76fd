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
