"""Reader of ai_engine's ``.sw`` model container.

The container (crates/ai-core/src/format/header.rs:1-14, parse_container
:56-90) is a 32-byte little-endian header -- magic ``SW1\\0``, version 1,
flags, blob alignment, JSON offset and length -- then the JSON graph
(``SwModel``, crates/ai-core/src/format/model.rs:217-260), zero padding to
the blob alignment, and the weight blob.  Every weight is a byte range
``{off, len}`` of the blob (``WRef``) in the converter's packed layouts
(crates/ai-core/src/pack.rs:68-184).

``load_sw`` turns a container into the node list, logical weights and I/O
names that ``ai_engine_b200.net.NetModel`` runs (ai-gpu-runtime's
``Model::load``, crates/ai-gpu-runtime/src/model.rs:56-120, lowering each
``SwOp``): convs (with concat-into-conv parts as a concat node), Binary
(tensor / scalar / cvec / cvec-tensor / pvec-tensor operands), Gpool,
Avgpool, Resize, Concat, Chcopy, Act, Mix, SeGate (as gpool + its FCs) and
channel aliases.  Ops outside the conv path (max pool, transpose,
relayout, tiled operands) raise ``NotImplementedError``.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from typing import Dict, List, Tuple

import numpy as np

from .conv import Conv2d
from .net import Node
from .pack import cg, unpack_weights_conv, unpack_weights_dw

MAGIC = b"SW1\x00"
HEADER_LEN = 32


class SwFormatError(ValueError):
    pass


@dataclass
class SwGraph:
    name: str
    nodes: List[Node]
    weights: Dict[str, Tuple[np.ndarray, np.ndarray]]
    consts: Dict[str, np.ndarray]
    inputs: Dict[str, Tuple[int, int, int]]
    outputs: List[str]
    states: Dict[str, str]
    tensor_names: Dict[str, str]   # node tensor name -> the model's tensor name


def parse_container(data: bytes) -> Tuple[dict, memoryview]:
    """Header check and split into (JSON graph, weight blob)."""
    if len(data) < HEADER_LEN:
        raise SwFormatError("truncated header")
    if data[:4] != MAGIC:
        raise SwFormatError("not a .sw container (bad magic)")
    version, _flags, align, json_off, json_len = struct.unpack_from("<IIIQQ", data, 4)
    if version != 1:
        raise SwFormatError(f"unsupported version {version}")
    if align == 0 or json_off + json_len > len(data):
        raise SwFormatError("truncated JSON")
    graph = json.loads(bytes(data[json_off:json_off + json_len]).decode("utf-8"))
    blob_off = -(-(json_off + json_len) // align) * align
    if blob_off > len(data):
        raise SwFormatError("truncated blob")
    return graph, memoryview(data)[blob_off:]


def _floats(blob: memoryview, wref: dict, dtype: str) -> np.ndarray:
    off, n = int(wref["off"]), int(wref["len"])
    if off + n > len(blob):
        raise SwFormatError(f"weight range {off}+{n} past the blob ({len(blob)} bytes)")
    dt = np.float16 if dtype == "f16" else np.float32
    return np.frombuffer(blob[off:off + n], dtype=dt).astype(np.float32)


def load_sw(data: bytes) -> SwGraph:
    g, blob = parse_container(data)
    dt_default = g.get("dt_default", "f32")
    dt_weights = g.get("dt_weights") or dt_default
    tensors = g["tensors"]
    names = {}
    for tid, t in enumerate(tensors):
        names[tid] = f"t{tid}"
    shapes = {tid: (t["h"], t["w"], t["c"]) for tid, t in enumerate(tensors)}
    nodes: List[Node] = []
    weights: Dict[str, Tuple[np.ndarray, np.ndarray]] = {}
    consts: Dict[str, np.ndarray] = {}

    def tn(tid):
        return names[int(tid)]

    def conv_weights(op, cin, cout, kh, kw, groups, wref, bref, kg_pad):
        if groups == 1:
            wp = _floats(blob, wref, dt_weights)
            w = unpack_weights_conv(wp, cout, cin, kh, kw, kg_pad)
        else:
            wp = _floats(blob, wref, dt_default)
            w = unpack_weights_dw(wp, cout, kh, kw)
        b = _floats(blob, bref, dt_default)[:cout]
        return w, np.ascontiguousarray(b)

    for i, op in enumerate(g["ops"]):
        k = op["kind"]
        if k == "conv":
            out = tn(op["out"])
            src = tn(op["in"])
            if op.get("srcs"):
                cat = f"{out}.srcs"
                nodes.append(Node("concat", cat, tuple(tn(p["in"]) for p in op["srcs"])))
                src = cat
            groups = int(op["groups"])
            cv = Conv2d(int(op["cin"]), int(op["cout"]), int(op["kh"]), int(op["kw"]), int(op["sh"]), int(op["sw"]),
                        tuple(int(p) for p in op["pad"]), int(op.get("d", 1)), groups, op["act"])
            weights[out] = conv_weights(op, cv.cin, cv.cout, cv.kh, cv.kw, groups, op["w"], op["b"],
                                        int(op.get("kg_pad", 0)))
            res = op.get("res")
            nodes.append(Node("conv", out, (src,), conv=cv, res=None if res is None else tn(res)))
        elif k == "binary":
            b = op["b"]
            (bk, bv), = b.items()
            a = tn(op["a"])
            if bk == "tensor":
                nodes.append(Node("binary", tn(op["out"]), (a, tn(bv["tid"])), op=op["op"], act=op["act"]))
            elif bk == "scalar":
                nodes.append(Node("binary", tn(op["out"]), (a,), op=op["op"], act=op["act"],
                                  bkind="scalar_first" if bv.get("first") else "scalar", scalar=float(bv["v"])))
            elif bk == "cvec":
                cname = f"const{i}"
                consts[cname] = _floats(blob, bv["w"], dt_default)[:int(bv["c"])]
                nodes.append(Node("binary", tn(op["out"]), (a, cname), op=op["op"], act=op["act"], bkind="cvec"))
            elif bk in ("cvectensor", "pvectensor"):
                nodes.append(Node("binary", tn(op["out"]), (a, tn(bv["tid"])), op=op["op"], act=op["act"],
                                  bkind="cvec_tensor" if bk == "cvectensor" else "pvec_tensor"))
            else:
                raise NotImplementedError(f"binary operand {bk}")
        elif k == "gpool":
            nodes.append(Node("gpool", tn(op["out"]), (tn(op["in"]),)))
        elif k == "avgpool":
            if any(op["pad"]):
                raise NotImplementedError("padded average pool")
            nodes.append(Node("avgpool", tn(op["out"]), (tn(op["in"]),), size=(op["kh"], op["kw"], op["sh"], op["sw"])))
        elif k == "resize":
            if op.get("mode", "half_pixel") != "half_pixel" or op.get("srcs"):
                raise NotImplementedError("resize other than plain half_pixel")
            nodes.append(Node("resize", tn(op["out"]), (tn(op["in"]),), size=(int(op["oh"]), int(op["ow"]))))
        elif k == "concat":
            nodes.append(Node("concat", tn(op["out"]), tuple(tn(p["in"]) for p in op["parts"])))
        elif k == "chcopy":
            nodes.append(Node("chcopy", tn(op["out"]), (tn(op["in"]),), parts=(int(op["src_c"]), int(op["n"]))))
        elif k == "act":
            c = shapes[int(op["in"])][2]
            nodes.append(Node("chcopy", tn(op["out"]), (tn(op["in"]),), act=op["act"], parts=(0, c)))
        elif k == "mix":
            nodes.append(Node("mix", tn(op["out"]), (tn(op["z"]), tn(op["a"]), tn(op["b"]))))
        elif k == "se_gate":
            src, out = tn(op["in"]), tn(op["out"])
            cin = shapes[int(op["in"])][2]
            nodes.append(Node("gpool", f"{out}.pool", (src,)))
            cm = int(op["c_mid"])
            fc1 = f"{out}.fc1" if op.get("fc2") else out
            w1 = unpack_weights_conv(_floats(blob, op["w1"], dt_weights), cm, cin, 1, 1, -(-cg(cin) // 4) * 4)
            weights[fc1] = (w1, _floats(blob, op["b1"], dt_default)[:cm])
            nodes.append(Node("conv", fc1, (f"{out}.pool",), conv=Conv2d.pointwise(cin, cm, op["act1"])))
            if op.get("fc2"):
                f2 = op["fc2"]
                co = int(f2["c_out"])
                w2 = unpack_weights_conv(_floats(blob, f2["w"], dt_weights), co, cm, 1, 1, -(-cg(cm) // 4) * 4)
                weights[out] = (w2, _floats(blob, f2["b"], dt_default)[:co])
                nodes.append(Node("conv", out, (fc1,), conv=Conv2d.pointwise(cm, co, f2["act"])))
        else:
            raise NotImplementedError(f"op kind {k} is outside the conv path")
    # channel aliases (SwTensor.alias, a channel-group offset into another tensor)
    alias_nodes = []
    for tid, t in enumerate(tensors):
        al = t.get("alias")
        if al:
            alias_nodes.append((tid, Node("view", tn(tid), (tn(al["of"]),), parts=(4 * int(al["cg_off"]), t["c"]))))
    for tid, nd in alias_nodes:
        # place each view right after its source's producer
        src = nd.ins[0]
        pos = next((j for j, x in enumerate(nodes) if x.out == src), -1)
        nodes.insert(pos + 1, nd)
    inputs = {tn(t): shapes[int(t)] for t in g["inputs"]}
    states = {}
    for st in g.get("states", []):  # SwState {input, output}, model.rs:50-55
        states[tn(st["input"])] = tn(st["output"])
        inputs[tn(st["input"])] = shapes[int(st["input"])]
    return SwGraph(g.get("name", ""), nodes, weights, consts, inputs, [tn(t) for t in g["outputs"]], states,
                   {names[tid]: t["name"] for tid, t in enumerate(tensors)})
