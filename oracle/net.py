"""CPU oracle execution of a node graph with recurrent state -- TEST
INFRASTRUCTURE ONLY.

Runs the node lists of ``ai_engine_b200.net`` (convs plus Binary / Mix /
Gpool / Avgpool / Resize / Concat / Split / Chcopy) on the C restatement of
ai-cpu, the way ``ai_cpu::Model::infer`` runs a recurrent .sw graph
(crates/ai-cpu/src/model.rs:114-144, dispatch :393-550): logical channel
counts (no padding), every op's output materialised, state outputs of step
t fed back as step t + 1's state inputs.

``run_node`` runs one node on given input arrays, so a test can feed the
oracle the GPU's own inputs of each op and compare op by op.

``tf32`` names convs whose operands the oracle first truncates to TF32 (the
low 13 mantissa bits of every activation and weight cleared), the operand
format the GPU's tensor cores read fp32 data in.  With the GPU's own TF32
convs named, the oracle chain follows the GPU's arithmetic closely enough
for end-to-end comparisons of deep graphs at a tight bound.
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence, Tuple

import numpy as np

from . import Plan, avgpool, binary, channel_copy, gpool, lib, mix, resize_bilinear


def tf32_truncate(a: np.ndarray) -> np.ndarray:
    """fp32 -> the fp32 value of its TF32 truncation (10 mantissa bits kept)."""
    b = np.ascontiguousarray(a, np.float32).view(np.uint32) & np.uint32(0xFFFFE000)
    return b.view(np.float32)


def _shapes(nodes, inputs):
    sh = dict(inputs)
    for nd in nodes:
        s0 = sh[nd.ins[0]] if nd.ins else None
        k = nd.kind
        if k == "conv":
            cv = nd.conv
            ekh, ekw = cv.dil * (cv.kh - 1) + 1, cv.dil * (cv.kw - 1) + 1
            sh[nd.out] = ((s0[0] + cv.pad[0] + cv.pad[2] - ekh) // cv.sh + 1,
                          (s0[1] + cv.pad[1] + cv.pad[3] - ekw) // cv.sw + 1, cv.cout)
        elif k in ("binary", "mix"):
            sh[nd.out] = s0
        elif k == "gpool":
            sh[nd.out] = (1, 1, s0[2])
        elif k == "avgpool":
            kh, kw, sy, sx = nd.size
            sh[nd.out] = ((s0[0] - kh) // sy + 1, (s0[1] - kw) // sx + 1, s0[2])
        elif k == "resize":
            sh[nd.out] = (nd.size[0], nd.size[1], s0[2])
        elif k == "concat":
            sh[nd.out] = (s0[0], s0[1], sum(sh[i][2] for i in nd.ins))
        elif k == "split":
            for name, c in zip(nd.out, nd.parts):
                sh[name] = (s0[0], s0[1], c)
        elif k in ("chcopy", "view"):
            sh[nd.out] = (s0[0], s0[1], nd.parts[1])
    return sh


class OracleNet:
    def __init__(self, nodes: Sequence, weights: Dict[str, Tuple[np.ndarray, np.ndarray]],
                 inputs: Dict[str, Tuple[int, int, int]], states: Optional[Dict[str, str]] = None,
                 consts: Optional[Dict[str, np.ndarray]] = None, tf32=()):
        lib()
        self.tf32 = set(tf32)
        self.nodes = list(nodes)
        self.states = dict(states or {})
        self.inputs = dict(inputs)
        self.shapes = _shapes(self.nodes, inputs)
        self.consts = {k: np.ascontiguousarray(v, np.float32) for k, v in (consts or {}).items()}
        self.plans = {}
        for nd in self.nodes:
            if nd.kind == "conv":
                h, w, _ = self.shapes[nd.ins[0]]
                wt, b = weights[nd.out]
                if nd.out in self.tf32:
                    wt = tf32_truncate(wt)
                self.plans[nd.out] = Plan(nd.conv, h, w, wt, b, True, nd.res is not None)

    def run_node(self, nd, t: Dict[str, np.ndarray], threads: int = 1) -> Dict[str, np.ndarray]:
        """Run one node on the arrays in `t` (name -> [n, h, w, c]); returns its outputs."""
        k = nd.kind
        x = t[nd.ins[0]] if nd.ins else None
        n = x.shape[0]

        def new(name):
            h, w, c = self.shapes[name]
            return np.empty((n, h, w, c), np.float32)

        if k == "conv":
            res = t[nd.res] if nd.res is not None else None
            if nd.out in self.tf32:
                x = tf32_truncate(x)
            return {nd.out: self.plans[nd.out].run(x, res, threads)}
        if k == "binary":
            y = new(nd.out)
            if nd.bkind == "tensor":
                b = t[nd.ins[1]]
            elif nd.bkind in ("scalar", "scalar_first"):
                b = nd.scalar
            elif nd.bkind == "cvec":
                b = self.consts[nd.ins[1]]
            else:
                b = np.ascontiguousarray(t[nd.ins[1]].reshape(n, -1))
            binary(nd.op, np.ascontiguousarray(x), b, y, nd.act, kind=nd.bkind)
            return {nd.out: y}
        if k == "mix":
            y = new(nd.out)
            mix(*(np.ascontiguousarray(t[i]) for i in nd.ins), y)
            return {nd.out: y}
        if k == "gpool":
            return {nd.out: gpool(np.ascontiguousarray(x)).reshape(n, 1, 1, -1)}
        if k == "avgpool":
            return {nd.out: avgpool(x, nd.size[:2], nd.size[2:])}
        if k == "resize":
            return {nd.out: resize_bilinear(x, nd.size[0], nd.size[1])}
        if k == "concat":
            y = new(nd.out)
            coff = 0
            for part in nd.ins:
                c = t[part].shape[-1]
                channel_copy(np.ascontiguousarray(t[part]), (y, coff, c))
                coff += c
            return {nd.out: y}
        if k == "split":
            out, coff = {}, 0
            for name, c in zip(nd.out, nd.parts):
                out[name] = np.ascontiguousarray(x[..., coff:coff + c])
                coff += c
            return out
        if k == "view":
            coff, c = nd.parts
            return {nd.out: np.ascontiguousarray(x[..., coff:coff + c])}
        if k == "chcopy":
            coff, c = nd.parts
            y = new(nd.out)
            channel_copy((np.ascontiguousarray(x), coff, c), y, nd.act)
            return {nd.out: y}
        raise ValueError(f"unknown node kind {k}")

    def step(self, feeds: Dict[str, np.ndarray], state: Dict[str, np.ndarray], threads: int = 1,
             keep: bool = False) -> Dict[str, np.ndarray]:
        """One step over a batch: feeds (per-frame inputs) and state (the
        recurrent inputs); returns every tensor when keep, else the state
        outputs and the graph's other outputs."""
        t = {k: np.ascontiguousarray(v, np.float32) for k, v in feeds.items()}
        t.update({k: np.ascontiguousarray(v, np.float32) for k, v in state.items()})
        for nd in self.nodes:
            t.update(self.run_node(nd, t, threads))
        return t

    def zero_state(self, n: int) -> Dict[str, np.ndarray]:
        return {k: np.zeros((n, *self.shapes[k]), np.float32) for k in self.states}
