"""CPU oracle execution of a conv graph -- TEST INFRASTRUCTURE ONLY.

Runs the same op list as ``ai_engine_b200.graph.Model`` frame by frame
through the ai-cpu restatement, the way ``ai_cpu::Model::infer`` runs a
.sw graph (crates/ai-cpu/src/model.rs:114-144, dispatch :393-550).  Used
for whole-network parity and as the timed CPU baseline, in ai-cpu's two
threading modes:

* row bands (model.rs:421-441): one frame at a time, each conv's output
  rows split across `threads`;
* throughput: one frame per thread, `threads` frames in flight.

ctypes releases the GIL while the C kernels run, so Python threads give
real parallelism here.
"""
from __future__ import annotations

import concurrent.futures as cf
from typing import Dict, Tuple

import numpy as np

from . import Plan, lib, resize_bilinear
from .net import tf32_truncate


def _shapes(graph, in_hwc):
    shapes = {"input": tuple(in_hwc)}
    for op in graph:
        h, w, c = shapes[op[2]]
        if op[0] == "conv":
            cv = op[3]
            ekh, ekw = cv.dil * (cv.kh - 1) + 1, cv.dil * (cv.kw - 1) + 1
            shapes[op[1]] = ((h + cv.pad[0] + cv.pad[2] - ekh) // cv.sh + 1,
                             (w + cv.pad[1] + cv.pad[3] - ekw) // cv.sw + 1, cv.cout)
        else:
            shapes[op[1]] = (op[3][0], op[3][1], c)
    return shapes


class OracleModel:
    """``tf32`` names convs whose operands are first truncated to TF32 (the
    low 13 mantissa bits of every activation and weight cleared), the
    operand format the GPU's tensor cores read fp32 data in; naming the
    GPU's own TF32 convs makes the chain follow the GPU's arithmetic."""

    def __init__(self, graph, weights: Dict[str, Tuple[np.ndarray, np.ndarray]], in_hwc, tf32=()):
        lib()
        self.graph = list(graph)
        self.shapes = _shapes(self.graph, in_hwc)
        self.tf32 = set(tf32)
        self.plans = {}
        for op in self.graph:
            if op[0] == "conv":
                h, w, _ = self.shapes[op[2]]
                wt, b = weights[op[1]]
                if op[1] in self.tf32:
                    wt = tf32_truncate(wt)
                self.plans[op[1]] = Plan(op[3], h, w, wt, b, True, op[4] is not None)
        self.output = self.graph[-1][1]

    def infer_frame(self, x: np.ndarray, threads: int = 1, keep: bool = False):
        """x: [h, w, c] one frame.  Returns the output (and every tensor when keep)."""
        t = {"input": np.ascontiguousarray(x, np.float32)}
        for op in self.graph:
            kind, out, src, res = op[0], op[1], op[2], op[4]
            oh, ow, oc = self.shapes[out]
            if kind == "conv":
                y = np.empty((oh, ow, oc), np.float32)
                xin = tf32_truncate(t[src]) if out in self.tf32 else t[src]
                self.plans[out].run_frame(xin, y, t[res] if res else None, threads=threads)
            else:
                y = resize_bilinear(t[src][None], oh, ow)[0]
                if res:
                    y = y + t[res]
            t[out] = y
        return (t[self.output], t) if keep else t[self.output]

    def run_batch(self, x: np.ndarray, threads: int = 1, mode: str = "throughput") -> np.ndarray:
        n = x.shape[0]
        oh, ow, oc = self.shapes[self.output]
        out = np.empty((n, oh, ow, oc), np.float32)
        if mode == "bands" or threads <= 1:
            for f in range(n):
                out[f] = self.infer_frame(x[f], threads=threads)
            return out
        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            futs = {ex.submit(self.infer_frame, x[f], 1): f for f in range(n)}
            for fu in cf.as_completed(futs):
                out[futs[fu]] = fu.result()
        return out
