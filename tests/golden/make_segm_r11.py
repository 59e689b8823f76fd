"""Generate tests/golden/segm_r11.npz -- ai_engine's shipped segmentation
model and the ai-cpu restatement's output on the reference's own test input.

The model is ``web/models/segm_r11_160x288.sw`` of the ai_engine tree (a
.sw container: header, JSON graph of 44 ops, f32 weight blob).  The input is
ai-gpu-runtime's graph-exec test input, XorShift32(77) over the 160x288x3
frame (crates/ai-gpu-runtime/tests/graph_exec.rs:36-39); the output is the
CPU oracle's run of the graph (OracleNet over load_sw's node list), which
tests/test_swfile.py pins on CPU and the GPU path is compared against
within the reference's own 2e-3 bar (graph_exec.rs:58-71).

    python tests/golden/make_segm_r11.py <ai_engine checkout>
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from ai_engine_b200.swfile import load_sw  # noqa: E402
from oracle.net import OracleNet  # noqa: E402

SEED = 77


def main(src_root: str) -> None:
    data = open(os.path.join(src_root, "web", "models", "segm_r11_160x288.sw"), "rb").read()
    sw = load_sw(data)
    (inp, (h, w, c)), = sw.inputs.items()
    x = oracle.XorShift32(SEED).vec_f32(h * w * c).reshape(1, h, w, c)
    t = OracleNet(sw.nodes, sw.weights, sw.inputs, sw.states, sw.consts).step({inp: x}, {})
    out = t[sw.outputs[0]][0]
    np.savez_compressed(os.path.join(HERE, "segm_r11.npz"), sw=np.frombuffer(data, np.uint8), seed=SEED,
                        output=out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_segm_r11.py <ai_engine checkout>")
    main(sys.argv[1])
