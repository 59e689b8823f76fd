"""Generate tests/golden/rvm_plan_layers.json -- the op list of ai_engine's
recurrent matting graph, the only form in which ai_engine ships it
(web/compare/assets/rvm_144x256.plan.json in the ai_engine tree; its
weights are absent).

For every op the fixture keeps its kind and shapes only: per Conv the
channels, kernel, stride, dilation, padding, depthwise flag and activation;
per other op its input / output shapes and mode.  tests/test_rvm.py checks
ai_engine_b200.rvm.build_graph() against it layer by layer.

    python tests/golden/make_rvm_layers.py <path to the ai_engine checkout>
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(root: str) -> None:
    plan = json.load(open(os.path.join(root, "web", "compare", "assets", "rvm_144x256.plan.json")))
    tensors = plan["tensors"]
    ops = []
    for o in plan["ops"]:
        shp = lambda names: [tensors[x]["shape"] if x in tensors else x for x in names]  # noqa: E731
        rec = {"type": o["type"], "in": shp(o["in"]), "out": shp(o["out"])}
        if o["type"] == "Conv":
            rec.update(cin=o["cout"] if o["dw"] else o["cin"], cout=o["cout"], k=o["k"], s=o["s"], dil=o["dil"],
                       pad=o["pad"], dw=o["dw"], act=o["act"])
        else:
            rec.update({k: v for k, v in o.items() if k not in ("type", "in", "out")})
        ops.append(rec)
    out = {"source": "web/compare/assets/rvm_144x256.plan.json", "inputs": plan["inputs"],
           "outputs": plan["outputs"], "consts": plan["consts"], "ops": ops}
    with open(os.path.join(HERE, "rvm_plan_layers.json"), "w") as f:
        json.dump(out, f, indent=0)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_rvm_layers.py <ai_engine checkout>")
    main(sys.argv[1])
