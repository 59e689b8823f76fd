"""Minimal graph executor over the conv path.

Plays the part of ai-gpu-runtime's ``Model`` (crates/ai-gpu-runtime/src/
model.rs:56-426) for graphs made of convs and bilinear resizes:

* ``load``: infer shapes, lower every conv (``ConvPlan`` = lower_op's Conv
  arm) and pack its weights, allocate every activation buffer once
  (no allocation per frame, model.rs:1-5);
* ``infer``: record all dispatches on one CUDA stream (kernel::record,
  crates/ai-gpu/src/kernel.rs:181-191), optionally replayed from a
  captured CUDA graph instead of being re-issued from Python.

A graph is a list of ops; tensors are named, ``"input"`` is the batch.
  ("conv",   out, src, Conv2d, res_or_None)
  ("resize", out, src, (oh, ow), add_or_None)
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .conv import Conv2d, ConvPlan, input_u8, resize_bilinear, run_dw_pw, run_mbconv, run_stem_pw


@dataclass
class OpRecord:
    kind: str
    out: str
    src: str
    conv: Optional[Conv2d] = None
    res: Optional[str] = None
    size: Optional[Tuple[int, int]] = None
    plan: Optional[ConvPlan] = None
    head: Optional[ConvPlan] = None   # kind "dwpw": the fused 1x1 (cout <= 4) after the depthwise plan
    up: Optional[str] = None          # kind "dwpw": source whose exact-2x resize is added to the depthwise input
    blk: Optional[Tuple[ConvPlan, ConvPlan, ConvPlan]] = None  # kind "mb": expand, depthwise, project plans
    out2: Optional[str] = None        # kind "stempw": the fused 1x1's output (its plan in `head`)
    members: Tuple[str, ...] = ()     # fused kinds: the graph's conv (and resize) names this launch runs


def infer_shapes(graph: Sequence[tuple], in_hwc: Tuple[int, int, int]) -> Dict[str, Tuple[int, int, int]]:
    shapes = {"input": tuple(in_hwc)}
    for op in graph:
        kind, out, src = op[0], op[1], op[2]
        h, w, c = shapes[src]
        if kind == "conv":
            cv: Conv2d = op[3]
            if cv.cin != c:
                raise ValueError(f"{out}: conv expects {cv.cin} channels, {src} has {c}")
            oh, ow = cv.out_hw(h, w)
            shapes[out] = (oh, ow, cv.cout)
            if op[4] is not None and shapes[op[4]] != shapes[out]:
                raise ValueError(f"{out}: residual {op[4]} shape {shapes[op[4]]} != {shapes[out]}")
        elif kind == "resize":
            oh, ow = op[3]
            shapes[out] = (oh, ow, c)
            if op[4] is not None and shapes[op[4]] != shapes[out]:
                raise ValueError(f"{out}: add operand shape mismatch")
        else:
            raise ValueError(f"unknown op kind {kind}")
    return shapes


class Model:
    """Load-time lowering + per-batch execution of a conv graph on one GPU."""

    def __init__(self, graph: Sequence[tuple], weights: Dict[str, Tuple[np.ndarray, np.ndarray]], n: int,
                 in_hwc: Tuple[int, int, int], *, math: str = "auto", fuse: bool = False, fuse_heads: bool = True,
                 fuse_tail: bool = True, fuse_blocks: bool = True, fuse_stem: bool = True, input_u8: bool = False,
                 device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.n = n
        self.graph = list(graph)
        self.shapes = infer_shapes(self.graph, in_hwc)
        self.output = self.graph[-1][1]
        self.ops: List[OpRecord] = []
        self.bufs: Dict[str, torch.Tensor] = {}
        # Resize -> Conv(res) fusion (fuse=True): a bilinear resize whose
        # output only feeds the next conv's residual is folded into that
        # conv's epilogue (the residual is sampled from the low-resolution
        # tensor directly).  Off by default: on B200 the per-row bilinear
        # gathers make the issue-bound GEMM epilogue slower than a separate
        # resize pass for the FPN's 32-64 channel laterals.
        uses: Dict[str, int] = {}
        for op in self.graph:
            for t in (op[2], op[4]):
                if t is not None:
                    uses[t] = uses.get(t, 0) + 1
        fused_resize: Dict[str, str] = {}  # resize output -> its source
        if fuse:
            for op in self.graph:
                if op[0] == "resize" and op[4] is None and uses.get(op[1], 0) == 1 and op[1] != self.output:
                    fused_resize[op[1]] = op[2]
        # Depthwise -> 1x1 head fusion (fuse_heads): a depthwise conv whose
        # output only feeds a 1x1 conv with cout <= 4 runs with it as one
        # launch (aie_conv_run_dw_pw) when both plans qualify.
        head_of: Dict[str, tuple] = {}  # depthwise output name -> the consuming 1x1 op
        if fuse_heads and math != "fp32_strict":
            for op in self.graph:
                if op[0] != "conv" or op[4] is not None:
                    continue
                cv: Conv2d = op[3]
                prev = next((p for p in self.graph if p[1] == op[2]), None)
                if (cv.kh == 1 and cv.kw == 1 and cv.sh == 1 and cv.sw == 1 and cv.cout <= 4 and cv.pad == (0, 0, 0, 0)
                        and prev is not None and prev[0] == "conv" and prev[3].is_depthwise() and prev[4] is None
                        and uses.get(prev[1], 0) == 1 and prev[1] != self.output and prev[3].cout <= 32
                        and prev[3].cout % 4 == 0):
                    head_of[prev[1]] = op
        # the fused head's plans, made up front: a head whose plans do not
        # qualify runs as its two convs (and keeps its producers as they are)
        head_plans: Dict[str, Tuple[ConvPlan, ConvPlan]] = {}
        for dw_out, hop in list(head_of.items()):
            dop = next(p for p in self.graph if p[1] == dw_out)
            h, w, _ = self.shapes[dop[2]]
            dplan = ConvPlan(dop[3], n, h, w, math=math, device=self.device).load_weights(*weights[dw_out])
            oh, ow, _ = self.shapes[dw_out]
            hplan = ConvPlan(hop[3], n, oh, ow, math=math, device=self.device).load_weights(*weights[hop[1]])
            if dplan.kernel == "dw" and hplan.kernel == "pw_dot" and dplan.math != "fp32_strict":
                head_plans[dw_out] = (dplan, hplan)
            else:
                del head_of[dw_out]
        fused_heads = set(op[1] for op in head_of.values())
        # Feature-pyramid tail (with the head fusion): the head's depthwise
        # input is a conv whose residual is an exact-2x resize used nowhere
        # else.  The conv then runs without its residual and the fused head
        # adds the up-sampled source in its staged input tile
        # (aie_conv_run_dw_pw_up2): neither the resize's output nor the sum
        # is written.
        tail_up: Dict[str, str] = {}       # lateral conv output -> resize source
        dropped_resize: set = set()
        for dw_out in (head_of if fuse_tail else {}):
            dop = next(p for p in self.graph if p[1] == dw_out)
            lat = next((p for p in self.graph if p[1] == dop[2]), None)
            if lat is None or lat[0] != "conv" or lat[4] is None or uses.get(lat[1], 0) != 1 or lat[1] == self.output:
                continue
            rz = next((p for p in self.graph if p[1] == lat[4]), None)
            if rz is None or rz[0] != "resize" or rz[4] is not None or uses.get(rz[1], 0) != 1 or rz[1] == self.output:
                continue
            sh_, sw_, sc_ = self.shapes[rz[2]]
            if tuple(rz[3]) != (2 * sh_, 2 * sw_) or self.shapes[lat[1]] != (2 * sh_, 2 * sw_, sc_):
                continue
            tail_up[lat[1]] = rz[2]
            dropped_resize.add(rz[1])
            fused_resize.pop(rz[1], None)  # the head takes it instead of the conv's epilogue
        # Inverted-bottleneck blocks on small frames (fuse_blocks): a 1x1
        # expand, a depthwise 3x3 (stride 1, pad 1) and a 1x1 project whose
        # intermediates feed nothing else, over frames up to 10 x 18, run as
        # one launch (aie_conv_run_mbconv) when the 1x1 plans resolve to TF32.
        block_of: Dict[str, tuple] = {}  # project output -> (expand op, depthwise op, project op, plans)
        block_inner: set = set()        # expand / depthwise outputs recorded with their block
        if fuse_blocks and math not in ("fp32_strict", "ffma"):
            def is_pw(cv):
                return cv.kh == 1 and cv.kw == 1 and cv.sh == 1 and cv.sw == 1 and cv.groups == 1 and \
                    tuple(cv.pad) == (0, 0, 0, 0)
            for op in self.graph:
                if op[0] != "conv" or not is_pw(op[3]) or op[3].cout > 128:
                    continue
                dop = next((p for p in self.graph if p[1] == op[2]), None)
                if dop is None or dop[0] != "conv" or dop[4] is not None or dop[1] in head_of:
                    continue
                dcv = dop[3]
                if not (dcv.is_depthwise() and dcv.kh == 3 and dcv.kw == 3 and dcv.sh == 1 and dcv.sw == 1
                        and dcv.dil == 1 and tuple(dcv.pad) == (1, 1, 1, 1)):
                    continue
                eop = next((p for p in self.graph if p[1] == dop[2]), None)
                if eop is None or eop[0] != "conv" or eop[4] is not None or not is_pw(eop[3]):
                    continue
                if uses.get(eop[1], 0) != 1 or uses.get(dop[1], 0) != 1 or self.output in (eop[1], dop[1]):
                    continue
                h, w, c = self.shapes[eop[2]]
                if h > 10 or w > 18 or c % 32:
                    continue
                ex = ConvPlan(eop[3], n, h, w, math=math, device=self.device).load_weights(*weights[eop[1]])
                dw = ConvPlan(dcv, n, h, w, math=math, device=self.device).load_weights(*weights[dop[1]])
                pj = ConvPlan(op[3], n, h, w, has_res=op[4] is not None, math=math,
                              device=self.device).load_weights(*weights[op[1]])
                if ex.math != "tf32" or pj.math != "tf32" or dw.kernel != "dw" or dw.math == "fp32_strict":
                    continue
                block_of[op[1]] = (eop, dop, op, (ex, dw, pj))
                block_inner.update((eop[1], dop[1]))
            # a 1x1 expand read only by a 1x1 project (no depthwise between
            # them: a wide head conv and the pyramid lateral on it) runs the
            # same way with the expanded tensor kept on chip
            for op in self.graph:
                if op[0] != "conv" or not is_pw(op[3]) or op[3].cout > 128 or op[1] in block_of:
                    continue
                if op[1] in tail_up or (op[4] is not None and (op[4] in fused_resize or op[4] in dropped_resize)):
                    continue  # its residual is an up-sampling folded elsewhere
                eop = next((p for p in self.graph if p[1] == op[2]), None)
                if eop is None or eop[0] != "conv" or eop[4] is not None or not is_pw(eop[3]):
                    continue
                if eop[1] in block_of or eop[1] in block_inner or eop[1] in head_of:
                    continue
                if uses.get(eop[1], 0) != 1 or self.output == eop[1]:
                    continue
                h, w, c = self.shapes[eop[2]]
                if h > 10 or w > 18 or c % 32:
                    continue
                ex = ConvPlan(eop[3], n, h, w, math=math, device=self.device).load_weights(*weights[eop[1]])
                pj = ConvPlan(op[3], n, h, w, has_res=op[4] is not None, math=math,
                              device=self.device).load_weights(*weights[op[1]])
                if ex.math != "tf32" or pj.math != "tf32":
                    continue
                block_of[op[1]] = (eop, None, op, (ex, None, pj))
                block_inner.add(eop[1])
        # input_u8: the batch arrives as u8 RGB frames ("input_u8", 3 bytes per
        # pixel); the first op normalises them into the f32 "input" (u8 / 255)
        self.input_u8 = input_u8
        self.input_name = "input_u8" if input_u8 else "input"
        with torch.cuda.device(self.device):
            self.bufs["input"] = torch.empty((n, *in_hwc), dtype=torch.float32, device=self.device)
            if input_u8:
                if in_hwc[2] != 3:
                    raise ValueError("u8 frames feed a 3-channel input")
                self.bufs["input_u8"] = torch.empty((n, *in_hwc), dtype=torch.uint8, device=self.device)
                self.ops.append(OpRecord("u8in", "input", "input_u8"))
            for op in self.graph:
                kind, out, src = op[0], op[1], op[2]
                h, w, c = self.shapes[src]
                if kind == "resize" and (out in fused_resize or out in dropped_resize):
                    continue
                if out in fused_heads or out in block_inner:
                    continue  # recorded with its depthwise producer / its block
                if out in block_of:
                    eop, dop, pop, plans = block_of[out]
                    rec = OpRecord("mb", out, eop[2], conv=pop[3], res=pop[4], blk=plans,
                                   members=(eop[1], pop[1]) if dop is None else (eop[1], dop[1], pop[1]))
                    self.bufs[out] = torch.empty((n, *self.shapes[out]), dtype=torch.float32, device=self.device)
                    self.ops.append(rec)
                    continue
                if out in head_of:
                    hop = head_of[out]
                    rec = OpRecord("dwpw", hop[1], src, conv=op[3], up=tail_up.get(src), members=(out, hop[1]))
                    rec.plan, rec.head = head_plans[out]
                    self.bufs[hop[1]] = torch.empty((n, *self.shapes[hop[1]]), dtype=torch.float32, device=self.device)
                    self.ops.append(rec)
                    continue
                rec = OpRecord(kind, out, src)
                if kind == "conv":
                    rec.conv, rec.res = op[3], (None if out in tail_up else op[4])
                    res_resize = None
                    if rec.res in fused_resize:
                        lo = fused_resize[rec.res]
                        res_resize = (self.shapes[lo][0], self.shapes[lo][1], "half_pixel")
                        rec.res = lo
                    rec.plan = ConvPlan(rec.conv, n, h, w, has_res=rec.res is not None, math=math,
                                        res_resize=res_resize, device=self.device)
                    wt, b = weights[out]
                    rec.plan.load_weights(wt, b)
                else:
                    rec.size, rec.res = op[3], op[4]
                self.bufs[out] = torch.empty((n, *self.shapes[out]), dtype=torch.float32, device=self.device)
                self.ops.append(rec)
        # Stem + 1x1 (fuse_stem): a 1x1 TF32 conv over the tensor-core stem's
        # output (cin 32, cout <= 32, no residual: a pyramid lateral on the
        # stem features) runs inside the stem's launch (aie_conv_run_stem_pw)
        # from the stem's staged tile instead of re-reading it from memory.
        if fuse_stem:
            for st in [r for r in self.ops if r.kind == "conv" and r.plan.info.variant == 2]:
                pw = next((r for r in self.ops if r.kind == "conv" and r.src == st.out and r.res is None
                           and r.plan.kernel == "pw" and r.plan.math == "tf32" and r.conv.cin == 32
                           and r.conv.cout <= 32 and r.conv.cout % 4 == 0), None)
                if pw is None:
                    continue
                st.kind, st.head, st.out2 = "stempw", pw.plan, pw.out
                st.members = (st.out, pw.out)
                self.ops.remove(pw)
        self.graph_exec = None

    # -- accounting ------------------------------------------------------------
    def conv_flops(self) -> int:
        total = 0
        for r in self.ops:
            if r.blk is not None:
                total += sum(p.flops for p in r.blk if p is not None)
            elif r.plan is not None:
                total += r.plan.flops + (r.head.flops if r.head is not None else 0)
        return total

    def tf32_convs(self) -> set:
        """Names of the graph's convs that run on the TF32 tensor cores
        (fused launches included): the convs whose operands a TF32-emulating
        oracle truncates."""
        names = set()
        for r in self.ops:
            if r.kind == "conv" and r.plan.math == "tf32":
                names.add(r.out)
            elif r.kind == "stempw":
                names.update(r.members)
            elif r.kind == "mb":  # the two 1x1 GEMMs; the depthwise between them runs on the CUDA cores
                ex, _, pj = r.blk
                names.update(m for m, p in ((r.members[0], ex), (r.members[-1], pj)) if p.math == "tf32")
            elif r.kind == "dwpw" and r.plan.math == "tf32":
                names.add(r.members[0])
        return names

    def layer_table(self):
        rows = []
        for r in self.ops:
            if r.plan is not None:
                rows.append((r.out, r.plan.kernel, r.plan.math, r.plan.flops, r.plan.min_bytes))
        return rows

    # -- execution -----------------------------------------------------------------
    def record(self, stream=None):
        """Issue every op of the graph on `stream` (default: current stream)."""
        for r in self.ops:
            src = self.bufs[r.src]
            out = self.bufs[r.out]
            if r.kind == "conv":
                r.plan(src, self.bufs[r.res] if r.res else None, out=out, stream=stream)
            elif r.kind == "dwpw":
                run_dw_pw(r.plan, r.head, src, out=out, stream=stream, up=self.bufs[r.up] if r.up else None)
            elif r.kind == "mb":
                run_mbconv(*r.blk, src, res=self.bufs[r.res] if r.res else None, out=out, stream=stream)
            elif r.kind == "stempw":
                run_stem_pw(r.plan, r.head, src, stem_out=out, pw_out=self.bufs[r.out2], stream=stream)
            elif r.kind == "u8in":
                input_u8(src, out=out, stream=stream)
            else:
                oh, ow = r.size
                resize_bilinear(src, oh, ow, add=self.bufs[r.res] if r.res else None, out=out, stream=stream)
        return self.bufs[self.output]

    def _capture_one(self):
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.record()  # warm-up outside capture
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.record()
        return g

    def capture(self):
        """Capture the whole batch as one CUDA graph (replaces the per-op
        Python dispatch; the kernels are the same)."""
        self.graph_exec = self._capture_one()
        return self.graph_exec

    def infer(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x is not None:
            self.bufs[self.input_name].copy_(x, non_blocking=True)
        if self.graph_exec is not None:
            self.graph_exec.replay()
        else:
            self.record()
        return self.bufs[self.output]

    # -- pipelined host -> device -> host ------------------------------------------
    def capture_slots(self, slots: int = 2):
        """One CUDA graph per I/O slot: graph s reads input slot s and writes
        output slot s; the intermediate activations are shared, so the graphs
        run one after another on the compute stream while the copies of the
        neighbouring batches use the other slots."""
        if slots < 2:
            raise ValueError("pipelining needs at least two slots")
        iname = self.input_name
        in0, out0 = self.bufs[iname], self.bufs[self.output]
        self.in_slots = [in0] + [torch.empty_like(in0) for _ in range(slots - 1)]
        self.out_slots = [out0] + [torch.empty_like(out0) for _ in range(slots - 1)]
        self.slot_graphs = []
        try:
            for s in range(slots):
                self.bufs[iname], self.bufs[self.output] = self.in_slots[s], self.out_slots[s]
                self.slot_graphs.append(self._capture_one())
        finally:
            self.bufs[iname], self.bufs[self.output] = in0, out0
        self._copy_in = torch.cuda.Stream(device=self.device)
        self._copy_out = torch.cuda.Stream(device=self.device)

    def run_pipelined(self, host_in: Sequence[torch.Tensor], host_out: Sequence[torch.Tensor], stream=None):
        """Run batch k = host_in[k] (pinned [n, h, w, c] frames: f32, or u8 RGB
        for a model built with input_u8) through the
        graph into host_out[k], end to end.  ai-gpu-runtime uploads, runs and
        reads back one frame per call (upload_input, infer and read_output,
        crates/ai-gpu-runtime/src/model.rs:387-470); here the upload of batch k+1 and the read-back of batch
        k-1 run on their own copy streams while batch k computes, so the
        steady state costs max(upload, compute, read-back) per batch.

        Asynchronous on `stream` (default: current stream): the outputs are
        complete once that stream is synchronised."""
        if len(host_in) != len(host_out):
            raise ValueError("one output buffer per input batch")
        if not getattr(self, "slot_graphs", None):
            self.capture_slots()
        S = len(self.slot_graphs)
        compute = torch.cuda.current_stream(self.device) if stream is None else stream
        cin, cout = self._copy_in, self._copy_out
        h2d = [torch.cuda.Event() for _ in range(S)]
        done = [torch.cuda.Event() for _ in range(S)]
        d2h = [torch.cuda.Event() for _ in range(S)]
        start = torch.cuda.Event()
        start.record(compute)
        cin.wait_event(start)
        cout.wait_event(start)
        for k, (hi, ho) in enumerate(zip(host_in, host_out)):
            s = k % S
            if k >= S:
                cin.wait_event(done[s])      # batch k-S no longer reads input slot s
            with torch.cuda.stream(cin):
                self.in_slots[s].copy_(hi, non_blocking=True)
            h2d[s].record(cin)
            compute.wait_event(h2d[s])
            if k >= S:
                compute.wait_event(d2h[s])   # output slot s of batch k-S has been read back
            with torch.cuda.stream(compute):
                self.slot_graphs[s].replay()
            done[s].record(compute)
            cout.wait_event(done[s])
            with torch.cuda.stream(cout):
                ho.copy_(self.out_slots[s], non_blocking=True)
            d2h[s].record(cout)
        for s in range(min(S, len(host_in))):
            compute.wait_event(d2h[s])
            compute.wait_event(h2d[s])
        return host_out

    def release(self):
        self.graph_exec = None
        self.slot_graphs = []
