"""Graph executor for conv graphs with glue ops and recurrent state.

Plays the part of ai-gpu-runtime's ``Model`` (crates/ai-gpu-runtime/src/
model.rs:56-426) for graphs that mix convs with the non-conv ops of
``SwOp`` (crates/ai-core/src/format/model.rs:78-214) -- the recurrent
matting net's SE gates, LR-ASPP, ConvGRU and output block -- and that carry
state from one frame to the next (``SwState``, the ``r1..r4 -> r1o..r4o``
pairs of a recurrent model; ai_cpu::Model keeps them the same way,
crates/ai-cpu/src/model.rs:114-144).

Load time lowers every conv (one ``ConvPlan`` each, packed weights on the
device) and allocates every tensor once; a step records one launch per op
on one CUDA stream, or replays a captured CUDA graph.  Recurrent state
ping-pongs between two buffers per state, so a step never copies it: the
executor captures one graph per parity.

Nodes (``Node.kind``):
  conv     out = conv(ins[0]) (+ res)                 SwOp::Conv
  binary   out = act(ins[0] o ins[1] | scalar | cvec)  SwOp::Binary
  mix      out = a + z (b - a), ins = (z, a, b)       SwOp::Mix
  gpool    out [1, 1, C] = channel means               SwOp::Gpool
  avgpool  window mean, k / s in ``size``              SwOp::Avgpool
  resize   bilinear to ``size`` (half_pixel)           SwOp::Resize
  concat   channel concat of ins                       SwOp::Concat
  split    outs = channel slices of ins[0] (views)     Split (an alias)
  chcopy   out = act(ins[0][coff : coff + c])          SwOp::Chcopy / Act
  view     out = ins[0][coff : coff + c], no copy       SwTensor.alias
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import elementwise as ew
from ._lib import AieError
from .conv import Conv2d, ConvPlan, View, resize_bilinear, run_parts


@dataclass
class Node:
    kind: str
    out: object                      # a tensor name (a tuple of names for split)
    ins: Tuple[str, ...]
    conv: Optional[Conv2d] = None
    res: Optional[str] = None
    op: str = "add"                  # binary op
    act: str = "none"
    bkind: str = "tensor"            # binary operand: tensor / scalar / scalar_first / cvec / cvec_tensor
    scalar: float = 0.0
    size: Tuple[int, ...] = ()       # resize (oh, ow); avgpool (kh, kw, sh, sw)
    parts: Tuple[int, ...] = ()      # split channel counts; chcopy (coff, c)


def infer_shapes(nodes: Sequence[Node], inputs: Dict[str, Tuple[int, int, int]]) -> Dict[str, Tuple[int, int, int]]:
    """(h, w, c) of every tensor, checking each op's operand shapes."""
    sh = dict(inputs)
    for nd in nodes:
        s0 = sh[nd.ins[0]] if nd.ins else None
        k = nd.kind
        if k == "conv":
            if s0[2] != nd.conv.cin:
                raise ValueError(f"{nd.out}: conv expects {nd.conv.cin} channels, {nd.ins[0]} has {s0[2]}")
            oh, ow = nd.conv.out_hw(s0[0], s0[1])
            sh[nd.out] = (oh, ow, nd.conv.cout)
            if nd.res is not None and sh[nd.res] != sh[nd.out]:
                raise ValueError(f"{nd.out}: residual shape {sh[nd.res]} != {sh[nd.out]}")
        elif k == "binary":
            if nd.bkind == "tensor" and sh[nd.ins[1]] != s0:
                raise ValueError(f"{nd.out}: operand shapes {s0} / {sh[nd.ins[1]]}")
            if nd.bkind == "cvec_tensor" and sh[nd.ins[1]] != (1, 1, s0[2]):
                raise ValueError(f"{nd.out}: channel vector {sh[nd.ins[1]]} for {s0}")
            sh[nd.out] = s0
        elif k == "mix":
            if not (sh[nd.ins[1]] == sh[nd.ins[2]] == s0):
                raise ValueError(f"{nd.out}: mix operand shapes differ")
            sh[nd.out] = s0
        elif k == "gpool":
            sh[nd.out] = (1, 1, s0[2])
        elif k == "avgpool":
            kh, kw, sy, sx = nd.size
            sh[nd.out] = ((s0[0] - kh) // sy + 1, (s0[1] - kw) // sx + 1, s0[2])
        elif k == "resize":
            sh[nd.out] = (nd.size[0], nd.size[1], s0[2])
        elif k == "concat":
            hw = {sh[i][:2] for i in nd.ins}
            if len(hw) != 1:
                raise ValueError(f"{nd.out}: concat parts differ in size {hw}")
            sh[nd.out] = (s0[0], s0[1], sum(sh[i][2] for i in nd.ins))
        elif k == "split":
            if sum(nd.parts) != s0[2]:
                raise ValueError(f"split of {nd.ins[0]}: parts {nd.parts} != {s0[2]} channels")
            for name, c in zip(nd.out, nd.parts):
                sh[name] = (s0[0], s0[1], c)
        elif k in ("chcopy", "view"):
            coff, c = nd.parts
            if coff + c > s0[2]:
                raise ValueError(f"{nd.out}: channels past the source")
            sh[nd.out] = (s0[0], s0[1], c)
        else:
            raise ValueError(f"unknown node kind {k}")
    return sh


def _pad4(c: int) -> int:
    return (c + 3) // 4 * 4


def _pad_narrow_inputs(nodes: List[Node], inputs: Dict[str, Tuple[int, int, int]]) -> Tuple[List[Node], set]:
    """A graph input whose channel count is not a multiple of 4 and that is
    a concat part (RVM's 3-channel frame in its output block's concat) gets
    a copy with its pixels padded to 4 lanes (a zero lane), made once per
    step by a one-part concat (which writes each padded pixel whole, the
    zero lane included, as one 16-byte store): the concat's part and the average pools that build the image
    pyramid from it (whose outputs are the other concats' parts) read the
    copy, so every such part is a TMA-compatible view and the concat can
    be read in place by its conv.  Returns the rewritten nodes and the
    names whose buffers carry the padding."""
    shapes = infer_shapes(nodes, inputs)
    narrow = {p for nd in nodes if nd.kind == "concat" for p in nd.ins
              if p in inputs and shapes[p][2] % 4}
    if not narrow:
        return nodes, set()
    shadow = {p: p + ".c4" for p in narrow}
    padded = set(shadow.values())
    out: List[Node] = [Node("concat", shadow[p], (p,)) for p in sorted(narrow)]
    for nd in nodes:
        if nd.kind == "concat" and any(p in shadow for p in nd.ins):
            nd = replace(nd, ins=tuple(shadow.get(p, p) for p in nd.ins))
        elif nd.kind == "avgpool" and nd.ins[0] in shadow:
            nd = replace(nd, ins=(shadow[nd.ins[0]],))
        if nd.kind == "avgpool" and nd.ins[0] in padded:
            padded.add(nd.out)  # pools the zero lane too: stays zero
        out.append(nd)
    return out, padded


@dataclass
class _Rec:
    node: Node
    plan: Optional[ConvPlan] = None


class NetModel:
    """Load-time lowering and per-step execution of a node graph on one GPU.

    inputs: {name: (h, w, c)} of the per-frame inputs; states: {in: out}
    pairs of recurrent tensors (out of step t is in of step t + 1, zero
    before the first step); outputs: the names a step returns."""

    def __init__(self, nodes: Sequence[Node], weights: Dict[str, Tuple[np.ndarray, np.ndarray]], n: int,
                 inputs: Dict[str, Tuple[int, int, int]], outputs: Sequence[str],
                 states: Optional[Dict[str, str]] = None, consts: Optional[Dict[str, np.ndarray]] = None, *,
                 math: str = "auto", device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.n = n
        self.nodes, padded = _pad_narrow_inputs(list(nodes), inputs)
        self.states = dict(states or {})
        self.outputs = list(outputs)
        self.shapes = infer_shapes(self.nodes, inputs)
        self.feeds = [k for k in inputs if k not in self.states]  # per-step inputs (not recurrent state)
        for si, so in self.states.items():
            if self.shapes[si] != self.shapes[so]:
                raise ValueError(f"state {si} {self.shapes[si]} != {so} {self.shapes[so]}")
        consumers: Dict[str, List[Node]] = {}
        for nd in self.nodes:
            for t in (*nd.ins, nd.res):
                if t is not None:
                    consumers.setdefault(t, []).append(nd)
        # a concat whose consumers are all convs gets its channels padded to a
        # multiple of 4 (zero lanes, zero weights): the conv then reads it
        # through TMA on the tensor cores
        self.cpad: Dict[str, int] = {name: _pad4(self.shapes[name][2]) for name in padded}
        for nd in self.nodes:
            if nd.kind == "concat":
                c = self.shapes[nd.out][2]
                users = consumers.get(nd.out, [])
                if c % 4 and users and all(u.kind == "conv" and u.ins[0] == nd.out for u in users) \
                        and nd.out not in self.outputs:
                    self.cpad[nd.out] = _pad4(c)
        # Concat-into-conv: a concat whose only consumer is one tensor-core
        # conv, with every part a 16-byte aligned view (pixel stride and
        # first channel multiples of 4), is not materialised: the conv reads
        # the parts in place (aie_conv_run_parts), as ai-gpu's implicit GEMM
        # reads its SrcView parts (crates/ai-gpu/src/kernels/conv_igemm.rs:49-76).
        # The other concats are written by one aie_concat pass.
        self.fused_concat: Dict[str, Tuple[str, ...]] = {}  # concat name -> its parts
        self.alias: Dict[str, Tuple[str, int, int]] = {}  # split output -> (base tensor, coff, c)
        self.bufs: Dict[str, torch.Tensor] = {}
        self.recs: List[_Rec] = []
        dev = self.device
        with torch.cuda.device(dev):
            def alloc(name, zero=False):
                h, w, c = self.shapes[name]
                c = self.cpad.get(name, c)
                self.bufs[name] = (torch.zeros if zero else torch.empty)((n, h, w, c), dtype=torch.float32, device=dev)

            for name in inputs:
                alloc(name, zero=name in self.states)
            concat_nodes = {nd.out: nd for nd in self.nodes if nd.kind == "concat"}
            for nd in self.nodes:
                rec = _Rec(nd)
                if nd.kind == "concat" and self._fusable_concat(nd, consumers, math):
                    self.fused_concat[nd.out] = tuple(nd.ins)
                    self.recs.append(rec)  # kept in the node list, issued by its conv
                    continue
                if nd.kind in ("split", "view"):
                    base, coff = self._base(nd.ins[0])
                    if nd.kind == "view":
                        self.alias[nd.out] = (base, coff + nd.parts[0], nd.parts[1])
                    else:
                        for name, c in zip(nd.out, nd.parts):
                            self.alias[name] = (base, coff, c)
                            coff += c
                    self.recs.append(rec)
                    continue
                alloc(nd.out, zero=nd.out in self.cpad)
                if nd.kind == "conv" and nd.ins[0] in self.fused_concat:
                    h, w, c = self.shapes[nd.ins[0]]
                    parts = [self.shapes[pn][2] for pn in self.fused_concat[nd.ins[0]]]
                    try:
                        rec.plan = ConvPlan(nd.conv, n, h, w, has_res=nd.res is not None, math=math, parts=parts,
                                            device=dev).load_weights(*weights[nd.out])
                    except AieError:
                        # not a tensor-core conv after all: materialise the concat
                        cn = concat_nodes[nd.ins[0]]
                        del self.fused_concat[cn.out]
                        alloc(cn.out)
                        rec.plan = None
                    if rec.plan is not None:
                        self.recs.append(rec)
                        continue
                if nd.kind == "conv":
                    src = nd.ins[0]
                    h, w, c = self.shapes[src]
                    cv = nd.conv
                    wt, b = weights[nd.out]
                    base, coff = self._base(src)
                    bc = self.bufs[base].shape[-1]
                    if src in self.cpad:  # padded concat: zero weight rows for the padding lanes
                        cp = self.cpad[src]
                        w4 = np.zeros((cv.cout, cp, cv.kh, cv.kw), np.float32)
                        w4[:, :c] = np.asarray(wt, np.float32).reshape(cv.cout, c, cv.kh, cv.kw)
                        wt = w4
                        cv = Conv2d(cp, cv.cout, cv.kh, cv.kw, cv.sh, cv.sw, cv.pad, cv.dil, cv.groups, cv.act)
                    in_view = View(bc, coff) if (base != src) else None
                    rec.plan = ConvPlan(cv, n, h, w, has_res=nd.res is not None, math=math, in_view=in_view,
                                        device=dev).load_weights(wt, b)
                self.recs.append(rec)
            for si, so in self.states.items():
                if so in self.alias:
                    raise ValueError(f"state output {so} must be a tensor, not a view")
        self.consts = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(dev)
                       for k, v in (consts or {}).items()}
        self.step_index = 0
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}

    def _fusable_concat(self, nd: Node, consumers, math: str) -> bool:
        users = consumers.get(nd.out, [])
        if math not in ("auto", "tf32") or len(nd.ins) > 3 or nd.out in self.outputs or nd.out in self.states.values():
            return False
        if len(users) != 1 or users[0].kind != "conv" or users[0].ins[0] != nd.out or users[0].conv.groups != 1:
            return False
        for pn in nd.ins:
            if pn in self.fused_concat:
                return False
            base, coff = self._base(pn)
            stride = self.shapes[base][2] if base not in self.cpad else self.cpad[base]
            if base in self.fused_concat or stride % 4 or coff % 4:
                return False
        # every part starts on a K block of the conv (16 channels when all
        # parts have at most 16, else 32): at most one K block more than the
        # concatenated tensor takes, or the extra MMAs cost more than the
        # concat pass saves
        cs = [self.shapes[pn][2] for pn in nd.ins]
        bk = 16 if max(cs) <= 16 else 32
        return sum((c + bk - 1) // bk * bk for c in cs) <= (sum(cs) + 31) // 32 * 32 + 32

    # -- tensors -----------------------------------------------------------------
    def _base(self, name: str) -> Tuple[str, int]:
        if name in self.alias:
            b, coff, _ = self.alias[name]
            return b, coff
        return name, 0

    def view(self, name: str) -> ew.ChView:
        if name in self.alias:
            b, coff, c = self.alias[name]
            return ew.ChView(self.bufs[b], coff, c)
        return ew.ChView(self.bufs[name], 0, self.shapes[name][2])

    def tensor(self, name: str) -> torch.Tensor:
        """The logical [n, h, w, c] tensor (a copy if it is a view or padded;
        a concat read in place by its conv is assembled from its parts)."""
        if name in self.fused_concat:
            return torch.cat([self.tensor(p) for p in self.fused_concat[name]], dim=-1)
        v = self.view(name)
        if v.coff == 0 and v.c == v.t.shape[-1]:
            return v.t
        return v.t[..., v.coff:v.coff + v.c].contiguous()

    @property
    def conv_flops(self) -> int:
        return sum(r.plan.flops for r in self.recs if r.plan is not None)

    # -- execution -----------------------------------------------------------------
    def record(self, stream=None, ops=None):
        """Issue every op of one step on `stream` (default: current stream),
        or only the records in `ops` (a per-op timing pass)."""
        for r in (self.recs if ops is None else ops):
            nd = r.node
            k = nd.kind
            if k in ("split", "view"):
                continue
            if k == "conv" and nd.ins[0] in self.fused_concat:
                parts = []
                for pn in self.fused_concat[nd.ins[0]]:
                    base, coff = self._base(pn)
                    parts.append((self.bufs[base], coff))
                run_parts(r.plan, parts, res=None if nd.res is None else self.bufs[nd.res], out=self.bufs[nd.out],
                          stream=stream)
            elif k == "conv":
                base, _ = self._base(nd.ins[0])
                r.plan(self.bufs[base], res=None if nd.res is None else self.bufs[nd.res], out=self.bufs[nd.out],
                       stream=stream)
            elif k == "binary":
                if nd.bkind == "tensor":
                    b = self.view(nd.ins[1])
                elif nd.bkind in ("scalar", "scalar_first"):
                    b = nd.scalar
                elif nd.bkind == "cvec":
                    b = self.consts[nd.ins[1]]
                else:
                    b = self.bufs[nd.ins[1]]
                ew.binary(nd.op, self.view(nd.ins[0]), b, self.view(nd.out), nd.act,
                          kind="scalar" if nd.bkind == "scalar_first" else nd.bkind,
                          scalar_first=nd.bkind == "scalar_first", stream=stream)
            elif k == "mix":
                ew.mix(self.view(nd.ins[0]), self.view(nd.ins[1]), self.view(nd.ins[2]), self.view(nd.out),
                       stream=stream)
            elif k == "gpool":
                ew.gpool(self.view(nd.ins[0]), self.bufs[nd.out], stream=stream)
            elif k == "avgpool":
                ew.avgpool(self.bufs[nd.ins[0]], self.bufs[nd.out], nd.size[:2], nd.size[2:], stream=stream)
            elif k == "resize":
                resize_bilinear(self.tensor_for_resize(nd.ins[0]), nd.size[0], nd.size[1], out=self.bufs[nd.out],
                                stream=stream)
            elif k == "concat" and nd.out not in self.fused_concat:
                ew.concat([self.view(p) for p in nd.ins], ew.ChView(self.bufs[nd.out]), stream=stream)
            elif k == "chcopy":
                coff, c = nd.parts
                b, boff = self._base(nd.ins[0])
                ew.channel_copy(ew.ChView(self.bufs[b], boff + coff, c), self.view(nd.out), nd.act, stream=stream)

    def tensor_for_resize(self, name: str) -> torch.Tensor:
        if name in self.alias or name in self.cpad:
            raise ValueError(f"resize reads a dense tensor, {name} is a view")
        return self.bufs[name]

    def advance(self):
        """Make this step's state outputs the next step's state inputs."""
        for si, so in self.states.items():
            self.bufs[si], self.bufs[so] = self.bufs[so], self.bufs[si]
        self.step_index += 1

    def reset_state(self):
        for si in self.states:
            self.bufs[si].zero_()
        self.step_index = 0

    def capture(self, io_slots: bool = False):
        """Capture one CUDA graph per state parity (the buffers swap roles
        every step).  Replays with `replay()`.  With io_slots the per-step
        inputs and the non-state outputs get a second buffer, graph p reading
        and writing slot p, so that `run_pipelined` can copy the neighbouring
        steps' frames and results while a step computes."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.record(s)  # warm-up outside capture (plans, allocator)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        io = []
        if io_slots:
            io = list(dict.fromkeys(self._io_name(k) for k in (*self.feeds, *self.outputs)
                                    if k not in self.states.values()))
            for k in io:
                if k in self.alias or k in self.cpad:
                    raise ValueError(f"{k} is a view; pipelined I/O needs whole tensors")
            self.io_slots = {k: [self.bufs[k], torch.empty_like(self.bufs[k])] for k in io}
        saved = {k: self.bufs[k] for k in (*self.states.keys(), *self.states.values(), *io)}
        try:
            for parity in (0, 1):
                for k in io:
                    self.bufs[k] = self.io_slots[k][parity]
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self.record()
                self.graphs[parity] = g
                for si, so in self.states.items():
                    self.bufs[si], self.bufs[so] = self.bufs[so], self.bufs[si]
        finally:
            self.bufs.update(saved)
        self.reset_state()

    def _io_name(self, k: str) -> str:
        """The tensor behind `k`: an alias spanning all of its base tensor's
        channels is that tensor (a .sw model's output alias)."""
        a = self.alias.get(k)
        if a is not None and a[1] == 0 and a[2] == self.bufs[a[0]].shape[-1]:
            return a[0]
        return k

    def run_pipelined(self, host_in: Sequence[Dict[str, torch.Tensor]], host_out: Sequence[Dict[str, torch.Tensor]],
                      stream=None):
        """Run consecutive steps end to end: step k copies host_in[k] (pinned
        tensors per per-step input) in, replays the graph of its state parity
        and copies its non-state outputs into host_out[k] (pinned).  The
        upload of step k+1 and the read-back of step k-1 run on their own
        copy streams while step k computes (ai-gpu-runtime uploads, infers and
        reads back one frame per call, crates/ai-gpu-runtime/src/model.rs:
        387-470).  Recurrent state advances by one step per entry.
        Asynchronous on `stream` (default: current stream)."""
        if len(host_in) != len(host_out):
            raise ValueError("one output set per input set")
        if not getattr(self, "io_slots", None):
            self.capture(io_slots=True)
        compute = torch.cuda.current_stream(self.device) if stream is None else stream
        if not hasattr(self, "_copy_in"):
            self._copy_in = torch.cuda.Stream(device=self.device)
            self._copy_out = torch.cuda.Stream(device=self.device)
        cin, cout = self._copy_in, self._copy_out
        h2d = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        d2h = [torch.cuda.Event() for _ in range(2)]
        start = torch.cuda.Event()
        start.record(compute)
        cin.wait_event(start)
        cout.wait_event(start)
        for k, (hi, ho) in enumerate(zip(host_in, host_out)):
            p = self.step_index % 2
            if k >= 2:
                cin.wait_event(done[p])      # step k-2 no longer reads input slot p
            with torch.cuda.stream(cin):
                for name, t in hi.items():
                    self.io_slots[self._io_name(name)][p].copy_(t, non_blocking=True)
            h2d[p].record(cin)
            compute.wait_event(h2d[p])
            if k >= 2:
                compute.wait_event(d2h[p])   # output slot p of step k-2 has been read back
            with torch.cuda.stream(compute):
                self.graphs[p].replay()
            self.advance()
            done[p].record(compute)
            cout.wait_event(done[p])
            with torch.cuda.stream(cout):
                for name, t in ho.items():
                    t.copy_(self.io_slots[self._io_name(name)][p], non_blocking=True)
            d2h[p].record(cout)
        for p in range(min(2, len(host_in))):
            compute.wait_event(d2h[p])
            compute.wait_event(h2d[p])
        return host_out

    def replay(self):
        """One step from the captured graphs (state advances)."""
        if getattr(self, "io_slots", None):
            raise RuntimeError("captured with I/O slots: step it with run_pipelined")
        self.graphs[self.step_index % 2].replay()
        self.advance()

    def step(self, inputs: Dict[str, torch.Tensor], stream=None) -> Dict[str, torch.Tensor]:
        """Copy the step's inputs in, run one step eagerly, return copies of
        the outputs (device tensors the next step does not overwrite)."""
        for k, v in inputs.items():
            self.bufs[k].copy_(v)
        self.record(stream)
        outs = {k: self.tensor(k).clone() for k in self.outputs}
        self.advance()
        return outs

    def tf32_convs(self):
        """Names of the convs that run on the TF32 tensor cores."""
        return {r.node.out for r in self.recs if r.plan is not None and r.plan.math == "tf32"}

    def release(self):
        self.graphs.clear()
        self.io_slots = None
