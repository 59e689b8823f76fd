"""GPU parity of the graph-glue kernels (aie_binary, aie_mix, aie_gpool,
aie_avgpool, aie_channel_copy) against the ai-cpu restatement, through the
C ABI.  These ops round every step like ai-cpu, so the bar is bit-exact,
except for sigmoid / tanh (CUDA's expf / tanhf against glibc's, each
within 2 ulp of the exact value): 4 ulp.  Dense 16-byte-aligned shapes take the vector path; odd channel
counts and channel views take the element path."""
import numpy as np
import pytest
import torch

import oracle
from ai_engine_b200 import elementwise as ew
from oracle import XorShift32

pytestmark = pytest.mark.gpu

ACTS = ["none", "relu", "sigmoid", "tanh", "hardswish", "hardsigmoid", "clamp01"]


def _check(got, want, act="none"):
    got = np.asarray(got)
    if act in ("sigmoid", "tanh"):
        ulp = np.spacing(np.abs(want).astype(np.float32))
        assert np.all(np.abs(got.astype(np.float64) - want) <= 4 * ulp), float(np.max(np.abs(got - want) / ulp))
    else:
        assert np.array_equal(got, want), float(np.max(np.abs(got - want)))


def _rand(rng, *shape, scale=4.0):
    return (rng.vec_f32(int(np.prod(shape))) * scale).reshape(shape)


@pytest.mark.parametrize("c", [8, 5])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "prelu"])
@pytest.mark.parametrize("kind", ["tensor", "scalar", "scalar_first", "cvec", "cvec_tensor", "pvec_tensor"])
def test_binary(cuda_ok, c, op, kind):
    rng = XorShift32(7001 + c)
    n, h, w = 3, 5, 7
    a = _rand(rng, n, h, w, c)
    b = {"tensor": lambda: _rand(rng, n, h, w, c), "scalar": lambda: np.float32(0.75),
         "scalar_first": lambda: np.float32(-1.25), "cvec": lambda: _rand(rng, c),
         "cvec_tensor": lambda: _rand(rng, n, c), "pvec_tensor": lambda: _rand(rng, n * h * w)}[kind]()
    for act in ACTS:
        want = np.empty_like(a)
        oracle.binary(op, a, b, want, act, kind=kind)
        ga = torch.from_numpy(a).cuda()
        out = torch.empty_like(ga)
        if kind in ("scalar", "scalar_first"):
            gb = float(b)
        else:
            gb = torch.from_numpy(np.ascontiguousarray(b)).cuda()
        ew.binary(op, ga, gb, out, act, kind="scalar" if kind == "scalar_first" else kind,
                  scalar_first=kind == "scalar_first")
        _check(out.cpu().numpy(), want, act)


def test_binary_channel_views(cuda_ok):
    """Operands and output as channel slices of wider tensors (ai-cpu's
    strided View, crates/ai-cpu/src/kernels/elementwise.rs:278-300), both at
    16-byte-aligned offsets (vector path) and odd ones."""
    rng = XorShift32(7101)
    n, h, w = 2, 4, 6
    big_a = _rand(rng, n, h, w, 20)
    big_b = _rand(rng, n, h, w, 12)
    for (ao, bo, oo, c) in [(4, 8, 0, 4), (3, 1, 5, 6), (8, 0, 4, 12)]:
        want = np.zeros((n, h, w, 24), np.float32)
        oracle.binary("mul", (big_a, ao, c), (big_b, bo, c), (want, oo, c), "hardswish")
        out = torch.zeros((n, h, w, 24), device="cuda")
        ew.binary("mul", ew.ChView(torch.from_numpy(big_a).cuda(), ao, c),
                  ew.ChView(torch.from_numpy(big_b).cuda(), bo, c), ew.ChView(out, oo, c), "hardswish")
        _check(out.cpu().numpy(), want)


def test_binary_in_place(cuda_ok):
    """out aliasing a (an SE gate applied in place)."""
    rng = XorShift32(7102)
    a = _rand(rng, 2, 3, 4, 16)
    g = _rand(rng, 2, 16)
    want = np.empty_like(a)
    oracle.binary("mul", a, g, want, kind="cvec_tensor")
    ga = torch.from_numpy(a).cuda()
    ew.binary("mul", ga, torch.from_numpy(g).cuda(), ga, kind="cvec_tensor")
    _check(ga.cpu().numpy(), want)


@pytest.mark.parametrize("c,views", [(8, False), (6, False), (16, True)])
def test_mix(cuda_ok, c, views):
    rng = XorShift32(7201 + c)
    n, h, w = 2, 5, 9
    z = rng.vec_f32(n * h * w * c).reshape(n, h, w, c) * 0.5 + 0.5
    a = _rand(rng, n, h, w, c)
    b = _rand(rng, n, h, w, c)
    want = np.empty_like(a)
    oracle.mix(z, a, b, want)
    out = torch.empty((n, h, w, c), device="cuda")
    if views:
        zz = np.concatenate([z, np.ones_like(z)], -1)  # z as the first half of a gate tensor
        ew.mix(ew.ChView(torch.from_numpy(zz).cuda(), 0, c), torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), out)
    else:
        ew.mix(torch.from_numpy(z).cuda(), torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), out)
    _check(out.cpu().numpy(), want)
    # a = h, b = c~: the ConvGRU update (1 - z) h + z c~ stays between its operands
    got = out.cpu().numpy()
    lo, hi = np.minimum(a, b), np.maximum(a, b)
    assert np.all(got >= lo - 1e-5 * np.abs(lo) - 1e-6) and np.all(got <= hi + 1e-5 * np.abs(hi) + 1e-6)


@pytest.mark.parametrize("n,h,w,c", [(3, 18, 32, 72), (2, 9, 16, 960), (2, 5, 7, 5), (1, 1, 1, 8), (4, 3, 3, 12),
                                     (2, 36, 64, 72), (3, 7, 9, 200), (2, 1, 1, 132)])
def test_gpool(cuda_ok, n, h, w, c):
    rng = XorShift32(7301 + c)
    x = _rand(rng, n, h, w, c)
    want = oracle.gpool(x)
    out = torch.empty((n, c), device="cuda")
    ew.gpool(torch.from_numpy(x).cuda(), out)
    _check(out.cpu().numpy(), want)


def test_gpool_channel_view(cuda_ok):
    rng = XorShift32(7310)
    x = _rand(rng, 2, 6, 10, 24)
    want = oracle.gpool((x, 8, 12))
    out = torch.empty((2, 12), device="cuda")
    ew.gpool(ew.ChView(torch.from_numpy(x).cuda(), 8, 12), out)
    _check(out.cpu().numpy(), want)


@pytest.mark.parametrize("c", [3, 8])
@pytest.mark.parametrize("k,s,pad", [((2, 2), (2, 2), (0, 0, 0, 0)), ((3, 3), (2, 2), (1, 1, 1, 1)),
                                     ((3, 2), (1, 2), (0, 1, 2, 0))])
def test_avgpool(cuda_ok, c, k, s, pad):
    rng = XorShift32(7401 + c)
    x = _rand(rng, 2, 9, 14, c)
    want = oracle.avgpool(x, k, s, pad)
    out = torch.empty(want.shape, device="cuda")
    ew.avgpool(torch.from_numpy(x).cuda(), out, k, s, pad)
    _check(out.cpu().numpy(), want)


@pytest.mark.parametrize("act", ACTS)
def test_channel_copy_concat(cuda_ok, act):
    """A 171-channel concat built part by part (128 + 40 + 3, RVM's decode3
    input), then a slice of it back out with an activation."""
    rng = XorShift32(7501)
    n, h, w = 2, 3, 5
    parts = [_rand(rng, n, h, w, c) for c in (128, 40, 3)]
    want = np.concatenate(parts, -1)
    cat = torch.zeros((n, h, w, 172), device="cuda")
    coff = 0
    for p in parts:
        ew.channel_copy(torch.from_numpy(p).cuda(), ew.ChView(cat, coff, p.shape[-1]))
        coff += p.shape[-1]
    got = cat.cpu().numpy()
    _check(got[..., :171], want)
    assert not got[..., 171].any()
    sl = np.empty((n, h, w, 41), np.float32)
    oracle.channel_copy((want, 129, 41), sl, act)
    out = torch.empty((n, h, w, 41), device="cuda")
    ew.channel_copy(ew.ChView(cat, 129, 41), out, act)
    _check(out.cpu().numpy(), sl, act)


def test_glue_rejects_bad_views(cuda_ok):
    x = torch.zeros((1, 2, 2, 8), device="cuda")
    with pytest.raises(ValueError):
        ew.ChView(x, 6, 4)
    with pytest.raises(ValueError):
        ew.binary("add", x, torch.zeros((1, 2, 2, 4), device="cuda"), x)
    with pytest.raises(ValueError):
        ew.binary("add", x, torch.zeros(3, device="cuda"), x, kind="cvec")


@pytest.mark.parametrize("widths,pad", [((128, 40, 3), 1), ((32, 3), 1), ((16, 16), 0), ((5, 7, 4), 0)])
def test_concat(cuda_ok, widths, pad):
    """aie_concat: the parts in one pass, trailing padding lanes zeroed;
    one part given as a channel view of a wider tensor."""
    rng = XorShift32(7601 + sum(widths))
    n, h, w = 2, 3, 5
    parts = [_rand(rng, n, h, w, c) for c in widths]
    wide = _rand(rng, n, h, w, widths[0] + 6)
    wide[..., 2:2 + widths[0]] = parts[0]
    want = np.concatenate(parts, -1)
    cout = want.shape[-1] + pad
    out = torch.full((n, h, w, cout), 7.0, device="cuda")
    gp = [ew.ChView(torch.from_numpy(wide).cuda(), 2, widths[0])] + [torch.from_numpy(p).cuda() for p in parts[1:]]
    ew.concat(gp, out)
    got = out.cpu().numpy()
    _check(got[..., :want.shape[-1]], want)
    assert not got[..., want.shape[-1]:].any()
