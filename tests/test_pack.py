"""Layout tests restated from crates/ai-core/src/pack.rs:186-289 and
crates/ai-core/src/tensor.rs:82-111 (no GPU)."""
import numpy as np

from ai_engine_b200 import pack
from oracle import XorShift32


def test_layout_math():
    """tensor.rs:86-98: c=6 -> cg=2; idx = (h*W + w)*cg + cg_i"""
    assert pack.cg(6) == 2
    h, w, c = 3, 5, 6
    x = np.arange(h * w * c, dtype=np.float32).reshape(h, w, c)
    p = pack.pack_nhwc(x)
    assert p.shape == (3, 5, 8)
    flat = p.reshape(-1, 4)  # vec4 units
    idx = lambda hh, ww, g: (hh * w + ww) * 2 + g
    assert flat[idx(2, 4, 1)][0] == x[2, 4, 4]
    assert flat[idx(1, 0, 0)][3] == x[1, 0, 3]


def test_nhwc_roundtrip_odd_shapes():
    """pack.rs:190-197"""
    data = XorShift32(1).vec_f32(3 * 5 * 6).reshape(3, 5, 6)
    assert np.array_equal(pack.unpack_nhwc(pack.pack_nhwc(data), 6), data)


def test_pack_padding_channels_are_zero():
    """pack.rs:210-219"""
    flat = pack.pack_nhwc(np.ones((1, 2, 3), np.float32)).reshape(-1)
    assert flat[3] == 0.0 and flat[7] == 0.0


def test_conv_weight_layout_pointwise_identity():
    """pack.rs:222-236"""
    w = np.eye(4, dtype=np.float32).reshape(-1)
    packed, kg = pack.pack_weights_conv(w, 4, 4, 1, 1, 1)
    assert kg == 1
    assert np.array_equal(packed[:16].reshape(4, 4), np.eye(4, dtype=np.float32))


def test_conv_weight_kg_alignment_pads_zero():
    """pack.rs:239-252"""
    w = XorShift32(3).vec_f32(8 * 6)
    packed, kg = pack.pack_weights_conv(w, 8, 6, 1, 1, 4)
    assert kg == 4
    ng = 2
    assert not packed[2 * ng * 16:4 * ng * 16].any()


def test_pack_unpack_roundtrip_conv_and_dw():
    """pack.rs:255-270"""
    rng = XorShift32(11)
    cout, cin, k = 10, 6, 3
    w = rng.vec_f32(cout * cin * k * k)
    packed, kg_pad = pack.pack_weights_conv(w, cout, cin, k, k, 4)
    assert np.array_equal(pack.unpack_weights_conv(packed, cout, cin, k, k, kg_pad), w)
    c = 7
    wd = rng.vec_f32(c * 9)
    assert np.array_equal(pack.unpack_weights_dw(pack.pack_weights_dw(wd, c, 3, 3), c, 3, 3), wd)
    b = rng.vec_f32(cout)
    assert np.array_equal(pack.pack_bias(b, cout)[:cout], b)


def test_dw_weight_layout():
    """pack.rs:273-288"""
    c, taps, cg = 5, 9, 2
    w = np.arange(c * taps, dtype=np.float32)
    flat = pack.pack_weights_dw(w, c, 3, 3)
    for t in range(taps):
        assert flat[(t * cg + 1) * 4] == 4 * taps + t
        assert flat[(t * cg + 1) * 4 + 1] == 0.0
