"""NHWC-C4 and .sw weight packing (crates/ai-core/src/pack.rs:34-184).

These produce the byte layouts that ai_engine's converter writes into a
.sw blob and its GPU runtime binds; ``aie_conv_pack_weights`` accepts the
packed weight form directly (``wfmt="sw"``) and the kernels read and write
NHWC-C4 activations (``layout="nhwc_c4"``).
"""
from __future__ import annotations

import numpy as np


def cg(c: int) -> int:
    return (c + 3) // 4


def pack_nhwc(data: np.ndarray) -> np.ndarray:
    """Logical [..., c] (NHWC) -> [..., cg*4] with zero padding lanes (pack.rs:34-47)."""
    x = np.asarray(data, np.float32)
    c = x.shape[-1]
    out = np.zeros(x.shape[:-1] + (cg(c) * 4,), np.float32)
    out[..., :c] = x
    return out


def unpack_nhwc(packed: np.ndarray, c: int) -> np.ndarray:
    """NHWC-C4 -> logical NHWC, padding lanes dropped (pack.rs:50-64)."""
    return np.ascontiguousarray(np.asarray(packed)[..., :c])


def pack_weights_conv(w_oihw: np.ndarray, cout: int, cin: int, kh: int, kw: int, kg_align: int = 4):
    """OIHW -> [tap][kg][ng][j][comp] vec4s, kg padded to kg_align groups
    (pack.rs:68-102).  Returns (flat float32 array, kg_padded)."""
    w = np.asarray(w_oihw, np.float32).reshape(cout, cin, kh, kw)
    kg = -(-cg(cin) // max(kg_align, 1)) * max(kg_align, 1)
    ng = cg(cout)
    out = np.zeros((kh * kw, kg, ng, 4, 4), np.float32)
    # out[t, kgi, ngi, j, comp] = w[ngi*4+j, kgi*4+comp, ky, kx]
    wt = np.zeros((ng * 4, kg * 4, kh, kw), np.float32)
    wt[:cout, :cin] = w
    wt = wt.reshape(ng, 4, kg, 4, kh * kw)               # [ngi, j, kgi, comp, t]
    out[:] = wt.transpose(4, 2, 0, 1, 3)                  # [t, kgi, ngi, j, comp]
    return out.reshape(-1), kg


def pack_weights_dw(w: np.ndarray, c: int, kh: int, kw: int) -> np.ndarray:
    """[c][kh][kw] -> tap-major [tap][cg][comp] (pack.rs:105-122)."""
    taps = kh * kw
    src = np.zeros((cg(c) * 4, taps), np.float32)
    src[:c] = np.asarray(w, np.float32).reshape(c, taps)
    return np.ascontiguousarray(src.reshape(cg(c), 4, taps).transpose(2, 0, 1)).reshape(-1)


def pack_bias(b: np.ndarray, cout: int) -> np.ndarray:
    """[cout] -> [ng] vec4s with zero padding (pack.rs:178-184)."""
    out = np.zeros(cg(cout) * 4, np.float32)
    out[:cout] = np.asarray(b, np.float32).reshape(-1)
    return out


def unpack_weights_conv(packed: np.ndarray, cout: int, cin: int, kh: int, kw: int, kg_pad: int) -> np.ndarray:
    """Inverse of pack_weights_conv (pack.rs:124-151)."""
    ng = cg(cout)
    p = np.asarray(packed, np.float32).reshape(kh * kw, kg_pad, ng, 4, 4)
    full = p.transpose(2, 3, 1, 4, 0).reshape(ng * 4, kg_pad * 4, kh, kw)
    return np.ascontiguousarray(full[:cout, :cin]).reshape(-1)


def unpack_weights_dw(packed: np.ndarray, c: int, kh: int, kw: int) -> np.ndarray:
    """Inverse of pack_weights_dw (pack.rs:153-164)."""
    p = np.asarray(packed, np.float32).reshape(kh * kw, cg(c) * 4)
    return np.ascontiguousarray(p.T[:c]).reshape(-1)
