"""B200-native (sm_100a) conv-as-GEMM hot path of ai_engine.

Kernels live in ``libaie_conv.so`` (C ABI: ``include/aie_conv.h``); this
package is the host-side mirror of ai_engine's conv operator surface.
"""
from .conv import ACTIVATIONS, Conv2d, ConvPlan, View, device_status, lower_conv, resize_bilinear  # noqa: F401

__all__ = ["ACTIVATIONS", "Conv2d", "ConvPlan", "View", "device_status", "lower_conv", "resize_bilinear"]
