// Shared device helpers for the conv hot path (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace aie {

// Activation ids follow ai-core's Activation enum
// (crates/ai-core/src/activation.rs:7-24).
enum Act : int {
    kNone = 0, kRelu, kSigmoid, kTanh, kHardswish, kHardsigmoid, kClamp01, kRelu6, kSqrt, kNeg, kRecip
};

// Epilogue activation (crates/ai-core/src/activation.rs:28-43).
__device__ __forceinline__ float act_apply(int act, float x)
{
    switch (act) {
    case kRelu: return fmaxf(x, 0.0f);
    case kSigmoid: return 1.0f / (1.0f + expf(-x));
    case kTanh: return tanhf(x);
    case kHardswish: return x * fminf(fmaxf(x * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
    case kHardsigmoid: return fminf(fmaxf(x * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
    case kClamp01: return fminf(fmaxf(x, 0.0f), 1.0f);
    case kRelu6: return fminf(fmaxf(x, 0.0f), 6.0f);
    case kSqrt: return sqrtf(fmaxf(x, 0.0f));
    case kNeg: return -x;
    case kRecip: return 1.0f / x;
    default: return x;
    }
}

// The same activation with ai-cpu's rounding: channels below 4*floor(c/4)
// take apply4's form (multiply by the f32 constant 1/6, unfused), the tail
// takes Activation::apply's form (divide by 6)
// (crates/ai-cpu/src/kernels/mod.rs:21-50, conv.rs:190-235).
__device__ __forceinline__ float act_apply_strict(int act, float x, int ch, int c)
{
    const bool lane4 = ch < (c & ~3);
    switch (act) {
    case kRelu: return fmaxf(x, 0.0f);
    case kSigmoid: return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    case kTanh: return tanhf(x);
    case kHardswish:
    case kHardsigmoid: {
        float t = lane4 ? __fmul_rn(x, 1.0f / 6.0f) : __fdiv_rn(x, 6.0f);
        t = __fadd_rn(t, 0.5f);
        t = fminf(fmaxf(t, 0.0f), 1.0f);
        return act == kHardswish ? __fmul_rn(x, t) : t;
    }
    case kClamp01: return fminf(fmaxf(x, 0.0f), 1.0f);
    case kRelu6: return fminf(fmaxf(x, 0.0f), 6.0f);
    case kSqrt: return __fsqrt_rn(fmaxf(x, 0.0f));
    case kNeg: return -x;
    case kRecip: return __fdiv_rn(1.0f, x);
    default: return x;
    }
}

// Multiply-add in either fused (FFMA) or ai-cpu order-faithful unfused form.
template <bool kStrict>
__device__ __forceinline__ float madd(float acc, float a, float b)
{
    if constexpr (kStrict) return __fadd_rn(acc, __fmul_rn(a, b));
    else return fmaf(a, b, acc);
}

template <bool kStrict>
__device__ __forceinline__ float epi_act(int act, float x, int ch, int c)
{
    if constexpr (kStrict) return act_apply_strict(act, x, ch, c);
    else return act_apply(act, x);
}

template <bool kStrict>
__device__ __forceinline__ float add_res(float v, float r)
{
    if constexpr (kStrict) return __fadd_rn(v, r);
    else return v + r;
}

// Device error word set by bounded waits that give up (read and cleared by
// aie_device_status).  Bit layout: [31:24] kernel id, [23:0] site code.
// The library is one translation unit, so the definition lives here.
__device__ uint32_t g_aie_error = 0;

__device__ __forceinline__ void report_error(uint32_t code) { atomicCAS(&g_aie_error, 0u, code); }

}  // namespace aie
