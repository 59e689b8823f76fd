// Shared device helpers for the conv hot path (sm_100a).
#pragma once

#include <cuda.h>
#include <mutex>
#include <type_traits>
#include <utility>
#include <vector>
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

// Activation over a register array.  The switch sits outside the loop: a
// per-element switch on a runtime id compiles to one indirect branch per
// element, which cost ~10K cycles per 32 elements in the GEMM epilogue.
template <int N>
__device__ __forceinline__ void act_apply_n(int act, float (&v)[N])
{
    switch (act) {
    case kNone: break;
    case kRelu:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fmaxf(v[i], 0.0f);
        break;
    case kSigmoid:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = 1.0f / (1.0f + expf(-v[i]));
        break;
    case kTanh:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = tanhf(v[i]);
        break;
    case kHardswish:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = v[i] * fminf(fmaxf(v[i] * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
        break;
    case kHardsigmoid:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fminf(fmaxf(v[i] * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
        break;
    case kClamp01:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fminf(fmaxf(v[i], 0.0f), 1.0f);
        break;
    case kRelu6:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fminf(fmaxf(v[i], 0.0f), 6.0f);
        break;
    case kSqrt:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = sqrtf(fmaxf(v[i], 0.0f));
        break;
    case kNeg:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = -v[i];
        break;
    case kRecip:
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = 1.0f / v[i];
        break;
    default: break;
    }
}

// Activation with a compile-time kind where a kernel is instantiated for it
// (ACT >= 0: kNone, kRelu or kRelu6), else act_apply_n's runtime switch
// (ACT < 0).  In unrolled code the switch inlines every kind at each call:
// enough code to miss the instruction cache.
template <int ACT, int N>
__device__ __forceinline__ void act_fixed_n(int act, float (&v)[N])
{
    if constexpr (ACT == kNone) {
    } else if constexpr (ACT == kRelu) {
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fmaxf(v[i], 0.0f);
    } else if constexpr (ACT == kRelu6) {
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fminf(fmaxf(v[i], 0.0f), 6.0f);
    } else {
        act_apply_n<N>(act, v);
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

// madd on one pair (a0, a1) += (x0, x1) * (w0, w1), see madd4
template <bool kStrict>
__device__ __forceinline__ void madd2(float &a0, float &a1, const float2 &x, const float2 &w)
{
    if constexpr (kStrict) {
        // separate scalar roundings (the packed multiply and add measured
        // not bit-identical to them)
        a0 = __fadd_rn(a0, __fmul_rn(x.x, w.x));
        a1 = __fadd_rn(a1, __fmul_rn(x.y, w.y));
    } else {
        const float2 a = __ffma2_rn(x, w, make_float2(a0, a1));
        a0 = a.x;
        a1 = a.y;
    }
}

// madd over four channels: the fused form as two packed pairs (sm_100's
// two-wide FP32 FMA, one instruction per pair, each lane rounded exactly as
// fmaf); the strict form as separate scalar multiplies and adds in ai-cpu's
// order.
template <bool kStrict>
__device__ __forceinline__ void madd4(float (&acc)[4], const float4 &x, const float4 &w)
{
    float2 a0 = make_float2(acc[0], acc[1]), a1 = make_float2(acc[2], acc[3]);
    const float2 x0 = make_float2(x.x, x.y), x1 = make_float2(x.z, x.w);
    const float2 w0 = make_float2(w.x, w.y), w1 = make_float2(w.z, w.w);
    if constexpr (kStrict) {
        acc[0] = __fadd_rn(acc[0], __fmul_rn(x.x, w.x));
        acc[1] = __fadd_rn(acc[1], __fmul_rn(x.y, w.y));
        acc[2] = __fadd_rn(acc[2], __fmul_rn(x.z, w.z));
        acc[3] = __fadd_rn(acc[3], __fmul_rn(x.w, w.w));
        return;
    } else {
        a0 = __ffma2_rn(x0, w0, a0);
        a1 = __ffma2_rn(x1, w1, a1);
    }
    acc[0] = a0.x; acc[1] = a0.y; acc[2] = a1.x; acc[3] = a1.y;
}

// act_apply_strict over N consecutive channels starting at ch0, switch hoisted.
template <int N>
__device__ __forceinline__ void act_apply_strict_n(int act, float (&v)[N], int ch0, int c)
{
    if (act == kNone) return;
    if (act == kRelu) {
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = fmaxf(v[i], 0.0f);
        return;
    }
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = act_apply_strict(act, v[i], ch0 + i, c);
}

template <bool kStrict, int N>
__device__ __forceinline__ void epi_act_n(int act, float (&v)[N], int ch0, int c)
{
    if constexpr (kStrict) act_apply_strict_n<N>(act, v, ch0, c);
    else act_apply_n<N>(act, v);
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

// Division by a run-time divisor as multiply-high + shift (valid for
// 0 <= n < 2^31): the divisor's (mul, shift) pair is computed on the host.
struct FastDiv {
    int d;
    unsigned mul, shr;
};

static inline FastDiv make_fastdiv(int d)
{
    FastDiv f;
    f.d = d;
    if (d <= 1) {
        f.mul = 0;
        f.shr = 0;
        return f;
    }
    unsigned l = 0;
    while ((1ull << l) < (unsigned long long)d) l++;  // ceil(log2 d)
    const unsigned p = 31 + l;
    f.mul = (unsigned)(((1ull << p) + (unsigned long long)d - 1) / (unsigned long long)d);
    f.shr = p - 32;
    return f;
}

__device__ __forceinline__ int fdiv(int n, const FastDiv &f)
{
    return f.d <= 1 ? n : (int)(__umulhi((unsigned)n, f.mul) >> f.shr);
}

// ------------------------------------------------- mbarrier and TMA ---

constexpr unsigned long long kWaitNs = 1000000000ull;  // bounded waits give up after 1 s

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long gtime()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: true when the phase completed, false after `limit_ns`.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, unsigned long long limit_ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtime();
    while (true) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (gtime() - t0 > limit_ns) return false;
    }
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) { return mbar_wait_for(bar, parity, kWaitNs); }

// try_wait with a suspend-time hint: the thread may sleep (up to hint_ns)
// until the phase completes instead of polling, which frees issue slots for
// the warps that do the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for waits many warps share (they sleep between checks).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity)
{
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtime();
    while (!mbar_try_wait_sleep(bar, parity, 2000u))
        if (gtime() - t0 > kWaitNs) return false;
    return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1, int c2)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1, int c2,
                                            int c3)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// Device error word set by bounded waits that give up (read and cleared by
// aie_device_status).  Bit layout: [31:24] kernel id, [23:0] site code.
// The library is one translation unit, so the definition lives here.
__device__ uint32_t g_aie_error = 0;

__device__ __forceinline__ void report_error(uint32_t code) { atomicCAS(&g_aie_error, 0u, code); }

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize, and the shared-memory
// carveout when asked) once per kernel and device: the attributes belong to
// the function in each device's context
static inline cudaError_t ensure_smem_attr(const void *func, int bytes, bool max_carveout = false)
{
    static std::mutex mu;
    static std::vector<std::pair<const void *, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    for (const auto &f : done)
        if (f.first == func && f.second == dev) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && max_carveout)
        e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess) done.emplace_back(func, dev);
    return e;
}

}  // namespace aie
