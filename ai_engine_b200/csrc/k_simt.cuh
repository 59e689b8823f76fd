// CUDA-core kernels of the conv path: implicit-GEMM conv / 1x1 GEMM on FFMA,
// the cout<=4 pointwise dot kernel, and the depthwise conv.
//
// All three accumulate every output starting from its bias and walk taps in
// (ky, kx) order, then input channels in ascending order -- the order of
// ai-cpu's conv_std / conv_dw (crates/ai-cpu/src/kernels/conv.rs:238-334,
// dw.rs:100-200).  With kStrict the multiply and add are rounded separately
// (__fmul_rn/__fadd_rn), which reproduces ai-cpu's x86 results bit for bit
// (transcendental activations aside); without it each step is one FFMA.
#pragma once

#include "common.cuh"

namespace aie {

struct ConvArgs {
    const float *x;
    const float *w;
    const float *bias;
    const float *res;
    float *y;
    int n, ih, iw, cin, oh, ow, cout;
    int kh, kw, sh, sw, dil, pt, pl;
    long long x_stride, y_stride, r_stride;  // pixel strides in floats
    int x_coff, y_coff, r_coff;              // first channel of each view
    int act;
    int y_pad_to;    // output lanes [cout, y_pad_to) are written as zero
    long long M;     // n * oh * ow
    int wn;          // weight row stride in floats (GEMM: cout padded to 4)
    int vec_x;       // float4 input loads are aligned
    int vec_y;       // float4 output / residual accesses are aligned
    int res_mode;    // 0: residual tensor of the output's shape; 1/2: bilinear
                     // sample (half_pixel / asymmetric) of an rh x rw tensor
    int rh, rw;
    float rsy, rsx;  // rh / oh, rw / ow (f32 division, as the reference)
    FastDiv div_ow, div_oh;  // output pixel -> (frame, row, column)
    int res_up2;     // half_pixel sample with oh == 2 rh and ow == 2 rw
};

// Residual of output pixel m, channels [col, col+4), sampled bilinearly
// from the rh x rw residual tensor.  Same arithmetic, rounded step by step,
// as resize_bilinear_kernel / reference/resize.rs:5-42, so the fused
// Resize -> Conv(res) equals the unfused pair bit for bit.
struct BiTap {
    const float *p00, *p01, *p10, *p11;  // the four source pixels, channel col
    float tx, ty;                        // weights of the right column / lower row
};

__device__ __forceinline__ BiTap bilinear_tap(const ConvArgs &c, int mi, int col)
{
    const int t = fdiv(mi, c.div_ow);
    const int ox = mi - t * c.ow;
    const int img = fdiv(t, c.div_oh);
    const int oy = t - img * c.oh;
    int y0, y1, x0, x1;
    float ty, tx;
    if (c.res_up2) {
        // exact 2x: (oy + 0.5) * 0.5 - 0.5 = oy / 2 - 1/4 exactly, so its
        // floor is (oy - 1) >> 1 and its fraction 0.75 (oy even) or 0.25
        // (odd); the same rows and weights as the float path below
        const int fy = (oy - 1) >> 1, fx = (ox - 1) >> 1;
        y0 = max(fy, 0); y1 = min(fy + 1, c.rh - 1);
        x0 = max(fx, 0); x1 = min(fx + 1, c.rw - 1);
        ty = (oy & 1) ? 0.25f : 0.75f;
        tx = (ox & 1) ? 0.25f : 0.75f;
    } else {
        const float fy = c.res_mode == 1 ? __fsub_rn(__fmul_rn(__fadd_rn((float)oy, 0.5f), c.rsy), 0.5f)
                                         : __fmul_rn((float)oy, c.rsy);
        const float fx = c.res_mode == 1 ? __fsub_rn(__fmul_rn(__fadd_rn((float)ox, 0.5f), c.rsx), 0.5f)
                                         : __fmul_rn((float)ox, c.rsx);
        const float fly = floorf(fy), flx = floorf(fx);
        y0 = min(max((int)fly, 0), c.rh - 1); y1 = min(max((int)fly + 1, 0), c.rh - 1);
        x0 = min(max((int)flx, 0), c.rw - 1); x1 = min(max((int)flx + 1, 0), c.rw - 1);
        ty = fminf(fmaxf(__fsub_rn(fy, fly), 0.0f), 1.0f);
        tx = fminf(fmaxf(__fsub_rn(fx, flx), 0.0f), 1.0f);
    }
    const float *rb = c.res + (long long)img * c.rh * c.rw * c.r_stride + c.r_coff + col;
    BiTap b;
    b.p00 = rb + ((long long)y0 * c.rw + x0) * c.r_stride; b.p01 = rb + ((long long)y0 * c.rw + x1) * c.r_stride;
    b.p10 = rb + ((long long)y1 * c.rw + x0) * c.r_stride; b.p11 = rb + ((long long)y1 * c.rw + x1) * c.r_stride;
    b.tx = tx; b.ty = ty;
    return b;
}

// top = g00 (1-tx) + g01 tx, bot likewise, top (1-ty) + bot ty: each product
// and sum rounded on its own, the reference's order
__device__ __forceinline__ float4 bilinear_mix4(float4 g00, float4 g01, float4 g10, float4 g11, float tx, float ty)
{
    const float ty1 = __fsub_rn(1.0f, ty), tx1 = __fsub_rn(1.0f, tx);
    auto mix = [&](float a, float b, float c, float d) {
        const float top = __fadd_rn(__fmul_rn(a, tx1), __fmul_rn(b, tx));
        const float bot = __fadd_rn(__fmul_rn(c, tx1), __fmul_rn(d, tx));
        return __fadd_rn(__fmul_rn(top, ty1), __fmul_rn(bot, ty));
    };
    return make_float4(mix(g00.x, g01.x, g10.x, g11.x), mix(g00.y, g01.y, g10.y, g11.y),
                       mix(g00.z, g01.z, g10.z, g11.z), mix(g00.w, g01.w, g10.w, g11.w));
}

__device__ __forceinline__ float4 bilinear_res4(const ConvArgs &c, long long m, int col, bool vec)
{
    const BiTap b = bilinear_tap(c, (int)m, col);  // pixel counts are < 2^31 (checked at plan time)
    const float *p00 = b.p00, *p01 = b.p01, *p10 = b.p10, *p11 = b.p11;
    const float tx = b.tx, ty = b.ty;
    const float ty1 = __fsub_rn(1.0f, ty), tx1 = __fsub_rn(1.0f, tx);
    float g00[4], g01[4], g10[4], g11[4];
    if (vec) {
        const float4 a0 = __ldg(reinterpret_cast<const float4 *>(p00)), a1 = __ldg(reinterpret_cast<const float4 *>(p01));
        const float4 b0 = __ldg(reinterpret_cast<const float4 *>(p10)), b1 = __ldg(reinterpret_cast<const float4 *>(p11));
        g00[0] = a0.x; g00[1] = a0.y; g00[2] = a0.z; g00[3] = a0.w;
        g01[0] = a1.x; g01[1] = a1.y; g01[2] = a1.z; g01[3] = a1.w;
        g10[0] = b0.x; g10[1] = b0.y; g10[2] = b0.z; g10[3] = b0.w;
        g11[0] = b1.x; g11[1] = b1.y; g11[2] = b1.z; g11[3] = b1.w;
    } else {
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const bool ok = col + l < c.cout;
            g00[l] = ok ? __ldg(p00 + l) : 0.0f; g01[l] = ok ? __ldg(p01 + l) : 0.0f;
            g10[l] = ok ? __ldg(p10 + l) : 0.0f; g11[l] = ok ? __ldg(p11 + l) : 0.0f;
        }
    }
    float v[4];
#pragma unroll
    for (int l = 0; l < 4; l++) {
        const float top = __fadd_rn(__fmul_rn(g00[l], tx1), __fmul_rn(g01[l], tx));
        const float bot = __fadd_rn(__fmul_rn(g10[l], tx1), __fmul_rn(g11[l], tx));
        v[l] = __fadd_rn(__fmul_rn(top, ty1), __fmul_rn(bot, ty));
    }
    return make_float4(v[0], v[1], v[2], v[3]);
}

// ---------------------------------------------------------------------------
// Implicit-GEMM conv on FFMA.  C[M, cout] = sum_taps X_tap[M, cin] W_tap[cin, cout].
// CTA tile 128 x 64, K step 16, 256 threads, 8 x 4 outputs per thread.
// Weights: [tap][cin][wn] (the K-major form of ai-cpu's repack_weights,
// conv.rs:44-66, with cout padded to 4 instead of 8).
// ---------------------------------------------------------------------------
constexpr int kFfmaBM = 128, kFfmaBN = 64, kFfmaBK = 16, kFfmaThreads = 256;

template <bool kStrict>
__global__ void __launch_bounds__(kFfmaThreads) igemm_ffma_kernel(const ConvArgs a)
{
    constexpr int BM = kFfmaBM, BN = kFfmaBN, BK = kFfmaBK;
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const long long m0 = (long long)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;

    // A-load role: one output pixel (row) and 8 consecutive channels of it.
    const int ar = tid >> 1, ah = (tid & 1) * 8;
    const long long am = m0 + ar;
    const bool am_ok = am < a.M;
    int iy0 = 0, ix0 = 0;
    const float *xb = a.x;
    if (am_ok) {
        const long long hw = (long long)a.oh * a.ow;
        const int img = (int)(am / hw);
        const int rem = (int)(am - (long long)img * hw);
        const int oy = rem / a.ow, ox = rem - (rem / a.ow) * a.ow;
        iy0 = oy * a.sh - a.pt;
        ix0 = ox * a.sw - a.pl;
        xb = a.x + (long long)img * a.ih * a.iw * a.x_stride + a.x_coff;
    }
    // B-load role: one K row, 4 consecutive output channels.
    const int bk = tid >> 4, bn = (tid & 15) * 4;
    // Compute role.
    const int ty = tid >> 4, tx = tid & 15;

    const int kblocks = (a.cin + BK - 1) / BK;
    const int iters = a.kh * a.kw * kblocks;

    float ra[8];
    float4 rb;

    auto load = [&](int it) {
        const int t = it / kblocks, kb = it - t * kblocks;
        const int ky = t / a.kw, kx = t - ky * a.kw;
        const int iy = iy0 + ky * a.dil, ix = ix0 + kx * a.dil;
        const int c0 = kb * BK + ah;
        const bool ok = am_ok && iy >= 0 && iy < a.ih && ix >= 0 && ix < a.iw;
        if (ok) {
            const float *p = xb + ((long long)iy * a.iw + ix) * a.x_stride + c0;
            if (a.vec_x && c0 + 8 <= a.cin) {
                const float4 v0 = __ldg(reinterpret_cast<const float4 *>(p));
                const float4 v1 = __ldg(reinterpret_cast<const float4 *>(p + 4));
                ra[0] = v0.x; ra[1] = v0.y; ra[2] = v0.z; ra[3] = v0.w;
                ra[4] = v1.x; ra[5] = v1.y; ra[6] = v1.z; ra[7] = v1.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) ra[j] = (c0 + j < a.cin) ? __ldg(p + j) : 0.0f;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) ra[j] = 0.0f;
        }
        const int kr = kb * BK + bk;
        const int col = n0 + bn;
        if (kr < a.cin && col < a.wn)
            rb = __ldg(reinterpret_cast<const float4 *>(a.w + ((long long)t * a.cin + kr) * a.wn + col));
        else
            rb = make_float4(0.f, 0.f, 0.f, 0.f);
    };

    float acc[8][4];
    {
        float bv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int col = n0 + tx * 4 + j;
            bv[j] = col < a.cout ? a.bias[col] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = bv[j];
    }

    if (iters > 0) load(0);
    for (int it = 0; it < iters; it++) {
        const int buf = it & 1;
#pragma unroll
        for (int j = 0; j < 8; j++) As[buf][ah + j][ar] = ra[j];
        *reinterpret_cast<float4 *>(&Bs[buf][bk][bn]) = rb;
        __syncthreads();
        if (it + 1 < iters) load(it + 1);
#pragma unroll
        for (int k = 0; k < BK; k++) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 8 + 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float2 b01 = make_float2(b.x, b.y), b23 = make_float2(b.z, b.w);
            // output columns in packed pairs (two-wide FP32 instructions);
            // every output still accumulates over k in order
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float2 ai = make_float2(av[i], av[i]);
                madd2<kStrict>(acc[i][0], acc[i][1], ai, b01);
                madd2<kStrict>(acc[i][2], acc[i][3], ai, b23);
            }
        }
    }

    // Epilogue: bias (already in acc) -> act -> +residual
    // (crates/ai-gpu/src/kernels/common/epilogue.rs:13-30).
    const int col0 = n0 + tx * 4;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const long long m = m0 + ty * 8 + i;
        if (m >= a.M) break;
        float *yr = a.y + m * a.y_stride + a.y_coff;
        const float *rr = a.res ? a.res + m * a.r_stride + a.r_coff : nullptr;
        float v[4] = {acc[i][0], acc[i][1], acc[i][2], acc[i][3]};
        epi_act_n<kStrict, 4>(a.act, v, col0, a.cout);
        const bool vec = a.vec_y && col0 + 4 <= a.cout;
        if (a.res && a.res_mode) {
            const float4 r = bilinear_res4(a, m, col0, vec);
            v[0] = add_res<kStrict>(v[0], r.x); v[1] = add_res<kStrict>(v[1], r.y);
            v[2] = add_res<kStrict>(v[2], r.z); v[3] = add_res<kStrict>(v[3], r.w);
            rr = nullptr;
        }
        if (vec) {
            if (rr) {
                const float4 r = __ldg(reinterpret_cast<const float4 *>(rr + col0));
                v[0] = add_res<kStrict>(v[0], r.x); v[1] = add_res<kStrict>(v[1], r.y);
                v[2] = add_res<kStrict>(v[2], r.z); v[3] = add_res<kStrict>(v[3], r.w);
            }
            *reinterpret_cast<float4 *>(yr + col0) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int col = col0 + j;
                if (col < a.cout) yr[col] = rr ? add_res<kStrict>(v[j], rr[col]) : v[j];
                else if (col < a.y_pad_to) yr[col] = 0.0f;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// 1x1 conv with cout <= 4: one thread per pixel, cout dot products over cin.
// Weights [cout][cin] staged in shared memory.  Order of
// crates/ai-cpu/src/kernels/pw_dot.rs:44-58: four lane accumulators from
// zero (channel c feeds lane c % 4), summed as (l0+l1)+(l2+l3), then the
// bias, then the scalar activation on every channel.
// ---------------------------------------------------------------------------
template <bool kStrict>
__global__ void __launch_bounds__(256) pw_dot_kernel(const ConvArgs a)
{
    extern __shared__ float ws[];  // [cout][cin]
    const int nw = a.cout * a.cin;
    for (int i = threadIdx.x; i < nw; i += blockDim.x) ws[i] = a.w[i];
    __syncthreads();
    const long long m = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= a.M) return;
    const float *xr = a.x + m * a.x_stride + a.x_coff;
    float lane[4][4];
#pragma unroll
    for (int o = 0; o < 4; o++)
#pragma unroll
        for (int l = 0; l < 4; l++) lane[o][l] = 0.0f;
    int c = 0;
    if (a.vec_x) {
        for (; c + 4 <= a.cin; c += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(xr + c));
#pragma unroll
            for (int o = 0; o < 4; o++) {
                if (o < a.cout) {
                    const float *wr = ws + o * a.cin + c;
                    lane[o][0] = madd<kStrict>(lane[o][0], v.x, wr[0]);
                    lane[o][1] = madd<kStrict>(lane[o][1], v.y, wr[1]);
                    lane[o][2] = madd<kStrict>(lane[o][2], v.z, wr[2]);
                    lane[o][3] = madd<kStrict>(lane[o][3], v.w, wr[3]);
                }
            }
        }
    }
    for (; c < a.cin; c++) {
        const float v = __ldg(xr + c);
#pragma unroll
        for (int o = 0; o < 4; o++)
            if (o < a.cout) lane[o][c & 3] = madd<kStrict>(lane[o][c & 3], v, ws[o * a.cin + c]);
    }
    float *yr = a.y + m * a.y_stride + a.y_coff;
    const float *rr = a.res ? a.res + m * a.r_stride + a.r_coff : nullptr;
    float v[4];
#pragma unroll
    for (int o = 0; o < 4; o++) {
        const float s = __fadd_rn(__fadd_rn(lane[o][0], lane[o][1]), __fadd_rn(lane[o][2], lane[o][3]));
        v[o] = __fadd_rn(s, o < a.cout ? a.bias[o] : 0.0f);
    }
    // scalar activation form on every channel (pw_dot.rs:57): channel 0 of c=0 selects it
    epi_act_n<kStrict, 4>(a.act, v, 0, 0);
#pragma unroll
    for (int o = 0; o < 4; o++) {
        if (o < a.cout) yr[o] = rr ? add_res<kStrict>(v[o], rr[o]) : v[o];
        else if (o < a.y_pad_to) yr[o] = 0.0f;
    }
}

// Same op, memory-efficient form for cin = 4*CG (CG = 2, 4, 8, 16), 16-byte
// aligned input rows: each warp stages 32 pixels' input rows in shared
// memory with coalesced 16-byte loads (consecutive lanes read consecutive
// chunks), then each lane reduces its own pixel exactly as pw_dot_kernel
// does (lanes 4c..4c+3 in channel order, (l0+l1)+(l2+l3), + bias, act).
// Chunk q of row r is stored at position q ^ (r mod CG) so that both the
// row-major writes and the per-lane row reads are bank-conflict free.
template <bool kStrict, int CG>
__global__ void __launch_bounds__(256) pw_dot_tile_kernel(const ConvArgs a)
{
    constexpr int CIN = 4 * CG;
    extern __shared__ float4 sm4[];
    float *ws = reinterpret_cast<float *>(sm4);  // [cout][CIN], cout <= 4
    float4 *buf = sm4 + CIN + (threadIdx.x >> 5) * 32 * CG;  // this warp's 32 rows
    for (int i = threadIdx.x; i < a.cout * CIN; i += 256) ws[i] = a.w[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const long long m0 = ((long long)blockIdx.x * 8 + (threadIdx.x >> 5)) * 32;
    if (m0 >= a.M) return;
    const float *xb = a.x + a.x_coff;
#pragma unroll
    for (int j = 0; j < CG; j++) {
        const int f = j * 32 + lane;
        const int r = f / CG, q = f % CG;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m0 + r < a.M) v = __ldg(reinterpret_cast<const float4 *>(xb + (m0 + r) * a.x_stride + 4 * q));
        buf[r * CG + (q ^ (r % CG))] = v;
    }
    __syncwarp();
    const long long m = m0 + lane;
    float acc[4][4];
#pragma unroll
    for (int o = 0; o < 4; o++)
#pragma unroll
        for (int l = 0; l < 4; l++) acc[o][l] = 0.0f;
#pragma unroll
    for (int q = 0; q < CG; q++) {
        const float4 v = buf[lane * CG + (q ^ (lane % CG))];
#pragma unroll
        for (int o = 0; o < 4; o++) {
            if (o < a.cout) {
                const float4 w = reinterpret_cast<const float4 *>(ws + o * CIN)[q];
                madd4<kStrict>(acc[o], v, w);
            }
        }
    }
    if (m >= a.M) return;
    float *yr = a.y + m * a.y_stride + a.y_coff;
    const float *rr = a.res ? a.res + m * a.r_stride + a.r_coff : nullptr;
    float v[4];
#pragma unroll
    for (int o = 0; o < 4; o++) {
        const float s = __fadd_rn(__fadd_rn(acc[o][0], acc[o][1]), __fadd_rn(acc[o][2], acc[o][3]));
        v[o] = __fadd_rn(s, o < a.cout ? a.bias[o] : 0.0f);
    }
    epi_act_n<kStrict, 4>(a.act, v, 0, 0);  // scalar activation form (pw_dot.rs:57)
#pragma unroll
    for (int o = 0; o < 4; o++) {
        if (o < a.cout) yr[o] = rr ? add_res<kStrict>(v[o], rr[o]) : v[o];
        else if (o < a.y_pad_to) yr[o] = 0.0f;
    }
}

// ---------------------------------------------------------------------------
// Depthwise conv: one thread per (output pixel, 4-channel group); adjacent
// threads take adjacent channel groups so every tap load is a coalesced
// 128-bit access.  Weights [tap][c_pad4] (crates/ai-cpu/src/kernels/dw.rs:22-34),
// bias [c_pad4].  Memory-bound: the accumulation is always done unfused in
// ai-cpu's order, which costs nothing here.
// ---------------------------------------------------------------------------
template <bool kStrict>
__global__ void __launch_bounds__(256) dw_kernel(const ConvArgs a)
{
    const int cg = (a.cout + 3) >> 2;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= a.M * cg) return;
    const int g = (int)(idx % cg);
    const long long m = idx / cg;
    const long long hw = (long long)a.oh * a.ow;
    const int img = (int)(m / hw);
    const int rem = (int)(m - (long long)img * hw);
    const int oy = rem / a.ow, ox = rem - (rem / a.ow) * a.ow;
    const int c0 = g * 4;
    const int cpad = cg * 4;
    const float4 b4 = __ldg(reinterpret_cast<const float4 *>(a.bias) + g);
    float acc[4] = {b4.x, b4.y, b4.z, b4.w};
    const float *xb = a.x + (long long)img * a.ih * a.iw * a.x_stride + a.x_coff + c0;
    const bool full = a.vec_x && c0 + 4 <= a.cout;
    for (int ky = 0; ky < a.kh; ky++) {
        const int iy = oy * a.sh - a.pt + ky * a.dil;
        if (iy < 0 || iy >= a.ih) continue;
        for (int kx = 0; kx < a.kw; kx++) {
            const int ix = ox * a.sw - a.pl + kx * a.dil;
            if (ix < 0 || ix >= a.iw) continue;
            const float *p = xb + ((long long)iy * a.iw + ix) * a.x_stride;
            const float4 w4 = __ldg(reinterpret_cast<const float4 *>(a.w + (ky * a.kw + kx) * cpad + c0));
            float xv[4];
            if (full) {
                const float4 v = __ldg(reinterpret_cast<const float4 *>(p));
                xv[0] = v.x; xv[1] = v.y; xv[2] = v.z; xv[3] = v.w;
            } else {
#pragma unroll
                for (int l = 0; l < 4; l++) xv[l] = c0 + l < a.cout ? __ldg(p + l) : 0.0f;
            }
            acc[0] = madd<true>(acc[0], xv[0], w4.x);
            acc[1] = madd<true>(acc[1], xv[1], w4.y);
            acc[2] = madd<true>(acc[2], xv[2], w4.z);
            acc[3] = madd<true>(acc[3], xv[3], w4.w);
        }
    }
    float *yr = a.y + m * a.y_stride + a.y_coff + c0;
    const float *rr = a.res ? a.res + m * a.r_stride + a.r_coff + c0 : nullptr;
    float v[4] = {acc[0], acc[1], acc[2], acc[3]};
    epi_act_n<kStrict, 4>(a.act, v, c0, a.cout);
    if (a.vec_y && c0 + 4 <= a.cout) {
        if (rr) {
            const float4 r = __ldg(reinterpret_cast<const float4 *>(rr));
            v[0] = add_res<true>(v[0], r.x); v[1] = add_res<true>(v[1], r.y);
            v[2] = add_res<true>(v[2], r.z); v[3] = add_res<true>(v[3], r.w);
        }
        *reinterpret_cast<float4 *>(yr) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const int ch = c0 + l;
            if (ch < a.cout) yr[l] = rr ? add_res<true>(v[l], rr[l]) : v[l];
            else if (ch < a.y_pad_to) yr[l] = 0.0f;
        }
    }
}

// ---------------------------------------------------------------------------
// Bilinear resize (crates/ai-core/src/reference/resize.rs:5-42) with an
// optional fused add and activation.  One thread per (pixel, 4 channels).
// Multiplies and adds are rounded separately in the reference's order, so
// the result equals the CPU restatement bit for bit.
// ---------------------------------------------------------------------------
struct ResizeArgs {
    const float *x;
    const float *add;
    float *y;
    int n, ih, iw, c, oh, ow, mode, act;
    float sy, sx;
    int vec;
    FastDiv div_cg, div_owg, div_oh;
    int px_per_thread;  // output pixels per thread along x: 4 (c == 1, or c % 4 == 0 with
                        // aligned rows: a run of 4 pixels for one channel group), else 1
};

// Source coordinate along one axis (reference/resize.rs:16-29), rounded step
// by step: index pair, weight of the far sample.
__device__ __forceinline__ void resize_axis(int o, float scale, int mode, int in, int &i0, int &i1, float &t)
{
    const float f = mode == 0 ? __fsub_rn(__fmul_rn(__fadd_rn((float)o, 0.5f), scale), 0.5f) : __fmul_rn((float)o, scale);
    const float fl = floorf(f);
    i0 = min(max((int)fl, 0), in - 1);
    i1 = min(max((int)fl + 1, 0), in - 1);
    t = fminf(fmaxf(__fsub_rn(f, fl), 0.0f), 1.0f);
}

__device__ __forceinline__ float lerp2(float g00, float g01, float g10, float g11, float tx, float tx1, float ty,
                                       float ty1)
{
    const float top = __fadd_rn(__fmul_rn(g00, tx1), __fmul_rn(g01, tx));
    const float bot = __fadd_rn(__fmul_rn(g10, tx1), __fmul_rn(g11, tx));
    return __fadd_rn(__fmul_rn(top, ty1), __fmul_rn(bot, ty));
}

// Input staging: interleaved u8 RGB (cin = 3) or RGBA (cin = 4, alpha
// dropped) frames -> NHWC f32 in [0, 1], value = u8 / 255 with IEEE division
// (the reference normalises camera frames the same way: `v as f32 / 255.0`
// on the CPU, unorm texture sampling in ai-tasks' preprocess.wgsl:11-16).
// One thread converts 4 pixels; the C4 layout writes the 4th lane as zero.
__global__ void __launch_bounds__(256) input_u8_kernel(const uint8_t *__restrict__ in, float *__restrict__ out,
                                                        long long npix, int cin, int cout_stride)
{
    const long long p0 = ((long long)blockIdx.x * 256 + threadIdx.x) * 4;
    if (p0 >= npix) return;
    const int np = (int)min(4ll, npix - p0);
    uint8_t px[16];
    if (np == 4 && cin == 3 && ((uintptr_t)(in + p0 * 3) & 3) == 0) {
        const uint32_t *w = reinterpret_cast<const uint32_t *>(in + p0 * 3);
#pragma unroll
        for (int i = 0; i < 3; i++) {
            const uint32_t v = __ldg(w + i);
            px[4 * i] = v & 255; px[4 * i + 1] = (v >> 8) & 255; px[4 * i + 2] = (v >> 16) & 255; px[4 * i + 3] = v >> 24;
        }
    } else if (np == 4 && cin == 4 && ((uintptr_t)(in + p0 * 4) & 15) == 0) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(in + p0 * 4));
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            px[4 * i] = vv[i] & 255; px[4 * i + 1] = (vv[i] >> 8) & 255; px[4 * i + 2] = (vv[i] >> 16) & 255;
            px[4 * i + 3] = vv[i] >> 24;
        }
    } else {
        for (int i = 0; i < np * cin; i++) px[i] = in[p0 * cin + i];
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
        if (q >= np) break;
        float *o = out + (p0 + q) * cout_stride;
        const float r = __fdiv_rn((float)px[q * cin], 255.0f), gch = __fdiv_rn((float)px[q * cin + 1], 255.0f),
                    b = __fdiv_rn((float)px[q * cin + 2], 255.0f);
        if (cout_stride == 4) *reinterpret_cast<float4 *>(o) = make_float4(r, gch, b, 0.0f);
        else { o[0] = r; o[1] = gch; o[2] = b; }
    }
}

// YUV 4:2:0 camera frames (I420 planar, or NV12 / NV21 with interleaved
// chroma) -> the network's f32 RGB input.  The reference converts on the
// CPU, I420 -> RGBA8 (crates/ai-ffi/src/yuv.rs:7-31: BT.601 full range, f32
// with separate multiplies and adds, clamped to [0, 255] and truncated),
// and the model then reads each byte as v / 255.  One thread owns the 2 x 2
// pixel block that shares a chroma sample: the chroma products are formed
// once (the same products the reference forms per pixel), every sum is
// rounded on its own, so the result is bit for bit the reference's bytes
// divided by 255.
struct Yuv420Args {
    const uint8_t *y, *u, *v;
    long long fy, fu, fv;     // bytes between frames' planes
    int sy, su, sv, uv_step;  // row strides; bytes between horizontal chroma samples (1 planar, 2 interleaved)
    int n, h, w, ch, cw;      // ch, cw: chroma rows / columns = ceil(h / 2), ceil(w / 2)
    float *out;
    int ostride;              // 3 (NHWC) or 4 (NHWC-C4, 4th lane 0)
};

__device__ __forceinline__ float yuv_unorm(float c)
{
    c = fminf(fmaxf(c, 0.0f), 255.0f);                // Rust's clamp(0.0, 255.0)
    return __fdiv_rn((float)__float2int_rz(c), 255.0f);  // `as u8`, then v / 255
}

__global__ void __launch_bounds__(256) input_yuv420_kernel(const Yuv420Args a)
{
    const long long t = (long long)blockIdx.x * 256 + threadIdx.x;
    const long long per = (long long)a.ch * a.cw;
    if (t >= per * a.n) return;
    const int f = (int)(t / per);
    const int r = (int)(t - (long long)f * per);
    const int ci = r / a.cw, cj = r - ci * a.cw;
    const float uv = (float)__ldg(a.u + f * a.fu + (long long)ci * a.su + (long long)cj * a.uv_step) - 128.0f;
    const float vv = (float)__ldg(a.v + f * a.fv + (long long)ci * a.sv + (long long)cj * a.uv_step) - 128.0f;
    const float rv = __fmul_rn(1.402f, vv), gu = __fmul_rn(0.344136f, uv), gv = __fmul_rn(0.714136f, vv),
                bu = __fmul_rn(1.772f, uv);
#pragma unroll
    for (int dy = 0; dy < 2; dy++) {
        const int yy = 2 * ci + dy;
        if (yy >= a.h) break;
        const uint8_t *yrow = a.y + f * a.fy + (long long)yy * a.sy;
        float *orow = a.out + ((long long)f * a.h + yy) * a.w * a.ostride;
#pragma unroll
        for (int dx = 0; dx < 2; dx++) {
            const int xx = 2 * cj + dx;
            if (xx >= a.w) break;
            const float yv = (float)__ldg(yrow + xx);
            const float rr = yuv_unorm(__fadd_rn(yv, rv));
            const float gg = yuv_unorm(__fsub_rn(__fsub_rn(yv, gu), gv));
            const float bb = yuv_unorm(__fadd_rn(yv, bu));
            float *o = orow + (long long)xx * a.ostride;
            if (a.ostride == 4) *reinterpret_cast<float4 *>(o) = make_float4(rr, gg, bb, 0.0f);
            else { o[0] = rr; o[1] = gg; o[2] = bb; }
        }
    }
}

// Exact 2x upsampling in half_pixel mode (oh = 2*ih, ow = 2*iw; the FPN's
// and the mask's resizes).  Output (2i+a, 2j+b) samples source rows
// clamp(i-1+a), clamp(i+a) and columns clamp(j-1+b), clamp(j+b) with far
// weight 0.75 (a = 0) or 0.25 (a = 1): exactly the values resize_axis
// computes for this scale, combined in lerp2's order, so the result is bit
// for bit the general kernel's.  One thread owns a source pixel and writes
// its 2x2 output block from its 3x3 neighbourhood (2.25 loads per output
// instead of 4); C4: 4 channels per thread (C % 4 == 0, aligned), else C == 1
// with 4 source pixels per thread (iw % 4 == 0, aligned).
struct Up2Args {
    const float *x, *add;
    float *y;
    int n, ih, iw, c, act;
    FastDiv div_g, div_w, div_h;  // thread -> (group, source column, source row)
};

__device__ __forceinline__ float up2_lerp(float g00, float g01, float g10, float g11, float tx, float ty)
{
    return lerp2(g00, g01, g10, g11, tx, __fsub_rn(1.0f, tx), ty, __fsub_rn(1.0f, ty));
}

template <bool C1>
__global__ void __launch_bounds__(256) resize_up2_kernel(const Up2Args a)
{
    const int G = C1 ? 1 : a.c >> 2;                 // channel groups (C4) / 1
    const int W = C1 ? a.iw >> 2 : a.iw;             // thread columns per source row
    const int idx = blockIdx.x * 256 + threadIdx.x;  // < n*ih*W*G < 2^31 (checked on the host)
    if (idx >= a.n * a.ih * W * G) return;
    const int t = fdiv(idx, a.div_g), g = idx - t * G;
    const int r = fdiv(t, a.div_w), jw = t - r * W;
    const int img = fdiv(r, a.div_h), i = r - img * a.ih;
    const int oh = 2 * a.ih, ow = 2 * a.iw;
    const int rows[3] = {max(i - 1, 0), i, min(i + 1, a.ih - 1)};
    const float *xb = a.x + (long long)img * a.ih * a.iw * a.c;
    if constexpr (!C1) {
        const int j = jw, c0 = g * 4;
        const int cols[3] = {max(j - 1, 0), j, min(j + 1, a.iw - 1)};
        float4 v[3][3];
#pragma unroll
        for (int rr = 0; rr < 3; rr++)
#pragma unroll
            for (int cc = 0; cc < 3; cc++)
                v[rr][cc] = __ldg(reinterpret_cast<const float4 *>(xb + ((long long)rows[rr] * a.iw + cols[cc]) * a.c + c0));
#pragma unroll
        for (int ar = 0; ar < 2; ar++) {
            const float ty = ar ? 0.25f : 0.75f;
#pragma unroll
            for (int bc = 0; bc < 2; bc++) {
                const float tx = bc ? 0.25f : 0.75f;
                const float4 g00 = v[ar][bc], g01 = v[ar][bc + 1], g10 = v[ar + 1][bc], g11 = v[ar + 1][bc + 1];
                float o[4] = {up2_lerp(g00.x, g01.x, g10.x, g11.x, tx, ty), up2_lerp(g00.y, g01.y, g10.y, g11.y, tx, ty),
                              up2_lerp(g00.z, g01.z, g10.z, g11.z, tx, ty), up2_lerp(g00.w, g01.w, g10.w, g11.w, tx, ty)};
                const long long px = ((long long)img * oh + 2 * i + ar) * ow + 2 * j + bc;
                if (a.add) {
                    const float4 ad = __ldg(reinterpret_cast<const float4 *>(a.add + px * a.c + c0));
                    o[0] = __fadd_rn(o[0], ad.x); o[1] = __fadd_rn(o[1], ad.y);
                    o[2] = __fadd_rn(o[2], ad.z); o[3] = __fadd_rn(o[3], ad.w);
                }
                act_apply_strict_n<4>(a.act, o, c0, a.c);
                *reinterpret_cast<float4 *>(a.y + px * a.c + c0) = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    } else {
        // 4 source pixels j0..j0+3 (one float4 per row) plus their left and
        // right neighbours -> 8 output columns x 2 output rows
        const int j0 = jw * 4;
        float s[3][6];
#pragma unroll
        for (int rr = 0; rr < 3; rr++) {
            const float *row = xb + (long long)rows[rr] * a.iw;
            const float4 m = __ldg(reinterpret_cast<const float4 *>(row + j0));
            s[rr][0] = __ldg(row + max(j0 - 1, 0));
            s[rr][1] = m.x; s[rr][2] = m.y; s[rr][3] = m.z; s[rr][4] = m.w;
            s[rr][5] = __ldg(row + min(j0 + 4, a.iw - 1));
        }
#pragma unroll
        for (int ar = 0; ar < 2; ar++) {
            const float ty = ar ? 0.25f : 0.75f;
            float o[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const int bc = q & 1, k = (q >> 1) + bc;  // source columns k, k+1 of s (s[.][0] = j0-1)
                const float tx = bc ? 0.25f : 0.75f;
                o[q] = up2_lerp(s[ar][k], s[ar][k + 1], s[ar + 1][k], s[ar + 1][k + 1], tx, ty);
            }
            const long long px = ((long long)img * oh + 2 * i + ar) * ow + 2 * j0;
            if (a.add) {
#pragma unroll
                for (int q = 0; q < 8; q++) o[q] = __fadd_rn(o[q], __ldg(a.add + px + q));
            }
            act_apply_strict_n<8>(a.act, o, 0, 0);
            float4 *yr = reinterpret_cast<float4 *>(a.y + px);
            yr[0] = make_float4(o[0], o[1], o[2], o[3]);
            yr[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
    }
}

// C == 2 (the shipped segmentation model's two logits): a thread owns two
// source pixels (one float4 per source row: both channels of pixels j0 and
// j0 + 1) plus their left and right neighbours and writes 4 output columns x
// 2 output rows x 2 channels, with the same weights and lerp order as the
// other cases (iw even, 16-byte aligned input and output).
__global__ void __launch_bounds__(256) resize_up2_c2_kernel(const Up2Args a)
{
    const int W = a.iw >> 1;                         // thread columns per source row
    const int idx = blockIdx.x * 256 + threadIdx.x;  // < n*ih*W < 2^31 (checked on the host)
    if (idx >= a.n * a.ih * W) return;
    const int r = fdiv(idx, a.div_w), jw = idx - r * W;
    const int img = fdiv(r, a.div_h), i = r - img * a.ih;
    const int oh = 2 * a.ih, ow = 2 * a.iw;
    const int rows[3] = {max(i - 1, 0), i, min(i + 1, a.ih - 1)};
    const float *xb = a.x + (long long)img * a.ih * a.iw * 2;
    const int j0 = jw * 2;
    float s[3][4][2];  // source rows i-1..i+1 x columns j0-1..j0+2 x channels
#pragma unroll
    for (int rr = 0; rr < 3; rr++) {
        const float *row = xb + (long long)rows[rr] * a.iw * 2;
        const float4 m = __ldg(reinterpret_cast<const float4 *>(row + j0 * 2));
        const float2 lf = __ldg(reinterpret_cast<const float2 *>(row + max(j0 - 1, 0) * 2));
        const float2 rt = __ldg(reinterpret_cast<const float2 *>(row + min(j0 + 2, a.iw - 1) * 2));
        s[rr][0][0] = lf.x; s[rr][0][1] = lf.y;
        s[rr][1][0] = m.x;  s[rr][1][1] = m.y;
        s[rr][2][0] = m.z;  s[rr][2][1] = m.w;
        s[rr][3][0] = rt.x; s[rr][3][1] = rt.y;
    }
#pragma unroll
    for (int ar = 0; ar < 2; ar++) {
        const float ty = ar ? 0.25f : 0.75f;
        float o[8];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int bc = q & 1, k = (q >> 1) + bc;  // source columns k, k+1 of s (s[.][0] = j0-1)
            const float tx = bc ? 0.25f : 0.75f;
#pragma unroll
            for (int ch = 0; ch < 2; ch++)
                o[2 * q + ch] = up2_lerp(s[ar][k][ch], s[ar][k + 1][ch], s[ar + 1][k][ch], s[ar + 1][k + 1][ch], tx, ty);
        }
        const long long px = ((long long)img * oh + 2 * i + ar) * ow + 2 * j0;
        if (a.add) {
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = __fadd_rn(o[e], __ldg(a.add + px * 2 + e));
        }
        act_apply_strict_n<8>(a.act, o, 0, 2);  // two channels: ai-cpu's scalar activation for both
        float4 *yr = reinterpret_cast<float4 *>(a.y + px * 2);
        yr[0] = make_float4(o[0], o[1], o[2], o[3]);
        yr[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
}

__global__ void __launch_bounds__(256) resize_bilinear_kernel(const ResizeArgs a)
{
    const int cg = (a.c + 3) >> 2;
    const int idx = blockIdx.x * 256 + threadIdx.x;
    const int total = a.n * a.oh * ((a.ow + a.px_per_thread - 1) / a.px_per_thread) * cg;
    if (idx >= total) return;
    const int pxg = fdiv(idx, a.div_cg);  // pixel group index
    const int g = idx - pxg * cg;
    const int owg = (a.ow + a.px_per_thread - 1) / a.px_per_thread;
    const int row = fdiv(pxg, a.div_owg);  // img * oh + oy
    const int ox0 = (pxg - row * owg) * a.px_per_thread;
    const int img = fdiv(row, a.div_oh);
    const int oy = row - img * a.oh;
    int y0, y1;
    float ty;
    resize_axis(oy, a.sy, a.mode, a.ih, y0, y1, ty);
    const float ty1 = __fsub_rn(1.0f, ty);
    const float *xb = a.x + (long long)img * a.ih * a.iw * a.c;
    const float *r0 = xb + (long long)y0 * a.iw * a.c, *r1 = xb + (long long)y1 * a.iw * a.c;
    if (a.px_per_thread > 1 && a.c % 4 == 0) {  // a run of 4 output pixels, channels 4g..4g+3
        const int c0 = g * 4;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int ox = ox0 + p;
            if (ox >= a.ow) break;
            int x0, x1;
            float tx;
            resize_axis(ox, a.sx, a.mode, a.iw, x0, x1, tx);
            const float tx1 = __fsub_rn(1.0f, tx);
            const float4 g00 = __ldg(reinterpret_cast<const float4 *>(r0 + x0 * a.c + c0));
            const float4 g01 = __ldg(reinterpret_cast<const float4 *>(r0 + x1 * a.c + c0));
            const float4 g10 = __ldg(reinterpret_cast<const float4 *>(r1 + x0 * a.c + c0));
            const float4 g11 = __ldg(reinterpret_cast<const float4 *>(r1 + x1 * a.c + c0));
            float v[4];
            v[0] = lerp2(g00.x, g01.x, g10.x, g11.x, tx, tx1, ty, ty1);
            v[1] = lerp2(g00.y, g01.y, g10.y, g11.y, tx, tx1, ty, ty1);
            v[2] = lerp2(g00.z, g01.z, g10.z, g11.z, tx, tx1, ty, ty1);
            v[3] = lerp2(g00.w, g01.w, g10.w, g11.w, tx, tx1, ty, ty1);
            const long long px = (long long)row * a.ow + ox;
            if (a.add) {
                const float4 ad = __ldg(reinterpret_cast<const float4 *>(a.add + px * a.c + c0));
                v[0] = __fadd_rn(v[0], ad.x); v[1] = __fadd_rn(v[1], ad.y);
                v[2] = __fadd_rn(v[2], ad.z); v[3] = __fadd_rn(v[3], ad.w);
            }
            act_apply_strict_n<4>(a.act, v, c0, a.c);
            *reinterpret_cast<float4 *>(a.y + px * a.c + c0) = make_float4(v[0], v[1], v[2], v[3]);
        }
        return;
    }
    if (a.px_per_thread > 1) {  // single channel: 4 adjacent output pixels
        float v[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int ox = min(ox0 + p, a.ow - 1);
            int x0, x1;
            float tx;
            resize_axis(ox, a.sx, a.mode, a.iw, x0, x1, tx);
            v[p] = lerp2(__ldg(r0 + x0), __ldg(r0 + x1), __ldg(r1 + x0), __ldg(r1 + x1), tx, __fsub_rn(1.0f, tx), ty, ty1);
        }
        const long long ob = (long long)row * a.ow + ox0;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            if (ox0 + p >= a.ow) break;
            if (a.add) v[p] = __fadd_rn(v[p], __ldg(a.add + ob + p));
        }
        act_apply_strict_n<4>(a.act, v, 0, 0);
        if (a.vec && ox0 + 4 <= a.ow) {
            *reinterpret_cast<float4 *>(a.y + ob) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int p = 0; p < 4; p++)
                if (ox0 + p < a.ow) a.y[ob + p] = v[p];
        }
        return;
    }
    int x0, x1;
    float tx;
    resize_axis(ox0, a.sx, a.mode, a.iw, x0, x1, tx);
    const float tx1 = __fsub_rn(1.0f, tx);
    const int c0 = g * 4;
    const long long px = (long long)row * a.ow + ox0;
    float *yr = a.y + px * a.c + c0;
    const float *ar = a.add ? a.add + px * a.c + c0 : nullptr;
    const int nl = min(4, a.c - c0);
    float v[4];
    if (a.vec && nl == 4) {
        const float4 g00 = __ldg(reinterpret_cast<const float4 *>(r0 + x0 * a.c + c0));
        const float4 g01 = __ldg(reinterpret_cast<const float4 *>(r0 + x1 * a.c + c0));
        const float4 g10 = __ldg(reinterpret_cast<const float4 *>(r1 + x0 * a.c + c0));
        const float4 g11 = __ldg(reinterpret_cast<const float4 *>(r1 + x1 * a.c + c0));
        v[0] = lerp2(g00.x, g01.x, g10.x, g11.x, tx, tx1, ty, ty1);
        v[1] = lerp2(g00.y, g01.y, g10.y, g11.y, tx, tx1, ty, ty1);
        v[2] = lerp2(g00.z, g01.z, g10.z, g11.z, tx, tx1, ty, ty1);
        v[3] = lerp2(g00.w, g01.w, g10.w, g11.w, tx, tx1, ty, ty1);
        if (ar) {
            const float4 ad = __ldg(reinterpret_cast<const float4 *>(ar));
            v[0] = __fadd_rn(v[0], ad.x); v[1] = __fadd_rn(v[1], ad.y);
            v[2] = __fadd_rn(v[2], ad.z); v[3] = __fadd_rn(v[3], ad.w);
        }
        act_apply_strict_n<4>(a.act, v, c0, a.c);
        *reinterpret_cast<float4 *>(yr) = make_float4(v[0], v[1], v[2], v[3]);
        return;
    }
#pragma unroll
    for (int l = 0; l < 4; l++) {
        if (l < nl) {
            v[l] = lerp2(__ldg(r0 + x0 * a.c + c0 + l), __ldg(r0 + x1 * a.c + c0 + l), __ldg(r1 + x0 * a.c + c0 + l),
                         __ldg(r1 + x1 * a.c + c0 + l), tx, tx1, ty, ty1);
            if (ar) v[l] = __fadd_rn(v[l], __ldg(ar + l));
        } else {
            v[l] = 0.0f;
        }
    }
    act_apply_strict_n<4>(a.act, v, c0, a.c);
#pragma unroll
    for (int l = 0; l < 4; l++)
        if (l < nl) yr[l] = v[l];
}

}  // namespace aie

namespace aie {

// ---------------------------------------------------------------------------
// Small-cin direct conv (the stem: cin <= 4, k x k).  Persistent: each CTA
// walks tile_h x tile_w blocks of output pixels (all cout channels), with the
// next block's input halo prefetched into a second shared-memory buffer by
// cp.async while the current one is computed.  Each thread owns 4 output
// channels (lane % (cout/4)) and keeps their KK = kh*kw*cin weights in
// registers for the whole kernel, so the inner loop is one shared load per
// KK step feeding 4 FMAs.
// cout/4 consecutive lanes share one pixel, so every output store
// instruction writes whole 128-byte rows.  Accumulation order is bias, then
// (ky, kx, ic) -- ai-cpu's im2row stem order (crates/ai-cpu/src/kernels/
// im2row.rs:22-85 feeding conv_std).  Weights use the FFMA layout
// [tap][cin][wn].
// ---------------------------------------------------------------------------
struct StemGeom {
    int tile_h, tile_w, halo_h, halo_w, tiles_x, tiles_y;
    FastDiv div_tpi, div_tx;  // tile -> (frame, tile row, tile column)
};

template <bool kStrict, int KH, int KW, int CIN, int S, int TH, int TW>
__global__ void __launch_bounds__(256, 1) stem_kernel(const ConvArgs a, const StemGeom g)
{
    constexpr int KK = KH * KW * CIN;
    constexpr int HH = (TH - 1) * S + KH, HW = (TW - 1) * S + KW;  // halo block (dilation 1)
    constexpr int HROW = HW * CIN, HN = HH * HROW;
    constexpr int NPX = TH * TW;
    extern __shared__ float halo[];  // 2 x [HH][HW][CIN]
    const int tiles_per_img = g.tiles_x * g.tiles_y;
    const int ntiles = a.n * tiles_per_img;

    // Stage tile t's input halo into buffer `buf` with 4-byte cp.async;
    // out-of-frame elements are zero-filled (src-size 0) = the padding.
    auto stage = [&](int t, int buf) {
        const int img = t / tiles_per_img, rem = t - img * tiles_per_img;
        const int ty = rem / g.tiles_x, tx = rem - ty * g.tiles_x;
        const int iy0 = ty * TH * S - a.pt, ix0 = tx * TW * S - a.pl;
        const float *xb = a.x + (long long)img * a.ih * a.iw * a.x_stride + a.x_coff;
        float *dst = halo + buf * HN;
        for (int i = threadIdx.x; i < HN; i += 256) {
            const int cc = i % CIN, p = i / CIN;
            const int hy = p / HW, hx = p - hy * HW;
            const int iy = iy0 + hy, ix = ix0 + hx;
            const bool ok = iy >= 0 && iy < a.ih && ix >= 0 && ix < a.iw;
            const float *src = ok ? xb + ((long long)iy * a.iw + ix) * a.x_stride + cc : xb;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(
                             (uint32_t)__cvta_generic_to_shared(dst + i)),
                         "l"(src), "r"(ok ? 4 : 0)
                         : "memory");
        }
    };

    const int lpp = a.cout >> 2;  // lanes per pixel
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = (lane % lpp) * 4;  // this thread's 4 output channels
    float w[KK][4];
#pragma unroll
    for (int k = 0; k < KK; k++) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(a.w + (long long)k * a.wn + c0));
        w[k][0] = v.x; w[k][1] = v.y; w[k][2] = v.z; w[k][3] = v.w;
    }
    const float4 b4 = __ldg(reinterpret_cast<const float4 *>(a.bias + c0));
    const int ppw = 32 / lpp;       // pixels per warp per step
    const int step = 8 * ppw;       // pixels per CTA per step

    auto store = [&](int img, int oy, int ox, float (&acc)[4]) {
        epi_act_n<kStrict, 4>(a.act, acc, c0, a.cout);
        const long long m = ((long long)img * a.oh + oy) * a.ow + ox;
        if (a.res) {
            const float4 r = __ldg(reinterpret_cast<const float4 *>(a.res + m * a.r_stride + a.r_coff + c0));
            acc[0] = add_res<kStrict>(acc[0], r.x); acc[1] = add_res<kStrict>(acc[1], r.y);
            acc[2] = add_res<kStrict>(acc[2], r.z); acc[3] = add_res<kStrict>(acc[3], r.w);
        }
        *reinterpret_cast<float4 *>(a.y + m * a.y_stride + a.y_coff + c0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    };

    int t = blockIdx.x;
    if (t < ntiles) stage(t, 0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int i = 0; t < ntiles; t += gridDim.x, i++) {
        const int tn = t + gridDim.x;
        if (tn < ntiles) stage(tn, (i + 1) & 1);  // prefetch the next tile's halo
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");  // this tile's halo has landed
        __syncthreads();
        const float *hb = halo + (i & 1) * HN;
        const int img = t / tiles_per_img, rem = t - img * tiles_per_img;
        const int ty = rem / g.tiles_x, tx = rem - ty * g.tiles_x;
        const int oy0 = ty * TH, ox0 = tx * TW;
        // two pixels per thread per pass: 8 independent accumulator chains
        for (int p = warp * ppw + lane / lpp; p < NPX; p += 2 * step) {
            const int q = p + step;
            const bool has_q = q < NPX;
            const int dyp = p / TW, dxp = p - dyp * TW;
            const int dyq = q / TW, dxq = q - dyq * TW;
            const float *hp = hb + (dyp * S) * HROW + (dxp * S) * CIN;
            const float *hq = hb + (dyq * S) * HROW + (dxq * S) * CIN;
            float accp[4] = {b4.x, b4.y, b4.z, b4.w};
            float accq[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int ky = 0; ky < KH; ky++)
#pragma unroll
                for (int kx = 0; kx < KW; kx++)
#pragma unroll
                    for (int ic = 0; ic < CIN; ic++) {
                        constexpr int dummy = 0;
                        (void)dummy;
                        const int off = ky * HROW + kx * CIN + ic;
                        const int k = (ky * KW + kx) * CIN + ic;
                        const float xp = hp[off];
                        const float xq = has_q ? hq[off] : 0.0f;
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            accp[j] = madd<kStrict>(accp[j], xp, w[k][j]);
                            accq[j] = madd<kStrict>(accq[j], xq, w[k][j]);
                        }
                    }
            if (oy0 + dyp < a.oh && ox0 + dxp < a.ow) store(img, oy0 + dyp, ox0 + dxp, accp);
            if (has_q && oy0 + dyq < a.oh && ox0 + dxq < a.ow) store(img, oy0 + dyq, ox0 + dxq, accq);
        }
        __syncthreads();  // every thread is done with this buffer before it is refilled
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

}  // namespace aie

namespace aie {

// ---------------------------------------------------------------------------
// Depthwise conv, register-blocked: one thread computes PB horizontally
// adjacent output pixels x 4 channels.  Each input column it loads feeds
// every one of its outputs that the column's taps touch, so a row costs
// (PB-1)*S + K loads for PB outputs instead of PB*K (the 4-pixel blocking of
// crates/ai-cpu/src/kernels/dw.rs:100-145 and conv_dw.rs's PB).  Adjacent
// threads take adjacent channel groups, so every load and store is a
// coalesced 128-bit access.  Taps accumulate in (ky, kx) order: unfused
// (bit-identical to ai-cpu's conv_dw) in strict mode, fused multiply-adds
// otherwise.  Requires C % 4 == 0, aligned views, dilation 1.
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Depthwise conv, shared-memory halo tiles.  A CTA owns an 8 x TW block of
// output pixels and one 32-channel slice; it stages the input halo
// ((8-1)*S+K) x ((TW-1)*S+K) pixels x 32 channels with 16-byte cp.async
// (coalesced 128-byte pixel slices, zero fill = padding), then each thread
// computes 4 horizontally adjacent pixels x 4 channels from shared memory:
// every input element is read from L2/HBM once per CTA and no per-tap global
// address arithmetic remains.  Taps accumulate in (ky, kx) order, unfused in
// strict mode (bit-identical to ai-cpu's conv_dw, dw.rs:40-204) and fused
// otherwise.  Requires C % 4 == 0, 16-byte aligned views, dilation 1.
// ---------------------------------------------------------------------------
struct DwTile {
    int tiles_x, tiles_y, slices;
    FastDiv div_slices, div_tx, div_ty;  // block -> (slice, tile column, tile row, frame)
};

template <int K, int S, int TW>
struct DwTileGeom {
    static constexpr int TH = 8, PB = 4, RUNS = TW / PB, NT = TH * RUNS * 8;
    static constexpr int HH = (TH - 1) * S + K, HW = (TW - 1) * S + K;
    static constexpr int SMEM = HH * HW * 8 * 16 + 128;  // + slack for 128-byte alignment
    // exact-2x residual source patch (up-sampled-input mode): the source rows
    // and columns that the halo's pixels sample
    static constexpr int HHQ = (HH + 4) / 2, HWQ = (HW + 4) / 2;
    static constexpr int QSMEM = HHQ * HWQ * 8 * 16;
};

// Up-sampled input (UP2 = true): the depthwise input is x + up2(q), with q a
// dense [n][rh][rw][C] tensor and up2 the exact-2x half_pixel bilinear resize
// (reference/resize.rs:5-42): the FPN's Resize -> Conv(res) -> depthwise
// chain, where x is the lateral conv's output without its residual.  The sum
// is formed in the staged halo, so neither the up-sampled tensor nor the sum
// is written to memory.
struct DwUp2 {
    int rh, rw;
};

// Head mode (HEAD = true): the depthwise output feeds a 1x1 conv with at most
// 4 outputs (a segmentation head) that is applied in the same kernel: each
// thread dots its 4 channels of each of its 4 pixels with the 1x1 weights,
// the 8 lanes of a pixel group (its 32 channels) reduce by warp shuffle, and
// lane 0 of the group adds the bias, applies the activation and writes the
// <= 4 outputs.  The depthwise output never reaches memory.
struct PwHead {
    const float *w;     // [cout][cin] (pw_dot packing), cin = the depthwise channels (<= 32)
    const float *bias;  // [cout_pad4]
    float *y;
    long long y_stride;
    int y_coff, cout, act, y_pad_to;
};

// UP2 prologue: halo += up2(q) at every in-range pixel (padding stays zero).
// Rows 2k-1 and 2k of the up-sampled tensor sample the same two source rows
// clamp(k-1), clamp(k) (with row weights 0.25 / 0.75 swapped), and columns
// likewise, so one thread takes a 2 x 2 block of halo pixels for one channel
// group: four corner loads, the resize's top / bot rows for its two columns,
// then each pixel's mix: each lerp is a multiply and a fused multiply-add,
// the final mix two fused multiply-adds into the halo value, two channels
// per packed instruction (the head runs on the fused FFMA path; its bar is
// the FFMA tolerance, not the separate resize kernel's bits).  A tile whose
// halo starts on an odd row and column (pairs aligned with the halo: one
// pixel of padding, stride 1), lies inside the frame and samples no clamped
// source row or column mixes every pair without per-pixel range checks or
// clamps (with 8 x 16 tiles: every tile away from the frame's edge, 62% of
// them at 80 x 144).  Edge tiles keep the checks: replicating the patch's
// edge and re-zeroing the padding instead measured 4% slower.  The caller
// synchronises afterwards.
struct Up2Mix {  // a 4-channel value as two packed pairs
    float2 lo, hi;
};

__device__ __forceinline__ Up2Mix up2_split(const float4 v) { return {make_float2(v.x, v.y), make_float2(v.z, v.w)}; }

// p (1 - w) + q w, w in {0.25, 0.75}
__device__ __forceinline__ Up2Mix up2_lerp(const float4 p, const float4 q, float w1, float w)
{
    const float2 ww1 = make_float2(w1, w1), ww = make_float2(w, w);
    const Up2Mix pp = up2_split(p), qq = up2_split(q);
    return {__ffma2_rn(qq.lo, ww, __fmul2_rn(pp.lo, ww1)), __ffma2_rn(qq.hi, ww, __fmul2_rn(pp.hi, ww1))};
}

// dst += top (1 - w) + bot w
__device__ __forceinline__ void up2_mix_add(float4 *dst, const Up2Mix &top, const Up2Mix &bot, float w1, float w)
{
    const float4 v = *dst;
    const float2 ww1 = make_float2(w1, w1), ww = make_float2(w, w);
    const float2 lo = __ffma2_rn(bot.lo, ww, __ffma2_rn(top.lo, ww1, make_float2(v.x, v.y)));
    const float2 hi = __ffma2_rn(bot.hi, ww, __ffma2_rn(top.hi, ww1, make_float2(v.z, v.w)));
    *dst = make_float4(lo.x, lo.y, hi.x, hi.y);
}

template <int K, int S, int TW>
__device__ __forceinline__ void dw_up2_add(float4 *halo4, const float4 *qp, const ConvArgs &a, const DwUp2 &up, int iy0,
                                           int ix0, int qy0, int qx0)
{
    using G = DwTileGeom<K, S, TW>;
    constexpr int NT = G::NT, HH = G::HH, HW = G::HW, HWQ = G::HWQ;
    // pairs (2k-1, 2k) overlapping the halo: at most HH / 2 + 1 of them
    constexpr int NKY = HH / 2 + 1, NKX = HW / 2 + 1;
    const int ky0 = (iy0 + 1) >> 1, kx0 = (ix0 + 1) >> 1;  // pair holding the first halo row / column
    // halo rows / columns inside the image: [hy_lo, hy_hi) x [hx_lo, hx_hi)
    const int hy_lo = max(0, -iy0), hy_hi = min(HH, a.ih - iy0);
    const int hx_lo = max(0, -ix0), hx_hi = min(HW, a.iw - ix0);
    // first halo row / column of pair 0 (-1 when the halo starts at its second row)
    const int hy_k0 = 2 * ky0 - 1 - iy0, hx_k0 = 2 * kx0 - 1 - ix0;
    if constexpr (HH % 2 == 0 && HW % 2 == 0) {
        if (hy_k0 == 0 && hx_k0 == 0 && hy_lo == 0 && hy_hi == HH && hx_lo == 0 && hx_hi == HW && ky0 >= 1 &&
            ky0 + HH / 2 <= up.rh && kx0 >= 1 && kx0 + HW / 2 <= up.rw) {
            // pair (kyi, kxi) covers halo rows 2 kyi, 2 kyi + 1 and columns
            // 2 kxi, 2 kxi + 1, and samples patch rows kyi, kyi + 1 and
            // columns kxi, kxi + 1 (the patch starts at source row ky0 - 1
            // and column kx0 - 1)
            constexpr int PY = HH / 2, PX = HW / 2;
            static_assert(PY + 1 <= G::HHQ && PX + 1 <= HWQ, "the pairs' source rows lie in the patch");
            for (int t = threadIdx.x; t < PY * PX * 8; t += NT) {
                const int cg = t & 7, pk = t >> 3;
                const int kyi = pk / PX, kxi = pk - kyi * PX;  // compile-time divisor
                const float4 *q = qp + (kyi * HWQ + kxi) * 8 + cg;
                const float4 g00 = q[0], g01 = q[8], g10 = q[HWQ * 8], g11 = q[HWQ * 8 + 8];
                const Up2Mix top0 = up2_lerp(g00, g01, 0.75f, 0.25f), top1 = up2_lerp(g00, g01, 0.25f, 0.75f);
                const Up2Mix bot0 = up2_lerp(g10, g11, 0.75f, 0.25f), bot1 = up2_lerp(g10, g11, 0.25f, 0.75f);
                float4 *h = halo4 + (2 * kyi * HW + 2 * kxi) * 8 + cg;
                up2_mix_add(h, top0, bot0, 0.75f, 0.25f);
                up2_mix_add(h + 8, top1, bot1, 0.75f, 0.25f);
                up2_mix_add(h + HW * 8, top0, bot0, 0.25f, 0.75f);
                up2_mix_add(h + HW * 8 + 8, top1, bot1, 0.25f, 0.75f);
            }
            return;
        }
    }
    for (int t = threadIdx.x; t < NKY * NKX * 8; t += NT) {
        const int cg = t & 7, pk = t >> 3;
        const int kyi = pk / NKX, kxi = pk - kyi * NKX;  // compile-time divisor
        const int hy0 = hy_k0 + 2 * kyi, hx0 = hx_k0 + 2 * kxi;  // halo row / column of the pair's first pixel
        // rows hy0, hy0 + 1 and columns hx0, hx0 + 1 that lie in the image and the halo
        const bool ry0 = hy0 >= hy_lo && hy0 < hy_hi, ry1 = hy0 + 1 >= hy_lo && hy0 + 1 < hy_hi;
        const bool rx0 = hx0 >= hx_lo && hx0 < hx_hi, rx1 = hx0 + 1 >= hx_lo && hx0 + 1 < hx_hi;
        if (!((ry0 || ry1) && (rx0 || rx1))) continue;
        const int k = ky0 + kyi, j = kx0 + kxi;
        const int r0 = max(k - 1, 0) - qy0, r1 = min(k, up.rh - 1) - qy0;
        const int c0 = max(j - 1, 0) - qx0, c1 = min(j, up.rw - 1) - qx0;
        const float4 g00 = qp[(r0 * HWQ + c0) * 8 + cg], g01 = qp[(r0 * HWQ + c1) * 8 + cg];
        const float4 g10 = qp[(r1 * HWQ + c0) * 8 + cg], g11 = qp[(r1 * HWQ + c1) * 8 + cg];
        // columns 2j-1 (weight 0.25 on column clamp(j)) and 2j (0.75); rows likewise
        const Up2Mix top0 = up2_lerp(g00, g01, 0.75f, 0.25f), top1 = up2_lerp(g00, g01, 0.25f, 0.75f);
        const Up2Mix bot0 = up2_lerp(g10, g11, 0.75f, 0.25f), bot1 = up2_lerp(g10, g11, 0.25f, 0.75f);
        float4 *h = halo4 + (hy0 * HW + hx0) * 8 + cg;
        if (ry0 && rx0) up2_mix_add(h, top0, bot0, 0.75f, 0.25f);
        if (ry0 && rx1) up2_mix_add(h + 8, top1, bot1, 0.75f, 0.25f);
        if (ry1 && rx0) up2_mix_add(h + HW * 8, top0, bot0, 0.25f, 0.75f);
        if (ry1 && rx1) up2_mix_add(h + HW * 8 + 8, top1, bot1, 0.25f, 0.75f);
    }
}

// The depthwise conv of one staged tile (and, in head mode, the 1x1 head).
// Every thread of the CTA calls it (head mode shuffles across lanes).
template <bool kStrict, int K, int S, int TW, bool HEAD>
__device__ __forceinline__ void dw_tile_compute(const float4 *halo4, const ConvArgs &a, const PwHead &hd, int img, int ty,
                                                int tx, int c0, int ncg)
{
    using G = DwTileGeom<K, S, TW>;
    constexpr int TH = G::TH, PB = G::PB, RUNS = G::RUNS, HW = G::HW;
    const int cgi = threadIdx.x & 7, run = (threadIdx.x >> 3) % RUNS, row = threadIdx.x / (8 * RUNS);
    const int oy = ty * TH + row, ox0 = tx * TW + run * PB;
    const bool valid = cgi < ncg && oy < a.oh && ox0 < a.ow;
    if (!HEAD && !valid) return;  // head mode: every lane takes part in the shuffles
    const int ch = c0 + (valid ? cgi : 0) * 4;
    const int cpad = ((a.cout + 3) >> 2) << 2;
    const float4 b4 = __ldg(reinterpret_cast<const float4 *>(a.bias + ch));
    float acc[PB][4];
#pragma unroll
    for (int p = 0; p < PB; p++) {
        acc[p][0] = b4.x; acc[p][1] = b4.y; acc[p][2] = b4.z; acc[p][3] = b4.w;
    }
    constexpr int NJ = (PB - 1) * S + K;
#pragma unroll
    for (int ky = 0; ky < K; ky++) {
        float4 wk[K];
#pragma unroll
        for (int kx = 0; kx < K; kx++) wk[kx] = __ldg(reinterpret_cast<const float4 *>(a.w + (ky * K + kx) * cpad + ch));
        const float4 *hr = halo4 + ((row * S + ky) * HW + run * PB * S) * 8 + cgi;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const float4 xv = hr[j * 8];
#pragma unroll
            for (int p = 0; p < PB; p++) {
                const int kx = j - p * S;
                if (kx >= 0 && kx < K) madd4<kStrict>(acc[p], xv, wk[kx]);
            }
        }
    }
    if constexpr (HEAD) {
        static_assert(PB == 4, "the head's reduce-scatter spreads 4 pixels over 8 lanes");
        // partial dots of this lane's 4 channels for each of the group's 4
        // pixels, then a reduce-scatter over the 8 lanes of the pixel group:
        // the xor-4 step sums pixels {0, 1} into lanes with bit 2 clear and
        // {2, 3} into the others, xor-2 halves that again and xor-1 finishes,
        // so lanes 2p and 2p + 1 hold pixel p's sum (4 shuffles per output
        // instead of 12 for an all-reduce of every pixel)
        const bool b2 = (cgi & 4) != 0, b1 = (cgi & 2) != 0;
#pragma unroll
        for (int p = 0; p < PB; p++) epi_act_n<kStrict, 4>(a.act, acc[p], ch, a.cout);
        float sum[4];
#pragma unroll
        for (int o = 0; o < 4; o++) {
            sum[o] = 0.0f;
            if (o < hd.cout) {
                const float4 w = valid ? __ldg(reinterpret_cast<const float4 *>(hd.w + o * a.cout + ch))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
                float d[PB];
#pragma unroll
                for (int p = 0; p < PB; p++)
                    d[p] = fmaf(acc[p][3], w.w, fmaf(acc[p][2], w.z, fmaf(acc[p][1], w.y, acc[p][0] * w.x)));
                float k0 = b2 ? d[2] : d[0], k1 = b2 ? d[3] : d[1];
                k0 += __shfl_xor_sync(0xffffffffu, b2 ? d[0] : d[2], 4);
                k1 += __shfl_xor_sync(0xffffffffu, b2 ? d[1] : d[3], 4);
                float k = b1 ? k1 : k0;
                k += __shfl_xor_sync(0xffffffffu, b1 ? k0 : k1, 2);
                k += __shfl_xor_sync(0xffffffffu, k, 1);
                sum[o] = k;
            }
        }
        // the even lane of each pair finishes its pixel: bias, activation on
        // the real outputs only, store (padding lanes of a C4 view are zero)
        const int ox = ox0 + (b2 ? 2 : 0) + (b1 ? 1 : 0);
        if (!(cgi & 1) && oy < a.oh && ox < a.ow) {
            float v[4];
#pragma unroll
            for (int o = 0; o < 4; o++) v[o] = o < hd.cout ? act_apply(hd.act, sum[o] + __ldg(hd.bias + o)) : 0.0f;
            float *yr = hd.y + (((long long)img * a.oh + oy) * a.ow + ox) * hd.y_stride + hd.y_coff;
#pragma unroll
            for (int o = 0; o < 4; o++)
                if (o < hd.y_pad_to) yr[o] = v[o];
        }
    } else {
#pragma unroll
        for (int p = 0; p < PB; p++) {
            const int ox = ox0 + p;
            if (ox >= a.ow) break;
            epi_act_n<kStrict, 4>(a.act, acc[p], ch, a.cout);
            const long long m = ((long long)img * a.oh + oy) * a.ow + ox;
            if (a.res) {
                const float4 r = __ldg(reinterpret_cast<const float4 *>(a.res + m * a.r_stride + a.r_coff + ch));
                acc[p][0] = add_res<kStrict>(acc[p][0], r.x); acc[p][1] = add_res<kStrict>(acc[p][1], r.y);
                acc[p][2] = add_res<kStrict>(acc[p][2], r.z); acc[p][3] = add_res<kStrict>(acc[p][3], r.w);
            }
            *reinterpret_cast<float4 *>(a.y + m * a.y_stride + a.y_coff + ch) =
                make_float4(acc[p][0], acc[p][1], acc[p][2], acc[p][3]);
        }
    }
}

// kTma: the halo is one 4-D TMA box (32 channels, HW, HH, 1) of the input's
// (cin, iw, ih, n) tensor map, issued by one thread -- out-of-range pixels and
// channels read as zeros -- instead of one 16-byte cp.async per chunk with its
// index arithmetic (the staging was a sixth of the kernel's instructions).
// The body of dw_tile_kernel and dw_tile_up2_kernel (below).
template <bool kStrict, int K, int S, int TW, bool HEAD, bool kTma, bool UP2>
__device__ __forceinline__ void dw_tile_body(const CUtensorMap &tmx, const CUtensorMap &tmq, const ConvArgs &a,
                                             const DwTile &g, const PwHead &hd, const DwUp2 &up)
{
    static_assert(!UP2 || kTma, "the up-sampled input is staged by TMA");
    static_assert(!UP2 || !kStrict, "the up-sampled input is mixed with fused multiply-adds");
    using G = DwTileGeom<K, S, TW>;
    constexpr int TH = G::TH, NT = G::NT, HH = G::HH, HW = G::HW;
    extern __shared__ __align__(128) uint8_t dw_smem_raw[];
    // [HH][HW][8 channel groups], 128-byte aligned (a TMA destination)
    float4 *halo4 = reinterpret_cast<float4 *>((reinterpret_cast<uintptr_t>(dw_smem_raw) + 127) & ~uintptr_t(127));
    __shared__ uint64_t halo_bar;
    int b = blockIdx.x;
    const int q1 = fdiv(b, g.div_slices), slice = b - q1 * g.slices;
    const int q2 = fdiv(q1, g.div_tx), tx = q1 - q2 * g.tiles_x;
    const int img = fdiv(q2, g.div_ty), ty = q2 - img * g.tiles_y;
    const int c0 = slice * 32;
    const int ncg = min(8, (a.cout - c0) >> 2);
    const int iy0 = ty * TH * S - a.pt, ix0 = tx * TW * S - a.pl;
    if constexpr (kTma) {
        if (threadIdx.x == 0) {
            mbar_init(&halo_bar, 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        // UP2: source patch rows / columns from floor((first halo row - 1) / 2)
        float4 *qp = halo4 + HH * HW * 8;  // [G::HHQ][G::HWQ][8 channel groups]
        const int qy0 = (iy0 - 1) >> 1, qx0 = (ix0 - 1) >> 1;
        if (threadIdx.x == 0) {
            mbar_expect_tx(&halo_bar, (uint32_t)(HH * HW * 128 + (UP2 ? G::QSMEM : 0)));
            tma_load_4d(halo4, &tmx, &halo_bar, c0, ix0, iy0, img);
            if constexpr (UP2) tma_load_4d(qp, &tmq, &halo_bar, c0, qx0, qy0, img);
        }
        // bounded wait; the outcome is made CTA-uniform (head mode shuffles)
        const bool landed = mbar_wait_sleep(&halo_bar, 0);
        if (!__syncthreads_and(landed)) {
            if (threadIdx.x == 0) report_error(0x04000001u);
            return;
        }
        if constexpr (UP2) {
            dw_up2_add<K, S, TW>(halo4, qp, a, up, iy0, ix0, qy0, qx0);
            __syncthreads();
        }
    } else {
        const float *xb = a.x + (long long)img * a.ih * a.iw * a.x_stride + a.x_coff + c0;
        for (int i = threadIdx.x; i < HH * HW * 8; i += NT) {
            const int cgi = i & 7, pix = i >> 3;
            const int hy = pix / HW, hx = pix - hy * HW;
            const int iy = iy0 + hy, ix = ix0 + hx;
            const bool ok = cgi < ncg && iy >= 0 && iy < a.ih && ix >= 0 && ix < a.iw;
            const float *src = ok ? xb + ((long long)iy * a.iw + ix) * a.x_stride + cgi * 4 : a.x;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                             (uint32_t)__cvta_generic_to_shared(halo4 + i)),
                         "l"(src), "r"(ok ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
    }
    dw_tile_compute<kStrict, K, S, TW, HEAD>(halo4, a, hd, img, ty, tx, c0, ncg);
}

template <bool kStrict, int K, int S, int TW, bool HEAD = false, bool kTma = false>
__global__ void __launch_bounds__(DwTileGeom<K, S, TW>::NT)
    dw_tile_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmq, const ConvArgs a,
                   const DwTile g, const PwHead hd, const DwUp2 up)
{
    dw_tile_body<kStrict, K, S, TW, HEAD, kTma, false>(tmx, tmq, a, g, hd, up);
}

// The fused head with the up-sampled input asks for five CTAs per SM (at most
// 51 registers, a few bytes of spill): a CTA waits for its two TMA boxes with
// nothing else to do, and the fifth CTA hides more of that wait (head 194.7
// -> 186.2 us at 256 frames).  The other tile kernels keep the compiler's
// own register choice (an explicit minimum of one block let it take 128
// registers and halve their occupancy: 164 -> 242 us on 80x144x32).
template <int K, int S, int TW>
__global__ void __launch_bounds__(DwTileGeom<K, S, TW>::NT, 5)
    dw_tile_up2_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmq,
                       const ConvArgs a, const DwTile g, const PwHead hd, const DwUp2 up)
{
    dw_tile_body<false, K, S, TW, true, true, true>(tmx, tmq, a, g, hd, up);
}

// Persistent fused head (head mode, TMA staging): a CTA walks the tiles
// blockIdx.x, + gridDim.x, ... with two staging buffers, so the TMA loads of
// the tiles two ahead land while this tile computes -- a one-tile CTA waits
// for its load with nothing else to do.  Tile order and arithmetic are those
// of dw_tile_kernel<false, K, S, TW, true, true>.  (Measured on B200 at
// 256 x 80 x 144 x 32: 153 us against 172 us one tile per CTA.  With the
// up-sampled input the doubled staging leaves three CTAs per SM and the
// one-tile kernel wins, 235 against 266 us, so that mode stays one tile per
// CTA.)
template <int K, int S, int TW>
__global__ void __launch_bounds__(DwTileGeom<K, S, TW>::NT)
    dw_head_persistent_kernel(const __grid_constant__ CUtensorMap tmx, const ConvArgs a, const DwTile g,
                              const PwHead hd, const int tiles)
{
    using G = DwTileGeom<K, S, TW>;
    constexpr int TH = G::TH, HH = G::HH, HW = G::HW;
    constexpr uint32_t BUF = HH * HW * 128;
    static_assert(BUF % 128 == 0, "staging buffers stay 128-byte aligned");
    extern __shared__ __align__(128) uint8_t dw_smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dw_smem_raw) + 127) & ~uintptr_t(127));
    __shared__ uint64_t full[2];
    const int ncg = min(8, a.cout >> 2);
    if (threadIdx.x == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // tile -> (frame, tile row, tile column): one channel slice in head mode
    auto origin = [&](int t, int &img, int &ty, int &tx) {
        const int q2 = fdiv(t, g.div_tx);
        tx = t - q2 * g.tiles_x;
        img = fdiv(q2, g.div_ty);
        ty = q2 - img * g.tiles_y;
    };
    bool pend[2] = {false, false};  // thread 0: loads in flight per buffer
    auto issue = [&](int bsel, int t) {
        int img, ty, tx;
        origin(t, img, ty, tx);
        // the CTA's reads of this buffer (ordered by the barrier before the
        // call) come before the copy's writes
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&full[bsel], BUF);
        tma_load_4d(base + bsel * BUF, &tmx, &full[bsel], 0, tx * TW * S - a.pl, ty * TH * S - a.pt, img);
        pend[bsel] = true;
    };
    if (threadIdx.x == 0) {
        if ((int)blockIdx.x < tiles) issue(0, blockIdx.x);
        if ((int)(blockIdx.x + gridDim.x) < tiles) issue(1, blockIdx.x + gridDim.x);
    }
    uint32_t it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
        const int bsel = it & 1;
        // bounded wait; the outcome is made CTA-uniform (the head shuffles)
        const bool landed = mbar_wait_sleep(&full[bsel], (it >> 1) & 1);
        if (!__syncthreads_and(landed)) {
            if (threadIdx.x == 0) report_error(0x04000002u);
            break;
        }
        if (threadIdx.x == 0) pend[bsel] = false;
        int img, ty, tx;
        origin(t, img, ty, tx);
        dw_tile_compute<false, K, S, TW, true>(reinterpret_cast<const float4 *>(base + bsel * BUF), a, hd, img, ty, tx,
                                               0, ncg);
        __syncthreads();  // the buffer is free: stage the tile after next into it
        if (threadIdx.x == 0 && t + 2 * (int)gridDim.x < tiles) issue(bsel, t + 2 * gridDim.x);
    }
    // no copy may land after exit: wait (bounded) for loads still in flight
    if (threadIdx.x == 0)
        for (int bsel = 0; bsel < 2; bsel++)
            if (pend[bsel] && !mbar_wait(&full[bsel], ((it + (bsel != (int)(it & 1))) >> 1) & 1))
                report_error(0x04000003u);
}

struct DwGrid {
    int segs_per_row, cg;
    FastDiv div_cg, div_segs, div_oh;
};

// At most 64 registers (four 256-thread blocks per SM): the k5 stride-2 case
// needs 79 unconstrained and fits three; with the cap (a few bytes of spill)
// every depthwise layer measured 3-9% faster (e3.dw5s2 65.6 -> 63.5 us,
// RVM's dilated 5x5 layers 526 -> 482 us).
template <bool kStrict, int K, int S, int PB, int D = 1>
__global__ void __launch_bounds__(256, 4) dw_block_kernel(const ConvArgs a, const DwGrid gd)
{
    const int idx = blockIdx.x * 256 + threadIdx.x;  // < 2^31 (checked on the host)
    const int t = fdiv(idx, gd.div_cg);
    const int g = idx - t * gd.cg;
    const int rowid = fdiv(t, gd.div_segs);          // img * oh + oy
    const int seg = t - rowid * gd.segs_per_row;
    if (rowid >= a.n * a.oh) return;
    const int img = fdiv(rowid, gd.div_oh), oy = rowid - img * a.oh;
    const int cg = gd.cg;
    const int ox0 = seg * PB;
    const int c0 = g * 4;
    const int cpad = cg * 4;
    const float4 b4 = __ldg(reinterpret_cast<const float4 *>(a.bias) + g);
    float acc[PB][4];
#pragma unroll
    for (int p = 0; p < PB; p++) {
        acc[p][0] = b4.x; acc[p][1] = b4.y; acc[p][2] = b4.z; acc[p][3] = b4.w;
    }
    constexpr int NJ = (PB - 1) * S + (K - 1) * D + 1;  // input columns one row needs (dilation D)
    const int ixb = ox0 * S - a.pl;
#pragma unroll
    for (int ky = 0; ky < K; ky++) {
        const int iy = oy * S - a.pt + ky * D;
        if (iy < 0 || iy >= a.ih) continue;
        const float *row = a.x + ((long long)(img * a.ih + iy) * a.iw) * a.x_stride + a.x_coff + c0;
        float4 wk[K];
#pragma unroll
        for (int kx = 0; kx < K; kx++)
            wk[kx] = __ldg(reinterpret_cast<const float4 *>(a.w + (ky * K + kx) * cpad + c0));
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int ix = ixb + j;
            float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ix >= 0 && ix < a.iw) xv = __ldg(reinterpret_cast<const float4 *>(row + (long long)ix * a.x_stride));
#pragma unroll
            for (int p = 0; p < PB; p++) {
                // column j feeds tap kx of pixel p when j = p S + kx D
                const int r = j - p * S;
                const int kx = r / D;
                if (r >= 0 && r % D == 0 && kx < K) madd4<kStrict>(acc[p], xv, wk[kx]);
            }
        }
    }
#pragma unroll
    for (int p = 0; p < PB; p++) {
        const int ox = ox0 + p;
        if (ox >= a.ow) break;
        epi_act_n<kStrict, 4>(a.act, acc[p], c0, a.cout);
        const long long m = (long long)rowid * a.ow + ox;
        if (a.res) {
            const float4 r = __ldg(reinterpret_cast<const float4 *>(a.res + m * a.r_stride + a.r_coff + c0));
            acc[p][0] = add_res<true>(acc[p][0], r.x); acc[p][1] = add_res<true>(acc[p][1], r.y);
            acc[p][2] = add_res<true>(acc[p][2], r.z); acc[p][3] = add_res<true>(acc[p][3], r.w);
        }
        *reinterpret_cast<float4 *>(a.y + m * a.y_stride + a.y_coff + c0) =
            make_float4(acc[p][0], acc[p][1], acc[p][2], acc[p][3]);
    }
}

}  // namespace aie
