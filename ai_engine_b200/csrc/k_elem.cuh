// Graph glue around the convs: elementwise binary ops, the ConvGRU mix,
// global / windowed average pooling and channel copies (concat parts,
// channel slices, stand-alone activations).  These are the non-conv ops of
// ai_engine's recurrent matting and segmentation graphs
// (crates/ai-core/src/format/model.rs:111-214: Binary, Gpool, Avgpool,
// Concat, Chcopy, Act, Mix).
//
// All of them are HBM-bound streams: one thread owns one pixel's group of
// four channels, loads it as one 16-byte vector where every view allows
// (pixel stride, first channel and base 16-byte aligned, c % 4 == 0), and
// otherwise element by element.  Each result is rounded exactly as ai-cpu's
// x86 scalar-fallback kernels round it (crates/ai-cpu/src/kernels/
// elementwise.rs, pool.rs; unfused multiply and add), so the outputs are
// bit-identical to the CPU restatement except for the transcendental
// activations (expf / tanhf), which differ by at most an ulp or two.
#pragma once

namespace aie {

// A channel view of an NHWC batch: element (pixel q, channel ch) of a view
// lives at p[q * stride + coff + ch], q running over all frames' pixels.
struct EView {
    const float *p;
    long long stride;
    int coff;
};

__device__ __forceinline__ float ld_view(const EView &v, long long q, int ch)
{
    return v.p[q * v.stride + v.coff + ch];
}

__device__ __forceinline__ float4 ld_view4(const EView &v, long long q, int ch)
{
    return *reinterpret_cast<const float4 *>(v.p + q * v.stride + v.coff + ch);
}

// ai-core's BinaryOp (crates/ai-core/src/ops/elementwise.rs:5-27) in ai-cpu's
// 4-lane form (crates/ai-cpu/src/kernels/elementwise.rs:14-27): Sub is
// a + b * (-1), which rounds like a - b; Prelu is a > 0 ? a : a * b.
enum BinOp : int { kBinAdd = 0, kBinSub = 1, kBinMul = 2, kBinPrelu = 3 };

__device__ __forceinline__ float bin_apply(int op, float a, float b)
{
    switch (op) {
    case kBinAdd: return __fadd_rn(a, b);
    case kBinSub: return __fsub_rn(a, b);
    case kBinMul: return __fmul_rn(a, b);
    default: return a > 0.0f ? a : __fmul_rn(a, b);
    }
}

// Operand kinds of a Binary op's second input (SwOperand,
// crates/ai-core/src/format/model.rs:60-75).
enum BinOperand : int {
    kOpndTensor = 0,       // same shape as a
    kOpndScalar = 1,       // a o s
    kOpndScalarFirst = 2,  // s o a
    kOpndCvec = 3,         // [c] channel vector, every frame
    kOpndCvecTensor = 4,   // [n][c] channel vector per frame (an SE gate)
    kOpndPvecTensor = 5,   // [n * px] scalar per pixel, every channel
};

struct BinArgs {
    EView a, b;
    float *y;
    long long y_stride;
    int y_coff;
    long long Q;      // n * px
    unsigned px;      // pixels per frame
    int c, groups;    // channels, ceil(c / 4)
    int op, bkind, act;
    float scalar;
    bool vec;
};

__global__ void __launch_bounds__(256) binary_kernel(BinArgs a)
{
    const long long total = a.Q * a.groups;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long q = i / a.groups;
        const int ch0 = (int)(i - q * a.groups) * 4;
        const int nc = min(4, a.c - ch0);
        float x[4], s[4];
        if (a.vec) {
            const float4 v = ld_view4(a.a, q, ch0);
            x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
            for (int k = 0; k < 4; k++) x[k] = k < nc ? ld_view(a.a, q, ch0 + k) : 0.0f;
        }
        switch (a.bkind) {
        case kOpndTensor:
            if (a.vec) {
                const float4 v = ld_view4(a.b, q, ch0);
                s[0] = v.x; s[1] = v.y; s[2] = v.z; s[3] = v.w;
            } else {
                for (int k = 0; k < 4; k++) s[k] = k < nc ? ld_view(a.b, q, ch0 + k) : 0.0f;
            }
            break;
        case kOpndCvec:
            for (int k = 0; k < 4; k++) s[k] = k < nc ? a.b.p[ch0 + k] : 0.0f;
            break;
        case kOpndCvecTensor: {
            const long long f = q / a.px;
            for (int k = 0; k < 4; k++) s[k] = k < nc ? a.b.p[f * a.c + ch0 + k] : 0.0f;
            break;
        }
        case kOpndPvecTensor:
            for (int k = 0; k < 4; k++) s[k] = a.b.p[q];
            break;
        default:
            for (int k = 0; k < 4; k++) s[k] = a.scalar;
            break;
        }
        float r[4];
        const bool first = a.bkind == kOpndScalarFirst;
#pragma unroll
        for (int k = 0; k < 4; k++)
            r[k] = act_apply_strict(a.act, first ? bin_apply(a.op, s[k], x[k]) : bin_apply(a.op, x[k], s[k]),
                                    ch0 + k, a.c);
        float *yp = a.y + q * a.y_stride + a.y_coff + ch0;
        if (a.vec) {
            *reinterpret_cast<float4 *>(yp) = make_float4(r[0], r[1], r[2], r[3]);
        } else {
            for (int k = 0; k < nc; k++) yp[k] = r[k];
        }
    }
}

// GRU mix out = a + z (b - a) (SwOp::Mix, crates/ai-core/src/format/
// model.rs:193-199) in ai-cpu's order (crates/ai-cpu/src/kernels/
// elementwise.rs:128-150): channels below 4 floor(c / 4) compute
// (a + z b) + (-z) a, the tail a + z (b - a), each step rounded.
struct MixArgs {
    EView z, a, b;
    float *y;
    long long y_stride;
    int y_coff;
    long long Q;
    int c, groups;
    bool vec;
};

__device__ __forceinline__ float mix_one(float z, float a, float b, bool lane4)
{
    if (lane4) return __fadd_rn(__fadd_rn(a, __fmul_rn(z, b)), __fmul_rn(-z, a));
    return __fadd_rn(a, __fmul_rn(z, __fsub_rn(b, a)));
}

__global__ void __launch_bounds__(256) mix_kernel(MixArgs m)
{
    const long long total = m.Q * m.groups;
    const int cv = m.c & ~3;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long q = i / m.groups;
        const int ch0 = (int)(i - q * m.groups) * 4;
        float *yp = m.y + q * m.y_stride + m.y_coff + ch0;
        if (m.vec) {
            const float4 z = ld_view4(m.z, q, ch0), a = ld_view4(m.a, q, ch0), b = ld_view4(m.b, q, ch0);
            *reinterpret_cast<float4 *>(yp) = make_float4(mix_one(z.x, a.x, b.x, true), mix_one(z.y, a.y, b.y, true),
                                                          mix_one(z.z, a.z, b.z, true), mix_one(z.w, a.w, b.w, true));
        } else {
            const int nc = min(4, m.c - ch0);
            for (int k = 0; k < nc; k++)
                yp[k] = mix_one(ld_view(m.z, q, ch0 + k), ld_view(m.a, q, ch0 + k), ld_view(m.b, q, ch0 + k),
                                ch0 + k < cv);
        }
    }
}

// Global average pool [n][px][c] -> [n][c] (SwOp::Gpool; ai-cpu's
// reduction, crates/ai-cpu/src/kernels/segate.rs:46-57 and
// crates/ai-core/src/reference/pool.rs:6-19): each channel is summed over
// the frame's pixels in pixel order, then multiplied by the f32 1 / px.
// One thread owns four channels of one frame and walks the pixels with
// eight loads in flight; neighbouring threads read neighbouring channels,
// so each pixel row is one coalesced segment.
struct GpoolArgs {
    EView x;
    float *y;       // [n][c]
    int n, c, groups;
    unsigned px;
    float inv;
    bool vec;
};

__global__ void __launch_bounds__(128) gpool_kernel(GpoolArgs g)
{
    const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (t >= (long long)g.n * g.groups) return;
    const int f = (int)(t / g.groups);
    const int ch0 = (int)(t - (long long)f * g.groups) * 4;
    const int nc = min(4, g.c - ch0);
    const long long q0 = (long long)f * g.px;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    if (g.vec) {
        unsigned p = 0;
        for (; p + 8 <= g.px; p += 8) {
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; k++) v[k] = ld_view4(g.x, q0 + p + k, ch0);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                s0 = __fadd_rn(s0, v[k].x); s1 = __fadd_rn(s1, v[k].y);
                s2 = __fadd_rn(s2, v[k].z); s3 = __fadd_rn(s3, v[k].w);
            }
        }
        for (; p < g.px; p++) {
            const float4 v = ld_view4(g.x, q0 + p, ch0);
            s0 = __fadd_rn(s0, v.x); s1 = __fadd_rn(s1, v.y); s2 = __fadd_rn(s2, v.z); s3 = __fadd_rn(s3, v.w);
        }
    } else {
        for (unsigned p = 0; p < g.px; p++) {
            s0 = __fadd_rn(s0, ld_view(g.x, q0 + p, ch0));
            if (nc > 1) s1 = __fadd_rn(s1, ld_view(g.x, q0 + p, ch0 + 1));
            if (nc > 2) s2 = __fadd_rn(s2, ld_view(g.x, q0 + p, ch0 + 2));
            if (nc > 3) s3 = __fadd_rn(s3, ld_view(g.x, q0 + p, ch0 + 3));
        }
    }
    float *yp = g.y + (long long)f * g.c + ch0;
    const float r[4] = {__fmul_rn(s0, g.inv), __fmul_rn(s1, g.inv), __fmul_rn(s2, g.inv), __fmul_rn(s3, g.inv)};
    for (int k = 0; k < nc; k++) yp[k] = r[k];
}

// The same pool for 16-byte channel views, fed through shared memory: a CTA
// owns one frame and a slab of up to 128 channels (32 groups of four).  All
// 256 threads stream the frame's pixels into a ring of kGpStages stages of
// kGpStage float4 each (as many pixels per stage as fit: 512 / groups) with
// 16-byte cp.async copies, and thread t < groups folds group t's four
// channels over each landed stage in pixel order -- the same additions in
// the same order as gpool_kernel, bit for bit.  One thread per channel group
// walking the frame itself keeps too few bytes in flight (RVM's 36 x 64 x 72
// pools: 4,608 threads, ~1.8 TB/s); here every thread of the CTA has copies
// in flight for the stages ahead of the fold.
constexpr int kGpSlab = 32;     // channel groups (of four) per CTA
constexpr int kGpStage = 512;   // float4 per ring stage (8 KB)
constexpr int kGpStages = 6;    // ring stages (48 KB)

__global__ void __launch_bounds__(256) gpool_staged_kernel(GpoolArgs g)
{
    __shared__ __align__(16) float4 ring[kGpStages][kGpStage];
    const int f = (int)blockIdx.y;
    const int gbase = (int)blockIdx.x * kGpSlab;
    const int gs = min(kGpSlab, g.groups - gbase);  // groups in this slab
    const int ppc = kGpStage / gs;                   // pixels per stage
    const long long q0 = (long long)f * g.px;
    const int nchunks = (int)((g.px + ppc - 1) / ppc);
    const int items = ppc * gs;
    auto issue = [&](int chunk) {
        if (chunk < nchunks) {
            const unsigned p0 = (unsigned)chunk * ppc;
            float4 *st = ring[chunk % kGpStages];
            for (int i = threadIdx.x; i < items; i += blockDim.x) {
                const int pp = i / gs, gr = i - pp * gs;
                const bool ok = p0 + pp < g.px;
                const float *src = ok ? g.x.p + (q0 + p0 + pp) * g.x.stride + g.x.coff + (gbase + gr) * 4 : g.x.p;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                                 (uint32_t)__cvta_generic_to_shared(st + i)),
                             "l"(src), "r"(ok ? 16 : 0)
                             : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");  // one group per stage, empty past the last
    };
    for (int c = 0; c < kGpStages - 1; c++) issue(c);
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    for (int j = 0; j < nchunks; j++) {
        issue(j + kGpStages - 1);
        asm volatile("cp.async.wait_group %0;" ::"n"(kGpStages - 1) : "memory");  // stage j (this thread's part)
        __syncthreads();                                                         // everyone's part of stage j
        if ((int)threadIdx.x < gs) {
            const unsigned p0 = (unsigned)j * ppc;
            const int np = (int)min((unsigned)ppc, g.px - p0);
            const float4 *st = ring[j % kGpStages] + threadIdx.x;
            for (int pp = 0; pp < np; pp++) {
                const float4 v = st[pp * gs];
                s0 = __fadd_rn(s0, v.x); s1 = __fadd_rn(s1, v.y); s2 = __fadd_rn(s2, v.z); s3 = __fadd_rn(s3, v.w);
            }
        }
        __syncthreads();  // stage j is refilled by the next issue
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if ((int)threadIdx.x < gs) {
        const float4 r = make_float4(__fmul_rn(s0, g.inv), __fmul_rn(s1, g.inv), __fmul_rn(s2, g.inv),
                                     __fmul_rn(s3, g.inv));
        const int ch0 = (gbase + (int)threadIdx.x) * 4;
        float *yp = g.y + (long long)f * g.c + ch0;
        if (ch0 + 4 <= g.c && ((uintptr_t)yp % 16) == 0) {
            *reinterpret_cast<float4 *>(yp) = r;
        } else {
            const float rr[4] = {r.x, r.y, r.z, r.w};
            for (int k = 0; k < 4 && ch0 + k < g.c; k++) yp[k] = rr[k];
        }
    }
}

// Average pool with a fixed kh * kw divisor (SwOp::Avgpool;
// crates/ai-core/src/reference/pool.rs:22-46, the form RVM's decoder uses
// for its 2x2 / stride-2 input pyramid): taps summed in (ky, kx) order from
// zero, skipping those outside the frame, then multiplied by the f32
// 1 / (kh kw).  One thread per output pixel and four-channel group.
struct AvgpoolArgs {
    const float *x;
    float *y;
    int n, ih, iw, c, groups, oh, ow, kh, kw, sh, sw, pt, pl;
    float inv;
    bool vec;
};

__global__ void __launch_bounds__(256) avgpool_kernel(AvgpoolArgs a)
{
    const long long total = (long long)a.n * a.oh * a.ow * a.groups;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        long long r = i / a.groups;
        const int ch0 = (int)(i - r * a.groups) * 4;
        const int ox = (int)(r % a.ow);
        r /= a.ow;
        const int oy = (int)(r % a.oh);
        const int f = (int)(r / a.oh);
        const int nc = min(4, a.c - ch0);
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int ky = 0; ky < a.kh; ky++) {
            const int iy = oy * a.sh + ky - a.pt;
            if (iy < 0 || iy >= a.ih) continue;
            for (int kx = 0; kx < a.kw; kx++) {
                const int ix = ox * a.sw + kx - a.pl;
                if (ix < 0 || ix >= a.iw) continue;
                const float *xp = a.x + (((long long)f * a.ih + iy) * a.iw + ix) * a.c + ch0;
                if (a.vec) {
                    const float4 v = *reinterpret_cast<const float4 *>(xp);
                    s[0] = __fadd_rn(s[0], v.x); s[1] = __fadd_rn(s[1], v.y);
                    s[2] = __fadd_rn(s[2], v.z); s[3] = __fadd_rn(s[3], v.w);
                } else {
                    for (int k = 0; k < nc; k++) s[k] = __fadd_rn(s[k], xp[k]);
                }
            }
        }
        float *yp = a.y + (((long long)f * a.oh + oy) * a.ow + ox) * a.c + ch0;
        if (a.vec) {
            *reinterpret_cast<float4 *>(yp) = make_float4(__fmul_rn(s[0], a.inv), __fmul_rn(s[1], a.inv),
                                                          __fmul_rn(s[2], a.inv), __fmul_rn(s[3], a.inv));
        } else {
            for (int k = 0; k < nc; k++) yp[k] = __fmul_rn(s[k], a.inv);
        }
    }
}

// Channel copy out[q, 0:c] = act(in[q, 0:c]) between two channel views: a
// concat part written at its channel offset (SwOp::Concat), a channel slice
// (SwOp::Chcopy), or a stand-alone activation (SwOp::Act, with ai-cpu's
// apply4 / apply split, crates/ai-cpu/src/kernels/elementwise.rs:103-126).
struct CopyArgs {
    EView x;
    float *y;
    long long y_stride;
    int y_coff;
    long long Q;
    int c, groups, act;
    bool vec;
};

__global__ void __launch_bounds__(256) chcopy_kernel(CopyArgs a)
{
    const long long total = a.Q * a.groups;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long q = i / a.groups;
        const int ch0 = (int)(i - q * a.groups) * 4;
        float *yp = a.y + q * a.y_stride + a.y_coff + ch0;
        if (a.vec) {
            const float4 v = ld_view4(a.x, q, ch0);
            float r[4] = {v.x, v.y, v.z, v.w};
            if (a.act != kNone)
                for (int k = 0; k < 4; k++) r[k] = act_apply_strict(a.act, r[k], ch0 + k, a.c);
            *reinterpret_cast<float4 *>(yp) = make_float4(r[0], r[1], r[2], r[3]);
        } else {
            const int nc = min(4, a.c - ch0);
            for (int k = 0; k < nc; k++) yp[k] = act_apply_strict(a.act, ld_view(a.x, q, ch0 + k), ch0 + k, a.c);
        }
    }
}

}  // namespace aie

namespace aie {

// Channel concat of up to kConcatMax parts into one output view, one pass:
// a thread owns one output pixel's group of four channels, gathers them
// from whichever parts hold them and writes the group as one 16-byte store
// where the output allows.  Lanes past the parts' total (the zero padding
// of a buffer rounded up to a multiple of 4 channels) are written as zero.
// Compared with one copy per part, every output row is written once and
// whole: a part narrower than a 32-byte sector (the 3-channel frame in
// RVM's decoder concats) no longer makes the L2 fill and write back partial
// sectors.  (SwOp::Concat, crates/ai-core/src/format/model.rs:156-160.)
constexpr int kConcatMax = 8;

struct ConcatArgs {
    EView part[kConcatMax];
    int poff[kConcatMax + 1];   // first output channel of each part; poff[nparts] = parts' total
    int nparts;
    float *y;
    long long y_stride;
    int y_coff;
    unsigned Q;                 // n * px (< 2^31 / groups)
    int c_out, groups;          // output channels (>= the parts' total), ceil(c_out / 4)
    bool y_vec;
};

__global__ void __launch_bounds__(256) concat_kernel(ConcatArgs a)
{
    const unsigned total = a.Q * (unsigned)a.groups;
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const unsigned q = i / (unsigned)a.groups;
        const int ch0 = (int)(i - q * (unsigned)a.groups) * 4;
        float r[4];
        int p = 0;
        while (p + 1 < a.nparts && a.poff[p + 1] <= ch0) p++;
        const int lc = ch0 - a.poff[p];
        const EView &v = a.part[p];
        if (ch0 + 4 <= a.poff[p + 1] && ((uintptr_t)(v.p + (long long)q * v.stride + v.coff + lc) & 15) == 0) {
            const float4 t = ld_view4(v, q, lc);
            r[0] = t.x; r[1] = t.y; r[2] = t.z; r[3] = t.w;
        } else {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int ch = ch0 + k;
                int pp = p;
                while (pp < a.nparts && a.poff[pp + 1] <= ch) pp++;
                r[k] = pp < a.nparts ? ld_view(a.part[pp], q, ch - a.poff[pp]) : 0.0f;
            }
        }
        float *yp = a.y + (long long)q * a.y_stride + a.y_coff + ch0;
        if (a.y_vec) {
            *reinterpret_cast<float4 *>(yp) = make_float4(r[0], r[1], r[2], r[3]);
        } else {
            const int nc = min(4, a.c_out - ch0);
            for (int k = 0; k < nc; k++) yp[k] = r[k];
        }
    }
}

}  // namespace aie
