// 1x1 conv on the FP32 pipes for small channel counts (cin, cout in {32, 64}):
// the lateral convs of a feature pyramid, with bias, activation and residual
// fused -- either a residual tensor of the output's shape or the exact-2x
// half_pixel bilinear upsampling of a half-size tensor, so that a graph's
// Resize -> Conv(res) pair (ai-gpu-runtime lowering.rs Resize + Conv arms,
// reference/resize.rs:5-42 for the sampling) runs as one pass that reads the
// small tensor instead of writing and re-reading the upsampled one.
//
// Why not the tensor-core GEMM: at K = 32-64 a 128-pixel tile is four to
// eight MMAs, and the bilinear residual turns the tensor-core kernel's
// epilogue (one CTA per SM, eight epilogue warps) into the bottleneck.  Here
// several CTAs of eight warps per SM share the work, and the FFMA count
// (cin x cout per pixel) stays under the HBM time of the pass.
//
// Layout and work split:
//   - a CTA owns tiles of TP consecutive output pixels (persistent over
//     tiles); a tile's input rows [TP][cin] arrive by TMA as cin/32 boxes of
//     [TP pixels][32 channels] with 128-byte swizzle, two buffers deep (the
//     next tile loads while this one computes);
//   - thread (q, g) computes the 4 pixels q + r*TP/4 (r < 4) x the 8 output
//     channels [8g, 8g+8), g < cout/8, so TP = 4 * 256 / (cout/8);
//   - per 8 input channels: 8 shared loads of 16 bytes for the pixels, 16
//     for the weights, 256 FFMA (91% of the issue slots are FFMA);
//   - weights sit in shared memory as [k][half][g][4] (half = channels 4-7 of
//     a group) so that the 16-byte weight loads of a quarter-warp hit
//     distinct banks; the swizzle does the same for the pixel loads.
//
// Accumulation: fma over k = 0..cin-1 from zero, then + bias, activation,
// + residual (each rounded once): the FFMA family's order.  The bilinear
// residual is bit for bit the resize kernels' value.
#pragma once

namespace aie {

constexpr int kPwsThreads = 256;

struct PwsGeom {
    int tiles;  // ceil(M / TP) (< 2^31, checked at launch)
};

template <int CIN, int COUT>
struct PwsShape {
    static constexpr int CG = COUT / 8;                  // channel groups of 8
    static constexpr int TP = 4 * kPwsThreads / CG;      // pixels per tile
    static constexpr int QS = TP / 4;                    // pixel stride between a thread's 4 pixels
    static constexpr uint32_t XBYTES = TP * CIN * 4;     // one input buffer
    static constexpr uint32_t WBYTES = CIN * COUT * 4;
    // [x buffer 0][x buffer 1][weights][bias][2 mbarriers]; buffers 1024-aligned
    static constexpr uint32_t W_OFF = 2 * XBYTES;
    static constexpr uint32_t B_OFF = W_OFF + WBYTES;
    static constexpr uint32_t BAR_OFF = B_OFF + COUT * 4;
    static constexpr uint32_t SMEM = BAR_OFF + 16 + 1024;  // + alignment slack
    static_assert(COUT % 8 == 0 && kPwsThreads % CG == 0 && TP <= 256, "tile shape");
    static_assert(XBYTES % 1024 == 0, "buffers stay 1024-aligned for the 128-byte swizzle");
};

// exact-2x half_pixel sample of the rh x rw residual at output pixel m,
// channels [col, col+8): rows clamp((oy-1)>>1) and the next, weight 0.75 on
// the lower row for even oy and 0.25 for odd, likewise for columns -- the
// values the general resize computes for this scale, mixed in its order
__device__ __forceinline__ void pws_up2_res8(const ConvArgs &c, int m, int col, float (&rv)[8])
{
    const int t = fdiv(m, c.div_ow), ox = m - t * c.ow;
    const int img = fdiv(t, c.div_oh), oy = t - img * c.oh;
    const int fy = (oy - 1) >> 1, fx = (ox - 1) >> 1;
    const int y0 = max(fy, 0), y1 = min(fy + 1, c.rh - 1);
    const int x0 = max(fx, 0), x1 = min(fx + 1, c.rw - 1);
    const float ty = (oy & 1) ? 0.25f : 0.75f, tx = (ox & 1) ? 0.25f : 0.75f;
    const float *rb = c.res + (long long)img * c.rh * c.rw * c.r_stride + c.r_coff + col;
    const float *r0 = rb + (long long)y0 * c.rw * c.r_stride, *r1 = rb + (long long)y1 * c.rw * c.r_stride;
    const long long o0 = (long long)x0 * c.r_stride, o1 = (long long)x1 * c.r_stride;
    float4 g[4][2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        g[0][h] = __ldg(reinterpret_cast<const float4 *>(r0 + o0 + 4 * h));
        g[1][h] = __ldg(reinterpret_cast<const float4 *>(r0 + o1 + 4 * h));
        g[2][h] = __ldg(reinterpret_cast<const float4 *>(r1 + o0 + 4 * h));
        g[3][h] = __ldg(reinterpret_cast<const float4 *>(r1 + o1 + 4 * h));
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const float4 v = bilinear_mix4(g[0][h], g[1][h], g[2][h], g[3][h], tx, ty);
        rv[4 * h] = v.x; rv[4 * h + 1] = v.y; rv[4 * h + 2] = v.z; rv[4 * h + 3] = v.w;
    }
}

// RES: 0 none, 1 residual tensor of the output's shape, 2 exact-2x half_pixel
// bilinear sample of an rh x rw tensor (oh = 2 rh, ow = 2 rw)
template <int CIN, int COUT, int RES>
__global__ void __launch_bounds__(kPwsThreads, 2)
    pw_simt_kernel(const __grid_constant__ CUtensorMap tmx, const ConvArgs a, const PwsGeom g)
{
    using S = PwsShape<CIN, COUT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *ws = reinterpret_cast<float *>(smem + S::W_OFF);
    float *bs = reinterpret_cast<float *>(smem + S::B_OFF);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::BAR_OFF);
    const int tid = threadIdx.x;
    const int grp = tid % S::CG, q = tid / S::CG;

    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    // weights [k][o] (global, FFMA packing: cout % 4 == 0 so wn == cout) ->
    // [k][half][group][4]; bias
    for (int i = tid; i < CIN * COUT; i += kPwsThreads) {
        const int k = i / COUT, o = i - k * COUT;
        const int og = o >> 3, h = (o >> 2) & 1, e = o & 3;
        ws[k * COUT + h * (S::CG * 4) + og * 4 + e] = __ldg(a.w + (long long)k * a.wn + o);
    }
    for (int i = tid; i < COUT; i += kPwsThreads) bs[i] = __ldg(a.bias + i);
    __syncthreads();

    // thread 0 keeps the loads in flight: two tiles ahead
    bool pend[2] = {false, false};
    auto issue = [&](int b, int tile) {
        // the CTA's reads of this buffer (ordered by the barrier before the
        // call) come before the copy's writes
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&full[b], S::XBYTES);
#pragma unroll
        for (int s = 0; s < CIN / 32; s++)
            tma_load_2d(smem + b * S::XBYTES + s * (S::TP * 128), &tmx, &full[b], s * 32, tile * S::TP);
        pend[b] = true;
    };
    if (tid == 0) {
        if ((int)blockIdx.x < g.tiles) issue(0, blockIdx.x);
        if ((int)(blockIdx.x + gridDim.x) < g.tiles) issue(1, blockIdx.x + gridDim.x);
    }
    float bias[8];
#pragma unroll
    for (int j = 0; j < 8; j++) bias[j] = bs[grp * 8 + j];

    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < g.tiles; tile += gridDim.x, it++) {
        const int b = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        // every thread observes the load; the decision to go on is uniform
        const bool landed = mbar_wait(&full[b], ph);
        if (!__syncthreads_and(landed)) {
            report_error(0x05000001);
            break;
        }
        if (tid == 0) pend[b] = false;
        const uint8_t *xb = smem + b * S::XBYTES;
        float acc[4][8];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int j = 0; j < 8; j++) acc[r][j] = 0.0f;
#pragma unroll 1
        for (int kb = 0; kb < CIN / 8; kb++) {
            const uint8_t *sub = xb + (kb >> 2) * (S::TP * 128);
            const int j0 = (kb & 3) * 2;
            float x[4][8];
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int p = q + r * S::QS;
                const float4 lo = *reinterpret_cast<const float4 *>(sub + p * 128 + ((j0 ^ (p & 7)) * 16));
                const float4 hi = *reinterpret_cast<const float4 *>(sub + p * 128 + (((j0 + 1) ^ (p & 7)) * 16));
                x[r][0] = lo.x; x[r][1] = lo.y; x[r][2] = lo.z; x[r][3] = lo.w;
                x[r][4] = hi.x; x[r][5] = hi.y; x[r][6] = hi.z; x[r][7] = hi.w;
            }
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float *wr = ws + (kb * 8 + k) * COUT + grp * 4;
                const float4 w0 = *reinterpret_cast<const float4 *>(wr);
                const float4 w1 = *reinterpret_cast<const float4 *>(wr + S::CG * 4);
                const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int r = 0; r < 4; r++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[r][j] = fmaf(x[r][k], w[j], acc[r][j]);
            }
        }
        __syncthreads();  // the buffer is free: load the tile after next into it
        if (tid == 0 && tile + 2 * (int)gridDim.x < g.tiles) issue(b, tile + 2 * gridDim.x);

        // epilogue: bias -> activation -> + residual, 2 x 16 bytes per pixel
        const long long m_base = (long long)tile * S::TP;
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const long long m = m_base + q + r * S::QS;
            if (m >= a.M) continue;
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = acc[r][j] + bias[j];
            act_apply_n<8>(a.act, v);
            if constexpr (RES == 1) {
                const float *rr = a.res + m * a.r_stride + a.r_coff + grp * 8;
                const float4 r0 = __ldg(reinterpret_cast<const float4 *>(rr));
                const float4 r1 = __ldg(reinterpret_cast<const float4 *>(rr + 4));
                v[0] += r0.x; v[1] += r0.y; v[2] += r0.z; v[3] += r0.w;
                v[4] += r1.x; v[5] += r1.y; v[6] += r1.z; v[7] += r1.w;
            } else if constexpr (RES == 2) {
                float rv[8];
                pws_up2_res8(a, (int)m, grp * 8, rv);
#pragma unroll
                for (int j = 0; j < 8; j++) v[j] += rv[j];
            }
            float *yr = a.y + m * a.y_stride + a.y_coff + grp * 8;
            *reinterpret_cast<float4 *>(yr) = make_float4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<float4 *>(yr + 4) = make_float4(v[4], v[5], v[6], v[7]);
        }
    }
    // no copy may land after exit: wait (bounded) for loads still in flight
    if (tid == 0) {
        for (int b = 0; b < 2; b++)
            if (pend[b] && !mbar_wait(&full[b], ((it + (b != (int)(it & 1))) >> 1) & 1)) report_error(0x05000002);
    }
}

}  // namespace aie
