// Fused inverted-bottleneck block on small frames: 1x1 expand -> depthwise
// 3x3 (stride 1, pad 1) -> 1x1 project (+ residual), one CTA per frame
// (persistent over frames), the expanded tensor never leaving the SM.
// ai-gpu-runtime dispatches the three convs one after another (lower_op's
// GemmPwSpec / ConvDwSpec arms, crates/ai-gpu-runtime/src/lowering.rs:99-187),
// writing and re-reading the expanded tensor twice.
//
// Both GEMMs are transposed so that the frame's pixels are the MMA's N side
// (N = 240: up to 10 rows at a stride of 24 pixels, up to 24 wide) and the
// channels its M side (M = 128):
//   E^T[c, p] = W_exp[c, :] . X[p, :]       (c: a 128-channel chunk of the
//                                            expanded dimension)
//   P^T[o, p] += W_proj[o, chunk] . D[p, chunk]
// so one tcgen05.mma covers 128 x 240 x 8 instead of 128 pixels x a narrow
// N: a chunk costs cin / 8 expand MMAs and 16 project MMAs per frame.
// The input frame arrives by TMA as [10 rows][24 px][32 ch] boxes (128-byte
// swizzle): columns and rows past the frame read as zeros, so pixel
// p = 24 y + x of the B operand is image pixel (y, x).
//
// Per chunk of 128 expanded channels (TMEM: E at columns [0, 240), P at
// [256, 496)):
//   1. the MMA warp accumulates E over cin (the producer streams the
//      [240][32] input K-blocks with the matching [128][32] expand-weight
//      K-blocks, two stages);
//   2. eight channel warps (thread = expanded channel; warp w reads TMEM
//      lanes 32 (w % 4).. and takes half the frame's rows) load E a frame
//      row at a time (three 8-column tcgen05.ld per row), add the expand
//      bias and activation, run the 3x3
//      depthwise on a sliding three-row register window (zero padding at the
//      frame's edges), add its bias and activation, and write D[p][channel]
//      into shared memory as the project GEMM's K-major B operand (128-byte
//      swizzle, one 32-channel K-block per warp);
//   3. the MMA warp accumulates P over the chunk's four K-blocks (the
//      producer streams the [128 out][32] project-weight K-blocks).
// After the last chunk the channel warps add the project bias, activation
// and residual and store the frame (thread = output channel: 32 lanes write
// one pixel's 128 contiguous bytes).
//
// Channels past the expanded width (the last chunk's padding) and output
// channels past cout read zero weights (TMA zero fill) and zero biases, so
// they contribute nothing.  Every wait is bounded; a wait that gives up
// sets the device error word and the CTA leaves its loop.
#pragma once

namespace aie {

constexpr int kMbRowStride = 24;                   // pixels per frame row in the N layout
constexpr int kMbRows = 10;                        // frame rows in the N layout
constexpr int kMbN = kMbRowStride * kMbRows;       // 240
constexpr int kMbChunk = 128;                      // expanded channels per chunk (MMA M)
constexpr uint32_t kMbXBytes = kMbN * 128;         // one [240][32] input K-block: 30 KB
constexpr uint32_t kMbWBytes = kMbChunk * 128;     // one [128][32] weight K-block: 16 KB
constexpr uint32_t kMbStage = kMbXBytes + kMbWBytes;
constexpr int kMbStages = 2;
constexpr uint32_t kMbDOff = kMbStages * kMbStage;  // D: 4 K-blocks of [240][32]
constexpr uint32_t kMbBarOff = kMbDOff + 4 * kMbXBytes;
constexpr uint32_t kMbSmem = kMbBarOff + 128 + 1024;  // + barriers + alignment slack
constexpr int kMbChanWarps = 8;                    // two per TMEM lane quarter: frame rows 0-4 / 5-9
constexpr int kMbHalfRows = kMbRows / 2;
constexpr int kMbThreads = 32 * (2 + kMbChanWarps);  // MMA, producer, channel warps
constexpr uint32_t kMbECol = 0, kMbPCol = 256;
static_assert(kMbStage % 1024 == 0 && kMbXBytes % 1024 == 0, "operand tiles stay 1024-aligned");
static_assert(kMbSmem <= 227 * 1024, "shared memory");

struct MbArgs {
    const float *x;        // [n][h][w][cin] dense
    const float *b_exp;    // [>= cexp]
    const float *w_dw;     // [9][cexp_pad4]
    const float *b_dw;     // [>= cexp]
    const float *b_proj;   // [>= cout]
    const float *res;      // [n][h][w][cout] dense, or nullptr
    float *y;              // [n][h][w][cout] dense
    int n, h, w, cin, cexp, cout, cexp_pad4;
    int act_exp, act_dw, act_proj;
};

struct MbShared {
    uint64_t full[kMbStages], empty[kMbStages];
    uint64_t e_full, e_empty, d_full, d_empty, p_full, p_empty, drain;
    uint32_t tmem_base;
    uint32_t abort;
};

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

// loads one frame row (24 columns) of this thread's TMEM lane
__device__ __forceinline__ void tmem_row24(uint32_t taddr, float (&v)[kMbRowStride])
{
    uint32_t r[24];
    tmem_ld8(taddr, *reinterpret_cast<uint32_t(*)[8]>(r));
    tmem_ld8(taddr + 8, *reinterpret_cast<uint32_t(*)[8]>(r + 8));
    tmem_ld8(taddr + 16, *reinterpret_cast<uint32_t(*)[8]>(r + 16));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23])
                 :
                 : "memory");
#pragma unroll
    for (int i = 0; i < kMbRowStride; i++) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kMbThreads, 1)
    mbconv_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmWe,
                  const __grid_constant__ CUtensorMap tmWp, const MbArgs a)
{
    extern __shared__ __align__(1024) uint8_t mb_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(mb_smem_raw) + 1023) & ~uintptr_t(1023));
    MbShared &sh = *reinterpret_cast<MbShared *>(smem + kMbBarOff);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunks = (a.cexp + kMbChunk - 1) / kMbChunk;
    const int kx = a.cin / 32;  // expand K-blocks (cin % 32 == 0, checked on the host)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMbStages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], 1);
        }
        mbar_init(&sh.e_full, 1);
        mbar_init(&sh.e_empty, kMbChanWarps);
        mbar_init(&sh.d_full, kMbChanWarps);
        mbar_init(&sh.d_empty, 1);
        mbar_init(&sh.p_full, 1);
        mbar_init(&sh.p_empty, kMbChanWarps);
        mbar_init(&sh.drain, 1);
        sh.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmWe)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmWp)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&sh.tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;
    volatile uint32_t *abort_flag = &sh.abort;

    if (warp == 1) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t it = 0;  // stages filled so far
            auto take = [&](uint32_t bytes, uint32_t &s) {
                s = it % kMbStages;
                if (!mbar_wait(&sh.empty[s], ((it / kMbStages) & 1) ^ 1)) return false;
                it++;
                mbar_expect_tx(&sh.full[s], bytes);
                return true;
            };
            bool ok = true;
            for (int f = blockIdx.x; ok && f < a.n; f += gridDim.x) {
                for (int ch = 0; ok && ch < nchunks; ch++) {
                    for (int kb = 0; ok && kb < kx; kb++) {
                        uint32_t s;
                        if (*abort_flag || !take(kMbStage, s)) { ok = false; break; }
                        uint8_t *st = smem + s * kMbStage;
                        tma_load_4d(st, &tmX, &sh.full[s], kb * 32, 0, 0, f);
                        tma_load_2d(st + kMbXBytes, &tmWe, &sh.full[s], kb * 32, ch * kMbChunk);
                    }
                    for (int kb = 0; ok && kb < 4; kb++) {
                        uint32_t s;
                        if (*abort_flag || !take(kMbWBytes, s)) { ok = false; break; }
                        tma_load_2d(smem + s * kMbStage + kMbXBytes, &tmWp, &sh.full[s], ch * kMbChunk + kb * 32, 0);
                    }
                }
            }
            if (!ok) {
                report_error(0x06000001u);
                *abort_flag = 1;
            }
            // no copy may land after exit: wait (bounded) for the last stages'
            // copies themselves (a stage is refilled only after its previous
            // copies were consumed, so earlier ones have landed)
            for (uint32_t j = it >= kMbStages ? it - kMbStages : 0; j < it; j++)
                mbar_wait(&sh.full[j % kMbStages], (j / kMbStages) & 1);
        }
    } else if (warp == 0) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32(128, kMbN);
            uint32_t it = 0, g = 0, j = 0;  // stages consumed, chunks, frames
            bool ok = true;
            auto stage = [&](uint32_t &s) {
                s = it % kMbStages;
                const uint32_t ph = (it / kMbStages) & 1;
                it++;
                return mbar_wait(&sh.full[s], ph);
            };
            for (int f = blockIdx.x; ok && f < a.n; f += gridDim.x, j++) {
                for (int ch = 0; ok && ch < nchunks; ch++, g++) {
                    // E is free once the channel warps have read the previous chunk's
                    if (g > 0 && !mbar_wait(&sh.e_empty, (g - 1) & 1)) { ok = false; break; }
                    tc_fence_after();
                    for (int kb = 0; kb < kx; kb++) {
                        uint32_t s;
                        if (*abort_flag || !stage(s)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t sx = smem_u32(smem + s * kMbStage), sw = sx + kMbXBytes;
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            mma_tf32(tmem + kMbECol, smem_desc_sw128(sw) + 2 * k, smem_desc_sw128(sx) + 2 * k, idesc,
                                     (kb > 0 || k > 0) ? 1u : 0u);
                        mma_commit(&sh.empty[s]);
                    }
                    if (!ok) break;
                    mma_commit(&sh.e_full);
                    // D of this chunk written; P free (first chunk of a frame)
                    if (!mbar_wait(&sh.d_full, g & 1)) { ok = false; break; }
                    if (ch == 0 && j > 0 && !mbar_wait(&sh.p_empty, (j - 1) & 1)) { ok = false; break; }
                    tc_fence_after();
                    for (int kb = 0; kb < 4; kb++) {
                        uint32_t s;
                        if (*abort_flag || !stage(s)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t sw = smem_u32(smem + s * kMbStage) + kMbXBytes;
                        const uint32_t sd = smem_u32(smem + kMbDOff + kb * kMbXBytes);
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            mma_tf32(tmem + kMbPCol, smem_desc_sw128(sw) + 2 * k, smem_desc_sw128(sd) + 2 * k, idesc,
                                     (ch > 0 || kb > 0 || k > 0) ? 1u : 0u);
                        mma_commit(&sh.empty[s]);
                    }
                    if (!ok) break;
                    mma_commit(&sh.d_empty);
                    if (ch == nchunks - 1) mma_commit(&sh.p_full);
                }
            }
            if (!ok) {
                report_error(0x06000002u);
                *abort_flag = 1;
            }
            // every MMA this thread issued completes before TMEM is freed
            mma_commit(&sh.drain);
            mbar_wait(&sh.drain, 0);
        }
    } else {
        // ------------------------------------------------------ channel warps
        // warp w reads TMEM lanes 32 (w % 4).. (one 32-channel K-block of D)
        // and takes frame rows [5 hf, 5 hf + 5), hf = (w - 2) / 4
        const int q = warp & 3;
        const int y0 = ((warp - 2) >> 2) * kMbHalfRows;
        const uint32_t tlane = tmem + ((uint32_t)(q * 32) << 16);
        uint8_t *dk = smem + kMbDOff + q * kMbXBytes;  // this warp's K-block of D
        // 128-byte swizzle: pixel p = 24 y + x has p % 8 == x % 8, so the
        // 16-byte chunk of this lane's channel in row p depends on x only
        const uint32_t lane_off = (uint32_t)((lane & 3) << 2);
        const int lane_chunk = lane >> 2;
        uint32_t g = 0, j = 0;
        bool ok = true;
        for (int f = blockIdx.x; ok && f < a.n; f += gridDim.x, j++) {
            for (int ch = 0; ch < nchunks; ch++, g++) {
                const int c = ch * kMbChunk + q * 32 + lane;  // expanded channel of this thread
                const bool cv = c < a.cexp;
                float wd[9];
#pragma unroll
                for (int t = 0; t < 9; t++) wd[t] = cv ? __ldg(a.w_dw + t * a.cexp_pad4 + c) : 0.0f;
                const float be = cv ? __ldg(a.b_exp + c) : 0.0f, bd = cv ? __ldg(a.b_dw + c) : 0.0f;
                // the warp's lanes decide together (the TMEM loads are warp-collective)
                if (!__all_sync(0xffffffffu, !*abort_flag && mbar_wait_sleep(&sh.e_full, g & 1))) { ok = false; break; }
                if (g > 0 && !__all_sync(0xffffffffu, mbar_wait_sleep(&sh.d_empty, (g - 1) & 1))) { ok = false; break; }
                tc_fence_after();
                // expand epilogue of frame row r: bias, activation, zero outside the frame
                auto erow = [&](int r, float (&v)[kMbRowStride]) {
                    if (r < 0 || r >= a.h) {
#pragma unroll
                        for (int x = 0; x < kMbRowStride; x++) v[x] = 0.0f;
                        return;
                    }
                    tmem_row24(tlane + kMbECol + r * kMbRowStride, v);
#pragma unroll
                    for (int x = 0; x < kMbRowStride; x++) v[x] += be;
                    act_apply_n<kMbRowStride>(a.act_exp, v);
#pragma unroll
                    for (int x = 0; x < kMbRowStride; x++)
                        if (x >= a.w) v[x] = 0.0f;
                };
                float rw[3][kMbRowStride];  // rows y-1, y, y+1 of the window (renamed by the unrolled loop)
                erow(y0 - 1, rw[0]);
                erow(y0, rw[1]);
#pragma unroll
                for (int i = 0; i < kMbHalfRows; i++) {
                    const int y = y0 + i;
                    float(&ra)[kMbRowStride] = rw[i % 3];
                    float(&rb)[kMbRowStride] = rw[(i + 1) % 3];
                    float(&rc)[kMbRowStride] = rw[(i + 2) % 3];
                    erow(y + 1, rc);
                    // taps in (ky, kx) order from the bias, as the depthwise kernels;
                    // half a row at a time (register budget)
                    uint8_t *drow = dk + y * (kMbRowStride * 128) + lane_off;
                    const bool yv = y < a.h;
#pragma unroll
                    for (int xh = 0; xh < kMbRowStride; xh += kMbRowStride / 2) {
                        float o[kMbRowStride / 2];
#pragma unroll
                        for (int xi = 0; xi < kMbRowStride / 2; xi++) {
                            const int x = xh + xi;
                            float acc = bd;
#pragma unroll
                            for (int dx = -1; dx <= 1; dx++)
                                if (x + dx >= 0 && x + dx < kMbRowStride) acc = fmaf(ra[x + dx], wd[dx + 1], acc);
#pragma unroll
                            for (int dx = -1; dx <= 1; dx++)
                                if (x + dx >= 0 && x + dx < kMbRowStride) acc = fmaf(rb[x + dx], wd[3 + dx + 1], acc);
#pragma unroll
                            for (int dx = -1; dx <= 1; dx++)
                                if (x + dx >= 0 && x + dx < kMbRowStride) acc = fmaf(rc[x + dx], wd[6 + dx + 1], acc);
                            o[xi] = acc;
                        }
                        act_apply_n<kMbRowStride / 2>(a.act_dw, o);
                        // D[p][lane], p = 24 y + x: K-major, 128-byte swizzle
#pragma unroll
                        for (int xi = 0; xi < kMbRowStride / 2; xi++) {
                            const int x = xh + xi;
                            *reinterpret_cast<float *>(drow + x * 128 + ((lane_chunk ^ (x & 7)) << 4)) =
                                (yv && x < a.w) ? o[xi] : 0.0f;
                        }
                    }
                }
                tc_fence_before();
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // D is read by the MMA (async proxy)
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sh.e_empty);
                    mbar_arrive(&sh.d_full);
                }
            }
            if (!ok) break;
            // ---- project epilogue of frame f: thread = output channel, this warp's rows
            if (!__all_sync(0xffffffffu, mbar_wait_sleep(&sh.p_full, j & 1))) { ok = false; break; }
            tc_fence_after();
            const int o = q * 32 + lane;
            const bool ov = o < a.cout;
            const float bp = ov ? __ldg(a.b_proj + o) : 0.0f;
            const long long fbase = (long long)f * a.h * a.w;
#pragma unroll 1
            for (int y = y0; y < min(y0 + kMbHalfRows, a.h); y++) {
                const long long m0 = fbase + (long long)y * a.w;
                float v[kMbRowStride];
                tmem_row24(tlane + kMbPCol + y * kMbRowStride, v);
#pragma unroll
                for (int x = 0; x < kMbRowStride; x++) v[x] += bp;
                act_apply_n<kMbRowStride>(a.act_proj, v);
                // residual after the activation; a half row of loads in flight at once
#pragma unroll
                for (int xh = 0; xh < kMbRowStride; xh += kMbRowStride / 2) {
                    float r[kMbRowStride / 2];
#pragma unroll
                    for (int xi = 0; xi < kMbRowStride / 2; xi++)
                        r[xi] = (a.res && ov && xh + xi < a.w) ? __ldg(a.res + (m0 + xh + xi) * a.cout + o) : 0.0f;
                    if (ov) {
#pragma unroll
                        for (int xi = 0; xi < kMbRowStride / 2; xi++)
                            if (xh + xi < a.w) a.y[(m0 + xh + xi) * a.cout + o] = v[xh + xi] + r[xi];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.p_empty);
        }
        if (!ok) {
            report_error(0x06000003u);
            *abort_flag = 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

}  // namespace aie
