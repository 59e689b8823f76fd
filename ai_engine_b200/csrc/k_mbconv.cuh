// Fused inverted-bottleneck block on small frames: 1x1 expand -> depthwise
// 3x3 (stride 1, pad 1) -> 1x1 project (+ residual), one CTA per frame
// (persistent over frames), the expanded tensor never leaving the SM.
// ai-gpu-runtime dispatches the three convs one after another (lower_op's
// GemmPwSpec / ConvDwSpec arms, crates/ai-gpu-runtime/src/lowering.rs:99-187),
// writing and re-reading the expanded tensor twice.
//
// Both GEMMs are transposed so that the frame's pixels are the MMA's N side
// (N = 192: up to 10 rows of up to 18 pixels, row-major, then 12 zero rows)
// and the channels its M side (M = 128):
//   E^T[c, p] = W_exp[c, :] . X[p, :]       (c: a 128-channel chunk of the
//                                            expanded dimension)
//   P^T[o, p] += W_proj[o, chunk] . D[p, chunk]
// so one tcgen05.mma covers 128 x 192 x 8 instead of 128 pixels x a narrow
// N: a chunk costs cin / 8 expand MMAs and 16 project MMAs per frame.
// The input frame arrives by TMA as [10 rows][18 px][32 ch] boxes (128-byte
// swizzle): columns and rows past the frame read as zeros, so pixel
// p = 18 y + x of the B operand is image pixel (y, x).
//
// Per chunk of 128 expanded channels (TMEM: E at columns [0, 192), P at
// [256, 448)):
//   1. the MMA warp accumulates E over cin from an input ring (two [192][32]
//      K-blocks) and a weight ring (two [128][32] K-blocks);
//   2. eight channel warps (thread = expanded channel; warp w reads TMEM
//      lanes 32 (w % 4).. and takes half the frame's rows) copy the seven E
//      rows their five output rows need into registers and release E at
//      once; then they add the expand bias and activation, run the 3x3
//      depthwise (zero padding at the frame's edges), add its bias and
//      activation, and write D[p][channel] into shared memory as the project
//      GEMM's K-major B operand (128-byte swizzle, one 32-channel K-block per
//      lane quarter, in a ring of six K-block slots);
//   3. the MMA warp accumulates P over the chunk's four K-blocks, each as
//      soon as its two warps have written it; a slot is free again when the
//      project MMAs that read it complete (per-slot barriers).
// The MMA warp issues the expand of chunk g + 1 before the project of chunk
// g, so the next chunk's expand GEMM overlaps this chunk's depthwise on the
// CUDA cores; the producer loads the weights in that same order.
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

template <int V>
using Int = std::integral_constant<int, V>;

constexpr int kMbRowStride = 18;                   // pixels per frame row in the N layout (frame width <= 18)
constexpr int kMbRows = 10;                        // frame rows (frame height <= 10)
constexpr int kMbPix = kMbRowStride * kMbRows;     // 180
constexpr int kMbN = 192;                          // MMA N: the frame's pixels + 12 zero rows
constexpr int kMbChunk = 128;                      // expanded channels per chunk (MMA M)
constexpr uint32_t kMbXBytes = kMbN * 128;         // one [192][32] operand K-block: 24 KB
constexpr uint32_t kMbXBox = kMbPix * 128;         // the bytes a [10][18][32] TMA box writes
constexpr uint32_t kMbWBytes = kMbChunk * 128;     // one [128][32] weight K-block: 16 KB
constexpr int kMbXStages = 2, kMbWStages = 2;
// D K-blocks ([192][32], one per lane quarter) rotate through six slots: the
// quarter-q block of chunk g takes slot (4 g + q) % 6, so the next chunk's
// first two quarters write while the project GEMM still reads this chunk's,
// and its last two wait only for this chunk's first two K-blocks
constexpr int kMbDSlots = 6;
constexpr uint32_t kMbWOff = kMbXStages * kMbXBytes;
constexpr uint32_t kMbDOff = kMbWOff + kMbWStages * kMbWBytes;  // D: kMbDSlots K-blocks of [192][32]
constexpr uint32_t kMbBarOff = kMbDOff + kMbDSlots * kMbXBytes;
constexpr uint32_t kMbSmem = kMbBarOff + 256 + 1024;  // + barriers + alignment slack
constexpr int kMbChanWarps = 8;                     // two per TMEM lane quarter: frame rows 0-4 / 5-9
constexpr int kMbHalfRows = kMbRows / 2;
constexpr int kMbThreads = 32 * (2 + kMbChanWarps);  // MMA, producer, channel warps
constexpr uint32_t kMbECol = 0, kMbPCol = 256;
static_assert(kMbXBytes % 1024 == 0 && kMbWBytes % 1024 == 0 && kMbWOff % 1024 == 0 && kMbDOff % 1024 == 0,
              "operand tiles stay 1024-aligned");
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
    uint64_t xfull[kMbXStages], xempty[kMbXStages], wfull[kMbWStages], wempty[kMbWStages];
    uint64_t d_full[kMbDSlots], d_empty[kMbDSlots];
    uint64_t e_full, e_empty, p_full, p_empty, drain;
    uint32_t tmem_base;
    uint32_t abort;
};
static_assert(sizeof(MbShared) <= 256, "barrier block");

__device__ __forceinline__ void tmem_ld2(uint32_t taddr, uint32_t &r0, uint32_t &r1)
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(taddr));
}

// one frame row (18 columns) of this thread's TMEM lane
__device__ __forceinline__ void tmem_row18(uint32_t taddr, float (&v)[kMbRowStride])
{
    uint32_t r[kMbRowStride];
#pragma unroll
    for (int k = 0; k < kMbRowStride / 2; k++) tmem_ld2(taddr + 2 * k, r[2 * k], r[2 * k + 1]);
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17])
                 :
                 : "memory");
#pragma unroll
    for (int i = 0; i < kMbRowStride; i++) v[i] = __uint_as_float(r[i]);
}

// tcgen05.wait::ld naming 18 load destinations as read-write operands, so
// no use of them moves above the wait (after the first wait the loads have
// all landed; further ones only pin their registers)
__device__ __forceinline__ void tmem_wait_pin18(uint32_t (&r)[kMbRowStride])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17])
                 :
                 : "memory");
}

// AE, AD: the expand and depthwise activations (kRelu / kRelu6 / kNone, or
// -1 for any kind at run time).  DW = false: no depthwise (a 1x1 expand
// straight into a 1x1 project): the channel warps store the activated E
// rows as D.
template <int AE, int AD, bool DW = true>
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
        for (int s = 0; s < kMbXStages; s++) {
            mbar_init(&sh.xfull[s], 1);
            mbar_init(&sh.xempty[s], 1);
        }
        for (int s = 0; s < kMbWStages; s++) {
            mbar_init(&sh.wfull[s], 1);
            mbar_init(&sh.wempty[s], 1);
        }
        mbar_init(&sh.e_full, 1);
        mbar_init(&sh.e_empty, kMbChanWarps);
        for (int s = 0; s < kMbDSlots; s++) {
            mbar_init(&sh.d_full[s], 2);  // the two warps of a lane quarter
            mbar_init(&sh.d_empty[s], 1);
        }
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
    // the operand rows past the frame's 180 pixels stay zero: the TMA boxes
    // and the depthwise never write them
    constexpr int kPadFloats = (kMbN - kMbPix) * 32;
    for (int i = threadIdx.x; i < (kMbXStages + kMbDSlots) * kPadFloats; i += kMbThreads) {
        const int blk = i / kPadFloats, e = i - blk * kPadFloats;
        const uint32_t base = blk < kMbXStages ? blk * kMbXBytes : kMbDOff + (blk - kMbXStages) * kMbXBytes;
        reinterpret_cast<float *>(smem + base + kMbXBox)[e] = 0.0f;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // seen by the MMA (async proxy)
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
            uint32_t xi = 0, wi = 0;  // input / weight stages filled so far
            auto take_x = [&](uint32_t &s) {
                s = xi % kMbXStages;
                if (!mbar_wait(&sh.xempty[s], ((xi / kMbXStages) & 1) ^ 1)) return false;
                xi++;
                mbar_expect_tx(&sh.xfull[s], kMbXBox);
                return true;
            };
            auto take_w = [&](uint32_t &s) {
                s = wi % kMbWStages;
                if (!mbar_wait(&sh.wempty[s], ((wi / kMbWStages) & 1) ^ 1)) return false;
                wi++;
                mbar_expect_tx(&sh.wfull[s], kMbWBytes);
                return true;
            };
            bool ok = true;
            // a chunk's project weights, loaded after the next chunk's expand operands
            auto load_project = [&](int pch) {
                for (int kb = 0; ok && kb < 4; kb++) {
                    uint32_t t;
                    if (*abort_flag || !take_w(t)) { ok = false; break; }
                    tma_load_2d(smem + kMbWOff + t * kMbWBytes, &tmWp, &sh.wfull[t], pch * kMbChunk + kb * 32, 0);
                }
            };
            int prev_ch = -1;
            for (int f = blockIdx.x; ok && f < a.n; f += gridDim.x) {
                for (int ch = 0; ok && ch < nchunks; ch++) {
                    for (int kb = 0; kb < kx; kb++) {
                        uint32_t s, t;
                        if (*abort_flag || !take_x(s)) { ok = false; break; }
                        tma_load_4d(smem + s * kMbXBytes, &tmX, &sh.xfull[s], kb * 32, 0, 0, f);
                        if (!take_w(t)) { ok = false; break; }
                        tma_load_2d(smem + kMbWOff + t * kMbWBytes, &tmWe, &sh.wfull[t], kb * 32, ch * kMbChunk);
                    }
                    if (ok && prev_ch >= 0) load_project(prev_ch);
                    prev_ch = ch;
                }
            }
            if (ok && prev_ch >= 0) load_project(prev_ch);
            if (!ok) {
                report_error(0x06000001u);
                *abort_flag = 1;
            }
            // no copy may land after exit: wait (bounded) for the last copies
            // of each ring (a slot is refilled only after its previous copy
            // was consumed, so earlier ones have landed)
            for (uint32_t j = xi >= kMbXStages ? xi - kMbXStages : 0; j < xi; j++)
                mbar_wait(&sh.xfull[j % kMbXStages], (j / kMbXStages) & 1);
            for (uint32_t j = wi >= kMbWStages ? wi - kMbWStages : 0; j < wi; j++)
                mbar_wait(&sh.wfull[j % kMbWStages], (j / kMbWStages) & 1);
        }
    } else if (warp == 0) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32(128, kMbN);
            uint32_t xi = 0, wi = 0, g = 0, j = 0;  // stages consumed, chunks, frames
            bool ok = true;
            auto xstage = [&](uint32_t &s) {
                s = xi % kMbXStages;
                const uint32_t ph = (xi / kMbXStages) & 1;
                xi++;
                return mbar_wait(&sh.xfull[s], ph);
            };
            auto wstage = [&](uint32_t &s) {
                s = wi % kMbWStages;
                const uint32_t ph = (wi / kMbWStages) & 1;
                wi++;
                return mbar_wait(&sh.wfull[s], ph);
            };
            // the project GEMM of chunk pg (chunk pch of the CTA's frame pj)
            auto project = [&](uint32_t pg, int pch, uint32_t pj) {
                // P free (first chunk of a frame)
                if (pch == 0 && pj > 0 && !mbar_wait(&sh.p_empty, (pj - 1) & 1)) { ok = false; return; }
                for (int kb = 0; kb < 4; kb++) {
                    // K-block kb of that chunk's D written (slot use u)
                    const uint32_t u = 4 * pg + kb, slot = u % kMbDSlots;
                    uint32_t t;
                    if (*abort_flag || !mbar_wait(&sh.d_full[slot], (u / kMbDSlots) & 1) || !wstage(t)) {
                        ok = false;
                        return;
                    }
                    tc_fence_after();
                    const uint32_t sw = smem_u32(smem + kMbWOff + t * kMbWBytes);
                    const uint32_t sd = smem_u32(smem + kMbDOff + slot * kMbXBytes);
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        mma_tf32(tmem + kMbPCol, smem_desc_sw128(sw) + 2 * k, smem_desc_sw128(sd) + 2 * k, idesc,
                                 (pch > 0 || kb > 0 || k > 0) ? 1u : 0u);
                    mma_commit(&sh.wempty[t]);
                    mma_commit(&sh.d_empty[slot]);
                }
                if (pch == nchunks - 1) mma_commit(&sh.p_full);
            };
            int prev_ch = -1;
            uint32_t prev_g = 0, prev_j = 0;
            for (int f = blockIdx.x; ok && f < a.n; f += gridDim.x, j++) {
                for (int ch = 0; ok && ch < nchunks; ch++, g++) {
                    // E is free once the channel warps have copied the previous chunk's
                    if (g > 0 && !mbar_wait(&sh.e_empty, (g - 1) & 1)) { ok = false; break; }
                    tc_fence_after();
                    for (int kb = 0; kb < kx; kb++) {
                        uint32_t s, t;
                        if (*abort_flag || !xstage(s) || !wstage(t)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t sx = smem_u32(smem + s * kMbXBytes);
                        const uint32_t sw = smem_u32(smem + kMbWOff + t * kMbWBytes);
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            mma_tf32(tmem + kMbECol, smem_desc_sw128(sw) + 2 * k, smem_desc_sw128(sx) + 2 * k, idesc,
                                     (kb > 0 || k > 0) ? 1u : 0u);
                        mma_commit(&sh.xempty[s]);
                        mma_commit(&sh.wempty[t]);
                    }
                    if (!ok) break;
                    mma_commit(&sh.e_full);
                    // the previous chunk's project GEMM, behind this expand
                    if (prev_ch >= 0) project(prev_g, prev_ch, prev_j);
                    prev_ch = ch;
                    prev_g = g;
                    prev_j = j;
                }
            }
            if (ok && prev_ch >= 0) project(prev_g, prev_ch, prev_j);
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
        // this warp's K-block of chunk g's D: slot (4 g + q) % kMbDSlots, free once
        // the project GEMM has read the slot's previous K-block (use u - 1)
        auto dslot = [&](uint32_t g) { return (4 * g + (uint32_t)q) % kMbDSlots; };
        auto d_free = [&](uint32_t g) {
            const uint32_t u = (4 * g + (uint32_t)q) / kMbDSlots;
            return u == 0 || mbar_wait_sleep(&sh.d_empty[dslot(g)], (u - 1) & 1);
        };
        // 128-byte swizzle: the 16-byte chunk of this lane's channel in row p
        // is (lane / 4) ^ (p % 8); p = 18 y + x, so p % 8 = (2 y + x) % 8
        const uint32_t lane_off = (uint32_t)((lane & 3) << 2);
        const int lane_chunk = lane >> 2;
        // this lane's D column in each of the eight swizzle phases (row p % 8),
        // as shared-memory addresses; a store adds the row's constant offset
        uint32_t dcol[8];
#pragma unroll
        for (int k = 0; k < 8; k++) dcol[k] = smem_u32(smem + kMbDOff) + lane_off + ((lane_chunk ^ k) << 4);
        auto st_d = [](uint32_t addr, float v) { asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory"); };
        // One chunk without a depthwise (DW = false): this warp's five E rows
        // (no halo: D[p] depends on E[p] alone; rows past the frame hold the
        // expand of zero fill and feed no stored output) become D after the
        // expand bias and activation.  Y0 (the warp's first row, 0 or 5) is
        // compile-time, so the D stores' swizzled addresses fold into constants.
        auto pw_chunk = [&](auto Y0, int ch, uint32_t g) -> bool {
            constexpr int yb = decltype(Y0)::value;
            const int c = ch * kMbChunk + q * 32 + lane;  // expanded channel of this thread
            const float be = c < a.cexp ? __ldg(a.b_exp + c) : 0.0f;
            if (!__all_sync(0xffffffffu, !*abort_flag && mbar_wait_sleep(&sh.e_full, g & 1))) return false;
            tc_fence_after();
            uint32_t wr[kMbHalfRows][kMbRowStride];
#pragma unroll
            for (int r = 0; r < kMbHalfRows; r++)
#pragma unroll
                for (int k = 0; k < kMbRowStride / 2; k++)
                    tmem_ld2(tlane + kMbECol + (yb + r) * kMbRowStride + 2 * k, wr[r][2 * k], wr[r][2 * k + 1]);
#pragma unroll
            for (int r = 0; r < kMbHalfRows; r++) tmem_wait_pin18(wr[r]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.e_empty);
            float v[kMbHalfRows][kMbRowStride];
#pragma unroll
            for (int r = 0; r < kMbHalfRows; r++) {
#pragma unroll
                for (int x = 0; x < kMbRowStride; x++) v[r][x] = __uint_as_float(wr[r][x]) + be;
                act_fixed_n<AE, kMbRowStride>(a.act_exp, v[r]);
            }
            // the D slot is free once the project GEMM has read its previous K-block
            if (!__all_sync(0xffffffffu, d_free(g))) return false;
            tc_fence_after();
            const uint32_t soff = dslot(g) * kMbXBytes;
#pragma unroll
            for (int r = 0; r < kMbHalfRows; r++) {
                const int y = yb + r;
#pragma unroll
                for (int x = 0; x < kMbRowStride; x++)
                    st_d(dcol[(2 * y + x) & 7] + soff + (y * kMbRowStride + x) * 128, v[r][x]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // D is read by the MMA (async proxy)
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.d_full[dslot(g)]);
            return true;
        };
        uint32_t g = 0, j = 0;
        bool ok = true;
        for (int f = blockIdx.x; ok && f < a.n; f += gridDim.x, j++) {
            for (int ch = 0; ch < nchunks; ch++, g++) {
                if constexpr (DW) {
                    const int c = ch * kMbChunk + q * 32 + lane;  // expanded channel of this thread
                    const bool cv = c < a.cexp;
                    float wd[9];
#pragma unroll
                    for (int t = 0; t < 9; t++) wd[t] = cv ? __ldg(a.w_dw + t * a.cexp_pad4 + c) : 0.0f;
                    const float be = cv ? __ldg(a.b_exp + c) : 0.0f, bd = cv ? __ldg(a.b_dw + c) : 0.0f;
                    // the warp's lanes decide together (the TMEM loads are warp-collective)
                    if (!__all_sync(0xffffffffu, !*abort_flag && mbar_wait_sleep(&sh.e_full, g & 1))) { ok = false; break; }
                    tc_fence_after();
                    // copy the seven E rows y0 - 1 .. y0 + 5 of this lane's channel
                    // into registers (rows outside the frame are not read), then
                    // release E so the next chunk's expand GEMM can start
                    constexpr int kWin = kMbHalfRows + 2;
                    uint32_t wr[kWin][kMbRowStride];
#pragma unroll
                    for (int r = 0; r < kWin; r++) {
                        const int row = y0 - 1 + r;
                        if (row >= 0 && row < a.h) {  // warp-uniform
#pragma unroll
                            for (int k = 0; k < kMbRowStride / 2; k++)
                                tmem_ld2(tlane + kMbECol + row * kMbRowStride + 2 * k, wr[r][2 * k], wr[r][2 * k + 1]);
                        } else {
#pragma unroll
                            for (int x = 0; x < kMbRowStride; x++) wr[r][x] = 0u;
                        }
                    }
#pragma unroll
                    for (int r = 0; r < kWin; r++) tmem_wait_pin18(wr[r]);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sh.e_empty);
                    // expand epilogue: bias, activation, zero outside the frame
                    float win[kWin][kMbRowStride];
#pragma unroll
                    for (int r = 0; r < kWin; r++) {
                        const int row = y0 - 1 + r;
                        const bool rv = row >= 0 && row < a.h;
#pragma unroll
                        for (int x = 0; x < kMbRowStride; x++) win[r][x] = __uint_as_float(wr[r][x]) + be;
                        act_fixed_n<AE, kMbRowStride>(a.act_exp, win[r]);
#pragma unroll
                        for (int x = 0; x < kMbRowStride; x++)
                            if (!rv || x >= a.w) win[r][x] = 0.0f;
                    }
                    // the D slot is free once the project GEMM has read its previous K-block
                    if (!__all_sync(0xffffffffu, d_free(g))) { ok = false; break; }
                    tc_fence_after();
                    uint8_t *dk = smem + kMbDOff + dslot(g) * kMbXBytes;
#pragma unroll
                    for (int i = 0; i < kMbHalfRows; i++) {
                        const int y = y0 + i;
                        const float(&ra)[kMbRowStride] = win[i];
                        const float(&rb)[kMbRowStride] = win[i + 1];
                        const float(&rc)[kMbRowStride] = win[i + 2];
                        // taps in (ky, kx) order from the bias, as the depthwise kernels
                        float o[kMbRowStride];
#pragma unroll
                        for (int x = 0; x < kMbRowStride; x++) {
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
                            o[x] = acc;
                        }
                        act_fixed_n<AD, kMbRowStride>(a.act_dw, o);
                        // D[p][lane], p = 18 y + x: K-major, 128-byte swizzle
                        uint8_t *drow = dk + y * (kMbRowStride * 128) + lane_off;
                        const bool yv = y < a.h;
                        const int ysw = 2 * y;
#pragma unroll
                        for (int x = 0; x < kMbRowStride; x++)
                            *reinterpret_cast<float *>(drow + x * 128 + ((lane_chunk ^ ((ysw + x) & 7)) << 4)) =
                                (yv && x < a.w) ? o[x] : 0.0f;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // D is read by the MMA (async proxy)
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sh.d_full[dslot(g)]);
                } else if (y0 == 0 ? !pw_chunk(Int<0>(), ch, g) : !pw_chunk(Int<kMbHalfRows>(), ch, g)) {
                    ok = false;
                    break;
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
                float r[kMbRowStride];
                // the residual row first: its loads overlap the TMEM read
#pragma unroll
                for (int x = 0; x < kMbRowStride; x++)
                    r[x] = (a.res && ov && x < a.w) ? __ldg(a.res + (m0 + x) * a.cout + o) : 0.0f;
                float v[kMbRowStride];
                tmem_row18(tlane + kMbPCol + y * kMbRowStride, v);
#pragma unroll
                for (int x = 0; x < kMbRowStride; x++) v[x] += bp;
                act_apply_n<kMbRowStride>(a.act_proj, v);
                if (ov) {
#pragma unroll
                    for (int x = 0; x < kMbRowStride; x++)
                        if (x < a.w) a.y[(m0 + x) * a.cout + o] = v[x] + r[x];  // residual after the activation
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
