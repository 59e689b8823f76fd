// Tensor-core stem: a 3x3 conv with cin <= 3 and cout = 32 (the network's
// first layer, crates/ai-cpu/src/kernels/conv.rs's conv_std on a 3-channel
// frame) as a TF32 GEMM with K = 9*cin <= 27, zero-padded to 32 so that
// one im2col row is exactly one 128-byte swizzle row.
//
// Per 16x16 output tile (256 pixels = two M=128 MMA tiles):
//   1. the input halo is staged with 4-byte cp.async (zero-fill = padding),
//      double-buffered across tiles;
//   2. each thread writes its pixel's 32-value im2col row into the A
//      operand (K-major, 128-byte swizzle) -- 27 shared loads, 8 stores;
//   3. one thread issues 2 x 4 tcgen05.mma (M=128, N=32, K=8) into TMEM;
//   4. each warp drains its 32 TMEM lanes, adds bias, applies the
//      activation, transposes through its own A rows and writes 512-byte
//      contiguous pieces of the NHWC output.
// Three CTAs share an SM so their phases overlap.  Every wait is bounded.
//
// With PW (aie_conv_run_stem_pw) the kernel also runs the 1x1 conv that
// reads the stem's output (cin 32, cout <= 32: a feature pyramid's lateral
// on the stem features): the staged tile of step 4 is exactly that GEMM's A
// operand (pixel rows, 32 channels, K-major, 128-byte swizzle), so one
// thread issues 2 x 4 more MMAs into a second pair of accumulators while the
// warps store the stem tile, and the warps then drain, add the 1x1's bias
// and activation and store its output the same way.  The stem output is
// still written (the encoder reads it); the 1x1's separate pass over it is
// saved.
#pragma once

namespace aie {

constexpr int kStemCout = 32;
constexpr int kStemTile = 16;
constexpr int kStemThreads = 256;                 // one thread per output pixel of a tile
constexpr uint32_t kStemABytes = 256 * 128;       // im2col rows; also the epilogue staging
constexpr uint32_t kStemBBytes = kStemCout * 128; // weights [n][k], K-major
constexpr uint32_t kStemTmemCols = 64;            // two 128 x 32 fp32 accumulators (128 with PW: four)

// The fused 1x1 conv after the stem (PW): dense [n][oh][ow][cout] output.
struct StemPw {
    const float *w;     // [cout][32], K-major rows (the TF32 1x1 packing)
    const float *bias;  // [>= cout]
    float *y;
    int cout, act;
};

template <int CIN, int S, bool PW = false>
struct StemTcLayout {
    static constexpr int HH = (kStemTile - 1) * S + 3, HW = HH;
    static constexpr int HROW = HW * CIN, HN = HH * HROW;
    // TMA halo rows: the row's floats from a 16-byte-aligned start (up to 3
    // floats early) rounded up to 16 bytes
    static constexpr int BX = (HROW + 3 + 3) / 4 * 4;
    static constexpr int HN_MAX = HH * BX > HN ? HH * BX : HN;
    static constexpr uint32_t kB2Off = kStemABytes + kStemBBytes;         // PW: the 1x1's weights
    static constexpr uint32_t kHaloOff = kStemABytes + (PW ? 2 : 1) * kStemBBytes;
    // each halo buffer starts 256-byte aligned (a TMA destination must be at
    // least 128-byte aligned)
    static constexpr uint32_t kHaloFloats = (HN_MAX + 63) / 64 * 64;
    static constexpr uint32_t kBiasOff = kHaloOff + 2 * kHaloFloats * 4;  // stem bias, then (PW) the 1x1's
    static constexpr uint32_t kBarOff = kBiasOff + (PW ? 2 : 1) * kStemCout * 4;
    // barriers: [0] stem MMA, [1..2] halo buffers, [3] the 1x1's MMA; then the TMEM slot
    static constexpr uint32_t kBytes = kBarOff + 48 + 1024;  // + slack to 1024-align the base
    static_assert(kHaloOff % 256 == 0 && (kHaloFloats * 4) % 256 == 0, "TMA halo buffers 256-byte aligned");
    static_assert(kBarOff % 8 == 0, "mbarriers 8-byte aligned");
};

// First float of the halo row for a tile starting at column ix0, rounded
// down to a 16-byte boundary (TMA's innermost coordinate rule).
__device__ __forceinline__ int stem_row_start(int ix0, int cin) { return (ix0 * cin) & ~3; }

// byte offset of element (row, k) in a K-major operand with 128-byte rows
// and the 128-byte swizzle (16-byte chunk index XOR row % 8)
__device__ __forceinline__ uint32_t sw128_off(int row, int k)
{
    return (uint32_t)(row * 128 + ((((k >> 2) ^ row) & 7) << 4) + ((k & 3) << 2));
}

// kTma: the dense input (pixel stride = cin, 16-byte aligned rows) is staged
// with one 3-D TMA box (W*cin floats, H, N) per tile -- out-of-frame rows and
// columns read as zeros -- instead of one 4-byte cp.async per element.
template <int CIN, int S, bool kTma, bool PW = false>
__global__ void __launch_bounds__(kStemThreads, 3)
    stem_tc_kernel(const __grid_constant__ CUtensorMap tmx, const ConvArgs a, const StemGeom g, const StemPw pw)
{
    using L = StemTcLayout<CIN, S, PW>;
    constexpr uint32_t kTmemCols = PW ? 2 * kStemTmemCols : kStemTmemCols;
    constexpr int K = 9 * CIN;
    static_assert(K <= 32, "im2col row must fit one 128-byte swizzle row");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + kStemABytes;
    float *halo = reinterpret_cast<float *>(smem + L::kHaloOff);
    float *sbias = reinterpret_cast<float *>(smem + L::kBiasOff);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
    uint64_t *hbar = bar + 1;  // [2] halo buffer full (TMA path)
    uint64_t *bar2 = bar + 3;  // PW: the 1x1's MMAs done
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kBarOff + 32);
    constexpr int ROW = kTma ? L::BX : L::HROW;  // halo row stride in floats
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tiles_per_img = g.tiles_x * g.tiles_y;
    const int ntiles = a.n * tiles_per_img;

    auto stage = [&](int t, int buf) {
        const int img = fdiv(t, g.div_tpi), rem = t - img * tiles_per_img;
        const int ty = fdiv(rem, g.div_tx), tx = rem - ty * g.tiles_x;
        const int iy0 = ty * kStemTile * S - a.pt, ix0 = tx * kStemTile * S - a.pl;
        const float *xb = a.x + (long long)img * a.ih * a.iw * a.x_stride + a.x_coff;
        float *dst = halo + buf * L::kHaloFloats;
        for (int i = tid; i < L::HN; i += kStemThreads) {
            const int cc = i % CIN, p = i / CIN;
            const int hy = p / L::HW, hx = p - hy * L::HW;
            const int iy = iy0 + hy, ix = ix0 + hx;
            const bool ok = iy >= 0 && iy < a.ih && ix >= 0 && ix < a.iw;
            const float *src = ok ? xb + ((long long)iy * a.iw + ix) * a.x_stride + cc : xb;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst + i)), "l"(src),
                         "r"(ok ? 4 : 0)
                         : "memory");
        }
    };

    // one TMA box per tile (thread 0): rows [iy0, iy0 + HH) of the frame,
    // floats [start, start + BX) of each row
    auto stage_tma = [&](int t, int buf) {
        const int img = fdiv(t, g.div_tpi), rem = t - img * tiles_per_img;
        const int ty = fdiv(rem, g.div_tx), tx = rem - ty * g.tiles_x;
        const int iy0 = ty * kStemTile * S - a.pt, ix0 = tx * kStemTile * S - a.pl;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier generic reads of the buffer
        mbar_expect_tx(&hbar[buf], (uint32_t)(L::HH * L::BX * 4));
        tma_load_3d(halo + buf * L::kHaloFloats, &tmx, &hbar[buf], stem_row_start(ix0, CIN), iy0, img);
    };

    // B operand: packed weights [k][wn] -> rows n (output channel), K-major
    for (int i = tid; i < kStemCout * 32; i += kStemThreads) {
        const int n = i >> 5, k = i & 31;
        *reinterpret_cast<float *>(sB + sw128_off(n, k)) = k < K ? __ldg(a.w + k * a.wn + n) : 0.0f;
    }
    if (tid < kStemCout) sbias[tid] = __ldg(a.bias + tid);
    if constexpr (PW) {
        // the 1x1's weights as a second B operand (rows past cout are zero)
        uint8_t *sB2 = smem + L::kB2Off;
        for (int i = tid; i < kStemCout * 32; i += kStemThreads) {
            const int n = i >> 5, k = i & 31;
            *reinterpret_cast<float *>(sB2 + sw128_off(n, k)) = n < pw.cout ? __ldg(pw.w + n * 32 + k) : 0.0f;
        }
        if (tid < kStemCout) sbias[kStemCout + tid] = tid < pw.cout ? __ldg(pw.bias + tid) : 0.0f;
    }
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_init(&hbar[0], 1);
        mbar_init(&hbar[1], 1);
        mbar_init(bar2, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = idesc_tf32(128, kStemCout);
    const uint64_t bdesc = smem_desc_sw128(smem_u32(sB));

    uint32_t phase = 0, phase2 = 0;
    bool failed = false, mma_pending = false, mma2_pending = false;
    uint32_t halo_pending = 0;  // TMA path, thread 0: buffers with a copy in flight
    uint32_t halo_parity = 0;   // ... and the phase parity each of those copies completes
    int t = blockIdx.x;
    if constexpr (kTma) {
        if (t < ntiles && tid == 0) {
            stage_tma(t, 0);
            halo_pending |= 1u;  // use 0 of buffer 0: parity 0
        }
    } else {
        if (t < ntiles) stage(t, 0);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int i = 0; t < ntiles; t += gridDim.x, i++) {
        const int tn = t + gridDim.x;
        const int t_img = fdiv(t, g.div_tpi), t_rem = t - t_img * tiles_per_img;
        const int t_ty = fdiv(t_rem, g.div_tx), t_tx = t_rem - t_ty * g.tiles_x;
        if constexpr (kTma) {
            // prefetch the next tile's halo: its buffer was last read by the
            // previous tile's im2col, which every thread finished before the
            // previous tile's MMA barrier
            if (tn < ntiles && tid == 0) {
                const int nb = (i + 1) & 1;
                stage_tma(tn, nb);
                halo_pending |= 1u << nb;
                halo_parity = (halo_parity & ~(1u << nb)) | ((((uint32_t)(i + 1) >> 1) & 1u) << nb);
            }
            if (!mbar_wait_sleep(&hbar[i & 1], (uint32_t)(i >> 1) & 1)) {
                report_error(0x03000002u);
                failed = true;
            } else if (tid == 0) {
                halo_pending &= ~(1u << (i & 1));
            }
        } else {
            if (tn < ntiles) stage(tn, (i + 1) & 1);  // prefetch the next tile's halo
            asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group 1;" ::: "memory");  // this tile's halo has landed
        }
        tc_fence_before();
        if (__syncthreads_or(failed)) break;
        tc_fence_after();

        // ---- im2col: this thread's pixel -> A row `tid`, k = (ky*3 + kx)*CIN + ic
        {
            int hoff = 0;  // TMA path: the row data starts up to 3 floats into the row
            if constexpr (kTma) {
                const int ix0 = t_tx * kStemTile * S - a.pl;
                hoff = ix0 * CIN - stem_row_start(ix0, CIN);
            }
            const float *hp = halo + (i & 1) * L::kHaloFloats + hoff + (tid >> 4) * S * ROW + (tid & 15) * S * CIN;
            float v[32];
#pragma unroll
            for (int k = 0; k < 32; k++) {
                if (k < K) {
                    const int tap = k / CIN, ic = k - tap * CIN;
                    v[k] = hp[(tap / 3) * ROW + (tap % 3) * CIN + ic];
                } else {
                    v[k] = 0.0f;
                }
            }
            uint8_t *row = sA + tid * 128;
#pragma unroll
            for (int c = 0; c < 8; c++)
                *reinterpret_cast<float4 *>(row + (((c ^ tid) & 7) << 4)) =
                    make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // A visible to the tensor core
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
#pragma unroll
            for (int m = 0; m < 2; m++) {
                const uint64_t adesc = smem_desc_sw128(smem_u32(sA + m * (kStemABytes / 2)));
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    mma_tf32(tmem + (uint32_t)(m * kStemCout), adesc + 2 * kk, bdesc + 2 * kk, idesc, kk > 0);
            }
            mma_commit(bar);
        }
        mma_pending = true;
        // warp-uniform outcome: the TMEM loads below are warp-collective
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(bar, phase))) {
            if (lane == 0) report_error(0x03000001u);
            failed = true;
            continue;  // the next tile's barrier turns this into a CTA-wide exit
        }
        mma_pending = false;
        phase ^= 1;
        tc_fence_after();

        // ---- epilogue: TMEM lanes (warp%4)*32.., accumulator warp/4 -> pixel
        // tid, in two halves of 16 channels; staged in this warp's own A rows
        // (free once the MMA completed), 128-byte swizzled
        const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * kStemCout);
        uint8_t *srow = sA + tid * 128;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint32_t r[16];
            tmem_ld16_issue(taddr + 16 * h, r);
            tmem_wait16(r);
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                const float4 b4 = *reinterpret_cast<const float4 *>(sbias + 16 * h + j);
                o[j] = __uint_as_float(r[j]) + b4.x;
                o[j + 1] = __uint_as_float(r[j + 1]) + b4.y;
                o[j + 2] = __uint_as_float(r[j + 2]) + b4.z;
                o[j + 3] = __uint_as_float(r[j + 3]) + b4.w;
            }
            act_apply_n<16>(a.act, o);
#pragma unroll
            for (int c = 0; c < 4; c++)
                *reinterpret_cast<float4 *>(srow + ((((4 * h + c) ^ tid) & 7) << 4)) =
                    make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
        }
        if constexpr (PW) {
            // the staged tile is the 1x1's A operand: every warp's rows must
            // be in place before thread 0 issues its MMAs
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                const uint64_t b2desc = smem_desc_sw128(smem_u32(smem + L::kB2Off));
#pragma unroll
                for (int m = 0; m < 2; m++) {
                    const uint64_t adesc = smem_desc_sw128(smem_u32(sA + m * (kStemABytes / 2)));
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_tf32(tmem + kStemTmemCols + (uint32_t)(m * kStemCout), adesc + 2 * kk, b2desc + 2 * kk,
                                 idesc, kk > 0);
                }
                mma_commit(bar2);
            }
            mma2_pending = true;
        } else {
            __syncwarp();
        }
        const int oy0 = t_ty * kStemTile, ox0 = t_tx * kStemTile;
        const int c = lane & 7;                          // this lane's 4-channel chunk
        const int mrow0 = (t_img * a.oh + oy0) * a.ow + ox0;  // first pixel of the tile (M < 2^31)
        float *ybase = a.y + a.y_coff + 4 * c;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int p = warp * 32 + j * 4 + (lane >> 3);  // pixel of the tile
            const float4 val = *reinterpret_cast<const float4 *>(sA + p * 128 + (((c ^ p) & 7) << 4));
            const int dy = p >> 4, dx = p & 15;
            if (oy0 + dy < a.oh && ox0 + dx < a.ow)
                *reinterpret_cast<float4 *>(ybase + (long long)(mrow0 + dy * a.ow + dx) * a.y_stride) = val;
        }
        if constexpr (PW) {
            // the 1x1's accumulators -> + bias -> activation -> this warp's own
            // A rows (its stores above have read them; the MMAs have too once
            // bar2 completes) -> 128-byte rows of the 1x1's output
            if (!__all_sync(0xffffffffu, mbar_wait_sleep(bar2, phase2))) {
                if (lane == 0) report_error(0x03000003u);
                failed = true;
                continue;
            }
            mma2_pending = false;
            phase2 ^= 1;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; h++) {
                uint32_t r[16];
                tmem_ld16_issue(taddr + kStemTmemCols + 16 * h, r);
                tmem_wait16(r);
                float o[16];
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    const float4 b4 = *reinterpret_cast<const float4 *>(sbias + kStemCout + 16 * h + j);
                    o[j] = __uint_as_float(r[j]) + b4.x;
                    o[j + 1] = __uint_as_float(r[j + 1]) + b4.y;
                    o[j + 2] = __uint_as_float(r[j + 2]) + b4.z;
                    o[j + 3] = __uint_as_float(r[j + 3]) + b4.w;
                }
                act_apply_n<16>(pw.act, o);
                __syncwarp();
#pragma unroll
                for (int cc = 0; cc < 4; cc++)
                    *reinterpret_cast<float4 *>(srow + ((((4 * h + cc) ^ tid) & 7) << 4)) =
                        make_float4(o[4 * cc], o[4 * cc + 1], o[4 * cc + 2], o[4 * cc + 3]);
            }
            __syncwarp();
            if (4 * c < pw.cout) {
                float *y2 = pw.y + 4 * c;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int p = warp * 32 + j * 4 + (lane >> 3);
                    const float4 val = *reinterpret_cast<const float4 *>(sA + p * 128 + (((c ^ p) & 7) << 4));
                    const int dy = p >> 4, dx = p & 15;
                    if (oy0 + dy < a.oh && ox0 + dx < a.ow)
                        *reinterpret_cast<float4 *>(y2 + (long long)(mrow0 + dy * a.ow + dx) * pw.cout) = val;
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (mma_pending && tid == 0) mbar_wait(bar, phase);  // drain before the TMEM is released
    if (PW && mma2_pending && tid == 0) mbar_wait(bar2, phase2);
    if constexpr (kTma) {
        // a prefetch left in flight by an early exit must land before the CTA ends
        for (int b = 0; b < 2; b++)
            if (tid == 0 && (halo_pending >> b & 1)) mbar_wait(&hbar[b], halo_parity >> b & 1);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// Host: launch one wave of kStemCtasPerSm resident CTAs per SM (persistent
// over tiles).  The occupancy API reports one CTA per SM for this kernel on
// B200 (driver 580) although registers (80 x 256 x 3) and shared memory
// (3 x (64 KB + 1 KB)) admit three; the grid is sized from those limits
// directly, and the strided tile loop stays correct however many are resident.
constexpr int kStemCtasPerSm = 3;

template <int CIN, int S, bool PW = false>
static int stem_tc_launch(const ConvArgs &a, const StemGeom &g, cudaStream_t s, const StemPw &pw = StemPw{})
{
    using L = StemTcLayout<CIN, S, PW>;
    static_assert(kStemCtasPerSm * (L::kBytes + 1024) <= 228 * 1024, "shared memory for three CTAs per SM");
    for (auto fn : {stem_tc_kernel<CIN, S, true, PW>, stem_tc_kernel<CIN, S, false, PW>})
        if (ensure_smem_attr((const void *)fn, (int)L::kBytes, true) != cudaSuccess) return -1;
    const long long ntiles = (long long)a.n * g.tiles_x * g.tiles_y;
    const unsigned grid = (unsigned)std::min<long long>(ntiles, (long long)kStemCtasPerSm * tc_sm_count());
    // TMA halo when the input is a dense, 16-byte aligned [n][ih][iw][cin] tensor
    CUtensorMap tm;
    memset(&tm, 0, sizeof tm);
    const uintptr_t base = (uintptr_t)(a.x + a.x_coff);
    const uint64_t row_bytes = (uint64_t)a.iw * CIN * 4;
    PFN_encodeTiled enc = tc_encoder();
    bool tma = enc && a.x_stride == CIN && a.x_coff == 0 && base % 16 == 0 && row_bytes % 16 == 0;
    if (tma) {
        const cuuint64_t dims[3] = {(cuuint64_t)a.iw * CIN, (cuuint64_t)a.ih, (cuuint64_t)a.n};
        const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)row_bytes * a.ih};
        const cuuint32_t box[3] = {(cuuint32_t)L::BX, (cuuint32_t)L::HH, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        tma = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (tma) stem_tc_kernel<CIN, S, true, PW><<<grid, kStemThreads, L::kBytes, s>>>(tm, a, g, pw);
    else stem_tc_kernel<CIN, S, false, PW><<<grid, kStemThreads, L::kBytes, s>>>(tm, a, g, pw);
    return 0;
}

}  // namespace aie
