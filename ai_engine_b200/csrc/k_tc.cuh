// tcgen05 / TMEM TF32 implicit-GEMM conv for sm_100a (1x1 and k x k).
//
//   C[M, N] = sum over (tap, k-block) of A_tap[M, 32] * B_tap[32, N]
//
// M = output pixels, N = cout, K = taps x cin.  Persistent, warp-specialised:
//   warp 0       TMEM allocator + MMA issuer (one elected lane)
//   warps 1..8   epilogue, two groups of four: group g drains TMEM
//                accumulator buffer g (every other tile), so two tiles'
//                epilogues overlap.  tcgen05.ld -> bias -> act, transposed
//                through shared memory -> +residual -> coalesced row stores
//   warp 9       TMA producer: up to 8 free-running lanes, each issuing
//                every 8th stage of its pipeline (TMA issue is limited per
//                issuing thread, about one box in flight each: on B200 one
//                lane moves ~0.65 us per 16 KB box per SM, four ~0.23 us)
//   warp 10      second MMA issuer.  One issuing thread sustains one
//                M=128 K=8 TF32 MMA per ~55-75 SM clocks at N <= 64 (~45 per
//                SM with two issuers), so narrow k x k tiles run two
//                pipelines: the CTA's even units use stage ring 0, MMA warp
//                0, accumulators 0-1 and epilogue group 0, the odd units ring
//                1, warp 10, accumulators 2-3 and group 1 (each pipeline's
//                tiles alternate between its two accumulators, so its MMAs
//                never wait for the epilogue of its previous tile).
// Accumulators are double-buffered in TMEM so the epilogue of one tile
// overlaps the mainloop of the next.  Operands are fp32 in HBM and are read
// by the tensor core as TF32; both are K-major with the 128-byte swizzle.
// With one n-tile and no K split the whole B is resident in shared memory
// (loaded once per CTA) and the stages carry only A.
//
// A operand (activations, NHWC):
//   1x1 conv : 2-D tensor map (cin, M), box (32, 128)
//   k x k    : 4-D tensor map (cin, iw, ih, n) with element strides
//              (1, sw, sh, 1), box (32, bw*sw, bh*sh, 1): one M tile is a
//              bh x bw block of output pixels of one frame, and each tap is
//              the same box shifted by (kx*dil - pl, ky*dil - pt).  TMA's
//              out-of-bounds zero fill is the convolution's zero padding.
//   flat     : k x k, stride 1, narrow N.  One box of (16 + kw - 1) x bhx
//              input pixels per K block serves every tap: the box's pixels
//              in row-major order are the A rows, so tap (ky, kx)'s A
//              operand is the 128 rows starting at row ky*bwx + kx, and
//              accumulator row r is output pixel (r / bwx, r % bwx) of the
//              tile (valid for r % bwx < 16 and r / bwx < 128 / bwx).  A
//              stage feeds kh*kw MMA groups from one copy.  The tensor core
//              applies the 128-byte swizzle to absolute shared-memory
//              addresses, as the TMA wrote them, so a start row that is not
//              a multiple of 8 reads the right bytes.
// Concat parts (up to 3): the input is the channel concat of separate
// views read in place, one A tensor map each; part p owns whole K blocks
// (its channels padded with zero fill to a multiple of the block width: 16
// when every part has at most 16 channels, else 32), so a K block's
// copy comes from one part's map at that part's own channel coordinate.
// B operand (weights [tap][cout][cin_pad]): 3-D map, box (32, bn, 1).
//
// Split-K (small M, deep K): units = m_tiles x n_tiles x split.  Each unit
// writes its raw partial tile to the workspace; the last unit of a tile
// (atomic ticket) sums the partials in split order -- deterministic -- and
// runs the epilogue.
//
// Every wait on an mbarrier is bounded (1 s of %globaltimer); on expiry the
// CTA records an error code in g_aie_error, stops issuing work, waits
// (bounded) for its own copies in flight, frees its TMEM and exits.
#pragma once
#include <atomic>

#include <cuda.h>

#include <cstring>
#include <type_traits>

#include "k_simt.cuh"

namespace aie {

constexpr int kTcProducers = 1;                   // one producer warp ...
constexpr int kTcIssueLanes = 8;                  // ... issuing from up to 8 lanes at once
constexpr int kTcEpiWarps = 8;
constexpr int kTcMmaWarp1 = 1 + kTcEpiWarps + kTcProducers;  // second MMA issuer (pipeline 1)
constexpr int kTcThreads = 32 * (kTcMmaWarp1 + 1);           // MMA 0, epilogue, producer, MMA 1
constexpr uint32_t kTcStageOut = 32 * 32 * 4;      // one 32x32 fp32 epilogue chunk per warp
constexpr int kTcBM = 128;
constexpr int kTcBK = 32;                 // fp32 elements per K block = 128 B (one swizzle row)
constexpr uint32_t kTcBResidentMax = 112 * 1024;   // largest B kept in shared memory for a whole kernel
constexpr int kTcPatchCols = 18;                   // source columns per segment of an exact-2x residual patch
constexpr uint32_t kTcPatchBytes = 2 * 2 * kTcPatchCols * 128;  // [segment][source row][column] x 32 channels

// Residual buffer kinds of a tensor-core plan (tc_plan's res_kind)
enum TcResKind : uint32_t {
    kTcResNone = 0,    // no residual, or one read directly by the epilogue
    kTcResTensor = 1,  // residual tensor of the output's shape, cp.async rows
    kTcResUp2 = 2,     // exact-2x half_pixel bilinear residual, cp.async patches
};

struct TcGeom {
    uint32_t bm, bn;
    uint32_t igemm;            // 0: 2-D A map (1x1), 1: 4-D A map (k x k)
    uint32_t bw, bh;           // M tile box (k x k)
    uint32_t tiles_x, tiles_y; // output-pixel tiles per frame (k x k)
    uint32_t m_tiles, n_tiles, split, k_iters, k_per_split, kblocks, taps;
    uint32_t stages, tmem_cols;
    uint64_t units, grid;
    uint64_t workspace_bytes;
    uint32_t smem_bytes;
    uint32_t b_bytes;
    uint32_t pipes;            // independent MMA pipelines (1 or 2), see tc_conv_kernel
    uint32_t bk;               // channels per K block: 32 (128-byte rows) or 16 (64-byte rows)
    uint32_t bias_smem;        // the epilogue warps keep the n-tile's bias in shared memory
    uint32_t halo;             // k x k stride 1: one A box per (kx, K block), see tc_conv_kernel
    uint32_t flat;             // k x k stride 1: one A box per K block serving every tap, see tc_conv_kernel
    uint32_t bwx, bhx;         // flat mode: the box's width and height in input pixels
    uint32_t a_bytes;          // A bytes per stage (flat: the box rounded up to 1 KB)
    uint32_t a_box;            // bytes the A copy of a stage writes
    uint32_t b_resident;       // 1: the CTA's whole B (all taps and K blocks) is loaded once
    uint32_t bres_off;         // shared-memory offset of the resident B
    uint32_t res_off;          // per-warp residual prefetch buffers (0 = none)
    uint32_t res_patch;        // the buffers hold exact-2x residual patches (kTcResUp2)
    uint32_t out_off, shared_off;
};

struct TcArgs {
    ConvArgs c;
    uint32_t bn, bw, bh, tiles_x, tiles_y, m_tiles, n_tiles, split, k_iters, k_per_split, kblocks;
    uint32_t stages, tmem_cols, b_bytes, igemm;
    uint32_t b_resident, bres_off, res_off, pipes, halo, a_bytes;
    uint32_t bias_smem;               // per-warp shared copies of the n-tile's bias (else L1 reads)
    uint32_t flat, bwx, a_box;        // flat mode (see tc_conv_kernel)
    uint32_t nparts, kb1, kb2;        // concat parts: 1-3 A tensor maps; parts 1 and 2 start at K blocks kb1, kb2
    uint32_t res_patch;               // RES 3 epilogue: residual from per-warp exact-2x patches
    uint64_t units;                   // < 2^31 (checked at launch)
    FastDiv div_ntiles, div_split;    // unit -> (m tile, n tile, split)
    FastDiv div_perimg, div_tilesx;   // m tile -> (frame, tile row, tile column)
    uint32_t lbw;                     // log2(bw): bw is a power of two
    float *ws;            // split-K partials [tile][split][128][bn]
    uint32_t *tickets;    // split-K tickets [tile][4 row quadrants]
    uint32_t out_off, shared_off;  // shared-memory carve-up (bytes)
};

// Exact-2x residual patch of one epilogue warp.  On 1x1 tiles a warp's 32
// rows are the consecutive output pixels m0..m0+31; with ow >= 32 they lie
// in at most two output rows: segment 0 (the row of m0, from column ox0)
// and segment 1 (the next row, from column 0).  Output column ox reads
// source columns clamp((ox - 1) >> 1) and the one after, so a segment's 32
// columns need at most 18 source columns, from qc0 (segment 0) or 0
// (segment 1), on two source rows each.
struct Up2Patch {
    int ox0, qc0;            // first output / source column of segment 0
    int img0, y00, y01;      // segment 0: frame and source rows
    int img1, y10, y11;      // segment 1 (frame clamped to the batch when past it)
    int odd0, odd1;          // output row parity: lower-row weight 0.25 if odd, else 0.75
};

__device__ __forceinline__ Up2Patch up2_patch(const ConvArgs &c, int m0)
{
    Up2Patch p;
    const int t = fdiv(m0, c.div_ow);
    p.ox0 = m0 - t * c.ow;
    p.img0 = fdiv(t, c.div_oh);
    const int oy0 = t - p.img0 * c.oh;
    int oy1 = oy0 + 1;
    p.img1 = p.img0;
    if (oy1 == c.oh) {
        oy1 = 0;
        p.img1 = min(p.img0 + 1, c.n - 1);
    }
    p.qc0 = max((p.ox0 - 1) >> 1, 0);
    const int f0 = (oy0 - 1) >> 1, f1 = (oy1 - 1) >> 1;
    p.y00 = max(f0, 0); p.y01 = min(f0 + 1, c.rh - 1);
    p.y10 = max(f1, 0); p.y11 = min(f1 + 1, c.rh - 1);
    p.odd0 = oy0 & 1; p.odd1 = oy1 & 1;
    return p;
}

// --------------------------------------------------------------- PTX ---

// Self-test of the bounded-wait path: one thread waits on an mbarrier that
// nothing ever arrives at.  The wait gives up after `limit_ns`, records
// kSelftestCode in the device error word and the kernel returns normally --
// the same path every role of tc_conv_kernel takes when a wait expires.
constexpr uint32_t kSelftestCode = 0x7F000001u;

__global__ void selftest_wait_kernel(unsigned long long limit_ns)
{
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (!mbar_wait_for(&bar, 0, limit_ns)) report_error(kSelftestCode);
    }
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 B apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);       // start address
    d |= (uint64_t)1 << 16;                        // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;              // stride byte offset
    d |= (uint64_t)1 << 46;                        // version
    d |= (uint64_t)2 << 61;                        // layout: SWIZZLE_128B
    return d;
}

// The same for 16-channel K blocks (64-byte rows, 64-byte swizzle: 8-row
// groups 512 bytes apart), and the descriptor of a K block of BK channels.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);       // start address
    d |= (uint64_t)1 << 16;                        // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(512 >> 4) << 32;               // stride byte offset
    d |= (uint64_t)1 << 46;                        // version
    d |= (uint64_t)4 << 61;                        // layout: SWIZZLE_64B
    return d;
}

template <int BK>
__device__ __forceinline__ uint64_t smem_desc_k(uint32_t saddr)
{
    if constexpr (BK == 16) return smem_desc_sw64(saddr);
    else return smem_desc_sw128(saddr);
}

// Instruction descriptor, kind::tf32: D f32, A/B tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t m, uint32_t n)
{
    return (1u << 4)            // D format f32
           | (2u << 7)          // A format tf32
           | (2u << 10)         // B format tf32
           | ((n >> 3) << 17)   // N / 8
           | ((m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// The same MMA with each descriptor given as its low word (start address
// and leading offset, which the k x k loops step with 32-bit adds) and its
// high word (stride offset, version, swizzle: constant per kernel).
__device__ __forceinline__ void mma_tf32_lo(uint32_t tmem_d, uint32_t alo, uint32_t blo, uint32_t hi, uint32_t idesc,
                                            uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .b64 ad, bd;\n\t.reg .pred p;\n\t"
        "mov.b64 ad, {%1, %3};\n\t"
        "mov.b64 bd, {%2, %3};\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], ad, bd, %4, p;\n\t}" ::"r"(tmem_d),
        "r"(alo), "r"(blo), "r"(hi), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// TMEM -> registers.  tcgen05.ld is asynchronous until tcgen05.wait::ld;
// the wait names the destination registers as read-write operands so the
// compiler cannot move any use of them above it.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t *r)
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait16(uint32_t *r)
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// compiler-only fence on 16 registers (a wait already covered them)
__device__ __forceinline__ void reg_fence16(uint32_t *r)
{
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
    uint32_t r[16];
    tmem_ld16_issue(taddr, r);
    tmem_wait16(r);
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Issue the load of 32 accumulator columns (16 when only `remaining` <= 16
// are inside the tile; columns past `bn` may lie outside the TMEM
// allocation).  Complete with tmem_wait32.
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, int remaining, uint32_t (&r)[32])
{
    tmem_ld16_issue(taddr, r);
    if (remaining > 16) tmem_ld16_issue(taddr + 16, r + 16);
}

__device__ __forceinline__ void tmem_wait32(int remaining, uint32_t (&r)[32])
{
    tmem_wait16(r);
    reg_fence16(r + 16);
    if (remaining <= 16) {
#pragma unroll
        for (int i = 16; i < 32; i++) r[i] = 0u;
    }
}

// --------------------------------------------------------------- kernel ---

struct TcShared {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t acc_full[4];
    uint64_t acc_empty[4];
    uint64_t bfull;  // resident B landed
    uint32_t tmem_base;
    uint32_t abort;
};

// Output rows of unit `u`: decode (m tile, n tile, split).
struct TcUnit {
    uint32_t mt, nt, s;
};

// 32-bit multiply-high divisions: a 64-bit division has no hardware divider
// and cost ~1 us per tile in the epilogue
__device__ __forceinline__ TcUnit tc_unit(const TcArgs &a, uint64_t u64)
{
    const int u = (int)u64;
    TcUnit t;
    const int r = fdiv(u, a.div_ntiles);
    t.nt = (uint32_t)(u - r * (int)a.n_tiles);
    const int q = fdiv(r, a.div_split);
    t.s = (uint32_t)(r - q * (int)a.split);
    t.mt = (uint32_t)q;
    return t;
}

// First output pixel (frame, row, column) of k x k M tile mt
struct TcOrigin {
    int img, oy0, ox0;
};

__device__ __forceinline__ TcOrigin tc_origin(const TcArgs &a, uint32_t mt)
{
    TcOrigin o;
    o.img = fdiv((int)mt, a.div_perimg);
    const int rem = (int)mt - o.img * (int)(a.tiles_x * a.tiles_y);
    const int ty = fdiv(rem, a.div_tilesx), tx = rem - ty * (int)a.tiles_x;
    o.oy0 = ty * (int)a.bh;
    o.ox0 = tx * (int)a.bw;
    return o;
}

// Output pixel of accumulator row `row` of M tile `mt` (origin o for k x k
// tiles), or -1 if outside.
template <bool FLAT>
__device__ __forceinline__ long long tc_row_pixel(const TcArgs &a, uint32_t mt, const TcOrigin &o, uint32_t row)
{
    if (!a.igemm) {
        const long long m = (long long)mt * kTcBM + row;
        return m < a.c.M ? m : -1;
    }
    int oy, ox;
    if constexpr (FLAT) {
        const uint32_t y = row / a.bwx, x = row - y * a.bwx;
        if (x >= a.bw || y >= a.bh) return -1;  // a column of the right halo, or past the tile's rows
        oy = o.oy0 + (int)y;
        ox = o.ox0 + (int)x;
    } else {
        oy = o.oy0 + (int)(row >> a.lbw);
        ox = o.ox0 + (int)(row & (a.bw - 1));
    }
    if (oy >= a.c.oh || ox >= a.c.ow) return -1;
    return ((long long)o.img * a.c.oh + oy) * a.c.ow + ox;
}

// RES (the epilogue's residual source, one kernel per kind so that each
// layer's epilogue carries only its own code): 0 none, 1 residual tensor,
// 2 bilinear sample read directly, 3 exact-2x sample from per-warp patches.
// ACT: the activation when it is kNone or kRelu, else -1 (any kind, chosen
// at run time)
template <int RES, int ACT, bool FLAT, bool GBIAS = false, int BK = 32>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const TcArgs a,
                   const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmA2)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-align the stage buffers (128-byte swizzle atoms)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // stage = A tile (+ B tile unless B is resident for the whole kernel)
    const uint32_t btiles = a.b_resident ? 0u : FLAT ? (uint32_t)(a.c.kh * a.c.kw) : a.halo ? (uint32_t)a.c.kh : 1u;
    const uint32_t stage_bytes = a.a_bytes + btiles * a.b_bytes;
    const uint32_t stage_tx = a.a_box + btiles * a.b_bytes;  // bytes the stage's copies write
    TcShared &sh = *reinterpret_cast<TcShared *>(smem + a.shared_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < a.stages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], 1);
        }
        for (int b = 0; b < 4; b++) {
            mbar_init(&sh.acc_full[b], 1);
            mbar_init(&sh.acc_empty[b], 4);
        }
        mbar_init(&sh.bfull, 1);
        sh.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
        if (a.nparts > 1) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA1)) : "memory");
        if (a.nparts > 2) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA2)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem_base)),
                     "r"(a.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;
    volatile uint32_t *abort_flag = &sh.abort;

    if (warp == 1 + kTcEpiWarps) {
        // ------------------------------------------------ TMA producer warp
        // Pipeline p owns stages [p*RS, (p+1)*RS) and the CTA's units j with
        // j % pipes == p.  Lane l serves pipeline p = l % pipes and issues
        // that pipeline's iterations q, q+LQ, q+2LQ, ... (q = l / pipes), each
        // lane on its own: a lane waits only for the stage it fills next.
        const uint32_t P = a.pipes, RS = a.stages / a.pipes;
        // the lanes of one warp issue in lockstep rounds and a round waits for
        // all of its stages, so a round leaves two stages of the ring in
        // flight; more than 4 lanes measured no faster (about one box in
        // flight per lane: 4 lanes already reach ~0.23 us per box per SM)
        const uint32_t LQ = max(1u, min(min((uint32_t)kTcIssueLanes / P, 4u), RS > 2 ? RS - 2 : 1u));
        const uint32_t pl = (uint32_t)lane % P, q = (uint32_t)lane / P;
        struct Cursor {
            uint32_t u;  // units < 2^32 (m tiles < 2^24)
            uint32_t k, k1;
        };
        auto enter = [&](Cursor &cu) {  // first K iteration of unit cu.u
            if (cu.u < a.units) {
                const TcUnit t = tc_unit(a, cu.u);
                cu.k = t.s * a.k_per_split;
                cu.k1 = min(a.k_iters, cu.k + a.k_per_split);
            }
        };
        auto advance = [&](Cursor &cu) {
            if (++cu.k >= cu.k1) {
                cu.u += P * gridDim.x;
                enter(cu);
            }
        };
        if (a.b_resident && lane == 0) {
            // the whole B of the (single) n-tile, one box per (tap, K block),
            // in k order: k = tap * kblocks + kb at bres_off + k * b_bytes
            const uint32_t nb = (uint32_t)(a.c.kh * a.c.kw) * a.kblocks;
            mbar_expect_tx(&sh.bfull, nb * a.b_bytes);
            for (uint32_t k = 0; k < nb; k++) {
                const uint32_t tap = k / a.kblocks, kb = k - tap * a.kblocks;
                tma_load_3d(smem + a.bres_off + k * a.b_bytes, &tmB, &sh.bfull, (int)(kb * BK), 0, (int)tap);
            }
        }
        uint32_t last_mine = 0xFFFFFFFFu;
        if (q < LQ) {
            Cursor cur{(uint32_t)blockIdx.x + pl * gridDim.x, 0u, 0u};
            enter(cur);
            uint32_t it = 0;  // this pipeline's iteration index
            for (uint32_t i = 0; i < q && cur.u < a.units; i++, it++) advance(cur);
            while (cur.u < a.units) {
                const uint32_t s = pl * RS + it % RS, ph = (it / RS) & 1;
                if (*abort_flag || !mbar_wait(&sh.empty[s], ph ^ 1)) {
                    report_error(0x01000001);
                    *abort_flag = 1;
                    break;
                }
                const TcUnit t = tc_unit(a, cur.u);
                uint8_t *sa = smem + s * stage_bytes;
                uint8_t *sb = sa + a.a_bytes;
                mbar_expect_tx(&sh.full[s], stage_tx);
                const uint32_t k = cur.k;
                const uint32_t tap = k / a.kblocks, kb = k - tap * a.kblocks;
                const int kc = (int)(kb * BK);
                // the A copy of K block kbx: its part's tensor map and channel coordinate
                auto amap = [&](uint32_t kbx, int &ac) -> const CUtensorMap * {
                    if (a.nparts > 2 && kbx >= a.kb2) {
                        ac = (int)((kbx - a.kb2) * BK);
                        return &tmA2;
                    }
                    if (a.nparts > 1 && kbx >= a.kb1) {
                        ac = (int)((kbx - a.kb1) * BK);
                        return &tmA1;
                    }
                    ac = (int)(kbx * BK);
                    return &tmA;
                };
                int ac;
                if (FLAT) {
                    // stage = K block k: the tile's whole input window, every tap's B
                    const TcOrigin o = tc_origin(a, t.mt);
                    const CUtensorMap *tm = amap(k, ac);
                    tma_load_4d(sa, tm, &sh.full[s], ac, o.ox0 - a.c.pl, o.oy0 - a.c.pt, o.img);
                    if (!a.b_resident)
                        for (int tp = 0; tp < a.c.kh * a.c.kw; tp++)
                            tma_load_3d(sb + tp * a.b_bytes, &tmB, &sh.full[s], (int)(k * BK), (int)(t.nt * a.bn),
                                        tp);
                } else if (a.halo) {
                    // stage = column shift kx (= tap here), K block kb: rows
                    // [ybase, ybase + bh + kh - 1) x the bw columns at xbase + kx
                    const TcOrigin o = tc_origin(a, t.mt);
                    const CUtensorMap *tm = amap(kb, ac);
                    tma_load_4d(sa, tm, &sh.full[s], ac, o.ox0 - a.c.pl + (int)tap, o.oy0 - a.c.pt, o.img);
                    if (!a.b_resident)
                        for (int ky = 0; ky < a.c.kh; ky++)
                            tma_load_3d(sb + ky * a.b_bytes, &tmB, &sh.full[s], kc, (int)(t.nt * a.bn),
                                        ky * a.c.kw + (int)tap);
                } else if (a.igemm) {
                    const TcOrigin o = tc_origin(a, t.mt);
                    const int ybase = o.oy0 * a.c.sh - a.c.pt;
                    const int xbase = o.ox0 * a.c.sw - a.c.pl;
                    const int ky = (int)(tap / a.c.kw), kx = (int)(tap - ky * a.c.kw);
                    const CUtensorMap *tm = amap(kb, ac);
                    tma_load_4d(sa, tm, &sh.full[s], ac, xbase + kx * a.c.dil, ybase + ky * a.c.dil, o.img);
                } else {
                    const CUtensorMap *tm = amap(kb, ac);
                    tma_load_2d(sa, tm, &sh.full[s], ac, (int)(t.mt * kTcBM));
                }
                if (!a.b_resident && !a.halo && !FLAT)
                    tma_load_3d(sb, &tmB, &sh.full[s], kc, (int)(t.nt * a.bn), (int)tap);
                last_mine = s | (ph << 16);
                for (uint32_t i = 0; i < LQ && cur.u < a.units; i++, it++) advance(cur);
            }
        }
        // drain: wait (bounded) until the copies this lane issued have landed
        if (last_mine != 0xFFFFFFFFu) mbar_wait(&sh.full[last_mine & 0xFFFF], last_mine >> 16);
        if (a.b_resident && lane == 0) mbar_wait(&sh.bfull, 0);
        __syncwarp();
    } else if (warp == 0 || warp == kTcMmaWarp1) {
        // ------------------------------------------------ MMA issuers
        // pipeline p: units j = p, p + pipes, ... of this CTA, stage ring p,
        // accumulator buffer (tile count) as the epilogue group that drains it
        auto mma_pipeline = [&](auto pc) {
        constexpr uint32_t p = decltype(pc)::value;
        if (lane == 0 && p < a.pipes) {
            const uint32_t P = a.pipes, RS = a.stages / a.pipes;
            const uint32_t idesc = idesc_tf32(kTcBM, a.bn);
            uint32_t it = 0, nt = 0;
            uint32_t rs_slot = 0, rs_phase = 0;  // it % RS, (it / RS) & 1
            bool ok = true;
            if (a.b_resident && blockIdx.x + p * gridDim.x < a.units) {
                if (*abort_flag || !mbar_wait(&sh.bfull, 0)) {
                    report_error(0x01000005);
                    *abort_flag = 1;
                    ok = false;
                }
            }
            for (uint64_t u = blockIdx.x + (uint64_t)p * gridDim.x; u < a.units && ok; u += (uint64_t)P * gridDim.x, nt++) {
                const TcUnit t = tc_unit(a, u);
                const uint32_t k0 = t.s * a.k_per_split;
                const uint32_t k1 = min(a.k_iters, k0 + a.k_per_split);
                // accumulator buffer: with two pipelines each owns two (its
                // tiles alternate between them, so a tile's MMAs never wait
                // for the epilogue of the pipeline's previous tile); with one,
                // tiles alternate between the two buffers
                const uint32_t ab = P == 2 ? p * 2 + (nt & 1) : (nt & 1), aph = (nt >> 1) & 1;
                if (*abort_flag || !mbar_wait(&sh.acc_empty[ab], aph ^ 1)) {
                    report_error(0x01000002);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + ab * a.bn;
                // halo mode: K iteration k = (column shift kx, K block kb)
                uint32_t hkx = k0 / a.kblocks, hkb = k0 - hkx * a.kblocks;
                for (uint32_t k = k0; k < k1; k++, it++) {
                    // (the ring slot and phase advance with the iteration; a
                    // role that gave up leaves this wait to run out, so the
                    // abort flag is read per tile, not per K block)
                    const uint32_t s = p * RS + rs_slot, ph = rs_phase;
                    if (++rs_slot == RS) {
                        rs_slot = 0;
                        rs_phase ^= 1u;
                    }
                    if (!mbar_wait(&sh.full[s], ph)) {
                        report_error(0x01000003);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * stage_bytes);
                    // one K block: bk / 8 MMAs, each 8 tf32 = 32 bytes further
                    // along K inside the swizzle row
                    constexpr uint32_t rowb = BK * 4;
                    auto kblock = [&](uint64_t ad, uint64_t bd, bool acc0) {
                        if constexpr (BK == 16) {
                            mma_tf32(d, ad, bd, idesc, acc0 ? 0u : 1u);
                            mma_tf32(d, ad + 2, bd + 2, idesc, 1u);
                        } else {
#pragma unroll
                            for (uint32_t kk = 0; kk < 4; kk++)
                                mma_tf32(d, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
                                         (acc0 && kk == 0) ? 0u : 1u);
                        }
                    };
                    // k x k stride-1 tiles, 32-channel K blocks: the descriptors'
                    // low words (start address / 16) step by 32-bit adds from tap
                    // to tap and by 2 (32 bytes) from MMA to MMA; the high word
                    // is constant (the issuing thread's instructions per MMA set
                    // the pace of these narrow tiles: fpn.smooth4 148 -> 130 us,
                    // RVM's d0.conv1 1422 -> 1231 us against 64-bit descriptors
                    // built per tap; 16-channel blocks measured slower this way,
                    // d0.conv2 638 -> 679 us, and keep them)
                    const uint64_t d0 = smem_desc_k<BK>(sa);
                    const uint32_t dhi = (uint32_t)(d0 >> 32);
                    auto kblock_lo = [&](uint32_t al, uint32_t bl, uint32_t acc) {
                        mma_tf32_lo(d, al, bl, dhi, idesc, acc);
#pragma unroll
                        for (uint32_t kk = 1; kk < BK / 8; kk++) mma_tf32_lo(d, al + kk * 2, bl + kk * 2, dhi, idesc, 1u);
                    };
                    if constexpr (FLAT && BK == 16) {
                        // K block k; tap (ky, kx) reads the box from row ky * bwx + kx
                        for (uint32_t ky = 0; ky < (uint32_t)a.c.kh; ky++)
                            for (uint32_t kx = 0; kx < (uint32_t)a.c.kw; kx++) {
                                const uint32_t tap = ky * a.c.kw + kx;
                                const uint32_t sb = a.b_resident
                                                        ? smem_u32(smem + a.bres_off + (tap * a.kblocks + k) * a.b_bytes)
                                                        : sa + a.a_bytes + tap * a.b_bytes;
                                kblock(smem_desc_k<BK>(sa + (ky * a.bwx + kx) * rowb), smem_desc_k<BK>(sb),
                                       k == k0 && tap == 0);
                            }
                    } else if constexpr (FLAT) {
                        // K block k; tap (ky, kx) reads the box from row ky * bwx + kx
                        // (a fully unrolled 3 x 3 loop with precomputed descriptors
                        // measured 10-50% slower: smooth4 141 -> 168 us)
                        const uint32_t a_lo = (uint32_t)d0;
                        uint32_t bl = (uint32_t)smem_desc_k<BK>(
                            a.b_resident ? smem_u32(smem + a.bres_off + k * a.b_bytes) : sa + a.a_bytes);
                        const uint32_t b_step = (a.b_resident ? a.kblocks * a.b_bytes : a.b_bytes) >> 4;
                        uint32_t acc = k == k0 ? 0u : 1u;
                        for (uint32_t ky = 0; ky < (uint32_t)a.c.kh; ky++) {
                            uint32_t al = a_lo + ky * a.bwx * (rowb >> 4);
                            for (uint32_t kx = 0; kx < (uint32_t)a.c.kw; kx++) {
                                kblock_lo(al, bl, acc);
                                acc = 1u;
                                al += rowb >> 4;
                                bl += b_step;
                            }
                        }
                    } else if (a.halo && BK == 16) {
                        // tap (ky, kx): the stage's copy shifted down ky rows
                        // (ky * bw A rows, a multiple of 8 rows: swizzle-aligned)
                        const uint32_t kx = hkx, kb = hkb;
                        for (uint32_t ky = 0; ky < (uint32_t)a.c.kh; ky++) {
                            const uint32_t tap = ky * a.c.kw + kx;
                            const uint32_t sb = a.b_resident
                                                    ? smem_u32(smem + a.bres_off + (tap * a.kblocks + kb) * a.b_bytes)
                                                    : sa + a.a_bytes + ky * a.b_bytes;
                            kblock(smem_desc_k<BK>(sa + ky * a.bw * rowb), smem_desc_k<BK>(sb), k == k0 && ky == 0);
                        }
                    } else if (a.halo) {
                        const uint32_t kx = hkx, kb = hkb;
                        uint32_t al = (uint32_t)d0;
                        uint32_t bl = (uint32_t)smem_desc_k<BK>(
                            a.b_resident ? smem_u32(smem + a.bres_off + (kx * a.kblocks + kb) * a.b_bytes) : sa + a.a_bytes);
                        const uint32_t a_step = (a.bw * rowb) >> 4;
                        const uint32_t b_step = (a.b_resident ? a.c.kw * a.kblocks * a.b_bytes : a.b_bytes) >> 4;
                        uint32_t acc = k == k0 ? 0u : 1u;
                        for (uint32_t ky = 0; ky < (uint32_t)a.c.kh; ky++) {
                            kblock_lo(al, bl, acc);
                            acc = 1u;
                            al += a_step;
                            bl += b_step;
                        }
                    } else if constexpr (BK == 16) {
                        const uint32_t sb = a.b_resident ? smem_u32(smem + a.bres_off + k * a.b_bytes) : sa + a.a_bytes;
                        kblock(smem_desc_k<BK>(sa), smem_desc_k<BK>(sb), k == k0);
                    } else {
                        const uint32_t sb = a.b_resident ? smem_u32(smem + a.bres_off + k * a.b_bytes) : sa + a.a_bytes;
                        kblock_lo((uint32_t)d0, (uint32_t)smem_desc_k<BK>(sb), k == k0 ? 0u : 1u);
                    }
                    if (++hkb == a.kblocks) {
                        hkb = 0;
                        hkx++;
                    }
                    mma_commit(&sh.empty[s]);
                }
                if (!ok) break;
                mma_commit(&sh.acc_full[ab]);
            }
            // drain: wait (bounded) for the MMAs this thread issued before the
            // TMEM they write can be freed
            if (it > 0) {
                const uint32_t last = it - 1;
                mbar_wait(&sh.empty[p * RS + last % RS], (last / RS) & 1);
            }
        }
        };
        if (warp == 0) mma_pipeline(std::integral_constant<uint32_t, 0>{});
        else mma_pipeline(std::integral_constant<uint32_t, 1>{});
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (warps 1..8)
        // Two groups of four warps; group g drains TMEM accumulator buffer g,
        // i.e. every other tile, so two tiles' epilogues run at once.  Within
        // a group, warp w owns TMEM lane quadrant w % 4 (= accumulator rows).
        const uint32_t ew = (uint32_t)(warp - 1);  // 0..7: staging buffer
        const uint32_t grp = ew >> 2;              // accumulator buffer this group drains
        const uint32_t quad = warp & 3;            // TMEM lane quadrant this warp may access
        uint8_t *obuf = smem + a.out_off + ew * kTcStageOut;  // 32 x 32 fp32 staging
        // this warp's copy of the n-tile's bias (zero past cout), reloaded
        // only when the n-tile changes; read as broadcasts
        float *bcache = reinterpret_cast<float *>(smem + a.out_off + 8 * kTcStageOut) + ew * 256;
        uint32_t bias_nt = 0xFFFFFFFFu;
        int bias_base = 0;  // first column of the cached bias
        const ConvArgs &c = a.c;
        const int seg = lane & 7;
        int mrow[8];  // output pixel of the 8 rows this lane stores, -1 outside (M < 2^31)

        // bias -> act on this lane's row, staged through shared memory, then
        // written back by the warp 8 lanes per 128-byte row segment so every
        // store (and residual load) instruction covers 4 whole rows instead
        // of 32 scattered 16-byte pieces; residual added after the activation
        // RES (the kernel's template argument) picks the residual source
        // residual tensor (RES 1, 16-byte aligned rows): the 8 x 16 bytes this
        // lane adds for the chunk at col0 are fetched with cp.async into this
        // warp's residual buffer ahead of use, so their latency overlaps the
        // MMA wait and the TMEM drain without holding registers; each lane
        // later reads back only what it fetched itself
        auto prefetch_res = [&](int col0) {
            const int col = col0 + seg * 4;
            const bool vec = c.vec_y && col + 4 <= c.cout;
            if (!a.res_off || !vec) return;
            uint8_t *rbuf = smem + a.res_off + ew * kTcStageOut;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int r = i * 4 + (lane >> 3);
                const bool ok = mrow[i] >= 0;
                const float *src = ok ? c.res + (long long)mrow[i] * c.r_stride + c.r_coff + col : c.res;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                                 smem_u32(rbuf + r * 128 + ((seg ^ (r & 7)) * 16))),
                             "l"(src), "r"(ok ? 16 : 0)
                             : "memory");
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };

        // exact-2x residual (RES 3): the source pixels of this warp's 32 rows
        // for the chunk at col0, [segment][row][column] x 128 bytes, fetched
        // with cp.async ahead of use like the residual rows above (columns
        // past the source's edge repeat its last column; channels past cout
        // are zero-filled)
        int wm0 = -1;  // first output pixel of this warp's rows (1x1 tiles), -1 past M
        auto prefetch_patch = [&](int col0) {
            if (wm0 < 0) return;
            const Up2Patch p = up2_patch(c, wm0);
            uint8_t *pb = smem + a.res_off + ew * kTcPatchBytes;
            const float *rb = c.res + c.r_coff + col0;
#pragma unroll 6
            for (int j = 0; j < (int)(kTcPatchBytes / 16 / 32); j++) {
                const int idx = j * 32 + lane;
                const int slot = idx >> 3, piece = idx & 7;
                const int sg = slot >= 2 * kTcPatchCols ? 1 : 0;
                const int rem = slot - 2 * kTcPatchCols * sg;
                const int ry = rem >= kTcPatchCols ? 1 : 0;
                const int cx = rem - kTcPatchCols * ry;
                const int img = sg ? p.img1 : p.img0;
                const int y = sg ? (ry ? p.y11 : p.y10) : (ry ? p.y01 : p.y00);
                const int x = min((sg ? 0 : p.qc0) + cx, c.rw - 1);
                const bool ok = col0 + piece * 4 < c.cout;
                const float *src = ok ? rb + (((long long)img * c.rh + y) * c.rw + x) * c.r_stride + piece * 4 : c.res;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(pb + slot * 128 + piece * 16)),
                             "l"(src), "r"(ok ? 16 : 0)
                             : "memory");
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        auto prefetch_any = [&](int col0) {
            if constexpr (RES == 3) prefetch_patch(col0);
            else if constexpr (RES == 1) prefetch_res(col0);
        };
        // row r of this warp (pixel wm0 + r), channels seg*4.. of the chunk
        auto patch_res4 = [&](const Up2Patch &p, int r) {
            const int oxr = p.ox0 + r;
            const int sg = oxr >= c.ow ? 1 : 0;
            const int ox = sg ? oxr - c.ow : oxr;
            const int fx = (ox - 1) >> 1, qc = sg ? 0 : p.qc0;
            const int x0 = max(fx, 0) - qc, x1 = min(fx + 1, c.rw - 1) - qc;
            const uint8_t *sb = smem + a.res_off + ew * kTcPatchBytes + sg * (2 * kTcPatchCols * 128) + seg * 16;
            const float4 g00 = *reinterpret_cast<const float4 *>(sb + x0 * 128);
            const float4 g01 = *reinterpret_cast<const float4 *>(sb + x1 * 128);
            const float4 g10 = *reinterpret_cast<const float4 *>(sb + (kTcPatchCols + x0) * 128);
            const float4 g11 = *reinterpret_cast<const float4 *>(sb + (kTcPatchCols + x1) * 128);
            return bilinear_mix4(g00, g01, g10, g11, (ox & 1) ? 0.25f : 0.75f, (sg ? p.odd1 : p.odd0) ? 0.25f : 0.75f);
        };

        auto emit = [&](int col0, float (&v)[32]) {
            const int col = col0 + seg * 4;
            const bool vec = c.vec_y && col + 4 <= c.cout;
            // the chunk's bias: the warp's shared copy, or read by every lane
            // from the same global addresses (L1 broadcasts; the bias is
            // 16-byte aligned, checked at launch), zero past cout
            if constexpr (!GBIAS) {
                const float4 *bb = reinterpret_cast<const float4 *>(bcache + (col0 - bias_base));
#pragma unroll
                for (int q4 = 0; q4 < 8; q4++) {
                    const float4 b = bb[q4];
                    v[4 * q4] += b.x; v[4 * q4 + 1] += b.y; v[4 * q4 + 2] += b.z; v[4 * q4 + 3] += b.w;
                }
            } else if (col0 + 32 <= c.cout) {
                const float4 *bb = reinterpret_cast<const float4 *>(c.bias + col0);
#pragma unroll
                for (int q4 = 0; q4 < 8; q4++) {
                    const float4 b = __ldg(bb + q4);
                    v[4 * q4] += b.x; v[4 * q4 + 1] += b.y; v[4 * q4 + 2] += b.z; v[4 * q4 + 3] += b.w;
                }
            } else {
#pragma unroll
                for (int q4 = 0; q4 < 8; q4++) {
                    const int cb = col0 + 4 * q4;
                    if (cb + 4 <= c.cout) {
                        const float4 b = __ldg(reinterpret_cast<const float4 *>(c.bias + cb));
                        v[4 * q4] += b.x; v[4 * q4 + 1] += b.y; v[4 * q4 + 2] += b.z; v[4 * q4 + 3] += b.w;
                    } else if (cb < c.cout) {
#pragma unroll
                        for (int i = 0; i < 4; i++) v[4 * q4 + i] += cb + i < c.cout ? __ldg(c.bias + cb + i) : 0.0f;
                    }
                }
            }
            act_fixed_n<ACT, 32>(c.act, v);
            __syncwarp();  // previous chunk's readers are done with the buffer
            uint8_t *st = obuf + lane * 128;
#pragma unroll
            for (int ch = 0; ch < 8; ch++)
                *reinterpret_cast<float4 *>(st + ((ch ^ (lane & 7)) * 16)) =
                    make_float4(v[4 * ch], v[4 * ch + 1], v[4 * ch + 2], v[4 * ch + 3]);
            __syncwarp();
            if constexpr (RES == 1) {
                if (a.res_off) asm volatile("cp.async.wait_all;" ::: "memory");  // this lane's prefetched rows
            }
            Up2Patch pt{};
            if constexpr (RES == 3) {
                asm volatile("cp.async.wait_all;" ::: "memory");
                __syncwarp();  // the patch was fetched by the whole warp
                pt = up2_patch(c, max(wm0, 0));
            }
            if (col >= c.y_pad_to) return;
            // four rows at a time: their residual loads are issued together
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float4 rv[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = 4 * h + q;
                    rv[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if constexpr (RES == 2) {
                        if (mrow[i] >= 0) rv[q] = bilinear_res4(c, mrow[i], col, vec);
                    } else if constexpr (RES == 3) {
                        if (mrow[i] >= 0) rv[q] = patch_res4(pt, i * 4 + (lane >> 3));
                    }
                    if constexpr (RES == 1) {
                        if (mrow[i] >= 0) {
                            if (a.res_off && vec) {
                                const int r = i * 4 + (lane >> 3);
                                rv[q] = *reinterpret_cast<const float4 *>(smem + a.res_off + ew * kTcStageOut + r * 128 +
                                                                          ((seg ^ (r & 7)) * 16));
                            } else {
                                const float *rr = c.res + (long long)mrow[i] * c.r_stride + c.r_coff + col;
                                if (vec) rv[q] = __ldg(reinterpret_cast<const float4 *>(rr));
                                else {
                                    float t4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                                    for (int l = 0; l < 4; l++)
                                        if (col + l < c.cout) t4[l] = __ldg(rr + l);
                                    rv[q] = make_float4(t4[0], t4[1], t4[2], t4[3]);
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int i = 4 * h + q;
                    const int r = i * 4 + (lane >> 3);
                    if (mrow[i] < 0) continue;
                    float4 x = *reinterpret_cast<const float4 *>(obuf + r * 128 + ((seg ^ (r & 7)) * 16));
                    if constexpr (RES != 0) {
                        x.x += rv[q].x; x.y += rv[q].y; x.z += rv[q].z; x.w += rv[q].w;  // residual after act
                    }
                    float *yr = c.y + (long long)mrow[i] * c.y_stride + c.y_coff + col;
                    if (vec) {
                        *reinterpret_cast<float4 *>(yr) = x;
                    } else {
                        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                        for (int l = 0; l < 4; l++) {
                            if (col + l < c.cout) yr[l] = xs[l];
                            else if (col + l < c.y_pad_to) yr[l] = 0.0f;
                        }
                    }
                }
            }
        };

        auto emit_any = [&](int col0, float (&v)[32]) { emit(col0, v); };
        // residuals fetched into the per-warp buffers ahead of use
        constexpr bool res_tensor = RES == 1 || RES == 3;

        uint32_t k = 0;  // tiles this group has drained: the phase of its buffer
        for (uint64_t u = blockIdx.x + (uint64_t)grp * gridDim.x; u < a.units; u += 2ull * gridDim.x, k++) {
            const TcUnit t = tc_unit(a, u);
            // the group's k-th tile: buffer grp (one pipeline) or 2 grp + k % 2
            // (two pipelines, pipeline grp's tiles), see the MMA issuers
            const uint32_t ab = a.pipes == 2 ? grp * 2 + (k & 1) : grp, aph = a.pipes == 2 ? (k >> 1) & 1 : k & 1;
            const int ncol = (int)min(a.bn, (uint32_t)c.y_pad_to - t.nt * a.bn);
            const int nbase = (int)(t.nt * a.bn);
            const uint32_t tbase = tmem + ((quad * 32) << 16) + ab * a.bn;
            const uint64_t tile = (uint64_t)t.mt * a.n_tiles + t.nt;
            const TcOrigin org = a.igemm ? tc_origin(a, t.mt) : TcOrigin{0, 0, 0};
#pragma unroll
            for (int i = 0; i < 8; i++) mrow[i] = (int)tc_row_pixel<FLAT>(a, t.mt, org, quad * 32 + i * 4 + (lane >> 3));
            if constexpr (RES == 3) {
                const long long m0 = (long long)t.mt * kTcBM + quad * 32;
                wm0 = m0 < c.M ? (int)m0 : -1;
            }
            if (!GBIAS && t.nt != bias_nt) {
                __syncwarp();
                for (int i = lane; i < 256; i += 32) bcache[i] = (nbase + i < c.cout) ? __ldg(c.bias + nbase + i) : 0.0f;
                __syncwarp();
                bias_nt = t.nt;
                bias_base = nbase;
            }
            if (res_tensor && a.split == 1) prefetch_any(nbase);  // first chunk, ahead of the MMA wait
            if (a.split == 1) {
                // the epilogue warps sleep on the accumulator barrier so that
                // their polling does not take issue slots from the MMA and
                // producer warps sharing their sub-partitions
                const bool ok = !*abort_flag && mbar_wait_sleep(&sh.acc_full[ab], aph);
                if (ok) {
                    tc_fence_after();
                    for (int c0 = 0; c0 < ncol; c0 += 32) {
                        uint32_t r[32];
                        tmem_ld32_issue(tbase + c0, (int)a.bn - c0, r);
                        tmem_wait32((int)a.bn - c0, r);
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
                        emit_any(nbase + c0, v);
                        if (res_tensor && c0 + 32 < ncol) {
                            __syncwarp();  // every lane has read its rows of the buffer
                            prefetch_any(nbase + c0 + 32);
                        }
                    }
                }
                if (!ok) {
                    asm volatile("cp.async.wait_all;" ::: "memory");  // no copy may land after exit
                    report_error(0x01000004);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.acc_empty[ab]);
            } else {
                if (*abort_flag || !mbar_wait_sleep(&sh.acc_full[ab], aph)) {
                    report_error(0x01000004);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                // raw partial -> workspace, release the accumulator, then take
                // this warp's ticket for its 32 rows (no cross-warp barrier:
                // every warp finishes on its own even if another gave up).
                // Layout [tile][split][quadrant][bn / 4][32 lanes] of float4:
                // the warp's 32 rows of one 4-column group are 512 contiguous
                // bytes, so every store (and every load of the reduction
                // below, made by the same lanes) is one coalesced transaction.
                const uint64_t qstride = (uint64_t)(a.bn / 4) * 32;  // float4s per (split, quadrant)
                float4 *wq = reinterpret_cast<float4 *>(a.ws) + ((tile * a.split + t.s) * 4 + quad) * qstride + lane;
                for (int c0 = 0; c0 < (int)a.bn; c0 += 16) {
                    float v[16];
                    tmem_ld16(tbase + c0, v);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        wq[(uint32_t)(c0 / 4 + q) * 32] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.acc_empty[ab]);
                __threadfence();
                __syncwarp();
                uint32_t *ticket = a.tickets + tile * 4 + quad;
                uint32_t last = 0;
                if (lane == 0) last = atomicAdd(ticket, 1u) == a.split - 1 ? 1u : 0u;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    // this warp's rows of split 0; split s is s * sstride further
                    const float4 *base = reinterpret_cast<const float4 *>(a.ws) + (tile * a.split * 4 + quad) * qstride + lane;
                    const uint64_t sstride = 4 * qstride;
                    for (int c0 = 0; c0 < ncol; c0 += 32) {  // a.bn is a multiple of 32
                        if (res_tensor) {
                            __syncwarp();  // every lane has read its rows of the buffer
                            prefetch_any(nbase + c0);  // lands while the partials are summed
                        }
                        const float4 *p = base + (uint32_t)(c0 / 4) * 32;
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = 0.0f;
                        // summed in split order from zero (deterministic); two
                        // splits' loads in flight at a time
                        uint32_t s = 0;
                        for (; s + 2 <= a.split; s += 2) {
                            float4 x0[8], x1[8];
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                x0[q] = __ldcg(p + s * sstride + q * 32);
                                x1[q] = __ldcg(p + (s + 1) * sstride + q * 32);
                            }
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                v[4 * q] += x0[q].x; v[4 * q + 1] += x0[q].y; v[4 * q + 2] += x0[q].z; v[4 * q + 3] += x0[q].w;
                            }
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                v[4 * q] += x1[q].x; v[4 * q + 1] += x1[q].y; v[4 * q + 2] += x1[q].z; v[4 * q + 3] += x1[q].w;
                            }
                        }
                        if (s < a.split) {
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                const float4 x = __ldcg(p + s * sstride + q * 32);
                                v[4 * q] += x.x; v[4 * q + 1] += x.y; v[4 * q + 2] += x.z; v[4 * q + 3] += x.w;
                            }
                        }
                        emit_any(nbase + c0, v);
                    }
                    __syncwarp();
                    if (lane == 0) *ticket = 0;  // reusable by the next launch
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols));
    }
}

// --------------------------------------------------------------- host ---

static inline uint32_t tc_pow2_ceil(uint32_t v)
{
    uint32_t p = 32;
    while (p < v) p <<= 1;
    return p;
}

static inline bool tc_available() { return true; }

// k x k geometries the tensor-core path takes: strides 1-2 (the TMA box
// spans bw*sw <= 256 elements).
static inline bool tc_igemm_supported(uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ow)
{
    (void)kh; (void)kw; (void)ow;
    return sh >= 1 && sh <= 2 && sw >= 1 && sw <= 2;
}

// Plan the tensor-core launch.  Returns 0 or a negative code.
static inline int tc_plan(uint32_t n, uint32_t ih, uint32_t iw, uint32_t cin, uint32_t cout, uint32_t kh, uint32_t kw,
                          uint32_t sh, uint32_t sw, uint32_t dil, uint32_t pt, uint32_t pl, uint32_t oh, uint32_t ow,
                          uint32_t split_req, uint32_t res_kind, TcGeom *g, bool allow_halo = true,
                          bool allow_flat = true, uint32_t bk_req = 0)
{
    (void)ih; (void)iw; (void)pt; (void)pl;
    *g = TcGeom{};
    g->bm = kTcBM;
    const bool pw = kh == 1 && kw == 1 && sh == 1 && sw == 1;
    g->igemm = pw ? 0 : 1;
    g->taps = kh * kw;
    // K blocks of 32 channels (128-byte rows); one block of 16 (64-byte
    // rows, 64-byte swizzle) for cin <= 16, whose 32-wide block would be
    // half or more zero fill: half the MMAs (bound by the A operand's
    // shared-memory reads, which cost the same for data and padding) for
    // the same number of K blocks.  Where 16-channel blocks would need more
    // blocks than 32-channel ones (36 channels: 3 against 2) the per-block
    // copies and waits cost more than the MMAs saved (RVM's 3x3 36 -> 16:
    // 1415 -> 1820 us), so those keep 32.
    // (bk_req: the K block width a concat-parts plan laid its weights out in)
    g->bk = bk_req ? bk_req : (cin <= 16 && res_kind != kTcResUp2) ? 16u : (uint32_t)kTcBK;
    g->kblocks = (cin + g->bk - 1) / g->bk;
    g->k_iters = g->taps * g->kblocks;
    // Halo mode (k x k, stride 1, dilation 1): a 16 x 8 pixel tile's A for
    // tap (ky, kx) is rows [ky*16, ky*16 + 128) of one (8 + kh - 1) x 16
    // pixel box shifted by kx, so a stage loads one box per (kx, K block)
    // and feeds kh MMA groups: kw x kblocks boxes per tile instead of
    // kh x kw x kblocks.
    g->halo = (allow_halo && !pw && sh == 1 && sw == 1 && dil == 1 && kh >= 2 && kh <= 7) ? 1u : 0u;
    g->a_bytes = kTcBM * g->bk * 4;
    // N tile: fewest tiles of <= 256 columns, each a multiple of 32 so the
    // epilogue's 32-column store boxes never reach into the next tile
    const uint32_t nt = (cout + 255) / 256;
    g->bn = ((cout + nt - 1) / nt + 31) / 32 * 32;
    g->n_tiles = (cout + g->bn - 1) / g->bn;
    // Flat mode for narrow k x k stride-1 convs (N <= 64): their MMAs are
    // short, so the per-tap (or per-kx) TMA boxes set the pace; one box per
    // K block, 16 + kw - 1 pixels wide, serves every tap.  Accumulator rows
    // past the tile's 16 columns (and its last partial row) are computed
    // and dropped: 112 of 128 rows are outputs for a 3 x 3 kernel.
    if (g->halo && allow_flat && g->bn <= 64 && kw <= 7) {
        const uint32_t bwx = 16 + kw - 1, tr = kTcBM / bwx;
        const uint32_t rows = ((kh - 1) * bwx + (kw - 1) + kTcBM + bwx - 1) / bwx;
        g->flat = 1;
        g->halo = 0;
        g->bwx = bwx;
        g->bhx = rows;
        g->bw = 16;
        g->bh = tr;
        g->k_iters = g->kblocks;
        g->a_box = bwx * rows * g->bk * 4;
        g->a_bytes = (g->a_box + 1023) / 1024 * 1024;  // the next stage's copy stays 1 KB aligned
    }
    if (g->halo) {
        g->k_iters = kw * g->kblocks;
        g->a_bytes = (8 + kh - 1) * 16 * g->bk * 4;
    }
    if (!g->flat) g->a_box = g->a_bytes;
    if (g->flat) {
        g->tiles_x = (ow + g->bw - 1) / g->bw;
        g->tiles_y = (oh + g->bh - 1) / g->bh;
        g->m_tiles = n * g->tiles_x * g->tiles_y;
    } else if (g->halo) {
        g->bw = 16;
        g->bh = 8;
        g->tiles_x = (ow + g->bw - 1) / g->bw;
        g->tiles_y = (oh + g->bh - 1) / g->bh;
        g->m_tiles = n * g->tiles_x * g->tiles_y;
    } else if (g->igemm) {
        // M tile = bh x bw output pixels of one frame, bh*bw = 128; pick the
        // shape that wastes the fewest rows
        double best = 1e30;
        for (uint32_t bw = 1; bw <= 128; bw <<= 1) {
            const uint32_t bh = 128 / bw;
            if (bw * sw > 256 || bh * sh > 256) continue;
            const double cover = (double)((ow + bw - 1) / bw * bw) * ((oh + bh - 1) / bh * bh);
            if (cover < best) {
                best = cover;
                g->bw = bw;
                g->bh = bh;
            }
        }
        g->tiles_x = (ow + g->bw - 1) / g->bw;
        g->tiles_y = (oh + g->bh - 1) / g->bh;
        g->m_tiles = n * g->tiles_x * g->tiles_y;
    } else {
        const uint64_t M = (uint64_t)n * oh * ow;
        g->m_tiles = (uint32_t)((M + kTcBM - 1) / kTcBM);
    }
    uint64_t tiles = (uint64_t)g->m_tiles * g->n_tiles;
    uint32_t split = 1;
    if (split_req == 0) {
        if (tiles < 148 && g->k_iters >= 8) {
            // Too few tiles to fill the SMs: split K, and for 1x1 GEMMs
            // consider narrower N tiles too (more tiles share the work, and
            // each tile's last arrival sums fewer partial bytes).  Pick the
            // (N tile, split) with the lowest modelled time per CTA: MMA
            // issue (~0.072 us per tcgen05.mma) against operand loads
            // (~100 GB/s per SM from HBM), whichever is longer, per wave of
            // units, plus the partial write (~200 GB/s per SM) and the
            // reduction's L2 round trips (~0.5 us per two splits of a
            // 32-column chunk).
            double best = 1e30;
            uint32_t best_bn = g->bn, best_split = 1;
            for (uint32_t bn = g->bn;; bn = std::max(64u, (bn / 2 + 31) / 32 * 32)) {
                const uint64_t nt2 = (cout + bn - 1) / bn, t2 = (uint64_t)g->m_tiles * nt2;
                uint32_t sp = (uint32_t)std::min<uint64_t>(16, std::max<uint64_t>(1, 148 / t2));
                sp = std::min(sp, g->k_iters / 4 ? g->k_iters / 4 : 1u);
                const uint32_t kps = (g->k_iters + sp - 1) / sp;
                const uint64_t waves = (t2 * ((g->k_iters + kps - 1) / kps) + 147) / 148;
                const double mma = kps * 4 * 0.072;
                const double load = kps * (double)(g->a_bytes + bn * g->bk * 4) / 1e5;
                double t = waves * std::max(mma, load);
                if (sp > 1) t += 128.0 * bn * 4 / 2e5 + 0.5 * ((sp + 1) / 2) * (bn / 32);
                if (t < best) {
                    best = t;
                    best_bn = bn;
                    best_split = sp;
                }
                if (g->igemm || bn <= 64) break;  // k x k tiles keep their N tile
            }
            if (best_bn != g->bn) {
                g->bn = best_bn;
                g->n_tiles = (cout + g->bn - 1) / g->bn;
                tiles = (uint64_t)g->m_tiles * g->n_tiles;
            }
            split = best_split;
        }
    } else {
        split = std::min(split_req, g->k_iters);
    }
    if (split < 1) split = 1;
    g->k_per_split = (g->k_iters + split - 1) / split;
    g->split = (g->k_iters + g->k_per_split - 1) / g->k_per_split;  // no empty splits
    g->units = tiles * g->split;
    g->b_bytes = g->bn * g->bk * 4;
    // shared memory: [stages][resident B][epilogue staging][barriers]; stage
    // buffers and the resident B are 1024-aligned.  Per epilogue warp: a
    // 32 x 32 staging tile, a copy of the n-tile's bias (+ residual prefetch
    // buffers).  Where the ring would have fewer than four stages and the
    // bias copies are what costs the next one, they are dropped (the
    // epilogue then reads the bias from global memory, L1 broadcasts): the
    // wide (N = 256) tiles get their fourth 48 KB stage that way (config 2
    // 128 -> 256: 444 -> 507 TFLOP/s), while the shallow-K layers keep the
    // copies (global bias reads slowed their epilogue: e3.exp 43 -> 52 us).
    const uint32_t res_buf = res_kind == kTcResTensor ? kTcStageOut : res_kind == kTcResUp2 ? kTcPatchBytes : 0u;
    const uint32_t bias_bytes = kTcEpiWarps * 256 * 4;
    uint32_t out_bytes = kTcEpiWarps * (kTcStageOut + res_buf) + bias_bytes;
    const uint32_t limit = 227 * 1024 - 1024 /*align slack*/ - 256 /*barriers*/;
    // Resident B: with one n-tile and no K split every unit of a CTA uses the
    // same B, so it is loaded once (one TMA box per tap and K block) and each
    // stage carries only its A tile -- half the TMA operations per stage.
    const uint64_t bres = (uint64_t)g->taps * g->kblocks * g->b_bytes;
    g->b_resident = (g->n_tiles == 1 && g->split == 1 && bres <= kTcBResidentMax &&
                     (limit - out_bytes - bres) / g->a_bytes >= 4) ? 1u : 0u;
    const uint32_t stage = g->a_bytes + (g->b_resident ? 0u : (g->flat ? kh * kw : g->halo ? kh : 1u) * g->b_bytes);
    const uint32_t fixed = out_bytes + (g->b_resident ? (uint32_t)bres : 0u);
    g->stages = std::min<uint32_t>(8, (limit - fixed) / stage);
    g->bias_smem = 1;
    if (g->stages < 4 && !g->flat && res_kind <= kTcResTensor && (limit - fixed + bias_bytes) / stage > g->stages) {
        g->stages = std::min<uint32_t>(8, (limit - fixed + bias_bytes) / stage);
        g->bias_smem = 0;
        out_bytes -= bias_bytes;
    }
    // flat tiles want the weights resident: streamed, a stage carries kh*kw
    // B tiles (36 KB for a 3 x 3 at N = 32) and the ring shrinks to three
    // stages (a 3 x 3 72 -> 32 at 40 x 72 took 346 us flat against 234 us
    // with the per-kx halo boxes, whose stages carry kh B tiles)
    if (g->flat && (g->stages < 3 || !g->b_resident))  // the per-kx halo boxes instead
        return tc_plan(n, ih, iw, cin, cout, kh, kw, sh, sw, dil, pt, pl, oh, ow, split_req, res_kind, g, true, false,
                       bk_req);
    if (g->halo && g->stages < 3)  // halo stages too large (wide N): per-tap boxes
        return tc_plan(n, ih, iw, cin, cout, kh, kw, sh, sw, dil, pt, pl, oh, ow, split_req, res_kind, g, false, false,
                       bk_req);
    if (g->stages < 2) return -2;
    // narrow k x k tiles (long K loops, N <= 128) are bound by the per-thread
    // MMA issue cost: two pipelines.  1x1 GEMMs keep one deep ring (their
    // short K loops are bound by load latency, which halved rings expose).
    g->pipes = (g->igemm && g->bn <= 128 && g->stages >= 4) ? 2u : 1u;
    g->bres_off = g->stages * stage;
    g->out_off = g->bres_off + (g->b_resident ? (uint32_t)bres : 0u);
    g->res_off = res_buf ? g->out_off + kTcEpiWarps * kTcStageOut + (g->bias_smem ? bias_bytes : 0u) : 0u;
    g->res_patch = (res_kind == kTcResUp2 && !g->igemm) ? 1u : 0u;
    g->shared_off = g->out_off + out_bytes;
    g->tmem_cols = tc_pow2_ceil((g->pipes == 2 ? 4 : 2) * g->bn);  // two accumulators per pipeline
    if (g->tmem_cols > 512) return -3;
    g->smem_bytes = g->shared_off + 1024 + (uint32_t)sizeof(TcShared);
    g->grid = std::min<uint64_t>(g->units, 148);
    if (g->split > 1) {
        const uint64_t ws = tiles * g->split * kTcBM * g->bn * 4;
        g->workspace_bytes = (ws + 255) / 256 * 256 + (tiles * 16 + 255) / 256 * 256;
    }
    return 0;
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled tc_encoder()
{
    static PFN_encodeTiled fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_encodeTiled)p;
    }
    return fn;
}

static int tc_sm_count()
{
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    }
    return n;
}

// Concat parts of a tensor-core conv's input (see tc_conv_kernel): part p is
// the channel view x[p] (pixel stride stride[p], first channel coff[p]) of
// c[p] channels, starting at K block kb0[p].
struct TcParts {
    int n = 0;
    const float *x[3] = {nullptr, nullptr, nullptr};
    long long stride[3] = {0, 0, 0};
    int coff[3] = {0, 0, 0};
    uint32_t c[3] = {0, 0, 0};
    uint32_t kb0[3] = {0, 0, 0};
};

static inline int tc_launch(const TcGeom &g, const ConvArgs &c, void *workspace, cudaStream_t stream, char *err,
                            size_t errlen, const TcParts *parts = nullptr)
{
    PFN_encodeTiled enc = tc_encoder();
    if (!enc) {
        snprintf(err, errlen, "cuTensorMapEncodeTiled unavailable");
        return -4;
    }
    if ((uintptr_t)c.w % 16) {
        snprintf(err, errlen, "TMA operands must be 16-byte aligned (weights)");
        return -5;
    }
    // one A map per concat part (a plain conv is one part: its input view)
    TcParts one;
    if (!parts) {
        one.n = 1;
        one.x[0] = c.x;
        one.stride[0] = c.x_stride;
        one.coff[0] = c.x_coff;
        one.c[0] = (uint32_t)c.cin;
        parts = &one;
    }
    CUtensorMap tmAp[3], tmB;
    CUresult r = CUDA_SUCCESS;
    // 128-byte rows for 32-channel K blocks, 64-byte rows for 16-channel ones
    const CUtensorMapSwizzle swz = g.bk == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    for (int pi = 0; pi < parts->n && r == CUDA_SUCCESS; pi++) {
        const uintptr_t abase = (uintptr_t)(parts->x[pi] + parts->coff[pi]);
        const long long xs = parts->stride[pi];
        if (abase % 16 || (xs * 4) % 16) {
            snprintf(err, errlen, "TMA operands must be 16-byte aligned (input part %d + channel offset, pixel stride)", pi);
            return -5;
        }
        if (g.igemm) {
            const cuuint64_t dims[4] = {(cuuint64_t)parts->c[pi], (cuuint64_t)c.iw, (cuuint64_t)c.ih, (cuuint64_t)c.n};
            const cuuint64_t strides[3] = {(cuuint64_t)xs * 4, (cuuint64_t)xs * 4 * c.iw, (cuuint64_t)xs * 4 * c.iw * c.ih};
            const cuuint32_t box[4] = {(cuuint32_t)g.bk, g.flat ? g.bwx : g.bw * (cuuint32_t)c.sw,
                                       g.flat ? g.bhx : g.halo ? g.bh + (cuuint32_t)c.kh - 1 : g.bh * (cuuint32_t)c.sh, 1};
            const cuuint32_t estr[4] = {1, (cuuint32_t)c.sw, (cuuint32_t)c.sh, 1};
            r = enc(&tmAp[pi], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void *)abase, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        } else {
            const cuuint64_t dims[2] = {(cuuint64_t)parts->c[pi], (cuuint64_t)c.M};
            const cuuint64_t strides[1] = {(cuuint64_t)xs * 4};
            const cuuint32_t box[2] = {(cuuint32_t)g.bk, (cuuint32_t)kTcBM};
            const cuuint32_t estr[2] = {1, 1};
            r = enc(&tmAp[pi], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)abase, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        }
    }
    for (int pi = parts->n; pi < 3; pi++) tmAp[pi] = tmAp[0];  // unused
    if (r != CUDA_SUCCESS) {
        snprintf(err, errlen, "cuTensorMapEncodeTiled(A) failed: %d", (int)r);
        return -4;
    }
    {
        // weights [tap][cout][kpad]: kpad = cin rounded up to 4, or with
        // parts every part's channels rounded up to whole K blocks
        const uint32_t cin_pad = parts != &one ? g.kblocks * g.bk : (c.cin + 3) / 4 * 4;
        const cuuint64_t dims[3] = {(cuuint64_t)cin_pad, (cuuint64_t)c.cout, (cuuint64_t)(c.kh * c.kw)};
        const cuuint64_t strides[2] = {(cuuint64_t)cin_pad * 4, (cuuint64_t)cin_pad * 4 * c.cout};
        const cuuint32_t box[3] = {(cuuint32_t)g.bk, g.bn, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        r = enc(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)c.w, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            snprintf(err, errlen, "cuTensorMapEncodeTiled(B) failed: %d", (int)r);
            return -4;
        }
    }
    TcArgs a;
    a.c = c;
    a.bn = g.bn; a.bw = g.bw; a.bh = g.bh; a.tiles_x = g.tiles_x; a.tiles_y = g.tiles_y;
    a.m_tiles = g.m_tiles; a.n_tiles = g.n_tiles; a.split = g.split; a.k_iters = g.k_iters;
    a.k_per_split = g.k_per_split; a.kblocks = g.kblocks; a.stages = g.stages; a.tmem_cols = g.tmem_cols;
    a.b_bytes = g.b_bytes; a.igemm = g.igemm; a.units = g.units;
    a.b_resident = g.b_resident; a.bres_off = g.bres_off; a.res_off = g.res_off; a.pipes = g.pipes; a.bias_smem = g.bias_smem;
    a.halo = g.halo; a.a_bytes = g.a_bytes;
    a.flat = g.flat; a.bwx = g.bwx; a.a_box = g.a_box;
    a.nparts = (uint32_t)parts->n;
    a.kb1 = parts->kb0[1];
    a.kb2 = parts->kb0[2];
    // patches need 16-byte residual rows (the plan checked the shapes)
    a.res_patch = (g.res_patch && c.res && c.res_mode && c.vec_y) ? 1u : 0u;
    if (g.units >= (1ull << 31) || (uint64_t)g.m_tiles * g.n_tiles * g.split >= (1ull << 31)) {
        snprintf(err, errlen, "too many tensor-core tiles in one call (%llu); split the batch",
                 (unsigned long long)g.units);
        return -2;
    }
    a.div_ntiles = make_fastdiv((int)g.n_tiles);
    a.div_split = make_fastdiv((int)g.split);
    a.div_perimg = make_fastdiv((int)std::max<uint32_t>(1, g.tiles_x * g.tiles_y));
    a.div_tilesx = make_fastdiv((int)std::max<uint32_t>(1, g.tiles_x));
    a.lbw = 0;
    while ((1u << a.lbw) < g.bw) a.lbw++;
    a.out_off = g.out_off; a.shared_off = g.shared_off;
    a.ws = nullptr;
    a.tickets = nullptr;
    if (g.split > 1) {
        if (!workspace || (uintptr_t)workspace % 256) {
            snprintf(err, errlen, "split-K workspace missing or not 256-byte aligned");
            return -2;
        }
        const uint64_t tiles = (uint64_t)g.m_tiles * g.n_tiles;
        const uint64_t ws = (tiles * g.split * kTcBM * g.bn * 4 + 255) / 256 * 256;
        a.ws = (float *)workspace;
        a.tickets = (uint32_t *)((uint8_t *)workspace + ws);
        cudaError_t e = cudaMemsetAsync(a.tickets, 0, tiles * 16, stream);
        if (e != cudaSuccess) {
            snprintf(err, errlen, "ticket reset: %s", cudaGetErrorString(e));
            return -4;
        }
    }
    const int kind = !c.res ? 0 : !c.res_mode ? 1 : a.res_patch ? 3 : 2;
    // the activation as a template argument where it is none or ReLU (one
    // inlined switch over every kind per chunk costs instruction-cache misses)
    // flat mode is its own instantiation, so the other layers' kernels
    // carry none of its code (1x1 GEMMs measured 25% slower with it inline)
    using Kern = void (*)(CUtensorMap, CUtensorMap, TcArgs, CUtensorMap, CUtensorMap);
    static const Kern kerns[4][3] = {
        {tc_conv_kernel<0, kNone, false>, tc_conv_kernel<0, kRelu, false>, tc_conv_kernel<0, -1, false>},
        {tc_conv_kernel<1, kNone, false>, tc_conv_kernel<1, kRelu, false>, tc_conv_kernel<1, -1, false>},
        {tc_conv_kernel<2, kNone, false>, tc_conv_kernel<2, kRelu, false>, tc_conv_kernel<2, -1, false>},
        {tc_conv_kernel<3, kNone, false>, tc_conv_kernel<3, kRelu, false>, tc_conv_kernel<3, -1, false>}};
    // global bias reads (the ring's fourth stage in place of the bias copies;
    // never with exact-2x residual patches, see tc_plan)
    static const Kern kerns_gbias[3][3] = {
        {tc_conv_kernel<0, kNone, false, true>, tc_conv_kernel<0, kRelu, false, true>, tc_conv_kernel<0, -1, false, true>},
        {tc_conv_kernel<1, kNone, false, true>, tc_conv_kernel<1, kRelu, false, true>, tc_conv_kernel<1, -1, false, true>},
        {tc_conv_kernel<2, kNone, false, true>, tc_conv_kernel<2, kRelu, false, true>, tc_conv_kernel<2, -1, false, true>}};
    // 16-channel K blocks (cin <= 16): the plain and flat kernels again
    static const Kern kerns_k16[3][3] = {
        {tc_conv_kernel<0, kNone, false, false, 16>, tc_conv_kernel<0, kRelu, false, false, 16>,
         tc_conv_kernel<0, -1, false, false, 16>},
        {tc_conv_kernel<1, kNone, false, false, 16>, tc_conv_kernel<1, kRelu, false, false, 16>,
         tc_conv_kernel<1, -1, false, false, 16>},
        {tc_conv_kernel<2, kNone, false, false, 16>, tc_conv_kernel<2, kRelu, false, false, 16>,
         tc_conv_kernel<2, -1, false, false, 16>}};
    static const Kern kerns_flat_k16[3][3] = {
        {tc_conv_kernel<0, kNone, true, false, 16>, tc_conv_kernel<0, kRelu, true, false, 16>,
         tc_conv_kernel<0, -1, true, false, 16>},
        {tc_conv_kernel<1, kNone, true, false, 16>, tc_conv_kernel<1, kRelu, true, false, 16>,
         tc_conv_kernel<1, -1, true, false, 16>},
        {tc_conv_kernel<2, kNone, true, false, 16>, tc_conv_kernel<2, kRelu, true, false, 16>,
         tc_conv_kernel<2, -1, true, false, 16>}};
    static const Kern kerns_flat[3][3] = {
        {tc_conv_kernel<0, kNone, true>, tc_conv_kernel<0, kRelu, true>, tc_conv_kernel<0, -1, true>},
        {tc_conv_kernel<1, kNone, true>, tc_conv_kernel<1, kRelu, true>, tc_conv_kernel<1, -1, true>},
        {tc_conv_kernel<2, kNone, true>, tc_conv_kernel<2, kRelu, true>, tc_conv_kernel<2, -1, true>}};
    const int ak = c.act == kNone ? 0 : c.act == kRelu ? 1 : 2;
    if ((g.flat || !g.bias_smem) && kind == 3) {
        snprintf(err, errlen, "flat tiles and global-bias tiles take no exact-2x residual patches");
        return -2;
    }
    if (g.bk == 16 && (kind == 3 || !g.bias_smem)) {
        snprintf(err, errlen, "16-channel K blocks take no exact-2x residual patches nor global bias reads");
        return -2;
    }
    auto kern = g.bk == 16 ? (g.flat ? kerns_flat_k16[kind][ak] : kerns_k16[kind][ak])
                : g.flat   ? kerns_flat[kind][ak]
                : !g.bias_smem ? kerns_gbias[kind][ak]
                               : kerns[kind][ak];
    {
        cudaError_t e = ensure_smem_attr((const void *)kern, 227 * 1024);
        if (e != cudaSuccess) {
            snprintf(err, errlen, "tc_conv_kernel shared-memory attribute: %s", cudaGetErrorString(e));
            return -4;
        }
    }
    const unsigned grid = (unsigned)std::min<uint64_t>(g.units, (uint64_t)tc_sm_count());
    kern<<<grid, kTcThreads, g.smem_bytes, stream>>>(tmAp[0], tmB, a, tmAp[1], tmAp[2]);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(err, errlen, "tc_conv_kernel launch: %s", cudaGetErrorString(e));
        return -4;
    }
    return 0;
}

}  // namespace aie
