// C ABI of the B200 conv hot path (declared in include/aie_conv.h).
//
// Host side: descriptor validation, kernel/math choice (the Conv arm of
// ai-gpu-runtime's lower_op, crates/ai-gpu-runtime/src/lowering.rs:99-187),
// weight packing, and launch dispatch.  Device side: the kernels in the
// included .cuh files.  Built as one translation unit for sm_100a.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "../../include/aie_conv.h"
#include "common.cuh"
#include "k_simt.cuh"
#include "k_tc.cuh"
#include "k_stem_tc.cuh"
#include "k_pw_simt.cuh"
#include "k_mbconv.cuh"
#include "k_elem.cuh"

using namespace aie;

// ------------------------------------------------------------ errors ---

static thread_local char t_err[512];

static int fail(int status, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof t_err, fmt, ap);
    va_end(ap);
    return status;
}

static int cuda_fail(cudaError_t e, const char *what)
{
    return fail(AIE_E_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define CUDA_TRY(call)                                  \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

// -------------------------------------------------------------- plan ---

struct aie_plan {
    aie_conv_desc d;
    int kernel;
    int math;  // AIE_MATH_FFMA, AIE_MATH_TF32, or kMathStrict
    bool strict;
    uint32_t oh, ow;
    long long M;
    long long x_stride, y_stride, r_stride;
    int x_coff, y_coff, r_coff;
    int y_pad_to;
    int wn;            // FFMA GEMM weight row stride
    int cin_pad;       // TF32 weight K stride within a tap
    uint32_t split, tile_m, tile_n;
    uint64_t wbytes, bbytes, wsbytes;
    uint64_t flops, min_bytes, grid;
    TcGeom tc;         // tensor-core launch geometry (TF32 only)
    bool stem;         // small-cin direct conv, see stem_kernel / stem_tc_kernel
    bool stem_tc;      // ... on the tensor cores (TF32, cin <= 3, cout = 32)
    StemGeom sg;
    uint32_t stem_smem;
    bool pws;          // 1x1 on the FP32 pipes for cin, cout in {32, 64}, see pw_simt_kernel
    // concat parts read in place (aie_conv_plan_parts): 0 = a plain plan
    uint32_t nparts;
    uint32_t part_c[3], part_kb0[3];
    uint32_t part_bk;  // channels per K block of a parts plan: 16 when every part has <= 16, else 32
};

static const int kMathStrict = AIE_MATH_FP32_STRICT;


static inline uint32_t rup(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

extern "C" int32_t aie_abi_version(void) { return AIE_ABI_VERSION; }

extern "C" const char *aie_build_info(void)
{
    return "aie_conv abi 2 sm_100a (tcgen05 TF32 GEMM, FFMA implicit GEMM, depthwise); nvcc " __DATE__;
}

extern "C" const char *aie_status_string(int s)
{
    switch (s) {
    case AIE_OK: return "ok";
    case AIE_E_FAILURE: return "failure";
    case AIE_E_INVALID: return "invalid argument";
    case AIE_E_UNSUPPORTED: return "unsupported convolution";
    case AIE_E_CUDA: return "CUDA error";
    case AIE_E_ALIGN: return "alignment requirement not met";
    case AIE_E_DEVICE_TIMEOUT: return "device-side wait timed out";
    case AIE_E_NOMEM: return "out of host memory";
    default: return "unknown status";
    }
}

extern "C" int aie_last_error(char *buf, size_t len)
{
    size_t n = strlen(t_err);
    if (buf && len) {
        size_t c = n < len - 1 ? n : len - 1;
        memcpy(buf, t_err, c);
        buf[c] = 0;
    }
    return (int)n;
}

static bool tf32_eligible(const aie_plan &p, const char **why)
{
    const aie_conv_desc &d = p.d;
    if (!tc_available()) { *why = "tensor-core kernel not built"; return false; }
    if (d.groups != 1) { *why = "depthwise"; return false; }
    if (d.cin % 4 || p.x_stride % 4 || p.x_coff % 4) { *why = "input channels/stride not a multiple of 4"; return false; }
    if (d.kh != 1 || d.kw != 1 || d.sh != 1 || d.sw != 1 || d.pad[0] || d.pad[1] || d.pad[2] || d.pad[3]) {
        if (!tc_igemm_supported(d.kh, d.kw, d.sh, d.sw, p.ow)) { *why = "conv geometry"; return false; }
    }
    return true;
}

// 4-D tensor map (cin, iw, ih, n) of a depthwise input view with a box of
// (32 channels, hw, hh, 1) for dw_tile_kernel's TMA halo; false when the
// view is not TMA-compatible (the kernel then stages with cp.async).
static bool dw_tile_tmap(const ConvArgs &a, int hw, int hh, CUtensorMap *tm)
{
    memset(tm, 0, sizeof *tm);
    PFN_encodeTiled enc = tc_encoder();
    const uintptr_t base = (uintptr_t)(a.x + a.x_coff);
    if (!enc || base % 16 || (a.x_stride * 4) % 16) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)a.cin, (cuuint64_t)a.iw, (cuuint64_t)a.ih, (cuuint64_t)a.n};
    const cuuint64_t strides[3] = {(cuuint64_t)a.x_stride * 4, (cuuint64_t)a.x_stride * 4 * a.iw,
                                   (cuuint64_t)a.x_stride * 4 * a.iw * a.ih};
    const cuuint32_t box[4] = {32, (cuuint32_t)hw, (cuuint32_t)hh, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void *)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// pw_simt_kernel<CIN, COUT, RES>: a 2-D tensor map (cin, M) over the input
// view with [TP pixels][32 channels] boxes and 128-byte swizzle; false when
// the operands are not TMA- and float4-compatible (the FFMA implicit GEMM
// runs the conv instead).
template <int CIN, int COUT, int RES>
static bool pws_launch_t(const ConvArgs &a, cudaStream_t s)
{
    using S = PwsShape<CIN, COUT>;
    PFN_encodeTiled enc = tc_encoder();
    const uintptr_t base = (uintptr_t)(a.x + a.x_coff);
    if (!enc || base % 16 || (a.x_stride * 4) % 16) return false;
    CUtensorMap tm;
    memset(&tm, 0, sizeof tm);
    const cuuint64_t dims[2] = {(cuuint64_t)CIN, (cuuint64_t)a.M};
    const cuuint64_t strides[1] = {(cuuint64_t)a.x_stride * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)S::TP};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return false;
    if (ensure_smem_attr((const void *)pw_simt_kernel<CIN, COUT, RES>, (int)S::SMEM) != cudaSuccess) return false;
    PwsGeom g;
    g.tiles = (int)((a.M + S::TP - 1) / S::TP);
    const unsigned grid = (unsigned)std::min<long long>(g.tiles, 2ll * tc_sm_count());
    pw_simt_kernel<CIN, COUT, RES><<<grid, kPwsThreads, S::SMEM, s>>>(tm, a, g);
    return true;
}

static bool pws_launch(const aie_plan *p, const ConvArgs &a, cudaStream_t s)
{
    if (!a.vec_y || a.y_stride % 4 || a.y_coff % 4 || (a.res && (a.r_stride % 4 || a.r_coff % 4))) return false;
    const int res = !a.res ? 0 : !a.res_mode ? 1 : 2;
    const int cin = (int)p->d.cin, cout = (int)p->d.cout;
#define AIE_PWS(CI, CO)                                                      \
    if (cin == CI && cout == CO)                                             \
        return res == 0 ? pws_launch_t<CI, CO, 0>(a, s) : res == 1 ? pws_launch_t<CI, CO, 1>(a, s) \
                                                              : pws_launch_t<CI, CO, 2>(a, s);
    AIE_PWS(32, 32) AIE_PWS(32, 64) AIE_PWS(64, 32) AIE_PWS(64, 64)
#undef AIE_PWS
    return false;
}

// 4-D tensor map (c, w, h, n) of a dense source tensor for the up-sampled
// depthwise input, box (32 channels, hwq, hhq, 1)
static bool dw_up2_tmap(const void *q, uint32_t n, uint32_t h, uint32_t w, uint32_t c, int hwq, int hhq,
                        CUtensorMap *tm)
{
    memset(tm, 0, sizeof *tm);
    PFN_encodeTiled enc = tc_encoder();
    if (!enc || (uintptr_t)q % 16 || (c * 4) % 16) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)n};
    const cuuint64_t strides[3] = {(cuuint64_t)c * 4, (cuuint64_t)c * 4 * w, (cuuint64_t)c * 4 * w * h};
    const cuuint32_t box[4] = {32, (cuuint32_t)hwq, (cuuint32_t)hhq, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void *)q, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// nparts > 0: the input is the channel concat of nparts views of part_c[i]
// channels (aie_conv_plan_parts); the plan must resolve to the tensor cores.
static int plan_impl(const aie_conv_desc *desc, uint32_t nparts, const uint32_t *part_c, aie_plan **out)
{
    if (!desc || !out) return fail(AIE_E_INVALID, "null argument");
    *out = nullptr;
    const aie_conv_desc &d = *desc;
    if (!d.n || !d.ih || !d.iw || !d.cin || !d.cout || !d.kh || !d.kw || !d.sh || !d.sw || !d.dil || !d.groups)
        return fail(AIE_E_INVALID, "zero-sized dimension in descriptor");
    if (d.act < 0 || d.act > AIE_ACT_RECIP) return fail(AIE_E_INVALID, "activation %d out of range", d.act);
    if (d.layout != AIE_LAYOUT_NHWC && d.layout != AIE_LAYOUT_NHWC_C4)
        return fail(AIE_E_INVALID, "layout %d out of range", d.layout);
    if (d.math < AIE_MATH_AUTO || d.math > kMathStrict) return fail(AIE_E_INVALID, "math %d out of range", d.math);
    if (d.kh > 16 || d.kw > 16) return fail(AIE_E_UNSUPPORTED, "kernel larger than 16x16");
    if (d.res_mode < AIE_RES_TENSOR || d.res_mode > AIE_RES_BILINEAR_ASYMMETRIC)
        return fail(AIE_E_INVALID, "res_mode %d out of range", d.res_mode);
    if (d.res_mode != AIE_RES_TENSOR && (!d.has_res || !d.res_h || !d.res_w))
        return fail(AIE_E_INVALID, "a bilinear residual needs has_res and res_h/res_w");
    // Conv2d::out_hw (crates/ai-core/src/ops/conv.rs:49-55)
    const long long ekh = (long long)d.dil * (d.kh - 1) + 1, ekw = (long long)d.dil * (d.kw - 1) + 1;
    const long long hh = (long long)d.ih + d.pad[0] + d.pad[2] - ekh;
    const long long ww = (long long)d.iw + d.pad[1] + d.pad[3] - ekw;
    if (hh < 0 || ww < 0) return fail(AIE_E_INVALID, "kernel larger than padded input");

    // concat parts: each part starts on a K block; 16-channel blocks when
    // every part has at most 16 channels (two 16-channel parts then fill
    // one 32-channel block's MMAs instead of two half-padded blocks)
    uint32_t kblocks_parts = 0, part_kb0[3] = {0, 0, 0}, part_bk = kTcBK;
    if (nparts) {
        if (nparts > 3 || !part_c) return fail(AIE_E_INVALID, "1 to 3 concat parts, got %u", nparts);
        uint64_t sum = 0;
        part_bk = 16;
        for (uint32_t i = 0; i < nparts; i++)
            if (part_c[i] > 16) part_bk = kTcBK;
        for (uint32_t i = 0; i < nparts; i++) {
            if (!part_c[i]) return fail(AIE_E_INVALID, "concat part %u has no channels", i);
            part_kb0[i] = kblocks_parts;
            kblocks_parts += (part_c[i] + part_bk - 1) / part_bk;
            sum += part_c[i];
        }
        if (sum != d.cin) return fail(AIE_E_INVALID, "concat parts hold %llu channels, cin is %u",
                                       (unsigned long long)sum, d.cin);
        if (d.groups != 1 || d.layout != AIE_LAYOUT_NHWC || d.in_stride || d.in_coff ||
            (d.math != AIE_MATH_AUTO && d.math != AIE_MATH_TF32))
            return fail(AIE_E_UNSUPPORTED, "concat parts need a dense-layout, non-grouped conv on the tensor cores "
                                           "(math auto or tf32; each part's view is given at run time)");
    }
    aie_plan *p = new (std::nothrow) aie_plan();
    if (!p) return fail(AIE_E_NOMEM, "plan allocation");
    p->d = d;
    p->nparts = nparts;
    p->part_bk = part_bk;
    for (uint32_t i = 0; i < nparts; i++) {
        p->part_c[i] = part_c[i];
        p->part_kb0[i] = part_kb0[i];
    }
    p->oh = (uint32_t)(hh / d.sh + 1);
    p->ow = (uint32_t)(ww / d.sw + 1);
    p->M = (long long)d.n * p->oh * p->ow;
    if (p->M >= (1ll << 31) || (long long)d.n * d.ih * d.iw >= (1ll << 31)) {
        delete p;
        return fail(AIE_E_UNSUPPORTED, "more than 2^31 pixels in one call; split the batch");
    }
    const bool c4 = d.layout == AIE_LAYOUT_NHWC_C4;
    p->x_stride = d.in_stride ? d.in_stride : (c4 ? rup(d.cin, 4) : d.cin);
    p->x_coff = d.in_coff;
    p->y_stride = d.out_stride ? d.out_stride : (c4 ? rup(d.cout, 4) : d.cout);
    p->y_coff = d.out_coff;
    p->r_stride = d.res_stride ? d.res_stride : (c4 ? rup(d.cout, 4) : d.cout);
    p->r_coff = d.res_coff;
    p->y_pad_to = (c4 && !d.out_stride) ? (int)rup(d.cout, 4) : (int)d.cout;
    if (p->x_coff + (long long)d.cin > p->x_stride || p->y_coff + (long long)d.cout > p->y_stride ||
        (d.has_res && p->r_coff + (long long)d.cout > p->r_stride)) {
        delete p;
        return fail(AIE_E_INVALID, "channel view exceeds its pixel stride");
    }

    // Kernel family: lowering.rs:130-168 (dw / 1x1 GEMM / implicit GEMM).
    const uint32_t taps = d.kh * d.kw;
    if (d.groups > 1) {
        if (d.groups != d.cin || d.cin != d.cout) {
            delete p;
            return fail(AIE_E_UNSUPPORTED, "grouped conv g=%u cin=%u cout=%u", d.groups, d.cin, d.cout);
        }
        p->kernel = AIE_KERNEL_DW;
    } else if (d.kh == 1 && d.kw == 1 && d.sh == 1 && d.sw == 1 && !d.pad[0] && !d.pad[1] && !d.pad[2] &&
               !d.pad[3]) {
        // cout <= 4 without a residual takes the dot kernel, as ai-cpu's
        // PwDot arm does (crates/ai-cpu/src/plan.rs:546-566)
        p->kernel = (d.cout <= 4 && !d.has_res) ? AIE_KERNEL_PW_DOT : AIE_KERNEL_PW;
    } else {
        p->kernel = AIE_KERNEL_IGEMM;
    }

    if (d.res_mode != AIE_RES_TENSOR && p->kernel != AIE_KERNEL_PW && p->kernel != AIE_KERNEL_IGEMM) {
        delete p;
        return fail(AIE_E_UNSUPPORTED, "a bilinear residual is fused into the GEMM kernels only");
    }

    // Small-cin 3x3 convs (the stem) take a direct-conv kernel: the GEMM's
    // per-tap K tiles would be mostly padding (cin=3 -> 3 of 32 lanes).
    const bool stem_shape = p->kernel == AIE_KERNEL_IGEMM && d.res_mode == AIE_RES_TENSOR && d.cin <= 4 &&
                            d.kh == 3 && d.kw == 3 && d.dil == 1 && d.sh == d.sw && (d.sh == 1 || d.sh == 2) &&
                            d.cout % 4 == 0 && d.cout / 4 >= 1 && d.cout / 4 <= 32 && 32 % (d.cout / 4) == 0;
    // cin <= 3 (K = 27 fits one 32-wide K row), cout = 32, no residual: the
    // tensor-core variant, an im2col GEMM of K = 32
    const bool stem_tc_shape = stem_shape && d.cin <= 3 && d.cout == (uint32_t)kStemCout && !d.has_res;

    // 1x1 shapes of the FP32-pipe pointwise kernel (pw_simt_kernel):
    // residual tensor or exact-2x half_pixel sample, 32-bit pixel indices
    const bool up2_res = d.has_res && d.res_mode == AIE_RES_BILINEAR_HALF_PIXEL &&
                         p->oh == 2 * (uint64_t)d.res_h && p->ow == 2 * (uint64_t)d.res_w;
    const bool pws_shape = p->kernel == AIE_KERNEL_PW && (d.cin == 32 || d.cin == 64) &&
                           (d.cout == 32 || d.cout == 64) && (d.res_mode == AIE_RES_TENSOR || up2_res) &&
                           p->M < (1ll << 31);

    // Math.
    const char *why = "";
    if (nparts) {
        // parts are read by the tensor-core GEMM's TMA copies only
        if (p->kernel != AIE_KERNEL_PW && p->kernel != AIE_KERNEL_IGEMM) {
            delete p;
            return fail(AIE_E_UNSUPPORTED, "concat parts: 1x1 with cout <= 4 runs the dot kernel; concat first");
        }
        if (d.sh > 2 || d.sw > 2 || !tc_igemm_supported(d.kh, d.kw, d.sh, d.sw, p->ow)) {
            delete p;
            return fail(AIE_E_UNSUPPORTED, "concat parts: conv geometry outside the tensor-core kernel");
        }
        p->math = AIE_MATH_TF32;
    } else if (stem_tc_shape && (d.math == AIE_MATH_AUTO || d.math == AIE_MATH_TF32)) {
        p->math = AIE_MATH_TF32;
        p->stem_tc = true;
    } else if (p->kernel == AIE_KERNEL_DW || p->kernel == AIE_KERNEL_PW_DOT) {
        p->math = d.math == kMathStrict ? kMathStrict : AIE_MATH_FFMA;
        if (d.math == AIE_MATH_TF32) {
            delete p;
            return fail(AIE_E_UNSUPPORTED, "TF32 requested for a memory-bound kernel (depthwise / cout<=4)");
        }
    } else if (d.math == AIE_MATH_FFMA || d.math == kMathStrict) {
        p->math = d.math;
        p->pws = pws_shape && d.math == AIE_MATH_FFMA;
    } else if (d.math == AIE_MATH_AUTO && pws_shape && up2_res) {
        // an FPN lateral with its upsampled coarser level as the residual:
        // the FP32-pipe kernel reads the half-size tensor directly, where the
        // tensor-core GEMM's epilogue would be the bottleneck
        p->math = AIE_MATH_FFMA;
        p->pws = true;
    } else if (tf32_eligible(*p, &why)) {
        p->math = AIE_MATH_TF32;
    } else if (d.math == AIE_MATH_TF32) {
        delete p;
        return fail(AIE_E_UNSUPPORTED, "TF32 path needs TMA-compatible operands: %s", why);
    } else {
        p->math = AIE_MATH_FFMA;
    }
    p->strict = p->math == kMathStrict;

    // Packed sizes and launch geometry.
    const uint32_t cpad4 = rup(d.cout, 4);
    p->bbytes = (uint64_t)cpad4 * 4;
    p->split = 1;
    if (p->kernel == AIE_KERNEL_DW) {
        p->wbytes = (uint64_t)taps * cpad4 * 4;
        p->grid = (uint64_t)((p->M * (cpad4 / 4) + 255) / 256);
    } else if (p->kernel == AIE_KERNEL_PW_DOT) {
        p->wbytes = (uint64_t)d.cout * d.cin * 4;
        p->grid = (uint64_t)((p->M + 255) / 256);
    } else if (p->math == AIE_MATH_TF32 && !p->stem_tc) {
        // weights [tap][cout][cin_pad]; with parts every part's channels
        // start on a K block (zero weight rows between parts)
        p->cin_pad = nparts ? (int)(kblocks_parts * part_bk) : (int)rup(d.cin, 4);
        p->wbytes = (uint64_t)taps * d.cout * p->cin_pad * 4;
        // residual buffers: rows of a residual tensor, or per-warp patches
        // of an exact-2x half_pixel residual on 1x1 tiles (32 consecutive
        // output pixels within two rows: ow >= 32; whole float4 pieces)
        const bool pw_tile = d.kh == 1 && d.kw == 1 && d.sh == 1 && d.sw == 1;
        const bool up2 = d.res_mode == AIE_RES_BILINEAR_HALF_PIXEL && p->oh == 2 * (uint64_t)d.res_h &&
                         p->ow == 2 * (uint64_t)d.res_w;
        const uint32_t res_kind = !d.has_res ? kTcResNone
                                  : d.res_mode == AIE_RES_TENSOR ? kTcResTensor
                                  : (up2 && pw_tile && p->ow >= 32 && d.cout % 4 == 0 && p->r_stride % 4 == 0 &&
                                     p->r_coff % 4 == 0)
                                      ? kTcResUp2
                                      : kTcResNone;
        int rc = tc_plan(d.n, d.ih, d.iw, nparts ? (uint32_t)p->cin_pad : d.cin, d.cout, d.kh, d.kw, d.sh, d.sw,
                         d.dil, d.pad[0], d.pad[1], p->oh, p->ow, d.split_k, res_kind, &p->tc, true, true,
                         nparts ? part_bk : 0u);
        if (rc) {
            delete p;
            return fail(AIE_E_UNSUPPORTED, "tensor-core geometry rejected (%d)", rc);
        }
        p->split = p->tc.split;
        p->tile_m = p->tc.bm;
        p->tile_n = p->tc.bn;
        p->wsbytes = p->tc.workspace_bytes;
        p->grid = p->tc.grid;
    } else {
        p->wn = (int)cpad4;
        p->wbytes = (uint64_t)taps * d.cin * p->wn * 4;
        // (the tensor-core stem reads the same [tap][cin][wn] packing)
        if (stem_shape) {
            p->stem = true;
            StemGeom &g = p->sg;
            g.tile_h = 16;
            g.tile_w = 16;
            g.halo_h = (g.tile_h - 1) * d.sh + d.kh;
            g.halo_w = (g.tile_w - 1) * d.sw + d.kw;
            g.tiles_x = (p->ow + g.tile_w - 1) / g.tile_w;
            g.tiles_y = (p->oh + g.tile_h - 1) / g.tile_h;
            g.div_tpi = make_fastdiv(g.tiles_x * g.tiles_y);
            g.div_tx = make_fastdiv(g.tiles_x);
            p->stem_smem = (uint32_t)(g.halo_h * g.halo_w * d.cin * 4);
            p->tile_m = g.tile_h * g.tile_w;
            p->tile_n = d.cout;
            p->grid = (uint64_t)d.n * g.tiles_x * g.tiles_y;
        }
    }
    if (!p->stem && (p->kernel == AIE_KERNEL_IGEMM || p->kernel == AIE_KERNEL_PW) && p->math != AIE_MATH_TF32) {
        p->tile_m = kFfmaBM;
        p->tile_n = kFfmaBN;
        p->grid = (uint64_t)((p->M + kFfmaBM - 1) / kFfmaBM) * ((d.cout + kFfmaBN - 1) / kFfmaBN);
    }
    // Algorithmic work (ai-cpu prof_meta rule, crates/ai-cpu/src/model.rs:249-260):
    // border taps counted as full; bytes = input + weights + bias + output (+ res).
    const uint64_t cin_g = d.cin / d.groups;
    p->flops = 2ull * (uint64_t)p->M * d.cout * cin_g * taps;
    const uint64_t res_px = !d.has_res ? 0 : (d.res_mode ? (uint64_t)d.n * d.res_h * d.res_w : (uint64_t)p->M);
    p->min_bytes = 4ull * ((uint64_t)d.n * d.ih * d.iw * d.cin + (uint64_t)d.cout * cin_g * taps + d.cout +
                           (uint64_t)p->M * d.cout + res_px * d.cout);
    *out = p;
    return AIE_OK;
}

extern "C" int aie_conv_plan(const aie_conv_desc *desc, aie_plan **out) { return plan_impl(desc, 0, nullptr, out); }

extern "C" int aie_conv_plan_parts(const aie_conv_desc *desc, uint32_t nparts, const uint32_t *part_c, aie_plan **out)
{
    if (!nparts) return fail(AIE_E_INVALID, "1 to 3 concat parts, got 0");
    return plan_impl(desc, nparts, part_c, out);
}

extern "C" int aie_conv_plan_info(const aie_plan *p, aie_plan_info *info)
{
    if (!p || !info) return fail(AIE_E_INVALID, "null argument");
    memset(info, 0, sizeof *info);
    info->kernel = p->kernel;
    info->math = p->math;
    info->oh = p->oh;
    info->ow = p->ow;
    info->split_k = p->split;
    info->tile_m = p->tile_m;
    info->tile_n = p->tile_n;
    info->variant = p->stem_tc ? 2u : p->stem ? 1u : p->pws ? 3u : 0u;
    info->weight_bytes = p->wbytes;
    info->bias_bytes = p->bbytes;
    info->workspace_bytes = p->wsbytes;
    info->flops = p->flops;
    info->min_bytes = p->min_bytes;
    info->grid_ctas = p->grid;
    return AIE_OK;
}

extern "C" void aie_plan_free(aie_plan *p) { delete p; }

// ------------------------------------------------------- weight packing ---

// Unpack the .sw blob layouts (crates/ai-core/src/pack.rs:124-184) to OIHW.
static void unpack_sw(const aie_conv_desc &d, const float *src, std::vector<float> &oihw)
{
    const uint32_t taps = d.kh * d.kw;
    if (d.groups > 1) {
        // depthwise [tap][cg][4] (pack.rs:105-122, unpack_weights_dw :153-164)
        const uint32_t cg = (d.cout + 3) / 4;
        oihw.assign((size_t)d.cout * taps, 0.f);
        for (uint32_t ch = 0; ch < d.cout; ch++)
            for (uint32_t t = 0; t < taps; t++) oihw[(size_t)ch * taps + t] = src[((size_t)t * cg + ch / 4) * 4 + ch % 4];
    } else {
        // [tap][kg_pad][ng][4][4] with kg_pad = ceil(cin/4) rounded up to 4
        // (pack.rs:68-102 with kg_align = 4, as ai-convert lower.rs:151 uses)
        const uint32_t kg = rup((d.cin + 3) / 4, 4), ng = (d.cout + 3) / 4;
        oihw.assign((size_t)d.cout * d.cin * taps, 0.f);
        for (uint32_t t = 0; t < taps; t++)
            for (uint32_t oc = 0; oc < d.cout; oc++)
                for (uint32_t ic = 0; ic < d.cin; ic++)
                    oihw[((size_t)oc * d.cin + ic) * taps + t] =
                        src[((((size_t)t * kg + ic / 4) * ng + oc / 4) * 4 + oc % 4) * 4 + ic % 4];
    }
}

extern "C" int aie_conv_pack_weights(const aie_plan *p, int32_t wfmt, const float *w_host, const float *bias_host,
                                     void *dev_w, void *dev_b, void *stream)
{
    if (!p || !w_host || !dev_w || !dev_b) return fail(AIE_E_INVALID, "null argument");
    if (wfmt != AIE_WFMT_OIHW && wfmt != AIE_WFMT_SW_PACKED) return fail(AIE_E_INVALID, "weight format %d", wfmt);
    const aie_conv_desc &d = p->d;
    const uint32_t taps = d.kh * d.kw;
    const uint32_t cin_g = d.cin / d.groups;
    std::vector<float> tmp;
    const float *w = w_host;
    if (wfmt == AIE_WFMT_SW_PACKED) {
        unpack_sw(d, w_host, tmp);
        w = tmp.data();
    }
    std::vector<float> pw(p->wbytes / 4, 0.f), pb(p->bbytes / 4, 0.f);
    if (p->kernel == AIE_KERNEL_DW) {
        const uint32_t cpad = rup(d.cout, 4);  // [tap][c_pad4], dw.rs:22-34
        for (uint32_t ch = 0; ch < d.cout; ch++)
            for (uint32_t t = 0; t < taps; t++) pw[(size_t)t * cpad + ch] = w[(size_t)ch * taps + t];
    } else if (p->kernel == AIE_KERNEL_PW_DOT) {
        memcpy(pw.data(), w, (size_t)d.cout * d.cin * 4);  // [cout][cin]
    } else if (p->math == AIE_MATH_TF32 && !p->stem_tc) {
        // [tap][cout][cin_pad]: K-major rows for the tcgen05 B operand; with
        // concat parts, input channel ic of part i sits at K position
        // part_bk * part_kb0[i] + (ic - the part's first channel)
        std::vector<uint32_t> kpos(d.cin);
        for (uint32_t ic = 0, i = 0, c0 = 0; ic < d.cin; ic++) {
            if (p->nparts) {
                while (ic >= c0 + p->part_c[i]) c0 += p->part_c[i++];
                kpos[ic] = p->part_kb0[i] * p->part_bk + (ic - c0);
            } else {
                kpos[ic] = ic;
            }
        }
        for (uint32_t t = 0; t < taps; t++)
            for (uint32_t oc = 0; oc < d.cout; oc++)
                for (uint32_t ic = 0; ic < d.cin; ic++)
                    pw[((size_t)t * d.cout + oc) * p->cin_pad + kpos[ic]] = w[((size_t)oc * cin_g + ic) * taps + t];
    } else {
        // [tap][cin][wn] (conv.rs:44-66 with cout padded to 4)
        for (uint32_t t = 0; t < taps; t++)
            for (uint32_t ic = 0; ic < d.cin; ic++)
                for (uint32_t oc = 0; oc < d.cout; oc++)
                    pw[((size_t)t * d.cin + ic) * p->wn + oc] = w[((size_t)oc * cin_g + ic) * taps + t];
    }
    if (bias_host) {
        if (wfmt == AIE_WFMT_SW_PACKED) memcpy(pb.data(), bias_host, p->bbytes);  // [ng][4]
        else memcpy(pb.data(), bias_host, (size_t)d.cout * 4);
        for (uint32_t i = d.cout; i < pb.size(); i++) pb[i] = 0.f;
    }
    cudaStream_t s = (cudaStream_t)stream;
    CUDA_TRY(cudaMemcpyAsync(dev_w, pw.data(), p->wbytes, cudaMemcpyHostToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(dev_b, pb.data(), p->bbytes, cudaMemcpyHostToDevice, s));
    CUDA_TRY(cudaStreamSynchronize(s));  // the host staging vectors die here
    return AIE_OK;
}

// ---------------------------------------------------------------- run ---

static ConvArgs make_args(const aie_plan *p, const void *in, const void *w, const void *b, const void *res,
                          void *out)
{
    const aie_conv_desc &d = p->d;
    ConvArgs a;
    a.x = (const float *)in;
    a.w = (const float *)w;
    a.bias = (const float *)b;
    a.res = d.has_res ? (const float *)res : nullptr;
    a.y = (float *)out;
    a.n = d.n; a.ih = d.ih; a.iw = d.iw; a.cin = d.cin; a.oh = p->oh; a.ow = p->ow; a.cout = d.cout;
    a.kh = d.kh; a.kw = d.kw; a.sh = d.sh; a.sw = d.sw; a.dil = d.dil; a.pt = d.pad[0]; a.pl = d.pad[1];
    a.x_stride = p->x_stride; a.y_stride = p->y_stride; a.r_stride = p->r_stride;
    a.x_coff = p->x_coff; a.y_coff = p->y_coff; a.r_coff = p->r_coff;
    a.act = d.act;
    a.y_pad_to = p->y_pad_to;
    a.M = p->M;
    a.wn = p->wn;
    const uintptr_t xa = (uintptr_t)(a.x + a.x_coff), ya = (uintptr_t)(a.y + a.y_coff);
    const uintptr_t ra = a.res ? (uintptr_t)(a.res + a.r_coff) : 0;
    a.res_mode = d.res_mode;
    a.rh = d.res_mode ? (int)d.res_h : (int)p->oh;
    a.rw = d.res_mode ? (int)d.res_w : (int)p->ow;
    a.div_ow = make_fastdiv((int)p->ow);
    a.div_oh = make_fastdiv((int)p->oh);
    a.rsy = (float)a.rh / (float)p->oh;
    a.rsx = (float)a.rw / (float)p->ow;
    a.res_up2 = d.res_mode == AIE_RES_BILINEAR_HALF_PIXEL && p->oh == 2 * (uint64_t)a.rh && p->ow == 2 * (uint64_t)a.rw;
    a.vec_x = (d.cin % 4 == 0 || d.groups > 1) && a.x_stride % 4 == 0 && xa % 16 == 0;
    a.vec_y = a.y_stride % 4 == 0 && ya % 16 == 0 && (!a.res || (a.r_stride % 4 == 0 && ra % 16 == 0));
    return a;
}

extern "C" int aie_conv_run(const aie_plan *p, const void *in, const void *w, const void *b, const void *res,
                            void *out, void *workspace, void *stream)
{
    if (!p || !in || !w || !b || !out) return fail(AIE_E_INVALID, "null tensor pointer");
    if (p->d.has_res && !res) return fail(AIE_E_INVALID, "plan has a residual but res is NULL");
    if (p->wsbytes && !workspace) return fail(AIE_E_INVALID, "plan needs %llu workspace bytes",
                                              (unsigned long long)p->wsbytes);
    if (p->nparts) return fail(AIE_E_INVALID, "the plan reads concat parts: run it with aie_conv_run_parts");
    if (((uintptr_t)w | (uintptr_t)b) % 16) return fail(AIE_E_ALIGN, "weights/bias must be 16-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    const ConvArgs a = make_args(p, in, w, b, res, out);
    if (p->kernel == AIE_KERNEL_DW) {
        const aie_conv_desc &d = p->d;
        const bool blocked = d.cout % 4 == 0 && a.vec_x && a.vec_y && a.x_coff % 4 == 0 && a.y_coff % 4 == 0 &&
                             (!a.res || (a.r_stride % 4 == 0 && a.r_coff % 4 == 0)) &&
                             (d.dil == 1 || (d.dil == 2 && d.sh == 1)) &&
                             d.kh == d.kw && d.sh == d.sw && (d.kh == 3 || d.kh == 5) && (d.sh == 1 || d.sh == 2) &&
                             (long long)d.n * p->oh * ((p->ow + 3) / 4) * (d.cout / 4) + 256 < (1ll << 31);
        // Large frames take the shared-memory halo tiles (8 x 16 output
        // pixels at stride 1, else 8 x 8; one 32-channel slice per CTA);
        // small frames (the deep 10x18 / 20x36 layers) would waste most of a
        // tile and re-read wide halos, and keep the register-blocked kernel,
        // as do channel counts whose last 32-channel slice would be mostly
        // idle lanes (44 channels: 20 of 64 lanes idle; the blocked kernel
        // works in groups of four).
        const bool tiled = blocked && d.dil == 1 && p->oh >= 40 && p->ow >= 64 &&
                           (d.cout % 32 == 0 || d.cout % 32 > 24);
        if (tiled) {
            DwTile tg;
            const bool wide = d.sh == 1 && p->ow > 12;
            const int TW = wide ? 16 : 8;
            tg.tiles_x = (int)((p->ow + TW - 1) / TW);
            tg.tiles_y = (int)((p->oh + 7) / 8);
            tg.slices = (int)((d.cout + 31) / 32);
            tg.div_slices = make_fastdiv(tg.slices);
            tg.div_tx = make_fastdiv(tg.tiles_x);
            tg.div_ty = make_fastdiv(tg.tiles_y);
            const long long blocks = (long long)d.n * tg.tiles_y * tg.tiles_x * tg.slices;
            if (blocks >= (1ll << 31)) return fail(AIE_E_UNSUPPORTED, "depthwise grid too large; split the batch");
#define AIE_DWT(S_, K_, ST_, TW_)                                                                             \
    do {                                                                                                      \
        using G_ = DwTileGeom<K_, ST_, TW_>;                                                                  \
        auto k1_ = dw_tile_kernel<S_, K_, ST_, TW_, false, true>;                                             \
        auto k0_ = dw_tile_kernel<S_, K_, ST_, TW_, false, false>;                                            \
        CUDA_TRY(ensure_smem_attr((const void *)k1_, G_::SMEM));                                              \
        CUDA_TRY(ensure_smem_attr((const void *)k0_, G_::SMEM));                                              \
        CUtensorMap tm_;                                                                                      \
        const bool tma_ = dw_tile_tmap(a, G_::HW, G_::HH, &tm_);                                              \
        (tma_ ? k1_ : k0_)<<<(unsigned)blocks, G_::NT, G_::SMEM, s>>>(tm_, tm_, a, tg, PwHead{}, DwUp2{0, 0}); \
    } while (0)
#define AIE_DWT2(S_)                                                         \
    if (d.kh == 3 && d.sh == 1) { if (wide) AIE_DWT(S_, 3, 1, 16); else AIE_DWT(S_, 3, 1, 8); } \
    else if (d.kh == 3) AIE_DWT(S_, 3, 2, 8);                               \
    else if (d.sh == 1) { if (wide) AIE_DWT(S_, 5, 1, 16); else AIE_DWT(S_, 5, 1, 8); } \
    else AIE_DWT(S_, 5, 2, 8);
            if (p->strict) { AIE_DWT2(true) } else { AIE_DWT2(false) }
#undef AIE_DWT2
#undef AIE_DWT
        } else if (blocked) {
            // 4 output pixels per thread (8 measured slower on B200: fewer
            // threads in flight for the same bytes)
            constexpr int PB = 4;
            DwGrid gd;
            gd.segs_per_row = (int)((p->ow + PB - 1) / PB);
            gd.cg = (int)(d.cout / 4);
            gd.div_cg = make_fastdiv(gd.cg);
            gd.div_segs = make_fastdiv(gd.segs_per_row);
            gd.div_oh = make_fastdiv((int)p->oh);
            const long long threads = (long long)d.n * p->oh * gd.segs_per_row * gd.cg;
            const unsigned grid = (unsigned)((threads + 255) / 256);
#define AIE_DW(S_, K_, ST_) dw_block_kernel<S_, K_, ST_, PB><<<grid, 256, 0, s>>>(a, gd)
#define AIE_DW2(S_)                                                                        \
    if (d.dil == 2) {                                                                      \
        if (d.kh == 3) dw_block_kernel<S_, 3, 1, PB, 2><<<grid, 256, 0, s>>>(a, gd);     \
        else dw_block_kernel<S_, 5, 1, PB, 2><<<grid, 256, 0, s>>>(a, gd);               \
    }                                                                                      \
    else if (d.kh == 3 && d.sh == 1) AIE_DW(S_, 3, 1);                                     \
    else if (d.kh == 3) AIE_DW(S_, 3, 2);                                                  \
    else if (d.sh == 1) AIE_DW(S_, 5, 1);                                                  \
    else AIE_DW(S_, 5, 2);
            if (p->strict) { AIE_DW2(true) } else { AIE_DW2(false) }
#undef AIE_DW2
#undef AIE_DW
        } else if (p->strict) dw_kernel<true><<<(unsigned)p->grid, 256, 0, s>>>(a);
        else dw_kernel<false><<<(unsigned)p->grid, 256, 0, s>>>(a);
    } else if (p->kernel == AIE_KERNEL_PW_DOT && a.vec_x && a.x_coff % 4 == 0 &&
               (p->d.cin == 8 || p->d.cin == 16 || p->d.cin == 32 || p->d.cin == 64) && p->M + 256 < (1ll << 31)) {
        // coalesced tile form: weights + 8 warps x 32 staged input rows
        const int cin = (int)p->d.cin;
        const size_t smem = (size_t)cin * 4 * 4 + (size_t)8 * 32 * cin * 4;
        const unsigned grid = (unsigned)((p->M + 255) / 256);
#define AIE_PWD(S_, CG_)                                                                                     \
    do {                                                                                                     \
        CUDA_TRY(ensure_smem_attr((const void *)pw_dot_tile_kernel<S_, CG_>, (int)smem));                     \
        pw_dot_tile_kernel<S_, CG_><<<grid, 256, smem, s>>>(a);                                              \
    } while (0)
        if (p->strict) {
            if (cin == 8) AIE_PWD(true, 2); else if (cin == 16) AIE_PWD(true, 4);
            else if (cin == 32) AIE_PWD(true, 8); else AIE_PWD(true, 16);
        } else {
            if (cin == 8) AIE_PWD(false, 2); else if (cin == 16) AIE_PWD(false, 4);
            else if (cin == 32) AIE_PWD(false, 8); else AIE_PWD(false, 16);
        }
#undef AIE_PWD
    } else if (p->kernel == AIE_KERNEL_PW_DOT) {
        const size_t smem = (size_t)p->d.cout * p->d.cin * 4;
        if (smem > 200 * 1024) return fail(AIE_E_UNSUPPORTED, "cout*cin too large for the dot kernel");
        if (smem > 48 * 1024) {
            CUDA_TRY(cudaFuncSetAttribute(pw_dot_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            CUDA_TRY(cudaFuncSetAttribute(pw_dot_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        }
        if (p->strict) pw_dot_kernel<true><<<(unsigned)p->grid, 256, smem, s>>>(a);
        else pw_dot_kernel<false><<<(unsigned)p->grid, 256, smem, s>>>(a);
    } else if (p->stem_tc && a.vec_y) {
        int rc;
        const int cin = (int)p->d.cin;
        if (p->d.sh == 1) rc = cin == 1 ? stem_tc_launch<1, 1>(a, p->sg, s) : cin == 2 ? stem_tc_launch<2, 1>(a, p->sg, s)
                                                                                      : stem_tc_launch<3, 1>(a, p->sg, s);
        else rc = cin == 1 ? stem_tc_launch<1, 2>(a, p->sg, s) : cin == 2 ? stem_tc_launch<2, 2>(a, p->sg, s)
                                                                         : stem_tc_launch<3, 2>(a, p->sg, s);
        if (rc) return cuda_fail(cudaGetLastError(), "tensor-core stem setup");
    } else if (p->math == AIE_MATH_TF32 && !p->stem_tc) {
        int rc = tc_launch(p->tc, a, workspace, s, t_err, sizeof t_err);
        if (rc) return rc;
    } else if (p->stem && !p->stem_tc && a.vec_y && (a.y_stride % 4 == 0) && !(a.res && (a.r_stride % 4 || a.r_coff % 4)) &&
               ((uintptr_t)w % 16 == 0)) {
        const unsigned stem_grid = (unsigned)std::min<uint64_t>(p->grid, (uint64_t)tc_sm_count());
        const unsigned smem = 2 * p->stem_smem;
#define AIE_STEM(S, C, ST) stem_kernel<S, 3, 3, C, ST, 16, 16><<<stem_grid, 256, smem, s>>>(a, p->sg)
#define AIE_STEM2(S, ST)                                        \
    if (cin == 1) AIE_STEM(S, 1, ST);                           \
    else if (cin == 2) AIE_STEM(S, 2, ST);                      \
    else if (cin == 3) AIE_STEM(S, 3, ST);                      \
    else AIE_STEM(S, 4, ST);
        const int cin = (int)p->d.cin;
        if (p->strict) {
            if (p->d.sh == 1) { AIE_STEM2(true, 1) } else { AIE_STEM2(true, 2) }
        } else {
            if (p->d.sh == 1) { AIE_STEM2(false, 1) } else { AIE_STEM2(false, 2) }
        }
#undef AIE_STEM2
#undef AIE_STEM
    } else if (p->pws && pws_launch(p, a, s)) {
        // launched: the FP32-pipe 1x1 kernel
    } else {
        dim3 grid((unsigned)((p->M + kFfmaBM - 1) / kFfmaBM), (p->d.cout + kFfmaBN - 1) / kFfmaBN);
        if (grid.y > 65535) return fail(AIE_E_UNSUPPORTED, "cout too large");
        if (p->strict) igemm_ffma_kernel<true><<<grid, kFfmaThreads, 0, s>>>(a);
        else igemm_ffma_kernel<false><<<grid, kFfmaThreads, 0, s>>>(a);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    return AIE_OK;
}

// up != NULL: the depthwise input is in + up2(up), up a dense [n][up_h][up_w][C]
// tensor with ih = 2 up_h, iw = 2 up_w (exact-2x half_pixel resize)
static int run_dw_pw(const aie_plan *dw, const aie_plan *pw, const void *in, const void *up, uint32_t up_h,
                     uint32_t up_w, const void *dw_w, const void *dw_b, const void *pw_w, const void *pw_b, void *out,
                     void *stream)
{
    if (!dw || !pw || !in || !dw_w || !dw_b || !pw_w || !pw_b || !out) return fail(AIE_E_INVALID, "null argument");
    const aie_conv_desc &d = dw->d, &q = pw->d;
    if (dw->kernel != AIE_KERNEL_DW || dw->strict || d.has_res || d.dil != 1 || d.kh != d.kw || d.sh != d.sw ||
        (d.kh != 3 && d.kh != 5) || (d.sh != 1 && d.sh != 2) || d.cout % 4 || d.cout > 32)
        return fail(AIE_E_UNSUPPORTED, "fused head: depthwise plan must be k3/k5, s1/s2, dil 1, cout %% 4 == 0 and <= 32, "
                                       "no residual, not FP32_STRICT");
    if (pw->kernel != AIE_KERNEL_PW_DOT || pw->strict || q.has_res || q.cin != d.cout || q.n != d.n ||
        q.ih != dw->oh || q.iw != dw->ow)
        return fail(AIE_E_UNSUPPORTED, "fused head: the 1x1 plan must be a cout <= 4 dot over the depthwise output "
                                       "(no residual, not FP32_STRICT)");
    if (((uintptr_t)dw_w | (uintptr_t)dw_b | (uintptr_t)pw_w | (uintptr_t)pw_b) % 16)
        return fail(AIE_E_ALIGN, "weights/bias must be 16-byte aligned");
    ConvArgs a = make_args(dw, in, dw_w, dw_b, nullptr, out);
    if (!a.vec_x || a.x_coff % 4 || a.x_stride % 4)
        return fail(AIE_E_ALIGN, "fused head: input rows must be 16-byte aligned");
    PwHead hd;
    hd.w = (const float *)pw_w;
    hd.bias = (const float *)pw_b;
    hd.y = (float *)out;
    hd.y_stride = pw->y_stride;
    hd.y_coff = pw->y_coff;
    hd.cout = (int)q.cout;
    hd.act = q.act;
    hd.y_pad_to = pw->y_pad_to;
    DwTile tg;
    const bool wide = d.sh == 1 && dw->ow > 12;
    const int TW = wide ? 16 : 8;
    tg.tiles_x = (int)((dw->ow + TW - 1) / TW);
    tg.tiles_y = (int)((dw->oh + 7) / 8);
    tg.slices = 1;
    tg.div_slices = make_fastdiv(1);
    tg.div_tx = make_fastdiv(tg.tiles_x);
    tg.div_ty = make_fastdiv(tg.tiles_y);
    const long long blocks = (long long)d.n * tg.tiles_y * tg.tiles_x;
    if (blocks >= (1ll << 31)) return fail(AIE_E_UNSUPPORTED, "fused head grid too large; split the batch");
    cudaStream_t s = (cudaStream_t)stream;
    CUtensorMap tmq;
    memset(&tmq, 0, sizeof tmq);
    if (up) {
        if ((uintptr_t)up % 16) return fail(AIE_E_ALIGN, "up-sampled input: source must be 16-byte aligned");
        if (!up_h || !up_w || d.ih != 2 * up_h || d.iw != 2 * up_w)
            return fail(AIE_E_UNSUPPORTED, "up-sampled input: source %ux%u is not half of the depthwise input %ux%u",
                        up_h, up_w, d.ih, d.iw);
        if ((long long)d.n * up_h * up_w * d.cin >= (1ll << 31))
            return fail(AIE_E_UNSUPPORTED, "up-sampled input larger than 2^31 elements; split the batch");
    }
#define AIE_DWH(K_, ST_, TW_)                                                                                 \
    do {                                                                                                      \
        using G_ = DwTileGeom<K_, ST_, TW_>;                                                                  \
        CUtensorMap tm_;                                                                                      \
        const bool tma_ = dw_tile_tmap(a, G_::HW, G_::HH, &tm_);                                              \
        if (up && (!tma_ || !dw_up2_tmap(up, d.n, up_h, up_w, d.cin, G_::HWQ, G_::HHQ, &tmq)))               \
            return fail(AIE_E_UNSUPPORTED, "up-sampled input: operands are not TMA-compatible");              \
        if (up) {                                                                                             \
            /* one tile per CTA: four CTAs per SM overlap their staging */                                   \
            auto ku_ = dw_tile_up2_kernel<K_, ST_, TW_>;                                 \
            CUDA_TRY(ensure_smem_attr((const void *)ku_, G_::SMEM + G_::QSMEM));                              \
            ku_<<<(unsigned)blocks, G_::NT, G_::SMEM + G_::QSMEM, s>>>(tm_, tmq, a, tg, hd,                   \
                                                                      DwUp2{(int)up_h, (int)up_w});           \
        } else if (tma_) {                                                                                    \
            /* persistent CTAs with double-buffered staging */                                               \
            auto kp_ = dw_head_persistent_kernel<K_, ST_, TW_>;                                               \
            const int smem_ = 2 * G_::HH * G_::HW * 128 + 128;                                                \
            CUDA_TRY(ensure_smem_attr((const void *)kp_, smem_));                                             \
            int occ_ = 0;                                                                                     \
            CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_, kp_, G_::NT, smem_));               \
            const long long grid_ = std::min<long long>(blocks, (long long)std::max(occ_, 1) * tc_sm_count()); \
            kp_<<<(unsigned)grid_, G_::NT, smem_, s>>>(tm_, a, tg, hd, (int)blocks);                          \
        } else {                                                                                              \
            auto k0_ = dw_tile_kernel<false, K_, ST_, TW_, true, false>;                                      \
            CUDA_TRY(ensure_smem_attr((const void *)k0_, G_::SMEM));                                          \
            k0_<<<(unsigned)blocks, G_::NT, G_::SMEM, s>>>(tm_, tm_, a, tg, hd, DwUp2{0, 0});                  \
        }                                                                                                     \
    } while (0)
    if (d.kh == 3 && d.sh == 1) { if (wide) AIE_DWH(3, 1, 16); else AIE_DWH(3, 1, 8); }
    else if (d.kh == 3) AIE_DWH(3, 2, 8);
    else if (d.sh == 1) { if (wide) AIE_DWH(5, 1, 16); else AIE_DWH(5, 1, 8); }
    else AIE_DWH(5, 2, 8);
#undef AIE_DWH
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "fused head launch");
    return AIE_OK;
}

extern "C" int aie_conv_run_parts(const aie_plan *p, const aie_tview *parts, const void *w, const void *b,
                                  const void *res, void *out, void *workspace, void *stream)
{
    if (!p || !parts || !w || !b || !out) return fail(AIE_E_INVALID, "null argument");
    if (!p->nparts) return fail(AIE_E_INVALID, "the plan was made without concat parts: run it with aie_conv_run");
    if (p->d.has_res && !res) return fail(AIE_E_INVALID, "plan has a residual but res is NULL");
    if (p->wsbytes && !workspace) return fail(AIE_E_INVALID, "plan needs %llu workspace bytes",
                                              (unsigned long long)p->wsbytes);
    if (((uintptr_t)w | (uintptr_t)b) % 16) return fail(AIE_E_ALIGN, "weights/bias must be 16-byte aligned");
    TcParts tp;
    tp.n = (int)p->nparts;
    for (uint32_t i = 0; i < p->nparts; i++) {
        if (!parts[i].data) return fail(AIE_E_INVALID, "concat part %u: null data", i);
        const long long st = parts[i].stride ? parts[i].stride : p->part_c[i];
        if ((long long)parts[i].coff + p->part_c[i] > st)
            return fail(AIE_E_INVALID, "concat part %u: channel view exceeds its pixel stride", i);
        tp.x[i] = (const float *)parts[i].data;
        tp.stride[i] = st;
        tp.coff[i] = (int)parts[i].coff;
        tp.c[i] = p->part_c[i];
        tp.kb0[i] = p->part_kb0[i];
    }
    ConvArgs a = make_args(p, parts[0].data, w, b, res, out);
    a.x_stride = tp.stride[0];
    a.x_coff = tp.coff[0];
    int rc = tc_launch(p->tc, a, workspace, (cudaStream_t)stream, t_err, sizeof t_err, &tp);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core conv launch");
    return AIE_OK;
}

extern "C" int aie_conv_run_dw_pw(const aie_plan *dw, const aie_plan *pw, const void *in, const void *dw_w,
                                  const void *dw_b, const void *pw_w, const void *pw_b, void *out, void *stream)
{
    return run_dw_pw(dw, pw, in, nullptr, 0, 0, dw_w, dw_b, pw_w, pw_b, out, stream);
}

extern "C" int aie_conv_run_dw_pw_up2(const aie_plan *dw, const aie_plan *pw, const void *in, const void *up,
                                      uint32_t up_h, uint32_t up_w, const void *dw_w, const void *dw_b,
                                      const void *pw_w, const void *pw_b, void *out, void *stream)
{
    if (!up) return fail(AIE_E_INVALID, "null up-sampled source");
    return run_dw_pw(dw, pw, in, up, up_h, up_w, dw_w, dw_b, pw_w, pw_b, out, stream);
}

extern "C" int aie_conv_run_stem_pw(const aie_plan *stem, const aie_plan *pw, const void *in, const void *stem_w,
                                    const void *stem_b, const void *pw_w, const void *pw_b, void *stem_out,
                                    void *pw_out, void *stream)
{
    if (!stem || !pw || !in || !stem_w || !stem_b || !pw_w || !pw_b || !stem_out || !pw_out)
        return fail(AIE_E_INVALID, "null argument");
    const aie_conv_desc &d = stem->d, &q = pw->d;
    if (!stem->stem_tc)
        return fail(AIE_E_UNSUPPORTED, "stem + 1x1: the first plan must run as the tensor-core stem "
                                       "(3x3, cin <= 3, cout 32, no residual, math AUTO or TF32)");
    if (pw->kernel != AIE_KERNEL_PW || pw->math != AIE_MATH_TF32 || q.has_res || q.cin != (uint32_t)kStemCout ||
        q.cout > (uint32_t)kStemCout || q.cout % 4 || q.n != d.n || q.ih != stem->oh || q.iw != stem->ow ||
        q.layout != AIE_LAYOUT_NHWC || pw->x_stride != (long long)q.cin || pw->x_coff ||
        pw->y_stride != (long long)q.cout || pw->y_coff || pw->cin_pad != (int)kStemCout)
        return fail(AIE_E_UNSUPPORTED, "stem + 1x1: the second plan must be a dense TF32 1x1 over the stem's output, "
                                       "cin 32, cout <= 32 and a multiple of 4, no residual");
    if (((uintptr_t)stem_w | (uintptr_t)stem_b | (uintptr_t)pw_w | (uintptr_t)pw_b | (uintptr_t)pw_out) % 16)
        return fail(AIE_E_ALIGN, "weights, biases and the 1x1 output must be 16-byte aligned");
    const ConvArgs a = make_args(stem, in, stem_w, stem_b, nullptr, stem_out);
    if (!a.vec_y) return fail(AIE_E_ALIGN, "the stem output must be 16-byte aligned with a pixel stride of 4k floats");
    StemPw sp;
    sp.w = (const float *)pw_w;
    sp.bias = (const float *)pw_b;
    sp.y = (float *)pw_out;
    sp.cout = (int)q.cout;
    sp.act = q.act;
    cudaStream_t s = (cudaStream_t)stream;
    const int cin = (int)d.cin;
    int rc;
    if (d.sh == 1)
        rc = cin == 1 ? stem_tc_launch<1, 1, true>(a, stem->sg, s, sp)
             : cin == 2 ? stem_tc_launch<2, 1, true>(a, stem->sg, s, sp) : stem_tc_launch<3, 1, true>(a, stem->sg, s, sp);
    else
        rc = cin == 1 ? stem_tc_launch<1, 2, true>(a, stem->sg, s, sp)
             : cin == 2 ? stem_tc_launch<2, 2, true>(a, stem->sg, s, sp) : stem_tc_launch<3, 2, true>(a, stem->sg, s, sp);
    if (rc) return cuda_fail(cudaGetLastError(), "tensor-core stem setup");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "stem + 1x1 launch");
    return AIE_OK;
}

extern "C" int aie_conv_run_mbconv(const aie_plan *ex, const aie_plan *dw, const aie_plan *pj, const void *in,
                                   const void *ex_w, const void *ex_b, const void *dw_w, const void *dw_b,
                                   const void *pj_w, const void *pj_b, const void *res, void *out, void *stream)
{
    if (!ex || !pj || !in || !ex_w || !ex_b || !pj_w || !pj_b || !out || (dw && (!dw_w || !dw_b)))
        return fail(AIE_E_INVALID, "null argument");
    const aie_conv_desc &e = ex->d, &q = pj->d;
    auto dense = [](const aie_plan *p) {
        return p->d.layout == AIE_LAYOUT_NHWC && p->x_stride == (long long)p->d.cin && p->x_coff == 0 &&
               p->y_stride == (long long)p->d.cout && p->y_coff == 0;
    };
    if (ex->kernel != AIE_KERNEL_PW || ex->math != AIE_MATH_TF32 || e.has_res || !dense(ex) || e.cin % 32)
        return fail(AIE_E_UNSUPPORTED, "fused block: the expand plan must be a dense TF32 1x1 without residual, "
                                       "cin %% 32 == 0");
    if (dw) {
        const aie_conv_desc &d = dw->d;
        if (dw->kernel != AIE_KERNEL_DW || dw->strict || d.has_res || d.kh != 3 || d.kw != 3 || d.sh != 1 ||
            d.sw != 1 || d.dil != 1 || d.pad[0] != 1 || d.pad[1] != 1 || d.pad[2] != 1 || d.pad[3] != 1 ||
            d.cin != e.cout || d.n != e.n || d.ih != e.ih || d.iw != e.iw || !dense(dw))
            return fail(AIE_E_UNSUPPORTED, "fused block: the depthwise plan must be a dense 3x3, stride 1, pad 1 "
                                           "conv over the expand output, not FP32_STRICT");
    }
    if (pj->kernel != AIE_KERNEL_PW || pj->math != AIE_MATH_TF32 || q.cin != e.cout || q.cout > 128 || q.n != e.n ||
        q.ih != e.ih || q.iw != e.iw || !dense(pj) || (q.has_res && q.res_mode != AIE_RES_TENSOR) ||
        (q.has_res && (pj->r_stride != (long long)q.cout || pj->r_coff != 0)))
        return fail(AIE_E_UNSUPPORTED, "fused block: the project plan must be a dense TF32 1x1 over the depthwise "
                                       "output with cout <= 128");
    if (e.ih > (uint32_t)kMbRows || e.iw > (uint32_t)kMbRowStride)
        return fail(AIE_E_UNSUPPORTED, "fused block: frames up to %dx%d, got %ux%u", kMbRows, kMbRowStride, e.ih, e.iw);
    if (q.has_res != (res != nullptr)) return fail(AIE_E_INVALID, "residual pointer does not match the project plan");
    if (((uintptr_t)in | (uintptr_t)ex_w | (uintptr_t)ex_b | (uintptr_t)dw_w | (uintptr_t)dw_b | (uintptr_t)pj_w |
         (uintptr_t)pj_b | (uintptr_t)res | (uintptr_t)out) % 16)
        return fail(AIE_E_ALIGN, "fused block: tensors must be 16-byte aligned");
    PFN_encodeTiled enc = tc_encoder();
    if (!enc) return fail(AIE_E_UNSUPPORTED, "tensor-map encoder unavailable");
    CUtensorMap tmX, tmWe, tmWp;
    memset(&tmX, 0, sizeof tmX);
    memset(&tmWe, 0, sizeof tmWe);
    memset(&tmWp, 0, sizeof tmWp);
    const cuuint32_t e1[4] = {1, 1, 1, 1};
    {
        const cuuint64_t dims[4] = {e.cin, e.iw, e.ih, e.n};
        const cuuint64_t str[3] = {(cuuint64_t)e.cin * 4, (cuuint64_t)e.cin * 4 * e.iw, (cuuint64_t)e.cin * 4 * e.iw * e.ih};
        const cuuint32_t box[4] = {32, (cuuint32_t)kMbRowStride, (cuuint32_t)kMbRows, 1};
        if (enc(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void *)in, dims, str, box, e1, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return fail(AIE_E_UNSUPPORTED, "fused block: input tensor map rejected");
    }
    auto wmap = [&](CUtensorMap *tm, const void *w, uint32_t k, uint32_t rows) {
        const cuuint64_t dims[2] = {k, rows};
        const cuuint64_t str[1] = {(cuuint64_t)k * 4};
        const cuuint32_t box[2] = {32, (cuuint32_t)kMbChunk};
        return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)w, dims, str, box, e1, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    // TF32 packing: [tap = 1][cout][cin_pad4], K-major rows
    if (!wmap(&tmWe, ex_w, (uint32_t)ex->cin_pad, e.cout) || !wmap(&tmWp, pj_w, (uint32_t)pj->cin_pad, q.cout))
        return fail(AIE_E_UNSUPPORTED, "fused block: weight tensor map rejected");
    MbArgs a;
    a.x = (const float *)in;
    a.b_exp = (const float *)ex_b;
    a.w_dw = (const float *)dw_w;
    a.b_dw = (const float *)dw_b;
    a.b_proj = (const float *)pj_b;
    a.res = (const float *)res;
    a.y = (float *)out;
    a.n = (int)e.n; a.h = (int)e.ih; a.w = (int)e.iw;
    a.cin = (int)e.cin; a.cexp = (int)e.cout; a.cout = (int)q.cout; a.cexp_pad4 = (int)rup(e.cout, 4);
    a.act_exp = e.act; a.act_dw = dw ? dw->d.act : AIE_ACT_NONE; a.act_proj = q.act;
    cudaStream_t s = (cudaStream_t)stream;
    // compile-time activations for the usual ReLU / ReLU6 blocks
    const int ad = a.act_dw;
    auto kern = !dw ? (e.act == AIE_ACT_RELU ? mbconv_kernel<kRelu, -1, false> : mbconv_kernel<-1, -1, false>)
                : (e.act == AIE_ACT_RELU && ad == AIE_ACT_RELU)      ? mbconv_kernel<kRelu, kRelu>
                : (e.act == AIE_ACT_RELU6 && ad == AIE_ACT_RELU6) ? mbconv_kernel<kRelu6, kRelu6>
                                                                  : mbconv_kernel<-1, -1>;
    CUDA_TRY(ensure_smem_attr((const void *)kern, (int)kMbSmem));
    const unsigned grid = (unsigned)std::min<long long>(e.n, tc_sm_count());
    kern<<<grid, kMbThreads, kMbSmem, s>>>(tmX, tmWe, tmWp, a);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, "fused block launch");
    return AIE_OK;
}

extern "C" int aie_input_u8(uint32_t n, uint32_t h, uint32_t w, uint32_t cin, const void *in, int32_t layout,
                            void *out, void *stream)
{
    if (!in || !out) return fail(AIE_E_INVALID, "null tensor pointer");
    if (!n || !h || !w) return fail(AIE_E_INVALID, "zero-sized frame batch");
    if (cin != 3 && cin != 4) return fail(AIE_E_INVALID, "u8 frames must be RGB (3) or RGBA (4), got %u", cin);
    if (layout != AIE_LAYOUT_NHWC && layout != AIE_LAYOUT_NHWC_C4)
        return fail(AIE_E_INVALID, "layout %d out of range", layout);
    const int stride = layout == AIE_LAYOUT_NHWC_C4 ? 4 : 3;
    if (stride == 4 && (uintptr_t)out % 16) return fail(AIE_E_ALIGN, "C4 output must be 16-byte aligned");
    const long long npix = (long long)n * h * w;
    const long long threads = (npix + 3) / 4;
    if (threads >= (1ll << 31) * 256ll) return fail(AIE_E_UNSUPPORTED, "frame batch too large");
    input_u8_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint8_t *)in, (float *)out, npix, (int)cin, stride);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "input staging launch");
    return AIE_OK;
}

extern "C" int aie_input_yuv420(uint32_t n, uint32_t h, uint32_t w, const aie_yuv420 *src, int32_t layout,
                                void *out, void *stream)
{
    if (!src || !out || !src->y || !src->u || !src->v) return fail(AIE_E_INVALID, "null plane or output pointer");
    if (!n || !h || !w) return fail(AIE_E_INVALID, "zero-sized frame batch");
    if (layout != AIE_LAYOUT_NHWC && layout != AIE_LAYOUT_NHWC_C4)
        return fail(AIE_E_INVALID, "layout %d out of range", layout);
    if (src->uv_step != 1 && src->uv_step != 2)
        return fail(AIE_E_INVALID, "uv_step must be 1 (I420) or 2 (NV12 / NV21), got %u", src->uv_step);
    const uint64_t ch = (h + 1) / 2, cw = (w + 1) / 2;
    if (src->stride_y < w) return fail(AIE_E_INVALID, "stride_y %u < width %u", src->stride_y, w);
    const uint64_t cbytes = (cw - 1) * src->uv_step + 1;  // bytes a chroma row spans
    if (src->stride_u < cbytes || src->stride_v < cbytes)
        return fail(AIE_E_INVALID, "chroma strides (%u, %u) shorter than a chroma row (%llu bytes)", src->stride_u,
                    src->stride_v, (unsigned long long)cbytes);
    const uint64_t fy = src->frame_y ? src->frame_y : (uint64_t)src->stride_y * h;
    const uint64_t fu = src->frame_u ? src->frame_u : (uint64_t)src->stride_u * ch;
    const uint64_t fv = src->frame_v ? src->frame_v : (uint64_t)src->stride_v * ch;
    if (fy < (uint64_t)src->stride_y * (h - 1) + w || fu < (uint64_t)src->stride_u * (ch - 1) + cbytes ||
        fv < (uint64_t)src->stride_v * (ch - 1) + cbytes)
        return fail(AIE_E_INVALID, "frame strides shorter than a frame's planes");
    const int stride = layout == AIE_LAYOUT_NHWC_C4 ? 4 : 3;
    if (stride == 4 && (uintptr_t)out % 16) return fail(AIE_E_ALIGN, "C4 output must be 16-byte aligned");
    const uint64_t threads = (uint64_t)n * ch * cw;
    if (threads >= (1ull << 31) * 256ull || (uint64_t)n * h * w * stride >= (1ull << 62))
        return fail(AIE_E_UNSUPPORTED, "frame batch too large");
    Yuv420Args a;
    a.y = (const uint8_t *)src->y;
    a.u = (const uint8_t *)src->u;
    a.v = (const uint8_t *)src->v;
    a.fy = (long long)fy; a.fu = (long long)fu; a.fv = (long long)fv;
    a.sy = (int)src->stride_y; a.su = (int)src->stride_u; a.sv = (int)src->stride_v; a.uv_step = (int)src->uv_step;
    a.n = (int)n; a.h = (int)h; a.w = (int)w; a.ch = (int)ch; a.cw = (int)cw;
    a.out = (float *)out;
    a.ostride = stride;
    input_yuv420_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "YUV input staging launch");
    return AIE_OK;
}

extern "C" int aie_resize_bilinear(uint32_t n, uint32_t ih, uint32_t iw, uint32_t c, const void *in, uint32_t oh,
                                   uint32_t ow, int32_t mode, const void *add, int32_t act, void *out, void *stream)
{
    if (!in || !out) return fail(AIE_E_INVALID, "null tensor pointer");
    if (!n || !ih || !iw || !c || !oh || !ow) return fail(AIE_E_INVALID, "zero-sized resize");
    if (mode != 0 && mode != 1) return fail(AIE_E_INVALID, "resize mode %d", mode);
    if (act < 0 || act > AIE_ACT_RECIP) return fail(AIE_E_INVALID, "activation %d", act);
    if ((long long)n * oh * ow * ((c + 3) / 4) >= (1ll << 31) || (long long)n * ih * iw * c >= (1ll << 31))
        return fail(AIE_E_UNSUPPORTED, "resize larger than 2^31 elements; split the batch");
    ResizeArgs a;
    a.x = (const float *)in;
    a.add = (const float *)add;
    a.y = (float *)out;
    a.n = n; a.ih = ih; a.iw = iw; a.c = c; a.oh = oh; a.ow = ow; a.mode = mode; a.act = act;
    a.sy = (float)ih / (float)oh;
    a.sx = (float)iw / (float)ow;
    const int cg = (int)((c + 3) / 4);
    a.vec = c == 1 ? ((uintptr_t)out % 16 == 0 && ow % 4 == 0)
                   : ((c % 4 == 0) && (uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0 &&
                      (!add || (uintptr_t)add % 16 == 0));
    // exact 2x half_pixel upsampling: the source-pixel-per-thread kernel
    if (mode == 0 && oh == 2 * ih && ow == 2 * iw) {
        const bool c4 = c % 4 == 0 && a.vec;
        const bool c1 = c == 1 && iw % 4 == 0 && (uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0;
        const bool c2 = c == 2 && iw % 2 == 0 && (uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0;
        if (c2) {
            Up2Args u;
            u.x = (const float *)in;
            u.add = (const float *)add;
            u.y = (float *)out;
            u.n = n; u.ih = ih; u.iw = iw; u.c = c; u.act = act;
            u.div_g = make_fastdiv(1);
            u.div_w = make_fastdiv((int)(iw / 2));
            u.div_h = make_fastdiv((int)ih);
            const long long threads = (long long)n * ih * (iw / 2);
            if (threads + 256 < (1ll << 31)) {
                resize_up2_c2_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(u);
                cudaError_t e = cudaGetLastError();
                if (e != cudaSuccess) return cuda_fail(e, "resize launch");
                return AIE_OK;
            }
        }
        if (c4 || c1) {
            Up2Args u;
            u.x = (const float *)in;
            u.add = (const float *)add;
            u.y = (float *)out;
            u.n = n; u.ih = ih; u.iw = iw; u.c = c; u.act = act;
            const int G = c1 ? 1 : (int)(c / 4), Wt = c1 ? (int)(iw / 4) : (int)iw;
            u.div_g = make_fastdiv(G);
            u.div_w = make_fastdiv(Wt);
            u.div_h = make_fastdiv((int)ih);
            const long long threads = (long long)n * ih * Wt * G;
            if (threads + 256 < (1ll << 31)) {
                const unsigned grid = (unsigned)((threads + 255) / 256);
                if (c1) resize_up2_kernel<true><<<grid, 256, 0, (cudaStream_t)stream>>>(u);
                else resize_up2_kernel<false><<<grid, 256, 0, (cudaStream_t)stream>>>(u);
                cudaError_t e = cudaGetLastError();
                if (e != cudaSuccess) return cuda_fail(e, "resize launch");
                return AIE_OK;
            }
        }
    }
    a.px_per_thread = (c == 1 || (c % 4 == 0 && a.vec)) ? 4 : 1;
    a.div_cg = make_fastdiv(cg);
    a.div_owg = make_fastdiv((int)((ow + a.px_per_thread - 1) / a.px_per_thread));
    a.div_oh = make_fastdiv((int)oh);
    const long long groups = (long long)n * oh * ((ow + a.px_per_thread - 1) / a.px_per_thread) * cg;
    resize_bilinear_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "resize launch");
    return AIE_OK;
}

// ------------------------------------------------------- graph glue ---

// Resolves a channel view of c channels; stride 0 = dense.  Fails on a null
// pointer or a view whose channels run past its pixel stride.
static int make_eview(const aie_tview &v, uint32_t c, const char *what, EView *out)
{
    if (!v.data) return fail(AIE_E_INVALID, "%s: null tensor pointer", what);
    const uint32_t stride = v.stride ? v.stride : c;
    if ((uint64_t)v.coff + c > stride)
        return fail(AIE_E_INVALID, "%s: channels [%u, %u) exceed the pixel stride %u", what, v.coff, v.coff + c,
                    stride);
    out->p = (const float *)v.data;
    out->stride = stride;
    out->coff = (int)v.coff;
    return AIE_OK;
}

static bool eview_vec(const EView &v)
{
    return (uintptr_t)v.p % 16 == 0 && v.stride % 4 == 0 && v.coff % 4 == 0;
}

// Grid for a grid-stride loop over `work` items of 256 threads: enough CTAs
// to fill the SMs several times over, no more than the work needs.
static unsigned elem_grid(long long work)
{
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    const long long need = (work + 255) / 256;
    return (unsigned)std::max(1ll, std::min(need, (long long)sms * 16));
}

static int elem_sizes(uint32_t n, uint32_t px, uint32_t c, const char *what)
{
    if (!n || !px || !c) return fail(AIE_E_INVALID, "%s: zero-sized tensor (n %u, px %u, c %u)", what, n, px, c);
    return AIE_OK;
}

extern "C" int aie_binary(uint32_t n, uint32_t px, uint32_t c, aie_tview a, int32_t op, int32_t b_kind, aie_tview b,
                          float scalar, int32_t act, aie_tview out, void *stream)
{
    int s;
    if ((s = elem_sizes(n, px, c, "binary"))) return s;
    if (op < AIE_BIN_ADD || op > AIE_BIN_PRELU) return fail(AIE_E_INVALID, "binary op %d out of range", op);
    if (b_kind < AIE_OPND_TENSOR || b_kind > AIE_OPND_PVEC_TENSOR)
        return fail(AIE_E_INVALID, "binary operand kind %d out of range", b_kind);
    if (act < 0 || act > AIE_ACT_RECIP) return fail(AIE_E_INVALID, "activation %d out of range", act);
    BinArgs g{};
    EView y;
    if ((s = make_eview(a, c, "binary a", &g.a)) || (s = make_eview(out, c, "binary out", &y))) return s;
    if (b_kind == AIE_OPND_TENSOR) {
        if ((s = make_eview(b, c, "binary b", &g.b))) return s;
    } else if (b_kind != AIE_OPND_SCALAR && b_kind != AIE_OPND_SCALAR_FIRST) {
        if (!b.data) return fail(AIE_E_INVALID, "binary b: null vector pointer");
        g.b.p = (const float *)b.data;
    }
    g.y = (float *)y.p;
    g.y_stride = y.stride;
    g.y_coff = y.coff;
    g.Q = (long long)n * px;
    g.px = px;
    g.c = (int)c;
    g.groups = (int)((c + 3) / 4);
    g.op = op; g.bkind = b_kind; g.act = act; g.scalar = scalar;
    g.vec = c % 4 == 0 && eview_vec(g.a) && eview_vec(y) && (b_kind != AIE_OPND_TENSOR || eview_vec(g.b));
    binary_kernel<<<elem_grid(g.Q * g.groups), 256, 0, (cudaStream_t)stream>>>(g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "binary launch");
    return AIE_OK;
}

extern "C" int aie_mix(uint32_t n, uint32_t px, uint32_t c, aie_tview z, aie_tview a, aie_tview b, aie_tview out,
                       void *stream)
{
    int s;
    if ((s = elem_sizes(n, px, c, "mix"))) return s;
    MixArgs m{};
    EView y;
    if ((s = make_eview(z, c, "mix z", &m.z)) || (s = make_eview(a, c, "mix a", &m.a)) ||
        (s = make_eview(b, c, "mix b", &m.b)) || (s = make_eview(out, c, "mix out", &y)))
        return s;
    m.y = (float *)y.p;
    m.y_stride = y.stride;
    m.y_coff = y.coff;
    m.Q = (long long)n * px;
    m.c = (int)c;
    m.groups = (int)((c + 3) / 4);
    m.vec = c % 4 == 0 && eview_vec(m.z) && eview_vec(m.a) && eview_vec(m.b) && eview_vec(y);
    mix_kernel<<<elem_grid(m.Q * m.groups), 256, 0, (cudaStream_t)stream>>>(m);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "mix launch");
    return AIE_OK;
}

extern "C" int aie_gpool(uint32_t n, uint32_t px, uint32_t c, aie_tview in, void *out, void *stream)
{
    int s;
    if ((s = elem_sizes(n, px, c, "gpool"))) return s;
    if (!out) return fail(AIE_E_INVALID, "gpool out: null tensor pointer");
    GpoolArgs g{};
    if ((s = make_eview(in, c, "gpool in", &g.x))) return s;
    g.y = (float *)out;
    g.n = (int)n;
    g.c = (int)c;
    g.groups = (int)((c + 3) / 4);
    g.px = px;
    g.inv = 1.0f / (float)px;
    g.vec = c % 4 == 0 && eview_vec(g.x);
    const long long threads = (long long)n * g.groups;
    if (threads >= (1ll << 31)) return fail(AIE_E_UNSUPPORTED, "gpool: too many frames x channel groups");
    if (g.vec && n <= 65535u)
        gpool_staged_kernel<<<dim3((unsigned)((g.groups + kGpSlab - 1) / kGpSlab), n), 256, 0, (cudaStream_t)stream>>>(g);
    else
        gpool_kernel<<<(unsigned)((threads + 127) / 128), 128, 0, (cudaStream_t)stream>>>(g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gpool launch");
    return AIE_OK;
}

extern "C" int aie_avgpool(uint32_t n, uint32_t ih, uint32_t iw, uint32_t c, uint32_t kh, uint32_t kw, uint32_t sh,
                           uint32_t sw, const uint32_t pad[4], const void *in, void *out, void *stream)
{
    if (!in || !out || !pad) return fail(AIE_E_INVALID, "avgpool: null pointer");
    if (!n || !ih || !iw || !c || !kh || !kw || !sh || !sw) return fail(AIE_E_INVALID, "avgpool: zero size");
    const long long eh = (long long)ih + pad[0] + pad[2], ew = (long long)iw + pad[1] + pad[3];
    if (eh < kh || ew < kw) return fail(AIE_E_INVALID, "avgpool: window larger than the padded frame");
    AvgpoolArgs a{};
    a.x = (const float *)in;
    a.y = (float *)out;
    a.n = (int)n; a.ih = (int)ih; a.iw = (int)iw; a.c = (int)c;
    a.groups = (int)((c + 3) / 4);
    a.oh = (int)((eh - kh) / sh + 1);
    a.ow = (int)((ew - kw) / sw + 1);
    a.kh = (int)kh; a.kw = (int)kw; a.sh = (int)sh; a.sw = (int)sw;
    a.pt = (int)pad[0]; a.pl = (int)pad[1];
    a.inv = 1.0f / (float)(kh * kw);
    a.vec = c % 4 == 0 && (uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0;
    avgpool_kernel<<<elem_grid((long long)n * a.oh * a.ow * a.groups), 256, 0, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "avgpool launch");
    return AIE_OK;
}

extern "C" int aie_channel_copy(uint32_t n, uint32_t px, uint32_t c, aie_tview in, int32_t act, aie_tview out,
                                void *stream)
{
    int s;
    if ((s = elem_sizes(n, px, c, "channel copy"))) return s;
    if (act < 0 || act > AIE_ACT_RECIP) return fail(AIE_E_INVALID, "activation %d out of range", act);
    CopyArgs a{};
    EView y;
    if ((s = make_eview(in, c, "channel copy in", &a.x)) || (s = make_eview(out, c, "channel copy out", &y)))
        return s;
    a.y = (float *)y.p;
    a.y_stride = y.stride;
    a.y_coff = y.coff;
    a.Q = (long long)n * px;
    a.c = (int)c;
    a.groups = (int)((c + 3) / 4);
    a.act = act;
    a.vec = c % 4 == 0 && eview_vec(a.x) && eview_vec(y);
    chcopy_kernel<<<elem_grid(a.Q * a.groups), 256, 0, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "channel copy launch");
    return AIE_OK;
}

extern "C" int aie_concat(uint32_t n, uint32_t px, uint32_t nparts, const aie_tview *parts, const uint32_t *part_c,
                          uint32_t out_c, aie_tview out, void *stream)
{
    int s;
    if ((s = elem_sizes(n, px, out_c, "concat"))) return s;
    if (!parts || !part_c) return fail(AIE_E_INVALID, "concat: null part list");
    if (nparts < 1 || nparts > (uint32_t)kConcatMax)
        return fail(AIE_E_INVALID, "concat: %u parts (1..%d)", nparts, kConcatMax);
    ConcatArgs a{};
    uint64_t total = 0;
    for (uint32_t i = 0; i < nparts; i++) {
        if (!part_c[i]) return fail(AIE_E_INVALID, "concat: part %u has no channels", i);
        if ((s = make_eview(parts[i], part_c[i], "concat part", &a.part[i]))) return s;
        a.poff[i] = (int)total;
        total += part_c[i];
    }
    if (total > out_c) return fail(AIE_E_INVALID, "concat: parts hold %llu channels, out_c is %u",
                                   (unsigned long long)total, out_c);
    a.poff[nparts] = (int)total;
    a.nparts = (int)nparts;
    EView y;
    if ((s = make_eview(out, out_c, "concat out", &y))) return s;
    a.y = (float *)y.p;
    a.y_stride = y.stride;
    a.y_coff = y.coff;
    a.c_out = (int)out_c;
    a.groups = (int)((out_c + 3) / 4);
    if ((uint64_t)n * px * a.groups >= (1ull << 31)) return fail(AIE_E_UNSUPPORTED, "concat larger than 2^31 groups");
    a.Q = n * px;
    a.y_vec = out_c % 4 == 0 && eview_vec(y);
    concat_kernel<<<elem_grid((long long)a.Q * a.groups), 256, 0, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "concat launch");
    return AIE_OK;
}

extern "C" int aie_selftest_wait_timeout(uint32_t timeout_us, void *stream)
{
    if (timeout_us == 0 || timeout_us > 2000000) return fail(AIE_E_INVALID, "timeout must be 1..2000000 us");
    selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((unsigned long long)timeout_us * 1000ull);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
    return AIE_OK;
}

extern "C" int aie_device_status(void *stream, uint32_t *code_out)
{
    CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    uint32_t v = 0, zero = 0;
    CUDA_TRY(cudaMemcpyFromSymbol(&v, g_aie_error, sizeof v));
    if (v) CUDA_TRY(cudaMemcpyToSymbol(g_aie_error, &zero, sizeof zero));
    if (code_out) *code_out = v;
    if (v) return fail(AIE_E_DEVICE_TIMEOUT, "device wait gave up, code 0x%08x", v);
    return AIE_OK;
}

// ------------------------------------------------- no-allocation entry ---
//
// Some callers cannot allocate device memory once they are running: a
// real-time frame loop whose latency budget cannot absorb cudaMalloc's
// implicit device synchronisation, or a plugin inside a host application
// that owns the device allocator and hands over only its own tensors.  For
// them the split-K scratch comes from this fixed array inside the library
// instead of a caller workspace.
//
// The array lives in the memory of every GPU that loads this library, from
// module load until process exit.  All calls share it and it keeps the
// previous call's contents: the split-K tickets are cleared on the stream
// before every launch and the partials are written before they are read,
// so no state leaks between calls -- but two calls that overlap on the GPU
// (e.g. on different streams) race on it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[AIE_NOALLOC_SCRATCH_BYTES];

typedef CUresult (*PFN_ctxGetCurrent)(CUcontext *);

static std::mutex g_noalloc_mu;
// The array's device address per device ordinal, with the context it was
// looked up in: after cudaDeviceReset (or under another context on the same
// ordinal) the address is looked up again instead of reused.
static void *g_noalloc_addr[64];
static CUcontext g_noalloc_ctx[64];

extern "C" int aie_conv_run_noalloc(const aie_plan *p, const void *in, const void *w, const void *b,
                                    const void *res, void *out, void *stream)
{
    if (!p) return fail(AIE_E_INVALID, "null plan");
    if (p->wsbytes > AIE_NOALLOC_SCRATCH_BYTES)
        return fail(AIE_E_UNSUPPORTED,
                    "plan needs %llu bytes of split-K scratch but the built-in scratch holds %u; "
                    "use aie_conv_run with a workspace, or plan with a smaller split_k",
                    (unsigned long long)p->wsbytes, (unsigned)AIE_NOALLOC_SCRATCH_BYTES);
    void *ws = nullptr;
    if (p->wsbytes) {
        int dev = -1;
        CUDA_TRY(cudaGetDevice(&dev));
        if (dev < 0 || dev >= 64) return fail(AIE_E_UNSUPPORTED, "device ordinal %d out of range", dev);
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        static PFN_ctxGetCurrent ctx_current = nullptr;
        if (!ctx_current) {
            void *fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
                q != cudaDriverEntryPointSuccess || !fn)
                return fail(AIE_E_CUDA, "cuCtxGetCurrent unavailable");
            ctx_current = (PFN_ctxGetCurrent)fn;
        }
        CUcontext ctx = nullptr;
        if (ctx_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
        if (!ctx || !g_noalloc_addr[dev] || g_noalloc_ctx[dev] != ctx) {
            // first call on this device (which is current) or in this context:
            // the array's name is only a host-side stand-in for it; ask the
            // runtime for its device address
            void *addr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
            // the lookup made the runtime's context current if none was
            if (!ctx && (ctx_current(&ctx) != CUDA_SUCCESS || !ctx))
                return fail(AIE_E_CUDA, "no current CUDA context");
            g_noalloc_addr[dev] = addr;
            g_noalloc_ctx[dev] = ctx;
        }
        ws = g_noalloc_addr[dev];
    }
    return aie_conv_run(p, in, w, b, res, out, ws, stream);
}
