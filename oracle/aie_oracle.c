/*
 * aie_oracle.c -- CPU restatement of ai_engine's convolution path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the timed
 * CPU baseline; it is never linked into, called by, or used as a fallback
 * for the CUDA library in ai_engine_b200/.  Only tests/, the smoke check in
 * __graft_entry__.py and bench.py's CPU-baseline leg load it.
 *
 * What it restates (paths relative to the ai_engine project root):
 *   - XorShift32 seeded generator            crates/ai-core/src/rng.rs:3-27
 *   - Activation::apply (scalar)             crates/ai-core/src/activation.rs:28-43
 *   - apply4 (4-lane epilogue activation)    crates/ai-cpu/src/kernels/mod.rs:21-50
 *   - naive conv2d (semantic reference)      crates/ai-core/src/reference/conv.rs:9-62
 *   - conv_std broadcast GEMM (MR x NR=8)    crates/ai-cpu/src/kernels/conv.rs:81-468
 *   - conv_dw                                crates/ai-cpu/src/kernels/dw.rs:40-272
 *   - conv_pw_dot (cout <= 4 head)           crates/ai-cpu/src/kernels/pw_dot.rs:32-61
 *   - im2row stem                            crates/ai-cpu/src/kernels/im2row.rs:22-102
 *   - kernel choice at load time             crates/ai-cpu/src/plan.rs:462-619
 *   - bilinear resize                        crates/ai-core/src/reference/resize.rs:5-42
 *   - binary add                             crates/ai-cpu/src/kernels/elementwise.rs:30-55
 *   - Binary (tensor/scalar/cvec/pvec), Mix, crates/ai-cpu/src/kernels/elementwise.rs,
 *     Act, Concat/Chcopy copies              crates/ai-core/src/reference/elementwise.rs:7-26
 *   - Gpool, Avgpool                         crates/ai-cpu/src/kernels/segate.rs:46-57,
 *                                            crates/ai-core/src/reference/pool.rs:5-46
 *   - I420 <-> RGBA8 frame conversion        crates/ai-ffi/src/yuv.rs:7-58
 *     (BT.601 full range)
 *
 * Rounding.  ai-cpu on x86 runs its scalar F32x4 fallback
 * (crates/ai-cpu/src/simd.rs:189-300): `fma` is a separate multiply then add,
 * and `sum` is (l0+l1)+(l2+l3).  This file is compiled with
 * -ffp-contract=off so gcc never fuses a multiply-add, which reproduces
 * that rounding.  Every output accumulates in the reference's order:
 * start from the bias, then valid taps in (ky, kx) order, then input
 * channels in ascending order.  The only departure: lanes that ai-cpu reads
 * past a pixel's last channel (zero-weight padding of the K axis) are
 * skipped here instead of being multiplied by a zero weight; the sum is
 * identical except possibly for the sign of an exact zero.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

enum {
    ACT_NONE = 0, ACT_RELU, ACT_SIGMOID, ACT_TANH, ACT_HARDSWISH, ACT_HARDSIGMOID,
    ACT_CLAMP01, ACT_RELU6, ACT_SQRT, ACT_NEG, ACT_RECIP, ACT_COUNT
};

typedef struct {
    uint32_t cin, cout, kh, kw, sh, sw;
    uint32_t pad[4]; /* top, left, bottom, right */
    uint32_t dil, groups;
    int32_t act;
} orc_conv;

/* channel-strided view of an NHWC tensor (crates/ai-cpu/src/view.rs:8-27) */
typedef struct {
    const float *data;
    size_t c_off;
    size_t stride;
    size_t c;
} orc_view;

static inline size_t vbase(const orc_view *v, size_t lin_px) { return lin_px * v->stride + v->c_off; }

/* ---------------------------------------------------------------- rng --- */

ORC_API uint32_t orc_xorshift32_next(uint32_t *state)
{
    uint32_t x = *state;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *state = x;
    return x;
}

ORC_API uint32_t orc_xorshift32_seed(uint32_t seed) { return seed == 0 ? 0x9e3779b9u : seed; }

/* next_f32: top 24 bits -> [0,1) -> [-1,1) (rng.rs:21-24) */
ORC_API void orc_fill_uniform(uint32_t *state, float *out, size_t n)
{
    const float inv = 1.0f / (float)(1u << 24);
    for (size_t i = 0; i < n; i++) {
        uint32_t u = orc_xorshift32_next(state) >> 8;
        out[i] = (float)u * inv * 2.0f - 1.0f;
    }
}

/* --------------------------------------------------------- activation --- */

static inline float clampf(float x, float lo, float hi)
{
    /* Rust f32::clamp: NaN passes through */
    if (x < lo) return lo;
    if (x > hi) return hi;
    return x;
}

/* Activation::apply (activation.rs:28-43) */
ORC_API float orc_act_apply(int act, float x)
{
    switch (act) {
    case ACT_NONE: return x;
    case ACT_RELU: return fmaxf(x, 0.0f);
    case ACT_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case ACT_TANH: return tanhf(x);
    case ACT_HARDSWISH: return x * clampf(x / 6.0f + 0.5f, 0.0f, 1.0f);
    case ACT_HARDSIGMOID: return clampf(x / 6.0f + 0.5f, 0.0f, 1.0f);
    case ACT_CLAMP01: return clampf(x, 0.0f, 1.0f);
    case ACT_RELU6: return clampf(x, 0.0f, 6.0f);
    case ACT_SQRT: return sqrtf(fmaxf(x, 0.0f));
    case ACT_NEG: return -x;
    case ACT_RECIP: return 1.0f / x;
    default: return x;
    }
}

/* one lane of apply4 (kernels/mod.rs:21-50): hard activations multiply by
 * the f32 constant 1/6 instead of dividing by 6, and use max-then-min. */
ORC_API float orc_act_apply4_lane(int act, float x)
{
    const float sixth = 1.0f / 6.0f;
    switch (act) {
    case ACT_NONE: return x;
    case ACT_RELU: return fmaxf(x, 0.0f);
    case ACT_HARDSWISH: return x * fminf(fmaxf(x * sixth + 0.5f, 0.0f), 1.0f);
    case ACT_HARDSIGMOID: return fminf(fmaxf(x * sixth + 0.5f, 0.0f), 1.0f);
    case ACT_CLAMP01: return fminf(fmaxf(x, 0.0f), 1.0f);
    case ACT_RELU6: return fminf(fmaxf(x, 0.0f), 6.0f);
    case ACT_NEG: return x * -1.0f;
    default: return orc_act_apply(act, x); /* sqrt/recip/sigmoid/tanh: scalar */
    }
}

/* ai-cpu epilogues apply the 4-lane form to channels below 4*floor(c/4) and
 * the scalar form to the tail (conv.rs:190-235, dw.rs:147-171). */
static inline float epi_act(int act, float v, size_t ch, size_t c)
{
    return ch < (c / 4) * 4 ? orc_act_apply4_lane(act, v) : orc_act_apply(act, v);
}

/* -------------------------------------------------------------- shape --- */

/* Conv2d::out_hw (ops/conv.rs:49-55) */
ORC_API int orc_out_hw(const orc_conv *op, uint32_t ih, uint32_t iw, uint32_t *oh, uint32_t *ow)
{
    int64_t ekh = (int64_t)op->dil * (op->kh - 1) + 1;
    int64_t ekw = (int64_t)op->dil * (op->kw - 1) + 1;
    int64_t h = (int64_t)ih + op->pad[0] + op->pad[2] - ekh;
    int64_t w = (int64_t)iw + op->pad[1] + op->pad[3] - ekw;
    if (h < 0 || w < 0 || op->sh == 0 || op->sw == 0) return -1;
    *oh = (uint32_t)(h / op->sh + 1);
    *ow = (uint32_t)(w / op->sw + 1);
    return 0;
}

/* ----------------------------------------------- naive reference conv --- */

/* reference::conv::conv2d (reference/conv.rs:9-62), one frame, dense NHWC,
 * OIHW weights.  bias / residual may be NULL. */
ORC_API int orc_conv2d_ref(const orc_conv *op, uint32_t ih, uint32_t iw, const float *input,
                           const float *weights, const float *bias, const float *residual,
                           float *out)
{
    uint32_t oh, ow;
    if (orc_out_hw(op, ih, iw, &oh, &ow)) return -1;
    if (op->groups == 0 || op->cin % op->groups || op->cout % op->groups) return -1;
    const uint32_t cin_g = op->cin / op->groups, cout_g = op->cout / op->groups;
    for (uint32_t oy = 0; oy < oh; oy++)
        for (uint32_t ox = 0; ox < ow; ox++)
            for (uint32_t oc = 0; oc < op->cout; oc++) {
                uint32_t g = oc / cout_g;
                float acc = bias ? bias[oc] : 0.0f;
                for (uint32_t ky = 0; ky < op->kh; ky++)
                    for (uint32_t kx = 0; kx < op->kw; kx++) {
                        int64_t iy = (int64_t)oy * op->sh + (int64_t)ky * op->dil - op->pad[0];
                        int64_t ix = (int64_t)ox * op->sw + (int64_t)kx * op->dil - op->pad[1];
                        if (iy < 0 || iy >= ih || ix < 0 || ix >= iw) continue;
                        for (uint32_t icg = 0; icg < cin_g; icg++) {
                            uint32_t ic = g * cin_g + icg;
                            float iv = input[((size_t)iy * iw + ix) * op->cin + ic];
                            float wv = weights[(((size_t)oc * cin_g + icg) * op->kh + ky) * op->kw + kx];
                            acc += iv * wv;
                        }
                    }
                size_t idx = ((size_t)oy * ow + ox) * op->cout + oc;
                float v = orc_act_apply(op->act, acc);
                if (residual) v += residual[idx];
                out[idx] = v;
            }
    return 0;
}

/* ------------------------------------------------ ai-cpu: conv_std --- */

#define NR 8

/* valid tap rows of output row oy: (tap row start, iy) */
static size_t ky_list(const orc_conv *op, uint32_t ih, size_t oy, size_t *t_row, size_t *iys)
{
    size_t n = 0;
    for (int64_t ky = 0; ky < op->kh; ky++) {
        int64_t iy = (int64_t)oy * op->sh + ky * op->dil - op->pad[0];
        if (iy >= 0 && iy < ih) {
            t_row[n] = (size_t)(ky * op->kw);
            iys[n] = (size_t)iy;
            n++;
        }
    }
    return n;
}

static inline int64_t div_euclid(int64_t a, int64_t b)
{
    int64_t q = a / b;
    if (a % b < 0) q -= 1;
    return q;
}

/* interior ox range [lo, hi] where every kx tap is inside (conv.rs:110-120) */
static void interior_range(const orc_conv *op, uint32_t iw, uint32_t ow, int64_t *lo_o, int64_t *hi_o)
{
    int64_t lo = 0, hi = (int64_t)ow - 1;
    int64_t sw = op->sw, dil = op->dil, pl = op->pad[1];
    for (int64_t kx = 0; kx < op->kw; kx++) {
        int64_t off = kx * dil - pl;
        int64_t mn = div_euclid(-off + sw - 1, sw);
        if (mn < 0) mn = 0;
        int64_t mx = div_euclid((int64_t)iw - 1 - off, sw);
        if (mn > lo) lo = mn;
        if (mx < hi) hi = mx;
    }
    *lo_o = lo;
    *hi_o = hi;
}

typedef struct {
    const orc_conv *op;
    uint32_t ih, iw, ow;
    orc_view x;
    size_t c4; /* weight K stride of the single part (>= x.c) */
    const float *wts;  /* [tap][c4][cout_pad] */
    const float *bias; /* [cout_pad] */
    size_t cout_pad;
    const orc_view *res;
    float *out; /* band slice starting at pixel px_base */
    size_t px_base;
    size_t cout;
} std_ctx;

static void std_store(const std_ctx *s, const float *acc, size_t px, size_t oc0)
{
    size_t o = (px - s->px_base) * s->cout + oc0;
    size_t nc = s->cout - oc0 < NR ? s->cout - oc0 : NR;
    for (size_t l = 0; l < nc; l++) {
        float v = epi_act(s->op->act, acc[l], oc0 + l, s->cout);
        if (s->res) v += s->res->data[vbase(s->res, px) + oc0 + l];
        s->out[o + l] = v;
    }
}

/* MR interior pixels x NR output channels (conv.rs:238-334). */
static void std_mr(const std_ctx *s, int MR, const size_t *t_rows, const size_t *iys, size_t nky,
                   size_t oy, size_t ox, size_t oc0)
{
    float acc[8][NR];
    for (int p = 0; p < MR; p++)
        for (int l = 0; l < NR; l++) acc[p][l] = s->bias[oc0 + l];
    const size_t sw = s->op->sw, dil = s->op->dil, pl = s->op->pad[1], kw = s->op->kw;
    const size_t pc = s->x.c;
    for (size_t r = 0; r < nky; r++) {
        for (size_t kx = 0; kx < kw; kx++) {
            size_t t = t_rows[r] + kx;
            size_t ix0 = ox * sw + kx * dil - pl;
            size_t row = iys[r] * s->iw;
            size_t base[8];
            for (int p = 0; p < MR; p++) base[p] = vbase(&s->x, row + ix0 + p * sw);
            const float *w = s->wts + t * s->c4 * s->cout_pad + oc0;
            for (size_t ic = 0; ic < pc; ic++) {
                const float *wr = w + ic * s->cout_pad;
                for (int p = 0; p < MR; p++) {
                    const float a = s->x.data[base[p] + ic];
                    for (int l = 0; l < NR; l++) acc[p][l] = acc[p][l] + a * wr[l];
                }
            }
        }
    }
    for (int p = 0; p < MR; p++) std_store(s, acc[p], oy * s->ow + ox + p, oc0);
}

/* one edge pixel, per-kx bounds check (conv.rs:405-468) */
static void std_mr1(const std_ctx *s, const size_t *t_rows, const size_t *iys, size_t nky, size_t oy,
                    size_t ox, size_t oc0)
{
    float acc[NR];
    for (int l = 0; l < NR; l++) acc[l] = s->bias[oc0 + l];
    const int64_t sw = s->op->sw, dil = s->op->dil, pl = s->op->pad[1];
    const size_t pc = s->x.c;
    for (size_t r = 0; r < nky; r++) {
        for (size_t kx = 0; kx < s->op->kw; kx++) {
            int64_t ix = (int64_t)ox * sw + (int64_t)kx * dil - pl;
            if (ix < 0 || ix >= s->iw) continue;
            size_t t = t_rows[r] + kx;
            size_t base = vbase(&s->x, iys[r] * s->iw + (size_t)ix);
            const float *w = s->wts + t * s->c4 * s->cout_pad + oc0;
            for (size_t ic = 0; ic < pc; ic++) {
                const float a = s->x.data[base + ic];
                const float *wr = w + ic * s->cout_pad;
                for (int l = 0; l < NR; l++) acc[l] = acc[l] + a * wr[l];
            }
        }
    }
    std_store(s, acc, oy * s->ow + ox, oc0);
}

/* conv_std over output rows [y0, y1) (conv.rs:81-185) */
static void conv_std_rows(const std_ctx *s, uint32_t y0, uint32_t y1)
{
    int64_t lo, hi;
    interior_range(s->op, s->iw, s->ow, &lo, &hi);
    size_t t_rows[16], iys[16];
    for (size_t oy = y0; oy < y1; oy++) {
        size_t nky = ky_list(s->op, s->ih, oy, t_rows, iys);
        for (size_t oc0 = 0; oc0 < s->cout; oc0 += NR) {
            size_t ox = 0;
            while (ox < s->ow) {
#define INB(n) ((int64_t)ox >= lo && (int64_t)(ox + (n) - 1) <= hi && ox + (n) <= s->ow)
                if (INB(8)) {
                    std_mr(s, 8, t_rows, iys, nky, oy, ox, oc0);
                    ox += 8;
                } else if (INB(4)) {
                    std_mr(s, 4, t_rows, iys, nky, oy, ox, oc0);
                    ox += 4;
                } else {
                    std_mr1(s, t_rows, iys, nky, oy, ox, oc0);
                    ox += 1;
                }
#undef INB
            }
        }
    }
}

/* ------------------------------------------------- ai-cpu: conv_dw --- */

typedef struct {
    const orc_conv *op;
    uint32_t ih, iw, ow;
    orc_view x;
    const float *wts;  /* [tap][c_pad4] */
    const float *bias; /* [c_pad4] */
    size_t c_pad;
    const orc_view *res;
    float *out;
    size_t px_base;
} dw_ctx;

/* one output pixel, all channels; taps in (ky, kx) order (dw.rs:209-272).
 * The interior fast path of dw.rs:100-200 accumulates in the same order. */
static void dw_px(const dw_ctx *s, const size_t *t_rows, const size_t *iys, size_t nky, size_t oy,
                  size_t ox)
{
    const size_t c = s->op->cout;
    const int64_t sw = s->op->sw, dil = s->op->dil, pl = s->op->pad[1];
    const size_t px_out = oy * s->ow + ox;
    float *o = s->out + (px_out - s->px_base) * c;
    float acc[64];
    for (size_t c0 = 0; c0 < c; c0 += 64) {
        size_t nc = c - c0 < 64 ? c - c0 : 64;
        for (size_t l = 0; l < nc; l++) acc[l] = s->bias[c0 + l];
        for (size_t r = 0; r < nky; r++)
            for (size_t kx = 0; kx < s->op->kw; kx++) {
                int64_t ix = (int64_t)ox * sw + (int64_t)kx * dil - pl;
                if (ix < 0 || ix >= s->iw) continue;
                const float *xv = s->x.data + vbase(&s->x, iys[r] * s->iw + (size_t)ix) + c0;
                const float *wv = s->wts + (t_rows[r] + kx) * s->c_pad + c0;
                for (size_t l = 0; l < nc; l++) acc[l] = acc[l] + xv[l] * wv[l];
            }
        for (size_t l = 0; l < nc; l++) {
            float v = epi_act(s->op->act, acc[l], c0 + l, c);
            if (s->res) v += s->res->data[vbase(s->res, px_out) + c0 + l];
            o[c0 + l] = v;
        }
    }
}

static void conv_dw_rows(const dw_ctx *s, uint32_t y0, uint32_t y1)
{
    size_t t_rows[16], iys[16];
    for (size_t oy = y0; oy < y1; oy++) {
        size_t nky = ky_list(s->op, s->ih, oy, t_rows, iys);
        for (size_t ox = 0; ox < s->ow; ox++) dw_px(s, t_rows, iys, nky, oy, ox);
    }
}

/* ---------------------------------------------------------- the plan --- */

enum { ORC_K_STD = 1, ORC_K_DW = 2, ORC_K_STEM = 3, ORC_K_PWDOT = 4 };

typedef struct {
    int kind;
    orc_conv op;
    orc_conv pw; /* stem: 1x1 over the patch matrix */
    uint32_t ih, iw, oh, ow;
    size_t cin_pad, cout_pad, k_pad, c_pad;
    float *w;
    float *b;
} orc_plan;

/* plan::lower Conv arm (plan.rs:462-619), restricted to single-part,
 * dense-or-view inputs.  w_oihw is logical OIHW; bias may be NULL. */
ORC_API orc_plan *orc_plan_create(const orc_conv *op, uint32_t ih, uint32_t iw, const float *w_oihw,
                                  const float *bias, int input_is_dense, int has_res)
{
    orc_plan *p = (orc_plan *)calloc(1, sizeof(orc_plan));
    if (!p) return NULL;
    p->op = *op;
    p->ih = ih;
    p->iw = iw;
    if (orc_out_hw(op, ih, iw, &p->oh, &p->ow)) {
        free(p);
        return NULL;
    }
    const size_t cout = op->cout, cin = op->cin, taps = (size_t)op->kh * op->kw;
    if (op->groups > 1) {
        if (op->groups != op->cin || op->cin != op->cout) {
            free(p);
            return NULL;
        }
        /* dw::repack_weights: [c][kh][kw] -> [tap][c_pad4] (dw.rs:22-34) */
        p->kind = ORC_K_DW;
        p->c_pad = (cout + 3) / 4 * 4;
        p->w = (float *)calloc(taps * p->c_pad, sizeof(float));
        p->b = (float *)calloc(p->c_pad, sizeof(float));
        for (size_t ch = 0; ch < cout; ch++)
            for (size_t t = 0; t < taps; t++) p->w[t * p->c_pad + ch] = w_oihw[ch * taps + t];
        if (bias) memcpy(p->b, bias, cout * sizeof(float));
    } else if (cin <= 4 && taps > 1 && op->dil == 1 && input_is_dense) {
        /* stem: im2row + 1x1 conv_std over K = kh*kw*cin (plan.rs:513-545) */
        p->kind = ORC_K_STEM;
        size_t k = taps * cin;
        p->k_pad = (k + 3) / 4 * 4;
        p->cout_pad = (cout + NR - 1) / NR * NR;
        p->w = (float *)calloc(p->k_pad * p->cout_pad, sizeof(float));
        p->b = (float *)calloc(p->cout_pad, sizeof(float));
        /* permute_weights: OIHW -> [cout][(ky,kx,ic)] then repack [k][cout_pad] */
        for (size_t oc = 0; oc < cout; oc++)
            for (size_t ic = 0; ic < cin; ic++)
                for (size_t t = 0; t < taps; t++)
                    p->w[(t * cin + ic) * p->cout_pad + oc] = w_oihw[(oc * cin + ic) * taps + t];
        if (bias) memcpy(p->b, bias, cout * sizeof(float));
        p->pw = *op;
        p->pw.cin = (uint32_t)k;
        p->pw.kh = p->pw.kw = p->pw.sh = p->pw.sw = p->pw.dil = 1;
        memset(p->pw.pad, 0, sizeof(p->pw.pad));
    } else if (op->kh == 1 && op->kw == 1 && op->sh == 1 && op->sw == 1 && !has_res && cout <= 4) {
        /* pw_dot::repack_weights: [cout][k_pad4] (pw_dot.rs:19-28) */
        p->kind = ORC_K_PWDOT;
        p->k_pad = (cin + 3) / 4 * 4;
        p->w = (float *)calloc(cout * p->k_pad, sizeof(float));
        p->b = (float *)calloc(cout, sizeof(float));
        for (size_t oc = 0; oc < cout; oc++) memcpy(p->w + oc * p->k_pad, w_oihw + oc * cin, cin * sizeof(float));
        if (bias) memcpy(p->b, bias, cout * sizeof(float));
    } else {
        /* conv::repack_weights: OIHW -> [tap][cin_pad][cout_pad] (conv.rs:44-66) */
        p->kind = ORC_K_STD;
        p->cin_pad = cin % 4 ? (cin + 3) / 4 * 4 : cin;
        p->cout_pad = (cout + NR - 1) / NR * NR;
        p->w = (float *)calloc(taps * p->cin_pad * p->cout_pad, sizeof(float));
        p->b = (float *)calloc(p->cout_pad, sizeof(float));
        for (size_t oc = 0; oc < cout; oc++)
            for (size_t ic = 0; ic < cin; ic++)
                for (size_t t = 0; t < taps; t++)
                    p->w[(t * p->cin_pad + ic) * p->cout_pad + oc] = w_oihw[(oc * cin + ic) * taps + t];
        if (bias) memcpy(p->b, bias, cout * sizeof(float));
    }
    if (!p->w || !p->b) {
        free(p->w);
        free(p->b);
        free(p);
        return NULL;
    }
    return p;
}

ORC_API void orc_plan_free(orc_plan *p)
{
    if (!p) return;
    free(p->w);
    free(p->b);
    free(p);
}

ORC_API int orc_plan_kind(const orc_plan *p) { return p->kind; }

/* im2row (im2row.rs:22-85): out [oh*ow][k_pad], K order (ky, kx, ic) */
static void im2row(const orc_plan *p, const orc_view *x, float *out)
{
    const orc_conv *op = &p->op;
    const size_t c = op->cin;
    for (size_t oy = 0; oy < p->oh; oy++)
        for (size_t ox = 0; ox < p->ow; ox++) {
            float *dst = out + (oy * p->ow + ox) * p->k_pad;
            size_t k = 0;
            for (size_t ky = 0; ky < op->kh; ky++) {
                int64_t iy = (int64_t)(oy * op->sh + ky) - op->pad[0];
                for (size_t kx = 0; kx < op->kw; kx++) {
                    int64_t ix = (int64_t)(ox * op->sw + kx) - op->pad[1];
                    int ok = iy >= 0 && iy < p->ih && ix >= 0 && ix < p->iw;
                    for (size_t ch = 0; ch < c; ch++)
                        dst[k++] = ok ? x->data[vbase(x, (size_t)iy * p->iw + (size_t)ix) + ch] : 0.0f;
                }
            }
            for (; k < p->k_pad; k++) dst[k] = 0.0f;
        }
}

typedef struct {
    const orc_plan *p;
    orc_view x, res;
    int has_res;
    float *out;
    float *scratch;
    uint32_t y0, y1;
} band_job;

static void run_band(const band_job *j)
{
    const orc_plan *p = j->p;
    const orc_view *res = j->has_res ? &j->res : NULL;
    float *out = j->out + (size_t)j->y0 * p->ow * p->op.cout;
    if (p->kind == ORC_K_DW) {
        dw_ctx s = {&p->op, p->ih, p->iw, p->ow, j->x, p->w, p->b, p->c_pad, res, out, (size_t)j->y0 * p->ow};
        conv_dw_rows(&s, j->y0, j->y1);
    } else if (p->kind == ORC_K_STD) {
        std_ctx s = {&p->op, p->ih, p->iw, p->ow, j->x, p->cin_pad, p->w, p->b, p->cout_pad, res, out,
                     (size_t)j->y0 * p->ow, p->op.cout};
        conv_std_rows(&s, j->y0, j->y1);
    } else if (p->kind == ORC_K_STEM) {
        orc_view pv = {j->scratch, 0, p->k_pad, p->k_pad};
        std_ctx s = {&p->pw, p->oh, p->ow, p->ow, pv, p->k_pad, p->w, p->b, p->cout_pad, res, out,
                     (size_t)j->y0 * p->ow, p->op.cout};
        conv_std_rows(&s, j->y0, j->y1);
    }
}

static void *band_thread(void *arg)
{
    run_band((const band_job *)arg);
    return NULL;
}

/* pw_dot (pw_dot.rs:32-61): 4 lane accumulators from zero, (l0+l1)+(l2+l3),
 * then + bias and the scalar activation */
static void run_pwdot(const orc_plan *p, const orc_view *x, float *out)
{
    const size_t cout = p->op.cout, cin = p->op.cin, px = (size_t)p->oh * p->ow;
    for (size_t q = 0; q < px; q++) {
        const float *xv = x->data + vbase(x, q);
        for (size_t oc = 0; oc < cout; oc++) {
            float a[4] = {0, 0, 0, 0};
            const float *w = p->w + oc * p->k_pad;
            for (size_t kc = 0; kc < p->k_pad; kc += 4)
                for (size_t l = 0; l < 4; l++)
                    if (kc + l < cin) a[l] = a[l] + xv[kc + l] * w[kc + l];
            float sum = (a[0] + a[1]) + (a[2] + a[3]);
            out[q * cout + oc] = orc_act_apply(p->op.act, sum + p->b[oc]);
        }
    }
}

/* Run one frame.  The input is a view (x_stride/x_coff: pixel stride and
 * channel offset in floats); res (nullable) likewise; out is dense NHWC.
 * threads > 1 splits output rows into bands as model.rs:421-441 does. */
ORC_API int orc_plan_run(const orc_plan *p, const float *x, size_t x_stride, size_t x_coff, const float *res,
                         size_t res_stride, size_t res_coff, float *out, int threads)
{
    orc_view xv = {x, x_coff, x_stride ? x_stride : p->op.cin, p->op.cin};
    orc_view rv = {res, res_coff, res_stride ? res_stride : p->op.cout, p->op.cout};
    if (p->kind == ORC_K_PWDOT) {
        run_pwdot(p, &xv, out);
        return 0;
    }
    float *scratch = NULL;
    if (p->kind == ORC_K_STEM) {
        scratch = (float *)malloc(((size_t)p->oh * p->ow * p->k_pad + 4) * sizeof(float));
        if (!scratch) return -1;
        im2row(p, &xv, scratch);
    }
    uint32_t rows = p->oh;
    band_job one = {p, xv, rv, res != NULL, out, scratch, 0, rows};
    if (threads > 1 && rows >= (uint32_t)threads) {
        uint32_t band = (rows + threads - 1) / threads;
        pthread_t tid[256];
        band_job jobs[256];
        int n = 0;
        for (uint32_t y0 = 0; y0 < rows && n < 256; y0 += band, n++) {
            jobs[n] = one;
            jobs[n].y0 = y0;
            jobs[n].y1 = y0 + band < rows ? y0 + band : rows;
        }
        int started[256] = {0};
        for (int i = 1; i < n; i++) {
            started[i] = pthread_create(&tid[i], NULL, band_thread, &jobs[i]) == 0;
            if (!started[i]) run_band(&jobs[i]);
        }
        run_band(&jobs[0]);
        for (int i = 1; i < n; i++)
            if (started[i]) pthread_join(tid[i], NULL);
    } else {
        run_band(&one);
    }
    free(scratch);
    return 0;
}

/* --------------------------------------------------- resize and add --- */

/* bilinear resize (reference/resize.rs:5-42); mode 0 = half_pixel,
 * 1 = asymmetric.  Dense NHWC in and out, one frame. */
ORC_API void orc_resize_bilinear(uint32_t ih, uint32_t iw, uint32_t c, const float *in, uint32_t oh, uint32_t ow,
                                 int mode, float *out)
{
    const float sy = (float)ih / (float)oh, sx = (float)iw / (float)ow;
    for (uint32_t oy = 0; oy < oh; oy++) {
        float fy = mode == 0 ? ((float)oy + 0.5f) * sy - 0.5f : (float)oy * sy;
        int64_t fl = (int64_t)floorf(fy);
        int64_t y0 = fl < 0 ? 0 : (fl > (int64_t)ih - 1 ? (int64_t)ih - 1 : fl);
        int64_t y1 = fl + 1 < 0 ? 0 : (fl + 1 > (int64_t)ih - 1 ? (int64_t)ih - 1 : fl + 1);
        float ty = clampf(fy - floorf(fy), 0.0f, 1.0f);
        for (uint32_t ox = 0; ox < ow; ox++) {
            float fx = mode == 0 ? ((float)ox + 0.5f) * sx - 0.5f : (float)ox * sx;
            int64_t fxl = (int64_t)floorf(fx);
            int64_t x0 = fxl < 0 ? 0 : (fxl > (int64_t)iw - 1 ? (int64_t)iw - 1 : fxl);
            int64_t x1 = fxl + 1 < 0 ? 0 : (fxl + 1 > (int64_t)iw - 1 ? (int64_t)iw - 1 : fxl + 1);
            float tx = clampf(fx - floorf(fx), 0.0f, 1.0f);
            for (uint32_t ch = 0; ch < c; ch++) {
                float g00 = in[((size_t)y0 * iw + x0) * c + ch], g01 = in[((size_t)y0 * iw + x1) * c + ch];
                float g10 = in[((size_t)y1 * iw + x0) * c + ch], g11 = in[((size_t)y1 * iw + x1) * c + ch];
                float top = g00 * (1.0f - tx) + g01 * tx;
                float bot = g10 * (1.0f - tx) + g11 * tx;
                out[((size_t)oy * ow + ox) * c + ch] = top * (1.0f - ty) + bot * ty;
            }
        }
    }
}

/* out = act(a + b), dense (elementwise.rs:30-55) */
ORC_API void orc_add(const float *a, const float *b, size_t n, size_t c, int act, float *out)
{
    for (size_t i = 0; i < n; i++) {
        size_t ch = c ? i % c : 0;
        out[i] = epi_act(act, a[i] + b[i], ch, c ? c : 4);
    }
}

/* ---- graph glue (crates/ai-cpu/src/kernels/elementwise.rs, segate.rs;
 * crates/ai-core/src/reference/{elementwise,pool}.rs).  Tensors are channel
 * views: element (pixel q, channel ch) at p[q * stride + off + ch], q over
 * all n * px pixels (ai-cpu's View, crates/ai-cpu/src/view.rs:8-16). */

/* BinaryOp::apply (crates/ai-core/src/ops/elementwise.rs:14-27).  ai-cpu's
 * 4-lane Sub is a + b * (-1) and rounds the same as a - b. */
static inline float bin_apply(int op, float a, float b)
{
    switch (op) {
    case 0: return a + b;
    case 1: return a - b;
    case 2: return a * b;
    default: return a > 0.0f ? a : a * b;
    }
}

/* SwOp::Binary: out = act(a o b).  kind: 0 tensor view, 1 a o scalar,
 * 2 scalar o a, 3 [c] channel vector, 4 [n][c] per-frame channel vector,
 * 5 [n * px] per-pixel scalar (binary_tensor / binary_scalar / binary_cvec /
 * binary_pvec, elementwise.rs:29-101 and the tail loops). */
ORC_API void orc_binary(size_t n, size_t px, size_t c, const float *a, size_t as, size_t ao, int op, int kind,
                        const float *b, size_t bs, size_t bo, float scalar, int act, float *out, size_t os,
                        size_t oo)
{
    for (size_t q = 0; q < n * px; q++) {
        for (size_t ch = 0; ch < c; ch++) {
            float x = a[q * as + ao + ch], s;
            switch (kind) {
            case 0: s = b[q * bs + bo + ch]; break;
            case 3: s = b[ch]; break;
            case 4: s = b[(q / px) * c + ch]; break;
            case 5: s = b[q]; break;
            default: s = scalar; break;
            }
            float v = kind == 2 ? bin_apply(op, s, x) : bin_apply(op, x, s);
            out[q * os + oo + ch] = epi_act(act, v, ch, c);
        }
    }
}

/* SwOp::Mix out = a + z (b - a), elementwise.rs:128-150: the 4-lane part is
 * (a + z b) + (-z) a, the tail a + z (b - a). */
ORC_API void orc_mix(size_t n, size_t px, size_t c, const float *z, size_t zs, size_t zo, const float *a, size_t as,
                     size_t ao, const float *b, size_t bs, size_t bo, float *out, size_t os, size_t oo)
{
    const size_t cv = c / 4 * 4;
    for (size_t q = 0; q < n * px; q++) {
        for (size_t ch = 0; ch < c; ch++) {
            float zv = z[q * zs + zo + ch], av = a[q * as + ao + ch], bv = b[q * bs + bo + ch];
            float r;
            if (ch < cv) {
                float t = av + zv * bv;
                r = t + (zv * -1.0f) * av;
            } else {
                r = av + zv * (bv - av);
            }
            out[q * os + oo + ch] = r;
        }
    }
}

/* SwOp::Gpool: per frame, channel sums in pixel order times 1/px
 * (segate.rs:46-57, reference/pool.rs:5-19).  out: [n][c] dense. */
ORC_API void orc_gpool(size_t n, size_t px, size_t c, const float *x, size_t xs, size_t xo, float *out)
{
    const float inv = 1.0f / (float)px;
    for (size_t f = 0; f < n; f++) {
        float *o = out + f * c;
        for (size_t ch = 0; ch < c; ch++) o[ch] = 0.0f;
        for (size_t p = 0; p < px; p++) {
            const float *row = x + (f * px + p) * xs + xo;
            for (size_t ch = 0; ch < c; ch++) o[ch] += row[ch];
        }
        for (size_t ch = 0; ch < c; ch++) o[ch] *= inv;
    }
}

/* SwOp::Avgpool, one dense frame [ih][iw][c] -> [oh][ow][c]
 * (reference/pool.rs:22-46): divisor kh*kw whatever the border. */
ORC_API void orc_avgpool(uint32_t ih, uint32_t iw, uint32_t c, uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw,
                         uint32_t pt, uint32_t pl, uint32_t oh, uint32_t ow, const float *x, float *out)
{
    const float inv = 1.0f / (float)(kh * kw);
    for (uint32_t oy = 0; oy < oh; oy++)
        for (uint32_t ox = 0; ox < ow; ox++)
            for (uint32_t ch = 0; ch < c; ch++) {
                float acc = 0.0f;
                for (uint32_t ky = 0; ky < kh; ky++)
                    for (uint32_t kx = 0; kx < kw; kx++) {
                        int64_t iy = (int64_t)(oy * sh + ky) - pt, ix = (int64_t)(ox * sw + kx) - pl;
                        if (iy >= 0 && iy < ih && ix >= 0 && ix < iw) acc += x[((size_t)iy * iw + ix) * c + ch];
                    }
                out[((size_t)oy * ow + ox) * c + ch] = acc * inv;
            }
}

/* SwOp::Concat part / Chcopy / Act: out = act(x) between views
 * (elementwise.rs:103-126 for the activation's apply4 / apply split). */
ORC_API void orc_channel_copy(size_t n, size_t px, size_t c, const float *x, size_t xs, size_t xo, int act,
                              float *out, size_t os, size_t oo)
{
    for (size_t q = 0; q < n * px; q++)
        for (size_t ch = 0; ch < c; ch++) out[q * os + oo + ch] = epi_act(act, x[q * xs + xo + ch], ch, c);
}

/* I420 (YUV 4:2:0, planar) -> RGBA8, alpha 255 (crates/ai-ffi/src/yuv.rs:7-31).
 * Chroma sample (y/2, x/2) serves pixel (y, x); each channel is computed in
 * f32 with unfused multiplies and adds, clamped to [0, 255] and truncated
 * (Rust's `as u8`). */
ORC_API void orc_i420_to_rgba(const uint8_t *y, const uint8_t *u, const uint8_t *v, size_t w, size_t h,
                              size_t stride_y, size_t stride_u, size_t stride_v, uint8_t *out)
{
    for (size_t yy = 0; yy < h; yy++)
        for (size_t xx = 0; xx < w; xx++) {
            const float yv = (float)y[yy * stride_y + xx];
            const float uv = (float)u[(yy / 2) * stride_u + xx / 2] - 128.0f;
            const float vv = (float)v[(yy / 2) * stride_v + xx / 2] - 128.0f;
            float r = yv + 1.402f * vv;
            float g = yv - 0.344136f * uv - 0.714136f * vv;
            float b = yv + 1.772f * uv;
            r = r < 0.0f ? 0.0f : r > 255.0f ? 255.0f : r;
            g = g < 0.0f ? 0.0f : g > 255.0f ? 255.0f : g;
            b = b < 0.0f ? 0.0f : b > 255.0f ? 255.0f : b;
            uint8_t *o = out + (yy * w + xx) * 4;
            o[0] = (uint8_t)r;
            o[1] = (uint8_t)g;
            o[2] = (uint8_t)b;
            o[3] = 255;
        }
}

/* RGBA8 -> I420 (crates/ai-ffi/src/yuv.rs:33-58): chroma from the top-left
 * pixel of each 2 x 2 block, not an average. */
ORC_API void orc_rgba_to_i420(const uint8_t *rgba, size_t w, size_t h, uint8_t *y, uint8_t *u, uint8_t *v,
                              size_t stride_y, size_t stride_u, size_t stride_v)
{
    for (size_t yy = 0; yy < h; yy++)
        for (size_t xx = 0; xx < w; xx++) {
            const uint8_t *px = rgba + (yy * w + xx) * 4;
            const float r = (float)px[0], g = (float)px[1], b = (float)px[2];
            float l = 0.299f * r + 0.587f * g + 0.114f * b;
            y[yy * stride_y + xx] = (uint8_t)(l < 0.0f ? 0.0f : l > 255.0f ? 255.0f : l);
            if (yy % 2 == 0 && xx % 2 == 0) {
                float cu = -0.168736f * r - 0.331264f * g + 0.5f * b + 128.0f;
                float cv = 0.5f * r - 0.418688f * g - 0.081312f * b + 128.0f;
                u[(yy / 2) * stride_u + xx / 2] = (uint8_t)(cu < 0.0f ? 0.0f : cu > 255.0f ? 255.0f : cu);
                v[(yy / 2) * stride_v + xx / 2] = (uint8_t)(cv < 0.0f ? 0.0f : cv > 255.0f ? 255.0f : cv);
            }
        }
}
