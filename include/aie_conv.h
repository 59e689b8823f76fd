/*
 * aie_conv.h -- C ABI of the B200 (sm_100a) convolution hot path.
 *
 * One plan per convolution layer; caller-owned device buffers; every call is
 * asynchronous on the caller's CUDA stream and returns an aie_status.  No
 * entry point aborts, and aie_conv_run allocates nothing.
 *
 * What each entry point replaces in ai_engine (paths relative to its root):
 *
 *   aie_conv_plan          the SwOp::Conv arm of ai-gpu-runtime's lower_op
 *                          (crates/ai-gpu-runtime/src/lowering.rs:99-187):
 *                          groups>1 -> depthwise (ConvDwSpec, conv_dw.rs:21),
 *                          kh==1 -> pointwise GEMM (GemmPwSpec + pick_variant,
 *                          gemm_pw.rs:91-149), else implicit GEMM
 *                          (ConvIgemmSpec::from_op, conv_igemm.rs:79).
 *   aie_conv_plan_info     KernelSpec::cache_key / workgroups introspection
 *                          (crates/ai-gpu/src/kernel.rs:26-36).
 *   aie_conv_pack_weights  the converter's weight packing
 *                          (crates/ai-core/src/pack.rs:68-184, consumed by
 *                          ai-convert plan/lower.rs:116-190); accepts the
 *                          logical OIHW form or the .sw blob's packed form.
 *   aie_conv_run           kernel::record of one OpDispatch
 *                          (crates/ai-gpu/src/kernel.rs:181-191) with the
 *                          binding order of lowering.rs:169-178:
 *                          input, weights, bias, optional residual, output.
 *   aie_resize_bilinear    ResizeBilinearSpec (crates/ai-gpu/src/kernels/
 *                          resize_bilinear.rs) fused with an optional Binary
 *                          add (crates/ai-gpu/src/kernels/elementwise.rs).
 *   aie_binary, aie_mix,   the non-conv SwOps between the convs: Binary, Mix,
 *   aie_gpool, aie_avgpool, Gpool, Avgpool, Concat, Chcopy / Act
 *   aie_concat,            (crates/ai-core/src/format/model.rs:111-214),
 *   aie_channel_copy       in ai-cpu's rounding (crates/ai-cpu/src/kernels/
 *                          elementwise.rs, segate.rs).
 *   aie_conv_plan_parts, aie_conv_run_parts
 *                          ConvIgemmSpec's concat parts (conv_igemm.rs:49-76)
 *                          read in place by the GEMM.
 *   aie_conv_run_dw_pw(_up2), aie_conv_run_mbconv, aie_conv_run_stem_pw
 *                          two or three consecutive dispatches of a lowered
 *                          graph as one launch (see each declaration).
 *   aie_status_string      RuntimeError's Display
 *                          (crates/ai-gpu-runtime/src/error.rs:5-13).
 *   aie_device_status      GpuContext::lost_reason polling
 *                          (crates/ai-gpu/src/context.rs:145).
 *
 * Status convention follows ai-ffi's VbResult (include/ai_engine_ffi.h:15-18
 * in ai_engine): 0 success, negative failure.
 */
#ifndef AIE_CONV_H
#define AIE_CONV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AIE_ABI_VERSION 2

#ifndef AIE_API
#define AIE_API __attribute__((visibility("default")))
#endif

typedef enum aie_status {
    AIE_OK = 0,
    AIE_E_FAILURE = -1,        /* VbResult::Failure */
    AIE_E_INVALID = -2,        /* bad descriptor, null pointer, bad size */
    AIE_E_UNSUPPORTED = -3,    /* valid conv this library does not run */
    AIE_E_CUDA = -4,           /* a CUDA runtime/driver call failed */
    AIE_E_ALIGN = -5,          /* pointer/stride alignment the kernel needs */
    AIE_E_DEVICE_TIMEOUT = -6, /* a bounded device-side wait gave up */
    AIE_E_NOMEM = -7           /* host allocation failed (plan time only) */
} aie_status;

/* Order of ai-core's Activation enum (crates/ai-core/src/activation.rs:7-24). */
typedef enum aie_act {
    AIE_ACT_NONE = 0,
    AIE_ACT_RELU = 1,
    AIE_ACT_SIGMOID = 2,
    AIE_ACT_TANH = 3,
    AIE_ACT_HARDSWISH = 4,
    AIE_ACT_HARDSIGMOID = 5,
    AIE_ACT_CLAMP01 = 6,
    AIE_ACT_RELU6 = 7,
    AIE_ACT_SQRT = 8,
    AIE_ACT_NEG = 9,
    AIE_ACT_RECIP = 10
} aie_act;

/* Activation memory layouts.  NHWC is ai-cpu's dense logical layout
 * (crates/ai-cpu/src/view.rs); NHWC_C4 is ai-gpu's layout with channels
 * zero-padded to a multiple of 4 (crates/ai-core/src/tensor.rs:1-9).  With
 * NHWC_C4 the output's padding lanes are written as zero, so the output
 * buffer equals pack_nhwc() of the logical result. */
typedef enum aie_layout { AIE_LAYOUT_NHWC = 0, AIE_LAYOUT_NHWC_C4 = 1 } aie_layout;

/* Arithmetic of the dense contractions.  FFMA: fp32 fused multiply-add on
 * the CUDA cores.  TF32: tcgen05 tensor cores, fp32 operands read as TF32,
 * fp32 accumulate in tensor memory.  FP32_STRICT: fp32 on the CUDA cores with
 * every multiply and add rounded separately, in ai-cpu's accumulation order
 * (bias, then taps in (ky, kx) order, then input channels ascending), which
 * reproduces ai-cpu's x86 results bit for bit apart from the transcendental
 * activations.  AUTO picks TF32 where the operand layout allows TMA, else
 * FFMA.  Depthwise runs the unfused order under every setting. */
typedef enum aie_math {
    AIE_MATH_AUTO = 0,
    AIE_MATH_FFMA = 1,
    AIE_MATH_TF32 = 2,
    AIE_MATH_FP32_STRICT = 3
} aie_math;

/* Kernel family chosen by aie_conv_plan. */
typedef enum aie_kernel {
    AIE_KERNEL_DW = 1,         /* depthwise */
    AIE_KERNEL_PW = 2,         /* 1x1 GEMM (M = n*h*w, K = cin, N = cout) */
    AIE_KERNEL_IGEMM = 3,      /* implicit-GEMM k x k conv */
    AIE_KERNEL_PW_DOT = 4      /* 1x1 with cout <= 4: per-pixel dot products */
} aie_kernel;

/* Weight formats accepted by aie_conv_pack_weights. */
typedef enum aie_wfmt {
    AIE_WFMT_OIHW = 0,     /* logical [cout][cin/groups][kh][kw], bias [cout] */
    AIE_WFMT_SW_PACKED = 1 /* .sw blob form: conv [tap][kg_pad][ng][4][4]
                              (pack.rs:68-102, kg_pad = ceil(cin/4) rounded up
                              to a multiple of 4), depthwise [tap][cg][4]
                              (pack.rs:105-122), bias [ng][4] (pack.rs:178) */
} aie_wfmt;

/* Conv2d (crates/ai-core/src/ops/conv.rs:6-21) plus batch, layout and math.
 * Zero view fields mean "dense per layout". */
typedef struct aie_conv_desc {
    uint32_t n;          /* frames in the batch (the reference is batch 1) */
    uint32_t ih, iw;     /* input spatial size */
    uint32_t cin, cout;
    uint32_t kh, kw;
    uint32_t sh, sw;
    uint32_t pad[4];     /* top, left, bottom, right */
    uint32_t dil;        /* isotropic dilation */
    uint32_t groups;     /* 1 = dense, cin (== cout) = depthwise */
    int32_t act;         /* aie_act; epilogue order bias -> act -> +residual */
    int32_t has_res;     /* residual tensor of the output's shape */
    int32_t layout;      /* aie_layout of in / res / out */
    int32_t math;        /* aie_math */
    uint32_t split_k;    /* tensor-core 1x1 GEMM K split; 0 = auto, 1 = off */
    /* channel views (SrcView, crates/ai-gpu/src/kernels/common/source.rs:17):
     * pixel stride and first channel, in floats */
    uint32_t in_stride, in_coff;
    uint32_t res_stride, res_coff;
    uint32_t out_stride, out_coff;
    /* residual source: AIE_RES_TENSOR reads a tensor of the output's shape;
     * AIE_RES_BILINEAR_* reads a [n][res_h][res_w][cout] tensor and samples
     * it bilinearly at every output pixel (crates/ai-core/src/reference/
     * resize.rs:5-42), i.e. the Resize -> Conv(res) pair of an FPN merge
     * fused into the conv epilogue. */
    int32_t res_mode;
    uint32_t res_h, res_w;
} aie_conv_desc;

typedef enum aie_res_mode {
    AIE_RES_TENSOR = 0,
    AIE_RES_BILINEAR_HALF_PIXEL = 1,
    AIE_RES_BILINEAR_ASYMMETRIC = 2
} aie_res_mode;

typedef struct aie_plan_info {
    int32_t kernel;            /* aie_kernel */
    int32_t math;              /* resolved aie_math (FFMA, TF32 or FP32_STRICT) */
    uint32_t oh, ow;
    uint32_t split_k;          /* resolved split (1 = none) */
    uint32_t tile_m, tile_n;   /* CTA tile of the GEMM kernels */
    uint32_t variant;          /* IGEMM run as a small-cin direct conv when the
                                  output is 16-byte aligned: 1 = FFMA (cin <= 4,
                                  3x3), 2 = tensor-core im2col GEMM (TF32,
                                  cin <= 3, cout = 32, no residual);
                                  3 = PW on the FP32 pipes with TMA-staged
                                  tiles (FFMA, cin and cout in {32, 64}:
                                  chosen by AUTO for an exact-2x half_pixel
                                  residual, and by FFMA);
                                  0 = the family's main kernel */
    uint64_t weight_bytes;     /* size of dev_w for aie_conv_pack_weights */
    uint64_t bias_bytes;       /* size of dev_b */
    uint64_t workspace_bytes;  /* scratch aie_conv_run needs (0 = none) */
    uint64_t flops;            /* algorithmic 2*MACs, border taps counted */
    uint64_t min_bytes;        /* input + weights + bias + output (+ res), fp32 */
    uint64_t grid_ctas;        /* CTAs of the main launch */
} aie_plan_info;

typedef struct aie_plan aie_plan;

/* ABI version and a build string. */
AIE_API int32_t aie_abi_version(void);
AIE_API const char *aie_build_info(void);

/* Validate a conv, choose its kernel and math, and allocate a host-side plan
 * (immutable, shareable across threads).  Replaces lowering.rs:99-187. */
AIE_API int aie_conv_plan(const aie_conv_desc *desc, aie_plan **out);
AIE_API int aie_conv_plan_info(const aie_plan *plan, aie_plan_info *info);
AIE_API void aie_plan_free(aie_plan *plan);

/* Pack host weights (format aie_wfmt) into the plan's device layout.
 * dev_w / dev_b must hold info.weight_bytes / info.bias_bytes; bias may be
 * NULL (zeros).  Synchronous with respect to the host buffers; the device
 * copy is ordered on `stream` (a cudaStream_t, NULL = legacy default). */
AIE_API int aie_conv_pack_weights(const aie_plan *plan, int32_t wfmt, const float *w_host, const float *bias_host,
                          void *dev_w, void *dev_b, void *stream);

/* Run one conv over the batch.  in / res / out are device pointers in the
 * plan's layout; workspace must hold info.workspace_bytes (may be NULL when
 * that is 0).  Asynchronous on `stream`. */
AIE_API int aie_conv_run(const aie_plan *plan, const void *in, const void *dev_w, const void *dev_b, const void *res,
                 void *out, void *workspace, void *stream);

/* Depthwise conv followed by the 1x1 conv that consumes its output, fused
 * into one launch: the depthwise result never reaches memory.  This is the
 * segmentation head of the MobileNet-style nets (dw k x k -> 1x1 to <= 4
 * logits/mask channels).  `dw` must be a depthwise plan (k 3 or 5, stride 1
 * or 2, dilation 1, cout a multiple of 4 and <= 32, no residual, not
 * FP32_STRICT) over a dense input; `pw` a plan of kind AIE_KERNEL_PW_DOT
 * over dw's output shape (cin = dw's cout, no residual, not FP32_STRICT).
 * Weights and biases as packed for each plan; `out` is pw's output.
 * Otherwise AIE_E_UNSUPPORTED: run the two plans with aie_conv_run.
 * No counterpart in the reference, which dispatches the two convs in turn
 * (ai-gpu-runtime's lower_op emits one spec per SwOp::Conv,
 * crates/ai-gpu-runtime/src/lowering.rs:99-187). */
AIE_API int aie_conv_run_dw_pw(const aie_plan *dw, const aie_plan *pw, const void *in, const void *dw_w,
                       const void *dw_b, const void *pw_w, const void *pw_b, void *out, void *stream);

/* aie_conv_run_dw_pw over the depthwise input in + up2(up): `up` is a dense
 * [n][up_h][up_w][C] tensor (C = the depthwise channels, 16-byte aligned)
 * with 2 up_h, 2 up_w the depthwise input's height and width, and up2 the
 * exact-2x half_pixel bilinear resize (crates/ai-core/src/reference/
 * resize.rs:5-42).  The sum is formed in the kernel's staged input tile
 * (the resize's lerps as fused multiply-adds: the FFMA path's rounding), so
 * neither the up-sampled tensor nor the sum reaches memory.  Replaces the tail of a feature pyramid that
 * the reference dispatches as Resize, Conv(residual = the resize's output),
 * depthwise Conv, 1x1 Conv (ai-gpu-runtime lowering.rs:99-187, one spec per
 * op): `in` is the lateral conv's output computed without its residual.
 * AIE_E_UNSUPPORTED when the shapes do not match or the operands are not
 * TMA-compatible (dense, 16-byte aligned). */
AIE_API int aie_conv_run_dw_pw_up2(const aie_plan *dw, const aie_plan *pw, const void *in, const void *up,
                           uint32_t up_h, uint32_t up_w, const void *dw_w, const void *dw_b, const void *pw_w,
                           const void *pw_b, void *out, void *stream);

/* A whole inverted-bottleneck block in one launch: 1x1 expand `ex` ->
 * depthwise 3x3 (stride 1, pad 1) `dw` -> 1x1 project `pj` (+ residual),
 * the expanded tensor never reaching memory.  For small frames (h <= 10,
 * w <= 18, e.g. the 10x18 stages of a 160x288 MobileNet): one CTA per
 * frame, tcgen05 TF32 GEMMs with the pixels as the MMA's N side, the
 * depthwise on the CUDA cores between them.  All three are ordinary
 * aie_conv_plan results over dense NHWC tensors: `ex` and `pj` 1x1 plans
 * that resolved to TF32 (cin % 32 == 0, pj cout <= 128), `dw` a non-strict
 * depthwise plan; weights and biases as packed for each plan; `res` is the
 * project plan's residual (NULL without one).  `dw` NULL (dw_w, dw_b
 * ignored): a 1x1 expand straight into a 1x1 project, e.g. a wide head conv
 * whose only reader is a pyramid lateral -- the wide tensor never reaches
 * memory either.  Otherwise AIE_E_UNSUPPORTED: run the plans with
 * aie_conv_run.  Replaces the three (two) dispatches ai-gpu-runtime's
 * lower_op makes for the block (GemmPwSpec, ConvDwSpec, GemmPwSpec;
 * crates/ai-gpu-runtime/src/lowering.rs:99-187). */
AIE_API int aie_conv_run_mbconv(const aie_plan *ex, const aie_plan *dw, const aie_plan *pj, const void *in,
                        const void *ex_w, const void *ex_b, const void *dw_w, const void *dw_b, const void *pj_w,
                        const void *pj_b, const void *res, void *out, void *stream);

/* The tensor-core stem (a plan with aie_plan_info.variant 2: 3x3, cin <= 3,
 * cout 32) and a TF32 1x1 conv that reads its output (cin 32, cout <= 32 and
 * a multiple of 4, no residual, dense) in one launch: the stem writes its
 * output to stem_out as aie_conv_run would, and the 1x1's result to pw_out,
 * computed from the stem's staged output tile without reading it back from
 * memory.  Replaces the two dispatches ai-gpu-runtime records for a stem
 * conv and a feature-pyramid lateral on its output
 * (crates/ai-gpu-runtime/src/lowering.rs:99-187, kernel.rs:181-191).
 * AIE_E_UNSUPPORTED for plans outside that shape. */
AIE_API int aie_conv_run_stem_pw(const aie_plan *stem, const aie_plan *pw, const void *in, const void *stem_w,
                                 const void *stem_b, const void *pw_w, const void *pw_b, void *stem_out,
                                 void *pw_out, void *stream);

/* Input staging: a batch of interleaved u8 RGB (cin = 3) or RGBA (cin = 4,
 * alpha dropped) frames [n, h, w, cin] -> the network's f32 input
 * [n, h, w, 3] (layout NHWC) or [n, h, w, 4] (NHWC_C4, 4th lane 0), each
 * value u8 / 255 (IEEE division).  Replaces the reference's frame
 * normalisation -- on the GPU, ai-tasks' preprocess pass
 * (crates/ai-tasks/src/features/vb/shaders/preprocess.wgsl:11-16, unorm
 * texture sample -> [0, 1]); on the CPU, `v as f32 / 255.0`
 * (crates/ai-tasks/src/detect/roi.rs:166) -- at the model's resolution.
 * Lets a caller upload 3 bytes per pixel instead of 12. */
AIE_API int aie_input_u8(uint32_t n, uint32_t h, uint32_t w, uint32_t cin, const void *in, int32_t layout,
                 void *out, void *stream);

/* A batch of YUV 4:2:0 camera frames, one set of planes per frame, all on
 * the device.  I420 (planar): u and v are separate planes, uv_step = 1.
 * NV12: u points at the interleaved chroma plane and v = u + 1, uv_step = 2
 * (NV21: v at the plane, u = v + 1).  Chroma planes hold ceil(h/2) rows of
 * ceil(w/2) samples.  Strides are in bytes; frame_* is the distance between
 * consecutive frames' planes (0 = stride * rows, tightly packed). */
typedef struct aie_yuv420 {
    const void *y, *u, *v;
    uint32_t stride_y, stride_u, stride_v;
    uint32_t uv_step;
    uint64_t frame_y, frame_u, frame_v;
} aie_yuv420;

/* Input staging from YUV 4:2:0 frames: [n] frames of h x w -> the network's
 * f32 RGB input [n, h, w, 3] (layout NHWC) or [n, h, w, 4] (NHWC_C4, 4th
 * lane 0).  Each pixel is converted exactly as ai-ffi's i420_to_rgba
 * (crates/ai-ffi/src/yuv.rs:7-31: BT.601 full range, chroma sample
 * (y/2, x/2), f32 arithmetic, clamped and truncated to a byte) and that byte
 * read as v / 255, as the model's input normalisation does -- on the GPU,
 * with no RGBA intermediate.  Replaces the reference's CPU round trip
 * (i420_to_rgba in ai-ffi, then the frame upload). */
AIE_API int aie_input_yuv420(uint32_t n, uint32_t h, uint32_t w, const aie_yuv420 *src, int32_t layout, void *out,
                             void *stream);

/* Bilinear resize of a dense NHWC batch [n, ih, iw, c] to [n, oh, ow, c]
 * (crates/ai-core/src/reference/resize.rs:5-42; mode 0 = half_pixel,
 * 1 = asymmetric), then out = act(resized + add) when add is non-NULL
 * (add has the output's shape), else act(resized). */
AIE_API int aie_resize_bilinear(uint32_t n, uint32_t ih, uint32_t iw, uint32_t c, const void *in, uint32_t oh,
                        uint32_t ow, int32_t mode, const void *add, int32_t act, void *out, void *stream);

/* ---- Graph glue: the non-conv ops of ai_engine's recurrent matting graph
 * (RVM) and its segmentation heads, on NHWC f32 batches.  Each is one
 * stream-ordered launch, allocates nothing, and rounds every result the way
 * ai-cpu's kernels do (unfused multiply and add), so results are
 * bit-identical to ai-cpu's except for sigmoid / tanh (libm's expf / tanhf
 * against CUDA's, an ulp or two).
 *
 * A tensor argument is a channel view of an NHWC buffer -- the runtime's
 * SrcView (crates/ai-gpu/src/kernels/common/source.rs:17-80) and ai-cpu's
 * View (crates/ai-cpu/src/view.rs:8-16): element (pixel q, channel ch), q running
 * over every frame's pixels, lives at data[q * stride + coff + ch].
 * stride = 0 means dense (stride = the op's channel count). */
typedef struct aie_tview {
    void *data;
    uint32_t stride;
    uint32_t coff;
} aie_tview;

/* ai-core's BinaryOp (crates/ai-core/src/ops/elementwise.rs:5-11). */
typedef enum aie_binop { AIE_BIN_ADD = 0, AIE_BIN_SUB = 1, AIE_BIN_MUL = 2, AIE_BIN_PRELU = 3 } aie_binop;

/* Kinds of a Binary op's second operand (SwOperand,
 * crates/ai-core/src/format/model.rs:60-75). */
typedef enum aie_operand {
    AIE_OPND_TENSOR = 0,       /* b: same shape as a (a view) */
    AIE_OPND_SCALAR = 1,       /* a o scalar */
    AIE_OPND_SCALAR_FIRST = 2, /* scalar o a */
    AIE_OPND_CVEC = 3,         /* b.data: [c] channel vector, all frames (Cvec) */
    AIE_OPND_CVEC_TENSOR = 4,  /* b.data: [n][c] per-frame channel vector (CvecTensor: an SE gate) */
    AIE_OPND_PVEC_TENSOR = 5   /* b.data: [n * px] per-pixel scalar, all channels (PvecTensor) */
} aie_operand;

/* out = act(a o b) over n frames of px pixels and c channels: SwOp::Binary
 * (crates/ai-core/src/format/model.rs:111-117; reference
 * crates/ai-core/src/reference/elementwise.rs:7-26; ai-cpu
 * crates/ai-cpu/src/kernels/elementwise.rs: binary_tensor, binary_scalar,
 * binary_cvec, binary_pvec).  out may alias a or b exactly. */
AIE_API int aie_binary(uint32_t n, uint32_t px, uint32_t c, aie_tview a, int32_t op, int32_t b_kind, aie_tview b,
                       float scalar, int32_t act, aie_tview out, void *stream);

/* ConvGRU mix out = a + z (b - a): SwOp::Mix (crates/ai-core/src/format/
 * model.rs:193-199), ai-cpu's elementwise::mix (elementwise.rs:128-150),
 * in its rounding order. */
AIE_API int aie_mix(uint32_t n, uint32_t px, uint32_t c, aie_tview z, aie_tview a, aie_tview b, aie_tview out,
                    void *stream);

/* Global average pool [n][px][c] -> out [n][c] (dense): SwOp::Gpool
 * (crates/ai-core/src/reference/pool.rs:5-19; ai-cpu segate.rs:46-57),
 * summed in pixel order then scaled by 1/px, bit-identical to ai-cpu.
 * Feeds an SE gate's 1x1 convs (run as aie_conv plans over n frames of
 * 1 x 1 pixels) and AIE_OPND_CVEC_TENSOR. */
AIE_API int aie_gpool(uint32_t n, uint32_t px, uint32_t c, aie_tview in, void *out, void *stream);

/* Average pool with the fixed kh*kw divisor (taps outside the frame add
 * nothing): SwOp::Avgpool (crates/ai-core/src/reference/pool.rs:22-46).
 * Dense NHWC [n, ih, iw, c] -> [n, oh, ow, c]; pad = {top, left, bottom,
 * right}; oh = (ih + pt + pb - kh) / sh + 1 (likewise ow). */
AIE_API int aie_avgpool(uint32_t n, uint32_t ih, uint32_t iw, uint32_t c, uint32_t kh, uint32_t kw, uint32_t sh,
                        uint32_t sw, const uint32_t pad[4], const void *in, void *out, void *stream);

/* out[q, 0:c] = act(in[q, 0:c]) between channel views: one part of a
 * channel concat written at its offset (SwOp::Concat), a channel slice
 * (SwOp::Chcopy) or a stand-alone activation (SwOp::Act)
 * (crates/ai-core/src/format/model.rs:156-175). */
AIE_API int aie_channel_copy(uint32_t n, uint32_t px, uint32_t c, aie_tview in, int32_t act, aie_tview out,
                             void *stream);

/* Channel concat of nparts (1..8) views, part i holding part_c[i] channels,
 * into out[q, 0:out_c] in one pass: SwOp::Concat (crates/ai-core/src/
 * format/model.rs:156-160) and the conv's concat-into-conv parts
 * (Conv.srcs, model.rs:83-86; SrcView, crates/ai-gpu/src/kernels/common/
 * source.rs:17-80).  out_c may exceed the parts' total: those trailing
 * lanes are written as zero (a buffer padded to a multiple of 4 channels). */
AIE_API int aie_concat(uint32_t n, uint32_t px, uint32_t nparts, const aie_tview *parts, const uint32_t *part_c,
                       uint32_t out_c, aie_tview out, void *stream);

/* ---- Concat-into-conv.  A conv whose input is the channel concat of up to
 * three separate views, read in place by the tensor-core GEMM: ai-gpu's
 * implicit-GEMM conv with concat parts (ConvIgemmSpec srcs, crates/ai-gpu/
 * src/kernels/conv_igemm.rs:49-76; SrcView, crates/ai-gpu/src/kernels/
 * common/source.rs:17-80; the Conv op's srcs, crates/ai-core/src/format/
 * model.rs:83-86), so the concatenated tensor is never written.
 *
 * aie_conv_plan_parts: desc describes the conv over the concatenated input
 * (cin = the sum of part_c[0..nparts), layout NHWC, no input view, math
 * AUTO or TF32, not depthwise); weights are packed from the ordinary OIHW /
 * .sw forms by aie_conv_pack_weights.  Returns AIE_E_UNSUPPORTED when the
 * conv does not run on the tensor cores (a 1x1 with cout <= 4, strides
 * above 2): concat first and use aie_conv_plan.
 * aie_conv_run_parts: parts[i] is part i's view (its data, pixel stride and
 * first channel; stride 0 = dense), 16-byte aligned with a pixel stride
 * that is a multiple of 4 channels (TMA); otherwise AIE_E_ALIGN.  The other
 * arguments are aie_conv_run's.  A parts plan is refused by aie_conv_run
 * and an ordinary plan by aie_conv_run_parts. */
AIE_API int aie_conv_plan_parts(const aie_conv_desc *desc, uint32_t nparts, const uint32_t *part_c, aie_plan **out);
AIE_API int aie_conv_run_parts(const aie_plan *plan, const aie_tview *parts, const void *dev_w, const void *dev_b,
                               const void *res, void *out, void *workspace, void *stream);

/* Human-readable status, and the detail message of this thread's last
 * failure (copied into buf, NUL-terminated; returns its full length). */
AIE_API const char *aie_status_string(int status);
AIE_API int aie_last_error(char *buf, size_t len);

/* Size of the library's built-in split-K scratch (16 MiB per GPU). */
#define AIE_NOALLOC_SCRATCH_BYTES (16u << 20)

/* aie_conv_run for callers that cannot allocate device memory while they
 * run: a real-time frame loop that cannot absorb cudaMalloc's implicit
 * device synchronisation, or a plugin inside a host application that owns
 * the device allocator and hands over only its own tensors.  No counterpart
 * in the reference.  Instead of a caller workspace, split-K partials use a
 * fixed AIE_NOALLOC_SCRATCH_BYTES array inside the library (held by every
 * GPU that loads it, until exit); plans needing more are rejected with
 * AIE_E_UNSUPPORTED.  The first call on each device (with that device
 * current, and `stream` belonging to it) looks up the array's device
 * address; make that first call before any stream capture.  All calls
 * share the array: calls that overlap on the GPU race on it.  Allocates
 * nothing. */
AIE_API int aie_conv_run_noalloc(const aie_plan *plan, const void *in, const void *dev_w, const void *dev_b,
                                 const void *res, void *out, void *stream);

/* Failure-detection self-test: launch a kernel whose only wait (an
 * mbarrier nothing arrives at) gives up after timeout_us (1..2e6), records
 * its code in the device error word and returns -- the bounded-wait path of
 * the conv kernels, exercised without a fault.  Follow with
 * aie_device_status, which must report AIE_E_DEVICE_TIMEOUT.  Counterpart
 * of ai-gpu's device-loss test (crates/ai-gpu/tests/device_lost.rs). */
AIE_API int aie_selftest_wait_timeout(uint32_t timeout_us, void *stream);

/* Read and clear the device error word that bounded device-side waits set
 * when they give up (synchronises `stream`).  AIE_OK or
 * AIE_E_DEVICE_TIMEOUT; *code_out (nullable) receives the raw word. */
AIE_API int aie_device_status(void *stream, uint32_t *code_out);

#ifdef __cplusplus
}
#endif

#endif /* AIE_CONV_H */
