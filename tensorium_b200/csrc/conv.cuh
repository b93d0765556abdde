// conv.cuh -- shared definitions of the implicit-GEMM convolution kernels.
//
// GEMM view of TTensor.Conv2D (source/ntensors.pas:8252-8349), per image:
//   Y[f][p] = sum_k W[f][k] * im2col(X)[k][p],  M = filters, N = out_h*out_w, K = c*kh*kw.
// Here the N dimension runs over all images of the batch (n = b*OHW + p), so one launch
// covers the whole batch; im2col is never materialised (the B tile is gathered from NCHW X).
//
// Packed weights (tb_conv_pack_weights): Wp[k][m], row length Mpad = round_up(F, 4), with
// two K orders:
//   RSC (channels >= 16): k = (r*kw + s)*Cpad + c, Cpad = round_up(C, 16): a 16-deep k tile
//        lies inside one kernel tap (r, s), so the im2col validity test is per tile.
//   CRS (small channel counts): k = (c*kh + r)*kw + s (the reference order), K padded to 16.
#pragma once
#include "common.cuh"

namespace tbi {

constexpr int CONV_BK = 16;
constexpr int CONV_CRS_MAX_K = 1024;  // CRS k-table lives in shared memory

enum ConvMode { MODE_CRS = 0, MODE_RSC = 1, MODE_1X1V = 2 };

struct ConvGeom {
    int64_t B, C, H, W, F, KH, KW, SY, SX, PY, PX, DY, DX, OH, OW;
    int64_t x_bs, y_bs, r_bs;
    bool rsc;
    int64_t Cpad, Kpad, Mpad;
};

struct ConvParams {
    const float* __restrict__ x;
    const float* __restrict__ w;
    const float* __restrict__ bias;
    const float* __restrict__ bn_scale;
    const float* __restrict__ bn_mean;
    const float* __restrict__ bn_var;
    const float* __restrict__ res;
    float* __restrict__ y;
    float* __restrict__ ws;
    int* __restrict__ tile_cnt;  // split-K arrival counters, one per output tile, left at 0
    int C, H, W, F, KH, KW, SY, SX, PY, PX, DY, DX, OH, OW, OHW;
    int Cpad, Kpad, Mpad;
    long long x_bs, y_bs, r_bs, Ntot;
    int ktiles, kt_per_split, splits;
    int act, yolo_classes;
    int vec_out;  // 1: OHW, y_bs, r_bs multiples of 4 and y/res 16-byte aligned
    int wrsc;     // packed weight order: 1 = RSC (k = (r*kw + s)*Cpad + c), 0 = CRS
};

inline bool conv_is_rsc(int64_t C, int64_t KH, int64_t KW) {
    return !(C < 16 && C * KH * KW <= CONV_CRS_MAX_K);
}

int conv_geom(const tb_conv_desc* d, ConvGeom* g);

// Launch the conv (FP32 SIMT mainloop) with the given epilogue settings.
// ws / ws_floats: split-K partial buffer (nullptr = use the context workspace).
// tile_cnt: split-K arrival counters (nullptr = the context's); tile_cnt_len entries.
int conv_fp32_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp,
                     const float* bias, const float* bn_scale, const float* bn_mean,
                     const float* bn_var, const float* res, float* y, int act, int yolo_classes,
                     float* ws, int64_t ws_floats, int64_t* launches, int* tile_cnt = nullptr,
                     int64_t tile_cnt_len = 0, bool allow_tma = true);
// Order-exact FP32 conv (conv_exact.cu): the reference's k order and one FMA chain per output
// (fma = false: the connected layer's separate multiply and add), no split of K, no scratch.
bool conv_exact_supported(const ConvGeom& g);
int conv_exact_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                      const float* bn_scale, const float* bn_mean, const float* bn_var, const float* res, float* y,
                      int act, int yolo_classes, bool fma, int64_t* launches);
int conv_exact_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, float* y, bool fma);
// Connected layer in the reference's sdot_avx2 order (layers.cu): g is a 1x1 conv over 1x1 inputs.
int fc_sdot_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                   const float* bn_scale, const float* bn_mean, const float* bn_var, float* y, int act,
                   int64_t* launches);
// TF32 tensor-core path (conv_tc.cu): convolutions with channels % 32 == 0 (any stride, dilation).
bool conv_tc_supported(const ConvGeom& g);
int64_t conv_tc_scratch_floats(const ConvGeom& g);
int conv_tc_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                   const float* bn_scale, const float* bn_mean, const float* bn_var, const float* res,
                   float* y, int act, int yolo_classes, float* scratch, int64_t* launches,
                   unsigned long long* phases = nullptr);
// Diagnostic: MMA issue rate (see conv_tc.cu).
int conv_tc_mma_rate(tb_ctx* ctx, int kmajor, double* tflops_at_clock, double* cycles_per_mma);
// FP32 conv fed by TMA (conv_fp32_tma.cu): RSC layers with more than one output pixel.
bool conv_fp32_tma_supported(const ConvGeom& g);
int64_t conv_fp32_tma_ws_floats(const ConvGeom& g, int splits);
int conv_fp32_tma_run(tb_ctx* ctx, const ConvGeom& g, ConvParams p, float* ws, int64_t ws_floats,
                      int64_t tile_cnt_len, int64_t* launches);
// Measure the tensor-core tile shapes of this geometry on x / y and keep the fastest.
int conv_tc_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, float* y);
// Round packed weights to TF32 (nearest, ties away) in place.
int conv_tc_round_weights(tb_ctx* ctx, float* packed, int64_t n);
// Measure the candidate (tile, split) choices of this geometry on x / y and keep the fastest.
int conv_fp32_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, float* y);
// TF32 tensor-core conv on NHWC activations with the A operand fetched by TMA im2col (conv_nhwc.cu).
// pair = 1: BF16-split operands (activations as bf16 (hi, lo) pairs in 32-bit slots, weights as two
// bf16 operands (hi, hi) and (lo, lo); kind::f16 MMAs accumulate all four partial products)
int64_t conv_nhwc_packed_count(const ConvGeom& g, int pair = 0);
bool conv_nhwc_supported(const ConvGeom& g, int64_t x_ps);
int conv_nhwc_pack(tb_ctx* ctx, const ConvGeom& g, const float* w, float* wp, int pair = 0);
int conv_nhwc_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, int64_t x_ps, const float* wp,
                     const float* bias, const float* res, int64_t r_ps, float* y, int64_t y_ps, int act,
                     int yolo_classes, unsigned long long* phases, int pair = 0);
int64_t conv_nhwc_ws_floats(tb_ctx* ctx, const ConvGeom& g, int64_t x_ps, int pair = 0);
int conv_nhwc_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, int64_t x_ps, const float* wp, float* y,
                       int64_t y_ps, int pair = 0);
// NHWC data-movement layers of the network's NHWC plan (nhwc_layers.cu); strides in floats per pixel.
int nhwc_from_nchw(tb_ctx* ctx, int64_t batch, int64_t c, int64_t h, int64_t w, const float* x, int64_t x_bs,
                   float* y, int64_t ps, int pair = 0);
// first layer with C * KH * KW <= 32: receptive fields as 32 channels of a 1x1 conv, and its weights
int nhwc_im2col_first(tb_ctx* ctx, int64_t B, int64_t C, int64_t H, int64_t W, int64_t KH, int64_t KW, int64_t SY,
                      int64_t SX, int64_t PY, int64_t PX, int64_t DY, int64_t DX, int64_t OH, int64_t OW,
                      const float* x, int64_t x_bs, float* y, int pair = 0);
int nhwc_pack_first(tb_ctx* ctx, int64_t F, int64_t C, int64_t KH, int64_t KW, const float* w, float* wp, int pair = 0);
// the first layer computed directly from the NCHW input into its NHWC output (C*KH*KW <= 32,
// F <= 128, leaky or linear, no residual); weights packed [k][F rounded up to 32] by
// nhwc_pack_first_direct (nhwc_first_direct_wcount floats)
bool nhwc_first_direct_supported(int64_t C, int64_t KH, int64_t KW, int64_t SY, int64_t SX, int64_t DY, int64_t DX,
                                 int64_t F, int64_t yps);
int64_t nhwc_first_direct_wcount(int64_t F, int64_t C, int64_t KH, int64_t KW);
int nhwc_pack_first_direct(tb_ctx* ctx, int64_t F, int64_t C, int64_t KH, int64_t KW, const float* w, float* wd,
                           int pair = 0);
int nhwc_first_direct(tb_ctx* ctx, int64_t B, int64_t C, int64_t H, int64_t W, int64_t KH, int64_t KW, int64_t SY,
                      int64_t SX, int64_t PY, int64_t PX, int64_t DY, int64_t DX, int64_t OH, int64_t OW,
                      const float* x, int64_t x_bs, const float* wd, const float* bias, int64_t F, int act, float* y,
                      int64_t yps, int pair = 0);
int nhwc_upsample(tb_ctx* ctx, int64_t batch, int64_t c, int64_t h, int64_t w, int64_t s, float scale,
                  const float* x, int64_t xps, float* y, int64_t yps, int pair = 0);
int nhwc_copy(tb_ctx* ctx, int64_t npix, int64_t c, const float* x, int64_t xps, float* y, int64_t yps);
int nhwc_shortcut(tb_ctx* ctx, int64_t npix, int64_t c, const float* a, int64_t aps, const float* b, int64_t bps,
                  float* y, int64_t yps, int act, int pair = 0);
// Direct convolution for short reductions (C*KH*KW <= 32, CRS-packed weights, no residual, no
// fused yolo): the first layer of an image network (conv_direct.cu).
bool conv_direct_supported(const ConvGeom& g, const float* res, int yolo_classes);
// The first-layer direct kernel (conv_direct.cu, k_first_direct): C*KH*KW <= 32, F <= 128, bias
// then leaky or linear; w[k * wstride + f] with k = (c * KH + r) * KW + s. Output NCHW planes
// (yps == 0, y_bs floats per image) or NHWC (yps floats per pixel, F % 4 == 0). fmt 0: fp32
// operands and outputs, one FMA chain per output in ascending k from 0 (bit-identical to the
// reference CPU path); 1: operands and outputs rounded to TF32; 2: fp32 operands, bf16-pair outputs.
struct FirstGeom {
    int64_t B, C, H, W, KH, KW, SY, SX, PY, PX, DY, DX, OH, OW;
};
bool first_direct_supported(int64_t C, int64_t KH, int64_t KW, int64_t SY, int64_t SX, int64_t DY, int64_t DX, int64_t F,
                            bool nhwc);
int first_direct_launch(tb_ctx* ctx, const FirstGeom& g, const float* x, int64_t x_bs, const float* w, int64_t wstride,
                        const float* bias, int64_t F, int act, float* y, int64_t y_bs, int64_t yps, int fmt);
int conv_direct_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                       const float* bn_scale, const float* bn_mean, const float* bn_var, float* y, int act,
                       int64_t* launches);
// Split-K partial floats this call would need (0 when it does not split), for a given x.
// allow_tma = false: only the gather kernels (callers whose scratch cannot hold a replica)
int64_t conv_fp32_ws_floats_for(tb_ctx* ctx, const ConvGeom& g, const float* x, bool allow_tma = true);
// The same for a caller-provided scratch of cap_floats partials and cap_tiles counters (the gather
// kernels, K split lowered until it fits; a split pinned by TB_CONV_FORCE is kept).
int64_t conv_fp32_ws_floats_fit(tb_ctx* ctx, const ConvGeom& g, const float* x, int64_t cap_floats,
                                int64_t cap_tiles);

// Floats of split-K workspace the FP32 path needs for this geometry (0 if it does not split).
int64_t conv_fp32_ws_floats(tb_ctx* ctx, const ConvGeom& g);

// TBaseLayer.batchNorm inference (source/nbaselayer.pas:336-370):
// (x - mean)/max(sqrt(var), 1e-6) * scale + bias, one rounding per step as the reference.
static __device__ __noinline__ float conv_bn(float v, float mean, float var, float scale, float bias) {
    float d = (float)sqrt((double)var);
    float sd = fmaxf(d, 0.000001f);
    float t = __fdiv_rn(__fsub_rn(v, mean), sd);
    t = __fmul_rn(t, scale);
    return __fadd_rn(t, bias);
}

// Epilogue of one output value: bias / unfused batchnorm, activation, fused yolo logistic.
__device__ __forceinline__ float conv_epilogue(float v, int m, const ConvParams& p) {
    if (p.bn_mean) {
        v = conv_bn(v, p.bn_mean[m], p.bn_var[m], p.bn_scale ? p.bn_scale[m] : 1.0f,
                    p.bias ? p.bias[m] : 0.0f);
    } else if (p.bias) {
        v = __fadd_rn(v, p.bias[m]);
    }
    if (p.yolo_classes > 0) {
        int e = m % (p.yolo_classes + 5);
        if (e != 2 && e != 3) v = tb_logistic(v);  // TYoloLayer.forward entries 0,1,4..
        return v;
    }
    if (p.act != TB_ACT_LINEAR) v = tb_activate_dev(v, p.act);
    return v;
}

// The epilogue of one value. simple: no unfused batchnorm, no yolo, leaky or linear -- then the
// row's bias bm (0 without bias) and the flags come from registers the caller loaded once,
// instead of re-reading the kernel parameters for every value.
__device__ __forceinline__ float conv_epi_value(float v, int m, const ConvParams& p, bool simple, bool has_bias,
                                                bool leaky, float bm) {
    if (!simple) return conv_epilogue(v, m, p);
    if (has_bias) v = __fadd_rn(v, bm);
    return (leaky && v < 0.f) ? __fmul_rn(v, 0.1f) : v;  // activate_array's leaky (leaky_array: v * 0.1f)
}

}  // namespace tbi
