// xnor.cu -- bit-packed XNOR convolution (TXNORConvolutionLayer, source/nxnorconvolutionlayer.pas).
//
// The reference packs im2col columns into bit rows (im2col_cpu_custom_bin :232-316,
// transpose_bin :457-478) and counts equal bits with 64-bit POPCNT
// (gemm_nn_custom_bin_mean_transposed :179-205): out = (2*count - K)*mean_f.
// Here:
//   * weights  -> Wb[f][tap][cw]  : bit j of word cw = (w[f][32*cw+j][tap] > 0)
//   * input    -> Xb[b][cw][pixel]: bit j = (x[b][32*cw+j][pixel] > 0)   (context workspace)
//   * counting mismatches instead of matches: pad channels are 0 in both operands, so they
//     never mismatch and need no mask; a padding pixel is an all-zero word (bit 0 = -1, as the
//     reference never sets it), so it mismatches exactly the weight's set bits.
//     2*count - K = K - 2*mismatches; both are integers, the fp32 multiply by mean_f is the
//     reference's single rounding.
#include "common.cuh"

using namespace tbi;

namespace {

// mean_f = (sum_i |w_fi|)/size in sequential fp32 order (binarize_weights :95-113) and the
// sign bits of every (filter, tap, channel word).
__global__ void k_xnor_pack_w(int F, int C, int KK, int Cw, const float* __restrict__ w,
                              uint32_t* __restrict__ wb, float* __restrict__ mean) {
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        const long long size = (long long)C * KK;
        const float* wf = w + (long long)f * size;
        float m = 0.0f;
        for (long long i = 0; i < size; ++i) m = __fadd_rn(m, fabsf(wf[i]));
        mean[f] = __fdiv_rn(m, (float)size);
        for (int tap = 0; tap < KK; ++tap)
            for (int cw = 0; cw < Cw; ++cw) {
                uint32_t bits = 0;
                for (int j = 0; j < 32; ++j) {
                    int c = cw * 32 + j;
                    if (c < C && wf[(long long)c * KK + tap] > 0.0f) bits |= 1u << j;
                }
                wb[((long long)f * KK + tap) * Cw + cw] = bits;
            }
    }
}

__global__ void k_xnor_pack_x(long long total, int C, int HW, int Cw, const float* __restrict__ x,
                              uint32_t* __restrict__ xb) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int pix = (int)(i % HW);
        long long t = i / HW;
        int cw = (int)(t % Cw);
        long long b = t / Cw;
        const float* src = x + (b * C + (long long)cw * 32) * HW + pix;
        uint32_t bits = 0;
        int lim = C - cw * 32 < 32 ? C - cw * 32 : 32;
        for (int j = 0; j < lim; ++j)
            if (src[(long long)j * HW] > 0.0f) bits |= 1u << j;
        xb[i] = bits;
    }
}

constexpr int XF = 32;   // filters per CTA
constexpr int XP = 128;  // output pixels per CTA (one per thread)

__global__ void __launch_bounds__(XP)
k_xnor_conv(int C, int H, int W, int F, int K, int stride, int pad, int OH, int OW, int Cw,
            int pad_mode, const uint32_t* __restrict__ xb, const uint32_t* __restrict__ wb,
            const float* __restrict__ mean, const float* __restrict__ bias, int act,
            int32_t* __restrict__ counts, float* __restrict__ y) {
    extern __shared__ __align__(16) uint32_t ws[];  // [tap][cw][XF]
    const int KK = K * K;
    const int f0 = blockIdx.y * XF;
    const int b = blockIdx.z;
    const int nf = min(XF, F - f0);
    for (int i = threadIdx.x; i < KK * Cw * XF; i += blockDim.x) {
        int f = i % XF, tc = i / XF;  // tc = tap*Cw + cw
        ws[i] = (f < nf) ? wb[((long long)(f0 + f) * KK) * Cw + tc] : 0u;
    }
    __syncthreads();
    const int OHW = OH * OW;
    const int p = blockIdx.x * XP + threadIdx.x;
    if (p >= OHW) return;
    const int oy = p / OW, ox = p - oy * OW;
    const uint32_t* xbb = xb + (long long)b * Cw * H * W;
    int mism[XF];
#pragma unroll
    for (int f = 0; f < XF; ++f) mism[f] = 0;
    int valid_taps = 0;
    for (int r = 0; r < K; ++r) {
        const int iy = oy * stride - pad + r;
        for (int s = 0; s < K; ++s) {
            const int ix = ox * stride - pad + s;
            const bool ok = (unsigned)iy < (unsigned)H && (unsigned)ix < (unsigned)W;
            if (!ok && pad_mode == TB_XNOR_PAD_ZERO) continue;
            valid_taps += ok ? 1 : 0;
            const uint32_t* wt = ws + (r * K + s) * Cw * XF;
            const uint32_t* xp = xbb + (ok ? (long long)iy * W + ix : 0);
            for (int cw = 0; cw < Cw; ++cw) {
                const uint32_t xw = ok ? __ldg(xp + (long long)cw * H * W) : 0u;
                const uint4* w4 = reinterpret_cast<const uint4*>(wt + cw * XF);
#pragma unroll
                for (int q = 0; q < XF / 4; ++q) {
                    uint4 wv = w4[q];
                    mism[4 * q + 0] += __popc(xw ^ wv.x);
                    mism[4 * q + 1] += __popc(xw ^ wv.y);
                    mism[4 * q + 2] += __popc(xw ^ wv.z);
                    mism[4 * q + 3] += __popc(xw ^ wv.w);
                }
            }
        }
    }
    const int Kbits = (pad_mode == TB_XNOR_PAD_ZERO) ? C * valid_taps : C * KK;
#pragma unroll
    for (int f = 0; f < XF; ++f) {
        if (f < nf) {
            const int fo = f0 + f;
            const int v = Kbits - 2 * mism[f];
            const long long oi = ((long long)b * F + fo) * OHW + p;
            if (counts) counts[oi] = v;
            float o = __fmul_rn((float)v, mean[fo]);
            if (bias) o = __fadd_rn(o, bias[fo]);
            if (act != TB_ACT_LINEAR) o = tb_activate_dev(o, act);
            y[oi] = o;
        }
    }
}

}  // namespace

extern "C" {

int tb_xnor_packed_weights_count(int64_t filters, int64_t channels, int64_t ksize, int64_t* count) {
    if (filters <= 0 || channels <= 0 || ksize <= 0 || !count) return fail(TB_ERR_INVALID, "xnor: bad shape");
    *count = filters * ksize * ksize * ceil_div(channels, 32);
    return TB_OK;
}

int tb_xnor_pack_weights(tb_ctx* ctx, int64_t filters, int64_t channels, int64_t ksize,
                         const float* weights, uint32_t* packed, float* mean) {
    TB_ENTER(ctx);
    if (filters <= 0 || channels <= 0 || ksize <= 0 || !weights || !packed || !mean)
        return fail(TB_ERR_INVALID, "xnor pack: bad arguments");
    const int64_t Cw = ceil_div(channels, 32);
    k_xnor_pack_w<<<grid_for(filters, 64, ctx->sm_count), 64, 0, ctx->stream>>>(
        (int)filters, (int)channels, (int)(ksize * ksize), (int)Cw, weights, packed, mean);
    return check_launch("k_xnor_pack_w");
}

int tb_xnor_conv_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                     int64_t filters, int64_t ksize, int64_t stride, int64_t pad, int64_t pad_mode,
                     const float* x, const uint32_t* packed_w, const float* mean, const float* bias,
                     int64_t activation, int32_t* popcount_out, float* y) {
    TB_ENTER(ctx);
    if (batch < 0 || channels <= 0 || h <= 0 || w <= 0 || filters <= 0 || ksize <= 0 ||
        stride <= 0 || pad < 0 || (pad_mode != TB_XNOR_PAD_BIT0 && pad_mode != TB_XNOR_PAD_ZERO))
        return fail(TB_ERR_INVALID, "xnor conv: bad shape");
    if (!act_supported(activation)) return fail(TB_ERR_UNSUPPORTED, "xnor conv: activation not supported");
    const int64_t oh = (h + 2 * pad - ksize) / stride + 1, ow = (w + 2 * pad - ksize) / stride + 1;
    if (oh <= 0 || ow <= 0) return fail(TB_ERR_INVALID, "xnor conv: empty output");
    if (batch == 0) return TB_OK;
    if (!x || !packed_w || !mean || !y) return fail(TB_ERR_INVALID, "xnor conv: null pointer");
    const int64_t Cw = ceil_div(channels, 32);
    const int64_t smem = ksize * ksize * Cw * XF * 4;
    if (smem > ctx->max_smem_optin)
        return fail(TB_ERR_UNSUPPORTED, "xnor conv: %lld channels x %lldx%lld kernel exceed shared memory",
                    (long long)channels, (long long)ksize, (long long)ksize);
    if (batch > 65535 || ceil_div(filters, XF) > 65535) return fail(TB_ERR_INVALID, "xnor conv: grid too large");
    const int64_t xwords = batch * Cw * h * w;
    int r = ensure_workspace(ctx, (size_t)xwords * 4);
    if (r != TB_OK) return r;
    uint32_t* xb = reinterpret_cast<uint32_t*>(ctx->ws);
    k_xnor_pack_x<<<grid_for(xwords, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
        xwords, (int)channels, (int)(h * w), (int)Cw, x, xb);
    r = check_launch("k_xnor_pack_x");
    if (r != TB_OK) return r;
    static bool attr_done[64] = {false};
    if (ctx->device < 64 && !attr_done[ctx->device]) {
        TB_CHECK_CUDA(cudaFuncSetAttribute(k_xnor_conv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           ctx->max_smem_optin));
        attr_done[ctx->device] = true;
    }
    dim3 grid((unsigned)ceil_div(oh * ow, XP), (unsigned)ceil_div(filters, XF), (unsigned)batch);
    k_xnor_conv<<<grid, XP, (size_t)smem, ctx->stream>>>(
        (int)channels, (int)h, (int)w, (int)filters, (int)ksize, (int)stride, (int)pad, (int)oh,
        (int)ow, (int)Cw, (int)pad_mode, xb, packed_w, mean, bias, (int)activation, popcount_out, y);
    return check_launch("k_xnor_conv");
}

}  // extern "C"
