// conv_direct.cu -- direct convolution for layers with a short reduction (C*KH*KW <= 32): the
// first layer of an image network (YOLOv3's 3 -> 32, 3x3 at 416x416; the MNIST 1 -> 32, 5x5).
//
// On the FP32 path. As a GEMM these layers have K <= 32 and a huge N (every output pixel), so a
// tiled GEMM spends its time filling tiles and running epilogues for a single k tile. Here a thread
// gathers the K input values of each of its output pixels once (from input rows staged in shared
// memory, zero for padding) into registers, then runs, per filter, the reference's dot product --
// one FMA per k in ascending (c, kh, kw) order starting from 0 (sim2Col + sgemm_nn's saxpy rows,
// source/ntensors.pas:11415-11532, 2061-2157, 1308-1435) -- followed by the usual epilogue. The
// result is bit-identical to the reference's CPU arithmetic.
#include "conv.cuh"

namespace tbi {

namespace {

constexpr int DIRECT_KMAX = 32;
constexpr int DIRECT_FMAX = 128;
constexpr int DIRECT_THREADS = 128;
constexpr int DIRECT_SEG = 4 * DIRECT_THREADS;  // widest row segment of one block (4 pixels per thread)
constexpr int DIRECT_SMEM_MAX = 96 * 1024;

// Columns of one staged input row for a segment of seg outputs.
__host__ __device__ inline int direct_cols(int SX, int KW, int DX, int seg) { return (seg - 1) * SX + (KW - 1) * DX + 1; }

// One block: DIRECT_SEG consecutive output pixels of one output row of one image. The C x KH input
// rows they read are staged in shared memory (zero where the window leaves the image), so the
// per-pixel gather is K plain shared-memory loads. Each thread then makes DIRECT_PPT pixels
// (DIRECT_THREADS apart, so every store instruction writes 128 consecutive pixels of one filter
// plane) for every filter, 8 filters at a time: per k two 16-byte broadcast loads of weights and
// 8 * DIRECT_PPT FMAs. KT > 0 fixes the reduction length at compile time (the common first layers:
// 3x3x3 = 27, 1x5x5 = 25), which keeps the k loop free of per-iteration guards.
// PPT: output pixels per thread (4 for large images; 1 when that would leave the GPU short of blocks).
template <int KT, int PPT>  // KT > 0: the reduction length as a compile-time constant (0: runtime, <= DIRECT_KMAX)
__global__ void __launch_bounds__(DIRECT_THREADS) k_conv_direct(const ConvParams p, int segs) {
    TB_GRID_DEP_ENTRY();
    constexpr int DIRECT_PPT = PPT, SEG = PPT * DIRECT_THREADS;
    extern __shared__ __align__(16) float dsm[];
    float* wsm = dsm;                                   // [k][f] (DIRECT_FMAX per k)
    float* xs = dsm + DIRECT_KMAX * DIRECT_FMAX;        // [c * KH + r][cols]
    __shared__ int ktab[DIRECT_KMAX];                   // per k: offset in xs of the tap
    const int K = KT > 0 ? KT : p.C * p.KH * p.KW;
    const int F8 = (p.F + 7) & ~7;
    const int cols = direct_cols(p.SX, p.KW, p.DX, SEG);
    const int seg = blockIdx.x % segs;
    const int oy = (blockIdx.x / segs) % p.OH;
    const long long b = blockIdx.x / ((long long)segs * p.OH);
    const int ox0 = seg * SEG;
    for (int i = threadIdx.x; i < K * F8; i += blockDim.x) {
        const int k = i / F8, f = i - k * F8;
        wsm[k * DIRECT_FMAX + f] = f < p.F ? p.w[(long long)k * p.Mpad + f] : 0.0f;
    }
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const int c = k / (p.KH * p.KW), rs = k - c * p.KH * p.KW;
        const int r = rs / p.KW, s = rs - r * p.KW;
        ktab[k] = (c * p.KH + r) * cols + s * p.DX;
    }
    const float* xb = p.x + b * p.x_bs;
    const int ix0 = ox0 * p.SX - p.PX;
    for (int i = threadIdx.x; i < p.C * p.KH * cols; i += blockDim.x) {
        const int row = i / cols, col = i - row * cols;
        const int c = row / p.KH, r = row - c * p.KH;
        const int iy = oy * p.SY - p.PY + r * p.DY, ix = ix0 + col;
        xs[i] = (iy >= 0 && iy < p.H && ix >= 0 && ix < p.W) ? __ldg(xb + ((long long)c * p.H + iy) * p.W + ix) : 0.0f;
    }
    __syncthreads();
    const int t = threadIdx.x;
    if (ox0 + t >= p.OW) return;  // no shared-memory barrier follows
    float xv[DIRECT_PPT][DIRECT_KMAX];
#pragma unroll
    for (int q = 0; q < DIRECT_PPT; ++q)
#pragma unroll
        for (int k = 0; k < DIRECT_KMAX; ++k) xv[q][k] = k < K ? xs[ktab[k] + (t + q * DIRECT_THREADS) * p.SX] : 0.0f;
    int nq = 0;  // pixels of this thread inside the row
#pragma unroll
    for (int q = 0; q < DIRECT_PPT; ++q) nq += ox0 + t + q * DIRECT_THREADS < p.OW;
    float* yrow = p.y + b * p.y_bs + (long long)oy * p.OW + ox0 + t;
    const bool simple = !p.bn_mean && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
    for (int f0 = 0; f0 < p.F; f0 += 8) {
        float acc[DIRECT_PPT][8];
#pragma unroll
        for (int q = 0; q < DIRECT_PPT; ++q)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[q][j] = 0.0f;
        // k runs to K exactly (a branch out of the unrolled loop: predicating the FMAs of
        // k >= K instead would cost a select per accumulator and k)
#pragma unroll
        for (int k = 0; k < DIRECT_KMAX; ++k) {
            if (k == K) break;
            const float4 wa = *reinterpret_cast<const float4*>(wsm + k * DIRECT_FMAX + f0);
            const float4 wb = *reinterpret_cast<const float4*>(wsm + k * DIRECT_FMAX + f0 + 4);
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int q = 0; q < DIRECT_PPT; ++q)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[q][j] = fmaf(wv[j], xv[q][k], acc[q][j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int f = f0 + j;
            if (f < p.F) {
                float* yf = yrow + (long long)f * p.OHW;
                const float bias = p.bias ? __ldg(p.bias + f) : 0.0f;
                // unfused batchnorm (TBaseLayer.batchNorm, as conv_bn): the filter's constants once
                float mean = 0.f, sd = 1.f, sc = 1.f;
                if (p.bn_mean) {
                    mean = __ldg(p.bn_mean + f);
                    sd = fmaxf((float)sqrt((double)__ldg(p.bn_var + f)), 0.000001f);
                    sc = p.bn_scale ? __ldg(p.bn_scale + f) : 1.0f;
                }
#pragma unroll
                for (int q = 0; q < DIRECT_PPT; ++q) {
                    if (q < nq) {
                        float o = acc[q][j];
                        if (simple) {  // bias, then leaky or linear (the common first layer)
                            if (p.bias) o = __fadd_rn(o, bias);
                            if (p.act == TB_ACT_LEAKY && o < 0.f) o = __fmul_rn(o, 0.1f);
                        } else if (p.bn_mean) {  // normalize, forwardScale, forwardBias, activation
                            o = __fadd_rn(__fmul_rn(__fdiv_rn(__fsub_rn(o, mean), sd), sc), bias);
                            if (p.act != TB_ACT_LINEAR) o = tb_activate_dev(o, p.act);
                        } else {
                            o = conv_epilogue(o, f, p);
                        }
                        __stcs(yf + q * DIRECT_THREADS, o);
                    }
                }
            }
        }
    }
}

}  // namespace

static int64_t direct_smem(const ConvGeom& g) {
    return (int64_t)(DIRECT_KMAX * DIRECT_FMAX + g.C * g.KH * direct_cols((int)g.SX, (int)g.KW, (int)g.DX, DIRECT_SEG)) * 4;
}

bool conv_direct_supported(const ConvGeom& g, const float* res, int yolo_classes) {
    return !g.rsc && g.C * g.KH * g.KW <= DIRECT_KMAX && g.F <= DIRECT_FMAX && !res && yolo_classes == 0 &&
           g.SX <= 4 && g.DX * (g.KW - 1) <= 64 && direct_smem(g) <= DIRECT_SMEM_MAX &&
           g.B * g.OH * ceil_div(g.OW, DIRECT_SEG) < ((int64_t)1 << 31) && g.C * g.H * g.W < ((int64_t)1 << 31) &&
           g.OH * g.OW < ((int64_t)1 << 31);
}

int conv_direct_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                       const float* bn_scale, const float* bn_mean, const float* bn_var, float* y, int act,
                       int64_t* launches) {
    ConvParams p{};
    p.x = x; p.w = wp; p.bias = bias; p.bn_scale = bn_scale; p.bn_mean = bn_mean; p.bn_var = bn_var;
    p.y = y;
    p.C = (int)g.C; p.H = (int)g.H; p.W = (int)g.W; p.F = (int)g.F; p.KH = (int)g.KH; p.KW = (int)g.KW;
    p.SY = (int)g.SY; p.SX = (int)g.SX; p.PY = (int)g.PY; p.PX = (int)g.PX; p.DY = (int)g.DY; p.DX = (int)g.DX;
    p.OH = (int)g.OH; p.OW = (int)g.OW; p.OHW = (int)(g.OH * g.OW);
    p.Mpad = (int)g.Mpad;
    p.x_bs = g.x_bs; p.y_bs = g.y_bs;
    p.act = act;
    const long long npix = g.B * g.OH * g.OW;
    (void)npix;
    // four pixels per thread while that still gives every SM a few blocks, else one
    const bool wide = g.B * g.OH * ceil_div(g.OW, DIRECT_SEG) >= 4 * (int64_t)ctx->sm_count;
    const int seg = wide ? DIRECT_SEG : DIRECT_THREADS;
    const int segs = (int)ceil_div(g.OW, seg);
    const int64_t blocks = g.B * g.OH * segs;
    const int64_t smem = (int64_t)(DIRECT_KMAX * DIRECT_FMAX + g.C * g.KH * direct_cols((int)g.SX, (int)g.KW, (int)g.DX, seg)) * 4;
    static bool attr[64] = {false};
    if (ctx->device < 64 && !attr[ctx->device]) {
        TB_CHECK_CUDA(cudaFuncSetAttribute(k_conv_direct<0, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, DIRECT_SMEM_MAX));
        TB_CHECK_CUDA(cudaFuncSetAttribute(k_conv_direct<27, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, DIRECT_SMEM_MAX));
        TB_CHECK_CUDA(cudaFuncSetAttribute(k_conv_direct<25, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, DIRECT_SMEM_MAX));
        TB_CHECK_CUDA(cudaFuncSetAttribute(k_conv_direct<0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, DIRECT_SMEM_MAX));
        TB_CHECK_CUDA(cudaFuncSetAttribute(k_conv_direct<27, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, DIRECT_SMEM_MAX));
        TB_CHECK_CUDA(cudaFuncSetAttribute(k_conv_direct<25, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, DIRECT_SMEM_MAX));
        attr[ctx->device] = true;
    }
    const int64_t K = g.C * g.KH * g.KW;
    const unsigned nb = (unsigned)blocks;
    auto kern = wide ? (K == 27 ? k_conv_direct<27, 4> : K == 25 ? k_conv_direct<25, 4> : k_conv_direct<0, 4>)
                     : (K == 27 ? k_conv_direct<27, 1> : K == 25 ? k_conv_direct<25, 1> : k_conv_direct<0, 1>);
    const int lr = launch(ctx, "k_conv_direct", kern, dim3(nb), dim3(DIRECT_THREADS), (size_t)smem, p, segs);
    if (lr != TB_OK) return lr;
    if (launches) ++*launches;
    return check_launch("k_conv_direct");
}

}  // namespace tbi
