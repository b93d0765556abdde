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

#include <cstdlib>
#include <mutex>

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


// ---- the first-layer kernel: bias + leaky / linear only, NCHW or NHWC output ----
//
// A block makes FK_ROWS output rows x FK_SEG consecutive output pixels of one image (FK_PPT
// pixels per thread, FK_THREADS apart). The weights ([k][filter], filters rounded up to FK_FG),
// the bias and every input row the block's output rows read (per channel, zero in the padding) are
// staged in shared memory once, behind one barrier; then for each output row each thread gathers
// the K inputs of its pixels into registers, then FK_FG filters at a time: per k, four 16-byte broadcast loads of weights and
// FK_FG x FK_PPT FMAs, each accumulator one chain in ascending k from 0 (the reference's order).
// NHWC outputs go through a per-warp staging tile so that each store instruction writes whole
// 64-byte pixel row pieces; NCHW outputs are stored per filter plane, 32 consecutive pixels per warp.
constexpr int FK_THREADS = 128, FK_PPT = 2, FK_SEG = FK_THREADS * FK_PPT, FK_ROWS = 8;
constexpr int FK_KMAX = 32, FK_FMAX = 128, FK_FG = 16;  // filters per pass
constexpr int FK_STG = FK_FG + 4;                        // staging row pitch (floats)

struct FirstParams {
    const float* x;
    long long x_bs;
    int C, H, W, KH, KW, SY, SX, PY, PX, DY, DX, OH, OW;
    int segs, row_blocks;  // blocks per output row segment / output-row groups per image
    const float* w;
    int wstride;
    const float* bias;
    int F, act;
    float* y;
    long long y_bs;
    int yps;  // NHWC: floats per pixel
    int fmt;  // 0: fp32, 1: TF32 operands and outputs, 2: fp32 operands, bf16-pair outputs
};

__host__ __device__ inline int fk_cols(int SX, int KW, int DX) { return (FK_SEG - 1) * SX + (KW - 1) * DX + 1; }
// input rows per channel that FK_ROWS consecutive output rows read
__host__ __device__ inline int fk_rows(int SY, int KH, int DY) { return (FK_ROWS - 1) * SY + (KH - 1) * DY + 1; }

// 4-byte asynchronous global -> shared copy; pred = false writes a zero.
__device__ __forceinline__ void fk_cp4(float* smem, const float* gmem, bool pred) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(gmem), "r"(pred ? 4 : 0) : "memory");
}

// KT: 27 = 3 channels, 3x3; 25 = 1 channel, 5x5 (the window, stride 1 and no dilation as
// compile-time constants); 0: any
// window with C * KH * KW <= 32. FMT: the operand / output format (FirstParams::fmt); NHWC output
// for FMT 1 and 2, NCHW planes for FMT 0.
template <int KT, int FMT>
__global__ void __launch_bounds__(FK_THREADS, 3) k_first_direct(const FirstParams p) {
    TB_GRID_DEP_ENTRY();
    constexpr bool NHWC = FMT != 0;
    constexpr int CT = KT == 27 ? 3 : KT == 25 ? 1 : 0, KWT = KT == 27 ? 3 : KT == 25 ? 5 : 0;
    extern __shared__ __align__(16) float fsm[];
    const int C = CT ? CT : p.C, KH = KWT ? KWT : p.KH, KW = KWT ? KWT : p.KW;
    const int K = KT > 0 ? KT : C * KH * KW;
    // the compile-time windows come with stride 1 and no dilation (the host checks), so every
    // shared-memory offset below folds into an immediate
    const int SX = KT ? 1 : p.SX, SY = KT ? 1 : p.SY, DX = KT ? 1 : p.DX, DY = KT ? 1 : p.DY;
    const int FG = (p.F + FK_FG - 1) & ~(FK_FG - 1);
    const int cols = fk_cols(SX, KW, DX);
    float* wsm = fsm;                                    // [K][FG]
    float* bsm = wsm + K * FG;                           // [FG]
    const int nrin = fk_rows(SY, KH, DY);
    float* xs = bsm + FG;                                // [c][nrin input rows][cols]
    float* stg = xs + ((C * nrin * cols + 3) & ~3);      // NHWC: per warp 32 x FK_STG
    const int seg = blockIdx.x % p.segs;
    const int rb = (blockIdx.x / p.segs) % p.row_blocks;
    const long long b = blockIdx.x / ((long long)p.segs * p.row_blocks);
    const int ox0 = seg * FK_SEG;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    // Staging: every copy is an asynchronous 4-byte cp.async (zero-filled where the weight column
    // or the input pixel does not exist), all in flight at once; a thread then waits for its own
    // copies, rounds them in place for the TF32 output format, and the block synchronises.
    const float* xb = p.x + b * p.x_bs;
    const int ix0 = ox0 * SX - p.PX;
    const int OHW = p.OH * p.OW;
    for (int i = t; i < K * FG; i += FK_THREADS) {
        const int k = i / FG, f = i - k * FG;
        const bool ok = f < p.F;
        fk_cp4(wsm + i, ok ? p.w + (long long)k * p.wstride + f : p.w, ok);
    }
    for (int f = t; f < FG; f += FK_THREADS) {
        const bool ok = p.bias && f < p.F;
        fk_cp4(bsm + f, ok ? p.bias + f : p.w, ok);
    }
    {
        const int iy0 = rb * FK_ROWS * SY - p.PY;  // first input row of the block
        const int n = C * nrin * cols;
        for (int i = t; i < n; i += FK_THREADS) {
            const int row = i / cols, col = i - row * cols;
            const int c = row / nrin, ri = row - c * nrin;
            const int iy = iy0 + ri, ix = ix0 + col;
            const bool ok = iy >= 0 && iy < p.H && ix >= 0 && ix < p.W;
            fk_cp4(xs + i, ok ? xb + ((long long)c * p.H + iy) * p.W + ix : p.x, ok);
        }
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    if constexpr (FMT == 1) {  // the TF32 operands: this thread's own copies, rounded in place
        for (int i = t; i < K * FG; i += FK_THREADS) wsm[i] = tb_tf32_rna(wsm[i]);
        for (int i = t; i < C * nrin * cols; i += FK_THREADS) xs[i] = tb_tf32_rna(xs[i]);
    }
    __syncthreads();
    for (int rr = 0; rr < FK_ROWS; ++rr) {
        const int oy = rb * FK_ROWS + rr;
        if (oy >= p.OH) break;  // the same for every thread of the block
        float xv[FK_PPT][FK_KMAX];
        {
            int c = 0, r = 0, s = 0;  // k = (c * KH + r) * KW + s
#pragma unroll
            for (int k = 0; k < FK_KMAX; ++k) {
                const int off = (c * nrin + rr * SY + r * DY) * cols + s * DX + t * SX;
#pragma unroll
                for (int q = 0; q < FK_PPT; ++q) xv[q][k] = k < K ? xs[off + q * FK_THREADS * SX] : 0.0f;
                if (k < K && ++s == KW) {
                    s = 0;
                    if (++r == KH) r = 0, ++c;
                }
            }
        }
        for (int f0 = 0; f0 < p.F; f0 += FK_FG) {
            float acc[FK_PPT][FK_FG];
#pragma unroll
            for (int q = 0; q < FK_PPT; ++q)
#pragma unroll
                for (int j = 0; j < FK_FG; ++j) acc[q][j] = 0.0f;
#pragma unroll
            for (int k = 0; k < FK_KMAX; ++k) {
                if (k == K) break;
                const float4* wk = reinterpret_cast<const float4*>(wsm + k * FG + f0);
#pragma unroll
                for (int j4 = 0; j4 < FK_FG / 4; ++j4) {
                    const float4 w4 = wk[j4];
#pragma unroll
                    for (int q = 0; q < FK_PPT; ++q) {
                        acc[q][4 * j4] = fmaf(w4.x, xv[q][k], acc[q][4 * j4]);
                        acc[q][4 * j4 + 1] = fmaf(w4.y, xv[q][k], acc[q][4 * j4 + 1]);
                        acc[q][4 * j4 + 2] = fmaf(w4.z, xv[q][k], acc[q][4 * j4 + 2]);
                        acc[q][4 * j4 + 3] = fmaf(w4.w, xv[q][k], acc[q][4 * j4 + 3]);
                    }
                }
            }
            const int nf = min(FK_FG, p.F - f0);
            const bool leaky = p.act == TB_ACT_LEAKY;
#pragma unroll
            for (int q = 0; q < FK_PPT; ++q) {
                float o[FK_FG];
#pragma unroll
                for (int j = 0; j < FK_FG; ++j) {
                    float v = __fadd_rn(acc[q][j], bsm[f0 + j]);  // forwardBias, then the activation
                    if (leaky && v < 0.f) v = __fmul_rn(v, 0.1f);
                    o[j] = FMT == 0 ? v : FMT == 1 ? tb_tf32_rna(v) : tb_pair_encode(v);
                }
                const int wox = ox0 + q * FK_THREADS + 32 * warp;  // this warp's first pixel
                if constexpr (NHWC) {
                    float* ws = stg + warp * 32 * FK_STG;
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < FK_FG; j += 4)
                        *reinterpret_cast<float4*>(ws + lane * FK_STG + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
                    __syncwarp();
                    // 32 pixels x nf filters: FK_FG / 4 lanes per pixel row
                    constexpr int LPR = FK_FG / 4, RPI = 32 / LPR;  // lanes per row, rows per instruction
                    const int nvalid = min(32, p.OW - wox);
                    float* yw = p.y + b * p.y_bs + ((long long)oy * p.OW + wox) * p.yps + f0;
#pragma unroll
                    for (int i = 0; i < 32 / RPI; ++i) {
                        const int px = i * RPI + lane / LPR, q4 = lane % LPR;
                        if (px < nvalid && 4 * q4 < nf)
                            *(reinterpret_cast<float4*>(yw + (long long)px * p.yps) + q4) =
                                *reinterpret_cast<const float4*>(ws + px * FK_STG + 4 * q4);  // the next layer reads it
                    }
                } else {
                    if (wox + lane < p.OW) {
                        float* yp = p.y + b * p.y_bs + (long long)oy * p.OW + wox + lane;
#pragma unroll
                        for (int j = 0; j < FK_FG; ++j)
                            if (j < nf) yp[(long long)(f0 + j) * OHW] = o[j];  // the next layer reads it
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


static int64_t first_smem(int64_t C, int64_t KH, int64_t KW, int64_t SY, int64_t SX, int64_t DY, int64_t DX, int64_t F,
                          bool nhwc) {
    const int64_t FG = round_up(F, FK_FG), cols = fk_cols((int)SX, (int)KW, (int)DX);
    const int64_t nrin = fk_rows((int)SY, (int)KH, (int)DY);
    return (C * KH * KW * FG + FG + round_up(C * nrin * cols, 4) + (nhwc ? 4 * 32 * FK_STG : 0)) * 4;
}

bool first_direct_supported(int64_t C, int64_t KH, int64_t KW, int64_t SY, int64_t SX, int64_t DY, int64_t DX, int64_t F,
                            bool nhwc) {
    return C * KH * KW <= FK_KMAX && F <= FK_FMAX && F > 0 && SX <= 4 && SY <= 4 && DX * (KW - 1) <= 64 &&
           DY * (KH - 1) <= 64 && first_smem(C, KH, KW, SY, SX, DY, DX, F, nhwc) <= 96 * 1024;
}

int first_direct_launch(tb_ctx* ctx, const FirstGeom& g, const float* x, int64_t x_bs, const float* w, int64_t wstride,
                        const float* bias, int64_t F, int act, float* y, int64_t y_bs, int64_t yps, int fmt) {
    const bool nhwc = yps > 0;
    if (!first_direct_supported(g.C, g.KH, g.KW, g.SY, g.SX, g.DY, g.DX, F, nhwc) || (act != TB_ACT_LEAKY && act != TB_ACT_LINEAR) ||
        (nhwc && (F % 4 || yps % 4 || !aligned16(y))) || wstride < F)
        return fail(TB_ERR_UNSUPPORTED, "first-layer direct conv: unsupported geometry");
    FirstParams p{};
    p.x = x; p.x_bs = x_bs;
    p.C = (int)g.C; p.H = (int)g.H; p.W = (int)g.W; p.KH = (int)g.KH; p.KW = (int)g.KW;
    p.SY = (int)g.SY; p.SX = (int)g.SX; p.PY = (int)g.PY; p.PX = (int)g.PX; p.DY = (int)g.DY; p.DX = (int)g.DX;
    p.OH = (int)g.OH; p.OW = (int)g.OW;
    p.segs = (int)ceil_div(g.OW, FK_SEG);
    p.row_blocks = (int)ceil_div(g.OH, FK_ROWS);
    p.w = w; p.wstride = (int)wstride; p.bias = bias; p.F = (int)F; p.act = act;
    p.y = y; p.y_bs = y_bs; p.yps = (int)yps; p.fmt = fmt;
    const int64_t blocks = g.B * p.row_blocks * p.segs;
    if (blocks == 0) return TB_OK;
    if (blocks >= ((int64_t)1 << 31) || g.B * g.C * g.H * g.W >= ((int64_t)1 << 40))
        return fail(TB_ERR_UNSUPPORTED, "first-layer direct conv: too many blocks");
    const int64_t smem = first_smem(g.C, g.KH, g.KW, g.SY, g.SX, g.DY, g.DX, F, nhwc);
    if (nhwc != (fmt != 0)) return fail(TB_ERR_UNSUPPORTED, "first-layer direct conv: NHWC goes with TF32 / pair outputs");
    const bool unit = g.SY == 1 && g.SX == 1 && g.DY == 1 && g.DX == 1;  // the compile-time windows' stride
    const int win = !unit ? 0 : g.C == 3 && g.KH == 3 && g.KW == 3 ? 27 : g.C == 1 && g.KH == 5 && g.KW == 5 ? 25 : 0;
    using Kern = void (*)(const FirstParams);
    static const Kern kerns[3][3] = {
        {k_first_direct<27, 0>, k_first_direct<27, 1>, k_first_direct<27, 2>},
        {k_first_direct<25, 0>, k_first_direct<25, 1>, k_first_direct<25, 2>},
        {k_first_direct<0, 0>, k_first_direct<0, 1>, k_first_direct<0, 2>}};
    const Kern kern = kerns[win == 27 ? 0 : win == 25 ? 1 : 2][fmt];
    static std::mutex mu;
    static bool done[64] = {false};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device >= 64 || !done[ctx->device]) {
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j)
                    TB_CHECK_CUDA(cudaFuncSetAttribute(kerns[i][j], cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
            if (ctx->device < 64) done[ctx->device] = true;
        }
    }
    return launch(ctx, "k_first_direct", kern, dim3((unsigned)blocks), dim3(FK_THREADS), (size_t)smem, p);
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
    // bias + leaky / linear (the common first layer): the first-layer kernel, same arithmetic
    if (!bn_mean && (act == TB_ACT_LEAKY || act == TB_ACT_LINEAR) &&
        first_direct_supported(g.C, g.KH, g.KW, g.SY, g.SX, g.DY, g.DX, g.F, false) && !getenv("TB_DIRECT_OLD")) {
        const FirstGeom fg{g.B, g.C, g.H, g.W, g.KH, g.KW, g.SY, g.SX, g.PY, g.PX, g.DY, g.DX, g.OH, g.OW};
        const int r = first_direct_launch(ctx, fg, x, g.x_bs, wp, g.Mpad, bias, g.F, act, y, g.y_bs, 0, 0);
        if (r == TB_OK && launches) ++*launches;
        return r;
    }
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
