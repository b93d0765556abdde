// compat.cu -- TNNCuda method shims (tbcompat_*) and the unfused batchnorm layer (tb_bn_fwd).
//
// The reference's layers call the methods of one global TNNCuda<single> object (source/
// nncuda.pas:35-158).  Each tbcompat_* function below has that method's argument list, in the
// same order and meaning (SizeInt -> int64_t, single -> float, boolean / longint / integer ->
// int32_t, TCUMem -> device pointer), preceded by the context that stands in for the object, so
// a Pascal TNNCuda replacement forwards every method with a one-line call.  Results follow the
// reference's CPU path (the parity target of this library), which its GPU kernels only
// approximate: the GEMMs keep the CPU routines' summation orders (s_nn / s_tn: C = beta*C, then
// one FMA of (alpha*a) per k in ascending order; s_nt: sdot_avx2's eight lanes; s_tt: a
// sequential sum of (alpha*a)*b), elementwise arithmetic is separately rounded, normalize
// divides by max(sqrt(var), 1e-6) as blockNormalize does.  Training-only methods (backward
// passes, upSample with isForward = 0) return TB_ERR_UNSUPPORTED.
#include "conv.cuh"

namespace tbi {
namespace {

enum { G_NN = 0, G_NT = 1, G_TN = 2, G_TT = 3 };

// One thread per C element, 16 x 16 outputs per block, 32-deep k chunks staged in shared memory.
template <int MODE>
__global__ void __launch_bounds__(256) k_compat_gemm(int64_t M, int64_t N, int64_t K, float alpha,
                                                      const float* __restrict__ A, int64_t lda, int64_t sA,
                                                      const float* __restrict__ B, int64_t ldb, int64_t sB,
                                                      float beta, float* __restrict__ Cm, int64_t ldc, int64_t sC) {
    __shared__ float As[16][33];  // As[i][k] = op(A)(i, k)
    __shared__ float Bs[32][17];  // Bs[k][j] = op(B)(k, j)
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t z = blockIdx.z;
    A += z * sA;
    B += z * sB;
    Cm += z * sC;
    const int64_t i0 = (int64_t)blockIdx.y * 16, j0 = (int64_t)blockIdx.x * 16;
    const int64_t i = i0 + ty, j = j0 + tx;
    float acc = 0.f, lane[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float c0 = 0.f;
    if (i < M && j < N) {
        c0 = Cm[i * ldc + j];
        if (beta != 1.0f) c0 = __fmul_rn(c0, beta);  // mulvs before the products
    }
    acc = c0;
    for (int64_t k0 = 0; k0 < K; k0 += 32) {
        for (int e = threadIdx.x; e < 16 * 32; e += 256) {
            const int r = e / 32, kk = e % 32;
            const int64_t gi = i0 + r, gk = k0 + kk;
            float v = 0.f;
            if (gi < M && gk < K) v = (MODE == G_NN || MODE == G_NT) ? A[gi * lda + gk] : A[gk * lda + gi];
            As[r][kk] = v;
        }
        for (int e = threadIdx.x; e < 32 * 16; e += 256) {
            const int kk = e / 16, cidx = e % 16;
            const int64_t gk = k0 + kk, gj = j0 + cidx;
            float v = 0.f;
            if (gk < K && gj < N) v = (MODE == G_NN || MODE == G_TN) ? B[gk * ldb + gj] : B[gj * ldb + gk];
            Bs[kk][cidx] = v;
        }
        __syncthreads();
        const int kn = (int)(K - k0 < 32 ? K - k0 : 32);
        if (MODE == G_NN || MODE == G_TN) {
            for (int kk = 0; kk < kn; ++kk) acc = fmaf(__fmul_rn(alpha, As[ty][kk]), Bs[kk][tx], acc);
        } else if (MODE == G_NT) {
            for (int kk = 0; kk < kn; ++kk) lane[kk & 7] = fmaf(As[ty][kk], Bs[kk][tx], lane[kk & 7]);
        } else {
            for (int kk = 0; kk < kn; ++kk) lane[0] = __fadd_rn(lane[0], __fmul_rn(__fmul_rn(alpha, As[ty][kk]), Bs[kk][tx]));
        }
        __syncthreads();
    }
    if (i >= M || j >= N) return;
    float out = acc;
    if (MODE == G_NT) {  // sdot_avx2 reduction, then C + alpha*sdot
        float t[4];
#pragma unroll
        for (int l = 0; l < 4; ++l) t[l] = __fadd_rn(lane[l], lane[l + 4]);
        const float s = __fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3]));
        out = __fadd_rn(c0, __fmul_rn(alpha, s));
    } else if (MODE == G_TT) {
        out = __fadd_rn(c0, lane[0]);
    }
    Cm[i * ldc + j] = out;
}

// col[(c*kh + r)*kw + s][oy*ow + ox] = im[c][oy*sy - ph + r*dy][ox*sx - pw + s*dx], 0 outside.
__global__ void k_im2col(int64_t C, int64_t H, int64_t W, int KH, int KW, int PH, int PW, int SY, int SX, int DY,
                         int DX, int64_t OH, int64_t OW, const float* __restrict__ im, float* __restrict__ col) {
    const int64_t total = C * KH * KW * OH * OW;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ox = e % OW, t1 = e / OW, oy = t1 % OH, row = t1 / OH;
        const int s = (int)(row % KW), r = (int)((row / KW) % KH);
        const int64_t c = row / ((int64_t)KW * KH);
        const int64_t iy = oy * SY - PH + (int64_t)r * DY, ix = ox * SX - PW + (int64_t)s * DX;
        col[e] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? im[(c * H + iy) * W + ix] : 0.f;
    }
}

// op: 0 forwardScale (x *= s[f]), 1 forwardScaleAdd (x = x*s[f] + b[f]), f = (i / block) % size.
__global__ void k_channel_affine(int64_t n, int64_t size, int64_t block, float* __restrict__ x,
                                 const float* __restrict__ s, const float* __restrict__ b, int64_t inc, int op) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t f = (i / block) % size;
        float v = __fmul_rn(x[i], s[f * inc]);
        if (op == 1) v = __fadd_rn(v, b[f * inc]);
        x[i] = v;
    }
}

// TNNCuda.normalize / blockNormalize: dst[g][i][j] = (dst - mean[i*ms]) / max(sqrt(var[i*vs]), 1e-6)
__global__ void k_normalize(int64_t n, int64_t size, int64_t block, const float* __restrict__ mean, int64_t ms,
                            const float* __restrict__ var, int64_t vs, float* __restrict__ dst) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = (e / block) % size;
        const float d = fmaxf((float)sqrt((double)var[i * vs]), 0.000001f);
        dst[e] = __fdiv_rn(__fsub_rn(dst[e], mean[i * ms]), d);
    }
}

// TBaseLayer.batchNorm inference (source/nbaselayer.pas:336-370): normalize, forwardScale,
// forwardBias as three separate roundings, over [batch][channels][spatial].
__global__ void k_bn(int64_t n, int64_t channels, int64_t spatial, const float* __restrict__ x,
                     const float* __restrict__ mean, const float* __restrict__ var, const float* __restrict__ scale,
                     const float* __restrict__ bias, float* __restrict__ y) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = (e / spatial) % channels;
        y[e] = conv_bn(x[e], mean[c], var[c], scale ? scale[c] : 1.0f, bias ? bias[c] : 0.0f);
    }
}

// softmaxBatch with the reference's strided group layout (source/cuda_sgemm.cu:934-952), each
// group in the CPU softmax order (max, exp((x - max)/temp) summed in order, divide).
__global__ void k_softmax_strided(int64_t n, int64_t batch, int64_t batch_size, int64_t groups, int64_t group_size,
                                  int64_t stride, float temp, const float* __restrict__ in, float* __restrict__ out) {
    const int64_t total = batch * groups;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = t / groups, g = t % groups;
        const float* x = in + b * batch_size + g * group_size;
        float* y = out + b * batch_size + g * group_size;
        if (n <= 0) continue;
        float largest = x[0];
        for (int64_t i = 1; i < n; ++i)
            if (x[i * stride] > largest) largest = x[i * stride];
        float sum = 0.0f;
        for (int64_t i = 0; i < n; ++i) {
            const float e = (float)exp((double)__fdiv_rn(__fsub_rn(x[i * stride], largest), temp));
            sum = __fadd_rn(sum, e);
            y[i * stride] = e;
        }
        for (int64_t i = 0; i < n; ++i) y[i * stride] = __fdiv_rn(y[i * stride], sum);
    }
}

int gemm_launch(tb_ctx* ctx, int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
                int64_t lda, int64_t sA, const float* B, int64_t ldb, int64_t sB, float beta, float* Cm, int64_t ldc,
                int64_t sC, int64_t batch) {
    if (M < 0 || N < 0 || K < 0 || batch < 0) return fail(TB_ERR_INVALID, "gemm: negative size");
    if (M == 0 || N == 0 || batch == 0) return TB_OK;
    if (!A || !B || !Cm) return fail(TB_ERR_INVALID, "gemm: null matrix");
    const int64_t ka = transA ? M : K, kb = transB ? K : N;
    if (lda < std::max<int64_t>(ka, 1) || ldb < std::max<int64_t>(kb, 1) || ldc < N)
        return fail(TB_ERR_INVALID, "gemm: leading dimension too small (lda %lld, ldb %lld, ldc %lld)",
                    (long long)lda, (long long)ldb, (long long)ldc);
    dim3 grid((unsigned)ceil_div(N, 16), (unsigned)ceil_div(M, 16), (unsigned)batch);
    if (grid.y > 65535 || grid.z > 65535) return fail(TB_ERR_INVALID, "gemm: too many rows or batches");
    const int mode = (transA ? 2 : 0) + (transB ? 1 : 0);
    switch (mode) {
    case G_NN: k_compat_gemm<G_NN><<<grid, 256, 0, ctx->stream>>>(M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, Cm, ldc, sC); break;
    case G_NT: k_compat_gemm<G_NT><<<grid, 256, 0, ctx->stream>>>(M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, Cm, ldc, sC); break;
    case G_TN: k_compat_gemm<G_TN><<<grid, 256, 0, ctx->stream>>>(M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, Cm, ldc, sC); break;
    default: k_compat_gemm<G_TT><<<grid, 256, 0, ctx->stream>>>(M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, Cm, ldc, sC); break;
    }
    return check_launch("k_compat_gemm");
}

}  // namespace
}  // namespace tbi

using namespace tbi;

extern "C" {

int tbcompat_createDeviceBuffer(tb_ctx* ctx, int64_t N, void** mem) { return tb_malloc(ctx, N, mem); }
int tbcompat_freeDeviceBuffer(tb_ctx* ctx, void* mem) { return tb_free(ctx, mem); }
int tbcompat_readBuffer(tb_ctx* ctx, const void* mem, int64_t bufferSize, void* buffer) {
    return tb_memcpy_d2h(ctx, buffer, mem, bufferSize);
}
int tbcompat_writeBuffer(tb_ctx* ctx, void* mem, int64_t bufferSize, const void* buffer) {
    int r = tb_memcpy_h2d(ctx, mem, buffer, bufferSize);
    return r != TB_OK ? r : tb_sync(ctx);  // writeBuffer is a blocking cudaMemcpy in the reference
}
int tbcompat_finish(tb_ctx* ctx) { return tb_sync(ctx); }

int tbcompat_ActivateArray(tb_ctx* ctx, int64_t N, float* x, int64_t offset, int32_t activation) {
    return tb_activate(ctx, N, x, offset, activation);
}

int tbcompat_forwardBias(tb_ctx* ctx, int64_t dstSize, float* dst, int64_t offset, int64_t srcSize, const float* src,
                         int64_t incb, int64_t batch) {
    return tb_forward_bias(ctx, dstSize, dst, offset, srcSize, src, incb, batch);
}

int tbcompat_forwardScale(tb_ctx* ctx, int64_t dstSize, float* dst, int64_t offset, int64_t scaleSize,
                          const float* scale, int64_t incb, int64_t batch) {
    TB_ENTER(ctx);
    if (dstSize < 0 || scaleSize <= 0 || batch <= 0 || dstSize % (scaleSize * batch))
        return fail(TB_ERR_INVALID, "forwardScale: dstSize must be a multiple of scaleSize*batch");
    if (dstSize == 0) return TB_OK;
    if (!dst || !scale) return fail(TB_ERR_INVALID, "forwardScale: null pointer");
    k_channel_affine<<<grid_for(dstSize, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
        dstSize, scaleSize, dstSize / (scaleSize * batch), dst + offset, scale, nullptr, incb > 0 ? incb : 1, 0);
    return check_launch("k_channel_affine");
}

int tbcompat_forwardScaleAdd(tb_ctx* ctx, int64_t dstSize, float* dst, int64_t offset, int64_t scaleSize,
                             const float* scales, const float* biases, int64_t incb, int64_t batch) {
    TB_ENTER(ctx);
    if (dstSize < 0 || scaleSize <= 0 || batch <= 0 || dstSize % (scaleSize * batch))
        return fail(TB_ERR_INVALID, "forwardScaleAdd: dstSize must be a multiple of scaleSize*batch");
    if (dstSize == 0) return TB_OK;
    if (!dst || !scales || !biases) return fail(TB_ERR_INVALID, "forwardScaleAdd: null pointer");
    k_channel_affine<<<grid_for(dstSize, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
        dstSize, scaleSize, dstSize / (scaleSize * batch), dst + offset, scales, biases, incb > 0 ? incb : 1, 1);
    return check_launch("k_channel_affine");
}

int tbcompat_normalize(tb_ctx* ctx, int64_t srcSize, int64_t dstSize, int64_t groups, const float* means,
                       int64_t meansStride, const float* vars, int64_t varsStride, float* dst, int64_t dstOffset) {
    TB_ENTER(ctx);
    if (srcSize <= 0 || groups <= 0 || dstSize < 0 || dstSize % (srcSize * groups))
        return fail(TB_ERR_INVALID, "normalize: dstSize must be a multiple of srcSize*groups");
    if (dstSize == 0) return TB_OK;
    if (!means || !vars || !dst) return fail(TB_ERR_INVALID, "normalize: null pointer");
    k_normalize<<<grid_for(dstSize, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
        dstSize, srcSize, dstSize / (srcSize * groups), means, meansStride, vars, varsStride, dst + dstOffset);
    return check_launch("k_normalize");
}

int tbcompat_gemm(tb_ctx* ctx, int32_t transA, int32_t transB, int64_t M, int64_t N, int64_t K, float ALPHA,
                  const float* A, int64_t aOffset, int64_t lda, const float* B, int64_t bOffset, int64_t ldb, float BETA,
                  float* C, int64_t cOffset, int64_t ldc) {
    TB_ENTER(ctx);
    return gemm_launch(ctx, transA, transB, M, N, K, ALPHA, A ? A + aOffset : A, lda, 0, B ? B + bOffset : B, ldb, 0,
                       BETA, C ? C + cOffset : C, ldc, 0, 1);
}

int tbcompat_gemmStridedBatched(tb_ctx* ctx, int32_t transA, int32_t transB, int64_t M, int64_t N, int64_t K,
                                float ALPHA, const float* A, int64_t aOffset, int64_t lda, int64_t strideA,
                                const float* B, int64_t bOffset, int64_t ldb, int64_t strideB, float BETA, float* C,
                                int64_t cOffset, int64_t ldc, int64_t strideC, int64_t batchCount) {
    TB_ENTER(ctx);
    return gemm_launch(ctx, transA, transB, M, N, K, ALPHA, A ? A + aOffset : A, lda, strideA, B ? B + bOffset : B,
                       ldb, strideB, BETA, C ? C + cOffset : C, ldc, strideC, batchCount);
}

int tbcompat_addvv(tb_ctx* ctx, int64_t N, const float* src1, int64_t src1Offset, int64_t inca, const float* src2,
                   int64_t src2Offset, int64_t incb, float* dst, int64_t dstOffset, int64_t incc) {
    return tb_addvv(ctx, N, src1, src1Offset, inca, src2, src2Offset, incb, dst, dstOffset, incc);
}

int tbcompat_fill(tb_ctx* ctx, int64_t N, float* x, int64_t offset, float val, int64_t stride) {
    return tb_fill(ctx, N, x, offset, val, stride);
}

int tbcompat_copy(tb_ctx* ctx, int64_t N, const float* src, int64_t srcOffset, int64_t inca, float* dst,
                  int64_t dstOffset, int64_t incb) {
    return tb_copy(ctx, N, src, srcOffset, inca, dst, dstOffset, incb);
}

int tbcompat_fmavss(tb_ctx* ctx, int64_t N, float* src, int64_t offset, float scalar, float bias, float* dst) {
    return tb_fmavss(ctx, N, src, offset, scalar, bias, dst);
}

int tbcompat_softmaxBatch(tb_ctx* ctx, int64_t N, const float* input, int64_t iOffset, int64_t batch,
                          int64_t batch_size, int64_t groups, int64_t group_size, int64_t stride, float temp,
                          float* output, int64_t oOffset) {
    TB_ENTER(ctx);
    if (N < 0 || batch < 0 || groups < 0 || stride <= 0) return fail(TB_ERR_INVALID, "softmaxBatch: bad sizes");
    if (N == 0 || batch == 0 || groups == 0) return TB_OK;
    if (!input || !output) return fail(TB_ERR_INVALID, "softmaxBatch: null pointer");
    const int64_t total = batch * groups;
    k_softmax_strided<<<grid_for(total, 128, ctx->sm_count), 128, 0, ctx->stream>>>(
        N, batch, batch_size, groups, group_size, stride, temp, input + iOffset, output + oOffset);
    return check_launch("k_softmax_strided");
}

int tbcompat_forwardMaxPool(tb_ctx* ctx, int64_t aBatch, int64_t outC, int64_t outH, int64_t outW, const float* input,
                            int64_t c, int64_t h, int64_t w, int64_t stride_x, int64_t stride_y, int64_t padding,
                            int64_t kernelSize, int64_t* indexes, float* output) {
    TB_ENTER(ctx);
    if (outC != c) return fail(TB_ERR_INVALID, "forwardMaxPool: outC (%lld) must equal c (%lld)", (long long)outC, (long long)c);
    if (stride_y <= 0 || stride_x <= 0 || kernelSize <= 0)
        return fail(TB_ERR_INVALID, "forwardMaxPool: bad window");
    if (outH != (h + padding - kernelSize) / stride_y + 1 || outW != (w + padding - kernelSize) / stride_x + 1)
        return fail(TB_ERR_INVALID, "forwardMaxPool: outH/outW do not follow (h + padding - size) div stride + 1");
    return tb_maxpool_fwd(ctx, aBatch, c, h, w, kernelSize, stride_x, stride_y, padding, input, output, indexes);
}

int tbcompat_im2col(tb_ctx* ctx, int64_t aChannels, int64_t aHeight, int64_t aWidth, int64_t kernelHeight,
                    int64_t kernelWidth, int64_t padHeight, int64_t padWidth, int64_t strideY, int64_t strideX,
                    int64_t dilationY, int64_t dilationX, const float* im, int64_t imOffset, float* col,
                    int64_t colOffset) {
    TB_ENTER(ctx);
    if (aChannels <= 0 || aHeight <= 0 || aWidth <= 0 || kernelHeight <= 0 || kernelWidth <= 0 || strideY <= 0 ||
        strideX <= 0 || dilationY <= 0 || dilationX <= 0 || padHeight < 0 || padWidth < 0)
        return fail(TB_ERR_INVALID, "im2col: bad geometry");
    if (!im || !col) return fail(TB_ERR_INVALID, "im2col: null pointer");
    // output size as TNNCuda.im2col (source/nncuda.pas:1144-1175): 1 when the window exceeds the padded input
    const int64_t sh = aHeight + 2 * padHeight, ph = dilationY * (kernelHeight - 1) + 1;
    const int64_t sw = aWidth + 2 * padWidth, pw = dilationX * (kernelWidth - 1) + 1;
    const int64_t OH = sh >= ph ? (sh - ph) / strideY + 1 : 1, OW = sw >= pw ? (sw - pw) / strideX + 1 : 1;
    const int64_t total = aChannels * kernelHeight * kernelWidth * OH * OW;
    k_im2col<<<grid_for(total, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
        aChannels, aHeight, aWidth, (int)kernelHeight, (int)kernelWidth, (int)padHeight, (int)padWidth, (int)strideY,
        (int)strideX, (int)dilationY, (int)dilationX, OH, OW, im + imOffset, col + colOffset);
    return check_launch("k_im2col");
}

int tbcompat_upSample(tb_ctx* ctx, int64_t aBatch, int64_t aChannels, int64_t outHeight, int64_t outWidth,
                      const float* in, int64_t stride, int32_t isForward, float scale, float* out, int32_t zeroIn) {
    (void)zeroIn;
    if (!isForward)
        return fail(TB_ERR_UNSUPPORTED, "upSample: the backward direction (isForward = 0) is training, not in this library");
    // the reference passes the input's height and width as outHeight / outWidth (its kernel
    // multiplies them by stride, source/nncuda.pas:1267-1286)
    return tb_upsample_fwd(ctx, aBatch, aChannels, outHeight, outWidth, stride, scale, in, out, 0);
}

int tb_bn_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t spatial, const float* x, const float* mean,
              const float* variance, const float* scales, const float* biases, float* y) {
    TB_ENTER(ctx);
    if (batch < 0 || channels <= 0 || spatial <= 0) return fail(TB_ERR_INVALID, "bn: bad shape");
    if (batch == 0) return TB_OK;
    if (!x || !mean || !variance || !y) return fail(TB_ERR_INVALID, "bn: null x, mean, variance or y");
    const int64_t n = batch * channels * spatial;
    k_bn<<<grid_for(n, 256, ctx->sm_count), 256, 0, ctx->stream>>>(n, channels, spatial, x, mean, variance, scales,
                                                                     biases, y);
    return check_launch("k_bn");
}

}  // extern "C"
