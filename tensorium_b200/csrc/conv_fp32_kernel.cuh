// conv_fp32_kernel.cuh -- FP32 CUDA-core implicit-GEMM convolution kernel template.
//
// Replaces the reference's GPU conv sequence (source/nConvolutionLayer.pas:1055-1122:
// per-image cuda.im2col, cublasSgemmStridedBatched, forwardBias / normalize+forwardScale,
// ActivateArray) and its CPU path (TTensor.Conv2D, source/ntensors.pas:8252-8349) by one
// kernel per layer:
//   * CTA tile BM x BN of (filters x pixels-over-the-batch), BK = 16 deep k tiles;
//   * a STAGES-deep cp.async ring in shared memory: the weight tile arrives as 16-byte
//     copies of the packed K-major weights, the activation tile is gathered straight from
//     NCHW X (zero-fill for padding), 16-byte copies for 1x1 stride-1 layers;
//   * each thread owns a TM x TN register tile (two TM/2 x TN/2 quads, BM/2 and BN/2 apart,
//     so every shared-memory read is a broadcast or a conflict-free float4);
//   * epilogue: bias or unfused batchnorm, activation, optional residual (shortcut) add,
//     optional YOLO logistic, float4 stores into NCHW Y at any batch stride (route slices);
//   * split-K over blockIdx.z when the tile grid is smaller than the machine; partial sums go
//     to a workspace and conv_splitk_reduce sums them in split order and runs the epilogue.
#pragma once
#include "conv.cuh"

#include <mutex>

namespace tbi {

__device__ __forceinline__ void cp_async4(float* smem, const float* gmem, bool pred) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    int sz = pred ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}

__device__ __forceinline__ void cp_async16(float* smem, const float* gmem, bool pred) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    int sz = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Output column quad n = nb .. nb+3 decoded once per thread: image b and pixel pix of nb.
struct ColQuad {
    int b, pix, nvalid;  // nvalid = how many of the 4 columns exist (0..4)
};

__device__ __forceinline__ ColQuad decode_quad(const ConvParams& p, long long nb) {
    ColQuad q;
    long long rem = p.Ntot - nb;
    q.nvalid = rem <= 0 ? 0 : (rem >= 4 ? 4 : (int)rem);
    if (q.nvalid == 0) { q.b = 0; q.pix = 0; return q; }
    unsigned n = (unsigned)nb;  // Ntot < 2^31 (checked on the host)
    q.b = (int)(n / (unsigned)p.OHW);
    q.pix = (int)(n - (unsigned)q.b * (unsigned)p.OHW);
    return q;
}

// Store the 4 outputs of column quad q in row m after the epilogue.
__device__ __forceinline__ void conv_store4(const ConvParams& p, int m, const ColQuad& q, const float* v,
                                            bool simple, bool has_bias, bool leaky, float bm) {
    if (q.nvalid == 0) return;
    if (p.vec_out && q.nvalid == 4) {  // OHW % 4 == 0: the quad lies in one image, 16-byte aligned
        float4 o;
        o.x = conv_epi_value(v[0], m, p, simple, has_bias, leaky, bm);
        o.y = conv_epi_value(v[1], m, p, simple, has_bias, leaky, bm);
        o.z = conv_epi_value(v[2], m, p, simple, has_bias, leaky, bm);
        o.w = conv_epi_value(v[3], m, p, simple, has_bias, leaky, bm);
        const long long off = (long long)m * p.OHW + q.pix;
        if (p.res) {
            float4 r = *reinterpret_cast<const float4*>(p.res + q.b * p.r_bs + off);
            o.x = __fadd_rn(o.x, r.x);
            o.y = __fadd_rn(o.y, r.y);
            o.z = __fadd_rn(o.z, r.z);
            o.w = __fadd_rn(o.w, r.w);
        }
        *reinterpret_cast<float4*>(p.y + q.b * p.y_bs + off) = o;
        return;
    }
    int b = q.b, pix = q.pix;
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // constant trip count: v (the accumulators) stays in registers
        if (k < q.nvalid) {
            while (pix >= p.OHW) { pix -= p.OHW; ++b; }
            const long long off = (long long)m * p.OHW + pix;
            float o = conv_epi_value(v[k], m, p, simple, has_bias, leaky, bm);
            if (p.res) o = __fadd_rn(o, p.res[b * p.r_bs + off]);
            p.y[b * p.y_bs + off] = o;
            ++pix;
        }
    }
}

template <int V>
struct VecT;
template <>
struct VecT<2> { typedef float2 T; };
template <>
struct VecT<4> { typedef float4 T; };

inline int conv_smem_bytes(int BM, int BN, int STAGES, int mode, int BK = CONV_BK) {
    return STAGES * BK * (BM + BN) * 4 + (mode == MODE_CRS ? CONV_CRS_MAX_K * 16 : 0);
}

template <int BM, int BN, int TM, int TN, int STAGES, int MODE, int BK = CONV_BK>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
conv_fp32_kernel(const ConvParams p) {
    constexpr int NT = (BM / TM) * (BN / TN);
    constexpr int TX = BN / TN;
    constexpr int TM2 = TM / 2, TN2 = TN / 2;
    static_assert(TN == 8, "epilogue stores quads of 4 columns");
    static_assert(TM == 4 || TM == 8, "TM must be 4 or 8");
    extern __shared__ __align__(16) float smem[];
    float* As = smem;                     // [STAGES][BK][BM]
    float* Bs = smem + STAGES * BK * BM;  // [STAGES][BK][BN]
    int4* ktab = reinterpret_cast<int4*>(Bs + STAGES * BK * BN);  // CRS k table

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const int m0 = blockIdx.y * BM;
    const long long n0 = (long long)blockIdx.x * BN;
    const int kt_begin = blockIdx.z * p.kt_per_split;
    const int kt_end = min(kt_begin + p.kt_per_split, p.ktiles);
    const int nkt = kt_end - kt_begin;
    const long long HW = (long long)p.H * p.W;

    if (MODE == MODE_CRS) {
        const int khw = p.KH * p.KW;
        for (int k = tid; k < p.Kpad; k += NT) {
            int c = k / khw, rs = k - c * khw, r = rs / p.KW, s = rs - r * p.KW;
            int dr = r * p.DY, ds = s * p.DX;
            ktab[k] = make_int4(c * (int)HW + dr * p.W + ds, dr, ds, c < p.C ? 1 : 0);
        }
        __syncthreads();
    }

    // ---- per-thread setup of the activation (B) gather ----
    constexpr int BCOLS = (MODE == MODE_1X1V) ? BN / 4 : BN;
    static_assert(NT % BCOLS == 0, "threads must cover the B tile columns");
    constexpr int KSTEP = NT / BCOLS;
    static_assert(BK % KSTEP == 0, "k rows per thread must be integral");
    constexpr int BEPT = BK / KSTEP;
    const int bcol = tid % BCOLS;
    const int krow0 = tid / BCOLS;
    const long long ncol = n0 + (MODE == MODE_1X1V ? 4 * bcol : bcol);
    const bool nvalid = ncol < p.Ntot;
    long long bimg = 0;
    int pix = 0, iy0 = 0, ix0 = 0;
    if (nvalid) {
        bimg = ncol / p.OHW;
        pix = (int)(ncol - bimg * p.OHW);
        int oy = pix / p.OW, ox = pix - oy * p.OW;
        iy0 = oy * p.SY - p.PY;
        ix0 = ox * p.SX - p.PX;
    }
    const float* xb = p.x + bimg * p.x_bs;

    // Loader state: k tiles are loaded in increasing order from kt_begin, so the weight pointer,
    // the tap (r, s) and the channel offset advance incrementally (no divisions per tile).
    constexpr int AITER = (BK * BM / 4 + NT - 1) / NT;
    static_assert(NT % (BM / 4) == 0, "a weight row of the tile is whole 16-byte copies");
    constexpr int AKSTEP = NT / (BM / 4);  // weight rows between a thread's copies
    const int a_kl0 = tid / (BM / 4), a_mq = tid - a_kl0 * (BM / 4);
    const bool a_ok = m0 + a_mq * 4 < p.Mpad;
    const int a_off = a_kl0 * p.Mpad + m0 + a_mq * 4;
    const float* wnext = p.w + (long long)kt_begin * BK * p.Mpad;
    int ld_c0 = 0, ld_s = 0, ld_iy = 0, ld_ix = 0;  // channel, kernel column, input row / column
    bool ld_okp = false;
    const float* ld_base = p.x;  // x at (ld_iy, ld_ix), channel krow0
    auto ld_tap = [&]() {
        ld_okp = nvalid && (unsigned)ld_iy < (unsigned)p.H && (unsigned)ld_ix < (unsigned)p.W;
        ld_base = xb + (ld_okp ? (long long)ld_iy * p.W + ld_ix : 0) + (long long)krow0 * HW;
    };
    if (MODE == MODE_RSC) {
        const int k0 = kt_begin * BK;
        const int rs = k0 / p.Cpad;
        ld_c0 = k0 - rs * p.Cpad;
        const int r = rs / p.KW;
        ld_s = rs - r * p.KW;
        ld_iy = iy0 + r * p.DY;
        ld_ix = ix0 + ld_s * p.DX;
        ld_tap();
    } else if (MODE == MODE_1X1V) {
        ld_c0 = kt_begin * BK;
    }

    auto load_tile = [&](int kt, int st) {
        // weights: BK rows of BM floats, 16-byte copies
        float* as = As + st * BK * BM;
#pragma unroll
        for (int i = 0; i < AITER; ++i) {
            const int kl = a_kl0 + i * AKSTEP;
            if (kl < BK)
                cp_async16(as + kl * BM + a_mq * 4, a_ok ? wnext + a_off + i * AKSTEP * p.Mpad : p.w, a_ok);
        }
        wnext += BK * p.Mpad;
        float* bs = Bs + st * BK * BN;
        if (MODE == MODE_CRS) {
#pragma unroll
            for (int e = 0; e < BEPT; ++e) {
                int kl = krow0 + e * KSTEP;
                int4 t = ktab[kt * BK + kl];
                int iy = iy0 + t.y, ix = ix0 + t.z;
                bool ok = nvalid && t.w && (unsigned)iy < (unsigned)p.H && (unsigned)ix < (unsigned)p.W;
                const float* src = ok ? xb + t.x + (long long)iy0 * p.W + ix0 : p.x;
                cp_async4(bs + kl * BN + bcol, src, ok);
            }
        } else if (MODE == MODE_RSC) {
            const float* cb = ld_base + (long long)ld_c0 * HW;
#pragma unroll
            for (int e = 0; e < BEPT; ++e) {
                const int kl = krow0 + e * KSTEP;
                const bool ok = ld_okp && ld_c0 + kl < p.C;
                cp_async4(bs + kl * BN + bcol, ok ? cb + (long long)e * KSTEP * HW : p.x, ok);
            }
            ld_c0 += BK;
            if (ld_c0 == p.Cpad) {
                ld_c0 = 0;
                ld_ix += p.DX;
                if (++ld_s == p.KW) ld_s = 0, ld_ix = ix0, ld_iy += p.DY;
                ld_tap();
            }
        } else {
            const float* cb = xb + pix + (long long)(ld_c0 + krow0) * HW;
#pragma unroll
            for (int e = 0; e < BEPT; ++e) {
                const int kl = krow0 + e * KSTEP;
                const bool ok = nvalid && ld_c0 + kl < p.C;
                cp_async16(bs + kl * BN + 4 * bcol, ok ? cb + (long long)e * KSTEP * HW : p.x, ok);
            }
            ld_c0 += BK;
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nkt) load_tile(kt_begin + s, s);
        cp_async_commit();
    }

    typedef typename VecT<TM2>::T AV;
    for (int t = 0; t < nkt; ++t) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        {
            int tn = t + STAGES - 1;
            if (tn < nkt) load_tile(kt_begin + tn, tn % STAGES);
            cp_async_commit();
        }
        const float* as = As + (t % STAGES) * BK * BM;
        const float* bs = Bs + (t % STAGES) * BK * BN;
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[TM], bv[TN];
            *reinterpret_cast<AV*>(&a[0]) = *reinterpret_cast<const AV*>(as + kk * BM + ty * TM2);
            *reinterpret_cast<AV*>(&a[TM2]) = *reinterpret_cast<const AV*>(as + kk * BM + BM / 2 + ty * TM2);
            *reinterpret_cast<float4*>(&bv[0]) = *reinterpret_cast<const float4*>(bs + kk * BN + tx * TN2);
            *reinterpret_cast<float4*>(&bv[TN2]) = *reinterpret_cast<const float4*>(bs + kk * BN + BN / 2 + tx * TN2);
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
        }
    }
    cp_async_wait<0>();

    // ---- epilogue ----
    const ColQuad cq[2] = {decode_quad(p, n0 + tx * TN2), decode_quad(p, n0 + BN / 2 + tx * TN2)};
    const bool simple = !p.bn_mean && p.yolo_classes == 0 && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
    const bool has_bias = p.bias != nullptr, leaky = p.act == TB_ACT_LEAKY;
    const float* __restrict__ biasp = p.bias;
    if (p.splits > 1) {
        // split-K: publish this split's partial tile, then the last CTA to arrive on the tile
        // sums all partials in split order 0..S-1 (deterministic, whatever the arrival order)
        // and runs the epilogue.  No CTA waits for another.
        const long long plane = (long long)p.F * p.Ntot;
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            int m = m0 + (i < TM2 ? ty * TM2 + i : BM / 2 + ty * TM2 + (i - TM2));
            if (m >= p.F) continue;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                long long nb = n0 + g * (BN / 2) + tx * TN2;
                if (nb >= p.Ntot) continue;
                const float* v = &acc[i][g * 4];
                float* dst = p.ws + blockIdx.z * plane + (long long)m * p.Ntot + nb;
                if ((p.Ntot & 3) == 0) {
                    __stcg(reinterpret_cast<float4*>(dst), make_float4(v[0], v[1], v[2], v[3]));
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if (nb + q < p.Ntot) __stcg(dst + q, v[q]);
                }
            }
        }
        __threadfence();
        __syncthreads();
        __shared__ int s_last;
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        if (tid == 0) {
            int prev = atomicAdd(&p.tile_cnt[tile], 1);
            s_last = (prev == p.splits - 1);
            if (s_last) p.tile_cnt[tile] = 0;  // ready for the next launch
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            int m = m0 + (i < TM2 ? ty * TM2 + i : BM / 2 + ty * TM2 + (i - TM2));
            if (m >= p.F) continue;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                long long nb = n0 + g * (BN / 2) + tx * TN2;
                if (nb >= p.Ntot) continue;
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                const float* src = p.ws + (long long)m * p.Ntot + nb;
                for (int z = 0; z < p.splits; ++z) {
                    if ((p.Ntot & 3) == 0) {
                        float4 t = __ldcg(reinterpret_cast<const float4*>(src + z * plane));
                        v[0] = __fadd_rn(v[0], t.x);
                        v[1] = __fadd_rn(v[1], t.y);
                        v[2] = __fadd_rn(v[2], t.z);
                        v[3] = __fadd_rn(v[3], t.w);
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            if (nb + q < p.Ntot) v[q] = __fadd_rn(v[q], __ldcg(src + z * plane + q));
                    }
                }
                conv_store4(p, m, cq[g], v, simple, has_bias, leaky, has_bias ? __ldg(biasp + m) : 0.f);
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        int m = m0 + (i < TM2 ? ty * TM2 + i : BM / 2 + ty * TM2 + (i - TM2));
        if (m >= p.F) continue;
        const float bm = has_bias ? __ldg(biasp + m) : 0.f;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            long long nb = n0 + g * (BN / 2) + tx * TN2;
            if (nb >= p.Ntot) continue;
            conv_store4(p, m, cq[g], &acc[i][g * 4], simple, has_bias, leaky, bm);
        }
    }
}

// CTAs of this configuration resident per SM (registers / shared memory), cached per device
template <int BM, int BN, int TM, int TN, int STAGES, int MODE, int BK = CONV_BK>
int conv_ctas_per_sm(tb_ctx* ctx) {
    static int cache[64] = {0};
    if (ctx->device < 64 && cache[ctx->device]) return cache[ctx->device];
    constexpr int NT = (BM / TM) * (BN / TN);
    const int smem = conv_smem_bytes(BM, BN, STAGES, MODE, BK);
    auto kern = conv_fp32_kernel<BM, BN, TM, TN, STAGES, MODE, BK>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int n = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, NT, smem) != cudaSuccess || n < 1) n = 1;
    if (ctx->device < 64) cache[ctx->device] = n;
    return n;
}

template <int BM, int BN, int TM, int TN, int STAGES, int MODE, int BK = CONV_BK>
int conv_launch_cfg(tb_ctx* ctx, const ConvParams& p, dim3 grid) {
    constexpr int NT = (BM / TM) * (BN / TN);
    const int smem = conv_smem_bytes(BM, BN, STAGES, MODE, BK);
    static std::mutex mu;
    static bool done[64] = {false};
    auto kern = conv_fp32_kernel<BM, BN, TM, TN, STAGES, MODE, BK>;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !done[ctx->device]) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(conv)");
            done[ctx->device] = true;
        }
    }
    kern<<<grid, NT, smem, ctx->stream>>>(p);
    return check_launch("conv_fp32_kernel");
}

template <int BM, int BN, int TM, int TN, int STAGES, int BK = CONV_BK>
int conv_occupancy_modes(tb_ctx* ctx, int mode) {
    switch (mode) {
    case MODE_CRS: return conv_ctas_per_sm<BM, BN, TM, TN, STAGES, MODE_CRS, CONV_BK>(ctx);
    case MODE_RSC: return conv_ctas_per_sm<BM, BN, TM, TN, STAGES, MODE_RSC, BK>(ctx);
    default: return conv_ctas_per_sm<BM, BN, TM, TN, STAGES, MODE_1X1V, BK>(ctx);
    }
}

// MODE_CRS (the small-channel first layer) always runs 16-deep k tiles: its K is padded to 16.
template <int BM, int BN, int TM, int TN, int STAGES, int BK = CONV_BK>
int conv_launch_modes(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode) {
    switch (mode) {
    case MODE_CRS: return conv_launch_cfg<BM, BN, TM, TN, STAGES, MODE_CRS, CONV_BK>(ctx, p, grid);
    case MODE_RSC: return conv_launch_cfg<BM, BN, TM, TN, STAGES, MODE_RSC, BK>(ctx, p, grid);
    default: return conv_launch_cfg<BM, BN, TM, TN, STAGES, MODE_1X1V, BK>(ctx, p, grid);
    }
}

// one entry per tile configuration, each compiled in its own translation unit;
// launch (grid.x > 0) or, with grid.x == 0, return the resident CTAs per SM
int conv_launch_128x128(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode);
int conv_launch_64x128(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode);
int conv_launch_64x64(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode);
int conv_launch_32x256(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode);

}  // namespace tbi
