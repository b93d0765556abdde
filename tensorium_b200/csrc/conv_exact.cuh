// conv_exact.cuh -- the order-exact FP32 implicit-GEMM convolution (the default FP32 path).
//
// The reference's CPU conv (TTensor.Conv2D, source/ntensors.pas:8252-8349) is im2col followed by
// cblas_sgemm -> sgemm_nn -> s_nn -> saxpy_avx2 (source/ntensors.pas:2231-2286, 2061-2157,
// 1308-1435): every output starts at 0 and receives one fused multiply-add per k, k ascending
// in the im2col row order k = (c*kh + r)*kw + s.  This kernel keeps exactly that chain for every
// output -- one fp32 accumulator, one fmaf per k, k in the same order, no split of K -- so its
// results are bit-identical to the reference's CPU path (the epilogue repeats the reference's
// separate roundings too).  Parallelism comes only from the filter x pixel tiles.
//
// Structure (one CTA = BM filters x BN output pixels over the flattened batch, 8x8 outputs per
// thread as two half-tile-apart quads, so shared-memory reads are broadcasts or conflict-free
// float4s):
//   * a stage is CC whole input channels: KS = CC*kh*kw consecutive k rows of the reference
//     order, so one barrier covers 1152-2304 FMAs per thread;
//   * weights arrive as 16-byte cp.async copies of the packed rows (either packed order: the
//     row of (c, r, s) is looked up once per thread, a stage then only advances the channel);
//   * activations are gathered per pixel: a thread owns one output pixel column and the taps of
//     one channel, so the tap offsets and their padding tests are computed once per thread and a
//     stage adds only the channel offset; 1x1 stride-1 layers copy 16-byte quads;
//   * 4-stage cp.async ring (3 for the generic tap count);
//   * fused epilogue (bias or unfused batchnorm, activation, residual, YOLO logistic) shared with
//     the tiled kernel.
// FMA = false gives the connected layer's order instead (sgemm_nt -> s_nt, source/ntensors.pas:
// 1957-2005: s = s + a*b, a separate multiply and add per k).
#pragma once
#include "conv_fp32_kernel.cuh"

namespace tbi {

enum ExactMode { EX_1X1V = 0, EX_1X1 = 1, EX_3X3 = 2, EX_GEN = 3 };
constexpr int EX_GEN_TAPS = 25;  // generic tap loop: kernel windows of at most 25 taps

// VAR selects the stage depth: 0 = 2 channels (3x3) / 16 channels (1x1) per stage, 4-deep ring;
// 1 = twice the channels per stage, 3-deep ring; 2 = the channels of 0, 3-deep ring; 3 = as 0,
// compiled for one resident CTA per SM (no register cap from occupancy).
template <int MODE, int G, int VAR = 0>
struct ExactShape {
    static constexpr int STAGES = (MODE == EX_GEN || VAR > 0) ? 3 : 4;
    static constexpr int CC = MODE == EX_3X3 ? (VAR == 1 ? 4 : 2) : (MODE == EX_GEN ? G : (VAR == 1 ? 32 : 16));
    static constexpr int KSMAX = MODE == EX_3X3 ? 9 * CC : (MODE == EX_GEN ? G * EX_GEN_TAPS : CC);
};

template <int BM, int BN, int TM, int TN>
__host__ __device__ constexpr int exact_threads() { return (BM / TM) * (BN / TN); }

template <int MODE, int G, int VAR>
inline int exact_smem_bytes(int BM, int BN) {
    using S = ExactShape<MODE, G, VAR>;
    return S::STAGES * S::KSMAX * (BM + BN) * 4;
}

// TM x TN outputs per thread: filters in two TM/2 quads BM/2 apart, pixels in TN/4 quads BN*4/TN
// apart (every shared-memory read a broadcast or a conflict-free float4).  TN = 16 tiles and VAR 3
// are compiled without an occupancy-derived register cap.
template <int BM, int BN, int TM, int TN, int MODE, bool FMA, int VAR>
__global__ void __launch_bounds__(exact_threads<BM, BN, TM, TN>(),
                                  (VAR == 3 || TN == 16) ? 1 : 512 / exact_threads<BM, BN, TM, TN>())
k_conv_exact(const ConvParams p) {
    constexpr int TX = BN / TN, TM2 = TM / 2, NQ = TN / 4, QS = BN / NQ;
    constexpr int NT = exact_threads<BM, BN, TM, TN>();
    constexpr int G = NT / BN;  // pixel-column groups of the activation loader
    static_assert(G == 1 || G == 2, "one or two threads per pixel column");
    using S = ExactShape<MODE, G, VAR>;
    constexpr int STAGES = S::STAGES, KSMAX = S::KSMAX, CC = S::CC;
    extern __shared__ __align__(16) float smem[];
    float* As = smem;                      // [STAGES][KSMAX][BM]
    float* Bs = smem + STAGES * KSMAX * BM;  // [STAGES][KSMAX][BN]
    TB_GRID_DEP_ENTRY();

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const int m0 = blockIdx.y * BM;
    const long long n0 = (long long)blockIdx.x * BN;
    const int KHKW = MODE == EX_3X3 ? 9 : (MODE == EX_GEN ? p.KH * p.KW : 1);
    const int KS = MODE == EX_GEN ? G * KHKW : KSMAX;
    const int nst = (p.C + CC - 1) / CC;  // stages: channel groups of CC
    const long long HW = (long long)p.H * p.W;

    // ---- weights: thread -> (16-byte column quad, rows w_r0 + i*RG) of every stage ----
    constexpr int MQ = BM / 4, RG = NT / MQ, WIT = (KSMAX + RG - 1) / RG;
    static_assert(NT % MQ == 0, "a weight row is whole 16-byte copies");
    const int w_mq = tid % MQ, w_r0 = tid / MQ;
    const bool w_mok = m0 + 4 * w_mq < p.Mpad;
    int w_off[WIT], w_cc[WIT];
#pragma unroll
    for (int i = 0; i < WIT; ++i) {
        const int row = w_r0 + i * RG;
        if (row < KS) {
            const int cc = row / KHKW, rs = row - cc * KHKW;
            // packed row of (channel cc, tap rs): RSC order k = rs*Cpad + c, CRS order k = c*khkw + rs
            w_off[i] = (p.wrsc ? rs * p.Cpad + cc : cc * KHKW + rs) * p.Mpad + m0 + 4 * w_mq;
            w_cc[i] = cc;
        } else {
            w_off[i] = 0;
            w_cc[i] = 1 << 29;  // no such row
        }
    }
    const long long wstep = (long long)(p.wrsc ? CC : CC * KHKW) * p.Mpad;

    // ---- activations: thread -> one pixel column, channel group g of the stage ----
    const int g = tid / (NT / G);  // 0 .. G-1
    int bcol;
    long long ncol;
    if (MODE == EX_1X1V) {
        bcol = 0;
        ncol = 0;
    } else {
        bcol = tid % BN;
        ncol = n0 + bcol;
    }
    const bool nvalid = MODE != EX_1X1V && ncol < p.Ntot;
    const float* xb = p.x;
    int iy0 = 0, ix0 = 0;
    if (nvalid) {
        const unsigned n = (unsigned)ncol;
        const unsigned b = n / (unsigned)p.OHW;
        const int pix = (int)(n - b * (unsigned)p.OHW);
        const int oy = pix / p.OW, ox = pix - oy * p.OW;
        iy0 = oy * p.SY - p.PY;
        ix0 = ox * p.SX - p.PX;
        xb = p.x + (long long)b * p.x_bs;
    }
    // 3x3: row / column offsets and in-image tests of the three kernel rows / columns
    int rowoff[3] = {0, 0, 0}, coloff[3] = {0, 0, 0};
    unsigned tapok = 0;
    if (MODE == EX_3X3) {
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const int iy = iy0 + r * p.DY;
            rowoff[r] = iy * p.W;
#pragma unroll
            for (int s = 0; s < 3; ++s) {
                const int ix = ix0 + s * p.DX;
                coloff[s] = ix;
                if (nvalid && (unsigned)iy < (unsigned)p.H && (unsigned)ix < (unsigned)p.W) tapok |= 1u << (r * 3 + s);
            }
        }
    }
    int pixoff = 0;
    bool pixok = false;
    if (MODE == EX_1X1) {
        pixok = nvalid && (unsigned)iy0 < (unsigned)p.H && (unsigned)ix0 < (unsigned)p.W;
        pixoff = pixok ? iy0 * p.W + ix0 : 0;
    }
    // 1x1 vectorised: thread -> (pixel quad, channel rows v_r0 + i*VRG)
    constexpr int BQ = BN / 4, VRG = NT / BQ, VIT = CC / VRG;
    static_assert(MODE != EX_1X1V || (NT % BQ == 0 && CC % VRG == 0), "1x1 quads cover the tile");
    const float* vq = p.x;
    bool vok = false;
    int v_r0 = 0;
    if (MODE == EX_1X1V) {
        const int q = tid % BQ;
        v_r0 = tid / BQ;
        const long long nq = n0 + 4 * q;
        vok = nq < p.Ntot;  // OHW % 4 == 0: a quad lies in one image
        if (vok) {
            const unsigned n = (unsigned)nq;
            const unsigned b = n / (unsigned)p.OHW;
            vq = p.x + (long long)b * p.x_bs + (n - b * (unsigned)p.OHW);
        }
    }

    auto load_stage = [&](int st_idx, int buf) {
        const int c0 = st_idx * CC;
        float* as = As + buf * KSMAX * BM;
        const float* wst = p.w + (long long)st_idx * wstep;
#pragma unroll
        for (int i = 0; i < WIT; ++i) {
            const int row = w_r0 + i * RG;
            if (row < KS) {
                const bool ok = w_mok && c0 + w_cc[i] < p.C;
                cp_async16(as + row * BM + 4 * w_mq, ok ? wst + w_off[i] : p.w, ok);
            }
        }
        float* bs = Bs + buf * KSMAX * BN;
        if (MODE == EX_1X1V) {
#pragma unroll
            for (int i = 0; i < VIT; ++i) {
                const int row = v_r0 + i * VRG;
                const bool ok = vok && c0 + row < p.C;
                cp_async16(bs + row * BN + 4 * (tid % BQ), ok ? vq + (long long)(c0 + row) * HW : p.x, ok);
            }
        } else if (MODE == EX_1X1) {
            constexpr int RPG = CC / G;
#pragma unroll
            for (int j = 0; j < RPG; ++j) {
                const int row = g * RPG + j;
                const bool ok = pixok && c0 + row < p.C;
                cp_async4(bs + row * BN + bcol, ok ? xb + (long long)(c0 + row) * HW + pixoff : p.x, ok);
            }
        } else if (MODE == EX_3X3) {
            constexpr int CPG = CC / G;  // channels of this thread per stage
#pragma unroll
            for (int cc = 0; cc < CPG; ++cc) {
                const int ch = g * CPG + cc;
                const bool cok = c0 + ch < p.C;
                const float* xc = xb + (long long)(c0 + ch) * HW;
#pragma unroll
                for (int r = 0; r < 3; ++r)
#pragma unroll
                    for (int s = 0; s < 3; ++s) {
                        const bool ok = cok && ((tapok >> (r * 3 + s)) & 1u);
                        cp_async4(bs + (ch * 9 + r * 3 + s) * BN + bcol, ok ? xc + rowoff[r] + coloff[s] : p.x, ok);
                    }
            }
        } else {  // generic window: one channel per group, taps in (r, s) order
            const int ch = g;
            const bool cok = nvalid && c0 + ch < p.C;
            const float* xc = xb + (long long)(c0 + ch) * HW;
            int r = 0, s = 0;
            for (int j = 0; j < KHKW; ++j) {
                const int iy = iy0 + r * p.DY, ix = ix0 + s * p.DX;
                const bool ok = cok && (unsigned)iy < (unsigned)p.H && (unsigned)ix < (unsigned)p.W;
                cp_async4(bs + (ch * KHKW + j) * BN + bcol, ok ? xc + iy * p.W + ix : p.x, ok);
                if (++s == p.KW) { s = 0; ++r; }
            }
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nst) load_stage(s, s);
        cp_async_commit();
    }

    typedef typename VecT<TM2>::T AV;
    auto kstep = [&](const float* as, const float* bs) {
        float a[TM], bv[TN];
        *reinterpret_cast<AV*>(&a[0]) = *reinterpret_cast<const AV*>(as + ty * TM2);
        *reinterpret_cast<AV*>(&a[TM2]) = *reinterpret_cast<const AV*>(as + BM / 2 + ty * TM2);
#pragma unroll
        for (int q = 0; q < NQ; ++q)
            *reinterpret_cast<float4*>(&bv[4 * q]) = *reinterpret_cast<const float4*>(bs + q * QS + tx * 4);
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                if (FMA) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
                else acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], bv[j]));
            }
    };

    for (int t = 0; t < nst; ++t) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        {
            const int tn = t + STAGES - 1;
            if (tn < nst) load_stage(tn, tn % STAGES);
            cp_async_commit();
        }
        const float* as = As + (t % STAGES) * KSMAX * BM;
        const float* bs = Bs + (t % STAGES) * KSMAX * BN;
        if (MODE == EX_GEN) {
#pragma unroll 1
            for (int kk = 0; kk < KS; ++kk) kstep(as + kk * BM, bs + kk * BN);
        } else {
#pragma unroll
            for (int kk = 0; kk < KSMAX; ++kk) kstep(as + kk * BM, bs + kk * BN);
        }
    }
    cp_async_wait<0>();

    // ---- epilogue (the tiled kernel's, without split-K) ----
    ColQuad cq[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) cq[q] = decode_quad(p, n0 + q * QS + tx * 4);
    const bool simple = !p.bn_mean && p.yolo_classes == 0 && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
    const bool has_bias = p.bias != nullptr, leaky = p.act == TB_ACT_LEAKY;
    const float* __restrict__ biasp = p.bias;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int m = m0 + (i < TM2 ? ty * TM2 + i : BM / 2 + ty * TM2 + (i - TM2));
        if (m >= p.F) continue;
        const float bm = has_bias ? __ldg(biasp + m) : 0.f;
#pragma unroll
        for (int gq = 0; gq < NQ; ++gq) conv_store4(p, m, cq[gq], &acc[i][gq * 4], simple, has_bias, leaky, bm);
    }
}

template <int BM, int BN, int TM, int TN, int MODE, bool FMA, int VAR>
int exact_launch_one(tb_ctx* ctx, const ConvParams& p, dim3 grid) {
    constexpr int NT = exact_threads<BM, BN, TM, TN>();
    const int smem = exact_smem_bytes<MODE, NT / BN, VAR>(BM, BN);
    auto kern = k_conv_exact<BM, BN, TM, TN, MODE, FMA, VAR>;
    static std::mutex mu;
    static bool done[64] = {false};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device >= 64) return fail(TB_ERR_UNSUPPORTED, "device index %d >= 64", ctx->device);
        if (!done[ctx->device]) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_conv_exact)");
            done[ctx->device] = true;
        }
    }
    if (grid.x == 0) {  // query: resident CTAs per SM
        int n = 1;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, NT, smem) != cudaSuccess || n < 1) n = 1;
        return n;
    }
    return launch(ctx, "k_conv_exact", kern, grid, dim3(NT), (size_t)smem, p);
}

// var: stage-depth variant (ExactShape) of the 3x3 and vectorised 1x1 modes
template <int BM, int BN, int TM, int TN>
int exact_launch_modes(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var) {
    switch (mode) {
    case EX_1X1V:
        if (!fma) return exact_launch_one<BM, BN, TM, TN, EX_1X1V, false, 0>(ctx, p, grid);
        if (var == 1) return exact_launch_one<BM, BN, TM, TN, EX_1X1V, true, 1>(ctx, p, grid);
        if (var == 2) return exact_launch_one<BM, BN, TM, TN, EX_1X1V, true, 2>(ctx, p, grid);
        return exact_launch_one<BM, BN, TM, TN, EX_1X1V, true, 0>(ctx, p, grid);
    case EX_1X1:
        return fma ? exact_launch_one<BM, BN, TM, TN, EX_1X1, true, 0>(ctx, p, grid)
                   : exact_launch_one<BM, BN, TM, TN, EX_1X1, false, 0>(ctx, p, grid);
    case EX_3X3:
        if (var == 1) return exact_launch_one<BM, BN, TM, TN, EX_3X3, true, 1>(ctx, p, grid);
        if (var == 2) return exact_launch_one<BM, BN, TM, TN, EX_3X3, true, 2>(ctx, p, grid);
        if (var == 3) return exact_launch_one<BM, BN, TM, TN, EX_3X3, true, 3>(ctx, p, grid);
        return exact_launch_one<BM, BN, TM, TN, EX_3X3, true, 0>(ctx, p, grid);
    default: return exact_launch_one<BM, BN, TM, TN, EX_GEN, true, 0>(ctx, p, grid);
    }
}

// one entry per tile shape (own translation units); grid.x == 0 returns resident CTAs per SM
int exact_launch_128x128(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var);
int exact_launch_64x128(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var);
int exact_launch_128x64(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var);
int exact_launch_64x64(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var);
int exact_launch_32x128(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var);
// 32 outputs per thread (conv_exact_small.cu)
int exact_launch_64x64n4(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var);
int exact_launch_64x128m4(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var);
// 3x3 stride-1 pad-1 windows with each input value staged once (conv_slide.cu): tiles
// 0..3 = 128x128, 128x64, 64x128, 64x64 (filters x positions) with a register window over one
// staged copy, 4..7 = the same tiles reading four shifted copies, 8..10 = register window with a
// relaxed register cap (128x64 at 2 and 3 CTAs per SM, 128x128 at 1)
constexpr int SLIDE_TILES = 17;  // 11..16: smaller thread tiles (8x4, 4x4, 4x8 outputs per thread)
bool conv_slide_supported(const ConvGeom& g, int tile);
int conv_slide_launch(tb_ctx* ctx, int tile, const ConvGeom& g, const ConvParams& p, bool query);
int slide_tile_bm(int tile);
int slide_tile_bn(int tile);
int slide_tile_nt(int tile);
// warp-specialised variant (conv_exact_ws.cu): 128 filters x bn (64 or 128) pixels per CTA
int exact_ws_launch(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, int bn);

}  // namespace tbi
