// conv_slide.cu -- order-exact FP32 convolution for 3x3 windows with stride 1, padding 1 and no
// dilation (the residual-block and head convs that carry ~77% of YOLOv3's FLOPs), with every input
// value staged once per CTA instead of once per tap.
//
// Summation order: as conv_exact.cuh -- every output is one fp32 accumulator that receives one fmaf
// per k in the reference's im2col order k = c*9 + r*3 + s (source/ntensors.pas:8252-8349 ->
// s_nn -> saxpy_avx2: one FMA per k, k ascending), so the result is bit-identical to the reference
// CPU path.  Padded taps multiply a staged zero, as the reference multiplies im2col's zeros.
//
// Position space.  Output pixel (b, y, x) sits at position q = (b*Hp + y)*Wp + x with Hp = H + 1 and
// a row pitch Wp >= W + 1: every image row is followed by Wp - W junk columns and every image by one
// junk row.  The input pixel that tap (r, s) of position q reads is then position
// q + (r-1)*Wp + (s-1) of the same space: the left/right padding lands in a junk column, the
// top/bottom padding in a junk row, and both are staged as zeros.  A CTA owns BN consecutive
// positions from P0 and stages, for each channel of a stage, the run of positions
// P0 - Wp - 1 .. P0 + BN + Wp (Ls floats, ~BN + 2*Wp) with 4-byte cp.async copies whose source
// offsets every thread computes once; the conv_exact 3x3 mode copies 9*BN gathered values instead.
//
// Mainloop.  A thread owns 8 filters (two quads BM/2 apart) x 8 positions (two quads BN/2 apart)
// (4-filter / 4-position tiles for small layers).
// For one (channel, kernel row r) it reads each position quad's 6-value input window with two
// 16-byte shared loads and runs the three taps s = 0, 1, 2 from registers: 4 shared loads of input
// and 6 of weights per 192 FMAs.  The window's misalignment (r*Wp) mod 4 is a compile-time constant
// (WPM = Wp mod 4 is a template parameter; the host picks Wp with Wp mod 4 != 3 so that it is at
// most 2 and two 16-byte loads always cover the window).  Junk positions are computed and dropped.
#include "conv_exact.cuh"

namespace tbi {

struct SlideParams {
    int Wp, Hp, Ls;  // row pitch, rows per image (H + 1), staged floats per channel (multiple of 4)
    int B;           // images
    long long npos;  // B * Hp * Wp positions
};

constexpr int SL_CC = 4;      // channels per stage: 36 k rows
constexpr int SL_STAGES = 3;  // cp.async ring depth
constexpr int SL_JMAX = 4;    // staged floats per channel <= SL_JMAX * threads

template <int BM, int BN, int TM, int TN>
__host__ __device__ constexpr int slide_threads() { return (BM / TM) * (BN / TN); }

// SH = 1 stages four copies of each channel's run, copy d shifted left by d floats, so that every
// tap's position quads are aligned float4s of one copy (the plain outer-product k step).
inline int slide_smem_bytes(int BM, int Ls, int SH) {
    return SL_STAGES * (9 * SL_CC * BM + (SH ? 4 : 1) * SL_CC * Ls) * 4;
}

// A thread owns TM filters (TM/4 quads, BM/2 apart when two) x TN positions (TN/4 quads, BN/2
// apart when two).  MB: resident CTAs per SM the register allocation is capped for (0: 512
// threads per SM).
template <int BM, int BN, int TM, int TN, int WPM, int SH, int MB>
__global__ void __launch_bounds__(slide_threads<BM, BN, TM, TN>(), MB ? MB : 512 / slide_threads<BM, BN, TM, TN>())
k_conv_slide(const ConvParams p, const SlideParams s) {
    constexpr int NT = slide_threads<BM, BN, TM, TN>(), TX = BN / TN, KS = 9 * SL_CC, NCOPY = SH ? 4 : 1;
    constexpr int QM = TM / 4, QN = TN / 4, MSTEP = BM / QM, NSTEP = BN / QN;
    static_assert((TM == 4 || TM == 8) && (TN == 4 || TN == 8), "thread tiles of 4 or 8");
    extern __shared__ __align__(16) float smem[];
    float* As = smem;                            // [STAGES][KS][BM]
    float* Bs = smem + SL_STAGES * KS * BM;      // [STAGES][NCOPY][CC][Ls]
    TB_GRID_DEP_ENTRY();

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const int m0 = blockIdx.y * BM;
    const long long P0 = (long long)blockIdx.x * BN;
    const int nst = p.C / SL_CC;  // the host admits C % SL_CC == 0 only
    const long long HW = (long long)p.H * p.W;
    const int Ls = s.Ls, Wp = s.Wp;

    // ---- weights: thread -> (16-byte column quad, rows w_r0 + i*RG) of every stage ----
    constexpr int MQ = BM / 4, RG = NT / MQ, WIT = (KS + RG - 1) / RG;
    static_assert(NT % MQ == 0, "a weight row is whole 16-byte copies");
    const int w_mq = tid % MQ, w_r0 = tid / MQ;
    const bool w_mok = m0 + 4 * w_mq < p.Mpad;
    int w_off[WIT];
#pragma unroll
    for (int i = 0; i < WIT; ++i) {
        const int row = w_r0 + i * RG;
        const int cc = row / 9, rs = row - cc * 9;
        // packed row of (channel cc, tap rs): RSC order k = rs*Cpad + c, CRS order k = c*9 + rs
        w_off[i] = row < KS ? (p.wrsc ? rs * p.Cpad + cc : cc * 9 + rs) * p.Mpad + m0 + 4 * w_mq : 0;
    }
    const long long wstep = (long long)(p.wrsc ? SL_CC : KS) * p.Mpad;

    // ---- activations: staged float j of a channel = position P0 - Wp - 1 + j ----
    int goff[SL_JMAX];  // offset of that input pixel in the batch (channel 0), or -1: a staged zero
#pragma unroll
    for (int i = 0; i < SL_JMAX; ++i) {
        const int j = tid + i * NT;
        goff[i] = -1;
        const long long v = P0 - Wp - 1 + j;
        if (j < Ls && v >= 0) {
            const long long row = v / Wp;
            const int xx = (int)(v - row * Wp);
            const int b = (int)(row / s.Hp), yy = (int)(row - (long long)b * s.Hp);
            if (xx < p.W && yy < p.H && b < s.B) goff[i] = (int)(b * p.x_bs) + yy * p.W + xx;
        }
    }

    auto load_stage = [&](int st, int buf) {
        float* as = As + buf * KS * BM;
        const float* wst = p.w + (long long)st * wstep;
#pragma unroll
        for (int i = 0; i < WIT; ++i) {
            const int row = w_r0 + i * RG;
            if (row < KS) cp_async16(as + row * BM + 4 * w_mq, w_mok ? wst + w_off[i] : p.w, w_mok);
        }
        float* bs = Bs + buf * NCOPY * SL_CC * Ls;
        const float* xs = p.x + (long long)st * SL_CC * HW;
#pragma unroll
        for (int cc = 0; cc < SL_CC; ++cc) {
#pragma unroll
            for (int i = 0; i < SL_JMAX; ++i) {
                const int j = tid + i * NT;
                if (j < Ls) {
                    const bool ok = goff[i] >= 0;
                    const float* src = ok ? xs + cc * HW + goff[i] : p.x;
#pragma unroll
                    for (int d = 0; d < NCOPY; ++d)  // copy d holds float j at j - d
                        if (j >= d) cp_async4(bs + (d * SL_CC + cc) * Ls + j - d, src, ok);
                }
            }
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

#pragma unroll
    for (int st = 0; st < SL_STAGES - 1; ++st) {
        if (st < nst) load_stage(st, st);
        cp_async_commit();
    }

    for (int t = 0; t < nst; ++t) {
        cp_async_wait<SL_STAGES - 2>();
        __syncthreads();
        {
            const int tn = t + SL_STAGES - 1;
            if (tn < nst) load_stage(tn, tn % SL_STAGES);
            cp_async_commit();
        }
        const float* as = As + (t % SL_STAGES) * KS * BM + ty * 4;
        const float* bs = Bs + (t % SL_STAGES) * NCOPY * SL_CC * Ls + 4 * tx;
        if constexpr (SH != 0) {
#pragma unroll 1
            for (int cc = 0; cc < SL_CC; ++cc)
#pragma unroll
                for (int r = 0; r < 3; ++r)
#pragma unroll
                    for (int sx = 0; sx < 3; ++sx) {
                        const int d = (r * WPM + sx) & 3;  // compile-time: the copy whose quads align
                        const float* bq = bs + (d * SL_CC + cc) * Ls + r * Wp + sx - d;
                        float a[TM], bv[TN];
                        const float* ar = as + (cc * 9 + r * 3 + sx) * BM;
#pragma unroll
                        for (int q = 0; q < QM; ++q)
                            *reinterpret_cast<float4*>(&a[4 * q]) = *reinterpret_cast<const float4*>(ar + q * MSTEP);
#pragma unroll
                        for (int q = 0; q < QN; ++q)
                            *reinterpret_cast<float4*>(&bv[4 * q]) = *reinterpret_cast<const float4*>(bq + q * NSTEP);
#pragma unroll
                        for (int i = 0; i < TM; ++i)
#pragma unroll
                            for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
                    }
        } else {
#pragma unroll 1
        for (int cc = 0; cc < SL_CC; ++cc) {
#pragma unroll
            for (int r = 0; r < 3; ++r) {
                const int o = (r * WPM) & 3;  // compile-time after unrolling: at most 2
                const float* w0 = bs + cc * Ls + r * Wp - o;  // 16-byte aligned
                float v[QN][8];  // each position quad's input window (6 of 8 values used)
#pragma unroll
                for (int q = 0; q < QN; ++q) {
                    *reinterpret_cast<float4*>(&v[q][0]) = *reinterpret_cast<const float4*>(w0 + q * NSTEP);
                    *reinterpret_cast<float4*>(&v[q][4]) = *reinterpret_cast<const float4*>(w0 + q * NSTEP + 4);
                }
#pragma unroll
                for (int sx = 0; sx < 3; ++sx) {
                    const float* ar = as + (cc * 9 + r * 3 + sx) * BM;
                    float a[TM];
#pragma unroll
                    for (int q = 0; q < QM; ++q)
                        *reinterpret_cast<float4*>(&a[4 * q]) = *reinterpret_cast<const float4*>(ar + q * MSTEP);
#pragma unroll
                    for (int i = 0; i < TM; ++i)
#pragma unroll
                        for (int q = 0; q < QN; ++q)
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                acc[i][4 * q + j] = fmaf(a[i], v[q][o + sx + j], acc[i][4 * q + j]);
                }
            }
        }
        }
    }
    cp_async_wait<0>();

    // ---- epilogue: the conv_exact epilogue arithmetic, junk positions dropped ----
    int ob[TN], opix[TN];  // image and pixel of the thread's positions (opix -1: junk)
#pragma unroll
    for (int e = 0; e < TN; ++e) {
        const long long q = P0 + (e / 4) * NSTEP + 4 * tx + (e % 4);
        const long long row = q / Wp;
        const int xx = (int)(q - row * Wp);
        const int b = (int)(row / s.Hp), yy = (int)(row - (long long)b * s.Hp);
        ob[e] = b;
        opix[e] = (q < s.npos && xx < p.W && yy < p.H && b < s.B) ? yy * p.W + xx : -1;
    }
    const bool simple = !p.bn_mean && p.yolo_classes == 0 && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
    const bool has_bias = p.bias != nullptr, leaky = p.act == TB_ACT_LEAKY;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int m = m0 + (i / 4) * MSTEP + ty * 4 + (i % 4);
        if (m >= p.F) continue;
        const float bm = has_bias ? __ldg(p.bias + m) : 0.f;
        float rv[TN];  // the row's residual values, all loads in flight before the first store
#pragma unroll
        for (int e = 0; e < TN; ++e)
            rv[e] = (p.res && opix[e] >= 0) ? __ldg(p.res + ob[e] * p.r_bs + (long long)m * p.OHW + opix[e]) : 0.f;
#pragma unroll
        for (int e = 0; e < TN; ++e) {
            if (opix[e] < 0) continue;
            const long long off = (long long)m * p.OHW + opix[e];
            float o = conv_epi_value(acc[i][e], m, p, simple, has_bias, leaky, bm);
            if (p.res) o = __fadd_rn(o, rv[e]);
            p.y[ob[e] * p.y_bs + off] = o;
        }
    }
}

namespace {

int slide_pitch(int64_t W) {
    int64_t wp = W + 1;
    if ((wp & 3) == 3) ++wp;  // (r * Wp) mod 4 <= 2 for r = 0, 1, 2
    return (int)wp;
}

template <int BM, int BN, int TM, int TN, int WPM, int SH, int MB>
int slide_launch_one(tb_ctx* ctx, const ConvParams& p, const SlideParams& s, bool query) {
    constexpr int NT = slide_threads<BM, BN, TM, TN>();
    const int smem = slide_smem_bytes(BM, s.Ls, SH);
    auto kern = k_conv_slide<BM, BN, TM, TN, WPM, SH, MB>;
    static std::mutex mu;
    static int done[64] = {0};  // largest dynamic shared memory enabled so far, per device
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device >= 64) return fail(TB_ERR_UNSUPPORTED, "device index %d >= 64", ctx->device);
        if (done[ctx->device] < smem) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_conv_slide)");
            done[ctx->device] = smem;
        }
    }
    if (query) {  // resident CTAs per SM
        int n = 1;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, NT, smem) != cudaSuccess || n < 1) n = 1;
        return n;
    }
    dim3 grid((unsigned)ceil_div(s.npos, (int64_t)BN), (unsigned)ceil_div((int64_t)p.F, (int64_t)BM), 1);
    if (grid.y > 65535) return fail(TB_ERR_INVALID, "conv: grid too large");
    return launch(ctx, "k_conv_slide", kern, grid, dim3(NT), (size_t)smem, p, s);
}

template <int BM, int BN, int SH, int MB = 0, int TM = 8, int TN = 8>
int slide_launch_tile(tb_ctx* ctx, const ConvParams& p, const SlideParams& s, bool query) {
    switch (s.Wp & 3) {
    case 0: return slide_launch_one<BM, BN, TM, TN, 0, SH, MB>(ctx, p, s, query);
    case 1: return slide_launch_one<BM, BN, TM, TN, 1, SH, MB>(ctx, p, s, query);
    default: return slide_launch_one<BM, BN, TM, TN, 2, SH, MB>(ctx, p, s, query);
    }
}

// tiles 0-3: register window; 4-7: the same CTA tiles with four shifted copies
// 8-10: register window, register cap relaxed: 128x64 for 2 and 3 CTAs per SM, 128x128 for 1;
// 11-16: smaller thread tiles (more warps for small layers): 64x64 at 8x4, 64x64 at 4x4, 32x64 at
// 4x4, 64x64 at 4x8, 128x64 at 8x4, 32x64 at 8x4
constexpr int kSlideBM[SLIDE_TILES] = {128, 128, 64, 64, 128, 128, 64, 64, 128, 128, 128, 64, 64, 32, 64, 128, 32};
constexpr int kSlideBN[SLIDE_TILES] = {128, 64, 128, 64, 128, 64, 128, 64, 64, 64, 128, 64, 64, 64, 64, 64, 64};
constexpr int kSlideTM[SLIDE_TILES] = {8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 4, 4, 4, 8, 8};
constexpr int kSlideTN[SLIDE_TILES] = {8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 4, 4, 4, 8, 4, 4};
constexpr int slide_sh(int tile) { return tile >= 4 && tile < 8 ? 1 : 0; }

SlideParams slide_params(const ConvGeom& g, int tile) {
    SlideParams s;
    s.Wp = slide_pitch(g.W);
    s.Hp = (int)g.H + 1;
    s.B = (int)g.B;
    s.npos = (long long)g.B * s.Hp * s.Wp;
    s.Ls = (int)((kSlideBN[tile] + 2 * s.Wp + 4 + 3) / 4 * 4);
    return s;
}

}  // namespace

bool conv_slide_supported(const ConvGeom& g, int tile) {
    if (tile < 0 || tile >= SLIDE_TILES) return false;
    if (!(g.KH == 3 && g.KW == 3 && g.SY == 1 && g.SX == 1 && g.PY == 1 && g.PX == 1 && g.DY == 1 && g.DX == 1))
        return false;
    if (g.OH != g.H || g.OW != g.W || g.C % SL_CC != 0 || g.C < SL_CC) return false;
    const SlideParams s = slide_params(g, tile);
    const int nt = (kSlideBM[tile] / kSlideTM[tile]) * (kSlideBN[tile] / kSlideTN[tile]);
    if (s.Ls > SL_JMAX * nt) return false;
    if (slide_smem_bytes(kSlideBM[tile], s.Ls, slide_sh(tile)) > 113 * 1024) return false;  // two CTAs per SM
    // 32-bit staged offsets and positions
    return g.B * g.x_bs < ((int64_t)1 << 31) && s.npos + kSlideBN[tile] < ((int64_t)1 << 31) &&
           (g.rsc ? 9 * g.Cpad : g.Kpad) * g.Mpad < ((int64_t)1 << 31);
}

int slide_tile_bm(int tile) { return kSlideBM[tile]; }
int slide_tile_nt(int tile) { return (kSlideBM[tile] / kSlideTM[tile]) * (kSlideBN[tile] / kSlideTN[tile]); }
int slide_tile_bn(int tile) { return kSlideBN[tile]; }

// query = true: resident CTAs per SM instead of a launch
int conv_slide_launch(tb_ctx* ctx, int tile, const ConvGeom& g, const ConvParams& p, bool query) {
    const SlideParams s = slide_params(g, tile);
    switch (tile) {
    case 0: return slide_launch_tile<128, 128, 0>(ctx, p, s, query);
    case 1: return slide_launch_tile<128, 64, 0>(ctx, p, s, query);
    case 2: return slide_launch_tile<64, 128, 0>(ctx, p, s, query);
    case 3: return slide_launch_tile<64, 64, 0>(ctx, p, s, query);
    case 4: return slide_launch_tile<128, 128, 1>(ctx, p, s, query);
    case 5: return slide_launch_tile<128, 64, 1>(ctx, p, s, query);
    case 6: return slide_launch_tile<64, 128, 1>(ctx, p, s, query);
    case 7: return slide_launch_tile<64, 64, 1>(ctx, p, s, query);
    case 8: return slide_launch_tile<128, 64, 0, 2>(ctx, p, s, query);
    case 9: return slide_launch_tile<128, 64, 0, 3>(ctx, p, s, query);
    case 10: return slide_launch_tile<128, 128, 0, 1>(ctx, p, s, query);
    case 11: return slide_launch_tile<64, 64, 0, 0, 8, 4>(ctx, p, s, query);
    case 12: return slide_launch_tile<64, 64, 0, 0, 4, 4>(ctx, p, s, query);
    case 13: return slide_launch_tile<32, 64, 0, 0, 4, 4>(ctx, p, s, query);
    case 14: return slide_launch_tile<64, 64, 0, 0, 4, 8>(ctx, p, s, query);
    case 15: return slide_launch_tile<128, 64, 0, 0, 8, 4>(ctx, p, s, query);
    default: return slide_launch_tile<32, 64, 0, 0, 8, 4>(ctx, p, s, query);
    }
}

}  // namespace tbi
