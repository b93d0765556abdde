// conv_tc.cu -- TF32 tensor-core (tcgen05 / TMEM) implicit-GEMM convolution, NCHW in and out.
//
// GEMM view (transposed against the FP32 path so that the output store is coalesced):
//   D[n = output pixel][f = filter] = sum_k A[n][k] * W[k][f],  K = (r, s, c), channel fastest,
// in the order of the packed weight rows Wp[k][Mpad] (RSC packing, C % 32 == 0).
//
// A (pixels x K) comes from "tap replicas" of the input, P[s][ph][b][c][Hrep][Wp]: for kernel
// column s and row phase ph (ph < stride_y), replica row R holds input row
// stride_y*(R - pad_top) + ph sampled at the output columns (ix = stride_x*x + s*dil_x - pad_x,
// zero outside the image and for x >= OW; Wp = round_up(OW, 4)).  Kernel row r then reads the
// plane of phase ph(r) shifted down by rowoff(r) rows, i.e. a run of consecutive elements that
// starts rowoff(r)*Wp past the pixel: for a fixed (r, s, c) a tile row of A is one contiguous
// 16-byte-aligned run, which TMA loads as boxes of 32 pixels x 32 channels.  Output pixels
// live on a padded grid: n = b*Lp + oy*Wp + ox, Lp = round_up(OH*Wp, 32); pixels with ox >= OW
// or past OH*Wp are computed and dropped.  A 1x1 stride-1 unpadded layer with W % 4 == 0 reads
// the input in place (no replica).
// B (K x filters) is the packed weight matrix, read by TMA as boxes of 32 filters x 32 k.
//
// One persistent CTA per SM (320 threads) walks the tiles (128 pixels x BN filters, filters
// fastest).  Warp 0: one thread issues the TMA loads into a STAGES-deep ring.  Warp 1: owns the
// TMEM allocation; one thread issues tcgen05.mma (M = 128, N = BN, K = 8, TF32 in, FP32
// accumulate) into one of two TMEM accumulators and commits each stage back to the producer.
// Warps 2-9: the epilogue, overlapped with the next tile's mainloop: tcgen05.ld of 32 filters of
// one pixel per thread, bias / batchnorm / activation / residual / yolo logistic, NCHW stores
// in which a warp writes 32 consecutive pixels of one filter.  Every wait is bounded: on timeout
// the kernel sets the context status word, drains the copies and MMAs in flight, frees its TMEM
// and returns.
#include "conv_tc.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace tbi {

constexpr int TC_BM = 128, TC_BK = 32, TC_THREADS = 320, TC_MAX_KH = 8;
constexpr int TC_BOX_BYTES = 32 * 32 * 4;

struct TcParams {
    const float* __restrict__ bias;
    const float* __restrict__ bn_scale;
    const float* __restrict__ bn_mean;
    const float* __restrict__ bn_var;
    const float* __restrict__ res;
    float* __restrict__ y;
    int* status;
    int B, F, KW, OH, OW, Wp, NPH, Lp, OHWp, OHW;
    int tiles_n, csteps, ktiles;
    int tiles_total;
    long long y_bs, r_bs;
    int act, yolo_classes;
    int rowoff[TC_MAX_KH], phase[TC_MAX_KH];
};

// Replica layout plan of one geometry.
struct TcPlan {
    int64_t Wp, NPH, pad_top, Hrep, Lp;
    bool inplace;
    int rowoff[TC_MAX_KH], phase[TC_MAX_KH];
};

static void tc_plan(const ConvGeom& g, TcPlan* pl) {
    pl->Wp = round_up(g.OW, 4);
    pl->NPH = g.SY;
    int64_t mn = 0, mx = 0;
    for (int r = 0; r < g.KH; ++r) {
        int64_t off = r * g.DY - g.PY;
        int64_t dr = off >= 0 ? off / g.SY : -((-off + g.SY - 1) / g.SY);  // floor(off / SY)
        pl->phase[r] = (int)(off - dr * g.SY);
        pl->rowoff[r] = (int)dr;
        mn = std::min(mn, dr);
        mx = std::max(mx, dr);
    }
    pl->pad_top = -mn;
    for (int r = 0; r < g.KH; ++r) pl->rowoff[r] += (int)pl->pad_top;
    pl->Hrep = g.OH + pl->pad_top + mx;
    pl->Lp = round_up(g.OH * pl->Wp, 32);
    pl->inplace = g.KH == 1 && g.KW == 1 && g.SY == 1 && g.SX == 1 && g.PY == 0 && g.PX == 0 && g.W % 4 == 0 &&
                  g.x_bs % 4 == 0;
}

// P[s][ph][b][c][Hrep][Wp]; each thread writes 4 consecutive columns (one 16-byte store).
__global__ void k_tc_repack(const float* __restrict__ x, long long x_bs, float* __restrict__ P, int B, int C, int H,
                            int W, int SY, int SX, int DX, int PX, int NPH, int pad_top, int Hrep, int Wp, int OW) {
    const int plane = Hrep * Wp;
    const int i4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i4 >= plane) return;
    const int c = blockIdx.y;
    const int zb = blockIdx.z;  // (s * NPH + ph) * B + b
    const int b = zb % B, sp = zb / B, ph = sp % NPH, s = sp / NPH;
    const int row = i4 / Wp, x0 = i4 - row * Wp;
    const int iy = SY * (row - pad_top) + ph;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if ((unsigned)iy < (unsigned)H) {
        const float* src = x + (long long)b * x_bs + ((long long)c * H + iy) * W;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int xx = x0 + j, ix = SX * xx + s * DX - PX;
            if (xx < OW && (unsigned)ix < (unsigned)W) v[j] = __ldg(src + ix);
        }
    }
    float4* dst = reinterpret_cast<float4*>(P + ((long long)zb * C + c) * plane + i4);
    *dst = make_float4(v[0], v[1], v[2], v[3]);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_conv_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const TcParams p) {
    constexpr int A_BYTES = TC_BM * TC_BK * 4;
    constexpr int B_BYTES = BN * TC_BK * 4;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr int NCHUNK = BN / 32;  // 32-filter column chunks of an accumulator
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - ((unsigned)__cvta_generic_to_shared(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], tfull_bar[2], tempty_bar[2], drain_bar;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const unsigned sbase = (unsigned)__cvta_generic_to_shared(smem);

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full_bar[s], 1);
            tc::mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull_bar[b], 1);
            tc::mbar_init(&tempty_bar[b], 256);
        }
        tc::mbar_init(&drain_bar, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 1) tc::tmem_alloc(&tmem_base, 2 * BN);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem0 = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.tiles_total; t += gridDim.x) {
                const int mt = t / p.tiles_n, nt = t - mt * p.tiles_n;
                const int n0 = mt * TC_BM, f0 = nt * BN;
                int bq[4], qq[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int n = n0 + 32 * j;
                    bq[j] = n / p.Lp;
                    qq[j] = n - bq[j] * p.Lp;
                }
                for (int kt = 0; kt < p.ktiles; ++kt, ++it) {
                    const int st = it % STAGES, use = it / STAGES;
                    if (use > 0 && !tc::mbar_wait_bounded(&empty_bar[st], (use - 1) & 1, &abort_flag, p.status, 911)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&full_bar[st], STAGE_BYTES);
                    const int rs = kt / p.csteps, c0 = (kt - rs * p.csteps) * TC_BK;
                    const int r = rs / p.KW, s = rs - r * p.KW;
                    const int xoff = p.rowoff[r] * p.Wp, z0 = (s * p.NPH + p.phase[r]) * p.B;
                    const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        tc::tma_load_3d(sa + j * TC_BOX_BYTES, &tmA, &full_bar[st], qq[j] + xoff, c0, z0 + bq[j]);
#pragma unroll
                    for (int j = 0; j < NCHUNK; ++j)
                        tc::tma_load_2d(sb + j * TC_BOX_BYTES, &tmB, &full_bar[st], f0 + 32 * j, kt * TC_BK);
                }
            }
            if (!ok) {  // an abort: let the copies already issued land before the CTA exits
                for (int j = it > STAGES ? it - STAGES : 0; j < it; ++j)
                    tc::mbar_wait_limit(&full_bar[j % STAGES], (j / STAGES) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = tc::idesc_tf32_mn(TC_BM, BN);
            int it = 0, tl = 0;
            bool ok = true, issued = false;
            for (int t = blockIdx.x; ok && t < p.tiles_total; t += gridDim.x, ++tl) {
                const int buf = tl & 1, u = tl >> 1;
                if (u > 0 && !tc::mbar_wait_bounded(&tempty_bar[buf], (u - 1) & 1, &abort_flag, p.status, 912)) break;
                tc::tc_fence_after();
                const uint32_t d = tmem0 + buf * BN;
                for (int kt = 0; kt < p.ktiles; ++kt, ++it) {
                    const int st = it % STAGES, use = it / STAGES;
                    if (!tc::mbar_wait_bounded(&full_bar[st], use & 1, &abort_flag, p.status, 913)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 8; ++kk) {
                        const uint64_t da = tc::smem_desc_mn_sw128_32b(sa + kk * 1024, TC_BOX_BYTES, 512);
                        const uint64_t db = tc::smem_desc_mn_sw128_32b(sb + kk * 1024, TC_BOX_BYTES, 512);
                        tc::mma_tf32(d, da, db, idesc, (kt | kk) ? 1u : 0u);
                    }
                    issued = true;
                    tc::mma_commit(&empty_bar[st]);
                }
                if (ok) tc::mma_commit(&tfull_bar[buf]);
            }
            if (issued) {  // every MMA has finished before TMEM is freed
                tc::mma_commit(&drain_bar);
                tc::mbar_wait_limit(&drain_bar, 0);
            }
        }
    } else {
        // ---------------- epilogue (warps 2-9) ----------------
        const int quarter = warp & 3;      // TMEM lanes 32*quarter .. +31 (a warp's lane window)
        const int half = (warp - 2) >> 2;  // column chunks half, half+2, ...
        ConvParams ep;
        ep.bias = p.bias;
        ep.bn_scale = p.bn_scale;
        ep.bn_mean = p.bn_mean;
        ep.bn_var = p.bn_var;
        ep.act = p.act;
        ep.yolo_classes = p.yolo_classes;
        int tl = 0;
        for (int t = blockIdx.x; t < p.tiles_total; t += gridDim.x, ++tl) {
            const int buf = tl & 1, u = tl >> 1;
            const bool ok = !abort_flag && tc::mbar_wait_bounded(&tfull_bar[buf], u & 1, &abort_flag, p.status, 914);
            if (!__all_sync(0xffffffffu, ok)) break;  // tcgen05.ld is warp-collective: all lanes or none
            tc::tc_fence_after();
            const int mt = t / p.tiles_n, nt = t - mt * p.tiles_n;
            const int n = mt * TC_BM + quarter * 32 + lane;
            const int b = n / p.Lp, q = n - b * p.Lp;
            const int oy = q / p.Wp, ox = q - oy * p.Wp;
            const bool valid = b < p.B && q < p.OHWp && ox < p.OW;
            const long long pix = (long long)oy * p.OW + ox;
            float* yb = p.y + (valid ? b * p.y_bs + pix : 0);
            const float* rb = p.res ? p.res + (valid ? b * p.r_bs + pix : 0) : nullptr;
            const uint32_t taddr = tmem0 + buf * BN + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
            for (int c = half; c < NCHUNK; c += 2) {
                float v[32];
                tc::tmem_ld32(taddr + c * 32, v);
                const int fb = nt * BN + c * 32;
                if (valid) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {  // fully unrolled: v stays in registers
                        const int f = fb + i;
                        if (f < p.F) {
                            float o = conv_epilogue(v[i], f, ep);
                            const long long off = (long long)f * p.OHW;
                            if (rb) o = __fadd_rn(o, rb[off]);
                            yb[off] = o;
                        }
                    }
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&tempty_bar[buf]);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem0, 2 * BN);
    }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// fp32 tensor map with boxes of 32 x 32 (x 1), 128-byte swizzle with 32-byte atoms, zero fill
static int encode_map(CUtensorMap* m, const float* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(TB_ERR_CUDA, "tensor-core conv: cuTensorMapEncodeTiled is not available");
    cuuint64_t d[3], s[2];
    cuuint32_t box[3] = {32, 32, 1}, es[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) d[i] = dims[i];
    for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<float*>(base), d, s, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TB_ERR_CUDA, "tensor-core conv: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TB_OK;
}

bool conv_tc_supported(const ConvGeom& g) {
    return g.rsc && g.C % TC_BK == 0 && g.Cpad == g.C && g.KH <= TC_MAX_KH && g.SY <= 4 &&
           g.B * round_up(g.OH * round_up(g.OW, 4), 32) < ((int64_t)1 << 31) - TC_BM;
}

int64_t conv_tc_scratch_floats(const ConvGeom& g) {
    TcPlan pl;  // in-place layers still get a replica when x is not 16-byte aligned
    tc_plan(g, &pl);
    return g.KW * pl.NPH * g.B * g.C * pl.Hrep * pl.Wp;
}

template <int BN, int STAGES>
static int launch_bn(tb_ctx* ctx, const CUtensorMap& a, const CUtensorMap& b, const TcParams& p) {
    constexpr int smem = STAGES * (TC_BM * TC_BK * 4 + BN * TC_BK * 4) + 1024;
    static std::mutex mu;
    static bool done[64] = {false};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !done[ctx->device]) {
            cudaError_t e = cudaFuncSetAttribute(k_conv_tc<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(conv_tc)");
            done[ctx->device] = true;
        }
    }
    const int grid = (int)std::min<int64_t>(p.tiles_total, ctx->sm_count);
    k_conv_tc<BN, STAGES><<<grid, TC_THREADS, smem, ctx->stream>>>(a, b, p);
    return check_launch("k_conv_tc");
}

// Filter-tile width: the smallest modelled time (waves of one CTA per SM x per-tile cost).
static int choose_bn(const ConvGeom& g, int64_t tiles_m, int sms) {
    int best = 32;
    double best_cost = 1e300;
    for (int bn : {32, 64, 128, 256}) {
        if (bn > round_up(g.F, 32) && bn != 32) break;
        const int64_t tiles = tiles_m * ceil_div(g.F, bn);
        const double cost = (double)ceil_div(tiles, sms) * (bn + 48);
        if (cost < best_cost) best = bn, best_cost = cost;
    }
    return best;
}

int conv_tc_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                   const float* bn_scale, const float* bn_mean, const float* bn_var, const float* res, float* y,
                   int act, int yolo_classes, float* scratch, int64_t* launches) {
    if (!conv_tc_supported(g)) return fail(TB_ERR_UNSUPPORTED, "tensor-core conv: unsupported geometry");
    if (g.B == 0) return TB_OK;
    TcPlan pl;
    tc_plan(g, &pl);
    const bool inplace = pl.inplace && aligned16(x);
    const float* src = x;
    uint64_t dims[3], strides[2];
    if (inplace) {
        dims[0] = (uint64_t)(g.H * g.W);
        dims[1] = (uint64_t)g.C;
        dims[2] = (uint64_t)g.B;
        strides[0] = (uint64_t)(g.H * g.W) * 4;
        strides[1] = (uint64_t)g.x_bs * 4;
    } else {
        if (!scratch || !aligned16(scratch))
            return fail(TB_ERR_INVALID, "tensor-core conv: this geometry needs a 16-byte-aligned replica buffer");
        const int64_t plane = pl.Hrep * pl.Wp;
        dim3 rg((unsigned)ceil_div(plane, 4 * 256), (unsigned)g.C, (unsigned)(g.KW * pl.NPH * g.B));
        if (rg.y > 65535 || rg.z > 65535) return fail(TB_ERR_UNSUPPORTED, "tensor-core conv: replica grid too large");
        k_tc_repack<<<rg, 256, 0, ctx->stream>>>(x, g.x_bs, scratch, (int)g.B, (int)g.C, (int)g.H, (int)g.W,
                                                 (int)g.SY, (int)g.SX, (int)g.DX, (int)g.PX, (int)pl.NPH,
                                                 (int)pl.pad_top, (int)pl.Hrep, (int)pl.Wp, (int)g.OW);
        int r = check_launch("k_tc_repack");
        if (r != TB_OK) return r;
        if (launches) ++*launches;
        src = scratch;
        dims[0] = (uint64_t)plane;
        dims[1] = (uint64_t)g.C;
        dims[2] = (uint64_t)(g.KW * pl.NPH * g.B);
        strides[0] = (uint64_t)plane * 4;
        strides[1] = (uint64_t)(g.C * plane) * 4;
    }
    CUtensorMap ta, tb;
    int r = encode_map(&ta, src, 3, dims, strides);
    if (r != TB_OK) return r;
    const uint64_t wd[2] = {(uint64_t)g.Mpad, (uint64_t)g.Kpad}, ws[1] = {(uint64_t)g.Mpad * 4};
    r = encode_map(&tb, wp, 2, wd, ws);
    if (r != TB_OK) return r;

    TcParams p{};
    p.bias = bias; p.bn_scale = bn_scale; p.bn_mean = bn_mean; p.bn_var = bn_var;
    p.res = res; p.y = y; p.status = ctx->d_status;
    p.B = (int)g.B; p.F = (int)g.F; p.KW = (int)g.KW; p.OH = (int)g.OH; p.OW = (int)g.OW;
    p.Wp = inplace ? (int)g.W : (int)pl.Wp;
    p.NPH = inplace ? 1 : (int)pl.NPH;
    p.Lp = (int)round_up(g.OH * p.Wp, 32);
    p.OHWp = (int)(g.OH * p.Wp);
    p.OHW = (int)(g.OH * g.OW);
    p.csteps = (int)(g.C / TC_BK);
    p.ktiles = (int)(g.KH * g.KW * p.csteps);
    p.y_bs = g.y_bs; p.r_bs = g.r_bs;
    p.act = act; p.yolo_classes = yolo_classes;
    for (int i = 0; i < TC_MAX_KH; ++i) {
        p.rowoff[i] = i < g.KH && !inplace ? pl.rowoff[i] : 0;
        p.phase[i] = i < g.KH && !inplace ? pl.phase[i] : 0;
    }
    const int64_t tiles_m = ceil_div(g.B * p.Lp, TC_BM);
    const int bn = choose_bn(g, tiles_m, ctx->sm_count);
    p.tiles_n = (int)ceil_div(g.F, bn);
    const int64_t tiles = tiles_m * p.tiles_n;
    if (tiles >= ((int64_t)1 << 31)) return fail(TB_ERR_UNSUPPORTED, "tensor-core conv: too many tiles");
    p.tiles_total = (int)tiles;
    switch (bn) {
    case 32: r = launch_bn<32, 8>(ctx, ta, tb, p); break;
    case 64: r = launch_bn<64, 8>(ctx, ta, tb, p); break;
    case 128: r = launch_bn<128, 6>(ctx, ta, tb, p); break;
    default: r = launch_bn<256, 4>(ctx, ta, tb, p); break;
    }
    if (r != TB_OK) return r;
    if (launches) ++*launches;
    return TB_OK;
}

}  // namespace tbi
