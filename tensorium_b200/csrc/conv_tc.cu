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
// one pixel per thread, bias / batchnorm / activation / yolo logistic, then a transpose through
// a per-warp shared slab so that residual loads and NCHW stores are 16-byte vectors of 4
// consecutive pixels of one filter.  Outputs are rounded to TF32 (nearest), so a following 1x1
// layer that reads them in place sees exact TF32 operands.  Every wait is bounded: on timeout
// the kernel sets the context status word, drains the copies and MMAs in flight, frees its TMEM
// and returns.
#include "conv_tc.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

namespace tbi {

constexpr int TC_BM = 128, TC_BK = 32, TC_THREADS = 320;
constexpr int TC_STG_LD = 36;                                // slab row stride (floats)
constexpr int TC_STG_BYTES = 8 * 16 * TC_STG_LD * 4;         // 8 epilogue warps x 16 x 36 floats
constexpr int TC_BIAS_BYTES = 8 * 256 * 4;                   // 8 epilogue warps x one tile's bias
constexpr int TC_BOX_BYTES = 32 * 32 * 4;

struct TcParams {
    const float* __restrict__ bias;
    const float* __restrict__ bn_scale;
    const float* __restrict__ bn_mean;
    const float* __restrict__ bn_var;
    const float* __restrict__ res;
    float* __restrict__ y;
    int* status;
    unsigned long long* phases;  // diagnostics: per-CTA cycle counters (null in normal launches)
    int B, C, F, KW, OH, OW, Wp, NPH, Lp, OHWp, OHW;
    int b_grouped;  // weights read as one 3-D box per stage (Mpad % 32 == 0)
    int vec_out;    // y (and res) take 16-byte stores of pixel quads: OW, OHW, batch strides % 4 == 0
    int g_full;     // 32-pixel groups per image that lie wholly inside it (a1/a4 maps); later
                    // groups are read through the bounds-checked tail map
    int tiles_n, csteps, ktiles;
    int tiles_total;
    int splits, kt_per_split, units;  // split-K: units = tiles_total * splits, unit w = tile w/splits
    float* part;                      // split-K partial tiles [unit][128 pixels][BN] (splits > 1)
    int* tile_cnt;                    // split-K arrival counters, one per tile, left at 0
    long long y_bs, r_bs;
    int act, yolo_classes;
    int phase[TC_MAX_KH];
};

// Tensor maps of one launch.  A (pixels x channels) is viewed 4-D as (32 pixels, channel,
// 32-pixel group, plane index) so that one copy brings a whole 128-pixel tile; one map per kernel
// row r has its base moved rowoff(r) replica rows down.  a4 maps copy 4 groups (a tile inside
// one image), a1 maps one group (tiles that straddle two images).  b views the packed weights as
// (32 filters, k, 32-filter group) with a box of BN/32 groups (bw: 2-D boxes of 32 x 32, for a
// filter count Mpad that is not a multiple of 32).
struct TcMaps {
    CUtensorMap a4[TC_MAX_KH];
    CUtensorMap a1[TC_MAX_KH];
    CUtensorMap tail;  // in-place x: (pixel, channel, image), bounds-checked, for a partial last group
    CUtensorMap b;
};

// cmul: channel multiple a tap replica needs (32 for the TF32 kernel's 32-deep k tiles; the FP32
// TMA kernel takes any RSC layer, its 16-deep tiles lying inside one tap by the packing)
void tc_plan(const ConvGeom& g, TcPlan* pl, int cmul) {
    for (int r = 0; r < TC_MAX_KH; ++r) pl->rowoff[r] = pl->phase[r] = 0;
    pl->NPH = 1;
    pl->pad_top = 0;
    if (g.KH == 1 && g.KW == 1 && g.SY == 1 && g.SX == 1 && g.PY == 0 && g.PX == 0 && (g.H * g.W) % 4 == 0 &&
        g.x_bs % 4 == 0 && g.rsc && g.C % cmul == 0) {
        pl->mode = TC_INPLACE;
        pl->Wp = g.H * g.W;  // one flat row: pixel q of the image is output pixel q
        pl->Hrep = 1;
        pl->Lp = round_up(pl->Wp, 32);
        pl->PS = 0;
        pl->Cr = g.C;
        return;
    }
    pl->Wp = round_up(g.OW, 4);
    pl->Lp = round_up(g.OH * pl->Wp, 32);
    if (!(g.rsc && g.C % cmul == 0)) {
        pl->mode = TC_IM2COL;
        pl->Hrep = g.OH;
        pl->Cr = round_up(g.Kpad, 32);
        pl->PS = round_up(g.OH * pl->Wp, 32) + 32;
        return;
    }
    pl->mode = TC_TAPS;
    pl->Cr = g.C;
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
    // a 32-pixel group read at a row offset never runs past its own plane
    pl->PS = round_up(pl->Hrep * pl->Wp, 32) + 32;
}

// Tap replicas P[s][ph][b][c][Hrep][Wp], planes PS elements apart (the tail of a plane is never
// written: it is read only for pixels that are dropped).  blockIdx.y = (ph * B + b) * C + c;
// one thread makes 4 consecutive columns of one row for every kernel column s: it reads the
// input window those need once (SX*3 + (KW-1)*DX + 1 <= 32 values) and writes one 16-byte quad
// per s, values rounded to TF32.
// SXC, DXC: compile-time column stride and dilation (0 = taken from SX, DX at run time)
template <int SXC, int DXC, bool ROUND>
__global__ void k_tc_repack_taps(const float* __restrict__ x, long long x_bs, float* __restrict__ P, int B, int C,
                                 int H, int W, int KW, int SY, int SX_, int DX_, int PX, int NPH, int pad_top,
                                 int Hrep, int Wp, int OW, int PS) {
    const int SX = SXC ? SXC : SX_, DX = DXC ? DXC : DX_;
    const int q4 = Wp >> 2;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= Hrep * q4) return;
    const int pc = blockIdx.y;
    const int c = pc % C, pb = pc / C, b = pb % B, ph = pb / B;
    const int row = j / q4, x0 = (j - row * q4) * 4;
    const int iy = SY * (row - pad_top) + ph;
    const bool rok = (unsigned)iy < (unsigned)H;
    const float* src = x + (long long)b * x_bs + ((long long)c * H + (rok ? iy : 0)) * W;
    const int ix0 = SX * x0 - PX;                  // input column of output column x0, tap 0
    const int span = SX * 3 + (KW - 1) * DX + 1;  // input columns the 4 outputs x KW taps read
    float win[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) {
        const int ix = ix0 + t;
        float v = (t < span && rok && (unsigned)ix < (unsigned)W) ? __ldg(src + ix) : 0.f;
        win[t] = ROUND ? tc::to_tf32_rna(v) : v;
    }
    const long long plane_z = (long long)ph * B + b;  // z of kernel column s is s*NPH*B + plane_z
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        if (s >= KW) break;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float w = 0.f;
            if (SXC && DXC) {
                w = win[(SXC * k + s * DXC) & 31];  // compile-time index (< span <= 32)
            } else {
                const int t = SX * k + s * DX;  // < span
#pragma unroll
                for (int u = 0; u < 32; ++u) w = (u == t) ? win[u] : w;  // register select, no local memory
            }
            v[k] = (x0 + k < OW) ? w : 0.f;
        }
        const long long z = (long long)s * NPH * B + plane_z;
        *reinterpret_cast<float4*>(P + (z * C + c) * PS + row * Wp + x0) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// im2col rows P[b][k][OH][Wp] in the k order of the packed weights (RSC with Cpad channels per
// tap, or CRS), rows past the real K zero; values rounded to TF32.
template <bool ROUND>
__global__ void k_tc_repack_im2col(const float* __restrict__ x, long long x_bs, float* __restrict__ P, int B, int C,
                                   int H, int W, int KH, int KW, int SY, int SX, int DY, int DX, int PY, int PX,
                                   int rsc, int Cpad, int Kreal, int Cr, int OH, int OW, int Wp, int PS) {
    const int q4 = Wp >> 2, per_plane = OH * q4;
    const long long total = (long long)B * Cr * per_plane;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int pk = (int)(i / per_plane);  // b * Cr + k
        const int j = (int)(i - (long long)pk * per_plane);
        const int oy = j / q4, x0 = (j - oy * q4) * 4;
        const int k = pk % Cr, b = pk / Cr;
        int c, r, s;
        if (rsc) {
            const int rs = k / Cpad;
            c = k - rs * Cpad;
            r = rs / KW;
            s = rs - r * KW;
        } else {
            c = k / (KH * KW);
            const int rs = k - c * KH * KW;
            r = rs / KW;
            s = rs - r * KW;
        }
        const bool kok = k < Kreal && c < C && r < KH;
        const int iy = oy * SY + r * DY - PY;
        const bool rok = kok && (unsigned)iy < (unsigned)H;
        const float* src = x + (long long)b * x_bs + ((long long)(rok ? c : 0) * H + (rok ? iy : 0)) * W;
        float v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int xx = x0 + t, ix = xx * SX + s * DX - PX;
            const float u = (rok && xx < OW && (unsigned)ix < (unsigned)W) ? __ldg(src + ix) : 0.f;
            v[t] = ROUND ? tc::to_tf32_rna(u) : u;
        }
        *reinterpret_cast<float4*>(P + (long long)pk * PS + oy * Wp + x0) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

__global__ void k_round_tf32(float* __restrict__ p, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        p[i] = tc::to_tf32_rna(p[i]);
}

// The epilogue of one pixel for 4 consecutive filters, for the less common cases (unfused batchnorm,
// yolo logistic, activations other than leaky / linear); out of line to keep the kernel small.
static __device__ __noinline__ float4 tc_epilogue4_f(float4 o, int f0, int F, const ConvParams ep) {
    if (ep.yolo_classes > 0 && !ep.bn_mean) {
        // fused yolo activation (TYoloLayer.forward: logistic on entries 0, 1, 4..): the result
        // is rounded to TF32, so the logistic runs in single precision here (the FP32 path keeps
        // the reference's double-precision exp)
        const int period = ep.yolo_classes + 5;
        int e = f0 % period;
        float v[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int f = min(f0 + i, F - 1);
            float t = ep.bias ? __fadd_rn(v[i], ep.bias[f]) : v[i];
            if (e != 2 && e != 3) t = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-t)));
            v[i] = t;
            e = e + 1 == period ? 0 : e + 1;
        }
        return make_float4(v[0], v[1], v[2], v[3]);
    }
    // filters f0 .. f0+3, clamped to F-1 (values past the last filter are never stored)
    o.x = conv_epilogue(o.x, min(f0, F - 1), ep);
    o.y = conv_epilogue(o.y, min(f0 + 1, F - 1), ep);
    o.z = conv_epilogue(o.z, min(f0 + 2, F - 1), ep);
    o.w = conv_epilogue(o.w, min(f0 + 3, F - 1), ep);
    return o;
}

// CTAS = 2: a cluster of two CTAs on two SMs computes a 256-pixel x BN tile with
// tcgen05.mma.cta_group::2 (M = 256): each CTA loads its own 128 pixels of A and BN/2 filters of
// B, so each SM receives half the B bytes per FLOP of a single-CTA tile; the even CTA's thread
// issues the MMAs, each CTA's TMEM holds the accumulator rows of its own pixels.
template <int BN, int STAGES, int CTAS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_conv_tc(const __grid_constant__ TcMaps maps, const TcParams p) {
    constexpr int A_BYTES = TC_BM * TC_BK * 4;
    constexpr int BNC = BN / CTAS;  // filters of B held by this CTA
    constexpr int B_BYTES = BNC * TC_BK * 4;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr int NBOX_B = BNC / 32;  // 32-filter boxes of this CTA's B tile
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - ((unsigned)__cvta_generic_to_shared(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], tfull_bar[2], tempty_bar[2], drain_bar;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    __shared__ volatile int last_unit;  // split-K: this CTA's unit is the last of its tile

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const unsigned sbase = (unsigned)__cvta_generic_to_shared(smem);
    const int rank = CTAS == 2 ? (int)tc::cluster_rank() : 0;
    const int t_first = blockIdx.x / CTAS, t_step = gridDim.x / CTAS;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full_bar[s], 1);
            tc::mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull_bar[b], 1);
            tc::mbar_init(&tempty_bar[b], 8 * CTAS);  // one arrival per epilogue warp of the pair
        }
        tc::mbar_init(&drain_bar, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&maps.b)) : "memory");
    }
    if (warp == 1) tc::tmem_alloc_g<CTAS>(&tmem_base, 2 * BN);
    tc::tc_fence_before();
    __syncthreads();
    if (CTAS == 2) tc::cluster_sync();  // the peer's barriers exist before anything signals them
    tc::tc_fence_after();
    const uint32_t tmem0 = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int it = 0;
            bool ok = true;
            const long long c_start = clock64();
            long long c_wait = 0;
            for (int w = t_first; ok && w < p.units; w += t_step) {
                const int t = w / p.splits, z = w - t * p.splits;
                const int kb = z * p.kt_per_split, ke = min(p.ktiles, kb + p.kt_per_split);
                const int mt = t / p.tiles_n, nt = t - mt * p.tiles_n;
                const int n0 = mt * (TC_BM * CTAS) + rank * TC_BM;
                int bq[4], gq[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int n = n0 + 32 * j;
                    bq[j] = n / p.Lp;
                    gq[j] = (n - bq[j] * p.Lp) >> 5;
                }
                const bool split = bq[0] != bq[3] || gq[3] >= p.g_full;
                // kernel tap (r, s) and first channel c0 of k tile kt
                const int rs0 = kb / p.csteps;
                int r = rs0 / p.KW, s = rs0 - r * p.KW, c0 = (kb - rs0 * p.csteps) * TC_BK;
                for (int kt = kb; kt < ke; ++kt, ++it) {
                    const int st = it % STAGES, use = it / STAGES;
                    const long long c0w = clock64();
                    if (use > 0 && !tc::mbar_wait_bounded(&empty_bar[st], (use - 1) & 1, &abort_flag, p.status, 911)) {
                        ok = false;
                        break;
                    }
                    c_wait += clock64() - c0w;
                    if (rank == 0) tc::mbar_arrive_expect_tx(&full_bar[st], STAGE_BYTES * CTAS);
                    const int z0 = (s * p.NPH + p.phase[r]) * p.B;
                    const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + A_BYTES;
                    if (!split) {
                        tc::tma_load_4d_g<CTAS>(sa, &maps.a4[r], &full_bar[st], 0, c0, gq[0], z0 + bq[0]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            if (gq[j] < p.g_full)
                                tc::tma_load_4d_g<CTAS>(sa + j * TC_BOX_BYTES, &maps.a1[r], &full_bar[st], 0, c0, gq[j], z0 + bq[j]);
                            else
                                tc::tma_load_3d_g<CTAS>(sa + j * TC_BOX_BYTES, &maps.tail, &full_bar[st], gq[j] * 32, c0, z0 + bq[j]);
                        }
                    }
                    if (p.b_grouped) {
                        tc::tma_load_3d_g<CTAS>(sb, &maps.b, &full_bar[st], 0, kt * TC_BK, nt * (BN / 32) + rank * NBOX_B);
                    } else {
#pragma unroll
                        for (int j = 0; j < NBOX_B; ++j)
                            tc::tma_load_2d_g<CTAS>(sb + j * TC_BOX_BYTES, &maps.b, &full_bar[st],
                                                    nt * BN + rank * BNC + 32 * j, kt * TC_BK);
                    }
                    c0 += TC_BK;
                    if (c0 == p.C) {
                        c0 = 0;
                        if (++s == p.KW) s = 0, ++r;
                    }
                }
            }
            if (p.phases) {
                p.phases[blockIdx.x * 12 + 0] = clock64() - c_start;
                p.phases[blockIdx.x * 12 + 1] = c_wait;
            }
            // an abort: let the copies already issued land before the CTA exits (a pair's odd CTA
            // cannot see its copies complete: they are counted on the even CTA's barriers)
            if (!ok && rank == 0) {
                for (int j = it > STAGES ? it - STAGES : 0; j < it; ++j)
                    tc::mbar_wait_limit(&full_bar[j % STAGES], (j / STAGES) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (the pair's even CTA) ----------------
            constexpr uint32_t idesc = tc::idesc_tf32_mn(TC_BM * CTAS, BN);
            int it = 0, tl = 0;
            bool ok = true, issued = false;
            const long long c_start = clock64();
            long long c_wf = 0, c_we = 0;
            for (int w = t_first; ok && w < p.units; w += t_step, ++tl) {
                const int z = w % p.splits;
                const int kb = z * p.kt_per_split, ke = min(p.ktiles, kb + p.kt_per_split);
                const int buf = tl & 1, u = tl >> 1;
                long long c0w = clock64();
                if (u > 0 && !tc::mbar_wait_bounded(&tempty_bar[buf], (u - 1) & 1, &abort_flag, p.status, 912)) break;
                c_we += clock64() - c0w;
                tc::tc_fence_after();
                const uint32_t d = tmem0 + buf * BN;
                for (int kt = kb; kt < ke; ++kt, ++it) {
                    const int st = it % STAGES, use = it / STAGES;
                    c0w = clock64();
                    if (!tc::mbar_wait_bounded(&full_bar[st], use & 1, &abort_flag, p.status, 913)) {
                        ok = false;
                        break;
                    }
                    c_wf += clock64() - c0w;
                    tc::tc_fence_after();
                    const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 8; ++kk) {
                        const uint64_t da = tc::smem_desc_mn_sw128_32b(sa + kk * 1024, TC_BOX_BYTES, 512);
                        const uint64_t db = tc::smem_desc_mn_sw128_32b(sb + kk * 1024, TC_BOX_BYTES, 512);
                        tc::mma_tf32_g<CTAS>(d, da, db, idesc, (kt != kb || kk) ? 1u : 0u);
                    }
                    issued = true;
                    tc::mma_commit_g<CTAS>(&empty_bar[st]);
                }
                if (ok) tc::mma_commit_g<CTAS>(&tfull_bar[buf]);
            }
            if (p.phases) {
                p.phases[blockIdx.x * 12 + 2] = clock64() - c_start;
                p.phases[blockIdx.x * 12 + 3] = c_wf;
                p.phases[blockIdx.x * 12 + 4] = c_we;
            }
            if (issued) {  // every MMA has finished before TMEM is freed
                tc::mma_commit_g<CTAS>(&drain_bar);
                tc::mbar_wait_limit(&drain_bar, 0);
            }
        }
    } else {
        // ---------------- epilogue (warps 2-9) ----------------
        // TMEM lane = pixel, column = filter.  Per 16-filter slab a warp moves its 32 pixels x 16
        // filters through a per-warp shared tile (filter-major); then each lane takes a quad of 4
        // consecutive pixels of one filter: bias / activation / residual / TF32 rounding on a
        // float4 and one 16-byte store.  The two warps of a TMEM lane window split the slabs.
        const int quarter = warp & 3;      // TMEM lanes 32*quarter .. +31 (a warp's lane window)
        const int half = (warp - 2) >> 2;  // slabs half, half+2, ...
        float* stg = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES) + (warp - 2) * (16 * TC_STG_LD);
        float* bsm = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + TC_STG_BYTES) + (warp - 2) * 256;
        ConvParams ep;
        ep.bias = p.bias;
        ep.bn_scale = p.bn_scale;
        ep.bn_mean = p.bn_mean;
        ep.bn_var = p.bn_var;
        ep.act = p.act;
        ep.yolo_classes = p.yolo_classes;
        // the common epilogue (folded batchnorm: bias, then leaky or linear) is inline
        const bool fast = !p.bn_mean && p.yolo_classes == 0 && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
        const bool leaky = p.act == TB_ACT_LEAKY;
        const int qd = lane & 7, frow = lane >> 3;  // this lane's pixel quad and first slab row
        int tl = 0;
        const long long c_start = clock64();
        long long c_wt = 0, c_ld = 0, c_st = 0, c_sts = 0;
        for (int w = t_first; w < p.units; w += t_step, ++tl) {
            const int t = w / p.splits;
            const int buf = tl & 1, u = tl >> 1;
            const long long c0w = clock64();
            const bool ok = !abort_flag && tc::mbar_wait_bounded(&tfull_bar[buf], u & 1, &abort_flag, p.status, 914);
            c_wt += clock64() - c0w;
            // all 8 epilogue warps leave together (tcgen05.ld is warp-collective, and the split-K
            // path below meets at a named barrier)
            if (tc::epi_any(!ok)) break;
            tc::tc_fence_after();
            const bool from_tmem = p.splits == 1;
            if (!from_tmem) {
                // split-K: this unit's raw accumulator rows -> partial tile, then free TMEM
                float* prow = p.part + ((size_t)w * TC_BM + quarter * 32 + lane) * BN;
#pragma unroll 1
                for (int sl = half; sl < BN / 16; sl += 2) {
                    uint32_t pr[16];
                    tc::tmem_ld16_issue(tmem0 + buf * BN + ((uint32_t)(quarter * 32) << 16) + sl * 16, pr);
                    tc::tmem_wait16(pr);
#pragma unroll
                    for (int i = 0; i < 16; i += 4)
                        __stcg(reinterpret_cast<float4*>(prow + sl * 16 + i),
                               make_float4(__uint_as_float(pr[i]), __uint_as_float(pr[i + 1]),
                                           __uint_as_float(pr[i + 2]), __uint_as_float(pr[i + 3])));
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty_bar[buf]);
                // the last unit of the tile to arrive sums the partials in split order
                __threadfence();
                tc::epi_sync();
                if (warp == 2 && lane == 0) {
                    const int prev = atomicAdd(&p.tile_cnt[t], 1);
                    last_unit = prev == p.splits - 1;
                    if (last_unit) p.tile_cnt[t] = 0;  // ready for the next launch
                }
                tc::epi_sync();
                if (!last_unit) continue;
                __threadfence();
            }
            const int mt = t / p.tiles_n, nt = t - mt * p.tiles_n;
            // this lane's quad: pixels n .. n+3 of the padded grid (one row, one image)
            const int n = mt * (TC_BM * CTAS) + rank * TC_BM + quarter * 32 + qd * 4;
            const int b = n / p.Lp, q = n - b * p.Lp;
            const int oy = q / p.Wp, ox = q - oy * p.Wp;
            const int nvalid = (b < p.B && q < p.OHWp) ? max(0, min(4, p.OW - ox)) : 0;
            const long long pix = (long long)oy * p.OW + ox;
            float* yq = p.y + (nvalid ? b * p.y_bs + pix : 0);
            const float* rq = p.res ? p.res + (nvalid ? b * p.r_bs + pix : 0) : nullptr;
            const bool vec = nvalid == 4 && p.vec_out;
            const uint32_t taddr = tmem0 + buf * BN + ((uint32_t)(quarter * 32) << 16);
            // this tile's bias values in the warp's own shared row (one latency per tile)
            const bool sbias = fast && p.bias;
            if (sbias) {
                for (int i = lane; i < BN; i += 32) {
                    const int f = nt * BN + i;
                    bsm[i] = f < p.F ? __ldg(p.bias + f) : 0.f;
                }
            }
            uint32_t vr[16];
            const long long c0l = clock64();
            if (from_tmem && half < BN / 16) tc::tmem_ld16_issue(taddr + half * 16, vr);
#pragma unroll 1
            for (int sl = half; sl < BN / 16; sl += 2) {
                const long long cw0 = clock64();
                if (from_tmem) {
                    tc::tmem_wait16(vr);
                } else {  // sum of the tile's partials, split 0 first
                    float acc[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
                    const float* pb = p.part + ((size_t)t * p.splits * TC_BM + quarter * 32 + lane) * BN + sl * 16;
                    for (int zz = 0; zz < p.splits; ++zz) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4) {
                            const float4 q4 = __ldcg(reinterpret_cast<const float4*>(pb + (size_t)zz * TC_BM * BN + i));
                            acc[i] = __fadd_rn(acc[i], q4.x);
                            acc[i + 1] = __fadd_rn(acc[i + 1], q4.y);
                            acc[i + 2] = __fadd_rn(acc[i + 2], q4.z);
                            acc[i + 3] = __fadd_rn(acc[i + 3], q4.w);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) vr[i] = __float_as_uint(acc[i]);
                }
                const long long cw1 = clock64();
                c_ld += cw1 - cw0;
                const int fb = nt * BN + sl * 16;
                // 1. this lane's pixel, 16 independent filters: bias, activation (and, without a
                //    residual, the TF32 rounding), into the filter-major slab
                if (fast) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float o = __uint_as_float(vr[i]);
                        if (sbias) o = __fadd_rn(o, bsm[sl * 16 + i]);
                        if (leaky && o < 0.f) o = __fmul_rn(o, 0.1f);  // rounded to TF32 below
                        stg[i * TC_STG_LD + lane] = rq ? o : tc::to_tf32_rna(o);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; i += 4) {
                        float4 o = make_float4(__uint_as_float(vr[i]), __uint_as_float(vr[i + 1]),
                                               __uint_as_float(vr[i + 2]), __uint_as_float(vr[i + 3]));
                        o = tc_epilogue4_f(o, fb + i, p.F, ep);
                        stg[i * TC_STG_LD + lane] = rq ? o.x : tc::to_tf32_rna(o.x);
                        stg[(i + 1) * TC_STG_LD + lane] = rq ? o.y : tc::to_tf32_rna(o.y);
                        stg[(i + 2) * TC_STG_LD + lane] = rq ? o.z : tc::to_tf32_rna(o.z);
                        stg[(i + 3) * TC_STG_LD + lane] = rq ? o.w : tc::to_tf32_rna(o.w);
                    }
                }
                // the next slab's TMEM load runs while this slab is stored
                if (from_tmem && sl + 2 < BN / 16) tc::tmem_ld16_issue(taddr + (sl + 2) * 16, vr);
                __syncwarp();
                c_sts += clock64() - cw1;
                // 2. 16 filters x 8 pixel quads: lane -> quad qd of filter rows frow, frow+4, ...
                float4 r4[4];
                if (rq && vec) {  // all residual loads of the slab before any arithmetic
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int f = min(fb + frow + 4 * j, p.F - 1);
                        r4[j] = __ldg(reinterpret_cast<const float4*>(rq + (long long)f * p.OHW));
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int f = fb + frow + 4 * j;
                    float4 o = *reinterpret_cast<const float4*>(stg + (frow + 4 * j) * TC_STG_LD + qd * 4);
                    if (f < p.F && nvalid) {
                        const long long off = (long long)f * p.OHW;
                        if (vec) {
                            if (rq) {
                                o.x = tc::to_tf32_rna(__fadd_rn(o.x, r4[j].x));
                                o.y = tc::to_tf32_rna(__fadd_rn(o.y, r4[j].y));
                                o.z = tc::to_tf32_rna(__fadd_rn(o.z, r4[j].z));
                                o.w = tc::to_tf32_rna(__fadd_rn(o.w, r4[j].w));
                            }
                            __stcs(reinterpret_cast<float4*>(yq + off), o);
                        } else {
                            const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                if (e < nvalid) {
                                    float w = ov[e];
                                    if (rq) w = tc::to_tf32_rna(__fadd_rn(w, __ldg(rq + off + e)));
                                    yq[off + e] = w;
                                }
                            }
                        }
                    }
                }
                __syncwarp();
            }
            c_st += clock64() - c0l;
            if (!from_tmem) continue;  // the accumulator was released after the partial was written
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) {  // this warp's TMEM reads are done: the accumulator may be reused
                if (CTAS == 1) tc::mbar_arrive(&tempty_bar[buf]);
                else tc::mbar_arrive_cluster(&tempty_bar[buf], 0);
            }
        }
        if (p.phases && warp == 2 && lane == 0) {
            p.phases[blockIdx.x * 12 + 5] = clock64() - c_start;
            p.phases[blockIdx.x * 12 + 6] = c_wt;
            p.phases[blockIdx.x * 12 + 7] = tl;
            p.phases[blockIdx.x * 12 + 8] = c_ld;
            p.phases[blockIdx.x * 12 + 9] = c_st;
            p.phases[blockIdx.x * 12 + 10] = c_sts;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    // neither CTA of a pair leaves while the other may still read its shared memory (MMA
    // operands) or signal its barriers
    if (CTAS == 2) tc::cluster_sync();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc_g<CTAS>(tmem0, 2 * BN);
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

// fp32 tensor map, 128-byte swizzle with 32-byte atoms, zero fill out of bounds
int encode_map(CUtensorMap* m, const float* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapSwizzle sw) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(TB_ERR_CUDA, "tensor-core conv: cuTensorMapEncodeTiled is not available");
    cuuint64_t d[4], s[3];
    cuuint32_t bx[4], es[4] = {1, 1, 1, 1};
    for (int i = 0; i < rank; ++i) d[i] = dims[i], bx[i] = box[i];
    for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<float*>(base), d, s, bx, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TB_ERR_CUDA, "tensor-core conv: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TB_OK;
}

bool conv_tc_supported(const ConvGeom& g) {
    // one output pixel per image (a connected layer) would fill one row of a 32-pixel group
    if (g.KH > TC_MAX_KH || g.SY > 4 || g.OH * g.OW == 1) return false;
    TcPlan pl;
    tc_plan(g, &pl, 32);
    if (pl.mode == TC_TAPS && (g.KW > 8 || g.SX * 3 + (g.KW - 1) * g.DX + 1 > 32 || pl.NPH * g.B * g.C > 65535))
        return false;
    return pl.Cr <= 4096 && g.B * pl.Lp < ((int64_t)1 << 31) - TC_BM &&
           g.KW * pl.NPH * g.B <= 65535 && g.B * pl.Cr * pl.PS < ((int64_t)1 << 40);
}

// Replica floats of a plan (rounded to 64 floats, so the split-K partials after it stay aligned).
int64_t replica_floats(const ConvGeom& g, const TcPlan& pl) {
    int64_t n;
    if (pl.mode == TC_INPLACE) {
        // x that is not 16-byte aligned is copied into a tap replica instead
        const int64_t Wp = round_up(g.OW, 4);
        n = g.B * g.C * (round_up(g.OH * Wp, 32) + 32);
    } else if (pl.mode == TC_IM2COL) {
        n = g.B * pl.Cr * pl.PS;
    } else {
        n = g.KW * pl.NPH * g.B * g.C * pl.PS;
    }
    return round_up(n, 64);
}

// split-K partial tiles live after the replica, up to this many floats (128 MB)
constexpr int64_t TC_PART_CAP = (int64_t)1 << 25;

int64_t conv_tc_scratch_floats(const ConvGeom& g) {
    TcPlan pl;
    tc_plan(g, &pl, 32);
    return replica_floats(g, pl) + TC_PART_CAP;
}

template <int BN, int STAGES, int CTAS>
static int launch_bn(tb_ctx* ctx, const TcMaps& maps, const TcParams& p) {
    constexpr int smem = STAGES * (TC_BM * TC_BK * 4 + (BN / CTAS) * TC_BK * 4) + TC_STG_BYTES + TC_BIAS_BYTES + 1024;
    static std::mutex mu;
    static bool done[64] = {false};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !done[ctx->device]) {
            cudaError_t e = cudaFuncSetAttribute(k_conv_tc<BN, STAGES, CTAS>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(conv_tc)");
            done[ctx->device] = true;
        }
    }
    const int slots = CTAS == 1 ? ctx->sm_count : (ctx->sm_count & ~1);
    const int grid = (int)std::min<int64_t>((int64_t)p.units * CTAS, slots);
    if constexpr (CTAS == 1) {
        k_conv_tc<BN, STAGES, 1><<<grid, TC_THREADS, smem, ctx->stream>>>(maps, p);
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = ctx->stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, k_conv_tc<BN, STAGES, CTAS>, maps, p);
        if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(conv_tc pair)");
    }
    return check_launch("k_conv_tc");
}

// Tile shape (filters per tile, CTAs per tile) with the smallest modelled time: waves of tiles
// over the SMs (or SM pairs) x per-tile cycles, a k tile costing the larger of its MMA time
// (2*BN cycles per SM) and its operand delivery (A 16 KB + this CTA's part of B at ~64 B/cycle).
struct TcShape { int bn, ctas, splits; };

// Shapes measured by conv_tc_autotune, per device and geometry; a shape pinned for one launch
// by the autotuner itself.
static std::mutex g_tc_mu;
static std::map<std::vector<int64_t>, TcShape> g_tc_tuned;
static thread_local const TcShape* t_tc_pin = nullptr;

static std::vector<int64_t> tc_key(int device, const ConvGeom& g, bool xa) {
    return {device, g.B, g.C, g.H, g.W, g.F, g.KH, g.KW, g.SY, g.SX, g.PY, g.PX, g.DY, g.DX, g.x_bs, g.y_bs, xa};
}

static TcShape choose_shape(const ConvGeom& g, int64_t npix, int ktiles, int sms, int device, bool xa) {
    TcShape best{32, 1, 1};
    double best_cost = 1e300;
    if (t_tc_pin) return *t_tc_pin;
    if (const char* f = getenv("TB_TC_FORCE")) {  // test hook "BN,CTAS[,SPLITS]"
        int bn = 0, ct = 0, sp = 1;
        if (sscanf(f, "%d,%d,%d", &bn, &ct, &sp) >= 2 && (bn == 32 || bn == 64 || bn == 128 || bn == 256) &&
            (ct == 1 || (ct == 2 && bn >= 64)) && sp >= 1 && sp <= 8)
            return TcShape{bn, ct, ct == 1 ? sp : 1};
    }
    {
        std::lock_guard<std::mutex> lk(g_tc_mu);
        auto it = g_tc_tuned.find(tc_key(device, g, xa));
        if (it != g_tc_tuned.end()) return it->second;
    }
    // CTA pairs (cta_group::2) are built and tested but not picked: at the batch sizes of the
    // bench a pair tile leaves fewer tiles per SM, and its tail epilogue is not hidden
    for (int ct : {1}) {
        for (int bn : {32, 64, 128, 256}) {
            if (bn > round_up(g.F, 32) && bn != 32) break;
            if (ct == 2 && bn < 64) continue;
            const int64_t tiles = ceil_div(npix, (int64_t)TC_BM * ct) * ceil_div(g.F, bn);
            const int64_t slots = ct == 1 ? sms : sms / 2;
            const double kc = std::max(2.0 * bn, (16384.0 + bn * 128.0 / ct) / 64.0);
            const double cost = (double)ceil_div(tiles, slots) * (ktiles * kc + 2500.0);
            if (cost < best_cost * 0.999) best = TcShape{bn, ct, 1}, best_cost = cost;
        }
    }
    return best;
}

// The A operand of a conv (pixels x k) as TMA maps: x in place (1x1 stride-1 layers), tap
// replicas or im2col rows built into `scratch` (values rounded to TF32 when `round`).  Maps: a4
// copies 4 32-pixel groups x box_k channels, a1 one group, `tail` a bounds-checked group of an
// in-place x; swizzle `sw`.  Shared by the TF32 kernel and the FP32 TMA kernel.
int tc_prepare_a(tb_ctx* ctx, const ConvGeom& g, const float* x, float* scratch, bool round, int box_k, int cmul,
                 CUtensorMapSwizzle sw, CUtensorMap* a4, CUtensorMap* a1, CUtensorMap* tail, TcPlan* plo,
                 int* kmaps_o, int* g_full_o, int64_t* launches) {
    TcPlan& pl = *plo;
    tc_plan(g, &pl, cmul);
    if (pl.mode == TC_INPLACE && !aligned16(x)) {  // same result through a (1-tap) replica
        ConvGeom g2 = g;
        g2.x_bs = g.x_bs + 1;  // any stride that is not a multiple of 4 selects the replica plan
        tc_plan(g2, &pl, cmul);
    }
    int r;
    int& kmaps = *kmaps_o;  // A maps in use (one per distinct kernel row for tap replicas)
    int& g_full = *g_full_o;
    kmaps = 1;
    g_full = 1 << 30;
    const uint32_t b4[4] = {32, (uint32_t)box_k, 4, 1}, b1[4] = {32, (uint32_t)box_k, 1, 1};
    if (pl.mode == TC_INPLACE) {
        // x itself: (32 pixels, channel, 32-pixel group, image); a partial last group of an
        // image goes through the bounds-checked (pixel, channel, image) tail map
        const int64_t HW = g.H * g.W;
        g_full = (int)(HW / 32);
        const uint64_t dims[4] = {32, (uint64_t)g.C, (uint64_t)std::max<int64_t>(g_full, 1), (uint64_t)g.B};
        const uint64_t st[3] = {(uint64_t)HW * 4, 128, (uint64_t)g.x_bs * 4};
        r = encode_map(&a4[0], x, 4, dims, st, b4, sw);
        if (r == TB_OK) r = encode_map(&a1[0], x, 4, dims, st, b1, sw);
        const uint64_t td[3] = {(uint64_t)HW, (uint64_t)g.C, (uint64_t)g.B};
        const uint64_t ts[2] = {(uint64_t)HW * 4, (uint64_t)g.x_bs * 4};
        const uint32_t tb[3] = {32, (uint32_t)box_k, 1};
        if (r == TB_OK) r = encode_map(tail, x, 3, td, ts, tb, sw);
        if (r != TB_OK) return r;
    } else {
        if (!scratch || !aligned16(scratch))
            return fail(TB_ERR_INVALID, "conv: this geometry needs a 16-byte-aligned replica buffer");
        int64_t Z;
        if (pl.mode == TC_IM2COL) {
            Z = g.B;
            const int64_t total = g.B * pl.Cr * g.OH * (pl.Wp / 4);
            (round ? k_tc_repack_im2col<true> : k_tc_repack_im2col<false>)<<<grid_for(total, 256, ctx->sm_count, 4), 256, 0, ctx->stream>>>(
                x, g.x_bs, scratch, (int)g.B, (int)g.C, (int)g.H, (int)g.W, (int)g.KH, (int)g.KW, (int)g.SY,
                (int)g.SX, (int)g.DY, (int)g.DX, (int)g.PY, (int)g.PX, g.rsc ? 1 : 0, (int)g.Cpad,
                (int)(g.rsc ? g.KH * g.KW * g.Cpad : g.C * g.KH * g.KW), (int)pl.Cr, (int)g.OH, (int)g.OW,
                (int)pl.Wp, (int)pl.PS);
        } else {
            Z = g.KW * pl.NPH * g.B;
            const int64_t rows4 = pl.Hrep * (pl.Wp / 4);
            dim3 rg((unsigned)ceil_div(rows4, 256), (unsigned)(pl.NPH * g.B * g.C));
            auto kern = (g.SX == 1 && g.DX == 1)   ? (round ? k_tc_repack_taps<1, 1, true> : k_tc_repack_taps<1, 1, false>)
                        : (g.SX == 2 && g.DX == 1) ? (round ? k_tc_repack_taps<2, 1, true> : k_tc_repack_taps<2, 1, false>)
                                                   : (round ? k_tc_repack_taps<0, 0, true> : k_tc_repack_taps<0, 0, false>);
            kern<<<rg, 256, 0, ctx->stream>>>(x, g.x_bs, scratch, (int)g.B, (int)g.C, (int)g.H, (int)g.W, (int)g.KW,
                                              (int)g.SY, (int)g.SX, (int)g.DX, (int)g.PX, (int)pl.NPH,
                                              (int)pl.pad_top, (int)pl.Hrep, (int)pl.Wp, (int)g.OW, (int)pl.PS);
            kmaps = (int)g.KH;
        }
        r = check_launch("k_tc_repack");
        if (r != TB_OK) return r;
        if (launches) ++*launches;
        // one view per kernel row: the base moves rowoff(r) replica rows down; a 32-pixel group
        // at a valid pixel then stays inside its plane (PS has 32 elements of slack)
        const uint64_t dims[4] = {32, (uint64_t)pl.Cr, (uint64_t)((pl.PS - 32) / 32), (uint64_t)Z};
        const uint64_t st[3] = {(uint64_t)pl.PS * 4, 128, (uint64_t)(pl.Cr * pl.PS) * 4};
        for (int k = 0; k < kmaps; ++k) {
            const float* base = scratch + (int64_t)pl.rowoff[k] * pl.Wp;
            r = encode_map(&a4[k], base, 4, dims, st, b4, sw);
            if (r == TB_OK) r = encode_map(&a1[k], base, 4, dims, st, b1, sw);
            if (r != TB_OK) return r;
        }
    }

    return TB_OK;
}

int conv_tc_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                   const float* bn_scale, const float* bn_mean, const float* bn_var, const float* res, float* y,
                   int act, int yolo_classes, float* scratch, int64_t* launches, unsigned long long* phases) {
    if (!conv_tc_supported(g)) return fail(TB_ERR_UNSUPPORTED, "tensor-core conv: unsupported geometry");
    if (g.B == 0) return TB_OK;
    TcPlan pl;
    TcMaps maps;
    memset(&maps, 0, sizeof(maps));
    int kmaps = 1, g_full = 1 << 30;
    int r = tc_prepare_a(ctx, g, x, scratch, true, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, maps.a4, maps.a1,
                         &maps.tail, &pl, &kmaps, &g_full, launches);
    if (r != TB_OK) return r;
    TcParams p{};
    p.bias = bias; p.bn_scale = bn_scale; p.bn_mean = bn_mean; p.bn_var = bn_var;
    p.res = res; p.y = y; p.status = ctx->d_status; p.phases = phases;
    p.B = (int)g.B; p.C = (int)pl.Cr; p.F = (int)g.F; p.OW = (int)(pl.mode == TC_INPLACE ? pl.Wp : g.OW);
    p.OH = (int)g.OH;
    p.Wp = (int)pl.Wp;
    p.NPH = (int)pl.NPH;
    p.Lp = (int)pl.Lp;
    p.OHWp = (int)(pl.mode == TC_INPLACE ? pl.Wp : g.OH * pl.Wp);
    p.OHW = (int)(g.OH * g.OW);
    p.g_full = g_full;
    {
        const bool ow4 = pl.mode == TC_INPLACE || g.OW % 4 == 0;
        p.vec_out = ow4 && (g.OH * g.OW) % 4 == 0 && g.y_bs % 4 == 0 && aligned16(y) &&
                    (!res || (g.r_bs % 4 == 0 && aligned16(res)));
    }
    p.csteps = (int)(pl.Cr / TC_BK);
    const int taps = pl.mode == TC_TAPS ? (int)(g.KH * g.KW) : 1;
    p.KW = pl.mode == TC_TAPS ? (int)g.KW : 1;
    p.ktiles = taps * p.csteps;
    p.y_bs = g.y_bs; p.r_bs = g.r_bs;
    p.act = act; p.yolo_classes = yolo_classes;
    for (int i = 0; i < TC_MAX_KH; ++i) p.phase[i] = pl.phase[i];
    const TcShape sh = choose_shape(g, g.B * p.Lp, p.ktiles, ctx->sm_count, ctx->device, aligned16(x));
    const int bn = sh.bn;
    const int64_t tiles_m = ceil_div(g.B * p.Lp, (int64_t)TC_BM * sh.ctas);
    p.tiles_n = (int)ceil_div(g.F, bn);
    const int64_t tiles = tiles_m * p.tiles_n;
    if (tiles >= ((int64_t)1 << 30)) return fail(TB_ERR_UNSUPPORTED, "tensor-core conv: too many tiles");
    p.tiles_total = (int)tiles;
    // split-K over units of kt_per_split k tiles (one CTA per tile; the counters and the partial
    // buffer bound it)
    int splits = std::min(sh.splits, p.ktiles);
    if (sh.ctas != 1 || !scratch || tiles > ctx->tile_cnt_len ||
        tiles * splits * TC_BM * bn > TC_PART_CAP)
        splits = 1;
    p.kt_per_split = (int)ceil_div(p.ktiles, splits);
    p.splits = (int)ceil_div(p.ktiles, p.kt_per_split);
    p.units = p.tiles_total * p.splits;
    p.part = p.splits > 1 ? scratch + replica_floats(g, pl) : nullptr;
    p.tile_cnt = ctx->tile_cnt;
    p.b_grouped = g.Mpad % 32 == 0;
    if (p.b_grouped) {  // (32 filters, k, filter group), one box of bn/32 groups per stage
        const uint64_t dims[3] = {32, (uint64_t)g.Kpad, (uint64_t)(g.Mpad / 32)};
        const uint64_t st[2] = {(uint64_t)g.Mpad * 4, 128};
        const uint32_t box[3] = {32, 32, (uint32_t)(bn / 32 / sh.ctas)};  // this CTA's filters
        r = encode_map(&maps.b, wp, 3, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    } else {
        const uint64_t dims[2] = {(uint64_t)g.Mpad, (uint64_t)g.Kpad};
        const uint64_t st[1] = {(uint64_t)g.Mpad * 4};
        const uint32_t box[2] = {32, 32};
        r = encode_map(&maps.b, wp, 2, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    }
    if (r != TB_OK) return r;
    if (sh.ctas == 1) {
        switch (bn) {
        case 32: r = launch_bn<32, 8, 1>(ctx, maps, p); break;
        case 64: r = launch_bn<64, 8, 1>(ctx, maps, p); break;
        case 128: r = launch_bn<128, 6, 1>(ctx, maps, p); break;
        default: r = launch_bn<256, 4, 1>(ctx, maps, p); break;
        }
    } else {
        switch (bn) {
        case 64: r = launch_bn<64, 8, 2>(ctx, maps, p); break;
        case 128: r = launch_bn<128, 8, 2>(ctx, maps, p); break;
        default: r = launch_bn<256, 6, 2>(ctx, maps, p); break;
        }
    }
    if (r != TB_OK) return r;
    if (launches) ++*launches;
    return TB_OK;
}


// ---------------------------------------------------------------------------------------
// Diagnostic: tcgen05.mma kind::tf32 issue rate on shared-memory operands already in place
// (no loads), M = 128, N = 256, K = 8, in the two operand layouts: both MN-major with the
// 32-byte-atom 128-byte swizzle (what k_conv_tc uses), or both K-major with the 128-byte
// swizzle.  One CTA per SM; batches of 64 MMAs committed to an mbarrier; cycles of the batches
// after the first.
__global__ void __launch_bounds__(128, 1) k_mma_rate(int kmajor, int batches, unsigned long long* cycles) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - ((unsigned)__cvta_generic_to_shared(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < (128 + 256) * 32; i += blockDim.x) reinterpret_cast<float*>(smem)[i] = 0.f;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    if (warp == 0) tc::tmem_alloc(&tmem_base, 256);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (threadIdx.x == 0) {
        const unsigned sa = (unsigned)__cvta_generic_to_shared(smem), sb = sa + 128 * 32 * 4;
        uint32_t idesc = tc::idesc_tf32_mn(128, 256);
        if (kmajor) idesc &= ~((1u << 15) | (1u << 16));
        long long t0 = 0;
        for (int b = 0; b < batches; ++b) {
            if (b == 1) t0 = clock64();
            for (int i = 0; i < 64; ++i) {
                const int kk = i & 3;
                uint64_t da, db;
                if (kmajor) {  // K-major SW128: rows of 32 fp32 along K, 8-row groups 1024 B apart
                    da = tc::smem_desc_mn_sw128_32b(sa + kk * 32, 16, 1024);
                    db = tc::smem_desc_mn_sw128_32b(sb + kk * 32, 16, 1024);
                    da = (da & ~(7ull << 61)) | (2ull << 61);
                    db = (db & ~(7ull << 61)) | (2ull << 61);
                } else {
                    da = tc::smem_desc_mn_sw128_32b(sa + kk * 1024, 4096, 512);
                    db = tc::smem_desc_mn_sw128_32b(sb + kk * 1024, 4096, 512);
                }
                tc::mma_tf32(tmem_base, da, db, idesc, i ? 1u : 0u);
            }
            tc::mma_commit(&bar);
            tc::mbar_wait_limit(&bar, b & 1);
        }
        cycles[blockIdx.x] = clock64() - t0;
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, 256);
    }
}

int conv_tc_mma_rate(tb_ctx* ctx, int kmajor, double* tflops_at_clock, double* cycles_per_mma) {
    const int batches = 65, smem = (128 + 256) * 32 * 4 + 1024;
    unsigned long long* d = nullptr;
    TB_CHECK_CUDA(cudaMalloc(&d, ctx->sm_count * sizeof(unsigned long long)));
    cudaFuncSetAttribute(k_mma_rate, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k_mma_rate<<<ctx->sm_count, 128, smem, ctx->stream>>>(kmajor, batches, d);
    std::vector<unsigned long long> h(ctx->sm_count);
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), d, h.size() * 8, cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e, "mma rate probe");
    double c = 0;
    for (auto v : h) c += (double)v;
    c /= h.size();
    *cycles_per_mma = c / ((batches - 1) * 64.0);
    // 2*128*256*8 FLOPs per MMA, per SM, at 1.965 GHz on every SM
    *tflops_at_clock = 2.0 * 128 * 256 * 8 / *cycles_per_mma * 1.965e9 * ctx->sm_count / 1e12;
    return TB_OK;
}

// Time every tile shape (filters per tile, CTAs per tile) of this geometry on the given buffers
// (bias, batchnorm, residual off) and keep the fastest for later launches.  Blocks; grows the
// workspace for the replica (not during stream capture).
int conv_tc_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, float* y) {
    if (g.B == 0 || !conv_tc_supported(g)) return TB_OK;
    int r = ensure_workspace(ctx, (size_t)conv_tc_scratch_floats(g) * sizeof(float));
    if (r != TB_OK) return r;
    std::vector<TcShape> cands;
    const int64_t ktiles = (g.rsc && g.C % 32 == 0) ? g.KH * g.KW * (g.C / 32) : round_up(g.Kpad, 32) / 32;
    for (int ct : {1, 2})
        for (int bn : {32, 64, 128, 256}) {
            if (ct == 2 && bn < 64) continue;
            if (bn > round_up(g.F, 32) && bn != 32) continue;
            for (int sp : {1, 2, 3, 4}) {
                if (sp > 1 && (ct != 1 || ktiles < 4 * sp)) continue;
                cands.push_back(TcShape{bn, ct, sp});
            }
        }
    cudaEvent_t e0, e1;
    TB_CHECK_CUDA(cudaEventCreate(&e0));
    TB_CHECK_CUDA(cudaEventCreate(&e1));
    float best_ms = 1e30f;
    TcShape best = cands[0];
    for (const TcShape& c : cands) {
        t_tc_pin = &c;
        float* ws = reinterpret_cast<float*>(ctx->ws);
        r = conv_tc_launch(ctx, g, x, wp, nullptr, nullptr, nullptr, nullptr, nullptr, y, TB_ACT_LINEAR, 0, ws, nullptr);
        stream_delay_us(ctx, 200);  // the timed launches queue behind it: device time only
        cudaEventRecord(e0, ctx->stream);
        for (int rep = 0; rep < 3 && r == TB_OK; ++rep)
            r = conv_tc_launch(ctx, g, x, wp, nullptr, nullptr, nullptr, nullptr, nullptr, y, TB_ACT_LINEAR, 0, ws,
                               nullptr);
        cudaEventRecord(e1, ctx->stream);
        t_tc_pin = nullptr;
        cudaError_t e = cudaEventSynchronize(e1);
        if (r != TB_OK) break;
        if (e != cudaSuccess) { r = cuda_fail(e, "tensor-core autotune"); break; }
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (getenv("TB_AUTOTUNE_VERBOSE"))
            fprintf(stderr, "tc autotune C%lld H%lld F%lld k%lld s%lld B%lld: bn %d ctas %d splits %d: %.4f ms\n",
                    (long long)g.C, (long long)g.H, (long long)g.F, (long long)g.KH, (long long)g.SY,
                    (long long)g.B, c.bn, c.ctas, c.splits, ms / 3);
        if (ms < best_ms) best_ms = ms, best = c;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (r != TB_OK) return r;
    std::lock_guard<std::mutex> lk(g_tc_mu);
    g_tc_tuned[tc_key(ctx->device, g, aligned16(x))] = best;
    return TB_OK;
}

int conv_tc_round_weights(tb_ctx* ctx, float* packed, int64_t n) {
    if (n <= 0) return TB_OK;
    k_round_tf32<<<grid_for(n, 256, ctx->sm_count), 256, 0, ctx->stream>>>(packed, n);
    return check_launch("k_round_tf32");
}

}  // namespace tbi
