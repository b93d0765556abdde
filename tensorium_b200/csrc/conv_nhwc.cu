// conv_nhwc.cu -- TF32 tensor-core convolution on NHWC activations, A operand fetched by TMA in
// im2col mode.
//
// The NCHW tensor-core kernel (conv_tc.cu) first copies its input into tap replicas, because a
// tap shift along W moves an NCHW pixel row by one float, which no TMA box can start at. With the
// channels innermost (NHWC) the pixel is an outer dimension: TMA's im2col mode walks 128
// consecutive output pixels (across row and image ends) and loads, for one kernel tap and 32
// channels, each pixel's input window start shifted by the tap offset, zero-filling whatever falls
// in the padding. So the operand tile arrives K-major (32 channels = one 128-byte swizzled row per
// pixel) straight from the activations: no replica pass, no padded pixel grid.
//
// Roles as in the NCHW kernel: warp 0 one thread issues the TMA ring (A by im2col, B = packed
// weights [F][KH][KW][Cp] K-major by a tiled 2-D map); warp 1 owns TMEM and one thread issues
// tcgen05.mma kind::tf32 (M = 128 pixels, N = BN filters, K = 8) into one of two accumulators;
// warps 2-9 run the epilogue of the previous tile while the next one accumulates. TMEM lane =
// pixel, so a thread holds 16 consecutive filters of one pixel after a 16-column load: NHWC
// stores are four 16-byte vectors per thread, NCHW stores (the yolo head convs) one float per
// filter with the warp's 32 lanes writing 32 consecutive pixels. No shared-memory transpose.
// Outputs are rounded to TF32 (nearest), so the next layer's operands are exact TF32 values.
// Every wait is bounded; on timeout the kernel sets the context status word, drains what is in
// flight, frees TMEM and returns.
#include "conv_tc.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <vector>

namespace tbi {

namespace {

constexpr int NH_BM = 128, NH_BK = 32, NH_THREADS = 320;
constexpr int NH_A_BYTES = NH_BM * NH_BK * 4;  // 16 KB: 128 pixels x 32 channels

struct NhwcParams {
    const float* __restrict__ bias;
    const float* __restrict__ res;  // NHWC, at the residual's channel offset (or null)
    float* __restrict__ y;          // NHWC: at the output's channel offset; NCHW: image 0, filter 0
    int* status;
    unsigned long long* phases;
    long long npix;                 // B * OH * OW
    long long y_bs;                 // NCHW output: floats between images
    int OW, OHW, SX, SY, PX, PY, KW, DX, DY;
    int F, csteps, ktiles;
    int tiles_n, tiles_total;
    // Work units: tiles 0 .. dp_tiles - 1 whole (unit w = tile w), then each remaining tile as
    // `splits` K ranges of kt_per_split k tiles (unit dp_tiles + q: tile dp_tiles + q / splits,
    // range q % splits), so the last partial wave of tiles is spread over every SM.
    int dp_tiles, splits, kt_per_split, units;
    float* part;                      // split units' partial tiles [q][BN / 4][128 pixels][4 filters]
    int* tile_cnt;                    // split-K arrival counters, one per tile, left at 0
    int out_nchw;
    int y_ps, r_ps;                 // NHWC pixel strides (floats) of the output and residual
    int vec;                        // NHWC: y / res 16-byte aligned and strides % 4 == 0
    int tma_out;                    // NHWC output written by TMA tensor stores (maps.y)
    int act, yolo_classes;
};

struct NhwcMaps {
    CUtensorMap a;  // im2col view of x: (C, W, H, N), 32 channels x 128 pixels per copy
    CUtensorMap b;  // packed weights (k, filter), box 32 x BN (pair mode: the (hi, hi) operand)
    CUtensorMap b2; // pair mode: the (lo, lo) weight operand
    CUtensorMap y;  // NHWC output (filter, pixel), box 16 x 32, 64-byte swizzle (tma_out)
};

// unit w of a launch: its tile, k tile range and partial slot (-1: a whole tile, stored directly)
struct NhUnit {
    int t, kb, ke, slot;
};

__device__ __forceinline__ NhUnit nh_unit(const NhwcParams& p, int w) {
    if (w < p.dp_tiles) return NhUnit{w, 0, p.ktiles, -1};
    const int q = w - p.dp_tiles, tq = q / p.splits, z = q - tq * p.splits;
    const int kb = z * p.kt_per_split;
    return NhUnit{p.dp_tiles + tq, kb, min(p.ktiles, kb + p.kt_per_split), q};
}

constexpr int NH_STG_BYTES = 8 * 2 * 32 * 64;  // per epilogue warp: two 32-pixel x 16-filter slabs

// K-major, 128-byte swizzle (layout type 2): rows of 32 fp32 along K, 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: 8 rows x 128 bytes
    d |= (uint64_t)1 << 46;            // version (Blackwell)
    d |= (uint64_t)2 << 61;            // SWIZZLE_128B
    return d;
}

// instruction descriptor: F32 accumulate, TF32 A and B, both K-major, M x N
__host__ __device__ constexpr uint32_t idesc_tf32_k(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// the same for kind::f16 with BF16 A and B
__host__ __device__ constexpr uint32_t idesc_bf16_k(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tma_load_im2col_4d(unsigned dst, const void* tmap, uint64_t* bar, int c, int w,
                                                   int h, int n, uint16_t ow, uint16_t oh) {
    unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(b), "r"(c), "r"(w), "r"(h), "r"(n), "h"(ow), "h"(oh)
        : "memory");
}

// the same for a CTA pair: the copy lands in this CTA's shared memory and its bytes are counted on
// the mbarrier of the pair's even CTA
template <int CTAS>
__device__ __forceinline__ void tma_load_im2col_4d_g(unsigned dst, const void* tmap, uint64_t* bar, int c, int w,
                                                     int h, int n, uint16_t ow, uint16_t oh) {
    if constexpr (CTAS == 1) {
        tma_load_im2col_4d(dst, tmap, bar, c, w, h, n, ow, oh);
    } else {
        asm volatile(
            "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};\n" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(tmap)), "r"(tc::tma_bar<2>(bar)), "r"(c), "r"(w), "r"(h), "r"(n), "h"(ow),
            "h"(oh)
            : "memory");
    }
}

// shared -> global tensor store of one box, tracked as a bulk group of this thread
__device__ __forceinline__ void tma_store_2d(const void* tmap, unsigned src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}

// wait until at most n of this thread's bulk groups still read their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ float nh_act(float o, int f, const NhwcParams& p) {
    if (p.yolo_classes > 0) {  // fused yolo activation (logistic on entries 0, 1, 4..), single precision
        const int e = f % (p.yolo_classes + 5);
        return (e != 2 && e != 3) ? __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-o))) : o;
    }
    if (p.act == TB_ACT_LEAKY) return o < 0.f ? __fmul_rn(o, 0.1f) : o;  // rounded to TF32 after
    if (p.act == TB_ACT_LINEAR) return o;
    return tb_activate_dev(o, p.act);
}

// PAIR: BF16-split operands. The 32-bit activation slots hold bf16 (hi, lo) pairs, so the same
// im2col box is a K-major tile of 64 bf16 (32 channels x (hi, lo)); the weights come as two
// operands (hi, hi) and (lo, lo), and per 32 channels 4 + 4 kind::f16 MMAs (K = 16) accumulate
// hi*w_hi + lo*w_hi + hi*w_lo + lo*w_lo = (hi + lo) * (w_hi + w_lo) in FP32.
//
// CTAS = 2: a cluster of two CTAs on two SMs computes a 256-pixel x BN tile with
// tcgen05.mma.cta_group::2 (M = 256). Each CTA loads its own 128 pixels of A and BN / 2 filters of
// B (the MMA reads B half from each CTA's shared memory), so an SM receives 3/4 (BN = 256) of the
// operand bytes per FLOP of a single-CTA tile; the even CTA's thread issues the MMAs and waits for
// both CTAs' copies on its own barriers; each CTA's TMEM holds the accumulator rows of its pixels
// and its epilogue warps store them. No split-K for pairs.
template <int BN, int STAGES, bool PAIR, int CTAS>
__global__ void __launch_bounds__(NH_THREADS, 1) k_conv_nhwc(const __grid_constant__ NhwcMaps maps, const NhwcParams p) {
    constexpr int BNC = BN / CTAS;  // filters of B held by this CTA
    constexpr int B_BYTES = BNC * NH_BK * 4;
    constexpr int STAGE_BYTES = NH_A_BYTES + (PAIR ? 2 : 1) * B_BYTES;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - ((unsigned)__cvta_generic_to_shared(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], tfull_bar[2], tempty_bar[2], drain_bar;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    __shared__ volatile int last_unit;  // split-K: this CTA's unit is the last of its tile

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (p.phases && tid == 0) p.phases[blockIdx.x * 12 + 10] = tc::global_ns();  // diagnostics: CTA start
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
            tc::mbar_init(&tempty_bar[b], 8 * CTAS);  // one arrival per epilogue warp (of the pair)
        }
        tc::mbar_init(&drain_bar, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&maps.a)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&maps.b)) : "memory");
    }
    if (warp == 1) tc::tmem_alloc_g<CTAS>(&tmem_base, 2 * BN);
    tc::tc_fence_before();
    __syncthreads();
    if (CTAS == 2) tc::cluster_sync();  // the peer's barriers exist before anything signals them
    tc::tc_fence_after();
    const uint32_t tmem0 = tmem_base;
    TB_GRID_DEP_ENTRY();  // set-up above overlaps the previous kernel's tail; activations only after it

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int it = 0;
            bool ok = true;
            const long long c_start = clock64();
            long long c_wait = 0;
            for (int w = t_first; ok && w < p.units; w += t_step) {
                const NhUnit un = nh_unit(p, w);
                const int t = un.t, kb = un.kb, ke = un.ke;
                const int mt = t / p.tiles_n, nt = t - mt * p.tiles_n;
                const long long m0 = (long long)mt * (NH_BM * CTAS) + rank * NH_BM;
                const int n0 = (int)(m0 / p.OHW);
                const int q = (int)(m0 - (long long)n0 * p.OHW);
                const int oy = q / p.OW, ox = q - oy * p.OW;
                const int w0 = ox * p.SX - p.PX, h0 = oy * p.SY - p.PY;
                const int rs0 = kb / p.csteps;  // tap (r, s) and channel step of k tile kb
                int r = rs0 / p.KW, s = rs0 - r * p.KW, c0 = kb - rs0 * p.csteps;
                for (int kt = kb; kt < ke; ++kt, ++it) {
                    const int st = it % STAGES, use = it / STAGES;
                    const long long c0w = clock64();
                    if (use > 0 && !tc::mbar_wait_bounded(&empty_bar[st], (use - 1) & 1, &abort_flag, p.status, 921)) {
                        ok = false;
                        break;
                    }
                    c_wait += clock64() - c0w;
                    if (rank == 0) tc::mbar_arrive_expect_tx(&full_bar[st], STAGE_BYTES * CTAS);
                    const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + NH_A_BYTES;
                    tma_load_im2col_4d_g<CTAS>(sa, &maps.a, &full_bar[st], c0 * NH_BK, w0, h0, n0,
                                               (uint16_t)(s * p.DX), (uint16_t)(r * p.DY));
                    tc::tma_load_2d_g<CTAS>(sb, &maps.b, &full_bar[st], kt * NH_BK, nt * BN + rank * BNC);
                    if (PAIR)
                        tc::tma_load_2d_g<CTAS>(sb + B_BYTES, &maps.b2, &full_bar[st], kt * NH_BK, nt * BN + rank * BNC);
                    if (++c0 == p.csteps) {  // next 32-channel step, then the next tap
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
            constexpr uint32_t idesc = PAIR ? idesc_bf16_k(NH_BM * CTAS, BN) : idesc_tf32_k(NH_BM * CTAS, BN);
            int it = 0, tl = 0;
            bool ok = true, issued = false;
            const long long c_start = clock64();
            long long c_wf = 0, c_we = 0;
            for (int w = t_first; ok && w < p.units; w += t_step, ++tl) {
                const NhUnit un = nh_unit(p, w);
                const int kb = un.kb, ke = un.ke;
                const int buf = tl & 1, u = tl >> 1;
                long long c0w = clock64();
                if (u > 0 && !tc::mbar_wait_bounded(&tempty_bar[buf], (u - 1) & 1, &abort_flag, p.status, 922)) break;
                c_we += clock64() - c0w;
                tc::tc_fence_after();
                const uint32_t d = tmem0 + buf * BN;
                for (int kt = kb; kt < ke; ++kt, ++it) {
                    const int st = it % STAGES, use = it / STAGES;
                    c0w = clock64();
                    if (!tc::mbar_wait_bounded(&full_bar[st], use & 1, &abort_flag, p.status, 923)) {
                        ok = false;
                        break;
                    }
                    c_wf += clock64() - c0w;
                    tc::tc_fence_after();
                    const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + NH_A_BYTES;
                    if (PAIR) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc::mma_bf16_g<CTAS>(d, smem_desc_k_sw128(sa + kk * 32), smem_desc_k_sw128(sb + kk * 32),
                                                 idesc, (kt != kb || kk) ? 1u : 0u);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc::mma_bf16_g<CTAS>(d, smem_desc_k_sw128(sa + kk * 32),
                                                 smem_desc_k_sw128(sb + B_BYTES + kk * 32), idesc, 1u);
                    } else {
#pragma unroll
                        for (int kk = 0; kk < NH_BK / 8; ++kk)
                            tc::mma_tf32_g<CTAS>(d, smem_desc_k_sw128(sa + kk * 32), smem_desc_k_sw128(sb + kk * 32),
                                                 idesc, (kt != kb || kk) ? 1u : 0u);
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
        const int quarter = warp & 3;      // TMEM lanes 32*quarter .. +31
        const int half = (warp - 2) >> 2;  // which half of the tile's filters this warp takes
        // this warp's two staging slabs (32 pixel rows x 64 bytes each, 64-byte swizzle: the
        // 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3), which the TMA store undoes)
        const unsigned stg0 = sbase + STAGES * STAGE_BYTES + (warp - 2) * 2 * 2048;
        // the common epilogue (bias, then leaky or linear, residual) is decided once here: read
        // per value from the parameter space, these flags cost a dependent constant load each
        const bool fast = p.yolo_classes == 0 && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
        const bool leaky = p.act == TB_ACT_LEAKY;
        const float* __restrict__ bias = p.bias;
        const int Fm1 = p.F - 1;
        const int period = p.yolo_classes > 0 ? p.yolo_classes + 5 : 0;
        int sbuf = 0;
        int tl = 0;
        const long long c_start = clock64();
        long long c_wt = 0, c_st = 0, c_ldw = 0;
        for (int w = t_first; w < p.units; w += t_step, ++tl) {
            const NhUnit un = nh_unit(p, w);
            const int t = un.t;
            const int buf = tl & 1, u = tl >> 1;
            const long long c0w = clock64();
            const bool ok = !abort_flag && tc::mbar_wait_bounded(&tfull_bar[buf], u & 1, &abort_flag, p.status, 924);
            c_wt += clock64() - c0w;
            if (tc::epi_any(!ok)) break;  // tcgen05.ld is warp-collective: all epilogue warps leave together
            tc::tc_fence_after();
            const bool from_tmem = un.slot < 0;
            if (!from_tmem) {
                // split unit: its raw accumulator -> its partial tile in groups of 4 filters (a warp's
                // 32 lanes write 32 consecutive pixels' float4s: 512-byte stores), then free TMEM
                float4* prow = reinterpret_cast<float4*>(p.part + (size_t)un.slot * NH_BM * BN) + quarter * 32 + lane;
                const uint32_t ta = tmem0 + buf * BN + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
                for (int sl = half; sl < BN / 16; sl += 2) {
                    uint32_t pr[16];
                    tc::tmem_ld16_issue(ta + sl * 16, pr);
                    tc::tmem_wait16(pr);
#pragma unroll
                    for (int i = 0; i < 16; i += 4)
                        __stcg(prow + (size_t)((sl * 16 + i) >> 2) * NH_BM,
                               make_float4(__uint_as_float(pr[i]), __uint_as_float(pr[i + 1]),
                                           __uint_as_float(pr[i + 2]), __uint_as_float(pr[i + 3])));
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty_bar[buf]);  // single CTAs only: pairs never split
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
            const long long mrow = (long long)mt * (NH_BM * CTAS) + rank * NH_BM + quarter * 32;  // this warp's pixels
            const long long m = mrow + lane;  // this lane's pixel
            const bool valid = m < p.npix;
            const long long b = valid ? m / p.OHW : 0;
            const int q = valid ? (int)(m - b * p.OHW) : 0;
            float* yp = p.out_nchw ? p.y + b * p.y_bs + q : p.y + (valid ? m : 0) * p.y_ps;
            const float* rp = p.res ? p.res + (valid ? m : 0) * p.r_ps : nullptr;
            const uint32_t taddr = tmem0 + buf * BN + ((uint32_t)(quarter * 32) << 16);
            const long long c0l = clock64();
            // this warp's slabs are contiguous and taken two at a time through one 32-column TMEM
            // load: one load latency per pair of slabs instead of one per slab
            constexpr int PER = BN / 32;  // slabs per warp (the two warps of a lane window split the tile)
            const int s_begin = half * PER;
            // TF32 mode rounds every output to TF32; pair mode writes NHWC outputs as bf16 pairs and
            // the NCHW yolo outputs as plain fp32
            auto store_fmt = [&](float o) { return PAIR ? (p.out_nchw ? o : tb_pair_encode(o)) : tc::to_tf32_rna(o); };
            auto process = [&](int sl, const float* vin) {
                float v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = vin[i];
                const int fb = nt * BN + sl * 16;
                const bool full = fb + 16 <= p.F;
                float rv[16];
                if (rp && valid) {
                    if (p.vec && full) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4) {
                            const float4 r4 = __ldg(reinterpret_cast<const float4*>(rp + fb + i));
                            rv[i] = tb_fmt_load(r4.x, PAIR); rv[i + 1] = tb_fmt_load(r4.y, PAIR);
                            rv[i + 2] = tb_fmt_load(r4.z, PAIR); rv[i + 3] = tb_fmt_load(r4.w, PAIR);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) rv[i] = fb + i < p.F ? tb_fmt_load(__ldg(rp + fb + i), PAIR) : 0.f;
                    }
                }
                if (fast) {  // bias, leaky or linear, residual: flags held in registers
                    float bv[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) bv[i] = bias ? __ldg(bias + min(fb + i, Fm1)) : 0.f;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float o = v[i];
                        if (bias) o = __fadd_rn(o, bv[i]);
                        if (leaky && o < 0.f) o = __fmul_rn(o, 0.1f);  // rounded to TF32 below
                        if (rp) o = __fadd_rn(o, rv[i]);
                        v[i] = store_fmt(o);
                    }
                } else if (period) {  // fused yolo head: logistic on entries 0, 1, 4.. of each anchor
                    int e = fb % period;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float o = v[i];
                        if (bias) o = __fadd_rn(o, __ldg(bias + min(fb + i, Fm1)));
                        if (e != 2 && e != 3) o = __frcp_rn(__fadd_rn(1.0f, __expf(-o)));  // rounded to TF32 below
                        v[i] = store_fmt(o);
                        e = e + 1 == period ? 0 : e + 1;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int f = min(fb + i, Fm1);
                        float o = v[i];
                        if (bias) o = __fadd_rn(o, __ldg(bias + f));
                        o = nh_act(o, f, p);
                        if (rp) o = __fadd_rn(o, rv[i]);
                        v[i] = store_fmt(o);
                    }
                }
                if (p.tma_out) {
                    // stage the slab, then one lane stores it as a 16 x 32 box (the map clips
                    // filters >= F and pixels past the end)
                    const unsigned slab = stg0 + sbuf * 2048;
                    if (lane == 0) bulk_wait_read<1>();  // the store that last read this slab is done
                    __syncwarp();
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const unsigned a = slab + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4);
                        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"r"(a), "f"(v[4 * c]),
                                     "f"(v[4 * c + 1]), "f"(v[4 * c + 2]), "f"(v[4 * c + 3])
                                     : "memory");
                    }
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) tma_store_2d(&maps.y, slab, fb, (int)mrow);
                    sbuf ^= 1;
                } else if (valid) {
                    if (p.out_nchw) {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (fb + i < p.F) __stcs(yp + (long long)(fb + i) * p.OHW, v[i]);
                    } else if (p.vec && full) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4)
                            __stcs(reinterpret_cast<float4*>(yp + fb + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (fb + i < p.F) yp[fb + i] = v[i];
                    }
                }
            };
            // the tile's accumulator columns [c0, c0 + n): from TMEM, or the sum of the split-K
            // partials in split order
            auto fetch = [&](int c0, float* out, int n) {
                if (from_tmem) {
                    if (n == 32) tc::tmem_ld32(taddr + c0, out);
                    else tc::tmem_ld16(taddr + c0, out);
                    return;
                }
                for (int i = 0; i < n; ++i) out[i] = 0.f;
                const int slot0 = un.slot - un.slot % p.splits;  // the tile's first split
                const float4* pb = reinterpret_cast<const float4*>(p.part + (size_t)slot0 * NH_BM * BN) +
                                   (size_t)(c0 >> 2) * NH_BM + quarter * 32 + lane;
                for (int zz = 0; zz < p.splits; ++zz) {
                    float4 q4[8];  // every load of this split in flight before the adds
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < n / 4) q4[j] = __ldcg(pb + (size_t)zz * (NH_BM * BN / 4) + (size_t)j * NH_BM);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (j >= n / 4) break;
                        out[4 * j] = __fadd_rn(out[4 * j], q4[j].x);
                        out[4 * j + 1] = __fadd_rn(out[4 * j + 1], q4[j].y);
                        out[4 * j + 2] = __fadd_rn(out[4 * j + 2], q4[j].z);
                        out[4 * j + 3] = __fadd_rn(out[4 * j + 3], q4[j].w);
                    }
                }
            };
            if constexpr (PER >= 2) {
#pragma unroll 1
                for (int sl = s_begin; sl < s_begin + PER; sl += 2) {
                    float vv[32];
                    const long long q0 = clock64();
                    fetch(sl * 16, vv, 32);
                    c_ldw += clock64() - q0;
                    process(sl, vv);
                    process(sl + 1, vv + 16);
                }
            } else {
                float vv[16];
                const long long q0 = clock64();
                fetch(s_begin * 16, vv, 16);
                c_ldw += clock64() - q0;
                process(s_begin, vv);
            }
            c_st += clock64() - c0l;
            if (!from_tmem) continue;  // the accumulator was released after the partial was written
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) {  // this warp's TMEM reads are done
                if (CTAS == 1) tc::mbar_arrive(&tempty_bar[buf]);
                else tc::mbar_arrive_cluster(&tempty_bar[buf], 0);
            }
        }
        if (lane == 0) bulk_wait_read<0>();  // the shared-memory slabs are read before the CTA exits
        if (p.phases && warp == 2 && lane == 0) {
            p.phases[blockIdx.x * 12 + 5] = clock64() - c_start;
            p.phases[blockIdx.x * 12 + 6] = c_wt;
            p.phases[blockIdx.x * 12 + 7] = tl;
            p.phases[blockIdx.x * 12 + 9] = c_st;
            p.phases[blockIdx.x * 12 + 8] = c_ldw;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (CTAS == 2) tc::cluster_sync();  // the pair's MMAs and its tempty arrivals are over
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc_g<CTAS>(tmem0, 2 * BN);
    }
    if (p.phases && tid == 0) p.phases[blockIdx.x * 12 + 11] = tc::global_ns();  // CTA end
}

// packed weights for the NHWC kernel: wp[f][(r * KW + s) * Cp + c] = tf32(w[f][c][r][s]), zero for c >= C;
// pair mode: that array of (hi, hi) bf16 pairs, then one of (lo, lo)
__global__ void k_pack_nhwc(const float* __restrict__ w, float* __restrict__ wp, int F, int C, int KH, int KW,
                            int Cp, int pair) {
    const long long kp = (long long)KH * KW * Cp, total = (long long)F * kp;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int f = (int)(i / kp);
        const int k = (int)(i - (long long)f * kp);
        const int rs = k / Cp, c = k - rs * Cp;
        const int r = rs / KW, s = rs - r * KW;
        const float v = c < C ? w[(((long long)f * C + c) * KH + r) * KW + s] : 0.0f;
        if (!pair) {
            wp[i] = tc::to_tf32_rna(v);
        } else {
            const uint32_t e = __float_as_uint(tb_pair_encode(v)), hi = e & 0xffffu, lo = e >> 16;
            wp[i] = __uint_as_float(hi | (hi << 16));
            wp[total + i] = __uint_as_float(lo | (lo << 16));
        }
    }
}

PFN_cuTensorMapEncodeIm2col_v12000 im2col_encoder() {
    static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(f);
    });
    return fn;
}

template <int BN, int STAGES, bool PAIR, int CTAS>
constexpr int nh_smem() {
    return STAGES * (NH_A_BYTES + (PAIR ? 2 : 1) * (BN / CTAS) * NH_BK * 4) + NH_STG_BYTES + 1024;
}

template <int BN, int STAGES, bool PAIR, int CTAS>
int nh_launch(tb_ctx* ctx, const NhwcMaps& maps, const NhwcParams& p) {
    constexpr int smem = nh_smem<BN, STAGES, PAIR, CTAS>();
    static_assert(smem <= 232448, "shared memory per CTA");
    static std::mutex mu;
    static bool done[64] = {false};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device >= 64 || !done[ctx->device]) {  // the attribute is set per device
            cudaError_t e = cudaFuncSetAttribute(k_conv_nhwc<BN, STAGES, PAIR, CTAS>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(conv_nhwc)");
            if (ctx->device < 64) done[ctx->device] = true;
        }
    }
    const int slots = CTAS == 1 ? ctx->sm_count : (ctx->sm_count & ~1);
    const int grid = (int)std::min<int64_t>((int64_t)p.units * CTAS, slots);
    if constexpr (CTAS == 1) {
        return launch(ctx, "k_conv_nhwc", k_conv_nhwc<BN, STAGES, PAIR, 1>, dim3((unsigned)grid), dim3(NH_THREADS),
                      (size_t)smem, maps, p);
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(NH_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = ctx->stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = ctx->pdl ? 2 : 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, k_conv_nhwc<BN, STAGES, PAIR, CTAS>, maps, p);
        if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(conv_nhwc pair)");
    }
    return check_launch("k_conv_nhwc");
}

}  // namespace

int64_t conv_nhwc_packed_count(const ConvGeom& g, int pair) { return (pair ? 2 : 1) * g.F * g.KH * g.KW * round_up(g.C, 32); }

bool conv_nhwc_supported(const ConvGeom& g, int64_t x_ps) {
    // im2col corner and offset fields of a 4-D map: corners in [-128, 127], offsets < 256
    const int64_t upx = g.PX - (g.KW - 1) * g.DX, upy = g.PY - (g.KH - 1) * g.DY;
    if (g.PX > 128 || g.PY > 128 || upx < -128 || upx > 127 || upy < -128 || upy > 127) return false;
    if ((g.KW - 1) * g.DX > 255 || (g.KH - 1) * g.DY > 255 || g.SX > 8 || g.SY > 8) return false;
    if (x_ps < g.C || x_ps % 4 != 0) return false;  // TMA strides are multiples of 16 bytes
    // small tensors keep the NCHW path (the im2col map is only used on tensors of >= 128 KB)
    if (g.B * g.H * g.W * x_ps * 4 < (128 << 10)) return false;
    return g.B * g.OH * g.OW < ((int64_t)1 << 31) - NH_BM && g.F <= 65535 && g.OH * g.OW > 1;
}

int conv_nhwc_pack(tb_ctx* ctx, const ConvGeom& g, const float* w, float* wp, int pair) {
    const int64_t total = conv_nhwc_packed_count(g, 0);
    k_pack_nhwc<<<grid_for(total, 256, ctx->sm_count), 256, 0, ctx->stream>>>(w, wp, (int)g.F, (int)g.C, (int)g.KH,
                                                                              (int)g.KW, (int)round_up(g.C, 32), pair);
    return check_launch("k_pack_nhwc");
}

// Tile shape of one NHWC conv launch: filters per tile, K splits, CTAs per tile (2: a cta_group::2
// pair on 256 pixels, never split).
struct NhShape {
    int bn, splits, ctas;
};

std::mutex g_nh_mu;
std::map<std::vector<int64_t>, NhShape> g_nh_tuned;  // measured at network set-up
thread_local const NhShape* t_nh_pin = nullptr;    // the autotuner's candidate under test

std::vector<int64_t> nh_key(int device, const ConvGeom& g, int64_t x_ps, int pair) {
    return {device, g.B, g.C, g.H, g.W, g.F, g.KH, g.KW, g.SY, g.SX, g.PY, g.PX, g.DY, g.DX, x_ps, pair};
}

int64_t nh_ktiles(const ConvGeom& g) { return g.KH * g.KW * (round_up(g.C, 32) / NH_BK); }

// split-K partial tiles of a shape (floats)
// tiles stored whole: every full wave over the SMs (the rest are split), all when not split
int64_t nh_dp_tiles(int64_t tiles, const NhShape& sh, int sms) {
    return sh.splits <= 1 ? tiles : (tiles / sms) * sms;
}

int64_t nh_part_floats(const ConvGeom& g, const NhShape& sh, int sms) {
    if (sh.splits <= 1) return 0;
    const int64_t tiles = ceil_div(g.B * g.OH * g.OW, NH_BM) * ceil_div(g.F, sh.bn);
    return (tiles - nh_dp_tiles(tiles, sh, sms)) * sh.splits * NH_BM * sh.bn;
}

constexpr int64_t NH_PART_CAP = (int64_t)1 << 26;  // 256 MiB of partial tiles at most

// default shape: the widest tile that does not leave most of it empty, no split
NhShape nh_default(const ConvGeom& g) { return NhShape{g.F > 128 ? 256 : g.F > 64 ? 128 : g.F > 32 ? 64 : 32, 1, 1}; }

NhShape nh_choose(tb_ctx* ctx, const ConvGeom& g, int64_t x_ps, int pair) {
    if (t_nh_pin) return *t_nh_pin;
    if (const char* f = getenv("TB_NHWC_FORCE")) {  // test hook: "BN,SPLITS[,CTAS]"
        NhShape sh{256, 1, 1};
        if (sscanf(f, "%d,%d,%d", &sh.bn, &sh.splits, &sh.ctas) >= 1 &&
            (sh.bn == 32 || sh.bn == 64 || sh.bn == 128 || sh.bn == 256)) {
            if (sh.splits < 1) sh.splits = 1;
            if (sh.ctas != 2 || sh.bn < 128) sh.ctas = 1;
            if (sh.ctas == 2) sh.splits = 1;
            return sh;
        }
    }
    std::lock_guard<std::mutex> lk(g_nh_mu);
    auto it = g_nh_tuned.find(nh_key(ctx->device, g, x_ps, pair));
    return it != g_nh_tuned.end() ? it->second : nh_default(g);
}

// x: NHWC with pixel stride x_ps (floats; x points at channel 0 of the conv's input);
// y: NHWC with pixel stride y_ps when y_ps > 0 (y at the output's channel offset), else NCHW
// with batch stride g.y_bs; res: NHWC with pixel stride r_ps (or null).
int conv_nhwc_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, int64_t x_ps, const float* wp,
                     const float* bias, const float* res, int64_t r_ps, float* y, int64_t y_ps, int act,
                     int yolo_classes, unsigned long long* phases, int pair) {
    if (!conv_nhwc_supported(g, x_ps)) return fail(TB_ERR_UNSUPPORTED, "NHWC tensor-core conv: unsupported geometry");
    if (g.B == 0) return TB_OK;
    if (!aligned16(x) || !aligned16(wp)) return fail(TB_ERR_INVALID, "NHWC conv: x and weights must be 16-byte aligned");
    if (y_ps > 0 && y_ps < g.F) return fail(TB_ERR_INVALID, "NHWC conv: output pixel stride below the filter count");
    auto enc = im2col_encoder();
    if (!enc) return fail(TB_ERR_CUDA, "NHWC conv: cuTensorMapEncodeIm2col is not available");
    const int64_t Cp = round_up(g.C, 32);
    NhwcMaps maps;
    memset(&maps, 0, sizeof(maps));
    {
        cuuint64_t dims[4] = {(cuuint64_t)g.C, (cuuint64_t)g.W, (cuuint64_t)g.H, (cuuint64_t)g.B};
        cuuint64_t strides[3] = {(cuuint64_t)(x_ps * 4), (cuuint64_t)(g.W * x_ps * 4), (cuuint64_t)(g.H * g.W * x_ps * 4)};
        int lower[2] = {(int)-g.PX, (int)-g.PY};
        int upper[2] = {(int)(g.PX - (g.KW - 1) * g.DX), (int)(g.PY - (g.KH - 1) * g.DY)};
        cuuint32_t es[4] = {1, (cuuint32_t)g.SX, (cuuint32_t)g.SY, 1};
        CUresult r = enc(&maps.a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(x), dims, strides, lower,
                         upper, NH_BK, NH_BM, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(TB_ERR_CUDA, "NHWC conv: cuTensorMapEncodeIm2col failed (%d)", (int)r);
    }
    NhShape sh = nh_choose(ctx, g, x_ps, pair);
    const int bn = sh.bn, ctas = sh.ctas == 2 ? 2 : 1;
    if (ctas == 2) sh.splits = 1;
    const int64_t ktiles = nh_ktiles(g);
    const int64_t tiles = ceil_div(g.B * g.OH * g.OW, NH_BM) * ceil_div(g.F, bn);
    if (sh.splits > ktiles) sh.splits = (int)ktiles;
    const int kps = (int)ceil_div(ktiles, sh.splits);
    sh.splits = (int)ceil_div(ktiles, kps);  // no empty split
    if (sh.splits > 1 && (tiles > ctx->tile_cnt_len || nh_part_floats(g, sh, ctx->sm_count) > NH_PART_CAP ||
                          (size_t)nh_part_floats(g, sh, ctx->sm_count) * sizeof(float) > ctx->ws_bytes))
        sh.splits = 1;  // no room for the partial tiles or counters: one unit per tile
    if (sh.splits > 1 && nh_dp_tiles(tiles, sh, ctx->sm_count) == tiles) sh.splits = 1;  // whole waves only
    {
        const uint64_t dims[2] = {(uint64_t)(g.KH * g.KW * Cp), (uint64_t)g.F};
        const uint64_t strides[1] = {(uint64_t)(g.KH * g.KW * Cp * 4)};
        const uint32_t box[2] = {(uint32_t)NH_BK, (uint32_t)(bn / ctas)};  // a pair's CTA holds half the filters
        int r = encode_map(&maps.b, wp, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (r != TB_OK) return r;
        if (pair) {  // the (lo, lo) operand follows the (hi, hi) one
            r = encode_map(&maps.b2, wp + conv_nhwc_packed_count(g, 0), 2, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
            if (r != TB_OK) return r;
        }
    }
    NhwcParams p{};
    static const bool no_tma_store = getenv("TB_NHWC_NO_TMA_STORE") != nullptr;  // experiment hook
    if (y_ps > 0 && y_ps % 4 == 0 && aligned16(y) && !no_tma_store) {
        const uint64_t dims[2] = {(uint64_t)g.F, (uint64_t)(g.B * g.OH * g.OW)};
        const uint64_t strides[1] = {(uint64_t)(y_ps * 4)};
        const uint32_t box[2] = {16, 32};
        int r = encode_map(&maps.y, y, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
        if (r != TB_OK) return r;
        p.tma_out = 1;
    }
    p.bias = bias; p.res = res; p.y = y; p.status = ctx->d_status; p.phases = phases;
    p.npix = g.B * g.OH * g.OW;
    p.y_bs = g.y_bs;
    p.OW = (int)g.OW; p.OHW = (int)(g.OH * g.OW);
    p.SX = (int)g.SX; p.SY = (int)g.SY; p.PX = (int)g.PX; p.PY = (int)g.PY;
    p.KW = (int)g.KW; p.DX = (int)g.DX; p.DY = (int)g.DY;
    p.F = (int)g.F;
    p.csteps = (int)(Cp / NH_BK);
    p.ktiles = (int)(g.KH * g.KW * p.csteps);
    p.tiles_n = (int)ceil_div(g.F, bn);
    p.tiles_total = (int)(ceil_div(p.npix, (int64_t)NH_BM * ctas) * p.tiles_n);
    p.splits = sh.splits;
    p.kt_per_split = sh.splits > 1 ? (int)ceil_div(ktiles, sh.splits) : (int)ktiles;
    p.dp_tiles = (int)nh_dp_tiles(p.tiles_total, sh, ctx->sm_count);
    p.units = p.dp_tiles + (p.tiles_total - p.dp_tiles) * p.splits;
    p.part = sh.splits > 1 ? reinterpret_cast<float*>(ctx->ws) : nullptr;
    p.tile_cnt = ctx->tile_cnt;
    p.out_nchw = y_ps > 0 ? 0 : 1;
    p.y_ps = (int)y_ps;
    p.r_ps = (int)r_ps;
    p.vec = y_ps % 4 == 0 && aligned16(y) && (!res || (r_ps % 4 == 0 && aligned16(res))) ? 1 : 0;
    p.act = act;
    p.yolo_classes = yolo_classes;
    if (ctas == 2) {
        if (pair) return bn == 256 ? nh_launch<256, 4, true, 2>(ctx, maps, p) : nh_launch<128, 6, true, 2>(ctx, maps, p);
        return bn == 256 ? nh_launch<256, 6, false, 2>(ctx, maps, p) : nh_launch<128, 8, false, 2>(ctx, maps, p);
    }
    if (pair) {
        if (bn == 256) return nh_launch<256, 2, true, 1>(ctx, maps, p);
        if (bn == 128) return nh_launch<128, 4, true, 1>(ctx, maps, p);
        if (bn == 32) return nh_launch<32, 8, true, 1>(ctx, maps, p);
        return nh_launch<64, 6, true, 1>(ctx, maps, p);
    }
    if (bn == 256) return nh_launch<256, 4, false, 1>(ctx, maps, p);
    if (bn == 128) return nh_launch<128, 6, false, 1>(ctx, maps, p);
    if (bn == 32) return nh_launch<32, 8, false, 1>(ctx, maps, p);
    return nh_launch<64, 8, false, 1>(ctx, maps, p);
}

// Workspace the NHWC conv of this geometry needs (split-K partials of its tuned shape).
int64_t conv_nhwc_ws_floats(tb_ctx* ctx, const ConvGeom& g, int64_t x_ps, int pair) {
    return nh_part_floats(g, nh_choose(ctx, g, x_ps, pair), ctx->sm_count);
}

// Time the tile shapes (filters per tile x K splits) of this geometry on the given buffers
// (bias and residual off) and keep the fastest for later launches. Blocks; grows the workspace.
int conv_nhwc_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, int64_t x_ps, const float* wp, float* y,
                       int64_t y_ps, int pair) {
    if (g.B == 0 || !conv_nhwc_supported(g, x_ps)) return TB_OK;
    const int64_t ktiles = nh_ktiles(g);
    std::vector<NhShape> cands;
    for (int bn : {32, 64, 128, 256}) {
        if (bn > 32 && bn / 2 >= g.F) continue;  // a tile at least half full
        const int64_t tiles = ceil_div(g.B * g.OH * g.OW, NH_BM) * ceil_div(g.F, bn);
        // splits cut only the tiles of the last partial wave: worth it while they fit one wave or two
        const int64_t rem = tiles - nh_dp_tiles(tiles, NhShape{bn, 2, 1}, ctx->sm_count);
        for (int sp : {1, 2, 3, 4, 6, 8}) {
            if (sp > 1 && (rem == 0 || ktiles < 2 * sp || tiles > ctx->tile_cnt_len || rem * sp > 2 * (int64_t)ctx->sm_count))
                continue;
            NhShape sh{bn, sp, 1};
            if (nh_part_floats(g, sh, ctx->sm_count) > NH_PART_CAP) continue;
            cands.push_back(sh);
        }
        if (bn >= 128) cands.push_back(NhShape{bn, 1, 2});  // a cta_group::2 pair on 256 pixels
    }
    if (cands.empty()) return TB_OK;
    int64_t ws = 0;
    for (const NhShape& c : cands) ws = std::max(ws, nh_part_floats(g, c, ctx->sm_count));
    int r = ensure_workspace(ctx, (size_t)std::max<int64_t>(ws, 1) * sizeof(float));
    if (r != TB_OK) return r;
    cudaEvent_t e0, e1;
    TB_CHECK_CUDA(cudaEventCreate(&e0));
    TB_CHECK_CUDA(cudaEventCreate(&e1));
    float best_ms = 1e30f;
    NhShape best = cands[0];
    for (const NhShape& c : cands) {
        t_nh_pin = &c;
        r = conv_nhwc_launch(ctx, g, x, x_ps, wp, nullptr, nullptr, 0, y, y_ps, TB_ACT_LINEAR, 0, nullptr, pair);
        stream_delay_us(ctx, 200);  // the timed launches queue behind it: device time only
        cudaEventRecord(e0, ctx->stream);
        for (int rep = 0; rep < 3 && r == TB_OK; ++rep)
            r = conv_nhwc_launch(ctx, g, x, x_ps, wp, nullptr, nullptr, 0, y, y_ps, TB_ACT_LINEAR, 0, nullptr, pair);
        cudaEventRecord(e1, ctx->stream);
        t_nh_pin = nullptr;
        cudaError_t e = cudaEventSynchronize(e1);
        if (r != TB_OK) break;
        if (e != cudaSuccess) { r = cuda_fail(e, "NHWC conv autotune"); break; }
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (getenv("TB_AUTOTUNE_VERBOSE"))
            fprintf(stderr, "nhwc autotune C%lld H%lld F%lld k%lld s%lld B%lld: bn %d splits %d ctas %d: %.4f ms\n",
                    (long long)g.C, (long long)g.H, (long long)g.F, (long long)g.KH, (long long)g.SY,
                    (long long)g.B, c.bn, c.splits, c.ctas, ms / 3);
        if (ms < best_ms) best_ms = ms, best = c;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (r != TB_OK) return r;
    std::lock_guard<std::mutex> lk(g_nh_mu);
    g_nh_tuned[nh_key(ctx->device, g, x_ps, pair)] = best;
    return TB_OK;
}

}  // namespace tbi

using namespace tbi;

extern "C" {

int tb_conv_nhwc_packed_count(const tb_conv_desc* d, int64_t* count) {
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!count) return fail(TB_ERR_INVALID, "null count");
    *count = conv_nhwc_packed_count(g);
    return TB_OK;
}

int tb_conv_pack_weights_nhwc(tb_ctx* ctx, const tb_conv_desc* d, const float* weights, float* packed) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!weights || !packed) return fail(TB_ERR_INVALID, "NHWC pack: null pointer");
    if (!aligned16(packed)) return fail(TB_ERR_INVALID, "NHWC pack: packed buffer must be 16-byte aligned");
    return conv_nhwc_pack(ctx, g, weights, packed);
}

int tb_conv2d_fwd_nhwc(tb_ctx* ctx, const tb_conv_desc* d, const float* x, int64_t x_pixel_stride,
                       const float* packed_w, const float* bias, const float* residual, int64_t res_pixel_stride,
                       float* y, int64_t y_pixel_stride) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!x || !packed_w || !y) return fail(TB_ERR_INVALID, "NHWC conv: null x, weights or y");
    if (residual && y_pixel_stride <= 0) return fail(TB_ERR_INVALID, "NHWC conv: a residual needs an NHWC output");
    if (!act_supported(d->activation)) return fail(TB_ERR_UNSUPPORTED, "NHWC conv: activation not supported");
    return conv_nhwc_launch(ctx, g, x, x_pixel_stride, packed_w, bias, residual, res_pixel_stride, y,
                            y_pixel_stride, (int)d->activation, 0, nullptr);
}

int tb_diag_conv_nhwc_phases(tb_ctx* ctx, const tb_conv_desc* d, const float* x, int64_t x_pixel_stride,
                             const float* packed_w, float* y, int64_t y_pixel_stride, double* out12) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!x || !packed_w || !y || !out12) return fail(TB_ERR_INVALID, "NHWC conv phases: null pointer");
    const int n = ctx->sm_count * 12;
    unsigned long long* dph = nullptr;
    TB_CHECK_CUDA(cudaMalloc(&dph, n * sizeof(unsigned long long)));
    cudaMemsetAsync(dph, 0, n * sizeof(unsigned long long), ctx->stream);
    r = conv_nhwc_launch(ctx, g, x, x_pixel_stride, packed_w, nullptr, nullptr, 0, y, y_pixel_stride,
                         (int)d->activation, 0, dph);
    std::vector<unsigned long long> h(n);
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), dph, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(dph);
    if (r != TB_OK) return r;
    if (e != cudaSuccess) return cuda_fail(e, "NHWC conv phases");
    int ctas = 0;
    for (int i = 0; i < 12; ++i) out12[i] = 0;
    for (int c = 0; c < ctx->sm_count; ++c) {
        if (h[c * 12 + 0] == 0) continue;
        ++ctas;
        for (int i = 0; i < 10; ++i) out12[i] += (double)h[c * 12 + i];
    }
    for (int i = 0; i < 10 && ctas; ++i) out12[i] /= ctas;
    // 10: the launch's span (first CTA start to last CTA end), 11: the longest CTA, both in ns
    unsigned long long t0 = ~0ull, t1 = 0, tmax = 0;
    for (int c = 0; c < ctx->sm_count; ++c) {
        if (h[c * 12 + 0] == 0) continue;
        t0 = std::min(t0, h[c * 12 + 10]);
        t1 = std::max(t1, h[c * 12 + 11]);
        tmax = std::max(tmax, h[c * 12 + 11] - h[c * 12 + 10]);
    }
    out12[10] = ctas ? (double)(t1 - t0) : 0.0;
    out12[11] = (double)tmax;
    return TB_OK;
}

}  // extern "C"
