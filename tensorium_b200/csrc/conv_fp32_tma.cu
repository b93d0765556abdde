// conv_fp32_tma.cu -- FP32 CUDA-core implicit-GEMM convolution fed by TMA (RSC layers).
//
// The same arithmetic as conv_fp32_kernel (M = filters, N = pixels, K = (r, s, c) in the packed
// weight order, one fmaf per k in ascending order per output, the reference-faithful epilogue),
// with the operand gather moved off the SMs: the A operand (weights [k][Mpad]) and the B operand
// (input pixels x channels) are copied by TMA from the packed weights and from x in place or its
// tap replicas (conv_tc.cu's tc_prepare_a, values not rounded), so the mainloop is shared-memory
// loads and FFMAs only.  Pixels live on the replica's padded grid n = b*Lp + oy*Wp + ox; padding
// pixels are computed and dropped.
//   * CTA tile 128 filters x 128 pixels, 256 threads, 8 x 8 outputs per thread (two 4-row and
//     two 4-column quads half a tile apart), 16-deep k tiles, STAGES-deep mbarrier ring;
//   * B stage layout [4 groups][16 k][32 pixels] (what a (32 pixels, channel, group, plane) box
//     writes); A stage layout [16 k][128 filters];
//   * split-K over blockIdx.z with the last-arriver fix-up of the gather kernel (partials summed
//     in split order 0..S-1).
// Every mbarrier wait is bounded; on timeout the CTA sets the context status word and stops.
#include "conv_tc.cuh"

#include <cstring>
#include <mutex>

namespace tbi {

namespace {

constexpr int FT_BM = 128, FT_BN = 128, FT_BK = 16, FT_THREADS = 256, FT_STAGES = 6;
constexpr int FT_A_BYTES = FT_BK * FT_BM * 4, FT_B_BYTES = FT_BK * FT_BN * 4;
constexpr int FT_STAGE_BYTES = FT_A_BYTES + FT_B_BYTES;

struct FtMaps {
    CUtensorMap a4[TC_MAX_KH];
    CUtensorMap a1[TC_MAX_KH];
    CUtensorMap tail;
    CUtensorMap w;  // packed weights (Mpad, Kpad), box 128 x 16
};

struct FtParams {
    ConvParams cp;  // epilogue fields, F, OHW, y_bs, r_bs, ws, tile_cnt, splits, kt_per_split, ktiles
    int* status;  // context status word (bounded waits that time out report here)
    int B, Lp, Wp, OW, OHWp, NPH, KW, csteps, g_full;
    long long Npad;
    int phase[TC_MAX_KH];
};

}  // namespace

__global__ void __launch_bounds__(FT_THREADS, 2)
    k_conv_fp32_tma(const __grid_constant__ FtMaps maps, const FtParams q) {
    const ConvParams& p = q.cp;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - ((unsigned)__cvta_generic_to_shared(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full_bar[FT_STAGES];
    __shared__ volatile int abort_flag;
    __shared__ int s_last;

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * FT_BM;
    const long long n0 = (long long)blockIdx.x * FT_BN;
    const int kb = blockIdx.z * p.kt_per_split, ke = min(p.ktiles, kb + p.kt_per_split);
    const int nkt = ke - kb;
    const unsigned sbase = (unsigned)__cvta_generic_to_shared(smem);

    // producer state, used by thread 0 only and kept in shared memory (not in every thread's
    // registers across the mainloop): this tile's 32-pixel groups, the tap (pr, ps) and channel
    // pc0 of the next k tile, copies issued
    __shared__ int bq[4], gq[4], split, pr, ps, pc0, issued;
    if (tid == 0) {
        issued = 0;
        for (int s = 0; s < FT_STAGES; ++s) tc::mbar_init(&full_bar[s], 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const long long n = n0 + 32 * j;
            bq[j] = (int)(n / q.Lp);
            gq[j] = (int)((n - (long long)bq[j] * q.Lp) >> 5);
        }
        split = bq[0] != bq[3] || gq[3] >= q.g_full;
        const int rs0 = kb / q.csteps;
        pr = rs0 / q.KW;
        ps = rs0 - pr * q.KW;
        pc0 = (kb - rs0 * q.csteps) * FT_BK;
    }
    auto issue = [&](int kt, int st) {  // thread 0: copies of k tile kt into stage st
        tc::mbar_arrive_expect_tx(&full_bar[st], FT_STAGE_BYTES);
        const unsigned sa = sbase + st * FT_STAGE_BYTES, sb = sa + FT_A_BYTES;
        tc::tma_load_2d(sa, &maps.w, &full_bar[st], m0, kt * FT_BK);
        const int z0 = (ps * q.NPH + q.phase[pr]) * q.B;
        if (!split) {
            tc::tma_load_4d(sb, &maps.a4[pr], &full_bar[st], 0, pc0, gq[0], z0 + bq[0]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (gq[j] < q.g_full)
                    tc::tma_load_4d(sb + j * (FT_B_BYTES / 4), &maps.a1[pr], &full_bar[st], 0, pc0, gq[j], z0 + bq[j]);
                else
                    tc::tma_load_3d(sb + j * (FT_B_BYTES / 4), &maps.tail, &full_bar[st], gq[j] * 32, pc0, z0 + bq[j]);
            }
        }
        ++issued;
        pc0 += FT_BK;
        if (pc0 >= q.csteps * FT_BK) {
            pc0 = 0;
            if (++ps == q.KW) ps = 0, ++pr;
        }
    };
    __syncthreads();
    if (tid == 0)
        for (int i = 0; i < FT_STAGES && i < nkt; ++i) issue(kb + i, i);

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    // B quads of this thread: pixel columns tx*4 and 64 + tx*4 -> group (tx>>3) and 2 + (tx>>3)
    const int boff0 = (tx >> 3) * (FT_BK * 32) + (tx & 7) * 4, boff1 = boff0 + 2 * (FT_BK * 32);
    bool ok = true;
    for (int t = 0; t < nkt; ++t) {
        const int st = t % FT_STAGES;
        ok = !abort_flag && tc::mbar_wait_bounded(&full_bar[st], (t / FT_STAGES) & 1, &abort_flag, q.status, 921);
        if (!ok) break;
        const float* as = reinterpret_cast<const float*>(smem + st * FT_STAGE_BYTES);
        const float* bs = reinterpret_cast<const float*>(smem + st * FT_STAGE_BYTES + FT_A_BYTES);
#pragma unroll
        for (int kk = 0; kk < FT_BK; ++kk) {
            float a[8], b[8];
            *reinterpret_cast<float4*>(&a[0]) = *reinterpret_cast<const float4*>(as + kk * FT_BM + ty * 4);
            *reinterpret_cast<float4*>(&a[4]) = *reinterpret_cast<const float4*>(as + kk * FT_BM + 64 + ty * 4);
            *reinterpret_cast<float4*>(&b[0]) = *reinterpret_cast<const float4*>(bs + boff0 + kk * 32);
            *reinterpret_cast<float4*>(&b[4]) = *reinterpret_cast<const float4*>(bs + boff1 + kk * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();  // every thread is done with stage st
        if (tid == 0 && t + FT_STAGES < nkt) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic reads before the refill
            issue(kb + t + FT_STAGES, st);
        }
    }
    ok = __syncthreads_and(ok);
    if (!ok) {  // a wait timed out: let the copies already issued land, then stop
        if (tid == 0)
            for (int j = issued > FT_STAGES ? issued - FT_STAGES : 0; j < issued; ++j)
                tc::mbar_wait_limit(&full_bar[j % FT_STAGES], (j / FT_STAGES) & 1);
        return;
    }

    // ---- epilogue: quads of 4 pixels of the padded grid (one row, one image) ----
    struct Quad { int b, oy, ox, nvalid; };
    Quad cq[2];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        const long long nb = n0 + g * 64 + tx * 4;
        const int b = (int)(nb / q.Lp), qq = (int)(nb - (long long)b * q.Lp);
        const int oy = qq / q.Wp, ox = qq - oy * q.Wp;
        cq[g].b = b;
        cq[g].oy = oy;
        cq[g].ox = ox;
        cq[g].nvalid = (ok && b < q.B && qq < q.OHWp) ? max(0, min(4, q.OW - ox)) : 0;
    }
    const bool simple = !p.bn_mean && p.yolo_classes == 0 && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
    const bool has_bias = p.bias != nullptr, leaky = p.act == TB_ACT_LEAKY;
    auto store4 = [&](int m, int g, const float* v) {
        const Quad& c = cq[g];
        if (c.nvalid == 0) return;
        const float bm = has_bias ? __ldg(p.bias + m) : 0.f;
        const long long off = (long long)m * p.OHW + (long long)c.oy * q.OW + c.ox;
        float* yb = p.y + c.b * p.y_bs;
        const float* rb = p.res ? p.res + c.b * p.r_bs : nullptr;
        if (p.vec_out && c.nvalid == 4) {
            float4 o;
            o.x = conv_epi_value(v[0], m, p, simple, has_bias, leaky, bm);
            o.y = conv_epi_value(v[1], m, p, simple, has_bias, leaky, bm);
            o.z = conv_epi_value(v[2], m, p, simple, has_bias, leaky, bm);
            o.w = conv_epi_value(v[3], m, p, simple, has_bias, leaky, bm);
            if (rb) {
                const float4 r = *reinterpret_cast<const float4*>(rb + off);
                o.x = __fadd_rn(o.x, r.x);
                o.y = __fadd_rn(o.y, r.y);
                o.z = __fadd_rn(o.z, r.z);
                o.w = __fadd_rn(o.w, r.w);
            }
            *reinterpret_cast<float4*>(yb + off) = o;
            return;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (e < c.nvalid) {
                float o = conv_epi_value(v[e], m, p, simple, has_bias, leaky, bm);
                if (rb) o = __fadd_rn(o, rb[off + e]);
                yb[off + e] = o;
            }
        }
    };
    if (p.splits > 1) {
        // split-K: publish this split's partial tile; the last CTA to arrive on the tile sums the
        // partials in split order 0..S-1 and runs the epilogue.  No CTA waits for another.
        const long long plane = (long long)p.F * q.Npad;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
            if (m >= p.F) continue;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                const long long nb = n0 + g * 64 + tx * 4;
                if (nb >= q.Npad) continue;
                __stcg(reinterpret_cast<float4*>(p.ws + blockIdx.z * plane + (long long)m * q.Npad + nb),
                       make_float4(acc[i][g * 4], acc[i][g * 4 + 1], acc[i][g * 4 + 2], acc[i][g * 4 + 3]));
            }
        }
        __threadfence();
        __syncthreads();
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        if (tid == 0) {
            const int prev = atomicAdd(&p.tile_cnt[tile], 1);
            s_last = prev == p.splits - 1;
            if (s_last) p.tile_cnt[tile] = 0;  // ready for the next launch
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
            if (m >= p.F) continue;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                const long long nb = n0 + g * 64 + tx * 4;
                if (nb >= q.Npad) continue;
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                const float* src = p.ws + (long long)m * q.Npad + nb;
                for (int z = 0; z < p.splits; ++z) {
                    const float4 t4 = __ldcg(reinterpret_cast<const float4*>(src + z * plane));
                    v[0] = __fadd_rn(v[0], t4.x);
                    v[1] = __fadd_rn(v[1], t4.y);
                    v[2] = __fadd_rn(v[2], t4.z);
                    v[3] = __fadd_rn(v[3], t4.w);
                }
                store4(m, g, v);
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= p.F) continue;
#pragma unroll
        for (int g = 0; g < 2; ++g) store4(m, g, &acc[i][g * 4]);
    }
}

}  // namespace tbi

namespace tbi {

bool conv_fp32_tma_supported(const ConvGeom& g) {
    if (!g.rsc || g.KH > TC_MAX_KH || g.SY > 4 || g.OH * g.OW == 1) return false;
    TcPlan pl;
    tc_plan(g, &pl, 1);
    if (pl.mode == TC_TAPS && (g.KW > 8 || g.SX * 3 + (g.KW - 1) * g.DX + 1 > 32 || pl.NPH * g.B * g.C > 65535))
        return false;
    return pl.mode != TC_IM2COL && g.B * pl.Lp < ((int64_t)1 << 31) - FT_BN && g.KW * pl.NPH * g.B <= 65535;
}

// workspace floats: the A-operand replica, then `splits` partial planes of F x (B*Lp)
int64_t conv_fp32_tma_ws_floats(const ConvGeom& g, int splits) {
    TcPlan pl;
    tc_plan(g, &pl, 1);
    const int64_t part = splits > 1 ? (int64_t)splits * g.F * round_up(g.B * pl.Lp, FT_BN) : 0;
    return replica_floats(g, pl) + part;
}

// p: the ConvParams of the gather kernel (x, w, epilogue, y, batch strides, splits,
// kt_per_split, tile_cnt, vec_out); ktiles is set here.  ws: workspace of
// conv_fp32_tma_ws_floats(g, p.splits) floats.
int conv_fp32_tma_run(tb_ctx* ctx, const ConvGeom& g, ConvParams p, float* ws, int64_t ws_floats,
                      int64_t tile_cnt_len, int64_t* launches) {
    if (!conv_fp32_tma_supported(g)) return fail(TB_ERR_UNSUPPORTED, "conv (TMA): unsupported geometry");
    if (!ws || !aligned16(ws)) return fail(TB_ERR_INVALID, "conv (TMA): needs a 16-byte-aligned workspace");
    if (ws_floats < conv_fp32_tma_ws_floats(g, p.splits))
        return fail(TB_ERR_INVALID, "conv (TMA): workspace too small");
    FtMaps maps;
    memset(&maps, 0, sizeof(maps));
    TcPlan pl;
    int kmaps = 1, g_full = 1 << 30;
    int r = tc_prepare_a(ctx, g, p.x, ws, false, FT_BK, 1, CU_TENSOR_MAP_SWIZZLE_NONE, maps.a4, maps.a1, &maps.tail,
                         &pl, &kmaps, &g_full, launches);
    if (r != TB_OK) return r;
    {
        const uint64_t dims[2] = {(uint64_t)g.Mpad, (uint64_t)g.Kpad};
        const uint64_t st[1] = {(uint64_t)g.Mpad * 4};
        const uint32_t box[2] = {FT_BM, FT_BK};
        r = encode_map(&maps.w, p.w, 2, dims, st, box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (r != TB_OK) return r;
    }
    FtParams q{};
    q.cp = p;
    q.cp.ktiles = (int)(g.Kpad / FT_BK);
    if (q.cp.kt_per_split <= 0) q.cp.kt_per_split = q.cp.ktiles;
    q.status = ctx->d_status;
    q.B = (int)g.B;
    q.Lp = (int)pl.Lp;
    q.Wp = (int)pl.Wp;
    q.OW = (int)(pl.mode == TC_INPLACE ? pl.Wp : g.OW);
    q.OHWp = (int)(pl.mode == TC_INPLACE ? pl.Wp : g.OH * pl.Wp);
    q.NPH = (int)pl.NPH;
    q.KW = pl.mode == TC_TAPS ? (int)g.KW : 1;
    q.csteps = (int)(g.Cpad / FT_BK);
    q.g_full = g_full;
    q.Npad = round_up(g.B * pl.Lp, FT_BN);
    for (int i = 0; i < TC_MAX_KH; ++i) q.phase[i] = pl.phase[i];
    q.cp.ws = p.splits > 1 ? ws + replica_floats(g, pl) : nullptr;
    {
        const bool ow4 = pl.mode == TC_INPLACE || g.OW % 4 == 0;
        q.cp.vec_out = ow4 && (g.OH * g.OW) % 4 == 0 && g.y_bs % 4 == 0 && aligned16(p.y) &&
                       (!p.res || (g.r_bs % 4 == 0 && aligned16(p.res)));
    }
    dim3 grid((unsigned)(q.Npad / FT_BN), (unsigned)ceil_div(g.F, FT_BM), (unsigned)p.splits);
    if (grid.y > 65535 || grid.z > 65535) return fail(TB_ERR_INVALID, "conv (TMA): grid too large");
    if (p.splits > 1 && (int64_t)grid.x * grid.y > tile_cnt_len)
        return fail(TB_ERR_INVALID, "conv (TMA): too many split-K tiles for the counters");
    constexpr int smem = FT_STAGES * FT_STAGE_BYTES + 1024;
    static std::mutex mu;
    static bool done[64] = {false};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !done[ctx->device]) {
            cudaError_t e = cudaFuncSetAttribute(k_conv_fp32_tma, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(conv TMA)");
            done[ctx->device] = true;
        }
    }
    k_conv_fp32_tma<<<grid, FT_THREADS, smem, ctx->stream>>>(maps, q);
    r = check_launch("k_conv_fp32_tma");
    if (r != TB_OK) return r;
    if (launches) ++*launches;
    return TB_OK;
}

}  // namespace tbi
