// conv_tc.cu -- TF32 tensor-core (tcgen05 / TMEM) implicit-GEMM convolution, NCHW.
//
// Same GEMM view as the FP32 path: D[m = filter][n = pixel over the batch], K = (r, s, c) with the
// channel fastest.  Operands reach shared memory by cp.async (16-byte copies only):
//   A (weights): the packed K-major weight rows Wp[k][Mpad], M contiguous -> MN-major tile;
//   B (activations): from the "tap replicas" P[s][b][c][H + 2p][Wp] made by k_tc_repack, where
//     P[s][.][y + p][x] = X[y][x + s - p] (0 outside) and Wp = round_up(W, 4): for a fixed (r, s, c)
//     the B row over the padded output grid n = (b, oy, ox < Wp) is one contiguous run, so every
//     16-byte chunk is aligned.  Columns ox >= OW of the padded grid are computed and discarded.
// Warp roles (160 threads): warps 0-3 produce the A/B ring (STAGES x BK=32) and later run the
// epilogue (tcgen05.ld from TMEM, bias / batchnorm / activation / residual / yolo, NCHW stores);
// warp 4 allocates TMEM and one of its threads issues tcgen05.mma (M = 128, N = BN, K = 8) and
// commits each stage back to the producers.  Every wait is bounded: on timeout the kernel sets
// the context status word, stops, frees its TMEM and returns.
// Stride-1 convolutions with channels % 32 == 0 take this path; the rest use the FP32 kernel.
#include "conv_tc.cuh"

#include <mutex>

namespace tbi {

struct TcParams {
    const float* __restrict__ w;   // packed weights [Kpad][Mpad]
    const float* __restrict__ p;   // tap replicas
    const float* __restrict__ bias;
    const float* __restrict__ bn_scale;
    const float* __restrict__ bn_mean;
    const float* __restrict__ bn_var;
    const float* __restrict__ res;
    float* __restrict__ y;
    int* status;
    int C, F, KH, KW, OH, OW, Wp, Hp, Mpad, ktiles;
    long long s_stride, b_stride, c_stride;  // replica strides (elements)
    long long Npad;                          // B * OH * Wp
    long long y_bs, r_bs;
    int act, yolo_classes;
};

constexpr int TC_BM = 128, TC_BK = 32, TC_STAGES = 4, TC_THREADS = 160;

// P[s][b][c][y][x] for s < KW, y < H + 2*pad, x < Wp
__global__ void k_tc_repack(const float* __restrict__ x, long long x_bs, float* __restrict__ P, int B, int C,
                            int H, int W, int KW, int pad, int Hp, int Wp) {
    const long long total = (long long)KW * B * C * Hp * Wp;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int xx = (int)(i % Wp);
        long long t = i / Wp;
        int yy = (int)(t % Hp);
        t /= Hp;
        int c = (int)(t % C);
        t /= C;
        int b = (int)(t % B);
        int s = (int)(t / B);
        int iy = yy - pad, ix = xx + s - pad;
        float v = 0.f;
        if (xx < W && (unsigned)iy < (unsigned)H && (unsigned)ix < (unsigned)W)
            v = x[b * x_bs + ((long long)c * H + iy) * W + ix];
        P[i] = v;
    }
}

template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1) k_conv_tc(const TcParams p) {
    constexpr int A_BYTES = TC_BK * TC_BM * 4;
    constexpr int B_BYTES = TC_BK * BN * 4;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment of the operand ring (swizzle atoms)
    unsigned char* smem = smem_raw + ((1024 - ((unsigned)__cvta_generic_to_shared(smem_raw) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full_bar[TC_STAGES], empty_bar[TC_STAGES], acc_bar;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * TC_BM;
    const long long n0 = (long long)blockIdx.x * BN;
    const unsigned sbase = (unsigned)__cvta_generic_to_shared(smem);

    if (tid == 0) {
        for (int s = 0; s < TC_STAGES; ++s) {
            tc::mbar_init(&full_bar[s], 128);
            tc::mbar_init(&empty_bar[s], 1);
        }
        tc::mbar_init(&acc_bar, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 4) tc::tmem_alloc(&tmem_base, BN);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_d = tmem_base;
    const int nkt = p.ktiles;
    const int csteps = p.C / TC_BK;  // k tiles per (r, s) tap

    if (warp < 4) {
        // ---------------- producers ----------------
        // per-thread B chunk assignment: 16-byte chunks (4 pixels) of the BK x BN tile
        for (int kt = 0; kt < nkt + 2; ++kt) {
            if (kt < nkt) {
                const int st = kt % TC_STAGES, use = kt / TC_STAGES;
                if (use > 0 && !tc::mbar_wait_bounded(&empty_bar[st], (use - 1) & 1, &abort_flag, p.status, 901))
                    break;
                const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + A_BYTES;
                // A: rows k0..k0+31 of Wp, columns m0..m0+127
                const float* wsrc = p.w + (long long)kt * TC_BK * p.Mpad + m0;
#pragma unroll
                for (int i = 0; i < (TC_BK * TC_BM / 4) / 128; ++i) {
                    int idx = tid + i * 128;
                    int k = idx / (TC_BM / 4), mq = (idx % (TC_BM / 4)) * 4;
                    bool ok = m0 + mq < p.Mpad;
                    const float* src = ok ? wsrc + (long long)k * p.Mpad + mq : p.w;
                    unsigned dst = sa + tc::sw128_32b_chunk(mq, k, TC_BM);
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                                 "r"(ok ? 16 : 0));
                }
                // B: tap (r, s) and channels c0..c0+31 of this k tile, pixels n0..n0+BN-1
                const int rs = kt / csteps, c0 = (kt - rs * csteps) * TC_BK;
                const int r = rs / p.KW, s = rs - r * p.KW;
                const long long img = (long long)p.OH * p.Wp;
#pragma unroll 4
                for (int i = 0; i < (TC_BK * BN / 4) / 128; ++i) {
                    int idx = tid + i * 128;
                    int k = idx / (BN / 4), nq = (idx % (BN / 4)) * 4;
                    long long n = n0 + nq;
                    bool ok = n < p.Npad;
                    const float* src = p.p;
                    if (ok) {
                        long long b = n / img, q = n - b * img;
                        src = p.p + s * p.s_stride + b * p.b_stride + (long long)(c0 + k) * p.c_stride +
                              (long long)r * p.Wp + q;
                    }
                    unsigned dst = sb + tc::sw128_32b_chunk(nq, k, BN);
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                                 "r"(ok ? 16 : 0));
                }
            }
            asm volatile("cp.async.commit_group;\n" ::);
            // stage kt-2 has landed: make it visible to the tensor core's async proxy, signal
            if (kt >= 2) {
                asm volatile("cp.async.wait_group 2;\n" ::: "memory");
                tc::fence_proxy_async();
                tc::mbar_arrive(&full_bar[(kt - 2) % TC_STAGES]);
            }
        }
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    } else if (warp == 4) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = tc::idesc_tf32_mn(TC_BM, BN);
        for (int kt = 0; kt < nkt; ++kt) {
            const int st = kt % TC_STAGES, use = kt / TC_STAGES;
            if (!tc::mbar_wait_bounded(&full_bar[st], use & 1, &abort_flag, p.status, 902)) break;
            tc::tc_fence_after();
            if (lane == 0) {
                const unsigned sa = sbase + st * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                for (int kk = 0; kk < TC_BK / 8; ++kk) {
                    // K = 8 per MMA: two 4-row K-groups of (MN/32)*512 bytes each
                    uint64_t da = tc::smem_desc_mn_sw128_32b(sa + kk * (TC_BM / 32) * 1024, 512, (TC_BM / 32) * 512);
                    uint64_t db = tc::smem_desc_mn_sw128_32b(sb + kk * (BN / 32) * 1024, 512, (BN / 32) * 512);
                    tc::mma_tf32(tmem_d, da, db, idesc, (kt | kk) ? 1u : 0u);
                }
                tc::mma_commit(&empty_bar[st]);
                if (kt == nkt - 1) tc::mma_commit(&acc_bar);
            }
            __syncwarp();
        }
    }

    // ---------------- epilogue (warps 0-3: TMEM lanes 32w .. 32w+31) ----------------
    if (warp < 4) {
        bool ok = !abort_flag && tc::mbar_wait_bounded(&acc_bar, 0, &abort_flag, p.status, 903);
        if (__all_sync(0xffffffffu, ok)) {  // tcgen05.ld is warp-collective: all lanes or none
            tc::tc_fence_after();
            const int m = m0 + warp * 32 + lane;
            const long long img = (long long)p.OH * p.Wp;
            const int OHW = p.OH * p.OW;
#pragma unroll 1
            for (int j = 0; j < BN / 32; ++j) {
                float v[32];
                tc::tmem_ld32(tmem_d + ((uint32_t)(warp * 32) << 16) + j * 32, v);
                if (m >= p.F) continue;
                const long long nb = n0 + j * 32;
#pragma unroll
                for (int q = 0; q < 32; ++q) {
                    long long n = nb + q;
                    if (n >= p.Npad) break;
                    long long b = n / img, rem = n - b * img;
                    int oy = (int)(rem / p.Wp), ox = (int)(rem - (long long)oy * p.Wp);
                    if (ox >= p.OW) continue;
                    ConvParams ep;  // only the epilogue fields are read
                    ep.bias = p.bias; ep.bn_scale = p.bn_scale; ep.bn_mean = p.bn_mean; ep.bn_var = p.bn_var;
                    ep.act = p.act; ep.yolo_classes = p.yolo_classes;
                    float o = conv_epilogue(v[q], m, ep);
                    const long long off = (long long)m * OHW + (long long)oy * p.OW + ox;
                    if (p.res) o = __fadd_rn(o, p.res[b * p.r_bs + off]);
                    p.y[b * p.y_bs + off] = o;
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 4) tc::tmem_dealloc(tmem_d, BN);
}

// ---------------------------------------------------------------------------------------
bool conv_tc_supported(const ConvGeom& g) {
    return g.SY == 1 && g.SX == 1 && g.DY == 1 && g.DX == 1 && g.C % TC_BK == 0 && g.rsc &&
           g.Cpad == g.C && g.KH == g.KW && g.PY == (g.KH - 1) / 2 && g.PX == g.PY &&
           g.OH == g.H && g.OW == g.W;
}

int64_t conv_tc_scratch_floats(const ConvGeom& g) {
    const int64_t Wp = round_up(g.W, 4), Hp = g.H + 2 * g.PY;
    return g.KW * g.B * g.C * Hp * Wp;
}

int conv_tc_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                   const float* bn_scale, const float* bn_mean, const float* bn_var, const float* res,
                   float* y, int act, int yolo_classes, float* scratch, int64_t* launches) {
    if (!conv_tc_supported(g)) return fail(TB_ERR_UNSUPPORTED, "tensor-core conv: unsupported geometry");
    const int64_t Wp = round_up(g.W, 4), Hp = g.H + 2 * g.PY;
    TcParams p{};
    p.w = wp; p.bias = bias; p.bn_scale = bn_scale; p.bn_mean = bn_mean; p.bn_var = bn_var;
    p.res = res; p.y = y; p.status = ctx->d_status;
    p.C = (int)g.C; p.F = (int)g.F; p.KH = (int)g.KH; p.KW = (int)g.KW; p.OH = (int)g.OH; p.OW = (int)g.OW;
    p.Wp = (int)Wp; p.Hp = (int)Hp; p.Mpad = (int)g.Mpad;
    p.ktiles = (int)(g.KH * g.KW * g.C / TC_BK);
    p.c_stride = Hp * Wp;
    p.b_stride = g.C * Hp * Wp;
    p.s_stride = g.B * g.C * Hp * Wp;
    p.Npad = g.B * g.OH * Wp;
    p.y_bs = g.y_bs; p.r_bs = g.r_bs;
    p.act = act; p.yolo_classes = yolo_classes;
    // tap replicas (a 1x1 layer whose rows are already 4-aligned reads x in place)
    if (g.KW == 1 && g.W % 4 == 0 && g.x_bs % 4 == 0 && aligned16(x)) {
        p.p = x;
        p.b_stride = g.x_bs;
    } else {
        const int64_t total = conv_tc_scratch_floats(g);
        k_tc_repack<<<grid_for(total, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
            x, g.x_bs, scratch, (int)g.B, (int)g.C, (int)g.H, (int)g.W, (int)g.KW, (int)g.PY, (int)Hp, (int)Wp);
        int r = check_launch("k_tc_repack");
        if (r != TB_OK) return r;
        if (launches) ++*launches;
        p.p = scratch;
    }
    const int BN = (ceil_div(p.Npad, 256) * ceil_div(g.F, TC_BM) >= ctx->sm_count) ? 256 : 128;
    const int smem = TC_STAGES * (TC_BK * TC_BM * 4 + TC_BK * BN * 4) + 1024;
    dim3 grid((unsigned)ceil_div(p.Npad, BN), (unsigned)ceil_div(g.F, TC_BM));
    static std::mutex mu;
    static bool done[2][64] = {{false}};
    {
        std::lock_guard<std::mutex> lk(mu);
        int which = BN == 256 ? 1 : 0;
        if (ctx->device < 64 && !done[which][ctx->device]) {
            cudaError_t e = BN == 256
                ? cudaFuncSetAttribute(k_conv_tc<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)
                : cudaFuncSetAttribute(k_conv_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(conv_tc)");
            done[which][ctx->device] = true;
        }
    }
    if (BN == 256) k_conv_tc<256><<<grid, TC_THREADS, smem, ctx->stream>>>(p);
    else k_conv_tc<128><<<grid, TC_THREADS, smem, ctx->stream>>>(p);
    int r = check_launch("k_conv_tc");
    if (r != TB_OK) return r;
    if (launches) ++*launches;
    return TB_OK;
}

}  // namespace tbi
