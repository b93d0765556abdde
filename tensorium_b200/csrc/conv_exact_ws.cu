// conv_exact_ws.cu -- warp-specialised variant of the order-exact FP32 convolution.
//
// Same arithmetic as k_conv_exact (conv_exact.cuh): k in the reference's im2col order, one fp32
// FMA chain per output, no split of K, the shared epilogue -- so the results are bit-identical.
// What changes is who moves the data: one producer warp issues every cp.async of a stage (the
// weight rows and the per-pixel activation gathers, with the address arithmetic and padding tests)
// and signals a "full" mbarrier per stage (cp.async.mbarrier.arrive.noinc: the arrival fires when
// the lane's copies have landed); the 4 or 8 compute warps only wait for "full", run the stage's
// LDS + FFMA stream and arrive on the stage's "empty" mbarrier.  No block-wide barrier remains in
// the mainloop, and the compute warps issue no loader instructions.  Every wait is bounded: on a
// timeout the CTA sets the context status word, lets the copies in flight land and returns.
#include "conv_exact.cuh"
#include "conv_tc.cuh"

namespace tbi {

namespace {

constexpr int WS_BM = 128, WS_STAGES = 4;

template <int MODE>
struct WsShape {
    static constexpr int CC = MODE == EX_3X3 ? 2 : 16;
    static constexpr int KS = MODE == EX_3X3 ? 18 : 16;
};

// Spin on mbarrier.test_wait (no suspension: these waits are short and on the FFMA stream's
// critical path), bounded like tc::mbar_wait_bounded.
__device__ __forceinline__ bool spin_wait(uint64_t* bar, unsigned parity, volatile int* abort, int* status, int code) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    const long long t0 = clock64();
    for (unsigned it = 0;; ++it) {
        unsigned ok;
        asm volatile(
            "{\n.reg .pred p;\nmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((it & 63) == 63) {
            if (*abort) return false;
            if (clock64() - t0 > (1ll << 32)) break;
        }
    }
    *abort = 1;
    if (status) atomicExch(status, code);
    return false;
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(a) : "memory");
}

template <int BN, int MODE>
__global__ void __launch_bounds__((WS_BM / 8) * (BN / 8) + 32, BN == 64 ? 3 : 1)
k_conv_exact_ws(const ConvParams p, int* status) {
    constexpr int BM = WS_BM, TM = 8, TN = 8, TM2 = 4, TX = BN / TN;
    constexpr int NC = (BM / TM) * (BN / TN);  // compute threads
    constexpr int KS = WsShape<MODE>::KS, CC = WsShape<MODE>::CC, S = WS_STAGES;
    extern __shared__ __align__(16) float smem[];
    float* As = smem;               // [S][KS][BM]
    float* Bs = smem + S * KS * BM;  // [S][KS][BN]
    __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S];
    __shared__ volatile int abort_flag;
    TB_GRID_DEP_ENTRY();

    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM;
    const long long n0 = (long long)blockIdx.x * BN;
    const int nst = (p.C + CC - 1) / CC;
    const long long HW = (long long)p.H * p.W;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(&full_bar[s], 32);       // one cp.async arrival per producer lane
            tc::mbar_init(&empty_bar[s], NC / 32);  // one arrival per compute warp
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();

    if (tid >= NC) {
        // ---------------- producer warp ----------------
        const int lane = tid - NC;
        // weights: this lane's 16-byte column quad of every row (RSC or CRS packed rows)
        const int KHKW = MODE == EX_3X3 ? 9 : 1;
        const bool w_ok = m0 + 4 * lane < p.Mpad;
        const long long wstep = (long long)(p.wrsc ? CC : CC * KHKW) * p.Mpad;
        // activations
        constexpr int PPL = BN / 32;  // 3x3: pixel columns per lane
        const float* pbase[PPL > 0 ? PPL : 1];
        unsigned tapok[PPL > 0 ? PPL : 1];
        const int rowstep = p.DY * p.W;
        if (MODE == EX_3X3) {
#pragma unroll
            for (int j = 0; j < PPL; ++j) {
                const long long n = n0 + lane + 32 * j;
                pbase[j] = p.x;
                tapok[j] = 0;
                if (n < p.Ntot) {
                    const unsigned b = (unsigned)n / (unsigned)p.OHW;
                    const int pix = (int)((unsigned)n - b * (unsigned)p.OHW);
                    const int oy = pix / p.OW, ox = pix - oy * p.OW;
                    const int iy0 = oy * p.SY - p.PY, ix0 = ox * p.SX - p.PX;
                    pbase[j] = p.x + (long long)b * p.x_bs + (long long)iy0 * p.W + ix0;
#pragma unroll
                    for (int r = 0; r < 3; ++r)
#pragma unroll
                        for (int s = 0; s < 3; ++s) {
                            const int iy = iy0 + r * p.DY, ix = ix0 + s * p.DX;
                            if ((unsigned)iy < (unsigned)p.H && (unsigned)ix < (unsigned)p.W) tapok[j] |= 1u << (r * 3 + s);
                        }
                }
            }
        }
        // 1x1 vectorised: this lane's pixel quad(s) (BN / 4 quads over 32 lanes)
        constexpr int QPL = BN / 128 > 0 ? BN / 128 : 1;
        const float* qbase[QPL];
        bool qok[QPL];
        if (MODE == EX_1X1V) {
#pragma unroll
            for (int j = 0; j < QPL; ++j) {
                const int q = lane + 32 * j;
                const long long nq = n0 + 4 * q;
                qok[j] = 4 * q < BN && nq < p.Ntot;
                qbase[j] = p.x;
                if (qok[j]) {
                    const unsigned b = (unsigned)nq / (unsigned)p.OHW;
                    qbase[j] = p.x + (long long)b * p.x_bs + ((unsigned)nq - b * (unsigned)p.OHW);
                }
            }
        }
        bool ok = true;
        int t = 0;
        for (; t < nst; ++t) {
            const int st = t % S, use = t / S;
            if (use > 0 && !spin_wait(&empty_bar[st], (use - 1) & 1, &abort_flag, status, 931)) {
                ok = false;
                break;
            }
            const int c0 = t * CC;
            float* as = As + st * KS * BM;
            float* bs = Bs + st * KS * BN;
            const float* wst = p.w + (long long)t * wstep;
#pragma unroll
            for (int row = 0; row < KS; ++row) {  // row = cc * KHKW + rs (the reference's k order)
                const int cc = row / KHKW, rs = row - cc * KHKW;
                const bool okw = w_ok && c0 + cc < p.C;
                const long long off = (long long)(p.wrsc ? rs * p.Cpad + cc : cc * KHKW + rs) * p.Mpad + m0 + 4 * lane;
                cp_async16(as + row * BM + 4 * lane, okw ? wst + off : p.w, okw);
            }
            if (MODE == EX_3X3) {
#pragma unroll
                for (int cc = 0; cc < CC; ++cc) {
                    const bool cok = c0 + cc < p.C;
                    const long long coff = (long long)(c0 + cc) * HW;
#pragma unroll
                    for (int j = 0; j < PPL; ++j)
#pragma unroll
                        for (int r = 0; r < 3; ++r)
#pragma unroll
                            for (int s = 0; s < 3; ++s) {
                                const bool okx = cok && ((tapok[j] >> (r * 3 + s)) & 1u);
                                const float* src = pbase[j] + coff + r * rowstep + s * p.DX;
                                cp_async4(bs + (cc * 9 + r * 3 + s) * BN + lane + 32 * j, okx ? src : p.x, okx);
                            }
                }
            } else {
#pragma unroll
                for (int row = 0; row < KS; ++row) {
                    const bool okc = c0 + row < p.C;
#pragma unroll
                    for (int j = 0; j < QPL; ++j)
                        if (4 * (lane + 32 * j) < BN)
                            cp_async16(bs + row * BN + 4 * (lane + 32 * j),
                                       (qok[j] && okc) ? qbase[j] + (long long)(c0 + row) * HW : p.x, qok[j] && okc);
                }
            }
            cp_async_arrive_noinc(&full_bar[st]);
        }
        cp_async_wait<0>();  // nothing in flight when the CTA leaves
        (void)ok;
        return;
    }

    // ---------------- compute warps ----------------
    const int tx = tid % TX, ty = tid / TX;
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;
    bool ok = true;
    for (int t = 0; t < nst; ++t) {
        const int st = t % S;
        if (!spin_wait(&full_bar[st], (t / S) & 1, &abort_flag, status, 932)) {
            ok = false;
            break;
        }
        const float* as = As + st * KS * BM;
        const float* bs = Bs + st * KS * BN;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            float a[TM], bv[TN];
            *reinterpret_cast<float4*>(&a[0]) = *reinterpret_cast<const float4*>(as + kk * BM + ty * TM2);
            *reinterpret_cast<float4*>(&a[4]) = *reinterpret_cast<const float4*>(as + kk * BM + BM / 2 + ty * TM2);
            *reinterpret_cast<float4*>(&bv[0]) = *reinterpret_cast<const float4*>(bs + kk * BN + tx * 4);
            *reinterpret_cast<float4*>(&bv[4]) = *reinterpret_cast<const float4*>(bs + kk * BN + BN / 2 + tx * 4);
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
        }
        __syncwarp();
        if ((tid & 31) == 0) tc::mbar_arrive(&empty_bar[st]);
    }
    if (!ok) return;

    // ---- epilogue (k_conv_exact's) ----
    const ColQuad cq[2] = {decode_quad(p, n0 + tx * 4), decode_quad(p, n0 + BN / 2 + tx * 4)};
    const bool simple = !p.bn_mean && p.yolo_classes == 0 && (p.act == TB_ACT_LEAKY || p.act == TB_ACT_LINEAR);
    const bool has_bias = p.bias != nullptr, leaky = p.act == TB_ACT_LEAKY;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int m = m0 + (i < TM2 ? ty * TM2 + i : BM / 2 + ty * TM2 + (i - TM2));
        if (m >= p.F) continue;
        const float bm = has_bias ? __ldg(p.bias + m) : 0.f;
#pragma unroll
        for (int gq = 0; gq < 2; ++gq) conv_store4(p, m, cq[gq], &acc[i][gq * 4], simple, has_bias, leaky, bm);
    }
}

template <int BN, int MODE>
int ws_launch_one(tb_ctx* ctx, const ConvParams& p, dim3 grid) {
    constexpr int NT = (WS_BM / 8) * (BN / 8) + 32;
    constexpr int smem = WS_STAGES * WsShape<MODE>::KS * (WS_BM + BN) * 4;
    auto kern = k_conv_exact_ws<BN, MODE>;
    static std::mutex mu;
    static bool done[64] = {false};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device >= 64) return fail(TB_ERR_UNSUPPORTED, "device index %d >= 64", ctx->device);
        if (!done[ctx->device]) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_conv_exact_ws)");
            done[ctx->device] = true;
        }
    }
    if (grid.x == 0) {
        int n = 1;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, NT, smem) != cudaSuccess || n < 1) n = 1;
        return n;
    }
    return launch(ctx, "k_conv_exact_ws", kern, grid, dim3(NT), (size_t)smem, p, ctx->d_status);
}

}  // namespace

// Warp-specialised exact conv (3x3 and vectorised 1x1 modes only): BN = 64 or 128 pixels per CTA,
// 128 filters. grid.x == 0 returns the resident CTAs per SM.
int exact_ws_launch(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, int bn) {
    if (mode == EX_3X3) return bn == 64 ? ws_launch_one<64, EX_3X3>(ctx, p, grid) : ws_launch_one<128, EX_3X3>(ctx, p, grid);
    if (mode == EX_1X1V) return bn == 64 ? ws_launch_one<64, EX_1X1V>(ctx, p, grid) : ws_launch_one<128, EX_1X1V>(ctx, p, grid);
    return fail(TB_ERR_UNSUPPORTED, "warp-specialised exact conv: mode %d", mode);
}

}  // namespace tbi
