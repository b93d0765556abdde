// conv_fp32.cu -- host side of the FP32 implicit-GEMM convolution: geometry, tile selection,
// split-K reduction, weight packing and the tb_conv_* entry points.
#include "conv_fp32_kernel.cuh"

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <vector>

namespace tbi {

__global__ void k_conv_pack(const float* __restrict__ w, float* __restrict__ wp, int F, int C,
                            int KH, int KW, int Cpad, long long Kpad, int Mpad, int rsc) {
    const long long total = Kpad * Mpad;
    const long long fs = (long long)C * KH * KW;
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        long long k = idx / Mpad;
        int m = (int)(idx - k * Mpad);
        float v = 0.0f;
        if (m < F) {
            int c, r, s;
            if (rsc) {
                int rs = (int)(k / Cpad);
                c = (int)(k - (long long)rs * Cpad);
                r = rs / KW;
                s = rs - r * KW;
            } else {
                int khw = KH * KW;
                c = (int)(k / khw);
                int rs = (int)(k - (long long)c * khw);
                r = rs / KW;
                s = rs - r * KW;
            }
            if (c < C) v = w[(long long)m * fs + ((long long)c * KH + r) * KW + s];
        }
        wp[idx] = v;
    }
}

int conv_geom(const tb_conv_desc* d, ConvGeom* g) {
    if (!d) return fail(TB_ERR_INVALID, "null conv descriptor");
    ConvGeom r;
    r.B = d->batch; r.C = d->channels; r.H = d->height; r.W = d->width;
    r.F = d->filters; r.KH = d->kernel_h; r.KW = d->kernel_w;
    r.SY = d->stride_y; r.SX = d->stride_x; r.PY = d->pad_y; r.PX = d->pad_x;
    r.DY = d->dilation_y > 0 ? d->dilation_y : 1;
    r.DX = d->dilation_x > 0 ? d->dilation_x : 1;
    if (r.B < 0 || r.C <= 0 || r.H <= 0 || r.W <= 0 || r.F <= 0 || r.KH <= 0 || r.KW <= 0 ||
        r.SY <= 0 || r.SX <= 0 || r.PY < 0 || r.PX < 0)
        return fail(TB_ERR_INVALID, "conv: bad shape (batch=%lld c=%lld h=%lld w=%lld f=%lld k=%lldx%lld s=%lldx%lld p=%lldx%lld)",
                    (long long)r.B, (long long)r.C, (long long)r.H, (long long)r.W, (long long)r.F,
                    (long long)r.KH, (long long)r.KW, (long long)r.SY, (long long)r.SX,
                    (long long)r.PY, (long long)r.PX);
    r.OH = (r.H + 2 * r.PY - (r.DY * (r.KH - 1) + 1)) / r.SY + 1;
    r.OW = (r.W + 2 * r.PX - (r.DX * (r.KW - 1) + 1)) / r.SX + 1;
    if (r.OH <= 0 || r.OW <= 0) return fail(TB_ERR_INVALID, "conv: empty output (kernel larger than padded input)");
    r.x_bs = d->in_batch_stride ? d->in_batch_stride : r.C * r.H * r.W;
    r.y_bs = d->out_batch_stride ? d->out_batch_stride : r.F * r.OH * r.OW;
    r.r_bs = d->res_batch_stride ? d->res_batch_stride : r.y_bs;
    if (r.x_bs < r.C * r.H * r.W || r.y_bs < r.F * r.OH * r.OW || r.r_bs < r.F * r.OH * r.OW)
        return fail(TB_ERR_INVALID, "conv: batch stride smaller than one image");
    const int64_t lim = (int64_t)1 << 31;
    if (r.C * r.H * r.W >= lim || r.F * r.OH * r.OW >= lim || r.B * r.OH * r.OW >= lim ||
        (r.B - 1) * std::max(r.x_bs, std::max(r.y_bs, r.r_bs)) >= lim * 64)
        return fail(TB_ERR_INVALID, "conv: tensor too large for this build");
    r.rsc = conv_is_rsc(r.C, r.KH, r.KW);
    if (r.rsc) {
        r.Cpad = round_up(r.C, CONV_BK);
        r.Kpad = r.KH * r.KW * r.Cpad;
    } else {
        r.Cpad = r.C;
        r.Kpad = round_up(r.C * r.KH * r.KW, CONV_BK);
    }
    r.Mpad = round_up(r.F, 4);
    if (r.Kpad >= lim / 4 || r.Kpad * r.Mpad >= lim * 2)
        return fail(TB_ERR_INVALID, "conv: weights too large for this build");
    *g = r;
    return TB_OK;
}

struct TileCfg {
    int BM, BN, splits, kt_per_split;
    int mode;
    int tma;  // 1: the TMA-fed kernel (conv_fp32_tma.cu, 128 x 128 tile); chosen only by measurement
};

static int conv_mode_of(const ConvGeom& g, bool x_aligned16) {
    if (g.KH == 1 && g.KW == 1 && g.SY == 1 && g.SX == 1 && g.PY == 0 && g.PX == 0 &&
        (g.OH * g.OW) % 4 == 0 && g.x_bs % 4 == 0 && x_aligned16)
        return MODE_1X1V;
    return g.rsc ? MODE_RSC : MODE_CRS;
}

static int ctas_per_sm(tb_ctx* ctx, int BM, int BN, int mode) {
    ConvParams dummy{};
    dim3 q(0, 0, 0);
    if (BM == 128) return conv_launch_128x128(ctx, dummy, q, mode);
    if (BM == 64 && BN == 128) return conv_launch_64x128(ctx, dummy, q, mode);
    if (BM == 64) return conv_launch_64x64(ctx, dummy, q, mode);
    return conv_launch_32x256(ctx, dummy, q, mode);
}

// Pick the CTA tile and the K split with a wave-quantisation cost model:
//   waves(s)  = ceil(tiles * s / (SMs * CTAs per SM))
//   time      = waves * (per-CTA FMAs of one split) * (CTAs per SM) / (SM FMA rate * tile eff.)
//             + split-K partial traffic (write + read of s partial planes)
// Larger tiles reuse operands better (efficiency factor); splitting K fills the last wave.
// Measured choices (conv_fp32_autotune), per device and geometry.
static std::mutex g_tune_mu;
static std::map<std::vector<int64_t>, TileCfg> g_tuned;

static std::vector<int64_t> tune_key(const tb_ctx* ctx, const ConvGeom& g, int mode) {
    return {ctx->device, g.B, g.C, g.H, g.W, g.F, g.KH, g.KW, g.SY, g.SX, g.PY, g.PX, g.DY, g.DX,
            g.x_bs, g.y_bs, mode};
}

static TileCfg choose_tiles(tb_ctx* ctx, const ConvGeom& g, bool x_aligned16, bool allow_tma = true) {
    TileCfg best{};
    best.mode = conv_mode_of(g, x_aligned16);
    if (!getenv("TB_CONV_FORCE")) {
        std::lock_guard<std::mutex> lk(g_tune_mu);
        auto it = g_tuned.find(tune_key(ctx, g, best.mode));
        if (it != g_tuned.end() && (allow_tma || !it->second.tma)) return it->second;
    }
    const int64_t M = g.F, N = g.B * g.OH * g.OW;
    const int64_t ktiles = g.Kpad / CONV_BK;
    struct Cand { int BM, BN; double eff; };
    const Cand cands[] = {{128, 128, 1.00}, {64, 128, 0.90}, {64, 64, 0.78}, {32, 256, 0.85}};
    double best_cost = 1e300;
    for (const Cand& c : cands) {
        if (M <= 32 && c.BM != 32) continue;           // waste more than half the rows
        if (M > 32 && M <= 64 && c.BM == 128) continue;
        if (M > 64 && c.BM == 32) continue;
        const int64_t tiles = ceil_div(M, c.BM) * ceil_div(N, c.BN);
        const int occ = ctas_per_sm(ctx, c.BM, c.BN, best.mode);
        const int64_t slots = (int64_t)ctx->sm_count * occ;
        // useful fraction of the tile (ragged M / N edges)
        const double fill = (double)M * (double)N / ((double)ceil_div(M, c.BM) * c.BM * (double)ceil_div(N, c.BN) * c.BN);
        int64_t smax = ktiles / 4;
        if (smax > 16) smax = 16;
        if (smax < 1) smax = 1;
        if (tiles >= 4 * slots) smax = 1;
        if (tiles * 1 > (ctx->tile_cnt_len)) smax = 1;
        for (int64_t sp = 1; sp <= smax; ++sp) {
            const int64_t kps = ceil_div(ktiles, sp);
            const int64_t s2 = ceil_div(ktiles, kps);
            if (s2 != sp) continue;
            const double waves = (double)ceil_div(tiles * sp, slots);
            const double cta_cycles = (double)c.BM * c.BN * (double)kps * CONV_BK * occ / (128.0 * c.eff * fill);
            double cost = waves * cta_cycles + 2000.0;  // + launch / prologue latency per wave
            if (sp > 1) cost += (double)sp * (double)M * (double)N * 8.0 / 3400.0 + 3000.0;
            if (cost < best_cost * 0.999) {
                best_cost = cost;
                best.BM = c.BM; best.BN = c.BN; best.splits = (int)sp; best.kt_per_split = (int)kps;
            }
        }
    }
    // test hook: TB_CONV_FORCE="BM,BN,splits" pins the tile configuration (parity tests of
    // every configuration); unset in normal use
    if (const char* f = getenv("TB_CONV_FORCE")) {
        int bm = 0, bn = 0, sp = 0, tma = 0;
        if (sscanf(f, "%d,%d,%d,%d", &bm, &bn, &sp, &tma) >= 3 &&
            ((bm == 128 && bn == 128) || (bm == 64 && bn == 128) || (bm == 64 && bn == 64) || (bm == 32 && bn == 256))) {
            best.BM = bm; best.BN = bn;
            best.tma = (tma == 1 && bm == 128 && bn == 128 && allow_tma && conv_fp32_tma_supported(g)) ? 1 : 0;
            int64_t spl = sp < 1 ? 1 : (sp > ktiles ? ktiles : sp);
            int64_t kps = ceil_div(ktiles, spl);
            best.kt_per_split = (int)kps;
            best.splits = (int)ceil_div(ktiles, kps);
        }
    }
    return best;
}

static int64_t ws_floats_of(const ConvGeom& g, const TileCfg& t) {
    if (t.tma) return conv_fp32_tma_ws_floats(g, t.splits);
    return t.splits > 1 ? (int64_t)t.splits * g.F * g.B * g.OH * g.OW : 0;
}

int64_t conv_fp32_ws_floats(tb_ctx* ctx, const ConvGeom& g) {
    return std::max(ws_floats_of(g, choose_tiles(ctx, g, true)), ws_floats_of(g, choose_tiles(ctx, g, false)));
}

int64_t conv_fp32_ws_floats_for(tb_ctx* ctx, const ConvGeom& g, const float* x, bool allow_tma) {
    return ws_floats_of(g, choose_tiles(ctx, g, aligned16(x), allow_tma));
}

// A caller-provided scratch of cap_floats partial sums and cap_tiles counters: keep the chosen
// tile but lower its K split to the largest count whose partial planes fit (down to 1, which
// needs none).  A split pinned through TB_CONV_FORCE is kept as it is.
static TileCfg fit_to_scratch(const ConvGeom& g, TileCfg t, int64_t cap_floats, int64_t cap_tiles) {
    if (t.tma || t.splits <= 1 || getenv("TB_CONV_FORCE")) return t;
    const int64_t ktiles = g.Kpad / CONV_BK;
    const int64_t tiles = ceil_div(g.F, t.BM) * ceil_div(g.B * g.OH * g.OW, t.BN);
    for (int64_t sp = t.splits; sp >= 1; --sp) {
        const int64_t kps = ceil_div(ktiles, sp);
        const int64_t s2 = ceil_div(ktiles, kps);
        if (s2 == 1 || (s2 * g.F * g.B * g.OH * g.OW <= cap_floats && tiles <= cap_tiles)) {
            t.splits = (int)s2;
            t.kt_per_split = (int)kps;
            return t;
        }
    }
    return t;
}

int64_t conv_fp32_ws_floats_fit(tb_ctx* ctx, const ConvGeom& g, const float* x, int64_t cap_floats,
                                int64_t cap_tiles) {
    return ws_floats_of(g, fit_to_scratch(g, choose_tiles(ctx, g, aligned16(x), false), cap_floats, cap_tiles));
}

static int launch_with(tb_ctx* ctx, const ConvGeom& g, const TileCfg& t, const float* x, const float* wp,
                       const float* bias, const float* bn_scale, const float* bn_mean,
                       const float* bn_var, const float* res, float* y, int act, int yolo_classes,
                       float* ws, int64_t ws_floats, int64_t* launches, int* tile_cnt,
                       int64_t tile_cnt_len) {
    ConvParams p{};
    p.x = x; p.w = wp; p.bias = bias; p.bn_scale = bn_scale; p.bn_mean = bn_mean; p.bn_var = bn_var;
    p.res = res; p.y = y; p.ws = nullptr;
    p.tile_cnt = tile_cnt ? tile_cnt : ctx->tile_cnt;
    const int64_t cnt_len = tile_cnt ? tile_cnt_len : ctx->tile_cnt_len;
    p.C = (int)g.C; p.H = (int)g.H; p.W = (int)g.W; p.F = (int)g.F;
    p.KH = (int)g.KH; p.KW = (int)g.KW; p.SY = (int)g.SY; p.SX = (int)g.SX;
    p.PY = (int)g.PY; p.PX = (int)g.PX; p.DY = (int)g.DY; p.DX = (int)g.DX;
    p.OH = (int)g.OH; p.OW = (int)g.OW; p.OHW = (int)(g.OH * g.OW);
    p.Cpad = (int)g.Cpad; p.Kpad = (int)g.Kpad; p.Mpad = (int)g.Mpad;
    p.x_bs = g.x_bs; p.y_bs = g.y_bs; p.r_bs = g.r_bs;
    p.Ntot = g.B * g.OH * g.OW;
    p.ktiles = (int)(g.Kpad / CONV_BK);
    p.kt_per_split = t.kt_per_split;
    p.splits = t.splits;
    p.act = act;
    p.yolo_classes = yolo_classes;
    p.vec_out = (p.OHW % 4 == 0 && g.y_bs % 4 == 0 && aligned16(y) &&
                 (!res || (g.r_bs % 4 == 0 && aligned16(res)))) ? 1 : 0;
    if (t.tma) {  // replica + split-K partials in the given scratch or the context workspace
        const int64_t need = conv_fp32_tma_ws_floats(g, t.splits);
        float* wsp = ws;
        int64_t wsf = ws_floats;
        if (!wsp) {
            int r = ensure_workspace(ctx, (size_t)need * sizeof(float));
            if (r != TB_OK) return r;
            wsp = reinterpret_cast<float*>(ctx->ws);
            wsf = need;
        }
        return conv_fp32_tma_run(ctx, g, p, wsp, wsf, cnt_len, launches);
    }
    dim3 grid((unsigned)ceil_div(p.Ntot, t.BN), (unsigned)ceil_div(g.F, t.BM), (unsigned)t.splits);
    if (grid.y > 65535 || grid.z > 65535) return fail(TB_ERR_INVALID, "conv: grid too large");
    if (t.splits > 1) {
        if ((int64_t)grid.x * grid.y > cnt_len)
            return fail(TB_ERR_INVALID, "conv: %lld split-K tiles exceed the counter array",
                        (long long)grid.x * grid.y);
        int64_t need = (int64_t)t.splits * g.F * p.Ntot;
        if (ws) {
            if (ws_floats < need) return fail(TB_ERR_INVALID, "conv: scratch of %lld floats too small (need %lld)",
                                              (long long)ws_floats, (long long)need);
            p.ws = ws;
        } else {
            int r = ensure_workspace(ctx, (size_t)need * sizeof(float));
            if (r != TB_OK) return r;
            p.ws = reinterpret_cast<float*>(ctx->ws);
        }
    }
    int r;
    if (t.BM == 128) r = conv_launch_128x128(ctx, p, grid, t.mode);
    else if (t.BM == 64 && t.BN == 128) r = conv_launch_64x128(ctx, p, grid, t.mode);
    else if (t.BM == 64) r = conv_launch_64x64(ctx, p, grid, t.mode);
    else r = conv_launch_32x256(ctx, p, grid, t.mode);
    if (r != TB_OK) return r;
    if (launches) ++*launches;
    return TB_OK;
}

int conv_fp32_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp,
                     const float* bias, const float* bn_scale, const float* bn_mean,
                     const float* bn_var, const float* res, float* y, int act, int yolo_classes,
                     float* ws, int64_t ws_floats, int64_t* launches, int* tile_cnt,
                     int64_t tile_cnt_len, bool allow_tma) {
    if (g.B == 0) return TB_OK;
    if (conv_direct_supported(g, res, yolo_classes) && !getenv("TB_CONV_FORCE"))
        return conv_direct_launch(ctx, g, x, wp, bias, bn_scale, bn_mean, bn_var, y, act, launches);
    TileCfg t = choose_tiles(ctx, g, aligned16(x), allow_tma);
    if (ws) t = fit_to_scratch(g, t, ws_floats, tile_cnt ? tile_cnt_len : ctx->tile_cnt_len);
    return launch_with(ctx, g, t, x, wp, bias, bn_scale, bn_mean, bn_var, res, y, act, yolo_classes,
                       ws, ws_floats, launches, tile_cnt, tile_cnt_len);
}

// Time every admissible (tile, split) of this geometry on the given buffers and remember the
// fastest; later launches of the same geometry use it.  Blocks; allocates the workspace the
// candidates need (not during stream capture).
int conv_fp32_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, float* y) {
    if (g.B == 0 || conv_direct_supported(g, nullptr, 0)) return TB_OK;
    const int mode = conv_mode_of(g, aligned16(x));
    const int64_t M = g.F, N = g.B * g.OH * g.OW;
    const int cfgs[4][2] = {{128, 128}, {64, 128}, {64, 64}, {32, 256}};
    const int split_list[] = {1, 2, 3, 4, 6, 8, 12, 16};
    std::vector<TileCfg> cands;
    for (auto& c : cfgs) {
        if (M <= 32 && c[0] != 32) continue;
        if (M > 64 && c[0] == 32) continue;
        const int64_t kt = g.Kpad / CONV_BK;
        const int64_t tiles = ceil_div(M, c[0]) * ceil_div(N, c[1]);
        for (int sp : split_list) {
            if (sp > 1 && (sp > kt / 2 || tiles > ctx->tile_cnt_len || tiles * sp > 64 * (int64_t)ctx->sm_count))
                continue;
            const int64_t kps = ceil_div(kt, sp);
            if (ceil_div(kt, kps) != sp) continue;
            if ((int64_t)sp * M * N * 4 > ((int64_t)512 << 20)) continue;  // 512 MiB scratch cap
            TileCfg t{};
            t.BM = c[0]; t.BN = c[1]; t.splits = sp; t.kt_per_split = (int)kps; t.mode = mode;
            cands.push_back(t);
            if (c[0] == 128 && conv_fp32_tma_supported(g)) {  // the TMA-fed kernel, same split
                t.tma = 1;
                cands.push_back(t);
            }
        }
    }
    if (cands.empty()) return TB_OK;
    int64_t ws_need = 0;
    for (auto& t : cands) ws_need = std::max<int64_t>(ws_need, ws_floats_of(g, t));
    if (ws_need) {
        int r = ensure_workspace(ctx, (size_t)ws_need * 4);
        if (r != TB_OK) return r;
    }
    cudaEvent_t e0, e1;
    TB_CHECK_CUDA(cudaEventCreate(&e0));
    TB_CHECK_CUDA(cudaEventCreate(&e1));
    float best_ms = 1e30f;
    TileCfg best = cands[0];
    int rc = TB_OK;
    for (auto& t : cands) {
        rc = launch_with(ctx, g, t, x, wp, nullptr, nullptr, nullptr, nullptr, nullptr, y, TB_ACT_LINEAR,
                         0, nullptr, 0, nullptr, nullptr, 0);  // warm-up
        if (rc != TB_OK) {
            if (t.tma) {  // a geometry the TMA maps cannot describe: keep the gather kernels
                rc = TB_OK;
                continue;
            }
            break;
        }
        stream_delay_us(ctx, 200);  // the timed launches queue behind it: device time only
        cudaEventRecord(e0, ctx->stream);
        for (int rep = 0; rep < 3 && rc == TB_OK; ++rep)
            rc = launch_with(ctx, g, t, x, wp, nullptr, nullptr, nullptr, nullptr, nullptr, y, TB_ACT_LINEAR,
                             0, nullptr, 0, nullptr, nullptr, 0);
        cudaEventRecord(e1, ctx->stream);
        cudaError_t e = cudaEventSynchronize(e1);
        if (rc != TB_OK) break;
        if (e != cudaSuccess) { rc = cuda_fail(e, "autotune"); break; }
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (getenv("TB_AUTOTUNE_VERBOSE"))
            fprintf(stderr, "autotune C%lld H%lld F%lld k%lld s%lld B%lld: %dx%d split %d mode %d tma %d: %.4f ms\n",
                    (long long)g.C, (long long)g.H, (long long)g.F, (long long)g.KH, (long long)g.SY,
                    (long long)g.B, t.BM, t.BN, t.splits, t.mode, t.tma, ms / 3);
        if (ms < best_ms) { best_ms = ms; best = t; }
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc != TB_OK) return rc;
    std::lock_guard<std::mutex> lk(g_tune_mu);
    g_tuned[tune_key(ctx, g, mode)] = best;
    return TB_OK;
}

}  // namespace tbi

using namespace tbi;

extern "C" {

int tb_conv_out_shape(const tb_conv_desc* d, int64_t* out_h, int64_t* out_w) {
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (out_h) *out_h = g.OH;
    if (out_w) *out_w = g.OW;
    return TB_OK;
}

int tb_conv_packed_weights_count(const tb_conv_desc* d, int64_t* count) {
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!count) return fail(TB_ERR_INVALID, "null count");
    *count = g.Kpad * g.Mpad;
    return TB_OK;
}

int tb_conv_pack_weights(tb_ctx* ctx, const tb_conv_desc* d, const float* weights, float* packed) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!weights || !packed) return fail(TB_ERR_INVALID, "conv pack: null pointer");
    if (!aligned16(packed)) return fail(TB_ERR_INVALID, "conv pack: packed buffer must be 16-byte aligned");
    int64_t total = g.Kpad * g.Mpad;
    k_conv_pack<<<grid_for(total, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
        weights, packed, (int)g.F, (int)g.C, (int)g.KH, (int)g.KW, (int)g.Cpad, (long long)g.Kpad,
        (int)g.Mpad, g.rsc ? 1 : 0);
    return check_launch("k_conv_pack");
}

int tb_conv_uses_tensor_cores(const tb_conv_desc* d, int64_t math_mode, int64_t* yes) {
    if (!yes) return fail(TB_ERR_INVALID, "tb_conv_uses_tensor_cores: null result pointer");
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    *yes = (math_mode == TB_MATH_TF32 && conv_tc_supported(g)) ? 1 : 0;
    return TB_OK;
}

int tb_conv_pack_weights_tf32(tb_ctx* ctx, const tb_conv_desc* d, const float* weights, float* packed) {
    int r = tb_conv_pack_weights(ctx, d, weights, packed);
    if (r != TB_OK) return r;
    ConvGeom g;
    conv_geom(d, &g);
    return conv_tc_round_weights(ctx, packed, g.Kpad * g.Mpad);
}

int tb_conv_fold_bn(int64_t filters, int64_t filter_size, float* weights, float* biases,
                    const float* scales, const float* mean, const float* variance) {
    if (filters <= 0 || filter_size <= 0 || !weights || !biases || !scales || !mean || !variance)
        return fail(TB_ERR_INVALID, "tb_conv_fold_bn: bad arguments");
    const float eps = 0.000001f;  // sEPSILON
    for (int64_t f = 0; f < filters; ++f) {
        float v = variance[f] > eps ? variance[f] : eps;
        float pre = (float)((double)scales[f] / sqrt((double)v));
        biases[f] = biases[f] - mean[f] * pre;
        float* w = weights + f * filter_size;
        for (int64_t i = 0; i < filter_size; ++i) w[i] = w[i] * pre;
    }
    return TB_OK;
}

int tb_conv_autotune(tb_ctx* ctx, const tb_conv_desc* d, const float* x, const float* packed_w, float* y) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!x || !packed_w || !y) return fail(TB_ERR_INVALID, "conv autotune: null pointer");
    if (ctx->math_mode != TB_MATH_FP32_TILED && conv_exact_supported(g))
        return conv_exact_autotune(ctx, g, x, packed_w, y, true);
    return conv_fp32_autotune(ctx, g, x, packed_w, y);
}

int tb_conv2d_fwd(tb_ctx* ctx, const tb_conv_desc* d, const float* x, const float* packed_w,
                  const float* bias, const float* bn_scale, const float* bn_mean,
                  const float* bn_variance, const float* residual, float* y, int64_t math_mode) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (g.B == 0) return TB_OK;
    if (!x || !packed_w || !y) return fail(TB_ERR_INVALID, "conv: null x, weights or y");
    if (bn_mean && !bn_variance) return fail(TB_ERR_INVALID, "conv: bn_mean given without bn_variance");
    if (!aligned16(packed_w)) return fail(TB_ERR_INVALID, "conv: packed weights must be 16-byte aligned");
    if (!act_supported(d->activation))
        return fail(TB_ERR_UNSUPPORTED, "conv: activation %lld not supported", (long long)d->activation);
    if (math_mode < 0) math_mode = ctx->math_mode;
    if (math_mode != TB_MATH_FP32 && math_mode != TB_MATH_TF32 && math_mode != TB_MATH_FP32_TILED)
        return fail(TB_ERR_UNSUPPORTED, "conv: math mode %lld is not available in this build", (long long)math_mode);
    if (math_mode == TB_MATH_TF32 && conv_tc_supported(g)) {
        r = ensure_workspace(ctx, (size_t)conv_tc_scratch_floats(g) * sizeof(float));
        if (r != TB_OK) return r;
        return conv_tc_launch(ctx, g, x, packed_w, bias, bn_scale, bn_mean, bn_variance, residual, y,
                              (int)d->activation, 0, reinterpret_cast<float*>(ctx->ws), nullptr);
    }
    if (math_mode != TB_MATH_FP32_TILED && conv_exact_supported(g))
        return conv_exact_launch(ctx, g, x, packed_w, bias, bn_scale, bn_mean, bn_variance, residual, y,
                                 (int)d->activation, 0, true, nullptr);
    return conv_fp32_launch(ctx, g, x, packed_w, bias, bn_scale, bn_mean, bn_variance, residual, y,
                            (int)d->activation, 0, nullptr, 0, nullptr);
}

int tb_diag_tc_mma_rate(tb_ctx* ctx, int64_t kmajor, double* tflops, double* cycles_per_mma) {
    TB_ENTER(ctx);
    if (!tflops || !cycles_per_mma) return fail(TB_ERR_INVALID, "null output");
    return conv_tc_mma_rate(ctx, (int)kmajor, tflops, cycles_per_mma);
}

int tb_diag_conv_tc_phases(tb_ctx* ctx, const tb_conv_desc* d, const float* x, const float* packed_w, float* y,
                           double* out12) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (!x || !packed_w || !y || !out12) return fail(TB_ERR_INVALID, "conv tc phases: null pointer");
    if (!conv_tc_supported(g)) return fail(TB_ERR_UNSUPPORTED, "conv tc phases: geometry not on the tensor-core path");
    r = ensure_workspace(ctx, (size_t)conv_tc_scratch_floats(g) * sizeof(float));
    if (r != TB_OK) return r;
    const int n = ctx->sm_count * 12;
    unsigned long long* dph = nullptr;
    TB_CHECK_CUDA(cudaMalloc(&dph, n * sizeof(unsigned long long)));
    cudaMemsetAsync(dph, 0, n * sizeof(unsigned long long), ctx->stream);
    r = conv_tc_launch(ctx, g, x, packed_w, nullptr, nullptr, nullptr, nullptr, nullptr, y, (int)d->activation, 0,
                       reinterpret_cast<float*>(ctx->ws), nullptr, dph);
    std::vector<unsigned long long> h(n);
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), dph, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(dph);
    if (r != TB_OK) return r;
    if (e != cudaSuccess) return cuda_fail(e, "conv tc phases");
    int ctas = 0;
    for (int i = 0; i < 12; ++i) out12[i] = 0;
    for (int c = 0; c < ctx->sm_count; ++c) {
        if (h[c * 12 + 0] == 0) continue;
        ++ctas;
        for (int i = 0; i < 12; ++i) out12[i] += (double)h[c * 12 + i];
    }
    for (int i = 0; i < 12 && ctas; ++i) out12[i] /= ctas;
    return TB_OK;
}

}  // extern "C"
