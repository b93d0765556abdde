// conv_exact.cu -- host side of the order-exact FP32 convolution (conv_exact.cuh): mode and
// tile selection, measured tile choice per geometry, launch.
#include "conv_exact.cuh"

#include <algorithm>
#include <map>
#include <mutex>
#include <vector>

namespace tbi {

namespace {

struct ExactTile {
    int BM, BN, NT;
};
constexpr ExactTile kTiles[] = {{128, 128, 256}, {64, 128, 128}, {128, 64, 128}, {64, 64, 64}, {32, 128, 128}};
constexpr int kNumTiles = 5;
constexpr int kNumVariants = 4;  // stage-depth variants (ExactShape) of the 3x3 and 1x1-vector modes

// configurations: t = variant * kNumTiles + tile
int num_configs(int mode, bool fma) {
    if (mode == EX_3X3) return kNumVariants * kNumTiles;
    return (mode == EX_1X1V && fma) ? 3 * kNumTiles : kNumTiles;
}

int exact_mode_of(const ConvGeom& g, const float* x) {
    if (g.KH == 1 && g.KW == 1) {
        if (g.SY == 1 && g.SX == 1 && g.PY == 0 && g.PX == 0 && (g.H * g.W) % 4 == 0 && g.x_bs % 4 == 0 &&
            aligned16(x))
            return EX_1X1V;
        return EX_1X1;
    }
    if (g.KH == 3 && g.KW == 3) return EX_3X3;
    return EX_GEN;
}

// configurations >= kWsBase: the warp-specialised kernel (conv_exact_ws.cu), 128 filters x 64 or
// 128 pixels, 3x3 and vectorised 1x1 modes
constexpr int kWsBase = 100;
bool ws_mode(int mode, bool fma) { return fma && (mode == EX_3X3 || mode == EX_1X1V); }
// configurations 110 / 111: 32 outputs per thread, 64 x 64 (8 x 4) and 64 x 128 (4 x 8)
constexpr int kSmallBase = 110;
// configurations 120 .. 120 + SLIDE_TILES - 1: the staged-once 3x3 stride-1 kernel (conv_slide.cu)
constexpr int kSlideBase = 120;
bool is_slide(int t) { return t >= kSlideBase && t < kSlideBase + SLIDE_TILES; }

// tile index t of kTiles plus a stage-depth variant (ExactShape) in t / kNumTiles
int run_tile(tb_ctx* ctx, int t, const ConvParams& p, dim3 grid, int mode, bool fma) {
    if (t == kSmallBase) return exact_launch_64x64n4(ctx, p, grid, mode, fma, 0);
    if (t == kSmallBase + 1) return exact_launch_64x128m4(ctx, p, grid, mode, fma, 0);
    if (t >= kWsBase) return exact_ws_launch(ctx, p, grid, mode, t == kWsBase ? 64 : 128);
    const int var = t / kNumTiles;
    switch (t % kNumTiles) {
    case 0: return exact_launch_128x128(ctx, p, grid, mode, fma, var);
    case 1: return exact_launch_64x128(ctx, p, grid, mode, fma, var);
    case 2: return exact_launch_128x64(ctx, p, grid, mode, fma, var);
    case 3: return exact_launch_64x64(ctx, p, grid, mode, fma, var);
    default: return exact_launch_32x128(ctx, p, grid, mode, fma, var);
    }
}

int tile_bm(int t) {
    if (is_slide(t)) return slide_tile_bm(t - kSlideBase);
    if (t == kSmallBase) return 64;
    if (t == kSmallBase + 1) return 64;
    return t >= kWsBase ? 128 : kTiles[t % kNumTiles].BM;
}
int tile_bn(int t) {
    if (is_slide(t)) return slide_tile_bn(t - kSlideBase);
    if (t == kSmallBase) return 64;
    if (t == kSmallBase + 1) return 128;
    return t >= kWsBase ? (t == kWsBase ? 64 : 128) : kTiles[t % kNumTiles].BN;
}
int tile_nt(int t) {
    if (is_slide(t)) return slide_tile_nt(t - kSlideBase);
    if (t == kSmallBase) return 128;
    if (t == kSmallBase + 1) return 256;
    return t >= kWsBase ? (t == kWsBase ? 128 : 256) : kTiles[t % kNumTiles].NT;
}

bool tile_admissible(int t, int64_t M) {
    const int BM = tile_bm(t);
    if (is_slide(t) && BM == 32) return true;  // the staged-once 32x64 tiles: more CTAs for small layers
    if (M <= 32) return BM == 32;
    if (M <= 64) return BM <= 64;
    return BM >= 64;
}

// Wave model: an SM that receives k CTAs of a tile runs them at a rate that grows with the warps
// resident (full from 12 warps up); the layer ends with the busiest SM.
double model_cost(tb_ctx* ctx, int t, const ConvGeom& g, int mode) {
    const ExactTile T{tile_bm(t), tile_bn(t), tile_nt(t)};
    const int64_t M = g.F, N = g.B * g.OH * g.OW;
    const int64_t tiles = ceil_div(M, T.BM) * ceil_div(N, T.BN);
    ConvParams dummy{};
    int occ = run_tile(ctx, t, dummy, dim3(0, 0, 0), mode, true);
    if (occ < 1) occ = 1;
    const int64_t per_sm = ceil_div(tiles, ctx->sm_count);
    const int64_t rounds = ceil_div(per_sm, occ);
    const int64_t resident = std::min<int64_t>(per_sm, occ);
    const double warps = (double)resident * T.NT / 32.0;
    const double rate = std::min(1.0, warps / 12.0);
    const double eff = (T.BM * T.BN >= 16384) ? 1.0 : (T.BM == 32 ? 0.85 : (T.BM * T.BN == 8192 ? 0.95 : 0.9));
    return (double)rounds * resident * T.BM * T.BN / (rate * eff);
}

std::mutex g_mu;
std::map<std::vector<int64_t>, int> g_tuned;

std::vector<int64_t> key_of(const tb_ctx* ctx, const ConvGeom& g, int mode, bool fma) {
    return {ctx->device, g.B, g.C, g.H, g.W, g.F, g.KH, g.KW, g.SY, g.SX, g.PY, g.PX, g.DY, g.DX, g.x_bs, mode,
            fma ? 1 : 0};
}

int choose_tile(tb_ctx* ctx, const ConvGeom& g, int mode, bool fma) {
    // test hook: TB_EXACT_FORCE=<configuration> pins the CTA tile (index % 5) and stage-depth
    // variant (index / 5) for the parity tests of every configuration
    if (const char* f = getenv("TB_EXACT_FORCE")) {
        int t = atoi(f);
        if (t >= kWsBase && t <= kWsBase + 1 && ws_mode(mode, fma) && tile_admissible(t, g.F)) return t;
        if (t >= kSmallBase && t <= kSmallBase + 1 && tile_admissible(t, g.F)) return t;
        if (is_slide(t) && fma && conv_slide_supported(g, t - kSlideBase) && tile_admissible(t, g.F)) return t;
        if (t >= 0 && t < num_configs(mode, fma) && tile_admissible(t, g.F)) return t;
        if (t >= 0 && tile_admissible(t % kNumTiles, g.F)) return t % kNumTiles;
    }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_tuned.find(key_of(ctx, g, mode, fma));
        if (it != g_tuned.end()) return it->second;
    }
    int best = -1;
    double best_cost = 1e300;
    for (int t = 0; t < kNumTiles; ++t) {
        if (!tile_admissible(t, g.F)) continue;
        const double c = model_cost(ctx, t, g, mode);
        if (c < best_cost * 0.999) { best_cost = c; best = t; }
    }
    return best < 0 ? 0 : best;
}

ConvParams params_of(const ConvGeom& g, const float* x, const float* wp, const float* bias, const float* bn_scale,
                     const float* bn_mean, const float* bn_var, const float* res, float* y, int act,
                     int yolo_classes) {
    ConvParams p{};
    p.x = x; p.w = wp; p.bias = bias; p.bn_scale = bn_scale; p.bn_mean = bn_mean; p.bn_var = bn_var;
    p.res = res; p.y = y;
    p.C = (int)g.C; p.H = (int)g.H; p.W = (int)g.W; p.F = (int)g.F;
    p.KH = (int)g.KH; p.KW = (int)g.KW; p.SY = (int)g.SY; p.SX = (int)g.SX;
    p.PY = (int)g.PY; p.PX = (int)g.PX; p.DY = (int)g.DY; p.DX = (int)g.DX;
    p.OH = (int)g.OH; p.OW = (int)g.OW; p.OHW = (int)(g.OH * g.OW);
    p.Cpad = (int)g.Cpad; p.Kpad = (int)g.Kpad; p.Mpad = (int)g.Mpad;
    p.x_bs = g.x_bs; p.y_bs = g.y_bs; p.r_bs = g.r_bs;
    p.Ntot = g.B * g.OH * g.OW;
    p.splits = 1;
    p.act = act;
    p.yolo_classes = yolo_classes;
    p.vec_out = (p.OHW % 4 == 0 && g.y_bs % 4 == 0 && aligned16(y) &&
                 (!res || (g.r_bs % 4 == 0 && aligned16(res)))) ? 1 : 0;
    p.wrsc = g.rsc ? 1 : 0;
    return p;
}

int launch_tile(tb_ctx* ctx, int t, const ConvGeom& g, const ConvParams& p, int mode, bool fma) {
    if (is_slide(t)) return conv_slide_launch(ctx, t - kSlideBase, g, p, false);
    const ExactTile T{tile_bm(t), tile_bn(t), tile_nt(t)};
    dim3 grid((unsigned)ceil_div(p.Ntot, T.BN), (unsigned)ceil_div(g.F, T.BM), 1);
    if (grid.y > 65535) return fail(TB_ERR_INVALID, "conv: grid too large");
    return run_tile(ctx, t, p, grid, mode, fma);
}

}  // namespace

bool conv_exact_supported(const ConvGeom& g) {
    if (g.KH * g.KW > EX_GEN_TAPS) return false;
    // per-stage weight row offsets are 32-bit
    const int64_t rows = g.rsc ? g.KH * g.KW * g.Cpad : g.Kpad;
    return rows * g.Mpad < ((int64_t)1 << 31) && g.B * g.OH * g.OW < ((int64_t)1 << 31);
}

int conv_exact_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                      const float* bn_scale, const float* bn_mean, const float* bn_var, const float* res, float* y,
                      int act, int yolo_classes, bool fma, int64_t* launches) {
    if (g.B == 0) return TB_OK;
    if (!conv_exact_supported(g))
        return fail(TB_ERR_UNSUPPORTED, "conv: a %lldx%lld window is beyond the order-exact FP32 kernel "
                    "(at most %d taps); use TB_MATH_FP32_TILED", (long long)g.KH, (long long)g.KW, EX_GEN_TAPS);
    if (fma && conv_direct_supported(g, res, yolo_classes))  // short reductions: the direct kernel, same order
        return conv_direct_launch(ctx, g, x, wp, bias, bn_scale, bn_mean, bn_var, y, act, launches);
    const int mode = exact_mode_of(g, x);
    const int t = choose_tile(ctx, g, mode, fma);
    ConvParams p = params_of(g, x, wp, bias, bn_scale, bn_mean, bn_var, res, y, act, yolo_classes);
    int r = launch_tile(ctx, t, g, p, mode, fma);
    if (r == TB_OK && launches) ++*launches;
    return r;
}

// Time every admissible configuration of this geometry on the given buffers (3 launches each,
// after one warm-up), time the three fastest again (10 launches each, twice in turn) and remember
// the fastest of those; a geometry already measured on this device is not measured again.
// Blocks; allocates nothing.
int conv_exact_autotune(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, float* y, bool fma) {
    if (g.B == 0 || !conv_exact_supported(g)) return TB_OK;
    if (fma && conv_direct_supported(g, nullptr, 0)) return TB_OK;
    const int mode = exact_mode_of(g, x);
    {  // one measurement per geometry: the layers that share it share the choice
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_tuned.count(key_of(ctx, g, mode, fma))) return TB_OK;
    }
    ConvParams p = params_of(g, x, wp, nullptr, nullptr, nullptr, nullptr, nullptr, y, TB_ACT_LINEAR, 0);
    cudaEvent_t e0, e1;
    TB_CHECK_CUDA(cudaEventCreate(&e0));
    TB_CHECK_CUDA(cudaEventCreate(&e1));
    int rc = TB_OK;
    std::vector<int> cfgs;
    for (int t = 0; t < num_configs(mode, fma); ++t) cfgs.push_back(t);
    if (ws_mode(mode, fma)) cfgs.push_back(kWsBase), cfgs.push_back(kWsBase + 1);
    cfgs.push_back(kSmallBase);
    cfgs.push_back(kSmallBase + 1);
    if (fma)
        for (int t = 0; t < SLIDE_TILES; ++t)
            if (conv_slide_supported(g, t)) cfgs.push_back(kSlideBase + t);
    // device time of `reps` back-to-back launches of configuration t, in ms per launch
    auto time_cfg = [&](int t, int reps, float* out) -> int {
        int r = launch_tile(ctx, t, g, p, mode, fma);  // warm-up
        if (r != TB_OK) return r;
        stream_delay_us(ctx, 200);  // the timed launches queue behind it: device time only
        cudaEventRecord(e0, ctx->stream);
        for (int rep = 0; rep < reps && r == TB_OK; ++rep) r = launch_tile(ctx, t, g, p, mode, fma);
        cudaEventRecord(e1, ctx->stream);
        cudaError_t e = cudaEventSynchronize(e1);
        if (r != TB_OK) return r;
        if (e != cudaSuccess) return cuda_fail(e, "exact conv autotune");
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        *out = ms / reps;
        return TB_OK;
    };
    // pass 1: every admissible configuration, 3 launches each
    std::vector<std::pair<float, int>> timed;
    for (int t : cfgs) {
        if (!tile_admissible(t, g.F)) continue;
        float ms = 0.f;
        rc = time_cfg(t, 3, &ms);
        if (rc != TB_OK) break;
        if (getenv("TB_AUTOTUNE_VERBOSE"))
            fprintf(stderr, "exact autotune C%lld H%lld F%lld k%lld s%lld B%lld: tile %dx%d var %d mode %d: %.4f ms\n",
                    (long long)g.C, (long long)g.H, (long long)g.F, (long long)g.KH, (long long)g.SY, (long long)g.B,
                    tile_bm(t), tile_bn(t), t >= kWsBase ? t : t / kNumTiles, mode, ms);
        timed.emplace_back(ms, t);
    }
    // pass 2: the three fastest again, 10 launches each, twice in turn; keep each one's best
    int best = -1;
    if (rc == TB_OK && !timed.empty()) {
        std::sort(timed.begin(), timed.end());
        const size_t top = std::min<size_t>(3, timed.size());
        std::vector<float> best_ms(top, 1e30f);
        for (int round = 0; round < 2 && rc == TB_OK; ++round)
            for (size_t i = 0; i < top && rc == TB_OK; ++i) {
                float ms = 0.f;
                rc = time_cfg(timed[i].second, 10, &ms);
                best_ms[i] = std::min(best_ms[i], ms);
            }
        size_t bi = 0;
        for (size_t i = 1; i < top; ++i)
            if (best_ms[i] < best_ms[bi]) bi = i;
        best = timed[bi].second;
        if (getenv("TB_AUTOTUNE_VERBOSE"))
            fprintf(stderr, "exact autotune C%lld H%lld F%lld k%lld s%lld B%lld: chose configuration %d (%.4f ms)\n",
                    (long long)g.C, (long long)g.H, (long long)g.F, (long long)g.KH, (long long)g.SY, (long long)g.B,
                    best, best_ms[bi]);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc != TB_OK) return rc;
    if (best >= 0) {
        std::lock_guard<std::mutex> lk(g_mu);
        g_tuned[key_of(ctx, g, mode, fma)] = best;
    }
    return TB_OK;
}

}  // namespace tbi
