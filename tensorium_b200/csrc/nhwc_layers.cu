// nhwc_layers.cu -- the data-movement layers of a network that runs its tensor-core convs on NHWC
// activations (net.cu's NHWC plan): input conversion, upsample, route copy and shortcut on
// [batch][h][w][pixel stride] buffers, where a layer's channels may be a slice of a wider
// (concatenation) buffer. Same arithmetic as the NCHW kernels: upsample multiplies by the scale
// (source/nupsamplelayer.pas:83-113), shortcut adds then activates (source/naddlayer.pas:667-725),
// route copies (source/nconcatlayer.pas:93-119).
#include "conv.cuh"

namespace tbi {

namespace {

// x: NCHW [b][c][h][w] (batch stride x_bs) -> y: NHWC, pixel stride ps >= c, channels c..ps-1
// zero; values rounded to TF32 (nearest), as every activation the tensor cores read
__global__ void k_nchw_to_nhwc(int64_t npix, int c, int hw, int ps, const float* __restrict__ x, int64_t x_bs,
                               float* __restrict__ y, int pair) {
    TB_GRID_DEP_ENTRY();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npix * ps;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pix = i / ps;
        const int ch = (int)(i - pix * ps);
        const int64_t b = pix / hw;
        const int q = (int)(pix - b * hw);
        const float v = ch < c ? __ldg(x + b * x_bs + (int64_t)ch * hw + q) : 0.0f;
        y[i] = tb_fmt_store(v, pair);
    }
}

// upsample: y[b][oy][ox][ch] = scale * x[b][oy/s][ox/s][ch], 4 channels per thread
__global__ void k_upsample_nhwc4(int64_t total4, int c4, int w, int h, int s, float scale,
                                 const float4* __restrict__ x, int xps4, float4* __restrict__ y, int yps4) {
    TB_GRID_DEP_ENTRY();
    const int ow = w * s, oh = h * s;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t opix = i / c4;
        const int q = (int)(i - opix * c4);
        const int ox = (int)(opix % ow);
        const int64_t t = opix / ow;
        const int oy = (int)(t % oh);
        const int64_t b = t / oh;
        const float4 v = __ldg(x + ((b * h + oy / s) * w + ox / s) * xps4 + q);
        y[opix * yps4 + q] = make_float4(scale * v.x, scale * v.y, scale * v.z, scale * v.w);
    }
}

// copy c channels per pixel between two pixel strides (route slices)
__global__ void k_copy_nhwc4(int64_t total4, int c4, const float4* __restrict__ x, int xps4, float4* __restrict__ y,
                             int yps4) {
    TB_GRID_DEP_ENTRY();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pix = i / c4;
        const int q = (int)(i - pix * c4);
        y[pix * yps4 + q] = __ldg(x + pix * xps4 + q);
    }
}

// shortcut: out = act(a + b) (bf16 pairs decoded, added in fp32, encoded again)
__global__ void k_shortcut_nhwc(int64_t total, int c, const float* __restrict__ a, int aps,
                                const float* __restrict__ b, int bps, float* __restrict__ y, int yps, int act,
                                int pair) {
    TB_GRID_DEP_ENTRY();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pix = i / c;
        const int ch = (int)(i - pix * c);
        float v = __fadd_rn(tb_fmt_load(__ldg(a + pix * aps + ch), pair), tb_fmt_load(__ldg(b + pix * bps + ch), pair));
        if (act != TB_ACT_LINEAR) v = tb_activate_dev(v, act);
        y[pix * yps + ch] = pair ? tb_pair_encode(v) : v;
    }
}

// The first layer of an image network (C * KH * KW <= 32) as a 1x1 conv over 32 "channels": output
// pixel (b, oy, ox) gets its whole receptive field, k = (r * KW + s) * C + c, zero past K and in
// the padding, rounded to TF32. One k tile instead of KH * KW mostly empty ones.
__global__ void k_im2col_first(int64_t npix, int C, int H, int W, int KW, int K, int OW, int OHW, int SY, int SX,
                               int PY, int PX, int DY, int DX, const float* __restrict__ x, int64_t x_bs,
                               float* __restrict__ y, int pair) {
    TB_GRID_DEP_ENTRY();
    // one thread per output pixel: the lanes of a warp read neighbouring pixels of the same tap
    // (coalesced) and each writes its 128-byte row of 32 values
    for (int64_t pix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; pix < npix; pix += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = pix / OHW;
        const int q = (int)(pix - b * OHW);
        const int oy = q / OW, ox = q - oy * OW;
        const float* xb = x + b * x_bs;
        float v[32];
        int c = 0, r = 0, s = 0;  // k = (r * KW + s) * C + c, in order
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            float t = 0.0f;
            if (k < K) {
                const int iy = oy * SY - PY + r * DY, ix = ox * SX - PX + s * DX;
                if (iy >= 0 && iy < H && ix >= 0 && ix < W) t = __ldg(xb + ((int64_t)c * H + iy) * W + ix);
                if (++c == C) {
                    c = 0;
                    if (++s == KW) s = 0, ++r;
                }
            }
            v[k] = tb_fmt_store(t, pair);
        }
        float4* yo = reinterpret_cast<float4*>(y + pix * 32);
#pragma unroll
        for (int k = 0; k < 32; k += 4) __stcs(yo + k / 4, make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]));
    }
}

// its weights: wp[f][k] = tf32(w[f][c][r][s]) for k = (r * KW + s) * C + c < K, zero up to 32; in
// pair mode two such operands, [F][32] of (hi, hi) and then [F][32] of (lo, lo) bf16 pairs
__global__ void k_pack_first(const float* __restrict__ w, float* __restrict__ wp, int F, int C, int KH, int KW,
                             int pair) {
    const int K = C * KH * KW;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < F * 32; i += gridDim.x * blockDim.x) {
        const int f = i >> 5, k = i & 31;
        float v = 0.0f;
        if (k < K) {
            const int rs = k / C, c = k - rs * C;
            const int r = rs / KW, s = rs - r * KW;
            v = w[(((int64_t)f * C + c) * KH + r) * KW + s];
        }
        if (!pair) {
            wp[i] = tb_tf32_rna(v);
        } else {
            const uint32_t s = __float_as_uint(tb_pair_encode(v)), hi = s & 0xffffu, lo = s >> 16;
            wp[i] = __uint_as_float(hi | (hi << 16));
            wp[(int64_t)F * 32 + i] = __uint_as_float(lo | (lo << 16));
        }
    }
}

// its weights: wd[k][f] for k = (c * KH + r) * KW + s, FG = F rounded up to 32 filters (zero
// past F); TF32 mode rounds them to TF32, pair mode keeps them exact
__global__ void k_pack_first_direct(const float* __restrict__ w, float* __restrict__ wd, int F, int K, int pair) {
    const int FG = (F + 31) & ~31;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < K * FG; i += gridDim.x * blockDim.x) {
        const int k = i / FG, f = i - k * FG;
        const float v = f < F ? w[(int64_t)f * K + k] : 0.0f;
        wd[i] = pair ? v : tb_tf32_rna(v);
    }
}

}  // namespace

bool nhwc_first_direct_supported(int64_t C, int64_t KH, int64_t KW, int64_t SY, int64_t SX, int64_t DY, int64_t DX,
                                 int64_t F, int64_t yps) {
    return F % 4 == 0 && yps % 4 == 0 && first_direct_supported(C, KH, KW, SY, SX, DY, DX, F, true);
}

int64_t nhwc_first_direct_wcount(int64_t F, int64_t C, int64_t KH, int64_t KW) { return C * KH * KW * round_up(F, 32); }

int nhwc_pack_first_direct(tb_ctx* ctx, int64_t F, int64_t C, int64_t KH, int64_t KW, const float* w, float* wd,
                           int pair) {
    const int64_t n = nhwc_first_direct_wcount(F, C, KH, KW);
    k_pack_first_direct<<<grid_for(n, 256, ctx->sm_count), 256, 0, ctx->stream>>>(w, wd, (int)F, (int)(C * KH * KW),
                                                                                   pair);
    return check_launch("k_pack_first_direct");
}

int nhwc_first_direct(tb_ctx* ctx, int64_t B, int64_t C, int64_t H, int64_t W, int64_t KH, int64_t KW, int64_t SY,
                      int64_t SX, int64_t PY, int64_t PX, int64_t DY, int64_t DX, int64_t OH, int64_t OW,
                      const float* x, int64_t x_bs, const float* wd, const float* bias, int64_t F, int act, float* y,
                      int64_t yps, int pair) {
    if (!nhwc_first_direct_supported(C, KH, KW, SY, SX, DY, DX, F, yps) || !aligned16(y))
        return fail(TB_ERR_UNSUPPORTED, "first-layer direct conv: unsupported geometry");
    FirstGeom fg{B, C, H, W, KH, KW, SY, SX, PY, PX, DY, DX, OH, OW};
    return first_direct_launch(ctx, fg, x, x_bs, wd, round_up(F, 32), bias, F, act, y, OH * OW * yps, yps,
                               pair ? 2 : 1);
}

int nhwc_im2col_first(tb_ctx* ctx, int64_t B, int64_t C, int64_t H, int64_t W, int64_t KH, int64_t KW, int64_t SY,
                      int64_t SX, int64_t PY, int64_t PX, int64_t DY, int64_t DX, int64_t OH, int64_t OW,
                      const float* x, int64_t x_bs, float* y, int pair) {
    const int64_t npix = B * OH * OW;
    if (npix == 0) return TB_OK;
    {
        const int _lr = launch(ctx, "k_im2col_first", k_im2col_first, dim3(grid_for(npix, 128, ctx->sm_count)), dim3(128), 0, npix, (int)C, (int)H, (int)W, (int)KW, (int)(C * KH * KW), (int)OW, (int)(OH * OW), (int)SY, (int)SX, (int)PY, (int)PX, (int)DY, (int)DX, x, x_bs, y, pair);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_im2col_first");
}

int nhwc_pack_first(tb_ctx* ctx, int64_t F, int64_t C, int64_t KH, int64_t KW, const float* w, float* wp, int pair) {
    k_pack_first<<<grid_for(F * 32, 256, ctx->sm_count), 256, 0, ctx->stream>>>(w, wp, (int)F, (int)C, (int)KH, (int)KW,
                                                                                pair);
    return check_launch("k_pack_first");
}

int nhwc_from_nchw(tb_ctx* ctx, int64_t batch, int64_t c, int64_t h, int64_t w, const float* x, int64_t x_bs,
                   float* y, int64_t ps, int pair) {
    const int64_t npix = batch * h * w;
    if (npix == 0) return TB_OK;
    {
        const int _lr = launch(ctx, "k_nchw_to_nhwc", k_nchw_to_nhwc, dim3(grid_for(npix * ps, 256, ctx->sm_count)), dim3(256), 0, npix, (int)c, (int)(h * w), (int)ps, x, x_bs, y, pair);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_nchw_to_nhwc");
}

int nhwc_upsample(tb_ctx* ctx, int64_t batch, int64_t c, int64_t h, int64_t w, int64_t s, float scale,
                  const float* x, int64_t xps, float* y, int64_t yps, int pair) {
    if (pair && scale != 1.0f) return fail(TB_ERR_UNSUPPORTED, "NHWC upsample: bf16-pair activations need scale 1");
    if (c % 4 || xps % 4 || yps % 4 || !aligned16(x) || !aligned16(y))
        return fail(TB_ERR_STATE, "NHWC upsample: channels, strides and pointers must be 16-byte multiples");
    const int64_t total4 = batch * h * s * w * s * (c / 4);
    if (total4 == 0) return TB_OK;
    {
        const int _lr = launch(ctx, "k_upsample_nhwc4", k_upsample_nhwc4, dim3(grid_for(total4, 256, ctx->sm_count)), dim3(256), 0, total4, (int)(c / 4), (int)w, (int)h, (int)s, scale, reinterpret_cast<const float4*>(x), (int)(xps / 4), reinterpret_cast<float4*>(y), (int)(yps / 4));
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_upsample_nhwc4");
}

int nhwc_copy(tb_ctx* ctx, int64_t npix, int64_t c, const float* x, int64_t xps, float* y, int64_t yps) {
    if (c % 4 || xps % 4 || yps % 4 || !aligned16(x) || !aligned16(y))
        return fail(TB_ERR_STATE, "NHWC copy: channels, strides and pointers must be 16-byte multiples");
    const int64_t total4 = npix * (c / 4);
    if (total4 == 0) return TB_OK;
    {
        const int _lr = launch(ctx, "k_copy_nhwc4", k_copy_nhwc4, dim3(grid_for(total4, 256, ctx->sm_count)), dim3(256), 0, total4, (int)(c / 4), reinterpret_cast<const float4*>(x), (int)(xps / 4), reinterpret_cast<float4*>(y), (int)(yps / 4));
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_copy_nhwc4");
}

int nhwc_shortcut(tb_ctx* ctx, int64_t npix, int64_t c, const float* a, int64_t aps, const float* b, int64_t bps,
                  float* y, int64_t yps, int act, int pair) {
    const int64_t total = npix * c;
    if (total == 0) return TB_OK;
    {
        const int _lr = launch(ctx, "k_shortcut_nhwc", k_shortcut_nhwc, dim3(grid_for(total, 256, ctx->sm_count)), dim3(256), 0, total, (int)c, a, (int)aps, b, (int)bps, y, (int)yps, act, pair);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_shortcut_nhwc");
}

}  // namespace tbi
