// layers.cu -- memory-bound layers of the conv inference path: maxpool, upsample, route,
// shortcut, yolo activation, softmax, global average pool, and the connected layer (run as a
// 1x1 convolution over 1x1 images through the conv kernel).
#include "conv.cuh"

#include <cfloat>

using namespace tbi;

// ---- maxpool: TMaxPoolLayer.forwardMaxPool / maxpoolMP (source/nMaxPoolLayer.pas:265-463) ----
// One thread per output; window scanned n-major, m-minor with strict '>' so the first maximum
// wins, out-of-image taps read -FLT_MAX (= -MaxSingle) and never win against it.
__global__ void k_maxpool(int64_t total, int c, int h, int w, int out_h, int out_w, int size,
                          int stride_x, int stride_y, int off, const float* __restrict__ x,
                          float* __restrict__ y, int64_t* __restrict__ idx) {
    TB_GRID_DEP_ENTRY();
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total;
         o += (int64_t)gridDim.x * blockDim.x) {
        int j = (int)(o % out_w);
        int64_t t = o / out_w;
        int i = (int)(t % out_h);
        int64_t bk = t / out_h;  // b*c + k
        float mx = -FLT_MAX;
        int64_t mi = -1;
        const int64_t plane = bk * (int64_t)h * w;
        for (int n = 0; n < size; ++n) {
            int cur_h = off + i * stride_y + n;
            for (int m = 0; m < size; ++m) {
                int cur_w = off + j * stride_x + m;
                int64_t index = plane + (int64_t)cur_h * w + cur_w;
                float val = (cur_h >= 0 && cur_h < h && cur_w >= 0 && cur_w < w) ? x[index] : -FLT_MAX;
                if (val > mx) {
                    mi = index;
                    mx = val;
                }
            }
        }
        y[o] = mx;
        if (idx) idx[o] = mi;
    }
}

// 2x2 stride-2 pad-0 fast path (configs 1-2): each thread makes 2 adjacent outputs from two
// float4 input rows. Same scan order and comparisons as the generic kernel.
__global__ void k_maxpool2x2(int64_t total2, int h, int w, int out_h, int out_w,
                             const float* __restrict__ x, float* __restrict__ y,
                             int64_t* __restrict__ idx) {
    TB_GRID_DEP_ENTRY();
    const int half = out_w / 2;
    for (int64_t o2 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o2 < total2;
         o2 += (int64_t)gridDim.x * blockDim.x) {
        int jj = (int)(o2 % half);
        int64_t t = o2 / half;
        int i = (int)(t % out_h);
        int64_t bk = t / out_h;
        const int64_t base = bk * (int64_t)h * w + (int64_t)(2 * i) * w + 4 * jj;
        float4 r0 = *reinterpret_cast<const float4*>(x + base);
        float4 r1 = *reinterpret_cast<const float4*>(x + base + w);
        float v0[4] = {r0.x, r0.y, r1.x, r1.y};
        float v1[4] = {r0.z, r0.w, r1.z, r1.w};
        int64_t off[4] = {0, 1, w, (int64_t)w + 1};
        float m0 = -FLT_MAX, m1 = -FLT_MAX;
        int64_t i0 = -1, i1 = -1;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (v0[q] > m0) { m0 = v0[q]; i0 = base + off[q]; }
            if (v1[q] > m1) { m1 = v1[q]; i1 = base + 2 + off[q]; }
        }
        int64_t ob = bk * (int64_t)out_h * out_w + (int64_t)i * out_w + 2 * jj;
        *reinterpret_cast<float2*>(y + ob) = make_float2(m0, m1);
        if (idx) {
            idx[ob] = i0;
            idx[ob + 1] = i1;
        }
    }
}

// ---- upsample: upsample() forward (source/nupsamplelayer.pas:83-113) ----
__global__ void k_upsample(int64_t total, int c, int h, int w, int s, float scale,
                           const float* __restrict__ x, float* __restrict__ y, int64_t y_bs) {
    TB_GRID_DEP_ENTRY();
    const int ow = w * s, oh = h * s;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total;
         o += (int64_t)gridDim.x * blockDim.x) {
        int xx = (int)(o % ow);
        int64_t t = o / ow;
        int yy = (int)(t % oh);
        int64_t cc = t / oh;  // b*c + ch
        int64_t b = cc / c, ch = cc - b * c;
        float v = x[(cc * h + yy / s) * w + xx / s];
        y[b * y_bs + (ch * oh + yy) * ow + xx] = scale * v;
    }
}

// stride-2 fast path: one thread reads 2 inputs and writes a float4 into each of 2 rows.
__global__ void k_upsample2(int64_t total2, int c, int h, int w, float scale,
                            const float* __restrict__ x, float* __restrict__ y, int64_t y_bs) {
    TB_GRID_DEP_ENTRY();
    const int ow = 2 * w, oh = 2 * h, half = w / 2;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t o0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o0 < total2; o0 += 4 * step) {
        float2 v[4];  // four input pairs per thread per round, loads first
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t o = o0 + r * step;
            if (o < total2) {
                const int xq = (int)(o % half);
                const int64_t t = o / half;
                v[r] = __ldcs(reinterpret_cast<const float2*>(x + t * w + 2 * xq));  // read once: evict-first
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t o = o0 + r * step;
            if (o >= total2) break;
            const int xq = (int)(o % half);
            const int64_t t = o / half;
            const int iy = (int)(t % h);
            const int64_t cc = t / h;
            const int64_t b = cc / c, ch = cc - b * c;
            const float a = scale * v[r].x, bb = scale * v[r].y;
            const float4 o4 = make_float4(a, a, bb, bb);
            float* dst = y + b * y_bs + (ch * oh + 2 * iy) * (int64_t)ow + 4 * xq;
            *reinterpret_cast<float4*>(dst) = o4;  // the next layer's input: default caching
            *reinterpret_cast<float4*>(dst + ow) = o4;
        }
    }
}

// ---- route / concat: copy rows of `n` elements from `batch` images ----
__global__ void k_copy_rows(int64_t batch, int64_t n, const float* __restrict__ src, int64_t src_bs,
                            float* __restrict__ dst, int64_t dst_bs) {
    TB_GRID_DEP_ENTRY();
    const int64_t total = batch * n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = i / n, e = i - b * n;
        dst[b * dst_bs + e] = src[b * src_bs + e];
    }
}

__global__ void k_copy_rows4(int64_t batch, int64_t n4, const float4* __restrict__ src, int64_t src_bs4,
                             float4* __restrict__ dst, int64_t dst_bs4) {
    TB_GRID_DEP_ENTRY();
    const int64_t total = batch * n4;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += 4 * step) {
        float4 v[4];  // four vectors per thread per round, loads first
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t i = i0 + r * step;
            if (i < total) {
                const int64_t b = i / n4, e = i - b * n4;
                v[r] = src[b * src_bs4 + e];  // a route source may be read again later
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t i = i0 + r * step;
            if (i >= total) break;
            const int64_t b = i / n4, e = i - b * n4;
            dst[b * dst_bs4 + e] = v[r];
        }
    }
}

// ---- shortcut: y = act(a + b) (source/naddlayer.pas:696-699) ----
__global__ void k_shortcut4(int64_t n4, const float4* __restrict__ a, const float4* __restrict__ b,
                            float4* __restrict__ y, int act) {
    TB_GRID_DEP_ENTRY();
    // four vectors per thread per round, all loads issued before any use (more bytes in flight)
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n4; i0 += 4 * step) {
        float4 u[4], v[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t i = i0 + r * step;
            if (i < n4) u[r] = a[i], v[r] = b[i];  // b (the residual source) may still be read later
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t i = i0 + r * step;
            if (i >= n4) break;
            float4 o;
            o.x = tb_activate_dev(u[r].x + v[r].x, act);
            o.y = tb_activate_dev(u[r].y + v[r].y, act);
            o.z = tb_activate_dev(u[r].z + v[r].z, act);
            o.w = tb_activate_dev(u[r].w + v[r].w, act);
            y[i] = o;
        }
    }
}

__global__ void k_shortcut(int64_t n, const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ y, int act) {
    TB_GRID_DEP_ENTRY();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        y[i] = tb_activate_dev(a[i] + b[i], act);
}

// ---- yolo: TYoloLayer.forward (source/nyololayer.pas:786-825) ----
// One (image, anchor, entry) plane of hw values per blockIdx.y, so the entry (and whether the
// logistic applies) is uniform in a block; float4 accesses when every plane is 16-byte aligned.
__global__ void k_yolo(int entries, int hw, int vec4, const float* __restrict__ x, float* __restrict__ y,
                       float scale_xy, float bias_xy) {
    TB_GRID_DEP_ENTRY();
    const int e = blockIdx.y % entries;
    const bool logi = e != 2 && e != 3, sxy = e < 2 && scale_xy != 1.0f;
    const int64_t base = (int64_t)blockIdx.y * hw;
    auto f = [&](float v) {
        // logistic_activate in double, as tb_logistic, inlined here: a call per element cost
        // more than the memory traffic it hides behind
        if (logi) v = (float)(1.0 / (1.0 + exp(-(double)v)));
        if (sxy) v = __fadd_rn(__fmul_rn(v, scale_xy), bias_xy);
        return v;
    };
    if (vec4) {
        const float4* x4 = reinterpret_cast<const float4*>(x + base);
        float4* y4 = reinterpret_cast<float4*>(y + base);
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hw / 4; i += gridDim.x * blockDim.x) {
            float4 v = __ldg(x4 + i);
            v.x = f(v.x);
            v.y = f(v.y);
            v.z = f(v.z);
            v.w = f(v.w);
            y4[i] = v;
        }
    } else {
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hw; i += gridDim.x * blockDim.x)
            y[base + i] = f(__ldg(x + base + i));
    }
}

// ---- softmax: softmaxBatch / softmax (source/nsoftmaxlayer.pas:83-137), sequential per group ----
__global__ void k_softmax(int64_t groups_total, int n, int groups, int64_t inputs, float temp,
                          const float* __restrict__ x, float* __restrict__ y) {
    TB_GRID_DEP_ENTRY();
    for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups_total;
         gi += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = gi / groups, g = gi - b * groups;
        const float* in = x + b * inputs + g * n;
        float* out = y + b * inputs + g * n;
        float largest = in[0];
        for (int i = 1; i < n; ++i)
            if (in[i] > largest) largest = in[i];
        float sum = 0.0f;
        for (int i = 0; i < n; ++i) {
            float e = (float)exp((double)__fdiv_rn(__fsub_rn(in[i], largest), temp));
            sum = __fadd_rn(sum, e);
            out[i] = e;
        }
        for (int i = 0; i < n; ++i) out[i] = __fdiv_rn(out[i], sum);
    }
}

// ---- global average pool (source/navgpoollayer.pas:60-84): Sum / (h*w), the sum in the order
// of vssum_avx2 (source/ntensors.pas:3592-3620), which vsSumI uses on AVX2 CPUs: eight lane sums
// over the whole blocks of 8, (l0+l4) .. (l3+l7), two horizontal adds, then the tail in order ----
__global__ void k_avgpool(int64_t total, int im, const float* __restrict__ x, float* __restrict__ y) {
    TB_GRID_DEP_ENTRY();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float* p = x + i * im;
        float lane[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const int nb = im / 8 * 8;
        for (int j = 0; j < nb; j += 8)
#pragma unroll
            for (int l = 0; l < 8; ++l) lane[l] = __fadd_rn(lane[l], p[j + l]);
        float t[4];
#pragma unroll
        for (int l = 0; l < 4; ++l) t[l] = __fadd_rn(lane[l], lane[l + 4]);
        float s = __fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3]));
        for (int j = nb; j < im; ++j) s = __fadd_rn(s, p[j]);
        y[i] = __fdiv_rn(s, (float)im);
    }
}

namespace tbi {
// Copy `n` elements per image from src (batch stride src_bs) to dst (batch stride dst_bs).
int copy_rows(tb_ctx* ctx, int64_t batch, int64_t n, const float* src, int64_t src_bs, float* dst,
              int64_t dst_bs) {
    if (batch == 0 || n == 0) return TB_OK;
    if (n % 4 == 0 && src_bs % 4 == 0 && dst_bs % 4 == 0 && aligned16(src) && aligned16(dst)) {
        {
            const int _lr = launch(ctx, "k_copy_rows4", k_copy_rows4, dim3(grid_for(batch * n / 4, 256, ctx->sm_count)), dim3(256), 0, batch, n / 4, reinterpret_cast<const float4*>(src), src_bs / 4, reinterpret_cast<float4*>(dst), dst_bs / 4);
            if (_lr != TB_OK) return _lr;
        }
    } else {
        {
            const int _lr = launch(ctx, "k_copy_rows", k_copy_rows, dim3(grid_for(batch * n, 256, ctx->sm_count)), dim3(256), 0, batch, n, src, src_bs, dst, dst_bs);
            if (_lr != TB_OK) return _lr;
        }
    }
    return check_launch("k_copy_rows");
}
}  // namespace tbi

extern "C" {

int tb_maxpool_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                   int64_t ksize, int64_t stride_x, int64_t stride_y, int64_t padding,
                   const float* x, float* y, int64_t* indexes) {
    TB_ENTER(ctx);
    if (batch < 0 || channels <= 0 || h <= 0 || w <= 0 || ksize <= 0 || stride_x <= 0 ||
        stride_y <= 0 || padding < 0)
        return fail(TB_ERR_INVALID, "maxpool: bad shape");
    const int64_t out_h = (h + padding - ksize) / stride_y + 1;
    const int64_t out_w = (w + padding - ksize) / stride_x + 1;
    if (out_h <= 0 || out_w <= 0) return fail(TB_ERR_INVALID, "maxpool: empty output");
    if (batch == 0) return TB_OK;
    if (!x || !y) return fail(TB_ERR_INVALID, "maxpool: null pointer");
    const int64_t total = batch * channels * out_h * out_w;
    const int off = -(int)(padding / 2);
    if (ksize == 2 && stride_x == 2 && stride_y == 2 && padding == 0 && w % 4 == 0 &&
        h == 2 * out_h && w == 2 * out_w && aligned16(x) && aligned16(y)) {
        const int64_t total2 = total / 2;
        {
            const int _lr = launch(ctx, "k_maxpool2x2", k_maxpool2x2, dim3(grid_for(total2, 256, ctx->sm_count)), dim3(256), 0, total2, (int)h, (int)w, (int)out_h, (int)out_w, x, y, indexes);
            if (_lr != TB_OK) return _lr;
        }
        return check_launch("k_maxpool2x2");
    }
    {
        const int _lr = launch(ctx, "k_maxpool", k_maxpool, dim3(grid_for(total, 256, ctx->sm_count)), dim3(256), 0, total, (int)channels, (int)h, (int)w, (int)out_h, (int)out_w, (int)ksize, (int)stride_x, (int)stride_y, off, x, y, indexes);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_maxpool");
}

int tb_upsample_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                    int64_t stride, float scale, const float* x, float* y, int64_t y_bs) {
    TB_ENTER(ctx);
    if (batch < 0 || channels <= 0 || h <= 0 || w <= 0 || stride <= 0)
        return fail(TB_ERR_INVALID, "upsample: bad shape (reverse / negative stride is not on the inference path)");
    const int64_t per = channels * h * w * stride * stride;
    if (y_bs == 0) y_bs = per;
    if (y_bs < per) return fail(TB_ERR_INVALID, "upsample: output batch stride smaller than one image");
    if (batch == 0) return TB_OK;
    if (!x || !y) return fail(TB_ERR_INVALID, "upsample: null pointer");
    if (stride == 2 && w % 2 == 0 && aligned16(y) && y_bs % 4 == 0 && ((uintptr_t)x & 7u) == 0) {
        const int64_t total2 = batch * channels * h * (w / 2);
        {
            const int _lr = launch(ctx, "k_upsample2", k_upsample2, dim3(grid_for(total2, 256, ctx->sm_count)), dim3(256), 0, total2, (int)channels, (int)h, (int)w, scale, x, y, y_bs);
            if (_lr != TB_OK) return _lr;
        }
        return check_launch("k_upsample2");
    }
    const int64_t total = batch * per;
    {
        const int _lr = launch(ctx, "k_upsample", k_upsample, dim3(grid_for(total, 256, ctx->sm_count)), dim3(256), 0, total, (int)channels, (int)h, (int)w, (int)stride, scale, x, y, y_bs);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_upsample");
}

int tb_route_fwd(tb_ctx* ctx, int64_t batch, int64_t n_inputs, const float* const* inputs,
                 const int64_t* sizes, float* y, int64_t per_sample) {
    TB_ENTER(ctx);
    if (batch < 0 || n_inputs <= 0 || !inputs || !sizes) return fail(TB_ERR_INVALID, "route: bad arguments");
    int64_t total = 0;
    for (int64_t i = 0; i < n_inputs; ++i) {
        if (sizes[i] < 0 || (sizes[i] > 0 && !inputs[i])) return fail(TB_ERR_INVALID, "route: bad input %lld", (long long)i);
        total += sizes[i];
    }
    if (batch == 0 || total == 0) return TB_OK;
    if (!y) return fail(TB_ERR_INVALID, "route: null output");
    int64_t off = 0;
    for (int64_t i = 0; i < n_inputs; ++i) {
        int r;
        if (per_sample)  // darknet per-image channel concatenation
            r = copy_rows(ctx, batch, sizes[i], inputs[i], sizes[i], y + off, total);
        else  // TTensor.concat: whole input tensors back to back
            r = copy_rows(ctx, 1, batch * sizes[i], inputs[i], 0, y + batch * off, 0);
        if (r != TB_OK) return r;
        off += sizes[i];
    }
    return TB_OK;
}

int tb_shortcut_fwd(tb_ctx* ctx, int64_t n, const float* a, const float* b, float* y, int64_t act) {
    TB_ENTER(ctx);
    if (n < 0 || (n > 0 && (!a || !b || !y))) return fail(TB_ERR_INVALID, "shortcut: bad arguments");
    if (!act_supported(act)) return fail(TB_ERR_UNSUPPORTED, "shortcut: activation %lld not supported", (long long)act);
    if (n == 0) return TB_OK;
    if (n % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(y)) {
        {
            const int _lr = launch(ctx, "k_shortcut4", k_shortcut4, dim3(grid_for(n / 4, 256, ctx->sm_count)), dim3(256), 0, n / 4, reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(y), (int)act);
            if (_lr != TB_OK) return _lr;
        }
    } else {
        {
            const int _lr = launch(ctx, "k_shortcut", k_shortcut, dim3(grid_for(n, 256, ctx->sm_count)), dim3(256), 0, n, a, b, y, (int)act);
            if (_lr != TB_OK) return _lr;
        }
    }
    return check_launch("k_shortcut");
}

int tb_yolo_fwd(tb_ctx* ctx, int64_t batch, int64_t n, int64_t classes, int64_t h, int64_t w,
                const float* x, float* y, float scale_xy) {
    TB_ENTER(ctx);
    if (batch < 0 || n <= 0 || classes < 0 || h <= 0 || w <= 0) return fail(TB_ERR_INVALID, "yolo: bad shape");
    if (batch == 0) return TB_OK;
    if (!x || !y) return fail(TB_ERR_INVALID, "yolo: null pointer");
    const int64_t planes = batch * n * (classes + 5), hw = h * w;
    if (planes > 2147483647 || hw > 2147483647) return fail(TB_ERR_UNSUPPORTED, "yolo: tensor too large");
    float bias_xy = (float)(0.5 * (1.0 - (double)scale_xy));
    const int vec4 = hw % 4 == 0 && aligned16(x) && aligned16(y);
    const int64_t per = vec4 ? hw / 4 : hw;
    dim3 grid((unsigned)std::min<int64_t>(ceil_div(per, 256), 64), (unsigned)planes);
    if (grid.y > 65535) {  // fall back to fewer, longer planes per block is not needed at darknet sizes
        return fail(TB_ERR_UNSUPPORTED, "yolo: more than 65535 (image, anchor, entry) planes");
    }
    {
        const int _lr = launch(ctx, "k_yolo", k_yolo, dim3(grid), dim3(256), 0, (int)(classes + 5), (int)hw, vec4, x, y, scale_xy, bias_xy);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_yolo");
}

int tb_softmax_fwd(tb_ctx* ctx, int64_t batch, int64_t inputs, int64_t groups, float temperature,
                   const float* x, float* y) {
    TB_ENTER(ctx);
    if (batch < 0 || inputs <= 0 || groups <= 0 || inputs % groups != 0)
        return fail(TB_ERR_INVALID, "softmax: bad shape");
    if (batch == 0) return TB_OK;
    if (!x || !y) return fail(TB_ERR_INVALID, "softmax: null pointer");
    const int64_t gt = batch * groups;
    {
        const int _lr = launch(ctx, "k_softmax", k_softmax, dim3(grid_for(gt, 128, ctx->sm_count)), dim3(128), 0, gt, (int)(inputs / groups), (int)groups, inputs, temperature, x, y);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_softmax");
}

int tb_avgpool_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                   const float* x, float* y) {
    TB_ENTER(ctx);
    if (batch < 0 || channels <= 0 || h <= 0 || w <= 0) return fail(TB_ERR_INVALID, "avgpool: bad shape");
    if (batch == 0) return TB_OK;
    if (!x || !y) return fail(TB_ERR_INVALID, "avgpool: null pointer");
    const int64_t total = batch * channels;
    {
        const int _lr = launch(ctx, "k_avgpool", k_avgpool, dim3(grid_for(total, 128, ctx->sm_count)), dim3(128), 0, total, (int)(h * w), x, y);
        if (_lr != TB_OK) return _lr;
    }
    return check_launch("k_avgpool");
}

}  // extern "C"

namespace tbi {

// TConnectedLayer.forward (source/nconnectedlayer.pas:157-184): y = x * W^T through sgemm_nt, whose
// dot product is sdot_avx2 (source/ntensors.pas:1233-1306) in the USE_AVX2 build the samples use:
// eight lane sums (lane l: k = l, l+8, ..., one FMA each), then (l0+l4) ... and two horizontal
// adds.  One thread per output keeps those eight lanes in registers; the block stages 64-deep k
// chunks of 8 images' inputs and 32 outputs' packed weights (Wp[k][m]) in shared memory.
__global__ void __launch_bounds__(256) k_fc_sdot8(const ConvParams p, int batch, int inputs) {
    TB_GRID_DEP_ENTRY();
    __shared__ float Xs[8][64];
    __shared__ float Ws[64][32];
    const int tid = threadIdx.x, ol = tid & 31, bl = tid >> 5;
    const int o = blockIdx.x * 32 + ol, b = blockIdx.y * 8 + bl;
    float lane[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < inputs; k0 += 64) {
        for (int e = tid; e < 8 * 64; e += 256) {
            const int bb = blockIdx.y * 8 + e / 64, kk = k0 + (e & 63);
            Xs[e / 64][e & 63] = (bb < batch && kk < inputs) ? p.x[(long long)bb * p.x_bs + kk] : 0.f;
        }
        for (int e = tid; e < 64 * 32; e += 256) {
            const int kk = k0 + e / 32, oo = blockIdx.x * 32 + (e & 31);
            Ws[e / 32][e & 31] = (kk < inputs && oo < p.F) ? p.w[(long long)kk * p.Mpad + oo] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 64; ++kk) lane[kk & 7] = fmaf(Xs[bl][kk], Ws[kk][ol], lane[kk & 7]);
        __syncthreads();
    }
    if (o >= p.F || b >= batch) return;
    float t[4];
#pragma unroll
    for (int l = 0; l < 4; ++l) t[l] = __fadd_rn(lane[l], lane[l + 4]);
    const float s = __fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3]));
    p.y[(long long)b * p.y_bs + o] = conv_epilogue(__fadd_rn(0.f, s), o, p);  // C := 0*C + alpha*sdot
}

int fc_sdot_launch(tb_ctx* ctx, const ConvGeom& g, const float* x, const float* wp, const float* bias,
                   const float* bn_scale, const float* bn_mean, const float* bn_var, float* y, int act,
                   int64_t* launches) {
    if (g.B == 0) return TB_OK;
    if (g.KH != 1 || g.KW != 1 || g.H != 1 || g.W != 1 || g.SY != 1 || g.SX != 1 || g.PY != 0 || g.PX != 0)
        return fail(TB_ERR_INVALID, "fc: not a 1x1 layer over 1x1 inputs");
    ConvParams p{};
    p.x = x; p.w = wp; p.bias = bias; p.bn_scale = bn_scale; p.bn_mean = bn_mean; p.bn_var = bn_var;
    p.y = y; p.F = (int)g.F; p.Mpad = (int)g.Mpad; p.x_bs = g.x_bs; p.y_bs = g.y_bs; p.act = act;
    dim3 grid((unsigned)ceil_div(g.F, 32), (unsigned)ceil_div(g.B, 8));
    if (grid.y > 65535) return fail(TB_ERR_INVALID, "fc: batch too large");
    {
        const int _lr = launch(ctx, "k_fc_sdot8", k_fc_sdot8, dim3(grid), dim3(256), 0, p, (int)g.B, (int)g.C);
        if (_lr != TB_OK) return _lr;
    }
    if (launches) ++*launches;
    return check_launch("k_fc_sdot8");
}

}  // namespace tbi

extern "C" {

int tb_fc_fwd(tb_ctx* ctx, int64_t batch, int64_t inputs, int64_t outputs, const float* x,
              const float* packed_w, const float* bias, int64_t activation, float* y) {
    TB_ENTER(ctx);
    tb_conv_desc d = {};
    d.batch = batch; d.channels = inputs; d.height = 1; d.width = 1;
    d.filters = outputs; d.kernel_h = 1; d.kernel_w = 1; d.stride_y = 1; d.stride_x = 1;
    d.activation = activation;
    if (batch == 0) return TB_OK;
    if (!x || !packed_w || !y) return fail(TB_ERR_INVALID, "fc: null x, weights or y");
    if (!act_supported(activation)) return fail(TB_ERR_UNSUPPORTED, "fc: activation %lld not supported", (long long)activation);
    ConvGeom g;
    int r = conv_geom(&d, &g);
    if (r != TB_OK) return r;
    return fc_sdot_launch(ctx, g, x, packed_w, bias, nullptr, nullptr, nullptr, y, (int)activation, nullptr);
}

}  // extern "C"
