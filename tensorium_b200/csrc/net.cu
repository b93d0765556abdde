// net.cu -- whole-network executor: the device-resident TNNet.forward / predict
// (source/nnet.pas:275-317, 452-472) for darknet conv networks.
//
// The reference runs layer.forwardGPU one after another, each a handful of launches
// (per-image im2col, GEMM, bias, activation, copies).  This executor:
//   * folds batchnorm on the host (TNNet.fuseBatchNorm, source/nnet.pas:268-273) when asked;
//   * fuses a shortcut into the epilogue of the conv before it (residual add) and the yolo
//     activation into the head conv, when that conv's raw output has no other reader;
//   * makes multi-input routes zero-copy: producers write straight into their channel slice of
//     the concat buffer and consumers read it with a batch stride;
//   * allocates every activation once (HBM is plentiful: YOLOv3-416 at batch 8 needs ~1.3 GB)
//     and replays the whole forward as one CUDA graph.
#include "conv.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <functional>
#include <vector>

namespace tbi {
int copy_rows(tb_ctx* ctx, int64_t batch, int64_t n, const float* src, int64_t src_bs, float* dst,
              int64_t dst_bs);
}
using namespace tbi;

namespace {

struct View {
    float* ptr = nullptr;
    int64_t bs = 0;  // elements between images
    int64_t ps = 0;  // 0: NCHW; > 0: NHWC with ps floats per pixel (ptr at the first channel)
};

struct Layer {
    int type = 0;
    int64_t c = 0, h = 0, w = 0;     // input shape
    int64_t oc = 0, oh = 0, ow = 0;  // output shape
    // conv / connected
    int64_t filters = 0, ksize = 0, stride = 0, pad = 0, act = TB_ACT_LINEAR;
    bool bn = false;
    std::vector<float> weights, biases, scales, mean, var;
    float *d_wp = nullptr, *d_bias = nullptr, *d_scale = nullptr, *d_mean = nullptr, *d_var = nullptr;
    // shortcut
    int64_t from = -1;
    // route
    std::vector<int64_t> inputs;
    bool route_zero_copy = false;
    // upsample
    float up_scale = 1.0f;
    // yolo
    int64_t classes = 0, n = 0;
    std::vector<int64_t> mask;
    std::vector<float> anchors;
    float scale_xy = 1.0f;
    // softmax
    int64_t groups = 1;
    float temperature = 1.0f;
    // plan
    bool absorbed = false;      // computed inside the previous conv's epilogue
    int64_t fuse_res = -1;      // conv: residual layer index
    int64_t fuse_yolo = 0;      // conv: yolo classes
    int64_t target = -1;        // conv: layer whose output view it writes (itself or next)
    View out;
    float* own = nullptr;       // allocation owned by this layer
    int64_t own_floats = 0;
    int64_t per_image() const { return oc * oh * ow; }
};

}  // namespace

struct tb_net {
    tb_ctx* ctx = nullptr;
    int64_t batch = 0, c = 0, h = 0, w = 0;
    std::vector<std::unique_ptr<Layer>> layers;
    bool fusion = true;
    bool finalized = false;
    int64_t math_mode = TB_MATH_FP32;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    const float* graph_x = nullptr;
    int64_t launches = 0, graph_launches = 0;
    double flops = 0.0;
    std::vector<float*> allocs;
    // NHWC plan (TF32 networks made of convs, shortcuts, routes, upsamples and fused yolo heads):
    // activations are NHWC, every conv runs on the NHWC tensor-core kernel, the input is
    // converted into x_nhwc (x_ps floats per pixel) first and the yolo heads are written NCHW
    bool nhwc = false;
    int pair = 0;  // NHWC plan in BF16-split mode: activations as bf16 (hi, lo) pairs
    float* x_nhwc = nullptr;
    int64_t x_ps = 0;
    // the first conv with C * KH * KW <= 32 runs as a 1x1 conv over its receptive fields
    // (x_nhwc holds [batch][oh][ow][32], made by the input conversion)
    bool first_im2col = false;
    // or, when it fits nhwc_first_direct (F <= 128, leaky or linear), computed straight from the
    // NCHW network input into its NHWC output (no x_nhwc, no receptive-field pass)
    bool first_direct = false;
    // Branch schedule (FP32 NCHW plans, whose kernels share no scratch memory): the layers on the
    // network's longest remaining path run on the launch stream, every other layer (e.g. the
    // tails of YOLOv3's 13x13 and 26x26 heads) on a second stream, concurrently with the next
    // scale's trunk; the edges that cross the two streams are ordered by events.
    bool branches = false;
    std::vector<int> lane;                    // per layer: 0 = launch stream, 1 = branch stream
    std::vector<std::vector<int64_t>> waits;  // per layer: producers on the other stream
    std::vector<cudaEvent_t> done;            // per layer: recorded after it when a consumer waits
    cudaStream_t side = nullptr;
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    // the branch stream's own split-K workspace and arrival counters (NHWC tensor-core plans, whose
    // split-K layers would otherwise share the context's with the launch stream's layers)
    void* side_ws = nullptr;
    size_t side_ws_bytes = 0;
    int* side_cnt = nullptr;
    int64_t side_cnt_len = 0;
};

namespace {
// geometry of the first layer run as a 1x1 conv over 32 receptive-field channels
ConvGeom first_as_1x1(const ConvGeom& g) {
    ConvGeom f = g;
    f.C = 32; f.H = g.OH; f.W = g.OW;
    f.KH = f.KW = 1; f.SY = f.SX = 1; f.PY = f.PX = 0; f.DY = f.DX = 1;
    return f;
}
}  // namespace

namespace {

int add_layer(tb_net* net, std::unique_ptr<Layer> L) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (net->finalized) return fail(TB_ERR_STATE, "net already finalized");
    net->layers.push_back(std::move(L));
    return (int)net->layers.size() - 1;
}

// output shape of every layer given the shapes of the layers before it
int infer_shapes(tb_net* net) {
    for (size_t i = 0; i < net->layers.size(); ++i) {
        Layer& L = *net->layers[i];
        if (i == 0) { L.c = net->c; L.h = net->h; L.w = net->w; }
        else { const Layer& P = *net->layers[i - 1]; L.c = P.oc; L.h = P.oh; L.w = P.ow; }
        switch (L.type) {
        case TB_LAYER_CONV: {
            if (L.weights.size() != (size_t)(L.filters * L.c * L.ksize * L.ksize))
                return fail(TB_ERR_INVALID, "layer %zu: conv weights hold %zu floats, expected %lld (c=%lld)",
                            i, L.weights.size(), (long long)(L.filters * L.c * L.ksize * L.ksize), (long long)L.c);
            L.oc = L.filters;
            L.oh = (L.h + 2 * L.pad - L.ksize) / L.stride + 1;
            L.ow = (L.w + 2 * L.pad - L.ksize) / L.stride + 1;
            if (L.oh <= 0 || L.ow <= 0) return fail(TB_ERR_INVALID, "layer %zu: empty conv output", i);
            break;
        }
        case TB_LAYER_SHORTCUT: {
            if (L.from < 0 || L.from >= (int64_t)i) return fail(TB_ERR_INVALID, "layer %zu: bad shortcut source", i);
            const Layer& F = *net->layers[L.from];
            if (F.oc != L.c || F.oh != L.h || F.ow != L.w)
                return fail(TB_ERR_UNSUPPORTED, "layer %zu: shortcut between different shapes", i);
            L.oc = L.c; L.oh = L.h; L.ow = L.w;
            break;
        }
        case TB_LAYER_ROUTE: {
            int64_t tc = 0, rh = -1, rw = -1;
            for (int64_t j : L.inputs) {
                if (j < 0 || j >= (int64_t)i) return fail(TB_ERR_INVALID, "layer %zu: bad route input", i);
                const Layer& S = *net->layers[j];
                if (rh < 0) { rh = S.oh; rw = S.ow; }
                if (S.oh != rh || S.ow != rw) return fail(TB_ERR_INVALID, "layer %zu: route inputs differ in size", i);
                tc += S.oc;
            }
            L.oc = tc; L.oh = rh; L.ow = rw;
            break;
        }
        case TB_LAYER_UPSAMPLE:
            L.oc = L.c; L.oh = L.h * L.stride; L.ow = L.w * L.stride;
            break;
        case TB_LAYER_YOLO:
            if (L.c != L.n * (L.classes + 5))
                return fail(TB_ERR_INVALID, "layer %zu: yolo expects %lld channels, got %lld", i,
                            (long long)(L.n * (L.classes + 5)), (long long)L.c);
            L.oc = L.c; L.oh = L.h; L.ow = L.w;
            break;
        case TB_LAYER_MAXPOOL:
            L.oc = L.c;
            L.oh = (L.h + L.pad - L.ksize) / L.stride + 1;
            L.ow = (L.w + L.pad - L.ksize) / L.stride + 1;
            break;
        case TB_LAYER_CONNECTED:
            if (L.weights.size() != (size_t)(L.filters * L.c * L.h * L.w))
                return fail(TB_ERR_INVALID, "layer %zu: connected weights hold %zu floats, expected %lld",
                            i, L.weights.size(), (long long)(L.filters * L.c * L.h * L.w));
            L.oc = L.filters; L.oh = 1; L.ow = 1;
            break;
        case TB_LAYER_SOFTMAX:
            L.oc = L.c; L.oh = L.h; L.ow = L.w;
            if ((L.c * L.h * L.w) % L.groups) return fail(TB_ERR_INVALID, "layer %zu: softmax groups", i);
            break;
        case TB_LAYER_AVGPOOL:
            L.oc = L.c; L.oh = 1; L.ow = 1;
            break;
        default:
            return fail(TB_ERR_INVALID, "layer %zu: unknown type", i);
        }
    }
    return TB_OK;
}

// readers[j] = layers that read layer j's output
std::vector<std::vector<int64_t>> readers_of(const tb_net* net) {
    const int64_t n = (int64_t)net->layers.size();
    std::vector<std::vector<int64_t>> r((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        const Layer& L = *net->layers[i];
        if (L.type == TB_LAYER_ROUTE) {
            for (int64_t j : L.inputs) r[j].push_back(i);
        } else {
            if (i > 0) r[i - 1].push_back(i);
            if (L.type == TB_LAYER_SHORTCUT) r[L.from].push_back(i);
        }
    }
    return r;
}

float* dev_upload(tb_net* net, const std::vector<float>& v, int* err) {
    if (v.empty()) return nullptr;
    float* p = nullptr;
    cudaError_t e = cudaMalloc(&p, v.size() * sizeof(float));
    if (e != cudaSuccess) { *err = cuda_fail(e, "cudaMalloc(weights)"); return nullptr; }
    net->allocs.push_back(p);
    e = cudaMemcpy(p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { *err = cuda_fail(e, "cudaMemcpy(weights)"); return nullptr; }
    return p;
}

void desc_of(const tb_net* net, const Layer& L, tb_conv_desc* d) {
    *d = tb_conv_desc{};
    d->batch = net->batch;
    if (L.type == TB_LAYER_CONV) {
        d->channels = L.c; d->height = L.h; d->width = L.w;
        d->kernel_h = L.ksize; d->kernel_w = L.ksize;
        d->stride_y = L.stride; d->stride_x = L.stride; d->pad_y = L.pad; d->pad_x = L.pad;
    } else {  // connected: a 1x1 conv over 1x1 images with c*h*w channels
        d->channels = L.c * L.h * L.w; d->height = 1; d->width = 1;
        d->kernel_h = d->kernel_w = 1; d->stride_y = d->stride_x = 1;
    }
    d->filters = L.filters;
    d->activation = L.act;
}

View input_view(tb_net* net, int64_t i, const float* x) {
    if (i == 0) {
        View v;
        if (net->nhwc) {
            v.ptr = net->x_nhwc;
            v.ps = net->x_ps;
            const Layer& L0 = *net->layers[0];
            v.bs = (net->first_im2col ? L0.oh * L0.ow : net->h * net->w) * net->x_ps;
            return v;
        }
        v.ptr = const_cast<float*>(x);
        v.bs = net->c * net->h * net->w;
        return v;
    }
    return net->layers[i - 1]->out;
}

// One layer of the NHWC plan.
int run_layer_nhwc(tb_net* net, int64_t i, const float* x) {
    tb_ctx* ctx = net->ctx;
    Layer& L = *net->layers[i];
    const int64_t B = net->batch;
    int r;
    if (i == 0 && net->first_direct) {
        const Layer& T = *net->layers[L.target];
        net->launches++;
        return nhwc_first_direct(ctx, B, net->c, net->h, net->w, L.ksize, L.ksize, L.stride, L.stride, L.pad, L.pad,
                                 1, 1, L.oh, L.ow, x, net->c * net->h * net->w, L.d_wp, L.d_bias, L.oc, (int)L.act,
                                 T.out.ptr, T.out.ps, net->pair);
    }
    if (i == 0) {  // the network input, NCHW, into the NHWC staging buffer (or its receptive fields)
        if (net->first_im2col)
            r = nhwc_im2col_first(ctx, B, net->c, net->h, net->w, L.ksize, L.ksize, L.stride, L.stride, L.pad, L.pad,
                                  1, 1, L.oh, L.ow, x, net->c * net->h * net->w, net->x_nhwc, net->pair);
        else
            r = nhwc_from_nchw(ctx, B, net->c, net->h, net->w, x, net->c * net->h * net->w, net->x_nhwc, net->x_ps,
                               net->pair);
        if (r != TB_OK) return r;
        net->launches++;
    }
    if (L.absorbed) return TB_OK;
    View in = input_view(net, i, x);
    switch (L.type) {
    case TB_LAYER_CONV: {
        tb_conv_desc d;
        desc_of(net, L, &d);
        const Layer& T = *net->layers[L.target];
        d.out_batch_stride = T.out.bs;
        ConvGeom g;
        r = conv_geom(&d, &g);
        if (r != TB_OK) return r;
        if (i == 0 && net->first_im2col) g = first_as_1x1(g);
        const float* res = nullptr;
        int64_t rps = 0;
        if (L.fuse_res >= 0) {
            res = net->layers[L.fuse_res]->out.ptr;
            rps = net->layers[L.fuse_res]->out.ps;
        }
        net->launches++;
        return conv_nhwc_launch(ctx, g, in.ptr, in.ps, L.d_wp, L.d_bias, res, rps, T.out.ptr, T.out.ps, (int)L.act,
                                (int)L.fuse_yolo, nullptr, net->pair);
    }
    case TB_LAYER_SHORTCUT: {
        const Layer& F = *net->layers[L.from];
        net->launches++;
        return nhwc_shortcut(ctx, B * L.oh * L.ow, L.oc, in.ptr, in.ps, F.out.ptr, F.out.ps, L.out.ptr, L.out.ps,
                             (int)L.act, net->pair);
    }
    case TB_LAYER_ROUTE: {
        if (L.route_zero_copy) return TB_OK;
        int64_t off = 0;
        for (int64_t j : L.inputs) {
            const Layer& S = *net->layers[j];
            r = nhwc_copy(ctx, B * L.oh * L.ow, S.oc, S.out.ptr, S.out.ps, L.out.ptr + off, L.out.ps);
            if (r != TB_OK) return r;
            net->launches++;
            off += S.oc;
        }
        return TB_OK;
    }
    case TB_LAYER_UPSAMPLE:
        net->launches++;
        return nhwc_upsample(ctx, B, L.c, L.h, L.w, L.stride, L.up_scale, in.ptr, in.ps, L.out.ptr, L.out.ps,
                             net->pair);
    }
    return fail(TB_ERR_STATE, "layer %lld: not on the NHWC plan", (long long)i);
}

int run_layer(tb_net* net, int64_t i, const float* x) {
    if (net->nhwc) return run_layer_nhwc(net, i, x);
    tb_ctx* ctx = net->ctx;
    Layer& L = *net->layers[i];
    if (L.absorbed) return TB_OK;
    const int64_t B = net->batch;
    View in = input_view(net, i, x);
    int r = TB_OK;
    switch (L.type) {
    case TB_LAYER_CONV:
    case TB_LAYER_CONNECTED: {
        tb_conv_desc d;
        desc_of(net, L, &d);
        const Layer& T = *net->layers[L.target];
        d.in_batch_stride = in.bs;
        d.out_batch_stride = T.out.bs;
        const float* res = nullptr;
        if (L.fuse_res >= 0) {
            res = net->layers[L.fuse_res]->out.ptr;
            d.res_batch_stride = net->layers[L.fuse_res]->out.bs;
        }
        ConvGeom g;
        r = conv_geom(&d, &g);
        if (r != TB_OK) return r;
        if (net->math_mode == TB_MATH_TF32 && conv_tc_supported(g))
            return conv_tc_launch(ctx, g, in.ptr, L.d_wp, L.d_bias, L.bn ? L.d_scale : nullptr,
                                  L.bn ? L.d_mean : nullptr, L.bn ? L.d_var : nullptr, res, T.out.ptr,
                                  (int)L.act, (int)L.fuse_yolo, reinterpret_cast<float*>(ctx->ws), &net->launches);
        if (L.type == TB_LAYER_CONNECTED && net->math_mode != TB_MATH_FP32_TILED)
            return fc_sdot_launch(ctx, g, in.ptr, L.d_wp, L.d_bias, L.bn ? L.d_scale : nullptr,
                                  L.bn ? L.d_mean : nullptr, L.bn ? L.d_var : nullptr, T.out.ptr, (int)L.act,
                                  &net->launches);
        if (net->math_mode != TB_MATH_FP32_TILED && conv_exact_supported(g))
            return conv_exact_launch(ctx, g, in.ptr, L.d_wp, L.d_bias, L.bn ? L.d_scale : nullptr,
                                     L.bn ? L.d_mean : nullptr, L.bn ? L.d_var : nullptr, res, T.out.ptr,
                                     (int)L.act, (int)L.fuse_yolo, true, &net->launches);
        return conv_fp32_launch(ctx, g, in.ptr, L.d_wp, L.d_bias, L.bn ? L.d_scale : nullptr,
                                L.bn ? L.d_mean : nullptr, L.bn ? L.d_var : nullptr, res, T.out.ptr,
                                (int)L.act, (int)L.fuse_yolo, nullptr, 0, &net->launches);
    }
    case TB_LAYER_SHORTCUT: {
        const Layer& F = *net->layers[L.from];
        if (in.bs != L.per_image() || F.out.bs != L.per_image() || L.out.bs != L.per_image())
            return fail(TB_ERR_STATE, "layer %lld: strided shortcut operands", (long long)i);
        r = tb_shortcut_fwd(ctx, B * L.per_image(), in.ptr, F.out.ptr, L.out.ptr, L.act);
        net->launches++;
        return r;
    }
    case TB_LAYER_ROUTE: {
        if (L.route_zero_copy) return TB_OK;
        int64_t off = 0;
        for (int64_t j : L.inputs) {
            const Layer& S = *net->layers[j];
            r = copy_rows(ctx, B, S.per_image(), S.out.ptr, S.out.bs, L.out.ptr + off, L.out.bs);
            if (r != TB_OK) return r;
            net->launches++;
            off += S.per_image();
        }
        return TB_OK;
    }
    case TB_LAYER_UPSAMPLE:
        if (in.bs != L.c * L.h * L.w) return fail(TB_ERR_STATE, "layer %lld: strided upsample input", (long long)i);
        r = tb_upsample_fwd(ctx, B, L.c, L.h, L.w, L.stride, L.up_scale, in.ptr, L.out.ptr, L.out.bs);
        net->launches++;
        return r;
    case TB_LAYER_YOLO:
        if (in.bs != L.c * L.h * L.w) return fail(TB_ERR_STATE, "layer %lld: strided yolo input", (long long)i);
        r = tb_yolo_fwd(ctx, B, L.n, L.classes, L.h, L.w, in.ptr, L.out.ptr, L.scale_xy);
        net->launches++;
        return r;
    case TB_LAYER_MAXPOOL:
        if (in.bs != L.c * L.h * L.w) return fail(TB_ERR_STATE, "layer %lld: strided maxpool input", (long long)i);
        r = tb_maxpool_fwd(ctx, B, L.c, L.h, L.w, L.ksize, L.stride, L.stride, L.pad, in.ptr, L.out.ptr, nullptr);
        net->launches++;
        return r;
    case TB_LAYER_SOFTMAX:
        if (in.bs != L.c * L.h * L.w) return fail(TB_ERR_STATE, "layer %lld: strided softmax input", (long long)i);
        r = tb_softmax_fwd(ctx, B, L.c * L.h * L.w, L.groups, L.temperature, in.ptr, L.out.ptr);
        net->launches++;
        return r;
    case TB_LAYER_AVGPOOL:
        if (in.bs != L.c * L.h * L.w) return fail(TB_ERR_STATE, "layer %lld: strided avgpool input", (long long)i);
        r = tb_avgpool_fwd(ctx, B, L.c, L.h, L.w, in.ptr, L.out.ptr);
        net->launches++;
        return r;
    }
    return fail(TB_ERR_INVALID, "layer %lld: unknown type", (long long)i);
}

int run_all(tb_net* net, const float* x) {
    net->launches = 0;
    const int64_t n = (int64_t)net->layers.size();
    if (!net->branches) {
        for (int64_t i = 0; i < n; ++i) {
            int r = run_layer(net, i, x);
            if (r != TB_OK) return r;
        }
        return TB_OK;
    }
    tb_ctx* ctx = net->ctx;
    cudaStream_t main = ctx->stream;
    TB_CHECK_CUDA(cudaEventRecord(net->fork_ev, main));
    TB_CHECK_CUDA(cudaStreamWaitEvent(net->side, net->fork_ev, 0));
    int r = TB_OK;
    for (int64_t i = 0; i < n && r == TB_OK; ++i) {
        cudaStream_t st = net->lane[i] ? net->side : main;
        for (int64_t p : net->waits[i])
            if (cudaStreamWaitEvent(st, net->done[p], 0) != cudaSuccess) r = fail(TB_ERR_CUDA, "branch wait");
        if (r != TB_OK) break;
        ctx->stream = st;
        void* ws = ctx->ws;
        const size_t wsb = ctx->ws_bytes;
        int* cnt = ctx->tile_cnt;
        const int64_t cnt_len = ctx->tile_cnt_len;
        if (net->lane[i] && net->side_ws) {
            ctx->ws = net->side_ws;
            ctx->ws_bytes = net->side_ws_bytes;
            ctx->tile_cnt = net->side_cnt;
            ctx->tile_cnt_len = net->side_cnt_len;
        }
        r = run_layer(net, i, x);
        ctx->stream = main;
        ctx->ws = ws;
        ctx->ws_bytes = wsb;
        ctx->tile_cnt = cnt;
        ctx->tile_cnt_len = cnt_len;
        if (r == TB_OK && net->done[i] && cudaEventRecord(net->done[i], st) != cudaSuccess)
            r = fail(TB_ERR_CUDA, "branch event");
    }
    // join the branch stream back in every case (a capture must end with it joined)
    cudaEventRecord(net->join_ev, net->side);
    cudaStreamWaitEvent(main, net->join_ev, 0);
    return r;
}

// The branch schedule of a finalized FP32 NCHW plan (see tb_net::branches).
int plan_branches(tb_net* net) {
    const int64_t n = (int64_t)net->layers.size();
    // launches[i]: layer i launches a kernel; src(j): the layers whose launches write j's output
    std::vector<char> launches((size_t)n, 0);
    for (int64_t i = 0; i < n; ++i) {
        const Layer& L = *net->layers[i];
        launches[i] = !L.absorbed && !(L.type == TB_LAYER_ROUTE && L.route_zero_copy);
    }
    std::function<void(int64_t, std::vector<int64_t>&)> src = [&](int64_t j, std::vector<int64_t>& out) {
        const Layer& L = *net->layers[j];
        if (L.absorbed) { out.push_back(j - 1); return; }  // written by the conv that absorbed it
        if (L.type == TB_LAYER_ROUTE && L.route_zero_copy) {
            for (int64_t k : L.inputs) src(k, out);
            return;
        }
        out.push_back(j);
    };
    std::vector<std::vector<int64_t>> prod((size_t)n), cons((size_t)n);
    std::vector<double> cost((size_t)n, 0.0);
    for (int64_t i = 0; i < n; ++i) {
        if (!launches[i]) continue;
        const Layer& L = *net->layers[i];
        std::vector<int64_t> p;
        if (L.type == TB_LAYER_ROUTE) {
            for (int64_t k : L.inputs) src(k, p);
        } else {
            if (i > 0) src(i - 1, p);
            if (L.type == TB_LAYER_SHORTCUT) src(L.from, p);
            if (L.fuse_res >= 0) src(L.fuse_res, p);
        }
        std::sort(p.begin(), p.end());
        p.erase(std::unique(p.begin(), p.end()), p.end());
        for (int64_t q : p) cons[q].push_back(i);
        prod[i] = p;
        cost[i] = (L.type == TB_LAYER_CONV || L.type == TB_LAYER_CONNECTED)
                      ? 2.0 * L.filters * L.oh * L.ow * L.c * L.ksize * L.ksize
                      : 1e5;
    }
    // longest remaining path (by FLOPs) from each launch; the trunk follows its maximum
    std::vector<double> rem((size_t)n, 0.0);
    for (int64_t i = n - 1; i >= 0; --i) {
        if (!launches[i]) continue;
        double m = 0.0;
        for (int64_t c : cons[i]) m = std::max(m, rem[c]);
        rem[i] = cost[i] + m;
    }
    net->lane.assign((size_t)n, 0);
    std::vector<char> trunk((size_t)n, 0);
    int64_t t = -1;
    for (int64_t i = 0; i < n && t < 0; ++i)
        if (launches[i]) t = i;
    while (t >= 0) {
        trunk[t] = 1;
        int64_t nx = -1;
        for (int64_t c : cons[t])
            if (nx < 0 || rem[c] > rem[nx]) nx = c;
        t = nx;
    }
    bool any = false;
    for (int64_t i = 0; i < n; ++i)
        if (launches[i] && !trunk[i]) { net->lane[i] = 1; any = true; }
    if (!any) return TB_OK;
    net->waits.assign((size_t)n, {});
    net->done.assign((size_t)n, nullptr);
    for (int64_t i = 0; i < n; ++i)
        for (int64_t q : prod[i])
            if (net->lane[q] != net->lane[i]) {
                net->waits[i].push_back(q);
                if (!net->done[q]) TB_CHECK_CUDA(cudaEventCreateWithFlags(&net->done[q], cudaEventDisableTiming));
            }
    TB_CHECK_CUDA(cudaStreamCreateWithFlags(&net->side, cudaStreamNonBlocking));
    TB_CHECK_CUDA(cudaEventCreateWithFlags(&net->fork_ev, cudaEventDisableTiming));
    TB_CHECK_CUDA(cudaEventCreateWithFlags(&net->join_ev, cudaEventDisableTiming));
    net->branches = true;
    return TB_OK;
}

void free_graph(tb_net* net) {
    if (net->exec) cudaGraphExecDestroy(net->exec);
    if (net->graph) cudaGraphDestroy(net->graph);
    net->exec = nullptr;
    net->graph = nullptr;
    net->graph_x = nullptr;
}

}  // namespace

extern "C" {

int tb_net_create(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t height, int64_t width, tb_net** out) {
    // ctx may be NULL: a host-only net that can be built, inspected and saved, not finalized
    if (ctx) TB_ENTER(ctx);
    if (!out || batch <= 0 || channels <= 0 || height <= 0 || width <= 0)
        return fail(TB_ERR_INVALID, "tb_net_create: bad arguments");
    tb_net* n = new tb_net();
    n->ctx = ctx;
    n->batch = batch; n->c = channels; n->h = height; n->w = width;
    n->math_mode = ctx ? ctx->math_mode : TB_MATH_FP32;
    *out = n;
    return TB_OK;
}

int tb_net_destroy(tb_net* net) {
    if (!net) return TB_OK;
    if (!net->ctx) { delete net; return TB_OK; }
    enter(net->ctx);
    cudaStreamSynchronize(net->ctx->stream);
    free_graph(net);
    if (net->side) cudaStreamSynchronize(net->side);
    for (cudaEvent_t e : net->done)
        if (e) cudaEventDestroy(e);
    if (net->fork_ev) cudaEventDestroy(net->fork_ev);
    if (net->join_ev) cudaEventDestroy(net->join_ev);
    if (net->side) cudaStreamDestroy(net->side);
    for (float* p : net->allocs) cudaFree(p);
    delete net;
    return TB_OK;
}

static int prev_channels(tb_net* net, int64_t* out) {
    if (net->layers.empty()) { *out = net->c; return TB_OK; }
    int r = infer_shapes(net);
    if (r != TB_OK) return r;
    *out = net->layers.back()->oc;
    return TB_OK;
}

int tb_net_add_conv(tb_net* net, int64_t filters, int64_t ksize, int64_t stride, int64_t pad,
                    int64_t activation, int64_t batch_normalize, const float* weights,
                    const float* biases, const float* scales, const float* mean, const float* var) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (filters <= 0 || ksize <= 0 || stride <= 0 || pad < 0 || !weights)
        return fail(TB_ERR_INVALID, "conv layer: bad arguments");
    if (!act_supported(activation)) return fail(TB_ERR_UNSUPPORTED, "conv layer: activation not supported");
    if (batch_normalize && (!scales || !mean || !var))
        return fail(TB_ERR_INVALID, "conv layer: batchnorm needs scales, mean and variance");
    int64_t cin;
    int r = prev_channels(net, &cin);
    if (r != TB_OK) return r;
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_CONV;
    L->filters = filters; L->ksize = ksize; L->stride = stride; L->pad = pad; L->act = activation;
    L->bn = batch_normalize != 0;
    L->weights.assign(weights, weights + filters * cin * ksize * ksize);
    L->biases = biases ? std::vector<float>(biases, biases + filters) : std::vector<float>((size_t)filters, 0.0f);
    if (L->bn) {
        L->scales.assign(scales, scales + filters);
        L->mean.assign(mean, mean + filters);
        L->var.assign(var, var + filters);
    }
    return add_layer(net, std::move(L));
}

int tb_net_add_shortcut(tb_net* net, int64_t from, int64_t activation) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (!act_supported(activation)) return fail(TB_ERR_UNSUPPORTED, "shortcut: activation not supported");
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_SHORTCUT;
    int64_t idx = (int64_t)net->layers.size();
    L->from = from < 0 ? idx + from : from;  // darknet: negative = relative
    L->act = activation;
    return add_layer(net, std::move(L));
}

int tb_net_add_route(tb_net* net, int64_t n, const int64_t* layers) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (n <= 0 || !layers) return fail(TB_ERR_INVALID, "route: bad arguments");
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_ROUTE;
    int64_t idx = (int64_t)net->layers.size();
    for (int64_t k = 0; k < n; ++k) L->inputs.push_back(layers[k] < 0 ? idx + layers[k] : layers[k]);
    return add_layer(net, std::move(L));
}

int tb_net_add_upsample(tb_net* net, int64_t stride, float scale) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (stride <= 0) return fail(TB_ERR_UNSUPPORTED, "upsample: only forward (positive) strides");
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_UPSAMPLE;
    L->stride = stride;
    L->up_scale = scale;
    return add_layer(net, std::move(L));
}

int tb_net_add_yolo(tb_net* net, int64_t classes, int64_t n, const int64_t* mask,
                    int64_t total_anchors, const float* anchors, float scale_xy) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (classes < 0 || n <= 0 || !mask || total_anchors <= 0 || !anchors)
        return fail(TB_ERR_INVALID, "yolo: bad arguments");
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_YOLO;
    L->classes = classes; L->n = n;
    L->mask.assign(mask, mask + n);
    for (int64_t m : L->mask)
        if (m < 0 || m >= total_anchors) return fail(TB_ERR_INVALID, "yolo: mask out of range");
    L->anchors.assign(anchors, anchors + 2 * total_anchors);
    L->scale_xy = scale_xy;
    return add_layer(net, std::move(L));
}

int tb_net_add_maxpool(tb_net* net, int64_t ksize, int64_t stride, int64_t padding) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (ksize <= 0 || stride <= 0 || padding < 0) return fail(TB_ERR_INVALID, "maxpool: bad arguments");
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_MAXPOOL;
    L->ksize = ksize; L->stride = stride; L->pad = padding;
    return add_layer(net, std::move(L));
}

int tb_net_add_connected(tb_net* net, int64_t outputs, int64_t activation, const float* weights,
                         const float* biases) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (outputs <= 0 || !weights) return fail(TB_ERR_INVALID, "connected: bad arguments");
    if (!act_supported(activation)) return fail(TB_ERR_UNSUPPORTED, "connected: activation not supported");
    int64_t inputs;
    if (net->layers.empty()) inputs = net->c * net->h * net->w;
    else {
        int r = infer_shapes(net);
        if (r != TB_OK) return r;
        const Layer& P = *net->layers.back();
        inputs = P.oc * P.oh * P.ow;
    }
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_CONNECTED;
    L->filters = outputs; L->act = activation;
    L->weights.assign(weights, weights + outputs * inputs);
    L->biases = biases ? std::vector<float>(biases, biases + outputs) : std::vector<float>((size_t)outputs, 0.0f);
    return add_layer(net, std::move(L));
}

int tb_net_add_softmax(tb_net* net, int64_t groups, float temperature) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (groups <= 0) return fail(TB_ERR_INVALID, "softmax: bad groups");
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_SOFTMAX;
    L->groups = groups;
    L->temperature = temperature;
    return add_layer(net, std::move(L));
}

int tb_net_add_avgpool(tb_net* net) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    auto L = std::make_unique<Layer>();
    L->type = TB_LAYER_AVGPOOL;
    return add_layer(net, std::move(L));
}

int tb_net_set_fusion(tb_net* net, int64_t enable) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (net->finalized) return fail(TB_ERR_STATE, "net already finalized");
    net->fusion = enable != 0;
    return TB_OK;
}

int tb_net_fuse_batchnorm(tb_net* net) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (net->finalized) return fail(TB_ERR_STATE, "net already finalized");
    int r = infer_shapes(net);
    if (r != TB_OK) return r;
    for (auto& Lp : net->layers) {
        Layer& L = *Lp;
        if (L.type != TB_LAYER_CONV || !L.bn) continue;
        r = tb_conv_fold_bn(L.filters, L.c * L.ksize * L.ksize, L.weights.data(), L.biases.data(),
                            L.scales.data(), L.mean.data(), L.var.data());
        if (r != TB_OK) return r;
        L.bn = false;
    }
    return TB_OK;
}

int tb_net_finalize(tb_net* net, int64_t math_mode) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (!net->ctx) return fail(TB_ERR_STATE, "net was created without a context (host-only)");
    TB_ENTER(net->ctx);
    if (net->finalized) return fail(TB_ERR_STATE, "net already finalized");
    if (net->layers.empty()) return fail(TB_ERR_INVALID, "empty net");
    if (math_mode != TB_MATH_FP32 && math_mode != TB_MATH_TF32 && math_mode != TB_MATH_FP32_TILED &&
        math_mode != TB_MATH_BF16_SPLIT)
        return fail(TB_ERR_UNSUPPORTED, "net: math mode %lld is not available in this build", (long long)math_mode);
    net->math_mode = math_mode;
    int r = infer_shapes(net);
    if (r != TB_OK) return r;
    const int64_t n = (int64_t)net->layers.size();
    const int64_t B = net->batch;
    auto rd = readers_of(net);

    // 1. fusion decisions: a conv whose only reader is the next layer absorbs a linear
    //    shortcut (residual epilogue) or a yolo layer (logistic epilogue)
    for (int64_t i = 0; i < n; ++i) net->layers[i]->target = i;
    if (net->fusion) {
        for (int64_t i = 0; i + 1 < n; ++i) {
            Layer& L = *net->layers[i];
            Layer& N = *net->layers[i + 1];
            if (L.type != TB_LAYER_CONV || rd[i].size() != 1 || rd[i][0] != i + 1) continue;
            if (N.type == TB_LAYER_SHORTCUT && N.act == TB_ACT_LINEAR && N.from != i) {
                L.fuse_res = N.from;
                L.target = i + 1;
                N.absorbed = true;
            } else if (N.type == TB_LAYER_YOLO && L.act == TB_ACT_LINEAR && N.scale_xy == 1.0f) {
                L.fuse_yolo = N.classes;
                L.target = i + 1;
                N.absorbed = true;
            }
        }
    }
    // 1b. the NHWC plan: a TF32 network made only of convs (batchnorm folded, geometries the
    //     NHWC tensor-core kernel takes), shortcuts, routes of 4-channel-multiple inputs,
    //     upsamples and fused yolo heads runs every activation in NHWC (TB_NET_NHWC=0: off)
    net->nhwc = false;
    net->first_im2col = false;
    net->first_direct = false;
    {
        const char* ev = getenv("TB_NET_NHWC");
        const bool tc_mode = math_mode == TB_MATH_TF32 || math_mode == TB_MATH_BF16_SPLIT;
        bool ok = tc_mode && net->fusion && !(ev && ev[0] == '0');
        for (int64_t i = 0; ok && i < n; ++i) {
            const Layer& L = *net->layers[i];
            switch (L.type) {
            case TB_LAYER_CONV: {
                tb_conv_desc d;
                desc_of(net, L, &d);
                ConvGeom g;
                if (L.bn || conv_geom(&d, &g) != TB_OK) { ok = false; break; }
                const char* fdv = getenv("TB_FIRST_DIRECT");
                if (i == 0 && L.target == 0 && (L.act == TB_ACT_LEAKY || L.act == TB_ACT_LINEAR) &&
                    !(fdv && fdv[0] == '0') &&
                    nhwc_first_direct_supported(L.c, L.ksize, L.ksize, L.stride, L.stride, 1, 1, L.oc, round_up(L.oc, 4))) {
                    net->first_direct = true;
                } else if (i == 0 && L.c * L.ksize * L.ksize <= 32) {
                    net->first_im2col = true;
                    if (!conv_nhwc_supported(first_as_1x1(g), 32)) ok = false;
                } else {
                    const int64_t xps = i == 0 ? round_up(net->c, 4) : round_up(L.c, 4);
                    if (!conv_nhwc_supported(g, xps) || (L.c % 4 && i > 0)) ok = false;
                }
                const Layer& T = *net->layers[L.target];
                if (T.type != TB_LAYER_YOLO && L.oc % 4) ok = false;
                break;
            }
            case TB_LAYER_SHORTCUT:
                if (L.oc % 4) ok = false;
                break;
            case TB_LAYER_UPSAMPLE:  // bf16 pairs are copied bit for bit: a scale needs decoding
                if (L.oc % 4 || (math_mode == TB_MATH_BF16_SPLIT && L.up_scale != 1.0f)) ok = false;
                break;
            case TB_LAYER_ROUTE:
                for (int64_t j : L.inputs)
                    if (net->layers[j]->oc % 4 || net->layers[j]->type == TB_LAYER_YOLO) ok = false;
                break;
            case TB_LAYER_YOLO:
                if (!L.absorbed) ok = false;
                break;
            default:
                ok = false;
            }
        }
        net->nhwc = ok;
        net->pair = ok && math_mode == TB_MATH_BF16_SPLIT ? 1 : 0;
        if (!ok) net->first_im2col = net->first_direct = false;
    }
    // floats per image and batch / pixel strides of a layer's own output buffer
    auto own_view = [&](Layer& L, float* ptr, int64_t channels_total) {
        View v;
        v.ptr = ptr;
        if (net->nhwc && L.type != TB_LAYER_YOLO) {
            v.ps = round_up(channels_total, 4);
            v.bs = L.oh * L.ow * v.ps;
        } else {
            v.bs = channels_total * L.oh * L.ow;
        }
        return v;
    };

    // producer[j]: the layer whose kernel writes j's output
    std::vector<int64_t> producer((size_t)n);
    for (int64_t i = 0; i < n; ++i) producer[i] = i;
    for (int64_t i = 0; i < n; ++i)
        if (net->layers[i]->target != i) producer[net->layers[i]->target] = i;
    // may j's output live in a route slice (batch stride > one image)? Every reader must take
    // a batch stride: a conv reading it as input, a conv reading it as residual (through an
    // absorbed shortcut), or a route copy.
    auto strided_reader_ok = [&](int64_t j) {
        for (int64_t k : rd[j]) {
            const Layer& R = *net->layers[k];
            if (R.type == TB_LAYER_ROUTE) continue;
            if (R.type == TB_LAYER_CONV && k == j + 1) continue;
            if (R.type == TB_LAYER_SHORTCUT && R.absorbed) continue;
            return false;
        }
        return true;
    };
    auto strided_writer_ok = [&](int64_t j) {
        const Layer& P = *net->layers[producer[j]];
        return P.type == TB_LAYER_CONV || P.type == TB_LAYER_UPSAMPLE;
    };

    // 2. buffers: multi-input routes first (their inputs may live inside them), then the rest
    std::vector<bool> placed((size_t)n, false);
    int err = TB_OK;
    auto alloc = [&](int64_t floats) -> float* {
        float* p = nullptr;
        cudaError_t e = cudaMalloc(&p, (size_t)floats * sizeof(float));
        if (e != cudaSuccess) { err = cuda_fail(e, "cudaMalloc(activations)"); return nullptr; }
        net->allocs.push_back(p);
        return p;
    };
    for (int64_t i = 0; i < n; ++i) {
        Layer& L = *net->layers[i];
        if (L.type != TB_LAYER_ROUTE || L.inputs.size() == 1) continue;
        L.out = own_view(L, nullptr, L.oc);
        L.own_floats = B * L.out.bs;
        L.own = alloc(L.own_floats);
        if (!L.own) return err;
        L.out.ptr = L.own;
        placed[i] = true;
        bool all = net->fusion;
        for (int64_t j : L.inputs)
            if (placed[j] || net->layers[j]->type == TB_LAYER_ROUTE || !strided_reader_ok(j) ||
                !strided_writer_ok(j))
                all = false;
        for (size_t a = 0; a < L.inputs.size(); ++a)
            for (size_t b = a + 1; b < L.inputs.size(); ++b)
                if (L.inputs[a] == L.inputs[b]) all = false;
        if (all) {
            int64_t off = 0;
            for (int64_t j : L.inputs) {
                Layer& S = *net->layers[j];
                S.out = L.out;  // NHWC: a channel slice; NCHW: a block of whole channel planes
                S.out.ptr = L.own + off;
                placed[j] = true;
                off += net->nhwc ? S.oc : S.per_image();
            }
            L.route_zero_copy = true;
        }
    }
    for (int64_t i = 0; i < n; ++i) {
        Layer& L = *net->layers[i];
        if (placed[i]) continue;
        if (L.type == TB_LAYER_ROUTE && L.inputs.size() == 1) {
            L.out = net->layers[L.inputs[0]]->out;  // alias; the input precedes the route
            L.route_zero_copy = true;
            placed[i] = true;
            continue;
        }
        if (L.target != i) {  // conv fused into the next layer: no buffer of its own
            placed[i] = true;
            continue;
        }
        L.out = own_view(L, nullptr, L.oc);
        L.own_floats = B * L.out.bs;
        L.own = alloc(L.own_floats);
        if (!L.own) return err;
        L.out.ptr = L.own;
        placed[i] = true;
    }
    if (net->nhwc && !net->first_direct) {
        const Layer& L0 = *net->layers[0];
        net->x_ps = net->first_im2col ? 32 : round_up(net->c, 4);
        net->x_nhwc = alloc(B * (net->first_im2col ? L0.oh * L0.ow : net->h * net->w) * net->x_ps);
        if (!net->x_nhwc) return err;
    }
    for (int64_t i = 0; i < n; ++i) {
        Layer& L = *net->layers[i];
        if (L.target != i) L.out = net->layers[L.target]->out;
    }

    // 3. weights, and the split-K workspace every conv will need
    int64_t ws_floats = 0;
    net->flops = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        Layer& L = *net->layers[i];
        if (L.type != TB_LAYER_CONV && L.type != TB_LAYER_CONNECTED) continue;
        tb_conv_desc d;
        desc_of(net, L, &d);
        ConvGeom g;
        r = conv_geom(&d, &g);
        if (r != TB_OK) return r;
        float* raw = dev_upload(net, L.weights, &err);
        if (!raw) return err;
        if (net->nhwc && i == 0 && net->first_direct) {
            L.d_wp = alloc(nhwc_first_direct_wcount(g.F, g.C, g.KH, g.KW));
            if (!L.d_wp) return err;
            r = nhwc_pack_first_direct(net->ctx, g.F, g.C, g.KH, g.KW, raw, L.d_wp, net->pair);
        } else if (net->nhwc && i == 0 && net->first_im2col) {
            L.d_wp = alloc(g.F * 32 * (net->pair ? 2 : 1));
            if (!L.d_wp) return err;
            r = nhwc_pack_first(net->ctx, g.F, g.C, g.KH, g.KW, raw, L.d_wp, net->pair);
        } else if (net->nhwc) {
            L.d_wp = alloc(conv_nhwc_packed_count(g, net->pair));
            if (!L.d_wp) return err;
            r = conv_nhwc_pack(net->ctx, g, raw, L.d_wp, net->pair);
        } else {
            L.d_wp = alloc(g.Kpad * g.Mpad);
            if (!L.d_wp) return err;
            r = tb_conv_pack_weights(net->ctx, &d, raw, L.d_wp);
            if (r == TB_OK && net->math_mode == TB_MATH_TF32 && conv_tc_supported(g))
                r = conv_tc_round_weights(net->ctx, L.d_wp, g.Kpad * g.Mpad);
        }
        if (r != TB_OK) return r;
        L.d_bias = dev_upload(net, L.biases, &err);
        if (err != TB_OK) return err;
        if (L.bn) {
            L.d_scale = dev_upload(net, L.scales, &err);
            L.d_mean = dev_upload(net, L.mean, &err);
            L.d_var = dev_upload(net, L.var, &err);
            if (err != TB_OK) return err;
        }
        if (net->math_mode == TB_MATH_FP32_TILED || !conv_exact_supported(g))
            ws_floats = std::max(ws_floats, conv_fp32_ws_floats(net->ctx, g));
        net->flops += 2.0 * (double)g.F * (double)(g.B * g.OH * g.OW) * (double)(g.C * g.KH * g.KW);
    }
    // 4. measure the tile / split choices of every conv geometry on the real buffers
    //    (TB_AUTOTUNE=0 keeps the cost model)
    const char* at = getenv("TB_AUTOTUNE");
    if (net->nhwc) {  // NHWC plan: tile width and K splits of every conv, measured on its buffers
        for (int64_t i = 0; i < n; ++i) {
            Layer& L = *net->layers[i];
            if (L.type != TB_LAYER_CONV || (i == 0 && net->first_direct)) continue;
            tb_conv_desc d;
            desc_of(net, L, &d);
            const Layer& T = *net->layers[L.target];
            d.out_batch_stride = T.out.bs;
            ConvGeom g;
            r = conv_geom(&d, &g);
            if (r != TB_OK) return r;
            if (i == 0 && net->first_im2col) g = first_as_1x1(g);
            const View in = input_view(net, i, nullptr);
            if (!(at && at[0] == '0')) {
                r = conv_nhwc_autotune(net->ctx, g, in.ptr, in.ps, L.d_wp, T.out.ptr, T.out.ps, net->pair);
                if (r != TB_OK) return r;
            }
            ws_floats = std::max(ws_floats, conv_nhwc_ws_floats(net->ctx, g, in.ps, net->pair));
        }
    }
    if (!(at && at[0] == '0') && !net->nhwc) {
        for (int64_t i = 0; i < n; ++i) {
            Layer& L = *net->layers[i];
            if (L.type != TB_LAYER_CONV && L.type != TB_LAYER_CONNECTED) continue;
            tb_conv_desc d;
            desc_of(net, L, &d);
            View in;
            float* tmp = nullptr;
            if (i == 0) {  // the network input is not known yet: tune on a zeroed stand-in
                in.bs = net->c * net->h * net->w;
                TB_CHECK_CUDA(cudaMalloc(&tmp, (size_t)(B * in.bs) * sizeof(float)));
                cudaMemset(tmp, 0, (size_t)(B * in.bs) * sizeof(float));
                in.ptr = tmp;
            } else {
                in = net->layers[i - 1]->out;
            }
            const Layer& T = *net->layers[L.target];
            d.in_batch_stride = in.bs;
            d.out_batch_stride = T.out.bs;
            ConvGeom g;
            r = conv_geom(&d, &g);
            if (r != TB_OK) { if (tmp) cudaFree(tmp); return r; }
            if (net->math_mode == TB_MATH_TF32 && conv_tc_supported(g)) {
                ws_floats = std::max(ws_floats, conv_tc_scratch_floats(g));
                r = conv_tc_autotune(net->ctx, g, in.ptr, L.d_wp, T.out.ptr);
                if (tmp) cudaFree(tmp);
                if (r != TB_OK) return r;
                continue;
            }
            if (net->math_mode != TB_MATH_FP32_TILED) {  // the order-exact kernels need no workspace
                r = L.type == TB_LAYER_CONNECTED ? TB_OK
                                                 : conv_exact_autotune(net->ctx, g, in.ptr, L.d_wp, T.out.ptr, true);
                if (tmp) cudaFree(tmp);
                if (r != TB_OK) return r;
                continue;
            }
            r = conv_fp32_autotune(net->ctx, g, in.ptr, L.d_wp, T.out.ptr);
            if (r == TB_OK) ws_floats = std::max(ws_floats, conv_fp32_ws_floats_for(net->ctx, g, in.ptr));
            if (tmp) cudaFree(tmp);
            if (r != TB_OK) return r;
        }
    }
    r = ensure_workspace(net->ctx, (size_t)std::max<int64_t>(ws_floats, 1) * sizeof(float));
    if (r != TB_OK) return r;
    // 5. branch schedule: FP32 NCHW plans whose convs all run on kernels without scratch memory
    //    (order-exact, direct, connected), and NHWC tensor-core plans, whose branch stream gets its
    //    own split-K workspace and counters; TB_NET_BRANCHES=0 keeps one stream
    {
        const char* bv = getenv("TB_NET_BRANCHES");
        const bool off = bv && bv[0] == '0';
        if (net->nhwc && !off) {
            r = plan_branches(net);
            if (r != TB_OK) return r;
            if (net->branches) {
                net->side_ws_bytes = net->ctx->ws_bytes;
                TB_CHECK_CUDA(cudaMalloc(&net->side_ws, std::max<size_t>(net->side_ws_bytes, 16)));
                net->allocs.push_back(reinterpret_cast<float*>(net->side_ws));
                net->side_cnt_len = net->ctx->tile_cnt_len;
                float* c = alloc(std::max<int64_t>(net->side_cnt_len, 1));
                if (!c) return err;
                net->side_cnt = reinterpret_cast<int*>(c);
                TB_CHECK_CUDA(cudaMemset(net->side_cnt, 0, (size_t)std::max<int64_t>(net->side_cnt_len, 1) * sizeof(int)));
            }
        }
        bool ok = !net->nhwc && math_mode == TB_MATH_FP32 && !off;
        for (int64_t i = 0; ok && i < n; ++i) {
            const Layer& L = *net->layers[i];
            if (L.type != TB_LAYER_CONV) continue;
            tb_conv_desc d;
            desc_of(net, L, &d);
            ConvGeom g;
            if (conv_geom(&d, &g) != TB_OK || !conv_exact_supported(g)) ok = false;
        }
        if (ok) {
            r = plan_branches(net);
            if (r != TB_OK) return r;
        }
    }
    TB_CHECK_CUDA(cudaStreamSynchronize(net->ctx->stream));
    net->finalized = true;
    return TB_OK;
}

int tb_net_forward(tb_net* net, const float* x, int64_t use_graph) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (!net->ctx) return fail(TB_ERR_STATE, "net was created without a context (host-only)");
    TB_ENTER(net->ctx);
    if (!net->finalized) return fail(TB_ERR_STATE, "net not finalized");
    if (!x) return fail(TB_ERR_INVALID, "null input");
    tb_ctx* ctx = net->ctx;
    if (!use_graph) return run_all(net, x);
    if (!(net->exec && net->graph_x == x)) {
        // capture on the context's own stream (the launch stream may be the legacy default
        // stream, which cannot be captured)
        free_graph(net);
        cudaStream_t saved = ctx->stream;
        ctx->stream = ctx->own_stream;
        cudaError_t e = cudaStreamBeginCapture(ctx->own_stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) { ctx->stream = saved; return cuda_fail(e, "cudaStreamBeginCapture"); }
        // TB_PDL=1: each layer's kernel may start while the previous one drains (programmatic
        // dependent launch; set-up overlaps that tail, reads wait for all of it). Off by default:
        // measured on YOLOv3 at batch 8 it gains nothing on the tensor-core plans and costs the
        // FP32 plan ~7% (dependent CTAs held resident beside the multi-wave FP32 grids).
        static const bool pdl = getenv("TB_PDL") != nullptr && atoi(getenv("TB_PDL")) != 0;
        ctx->pdl = pdl ? 1 : 0;
        int r = run_all(net, x);
        ctx->pdl = 0;
        cudaGraph_t g = nullptr;
        e = cudaStreamEndCapture(ctx->own_stream, &g);
        ctx->stream = saved;
        if (r != TB_OK) { if (g) cudaGraphDestroy(g); return r; }
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
        net->graph = g;
        e = cudaGraphInstantiate(&net->exec, g, 0);
        if (e != cudaSuccess) { free_graph(net); return cuda_fail(e, "cudaGraphInstantiate"); }
        net->graph_x = x;
        net->graph_launches = net->launches;
    }
    // fork from the launch stream, replay, join back
    TB_CHECK_CUDA(cudaEventRecord(ctx->fork, ctx->stream));
    TB_CHECK_CUDA(cudaStreamWaitEvent(ctx->own_stream, ctx->fork, 0));
    TB_CHECK_CUDA(cudaGraphLaunch(net->exec, ctx->own_stream));
    TB_CHECK_CUDA(cudaEventRecord(ctx->join, ctx->own_stream));
    TB_CHECK_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->join, 0));
    net->launches = net->graph_launches;
    return TB_OK;
}

int tb_net_profile(tb_net* net, const float* x, double* ms_out) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (!net->ctx) return fail(TB_ERR_STATE, "net was created without a context (host-only)");
    TB_ENTER(net->ctx);
    if (!net->finalized) return fail(TB_ERR_STATE, "net not finalized");
    if (!x || !ms_out) return fail(TB_ERR_INVALID, "null argument");
    const int64_t n = (int64_t)net->layers.size();
    cudaStream_t s = net->ctx->stream;
    std::vector<cudaEvent_t> ev((size_t)n + 1);
    for (auto& e : ev) TB_CHECK_CUDA(cudaEventCreate(&e));
    int r = TB_OK;
    net->launches = 0;
    cudaEventRecord(ev[0], s);
    for (int64_t i = 0; i < n && r == TB_OK; ++i) {
        r = run_layer(net, i, x);
        cudaEventRecord(ev[i + 1], s);
    }
    cudaError_t e = cudaEventSynchronize(ev[n]);
    for (int64_t i = 0; i < n; ++i) {
        float ms = 0.f;
        if (r == TB_OK && e == cudaSuccess) cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
        ms_out[i] = ms;
    }
    for (auto& ee : ev) cudaEventDestroy(ee);
    if (r != TB_OK) return r;
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize");
    return TB_OK;
}

int tb_net_layer_output(tb_net* net, int64_t layer, const float** ptr, int64_t* count, int64_t* bs) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (!net->finalized) return fail(TB_ERR_STATE, "net not finalized");
    if (layer < 0 || layer >= (int64_t)net->layers.size()) return fail(TB_ERR_INVALID, "layer out of range");
    const Layer& L = *net->layers[layer];
    if (L.target != layer)
        return fail(TB_ERR_STATE, "layer %lld is fused into layer %lld; its raw output is not materialised",
                    (long long)layer, (long long)L.target);
    if (ptr) *ptr = L.out.ptr;
    if (count) *count = L.per_image();
    if (bs) *bs = L.out.bs;
    return TB_OK;
}

int tb_net_layer_layout(tb_net* net, int64_t layer, int64_t* pixel_stride) {
    if (!net || !pixel_stride) return fail(TB_ERR_INVALID, "null argument");
    if (!net->finalized) return fail(TB_ERR_STATE, "net not finalized");
    if (layer < 0 || layer >= (int64_t)net->layers.size()) return fail(TB_ERR_INVALID, "layer out of range");
    *pixel_stride = net->layers[layer]->out.ps;
    return TB_OK;
}

int tb_net_layer_count(tb_net* net, int64_t* count) {
    if (!net || !count) return fail(TB_ERR_INVALID, "null argument");
    *count = (int64_t)net->layers.size();
    return TB_OK;
}

int tb_net_launch_count(tb_net* net, int64_t* count) {
    if (!net || !count) return fail(TB_ERR_INVALID, "null argument");
    *count = net->launches;
    return TB_OK;
}

int tb_net_flops(tb_net* net, double* flops) {
    if (!net || !flops) return fail(TB_ERR_INVALID, "null argument");
    if (!net->finalized) return fail(TB_ERR_STATE, "net not finalized");
    *flops = net->flops;
    return TB_OK;
}

int tb_net_input_shape(tb_net* net, int64_t* batch, int64_t* channels, int64_t* height, int64_t* width) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (batch) *batch = net->batch;
    if (channels) *channels = net->c;
    if (height) *height = net->h;
    if (width) *width = net->w;
    return TB_OK;
}

int tb_net_layer_info(tb_net* net, int64_t layer, tb_layer_info* out) {
    if (!net || !out) return fail(TB_ERR_INVALID, "null argument");
    if (layer < 0 || layer >= (int64_t)net->layers.size()) return fail(TB_ERR_INVALID, "layer out of range");
    int r = infer_shapes(net);
    if (r != TB_OK) return r;
    const Layer& L = *net->layers[layer];
    tb_layer_info d{};
    d.type = L.type;
    d.c = L.c; d.h = L.h; d.w = L.w;
    d.out_c = L.oc; d.out_h = L.oh; d.out_w = L.ow;
    d.filters = L.filters; d.ksize = L.ksize; d.stride = L.stride; d.pad = L.pad;
    d.activation = L.act; d.batch_normalize = L.bn ? 1 : 0;
    d.from = L.from;
    d.n_inputs = (int64_t)L.inputs.size();
    d.classes = L.classes; d.n = L.n; d.total_anchors = (int64_t)L.anchors.size() / 2;
    d.groups = L.groups;
    d.scale = L.type == TB_LAYER_UPSAMPLE ? L.up_scale
            : L.type == TB_LAYER_YOLO     ? L.scale_xy
            : L.type == TB_LAYER_SOFTMAX  ? L.temperature : 0.0f;
    d.weights_count = (int64_t)L.weights.size();
    *out = d;
    return TB_OK;
}

int tb_net_layer_param(tb_net* net, int64_t layer, int64_t which, void* dst, int64_t capacity,
                       int64_t* count) {
    if (!net) return fail(TB_ERR_INVALID, "null net");
    if (layer < 0 || layer >= (int64_t)net->layers.size()) return fail(TB_ERR_INVALID, "layer out of range");
    const Layer& L = *net->layers[layer];
    const void* src = nullptr;
    int64_t n = 0, esz = 4;
    switch (which) {
    case TB_PARAM_WEIGHTS:       src = L.weights.data(); n = (int64_t)L.weights.size(); break;
    case TB_PARAM_BIASES:        src = L.biases.data();  n = (int64_t)L.biases.size();  break;
    case TB_PARAM_SCALES:        src = L.scales.data();  n = L.bn ? (int64_t)L.scales.size() : 0; break;
    case TB_PARAM_ROLLING_MEAN:  src = L.mean.data();    n = L.bn ? (int64_t)L.mean.size() : 0;   break;
    case TB_PARAM_ROLLING_VAR:   src = L.var.data();     n = L.bn ? (int64_t)L.var.size() : 0;    break;
    case TB_PARAM_ROUTE_INPUTS:  src = L.inputs.data();  n = (int64_t)L.inputs.size(); esz = 8; break;
    case TB_PARAM_YOLO_MASK:     src = L.mask.data();    n = (int64_t)L.mask.size();   esz = 8; break;
    case TB_PARAM_YOLO_ANCHORS:  src = L.anchors.data(); n = (int64_t)L.anchors.size(); break;
    default: return fail(TB_ERR_INVALID, "unknown parameter %lld", (long long)which);
    }
    if (count) *count = n;
    if (!dst) return TB_OK;
    if (capacity < n) return fail(TB_ERR_INVALID, "parameter holds %lld elements, capacity %lld",
                                  (long long)n, (long long)capacity);
    if (n) std::memcpy(dst, src, (size_t)(n * esz));
    return TB_OK;
}

}  // extern "C"
