// yolo_detect.cu -- GPU detection extraction: TYoloLayer.getDetections + getBox + correctBoxes
// (source/nyololayer.pas:105-122, 399-498) for every yolo head and image, compacted on the
// device in the reference's order (heads in layer order, location i ascending, anchor minor;
// source/nnet.pas:647-653).  The reference pulls every head to the host and scans it there.
#include "common.cuh"

#include <cstring>
#include <mutex>
#include <vector>

using namespace tbi;

namespace {

constexpr int MAX_HEADS = 8;
constexpr int MAX_ANCH = 16;

struct HeadDev {
    const float* out;
    int n, classes, h, w;
    float aw[MAX_ANCH], ah[MAX_ANCH];
    int new_coords;
};

struct DetectArgs {
    HeadDev heads[MAX_HEADS];
    int n_heads;
    int img_w, img_h, net_w, net_h;
    int relative, letter;
    float thresh;
    long long capacity;
    float deltaw, deltah, ratiow, ratioh;
};

__device__ __forceinline__ long long head_outputs(const HeadDev& hd) {
    return (long long)hd.n * (hd.classes + 5) * hd.h * hd.w;
}

// counts[b*n_heads + h] = number of candidates with objectness > thresh
__global__ void k_yolo_count(const DetectArgs a, int* __restrict__ counts) {
    const int hi = blockIdx.x, b = blockIdx.y;
    const HeadDev& hd = a.heads[hi];
    const int hw = hd.h * hd.w, L = hw * hd.n;
    const float* out = hd.out + b * head_outputs(hd);
    int c = 0;
    for (int q = threadIdx.x; q < L; q += blockDim.x) {
        int i = q / hd.n, an = q - i * hd.n;
        float obj = out[(long long)an * (hd.classes + 5) * hw + 4LL * hw + i];
        c += (obj > a.thresh) ? 1 : 0;
    }
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    __shared__ int ws[32];
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += ws[i];
        counts[b * a.n_heads + hi] = t;
    }
}

// Ordered compaction (block scan per 256-candidate chunk) + box decode + correctBoxes.
__global__ void __launch_bounds__(256) k_yolo_write(const DetectArgs a, const int* __restrict__ counts,
                                                   tb_detection* __restrict__ dets, float* __restrict__ prob,
                                                   int max_classes) {
    const int hi = blockIdx.x, b = blockIdx.y;
    const HeadDev& hd = a.heads[hi];
    const int hw = hd.h * hd.w, L = hw * hd.n;
    const float* out = hd.out + b * head_outputs(hd);
    long long base = 0;
    for (int j = 0; j < hi; ++j) base += counts[b * a.n_heads + j];
    __shared__ int warp_tot[8];
    __shared__ long long running;
    if (threadIdx.x == 0) running = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int q0 = 0; q0 < L; q0 += 256) {
        int q = q0 + threadIdx.x;
        int i = 0, an = 0;
        float obj = 0.f;
        bool hit = false;
        if (q < L) {
            i = q / hd.n;
            an = q - i * hd.n;
            obj = out[(long long)an * (hd.classes + 5) * hw + 4LL * hw + i];
            hit = obj > a.thresh;
        }
        unsigned bal = __ballot_sync(0xffffffffu, hit);
        int before = __popc(bal & ((1u << lane) - 1u));
        if (lane == 0) warp_tot[wid] = __popc(bal);
        __syncthreads();
        int woff = 0, tot = 0;
        for (int w2 = 0; w2 < 8; ++w2) {
            if (w2 < wid) woff += warp_tot[w2];
            tot += warp_tot[w2];
        }
        long long pos = base + running + woff + before;
        if (hit && pos < a.capacity) {
            const long long st = hw;
            const float* bx = out + (long long)an * (hd.classes + 5) * hw + i;
            int row = i / hd.w, col = i - row * hd.w;
            // getBox (:105-122)
            float x = (float)(((double)col + (double)bx[0]) / (double)hd.w);
            float y = (float)(((double)row + (double)bx[st]) / (double)hd.h);
            float w, h;
            if (hd.new_coords) {
                double tw = (double)bx[2 * st], th = (double)bx[3 * st];
                w = (float)(tw * tw * 4.0 * (double)hd.aw[an] / (double)a.net_w);
                h = (float)(th * th * 4.0 * (double)hd.ah[an] / (double)a.net_h);
            } else {
                w = (float)(exp((double)bx[2 * st]) * (double)hd.aw[an] / (double)a.net_w);
                h = (float)(exp((double)bx[3 * st]) * (double)hd.ah[an] / (double)a.net_h);
            }
            // correctBoxes (:452-498)
            x = (float)(((double)x - (double)a.deltaw / 2.0 / (double)a.net_w) / (double)a.ratiow);
            y = (float)(((double)y - (double)a.deltah / 2.0 / (double)a.net_h) / (double)a.ratioh);
            w = (float)((double)w * (1.0 / (double)a.ratiow));
            h = (float)((double)h * (1.0 / (double)a.ratioh));
            if (!a.relative) {
                x = x * (float)a.img_w;
                w = w * (float)a.img_w;
                y = y * (float)a.img_h;
                h = h * (float)a.img_h;
            }
            long long di = (long long)b * a.capacity + pos;
            tb_detection d;
            d.x = x; d.y = y; d.w = w; d.h = h;
            d.objectness = obj;
            d.batch = b; d.head = hi; d.index = i; d.anchor = an;
            d.reserved[0] = d.reserved[1] = d.reserved[2] = 0;
            dets[di] = d;
            if (prob) {
                float* pr = prob + di * max_classes;
                for (int j = 0; j < hd.classes; ++j) {
                    float p = __fmul_rn(obj, bx[(5LL + j) * st]);
                    pr[j] = (p > a.thresh) ? p : 0.0f;
                }
                for (int j = hd.classes; j < max_classes; ++j) pr[j] = 0.0f;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) running += tot;
        __syncthreads();
    }
}

}  // namespace

// per image: the detections found over all heads (may exceed the capacity)
__global__ void k_yolo_totals(const int* __restrict__ per_head, int n_heads, int batch, int64_t* __restrict__ out) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= batch) return;
    int64_t t = 0;
    for (int h = 0; h < n_heads; ++h) t += per_head[b * n_heads + h];
    out[b] = t;
}

static int yolo_detect_impl(tb_ctx* ctx, int64_t batch, int64_t n_heads, const tb_yolo_head* heads, int64_t img_w,
                            int64_t img_h, int64_t net_w, int64_t net_h, float thresh, int64_t relative,
                            int64_t letter, int64_t capacity, tb_detection* dets, float* prob, int64_t* counts_host,
                            int64_t* counts_dev);

extern "C" int tb_yolo_detect(tb_ctx* ctx, int64_t batch, int64_t n_heads, const tb_yolo_head* heads,
                              int64_t img_w, int64_t img_h, int64_t net_w, int64_t net_h, float thresh,
                              int64_t relative, int64_t letter, int64_t capacity, tb_detection* dets,
                              float* prob, int64_t* counts_host) {
    if (!counts_host) return fail(TB_ERR_INVALID, "yolo_detect: null counts");
    return yolo_detect_impl(ctx, batch, n_heads, heads, img_w, img_h, net_w, net_h, thresh, relative, letter,
                            capacity, dets, prob, counts_host, nullptr);
}

extern "C" int tb_yolo_detect_device(tb_ctx* ctx, int64_t batch, int64_t n_heads, const tb_yolo_head* heads,
                                     int64_t img_w, int64_t img_h, int64_t net_w, int64_t net_h, float thresh,
                                     int64_t relative, int64_t letter, int64_t capacity, tb_detection* dets,
                                     float* prob, int64_t* counts_dev) {
    if (!counts_dev) return fail(TB_ERR_INVALID, "yolo_detect: null counts");
    return yolo_detect_impl(ctx, batch, n_heads, heads, img_w, img_h, net_w, net_h, thresh, relative, letter,
                            capacity, dets, prob, nullptr, counts_dev);
}

static int yolo_detect_impl(tb_ctx* ctx, int64_t batch, int64_t n_heads, const tb_yolo_head* heads, int64_t img_w,
                            int64_t img_h, int64_t net_w, int64_t net_h, float thresh, int64_t relative,
                            int64_t letter, int64_t capacity, tb_detection* dets, float* prob, int64_t* counts_host,
                            int64_t* counts_dev) {
    TB_ENTER(ctx);
    if (batch < 0 || n_heads <= 0 || n_heads > MAX_HEADS || !heads || img_w <= 0 || img_h <= 0 ||
        net_w <= 0 || net_h <= 0 || capacity < 0 || (capacity > 0 && !dets))
        return fail(TB_ERR_INVALID, "yolo_detect: bad arguments (at most %d heads)", MAX_HEADS);
    if (batch == 0) return TB_OK;
    if (batch > 65535) return fail(TB_ERR_INVALID, "yolo_detect: batch too large");
    DetectArgs a;
    memset(&a, 0, sizeof(a));
    int max_classes = 0;
    for (int64_t h = 0; h < n_heads; ++h) {
        const tb_yolo_head& s = heads[h];
        if (!s.output || s.n <= 0 || s.n > MAX_ANCH || s.classes < 0 || s.h <= 0 || s.w <= 0 ||
            !s.mask_host || !s.anchors_host)
            return fail(TB_ERR_INVALID, "yolo_detect: bad head %lld", (long long)h);
        HeadDev& d = a.heads[h];
        d.out = s.output;
        d.n = (int)s.n; d.classes = (int)s.classes; d.h = (int)s.h; d.w = (int)s.w;
        d.new_coords = (int)s.new_coords;
        for (int64_t k = 0; k < s.n; ++k) {
            int64_t m = s.mask_host[k];
            if (m < 0) return fail(TB_ERR_INVALID, "yolo_detect: negative mask");
            d.aw[k] = s.anchors_host[2 * m];
            d.ah[k] = s.anchors_host[2 * m + 1];
        }
        if (s.classes > max_classes) max_classes = (int)s.classes;
    }
    a.n_heads = (int)n_heads;
    a.img_w = (int)img_w; a.img_h = (int)img_h; a.net_w = (int)net_w; a.net_h = (int)net_h;
    a.relative = relative ? 1 : 0;
    a.letter = letter ? 1 : 0;
    a.thresh = thresh;
    a.capacity = capacity;
    int64_t new_w, new_h;
    if (letter) {
        if ((double)net_w / (double)img_w < (double)net_h / (double)img_h) {
            new_w = net_w;
            new_h = (img_h * net_w) / img_w;
        } else {
            new_h = net_h;
            new_w = (img_w * net_h) / img_h;
        }
    } else {
        new_w = net_w;
        new_h = net_h;
    }
    a.deltaw = (float)(net_w - new_w);
    a.deltah = (float)(net_h - new_h);
    a.ratiow = (float)((double)new_w / (double)net_w);
    a.ratioh = (float)((double)new_h / (double)net_h);

    const int64_t ncounts = batch * n_heads;
    int r = ensure_workspace(ctx, sizeof(int) * (size_t)ncounts);
    if (r != TB_OK) return r;
    int* d_counts = reinterpret_cast<int*>(ctx->ws);
    dim3 grid((unsigned)n_heads, (unsigned)batch);
    k_yolo_count<<<grid, 256, 0, ctx->stream>>>(a, d_counts);
    r = check_launch("k_yolo_count");
    if (r != TB_OK) return r;
    if (capacity > 0) {
        k_yolo_write<<<grid, 256, 0, ctx->stream>>>(a, d_counts, dets, prob, max_classes);
        r = check_launch("k_yolo_write");
        if (r != TB_OK) return r;
    }
    if (counts_dev) {  // per-image totals stay on the device; nothing waits
        k_yolo_totals<<<(unsigned)ceil_div(batch, 128), 128, 0, ctx->stream>>>(d_counts, (int)n_heads, (int)batch,
                                                                              counts_dev);
        return check_launch("k_yolo_totals");
    }
    std::vector<int> hc((size_t)ncounts);
    TB_CHECK_CUDA(cudaMemcpyAsync(hc.data(), d_counts, sizeof(int) * (size_t)ncounts,
                                  cudaMemcpyDeviceToHost, ctx->stream));
    TB_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
    for (int64_t b = 0; b < batch; ++b) {
        int64_t t = 0;
        for (int64_t h = 0; h < n_heads; ++h) t += hc[(size_t)(b * n_heads + h)];
        counts_host[b] = t;
    }
    return TB_OK;
}

// ---------------------------------------------------------------------------------------
// Class-wise NMS: TDetectionsHelper.doNMSSort (source/ntypes.pas:1621-1649) on the device.
// One block per (class) and launch per image: the candidates of the class (objectness > 0,
// prob > 0) are sorted by probability, highest first, in shared memory (bitonic sort; equal
// probabilities in detection order), then walked in that order: a candidate that is still
// unsuppressed zeroes the class probability of every later candidate whose box IoU with it
// exceeds the threshold (the inner comparisons run in parallel, one barrier per candidate).
// The reference sorts the whole record array with an unstable quicksort that carries the
// previous class's order, so among exactly equal probabilities its order is the partition
// history's; this keeps the detection order for them.  It also leaves the records sorted by the
// last class; this leaves them in place.  Box IoU as box_iou (source/ntypes.pas:1059-1108).
// ---------------------------------------------------------------------------------------
namespace {

constexpr int NMS_THREADS = 256;
constexpr int NMS_MAX = 8192;  // detections per image one block can sort in shared memory

__device__ __forceinline__ float nms_overlap(float x1, float w1, float x2, float w2) {
    const float l1 = __fsub_rn(x1, w1 * 0.5f), l2 = __fsub_rn(x2, w2 * 0.5f);
    const float left = l1 > l2 ? l1 : l2;
    const float r1 = __fadd_rn(x1, w1 * 0.5f), r2 = __fadd_rn(x2, w2 * 0.5f);
    const float right = r1 < r2 ? r1 : r2;
    return __fsub_rn(right, left);
}

__device__ __forceinline__ float nms_iou(const tb_detection& a, const tb_detection& b) {
    const float w = nms_overlap(a.x, a.w, b.x, b.w);
    const float h = nms_overlap(a.y, a.h, b.y, b.h);
    const float i = (w < 0.0f || h < 0.0f) ? 0.0f : __fmul_rn(w, h);
    const float u = __fsub_rn(__fadd_rn(__fmul_rn(a.w, a.h), __fmul_rn(b.w, b.h)), i);
    if (i == 0.0f || u == 0.0f) return 0.0f;
    return __fdiv_rn(i, u);
}

// (ka, ia) comes before (kb, ib): higher probability first, then lower detection index
__device__ __forceinline__ bool nms_before(float ka, int ia, float kb, int ib) {
    return ka > kb || (ka == kb && ia < ib);
}

__global__ void __launch_bounds__(NMS_THREADS)
    k_yolo_nms(const tb_detection* __restrict__ dets, float* __restrict__ prob, int n, int classes, int P,
               float thresh) {
    extern __shared__ __align__(16) unsigned char nsm[];
    float* key = reinterpret_cast<float*>(nsm);
    int* idx = reinterpret_cast<int*>(key + P);
    unsigned char* supp = reinterpret_cast<unsigned char*>(idx + P);
    __shared__ int m_sh;
    const int k = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) m_sh = 0;
    __syncthreads();
    for (int j = tid; j < n; j += NMS_THREADS) {  // candidates, in any slot order (sorted below)
        const float pk = prob[(long long)j * classes + k];
        if (dets[j].objectness != 0.0f && pk != 0.0f) {
            const int s = atomicAdd(&m_sh, 1);
            key[s] = pk;
            idx[s] = j;
        }
    }
    __syncthreads();
    const int m = m_sh;
    if (m < 2) return;  // nothing to suppress
    int P2 = 2;
    while (P2 < m) P2 <<= 1;
    for (int s = m + tid; s < P2; s += NMS_THREADS) {
        key[s] = -1.0f;  // below every probability
        idx[s] = 0x7fffffff;
    }
    __syncthreads();
    for (int size = 2; size <= P2; size <<= 1) {  // bitonic sort into "before" order
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = tid; t < P2 / 2; t += NMS_THREADS) {
                const int lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
                const bool up = (lo & size) == 0;  // this run ends in "before" order
                const bool swap = up ? nms_before(key[hi], idx[hi], key[lo], idx[lo])
                                     : nms_before(key[lo], idx[lo], key[hi], idx[hi]);
                if (swap) {
                    const float tk = key[lo];
                    key[lo] = key[hi];
                    key[hi] = tk;
                    const int ti = idx[lo];
                    idx[lo] = idx[hi];
                    idx[hi] = ti;
                }
            }
            __syncthreads();
        }
    }
    for (int s = tid; s < m; s += NMS_THREADS) supp[s] = 0;
    __syncthreads();
    for (int i = 0; i < m - 1; ++i) {
        if (!supp[i]) {  // uniform: read after the barrier that ended the previous step
            const tb_detection a = dets[idx[i]];
            for (int j = i + 1 + tid; j < m; j += NMS_THREADS)
                if (nms_iou(a, dets[idx[j]]) > thresh) supp[j] = 1;
        }
        __syncthreads();
    }
    for (int s = tid; s < m; s += NMS_THREADS)
        if (supp[s]) prob[(long long)idx[s] * classes + k] = 0.0f;
}

}  // namespace

extern "C" int tb_yolo_nms(tb_ctx* ctx, int64_t batch, int64_t capacity, const int64_t* counts_host, int64_t classes,
                           float thresh, const tb_detection* dets, float* prob) {
    TB_ENTER(ctx);
    if (batch < 0 || capacity < 0 || classes <= 0 || (batch > 0 && !counts_host))
        return fail(TB_ERR_INVALID, "nms: bad arguments");
    if (batch == 0 || capacity == 0) return TB_OK;
    if (!dets || !prob) return fail(TB_ERR_INVALID, "nms: null detections or probabilities");
    if (classes > 65535) return fail(TB_ERR_UNSUPPORTED, "nms: more than 65535 classes");
    static std::mutex mu;
    static bool done[64] = {false};
    const int smem_max = NMS_MAX * 9;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !done[ctx->device]) {
            cudaError_t e = cudaFuncSetAttribute(k_yolo_nms, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(nms)");
            done[ctx->device] = true;
        }
    }
    for (int64_t b = 0; b < batch; ++b) {
        const int64_t n = counts_host[b] < capacity ? counts_host[b] : capacity;
        if (n < 0) return fail(TB_ERR_INVALID, "nms: negative count");
        if (n > NMS_MAX)
            return fail(TB_ERR_UNSUPPORTED, "nms: %lld detections in image %lld (at most %d)", (long long)n,
                        (long long)b, NMS_MAX);
        if (n < 2) continue;
        int P = 2;
        while (P < n) P <<= 1;
        k_yolo_nms<<<(unsigned)classes, NMS_THREADS, (size_t)P * 9, ctx->stream>>>(
            dets + b * capacity, prob + b * capacity * classes, (int)n, (int)classes, P, thresh);
        int r = check_launch("k_yolo_nms");
        if (r != TB_OK) return r;
    }
    return TB_OK;
}
