// oracle.cpp -- CPU restatement of the reference's darknet conv-forward inference path.
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
// leg (--impl reference / cpu_baseline) may load this library, and only as the checker or as
// the timed CPU baseline; the product (tensorium_b200/) never calls it.
//
// PARITY UNPINNED: the reference is FreePascal and cannot be compiled here, and it ships no
// tests, golden vectors or fixtures.  Every function below restates the cited Pascal code
// (paths relative to the reference project root); the known-answer tests in tests/ check the
// restatement against hand-derived results.
//
// Numeric conventions (FreePascal on x86-64, USE_AVX2 build):
//  * single-precision arithmetic on single operands (SSE), no FMA contraction, except where
//    the reference uses vfmadd231ps explicitly (saxpy_avx2, source/ntensors.pas:1308-1435);
//  * untyped real constants (0.1, 1, 0.5) and the System unit's exp/sqrt are evaluated in
//    double and rounded to single on assignment -- restated with explicit double arithmetic.
//
// Build: oracle/Makefile (g++ -O3 -mavx2 -mfma -fopenmp, no -ffast-math, -ffp-contract=off).

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#endif

extern "C" {

// ---------------------------------------------------------------------------------------
// activations (source/nactivation.pas)
// ---------------------------------------------------------------------------------------
enum {
    acLOGISTIC = 0, acRELU = 1, acRELU6 = 2, acRELIE = 3, acLINEAR = 4, acRAMP = 5, acTANH = 6,
    acPLSE = 7, acREVLEAKY = 8, acLEAKY = 9, acELU = 10, acLOGGY = 11, acHARDTAN = 13,
    acLHTAN = 14, acSELU = 15
};

static inline float act_scalar(float x, int a) {
    switch (a) {
    case acLOGISTIC:  // logistic_activate :293-297, 1/(1+exp(-x)) with ValReal exp
        return (float)(1.0 / (1.0 + std::exp(-(double)x)));
    case acRELU:  // relu_activate: x*SizeInt(x>0)
        return x > 0 ? x : x * 0.0f;
    case acRELU6:
        return (x > 0 && x <= 6) ? x : x * 0.0f;
    case acRELIE:
        return x > 0 ? x : (float)(0.01 * (double)x);
    case acLINEAR:
        return x;
    case acRAMP:  // x*SizeInt(x>0)+0.1*x
        return (float)((double)(x > 0 ? x : x * 0.0f) + 0.1 * (double)x);
    case acTANH: {
        double px = std::exp((double)x), nx = std::exp(-(double)x);
        float fpx = (float)px, fnx = (float)nx;  // px, nx are single variables
        return (fpx - fnx) / (fpx + fnx);
    }
    case acPLSE:
        if (x < -4) return (float)(0.01 * ((double)x + 4));
        if (x > 4) return (float)(0.01 * ((double)x - 4) + 1);
        return (float)(0.125 * (double)x + 0.5);
    case acREVLEAKY:
    case acLEAKY:  // activate_array :555-566 -> leaky_array (:234-267, the USE_AVX2 build every
                   // sample project defines): x < 0 -> x * f with f: single = 0.1 (vmulps)
        return x < 0 ? x * 0.1f : x;
    case acELU:
        return (float)((x >= 0 ? (double)x : 0.0) + (x < 0 ? std::exp((double)x) - 1.0 : 0.0));
    case acLOGGY:
        return (float)(2.0 / (1.0 + std::exp(-(double)x)) - 1.0);
    case acHARDTAN:
        if (x < -1) return -1.0f;
        if (x > 1) return 1.0f;
        return x;
    case acLHTAN:
        if (x < 0) return (float)(0.001 * (double)x);
        if (x > 1) return (float)(0.001 * ((double)x - 1) + 1);
        return x;
    case acSELU:
        return (float)((x >= 0 ? 1.0507 * (double)x : 0.0) +
                       (x < 0 ? 1.0507 * 1.6732 * (std::exp((double)x) - 1.0) : 0.0));
    default:
        return x;
    }
}

// activate_array (source/nactivation.pas:508-621), scalar forms.
void or_activate(int64_t n, float* x, int64_t act) {
    if (act == acLINEAR) return;
    for (int64_t i = 0; i < n; ++i) x[i] = act_scalar(x[i], (int)act);
}

// ---------------------------------------------------------------------------------------
// im2col: sim2Col (source/ntensors.pas:11415-11470). col[c][kh][kw][oh][ow].
// ---------------------------------------------------------------------------------------
void or_im2col(int64_t channels, int64_t height, int64_t width, int64_t kh, int64_t kw,
               int64_t pad_h, int64_t pad_w, int64_t stride_y, int64_t stride_x,
               int64_t dil_y, int64_t dil_x, const float* im, float* col) {
    const int64_t out_w = (width + 2 * pad_w - (dil_x * (kw - 1) + 1)) / stride_x + 1;
    const int64_t out_h = (height + 2 * pad_h - (dil_y * (kh - 1) + 1)) / stride_y + 1;
    const int64_t channel_size = height * width, out_size = out_w * out_h;
#pragma omp parallel for schedule(static) if (channels >= 8)
    for (int64_t ch = 0; ch < channels; ++ch) {
        const float* d_im = im + channel_size * ch;
        float* d_col = col + kh * kw * out_size * ch;
        for (int64_t r = 0; r < kh; ++r)
            for (int64_t s = 0; s < kw; ++s) {
                int64_t in_row = -pad_h + r * dil_y;
                for (int64_t oy = 0; oy < out_h; ++oy) {
                    if ((uint64_t)in_row < (uint64_t)height) {
                        int64_t in_col = -pad_w + s * dil_x;
                        for (int64_t ox = 0; ox < out_w; ++ox, in_col += stride_x)
                            d_col[ox] = ((uint64_t)in_col < (uint64_t)width)
                                            ? d_im[in_row * width + in_col] : 0.0f;
                    } else {
                        for (int64_t ox = 0; ox < out_w; ++ox) d_col[ox] = 0.0f;
                    }
                    d_col += out_w;
                    in_row += stride_y;
                }
            }
    }
}

// ---------------------------------------------------------------------------------------
// SGEMM NN: cblas_sgemm -> sgemm_nn -> s_nn -> saxpy_avx2 (source/ntensors.pas:2231-2286,
// 2136-2157, 2061-2133, 1308-1435). C = beta*C (when beta != 1), then for every row i and
// k = 0..K-1 ascending: C[i,:] = fma(alpha*A[i,k], B[k,:], C[i,:]).  Rows are split across
// threads in contiguous chunks (TOPool.&For, source/steroids.pas:606-641); the element
// results do not depend on the split or on vector width.
// ---------------------------------------------------------------------------------------
static inline void saxpy_fma(int64_t n, float a, const float* x, float* y) {
    int64_t j = 0;
#if defined(__AVX2__) && defined(__FMA__)
    const __m256 va = _mm256_set1_ps(a);
    for (; j + 8 <= n; j += 8)
        _mm256_storeu_ps(y + j, _mm256_fmadd_ps(va, _mm256_loadu_ps(x + j), _mm256_loadu_ps(y + j)));
#endif
    for (; j < n; ++j) y[j] = std::fmaf(a, x[j], y[j]);
}

void or_sgemm_nn(int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
                 const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
        float* c = C + i * ldc;
        if (beta != 1.0f)
            for (int64_t j = 0; j < N; ++j) c[j] = c[j] * beta;  // mulvs
        const float* a = A + i * lda;
        for (int64_t k = 0; k < K; ++k) saxpy_fma(N, alpha * a[k], B + k * ldb, c);
    }
}

// SGEMM NT: sgemm_nt -> s_nt (source/ntensors.pas:1957-2005): C[i,j] = beta*C[i,j] +
// alpha*sdot(A_i, B_j).  sdot is sdot_avx2 (source/ntensors.pas:1233-1306, SIMD_REGS = 8) in the
// USE_AVX2 build every sample project defines: eight lane sums, lane l taking k = l, l+8, ...
// with one fused multiply-add each (the masked tail block adds its k = 8*floor(K/8) + l to lane
// l), then lanes l and l+4 are added (vextractf128 + vaddps) and the four sums reduced by two
// vhaddps: ((s0+s1) + (s2+s3)).
// ---------------------------------------------------------------------------------------
static inline float sdot_avx2_order(int64_t K, const float* a, const float* b) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t k = 0; k < K; ++k) lane[k & 7] = std::fmaf(a[k], b[k], lane[k & 7]);
    float t[4];
    for (int l = 0; l < 4; ++l) t[l] = lane[l] + lane[l + 4];
    return (t[0] + t[1]) + (t[2] + t[3]);
}

void or_sgemm_nt(int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
                 const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
        float* c = C + i * ldc;
        if (beta != 1.0f)
            for (int64_t j = 0; j < N; ++j) c[j] = c[j] * beta;
        for (int64_t j = 0; j < N; ++j) {
            const float s = alpha * sdot_avx2_order(K, A + i * lda, B + j * ldb);
            c[j] = c[j] + s;
        }
    }
}

// SGEMM TN: sgemm_tn -> s_tn (source/ntensors.pas:2007-2040): per row i and k ascending,
// saxpy(N, alpha*A[k*lda + i], B_k, C_i) -- one FMA per k, as s_nn.
void or_sgemm_tn(int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
                 const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
        float* c = C + i * ldc;
        if (beta != 1.0f)
            for (int64_t j = 0; j < N; ++j) c[j] = c[j] * beta;
        for (int64_t k = 0; k < K; ++k) saxpy_fma(N, alpha * A[k * lda + i], B + k * ldb, c);
    }
}

// SGEMM TT: sgemm_tt -> s_tt (source/ntensors.pas:2159-2183): sum := sum + ALPHA*A[i + kk*lda]*
// B[kk + j*ldb] (single products, left to right), C += sum.
void or_sgemm_tt(int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
                 const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
        float* c = C + i * ldc;
        if (beta != 1.0f)
            for (int64_t j = 0; j < N; ++j) c[j] = c[j] * beta;
        for (int64_t j = 0; j < N; ++j) {
            float sum = 0.0f;
            for (int64_t k = 0; k < K; ++k) {
                const float t = alpha * A[i + k * lda];
                sum = sum + t * B[k + j * ldb];
            }
            c[j] = c[j] + sum;
        }
    }
}

// ---------------------------------------------------------------------------------------
// Batchnorm fold: TBaseConvolutionalLayer.fuseBatchNorm (source/nConvolutionLayer.pas:
// 102-126): precomputed := scales/sqrt(max(var, sEPSILON)) (ValReal sqrt and divide, stored
// as single); biases -= mean*precomputed; weights *= precomputed.
// ---------------------------------------------------------------------------------------
void or_fuse_bn(int64_t filters, int64_t filter_size, float* weights, float* biases,
                const float* scales, const float* mean, const float* variance) {
    const float eps = 0.000001f;  // sEPSILON, source/ntensors.pas:95
    for (int64_t f = 0; f < filters; ++f) {
        float v = std::max(variance[f], eps);
        float pre = (float)((double)scales[f] / std::sqrt((double)v));
        biases[f] = biases[f] - mean[f] * pre;
        for (int64_t i = 0; i < filter_size; ++i) weights[f * filter_size + i] *= pre;
    }
}

// ---------------------------------------------------------------------------------------
// Conv forward: TConvolutionalLayer.forward (source/nConvolutionLayer.pas:457-569) ->
// TTensor.Conv2D (source/ntensors.pas:8252-8349) per image: im2col (skipped for 1x1 /
// stride 1 / dilation 1), gemm NN with beta = 0, then either batchNorm (inference:
// blockNormalize -> forwardScale -> forwardBias, source/nbaselayer.pas:336-370,
// source/ntensors.pas:4357-4382, 8693-8718, 7687-7727) or forwardBias, then activation.
// bn_mean == NULL selects the bias-only path.  bias may be NULL (no bias).
// ---------------------------------------------------------------------------------------
void or_conv2d_fwd(int64_t batch, int64_t channels, int64_t height, int64_t width,
                   int64_t filters, int64_t kh, int64_t kw, int64_t stride_y, int64_t stride_x,
                   int64_t pad_y, int64_t pad_x, int64_t dil_y, int64_t dil_x, const float* x,
                   const float* w, const float* bias, const float* bn_scale,
                   const float* bn_mean, const float* bn_var, int64_t activation, float* y) {
    if (dil_y <= 0) dil_y = 1;
    if (dil_x <= 0) dil_x = 1;
    const int64_t oh = (height + 2 * pad_y - (dil_y * (kh - 1) + 1)) / stride_y + 1;
    const int64_t ow = (width + 2 * pad_x - (dil_x * (kw - 1) + 1)) / stride_x + 1;
    const int64_t K = channels * kh * kw, N = oh * ow;
    const bool direct = (kh == 1 && kw == 1 && stride_x == 1 && stride_y == 1 &&
                         dil_x == 1 && dil_y == 1 && pad_x == 0 && pad_y == 0);
    std::vector<float> col;
    if (!direct) col.resize((size_t)(K * N));
    for (int64_t b = 0; b < batch; ++b) {
        const float* xb = x + b * channels * height * width;
        float* yb = y + b * filters * N;
        const float* B;
        if (direct) {
            B = xb;
        } else {
            or_im2col(channels, height, width, kh, kw, pad_y, pad_x, stride_y, stride_x, dil_y,
                      dil_x, xb, col.data());
            B = col.data();
        }
        or_sgemm_nn(filters, N, K, 1.0f, w, K, B, N, 0.0f, yb, N);
        for (int64_t f = 0; f < filters; ++f) {
            float* o = yb + f * N;
            if (bn_mean) {
                // _snormblkvv scalar: d := sqrt(variance); snormvss(o, mean, max(d, eps))
                float d = (float)std::sqrt((double)bn_var[f]);
                float sd = std::max(d, 0.000001f);
                float sc = bn_scale ? bn_scale[f] : 1.0f;
                float bi = bias ? bias[f] : 0.0f;
                for (int64_t j = 0; j < N; ++j) {
                    float t = (o[j] - bn_mean[f]) / sd;
                    t = t * sc;
                    o[j] = t + bi;
                }
            } else if (bias) {
                for (int64_t j = 0; j < N; ++j) o[j] = o[j] + bias[f];
            }
        }
        or_activate(filters * N, yb, activation);
    }
}

// ---------------------------------------------------------------------------------------
// Maxpool: maxpoolMP / forwardMaxPool (source/nMaxPoolLayer.pas:265-463). Offsets
// -padding div 2, out-of-image = -MaxSingle, strict '>', argmax = flat input index.
// ---------------------------------------------------------------------------------------
void or_maxpool(int64_t batch, int64_t c, int64_t h, int64_t w, int64_t size, int64_t stride_x,
                int64_t stride_y, int64_t padding, const float* src, float* dst,
                int64_t* indexes) {
    const int64_t out_h = (h + padding - size) / stride_y + 1;
    const int64_t out_w = (w + padding - size) / stride_x + 1;
    const int64_t w_off = -(padding / 2), h_off = -(padding / 2);
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t k = 0; k < c; ++k)
            for (int64_t i = 0; i < out_h; ++i)
                for (int64_t j = 0; j < out_w; ++j) {
                    int64_t out_index = j + out_w * (i + out_h * (k + c * b));
                    float mx = -FLT_MAX;
                    int64_t max_i = -1;
                    for (int64_t n = 0; n < size; ++n)
                        for (int64_t m = 0; m < size; ++m) {
                            int64_t cur_h = h_off + i * stride_y + n;
                            int64_t cur_w = w_off + j * stride_x + m;
                            int64_t index = cur_w + w * (cur_h + h * (k + b * c));
                            float val = (cur_h >= 0 && cur_h < h && cur_w >= 0 && cur_w < w)
                                            ? src[index] : -FLT_MAX;
                            if (val > mx) {
                                max_i = index;
                                mx = val;
                            }
                        }
                    dst[out_index] = mx;
                    if (indexes) indexes[out_index] = max_i;
                }
}

// Upsample: upsample() forward (source/nupsamplelayer.pas:83-113).
void or_upsample(int64_t batch, int64_t c, int64_t h, int64_t w, int64_t stride, float scale,
                 const float* in, float* out) {
    for (int64_t cc = 0; cc < batch * c; ++cc)
        for (int64_t y = 0; y < h * stride; ++y)
            for (int64_t x = 0; x < w * stride; ++x) {
                int64_t in_index = (cc * h + y / stride) * w + x / stride;
                int64_t out_index = (cc * h * stride + y) * stride * w + x;
                out[out_index] = scale * in[in_index];
            }
}

// Route, reference form: TTensor.concat (source/ntensors.pas:12045-12061), whole inputs
// back to back.  sizes[i] = total elements of input i.
void or_concat(int64_t n_inputs, const float* const* inputs, const int64_t* sizes, float* out) {
    int64_t off = 0;
    for (int64_t i = 0; i < n_inputs; ++i) {
        std::memcpy(out + off, inputs[i], sizeof(float) * (size_t)sizes[i]);
        off += sizes[i];
    }
}

// Shortcut: TAddLayer.forward single-input branch (source/naddlayer.pas:696-699), then
// activate().
void or_shortcut(int64_t n, const float* a, const float* b, float* out, int64_t act) {
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
    or_activate(n, out, act);
}

// YOLO forward: TYoloLayer.forward (source/nyololayer.pas:786-825) for newCoords = false.
void or_yolo_fwd(int64_t batch, int64_t n, int64_t classes, int64_t h, int64_t w,
                 const float* in, float* out, float scale_xy) {
    const int64_t outputs = n * (classes + 5) * h * w;
    std::memcpy(out, in, sizeof(float) * (size_t)(batch * outputs));
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t a = 0; a < n; ++a) {
            // entryIndex (:97-103): aBatch*outputs + _n*(classes+5)*w*h + entry*w*h + loc
            float* box = out + b * outputs + a * (classes + 5) * w * h;
            or_activate(2 * w * h, box, acLOGISTIC);
            or_activate((1 + classes) * w * h, box + 4 * w * h, acLOGISTIC);
            if (scale_xy != 1.0f) {
                // FusedMultiplyAdd(scaleXY, 0.5*(1-scaleXY)): v*s + b on 2*w*h values
                float bb = (float)(0.5 * (1.0 - (double)scale_xy));
                for (int64_t i = 0; i < 2 * w * h; ++i) box[i] = box[i] * scale_xy + bb;
            }
        }
}

// Detections: getDetections + getBox + correctBoxes (source/nyololayer.pas:105-122,
// 399-498).  Writes up to `capacity` records: box[5] = {x,y,w,h,objectness}, meta[3] =
// {index i, anchor n, det id}, prob[classes]. Returns the number found.
int64_t or_yolo_detections(const float* out, int64_t batch_index, int64_t n, int64_t classes,
                           int64_t h, int64_t w, const int64_t* mask, const float* anchors,
                           int64_t img_w, int64_t img_h, int64_t net_w, int64_t net_h,
                           float thresh, int64_t relative, int64_t letter, int64_t capacity,
                           float* boxes, int64_t* meta, float* probs) {
    const int64_t outputs = n * (classes + 5) * h * w;
    auto entry = [&](int64_t location, int64_t e) {
        int64_t nn = location / (w * h), loc = location % (w * h);
        return batch_index * outputs + nn * (classes + 5) * w * h + e * w * h + loc;
    };
    int64_t count = 0;
    for (int64_t i = 0; i < w * h; ++i) {
        int64_t row = i / w, col = i % w;
        for (int64_t a = 0; a < n; ++a) {
            float obj = out[entry(a * w * h + i, 4)];
            if (!(obj > thresh)) continue;
            if (count < capacity) {
                int64_t bi = entry(a * w * h + i, 0);
                int64_t st = w * h;
                int64_t n2 = 2 * mask[a];
                float bx = (float)(((double)col + (double)out[bi]) / (double)w);
                float by = (float)(((double)row + (double)out[bi + st]) / (double)h);
                float bw = (float)(std::exp((double)out[bi + 2 * st]) * (double)anchors[n2] / (double)net_w);
                float bh = (float)(std::exp((double)out[bi + 3 * st]) * (double)anchors[n2 + 1] / (double)net_h);
                float* B = boxes + count * 5;
                B[0] = bx; B[1] = by; B[2] = bw; B[3] = bh; B[4] = obj;
                meta[count * 3 + 0] = i;
                meta[count * 3 + 1] = a;
                meta[count * 3 + 2] = count;
                for (int64_t j = 0; j < classes; ++j) {
                    float p = obj * out[entry(a * w * h + i, 5 + j)];
                    probs[count * classes + j] = (p > thresh) ? p : 0.0f;
                }
            }
            ++count;
        }
    }
    // correctBoxes (:452-498)
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
    float deltaw = (float)(net_w - new_w), deltah = (float)(net_h - new_h);
    float ratiow = (float)((double)new_w / (double)net_w);
    float ratioh = (float)((double)new_h / (double)net_h);
    int64_t written = std::min(count, capacity);
    for (int64_t k = 0; k < written; ++k) {
        float* B = boxes + k * 5;
        B[0] = (float)(((double)B[0] - (double)deltaw / 2.0 / (double)net_w) / (double)ratiow);
        B[1] = (float)(((double)B[1] - (double)deltah / 2.0 / (double)net_h) / (double)ratioh);
        B[2] = (float)((double)B[2] * (1.0 / (double)ratiow));
        B[3] = (float)((double)B[3] * (1.0 / (double)ratioh));
        if (!relative) {
            B[0] = B[0] * (float)img_w;
            B[2] = B[2] * (float)img_w;
            B[1] = B[1] * (float)img_h;
            B[3] = B[3] * (float)img_h;
        }
    }
    return count;
}

// Connected: TConnectedLayer.forward (source/nconnectedlayer.pas:157-184) without BN:
// gemm(NoTrans, Trans, batch, outputs, inputs, beta = 0) + forwardBias + activation.
void or_connected(int64_t batch, int64_t inputs, int64_t outputs, const float* x, const float* w,
                  const float* bias, int64_t act, float* y) {
    or_sgemm_nt(batch, outputs, inputs, 1.0f, x, inputs, w, inputs, 0.0f, y, outputs);
    if (bias)
        for (int64_t b = 0; b < batch; ++b)
            for (int64_t o = 0; o < outputs; ++o) y[b * outputs + o] = y[b * outputs + o] + bias[o];
    or_activate(batch * outputs, y, act);
}

// Softmax: softmax / softmaxBatch (source/nsoftmaxlayer.pas:83-137), stride 1.
void or_softmax(int64_t batch, int64_t inputs, int64_t groups, float temp, const float* x,
                float* y) {
    const int64_t n = inputs / groups;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t g = 0; g < groups; ++g) {
            const float* in = x + b * inputs + g * n;
            float* out = y + b * inputs + g * n;
            if (n == 0) continue;
            float largest = in[0];
            for (int64_t i = 1; i < n; ++i)
                if (in[i] > largest) largest = in[i];
            float sum = 0.0f;
            for (int64_t i = 0; i < n; ++i) {
                float e = (float)std::exp((double)((in[i] - largest) / temp));
                sum = sum + e;
                out[i] = e;
            }
            for (int64_t i = 0; i < n; ++i) out[i] = out[i] / sum;
        }
}

// Global average pool: TAvgPoolLayer.forward (source/navgpoollayer.pas:60-84): Sum(1, h*w,
// offset) / (h*w).  TTensor<single>.sumv is vsSumI (source/ntensors.pas:3624-3634), which on an
// AVX2 CPU with unit stride is vssum_avx2 (:3592-3620): eight lane sums over the whole blocks of
// 8 (vaddps), lanes l and l+4 added, two haddps ((s0+s1) + (s2+s3)), then the N mod 8 tail added
// one by one.
static inline float vssum_avx2_order(int64_t n, const float* a) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int64_t nb = n / 8 * 8;
    for (int64_t k = 0; k < nb; ++k) lane[k & 7] = lane[k & 7] + a[k];
    float t[4];
    for (int l = 0; l < 4; ++l) t[l] = lane[l] + lane[l + 4];
    float s = (t[0] + t[1]) + (t[2] + t[3]);
    for (int64_t k = nb; k < n; ++k) s = s + a[k];
    return s;
}

void or_avgpool(int64_t batch, int64_t c, int64_t h, int64_t w, const float* x, float* y) {
    const int64_t im = h * w;
    for (int64_t i = 0; i < batch * c; ++i) y[i] = vssum_avx2_order(im, x + i * im) / (float)im;
}

// ---------------------------------------------------------------------------------------
// XNOR conv (source/nxnorconvolutionlayer.pas).  binarize_weights (:95-113) gives the
// per-filter mean = (sum |w|)/size, sequential fp32 sum.  The popcount GEMM
// gemm_nn_custom_bin_mean_transposed (:179-205) computes, per output,
// (2*count - K)*mean where count = number of equal sign bits over the K = c*k*k im2col
// positions; input bit = x > 0 (threshold :793-794), weight bit = w > 0, and a padding
// position is bit 0 (im2col_cpu_custom_bin :232-316 never sets it).  pad_mode 1 instead
// drops padding positions (float fallback :860-868 with zero padding):
//   value = (#equal - #different over valid positions) * mean.
// ---------------------------------------------------------------------------------------
void or_xnor_mean(int64_t filters, int64_t size, const float* w, float* mean) {
    for (int64_t f = 0; f < filters; ++f) {
        float m = 0.0f;
        for (int64_t i = 0; i < size; ++i) m = m + std::fabs(w[f * size + i]);
        mean[f] = m / (float)size;
    }
}

void or_xnor_conv(int64_t batch, int64_t c, int64_t h, int64_t w, int64_t filters, int64_t ksize,
                  int64_t stride, int64_t pad, int64_t pad_mode, const float* x,
                  const float* weights, const float* mean, int32_t* counts, float* y) {
    const int64_t oh = (h + 2 * pad - ksize) / stride + 1;
    const int64_t ow = (w + 2 * pad - ksize) / stride + 1;
    const int64_t K = c * ksize * ksize;
    const int64_t words = (K + 63) / 64;
    std::vector<uint64_t> wb((size_t)(filters * words), 0);
    for (int64_t f = 0; f < filters; ++f)
        for (int64_t k = 0; k < K; ++k)
            if (weights[f * K + k] > 0) wb[f * words + k / 64] |= 1ull << (k % 64);
#pragma omp parallel for schedule(static)
    for (int64_t bp = 0; bp < batch * oh * ow; ++bp) {
        std::vector<uint64_t> xb((size_t)words), vb((size_t)words);
        int64_t b = bp / (oh * ow), p = bp % (oh * ow), oy = p / ow, ox = p % ow;
        std::fill(xb.begin(), xb.end(), 0);
        std::fill(vb.begin(), vb.end(), 0);
        int64_t nvalid = 0;
        for (int64_t ch = 0; ch < c; ++ch)
            for (int64_t r = 0; r < ksize; ++r)
                for (int64_t s = 0; s < ksize; ++s) {
                    int64_t k = (ch * ksize + r) * ksize + s;
                    int64_t iy = oy * stride - pad + r, ix = ox * stride - pad + s;
                    if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
                        vb[k / 64] |= 1ull << (k % 64);
                        ++nvalid;
                        if (x[((b * c + ch) * h + iy) * w + ix] > 0) xb[k / 64] |= 1ull << (k % 64);
                    }
                }
        for (int64_t f = 0; f < filters; ++f) {
            int64_t count = 0, diff_valid = 0;
            for (int64_t q = 0; q < words; ++q) {
                uint64_t nx = ~(wb[f * words + q] ^ xb[q]);
                int64_t tmp = __builtin_popcountll(nx);
                if (K - q * 64 < 64) tmp -= 64 - (K - q * 64);  // tail correction (:197-198)
                count += tmp;
                diff_valid += __builtin_popcountll((wb[f * words + q] ^ xb[q]) & vb[q]);
            }
            int64_t v;
            if (pad_mode == 0) v = 2 * count - K;
            else v = (nvalid - diff_valid) - diff_valid;
            int64_t oi = (b * filters + f) * oh * ow + p;
            if (counts) counts[oi] = (int32_t)v;
            y[oi] = (float)v * mean[f];
        }
    }
}


// ---- NMS: TDetectionsHelper.doNMSSort (source/ntypes.pas:1621-1649), with box_iou
// (source/ntypes.pas:1059-1108), TDetectionsHelper.Comparer (:1554-1566) and
// TTools<T>.QuickSort (source/ntensors.pas:2483-2526). The record array is represented by a
// permutation of detection indices: QuickSort swaps records, the comparator reads prob /
// objectness through them, so swapping indices is the same algorithm. Output: probs (in the
// original detection order) with the suppressed (detection, class) entries zeroed; order
// receives the final record order (the reference leaves the array in that order).
static float nms_overlap(float x1, float w1, float x2, float w2) {
    const float l1 = x1 - w1 / 2.0f, l2 = x2 - w2 / 2.0f;
    const float left = (l1 > l2) ? l1 : l2;
    const float r1 = x1 + w1 / 2.0f, r2 = x2 + w2 / 2.0f;
    const float right = (r1 < r2) ? r1 : r2;
    return right - left;
}

static float nms_iou(const float* a, const float* b) {
    const float w = nms_overlap(a[0], a[2], b[0], b[2]);
    const float h = nms_overlap(a[1], a[3], b[1], b[3]);
    const float i = (w < 0.0f || h < 0.0f) ? 0.0f : w * h;
    const float i2 = i;  // box_union recomputes the same intersection
    const float u = a[2] * a[3] + b[2] * b[3] - i2;
    if (i == 0.0f || u == 0.0f) return 0.0f;
    return i / u;
}

struct NmsCtx {
    const float* probs;
    const float* obj;
    int64_t classes;
    int64_t sort_class;
};

// Comparer: 1 when a sorts after b (smaller prob / objectness), -1 before, 0 equal
static int nms_cmp(const NmsCtx& c, int64_t a, int64_t b) {
    float diff;
    if (c.sort_class >= 0)
        diff = c.probs[a * c.classes + c.sort_class] - c.probs[b * c.classes + c.sort_class];
    else
        diff = c.obj[a] - c.obj[b];
    if (diff < 0) return 1;
    if (diff > 0) return -1;
    return 0;
}

static void nms_quicksort(const NmsCtx& c, int64_t* arr, int64_t L, int64_t R) {
    do {
        int64_t I = L, J = R;
        const int64_t P = arr[(L + R) >> 1];
        do {
            while (I <= R && nms_cmp(c, P, arr[I]) > 0) ++I;
            while (J >= 0 && nms_cmp(c, P, arr[J]) < 0) --J;
            if (I <= J) {
                const int64_t q = arr[I];
                arr[I] = arr[J];
                arr[J] = q;
                ++I;
                --J;
            }
        } while (I <= J);
        if (J - L < R - I) {
            if (L < J) nms_quicksort(c, arr, L, J);
            L = I;
        } else {
            if (I < R) nms_quicksort(c, arr, I, R);
            R = J;
        }
    } while (L < R);
}

void or_nms_sort(int64_t n, int64_t classes, const float* boxes, const float* objectness, float* probs,
                 float thresh, int64_t* order) {
    std::vector<int64_t> arr(n);
    for (int64_t i = 0; i < n; ++i) arr[i] = i;
    // detections with objectness 0 go to the end (swap with the last, re-examine the swapped-in one)
    int64_t total = n - 1, k = total, i = 0;
    while (i <= k) {
        if (objectness[arr[i]] == 0.0f) {
            std::swap(arr[i], arr[k]);
            --k;
            --i;
        }
        ++i;
    }
    total = k + 1;
    NmsCtx c{probs, objectness, classes, -1};
    for (int64_t cl = 0; cl < classes; ++cl) {
        c.sort_class = cl;
        if (total > 0) nms_quicksort(c, arr.data(), 0, total - 1);
        for (int64_t a = 0; a < total; ++a) {
            if (probs[arr[a] * classes + cl] == 0.0f) continue;
            const float* ba = boxes + arr[a] * 4;
            for (int64_t b = a + 1; b < total; ++b)
                if (nms_iou(ba, boxes + arr[b] * 4) > thresh) probs[arr[b] * classes + cl] = 0.0f;
        }
    }
    if (order)
        for (int64_t j = 0; j < n; ++j) order[j] = arr[j];
}

// ---------------------------------------------------------------------------------------
// input images (source/ntypes.pas TImageData)
// ---------------------------------------------------------------------------------------
// TImageData.loadFromFile (:669-694, FPC build): planar RGB floats from the decoder's colours.
// FPImage (FreePascal's fcl-image, not part of the reference) holds 16-bit channels and widens
// an 8-bit value v to v * 257; the reference divides by $ff00, so a pixel byte becomes
// v * 257 / 65280 (double division, rounded to single on the store). The Delphi build
// (:696-724) divides the 8-bit value by $ff: pixel_scale 1.
// src: interleaved rows (row_stride bytes apart), bpp bytes per pixel (1 gray, 3, 4), bgr:
// byte order B, G, R. out: [3][h][w].
void or_image_from_bytes(int64_t w, int64_t h, const uint8_t* src, int64_t row_stride, int64_t bpp,
                         int64_t bgr, int64_t pixel_scale, float* out) {
    const int64_t plane = w * h;
    for (int64_t y = 0; y < h; ++y)
        for (int64_t x = 0; x < w; ++x) {
            const uint8_t* p = src + y * row_stride + x * bpp;
            int v[3];
            if (bpp == 1) v[0] = v[1] = v[2] = p[0];
            else if (bgr) { v[0] = p[2]; v[1] = p[1]; v[2] = p[0]; }
            else { v[0] = p[0]; v[1] = p[1]; v[2] = p[2]; }
            for (int k = 0; k < 3; ++k)
                out[k * plane + y * w + x] = pixel_scale == 0 ? (float)((double)(v[k] * 257) / 65280.0)
                                                              : (float)((double)v[k] / 255.0);
        }
}

// TImageData.resize (:837-897): separable bilinear, columns first into `part` [c][h][aw], then
// rows. Single-precision arithmetic; w_scale / h_scale are integer quotients stored to single.
void or_resize(int64_t c, int64_t h, int64_t w, const float* src, int64_t aw, int64_t ah, float* out) {
    std::vector<float> part((size_t)(c * h * aw));
    const float w_scale = (float)((double)(w - 1) / (double)(aw - 1));
    const float h_scale = (float)((double)(h - 1) / (double)(ah - 1));
    for (int64_t k = 0; k < c; ++k)
        for (int64_t r = 0; r < h; ++r)
            for (int64_t cc = 0; cc < aw; ++cc) {
                float val;
                if (cc == aw - 1 || w == 1) {
                    val = src[(k * h + r) * w + (w - 1)];
                } else {
                    const float sx = (float)cc * w_scale;
                    const int64_t ix = (int64_t)sx;  // trunc
                    const float dx = sx - (float)ix;
                    val = (1.0f - dx) * src[(k * h + r) * w + ix] + dx * src[(k * h + r) * w + ix + 1];
                }
                part[(size_t)((k * h + r) * aw + cc)] = val;
            }
    for (int64_t k = 0; k < c; ++k)
        for (int64_t r = 0; r < ah; ++r) {
            const float sy = (float)r * h_scale;
            const int64_t iy = (int64_t)sy;
            const float dy = sy - (float)iy;
            for (int64_t cc = 0; cc < aw; ++cc)
                out[(k * ah + r) * aw + cc] = (1.0f - dy) * part[(size_t)((k * h + iy) * aw + cc)];
            if (r == ah - 1 || h == 1) continue;
            for (int64_t cc = 0; cc < aw; ++cc)
                out[(k * ah + r) * aw + cc] = out[(k * ah + r) * aw + cc] + dy * part[(size_t)((k * h + iy + 1) * aw + cc)];
        }
}

// TImageData.letterBoxEx (:922-943): keep the aspect ratio, resize, embed centred into an
// image filled with 0.5. meta_out: new_w, new_h, dx, dy; ratio_out: the scale (single).
void or_letterbox(int64_t c, int64_t h, int64_t w, const float* src, int64_t aw, int64_t ah, float* out,
                  int64_t* meta_out, float* ratio_out) {
    int64_t new_w = w, new_h = h;
    float ratio;
    if ((double)aw / (double)w < (double)ah / (double)h) {
        new_w = aw;
        new_h = (h * aw) / w;
        ratio = (float)((double)aw / (double)w);
    } else {
        new_h = ah;
        new_w = (w * ah) / h;
        ratio = (float)((double)ah / (double)h);
    }
    std::vector<float> resized((size_t)(c * new_h * new_w));
    or_resize(c, h, w, src, new_w, new_h, resized.data());
    for (int64_t i = 0; i < c * ah * aw; ++i) out[i] = 0.5f;
    const int64_t dx = (aw - new_w) / 2, dy = (ah - new_h) / 2;
    for (int64_t k = 0; k < c; ++k)
        for (int64_t y = 0; y < new_h; ++y)
            for (int64_t x = 0; x < new_w; ++x) {
                const int64_t ox = dx + x, oy = dy + y;  // Setpixels drops out-of-range writes
                if (ox < 0 || oy < 0 || ox >= aw || oy >= ah) continue;
                out[(k * ah + oy) * aw + ox] = resized[(size_t)((k * new_h + y) * new_w + x)];
            }
    if (meta_out) { meta_out[0] = new_w; meta_out[1] = new_h; meta_out[2] = dx; meta_out[3] = dy; }
    if (ratio_out) *ratio_out = ratio;
}

int64_t or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_threads(int64_t n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads((int)n);
#else
    (void)n;
#endif
}

}  // extern "C"
