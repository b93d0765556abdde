/*
 * tensorium_b200.h -- C ABI of the B200 (sm_100a) backend for Tensorium's darknet-style
 * convolution-forward inference path.
 *
 * This library replaces the CUDA half of the reference's layer dispatch: the TNNCuda<T>
 * methods in source/nncuda.pas:100-158 that TConvolutionalLayer, TMaxPoolLayer,
 * TUpSampleLayer, TConcatLayer (route), TAddLayer (shortcut), TYoloLayer and
 * TXNORConvolutionLayer call from their forwardGPU methods.  The Pascal host keeps its
 * TSingleTensor / layer API and binds these functions as `external 'tensorium_b200' ... cdecl`.
 *
 * Conventions (all entry points):
 *   - cdecl, plain C types only; every size is int64_t (the reference's SizeInt on x86-64).
 *   - float pointers are device pointers unless the name ends in _host.
 *   - tensors are NCHW fp32, as TSingleTensor stores them.
 *   - every function returns int: TB_OK (0) on success, a negative TB_ERR_* otherwise; the
 *     message of the last failure on the calling thread is tb_last_error().
 *     (The reference asserts instead: SAFE_CALL in source/nncuda.pas:237-273.)
 *   - launches are asynchronous on the context's stream; only tb_sync, tb_memcpy_d2h and the
 *     functions that say so block.
 *   - device memory is allocated only by tb_malloc, tb_init, tb_workspace_reserve and
 *     tb_net_finalize, and by the context's scratch workspace growing on demand inside
 *     tb_conv2d_fwd (split-K partials), tb_xnor_conv_fwd (packed input bits) and
 *     tb_yolo_detect (counters). Growth is refused (TB_ERR_STATE) while the stream is being
 *     captured into a CUDA graph; reserve first with tb_workspace_reserve.
 */
#ifndef TENSORIUM_B200_H
#define TENSORIUM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_VERSION 100

/* ---- status codes ------------------------------------------------------------------ */
#define TB_OK               0
#define TB_ERR_INVALID     -1   /* bad argument (null pointer, bad size, unsupported shape) */
#define TB_ERR_CUDA        -2   /* a CUDA runtime call failed */
#define TB_ERR_UNSUPPORTED -3   /* valid request that this build does not implement */
#define TB_ERR_OOM         -4   /* device allocation failed */
#define TB_ERR_TIMEOUT     -5   /* a bounded wait ran out (collectives) */
#define TB_ERR_STATE       -6   /* call made in the wrong state (e.g. net not finalized) */
#define TB_ERR_DEVICE      -7   /* a kernel reported an error through the device status word */

/* ---- activations: same ordinals as TActivationType (source/ntypes.pas:66-71) ----------- */
#define TB_ACT_LOGISTIC  0
#define TB_ACT_RELU      1
#define TB_ACT_RELU6     2
#define TB_ACT_RELIE     3
#define TB_ACT_LINEAR    4
#define TB_ACT_RAMP      5
#define TB_ACT_TANH      6
#define TB_ACT_PLSE      7
#define TB_ACT_REVLEAKY  8
#define TB_ACT_LEAKY     9
#define TB_ACT_ELU      10
#define TB_ACT_LOGGY    11
#define TB_ACT_HARDTAN  13
#define TB_ACT_LHTAN    14
#define TB_ACT_SELU     15

/* ---- math modes of the convolution mainloop ---------------------------------------- */
#define TB_MATH_FP32  0   /* FP32 CUDA-core mainloop in the reference's order: one FMA per k,
                             k ascending as im2col rows (c, kh, kw), no split of K -- results
                             bit-identical to the reference CPU path (default) */
#define TB_MATH_TF32  1   /* tcgen05 tensor-core mainloop, TF32 operands, FP32 accumulate */
#define TB_MATH_BF16_SPLIT 3  /* tcgen05 kind::f16 tensor cores on BF16-split operands: every fp32
                             value carried as a pair of bf16 (hi = bf16(v), lo = bf16(v - hi)), all
                             four partial products accumulated in FP32 (~16-bit operand precision,
                             twice the MMAs of TF32). Networks only (tb_net_finalize, NHWC plan);
                             nets or layers that plan cannot take run on the FP32 path */
#define TB_MATH_FP32_TILED 2  /* FP32 CUDA-core mainloop with the summation reordered (k tiles
                             in (kh, kw, c) order, split-K with partial sums in scratch): within
                             the reference's 1e-4 per map, not bit-identical */

/* ---- context ------------------------------------------------------------------------- */
typedef struct tb_ctx tb_ctx;

typedef struct tb_options {
    int64_t math_mode;        /* TB_MATH_* used by tb_conv2d_fwd when a call does not override */
    int64_t workspace_bytes;  /* initial split-K workspace; 0 = library default (64 MiB) */
    int64_t flags;            /* reserved, must be 0 */
} tb_options;

/* Last error message of the calling thread ("" if none). */
const char* tb_last_error(void);
int tb_version(void);
/* Replaces TNNCuda.deviceCount (source/nncuda.pas:100). */
int tb_device_count(int64_t* count);
/* Replaces TNNCuda.Create(deviceIndex) (source/nncuda.pas:448-467): selects the device,
 * creates a stream and the split-K workspace. opts may be NULL. */
int tb_init(int64_t device, const tb_options* opts, tb_ctx** out);
/* Replaces TNNCuda.Destroy. */
int tb_shutdown(tb_ctx* ctx);
/* Run subsequent launches on an existing cudaStream_t; NULL selects the legacy default stream.
 * Until this is called the context launches on a stream of its own. */
int tb_set_stream(tb_ctx* ctx, void* cuda_stream);
void* tb_get_stream(tb_ctx* ctx);
/* Replaces TNNCuda.finish (source/nncuda.pas:1575-1584); also surfaces device status errors. */
int tb_sync(tb_ctx* ctx);
/* Replaces createDeviceBuffer / freeDeviceBuffer (source/nncuda.pas:103-104). */
int tb_malloc(tb_ctx* ctx, int64_t bytes, void** ptr);
int tb_free(tb_ctx* ctx, void* ptr);
/* Replaces writeBuffer / readBuffer (source/nncuda.pas:105-106). h2d is asynchronous
 * (ordered on the stream); d2h blocks until the bytes are on the host. */
int tb_memcpy_h2d(tb_ctx* ctx, void* dst, const void* src_host, int64_t bytes);
int tb_memcpy_d2h(tb_ctx* ctx, void* dst_host, const void* src, int64_t bytes);
/* Grow the split-K workspace to at least `bytes` (allocates; call before graph capture). */
int tb_workspace_reserve(tb_ctx* ctx, int64_t bytes);
/* Bytes the context's scratch workspace holds now (no counterpart in the reference). */
int tb_workspace_size(tb_ctx* ctx, int64_t* bytes);

/* ---- elementwise / BLAS-1 helpers used by the layers on the path -------------------- */
/* TNNCuda.ActivateArray(N, x, offset, activation) (source/nncuda.pas:108). */
int tb_activate(tb_ctx* ctx, int64_t n, float* x, int64_t offset, int64_t activation);
/* TNNCuda.forwardBias (source/nncuda.pas:110): dst[b][i][j] += bias[i], i < bias_size,
 * j < dst_size/(batch*bias_size). */
int tb_forward_bias(tb_ctx* ctx, int64_t dst_size, float* dst, int64_t offset,
                    int64_t bias_size, const float* bias, int64_t incb, int64_t batch);
/* TNNCuda.copy (source/nncuda.pas:123). */
int tb_copy(tb_ctx* ctx, int64_t n, const float* src, int64_t src_offset, int64_t inca,
            float* dst, int64_t dst_offset, int64_t incb);
/* TNNCuda.fill (source/nncuda.pas:122). */
int tb_fill(tb_ctx* ctx, int64_t n, float* x, int64_t offset, float val, int64_t stride);
/* TNNCuda.addvv (source/nncuda.pas:116): dst = src1 + src2 elementwise (strided). */
int tb_addvv(tb_ctx* ctx, int64_t n, const float* src1, int64_t src1_offset, int64_t inca,
             const float* src2, int64_t src2_offset, int64_t incb,
             float* dst, int64_t dst_offset, int64_t incc);
/* TNNCuda.fmavss (source/nncuda.pas:137): dst = src*scalar + bias on n elements at offset. */
int tb_fmavss(tb_ctx* ctx, int64_t n, float* src, int64_t offset, float scalar, float bias, float* dst);

/* ---- convolution (TConvolutionalLayer.forward / forwardGPU) --------------------------- */
typedef struct tb_conv_desc {
    int64_t batch, channels, height, width;        /* input  [batch, channels, height, width] */
    int64_t filters, kernel_h, kernel_w;           /* weights [filters][channels*kernel_h*kernel_w] */
    int64_t stride_y, stride_x, pad_y, pad_x;
    int64_t dilation_y, dilation_x;                /* 0 is read as 1 */
    int64_t activation;                            /* TB_ACT_* applied after bias / batchnorm */
    int64_t in_batch_stride;   /* elements between images of x; 0 = channels*height*width */
    int64_t out_batch_stride;  /* elements between images of y; 0 = filters*out_h*out_w */
    int64_t res_batch_stride;  /* elements between images of residual; 0 = like y */
} tb_conv_desc;

/* Output size (h + 2p - dil*(k-1) - 1) div s + 1, as TBaseConvolutionalLayer.outHeight /
 * outWidth (source/nConvolutionLayer.pas:92-100). */
int tb_conv_out_shape(const tb_conv_desc* d, int64_t* out_h, int64_t* out_w);
/* Number of floats of the packed weight buffer tb_conv_pack_weights writes. */
int tb_conv_packed_weights_count(const tb_conv_desc* d, int64_t* count);
/* Re-lay the reference weights (row-major [filters][channels][kh][kw], the order of
 * source/nConvolutionLayer.pas:206 and the darknet .weights file) into the K-major tile layout
 * the conv kernels read. Device to device, once per weight load (the reference's one-time
 * weights.pushToDevice, source/nConvolutionLayer.pas:1034-1036). */
int tb_conv_pack_weights(tb_ctx* ctx, const tb_conv_desc* d, const float* weights, float* packed);
/* tb_conv_pack_weights followed by rounding every packed weight to TF32 (nearest, ties away):
 * the weights for TB_MATH_TF32 calls. The tensor core would otherwise truncate them, a bias
 * toward zero that adds up over a deep network. Same layout and count. (The reference has no
 * tensor-core path; this replaces the same weights.pushToDevice step.) */
int tb_conv_pack_weights_tf32(tb_ctx* ctx, const tb_conv_desc* d, const float* weights, float* packed);
/* *yes = 1 when tb_conv2d_fwd with this descriptor and math mode runs the tensor-core mainloop
 * (TB_MATH_TF32 and channels % 32 == 0), 0 when it runs the FP32 kernel: which packing the
 * caller should hand it (no reference counterpart). */
int tb_conv_uses_tensor_cores(const tb_conv_desc* d, int64_t math_mode, int64_t* yes);
/* ---- TF32 tensor-core conv on NHWC activations (no reference counterpart: the layout the
 * B200 tensor-core path uses inside a network) ----
 * x is [batch][h][w][...] with x_pixel_stride floats per pixel (x points at the conv's first
 * input channel; a multiple of 4); y is NHWC with y_pixel_stride floats per pixel (y at the
 * output's first channel) or, with y_pixel_stride == 0, NCHW with the descriptor's
 * out_batch_stride. The residual (NHWC, res_pixel_stride) is added after the activation, the
 * shortcut order. Weights are packed by tb_conv_pack_weights_nhwc ([F][KH][KW][C rounded up to
 * 32], rounded to TF32). Operands are read as TF32; outputs are rounded to TF32. Geometries the
 * kernel cannot take (corner or tap offsets outside the im2col map's range, inputs under 128 KB)
 * return TB_ERR_UNSUPPORTED. The descriptor's in/res batch strides are ignored. */
int tb_conv_nhwc_packed_count(const tb_conv_desc* d, int64_t* count);
int tb_conv_pack_weights_nhwc(tb_ctx* ctx, const tb_conv_desc* d, const float* weights_host_or_dev,
                              float* packed);
int tb_conv2d_fwd_nhwc(tb_ctx* ctx, const tb_conv_desc* d, const float* x, int64_t x_pixel_stride,
                       const float* packed_w, const float* bias, const float* residual,
                       int64_t res_pixel_stride, float* y, int64_t y_pixel_stride);
/* Host helper: fold batchnorm into weights and biases in place, the arithmetic of
 * TBaseConvolutionalLayer.fuseBatchNorm (source/nConvolutionLayer.pas:102-126). */
int tb_conv_fold_bn(int64_t filters, int64_t filter_size, float* weights_host, float* biases_host,
                    const float* scales_host, const float* rolling_mean_host,
                    const float* rolling_variance_host);
/* Time the admissible CTA-tile / split-K choices of this geometry on the given buffers (y is
 * overwritten) and use the fastest for every later call with the same geometry on this device.
 * Optional: without it a cost model chooses. Blocks; may grow the workspace. (The reference has
 * no tuning step; its GPU conv is a fixed cuBLAS call, source/nncuda.pas:846.) */
int tb_conv_autotune(tb_ctx* ctx, const tb_conv_desc* d, const float* x, const float* packed_w, float* y);
/* Fused conv forward: y = act(conv(x, w) + epilogue) [+ residual].
 * Replaces, in one launch (two with split-K), the reference sequence
 *   cuda.im2col per image -> cuda.gemmStridedBatched -> [normalize, forwardScale] ->
 *   forwardBias -> ActivateArray   (source/nConvolutionLayer.pas:1055-1122)
 * epilogue: if bn_mean != NULL: v = ((acc - mean)/max(sqrt(var),1e-6))*bn_scale + bias
 *           (TBaseLayer.batchNorm inference, source/nbaselayer.pas:336-370)
 *           else v = acc + bias (bias may be NULL = 0; source/ntensors.pas:7709-7727);
 *           v = act(v); if residual != NULL: v += residual (TAddLayer.forward,
 *           source/naddlayer.pas:696-699, with a linear shortcut activation).
 * math_mode: TB_MATH_* or -1 for the context default. */
int tb_conv2d_fwd(tb_ctx* ctx, const tb_conv_desc* d, const float* x, const float* packed_w,
                  const float* bias, const float* bn_scale, const float* bn_mean,
                  const float* bn_variance, const float* residual, float* y, int64_t math_mode);

/* tb_conv2d_fwd without any device allocation, for callers that cannot call cudaMalloc
 * (device memory handed out up front by an arena, an allocator held by another component, or
 * a loop where an allocation's latency or failure is not acceptable). No counterpart in the
 * reference. Same arguments as tb_conv2d_fwd and the results of tb_conv2d_fwd with
 * math_mode TB_MATH_FP32_TILED (the tiled kernels with split-K); the split-K scratch is a fixed
 * array inside the library (16 MiB of partial sums + 16384 tile counters, held on every GPU that
 * loads the library until exit). A layer whose chosen split needs more scratch than that runs
 * with its split lowered until the partial sums fit (split 1 needs none); a split pinned through
 * the TB_CONV_FORCE test hook that does not fit is rejected with TB_ERR_INVALID. The first call
 * on a device looks up the array's device address; make that first call before any stream
 * capture; cudaDeviceReset of that device is not supported afterwards. All calls share the one
 * array: calls that overlap on the GPU (other streams, other contexts on the same device) race. */
int tb_conv2d_fwd_noalloc(tb_ctx* ctx, const tb_conv_desc* d, const float* x, const float* packed_w,
                          const float* bias, const float* bn_scale, const float* bn_mean,
                          const float* bn_variance, const float* residual, float* y);

/* ---- memory-bound layers -------------------------------------------------------------- */
/* TNNCuda.forwardMaxPool (source/nncuda.pas:132; CPU semantics source/nMaxPoolLayer.pas:
 * 265-463): out = max over the k x k window at (i*stride_y + n - padding div 2,
 * j*stride_x + m - padding div 2), out-of-image = -FLT_MAX, strict '>' (first max wins).
 * out_h = (h + padding - k) div stride_y + 1. indexes (int64, may be NULL) receives the flat
 * input index of the max (-1 if none). */
int tb_maxpool_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                   int64_t ksize, int64_t stride_x, int64_t stride_y, int64_t padding,
                   const float* x, float* y, int64_t* indexes);
/* TUpSampleLayer.forward (source/nupsamplelayer.pas:83-131): y[c][yy][xx] =
 * scale * x[c][yy div s][xx div s]. y_batch_stride (0 = dense) lets the result land in a
 * slice of a route (concat) buffer. */
int tb_upsample_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                    int64_t stride, float scale, const float* x, float* y, int64_t y_batch_stride);
/* TConcatLayer.forward (source/nconcatlayer.pas:93-119). per_sample != 0: darknet channel
 * concatenation per image (out[b] = in0[b] | in1[b] | ...). per_sample == 0: the reference's
 * TTensor.concat (source/ntensors.pas:12045-12061), whole tensors back to back.
 * sizes[i] = elements per image of input i. */
int tb_route_fwd(tb_ctx* ctx, int64_t batch, int64_t n_inputs, const float* const* inputs,
                 const int64_t* sizes, float* y, int64_t per_sample);
/* TAddLayer.forward single-input branch (source/naddlayer.pas:696-699) + activate():
 * y = act(a + b) over n elements. */
int tb_shortcut_fwd(tb_ctx* ctx, int64_t n, const float* a, const float* b, float* y,
                    int64_t activation);
/* TYoloLayer.forward (source/nyololayer.pas:786-825): copy x to y, logistic on entries
 * 0,1 (x,y) and 4..4+classes (objectness, classes) of every anchor, then if scale_xy != 1:
 * v*scale_xy - 0.5*(scale_xy-1) on entries 0,1. Layout [batch][n][classes+5][h][w]. */
int tb_yolo_fwd(tb_ctx* ctx, int64_t batch, int64_t n, int64_t classes, int64_t h, int64_t w,
                const float* x, float* y, float scale_xy);

/* One detection, as TDetection (source/ntypes.pas:278) without the per-class array, which is
 * written separately (prob[det][classes]). */
typedef struct tb_detection {
    float x, y, w, h;        /* TBox after correctBoxes */
    float objectness;
    int32_t batch;           /* image */
    int32_t head;            /* index of the yolo layer in the call */
    int32_t index;           /* location i = row*w + col */
    int32_t anchor;          /* _n */
    int32_t reserved[3];
} tb_detection;

typedef struct tb_yolo_head {
    const float* output;     /* activated yolo output [batch][n][classes+5][h][w] */
    int64_t n, classes, h, w;
    const int64_t* mask_host;    /* n anchor ids */
    const float* anchors_host;   /* all anchors (w,h pairs) of the layer, >= 2*max(mask)+2 */
    int64_t new_coords;
} tb_yolo_head;

/* TYoloLayer.getDetections + correctBoxes over every head (source/nyololayer.pas:399-498),
 * for every image, in the reference order (heads in layer order, i-major, anchor-minor,
 * source/nnet.pas:647-653). Writes at most `capacity` detections per image to
 * dets[b*capacity + k] and prob[(b*capacity + k)*classes + j]; counts[b] = number found
 * (may exceed capacity: then only the first `capacity` are written). Blocks until counts are
 * on the host (counts_host). */
int tb_yolo_detect(tb_ctx* ctx, int64_t batch, int64_t n_heads, const tb_yolo_head* heads,
                   int64_t img_w, int64_t img_h, int64_t net_w, int64_t net_h, float thresh,
                   int64_t relative, int64_t letter, int64_t capacity,
                   tb_detection* dets, float* prob, int64_t* counts_host);
/* tb_yolo_detect without the host round trip (no counterpart in the reference): the per-image
 * totals go to counts_dev (int64 [batch], device memory) and nothing waits, so detection
 * extraction, a gather to rank 0 (tb_group_gather_async) and the copy of the result can be queued
 * behind the forward. */
int tb_yolo_detect_device(tb_ctx* ctx, int64_t batch, int64_t n_heads, const tb_yolo_head* heads,
                          int64_t img_w, int64_t img_h, int64_t net_w, int64_t net_h, float thresh,
                          int64_t relative, int64_t letter, int64_t capacity, tb_detection* dets, float* prob,
                          int64_t* counts_dev);
/* Class-wise non-maximum suppression on the detections tb_yolo_detect wrote, replacing
 * TDetectionsHelper.doNMSSort (source/ntypes.pas:1621-1649): for every image and class, the
 * detections with a non-zero probability of the class are taken in order of decreasing
 * probability; each one not yet suppressed zeroes the class probability of every later one
 * whose box IoU with it (box_iou, source/ntypes.pas:1059-1108) exceeds `thresh`. Detections
 * with objectness 0 take no part. prob is updated in place; the records keep their order (the
 * reference leaves them sorted by the last class). Equal probabilities are taken in detection
 * order (the reference's quicksort leaves their order to its partition history). At most 8192
 * detections per image (min(counts_host[b], capacity)). Asynchronous on the context stream. */
int tb_yolo_nms(tb_ctx* ctx, int64_t batch, int64_t capacity, const int64_t* counts_host, int64_t classes,
                float thresh, const tb_detection* dets, float* prob);

/* ---- XNOR binary convolution (TXNORConvolutionLayer, source/nxnorconvolutionlayer.pas) --- */
#define TB_XNOR_PAD_BIT0 0   /* padding pixels are bit 0 (= -1), as im2col_cpu_custom_bin :232-316 */
#define TB_XNOR_PAD_ZERO 1   /* padding pixels contribute 0, as the float fallback :860-868 */
/* Words (uint32) of the packed weight buffer. */
int tb_xnor_packed_weights_count(int64_t filters, int64_t channels, int64_t ksize, int64_t* count);
/* Sign-pack weights (bit = w > 0) and compute mean_f = (sum_i |w_fi|)/size in the reference's
 * sequential fp32 order (binarize_weights, :95-113). weights and mean are device pointers. */
int tb_xnor_pack_weights(tb_ctx* ctx, int64_t filters, int64_t channels, int64_t ksize,
                         const float* weights, uint32_t* packed, float* mean);
/* out[b][f][p] = (2*matches - K) * mean[f] (gemm_nn_custom_bin_mean_transposed :179-205),
 * input bit = x > 0 (:793-794); then + bias (may be NULL) and activation. popcount_out
 * (int32 [batch][filters][oh][ow], may be NULL) receives 2*matches - K. Scratch: the packed
 * input bits live in the context workspace. */
int tb_xnor_conv_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                     int64_t filters, int64_t ksize, int64_t stride, int64_t pad, int64_t pad_mode,
                     const float* x, const uint32_t* packed_w, const float* mean,
                     const float* bias, int64_t activation, int32_t* popcount_out, float* y);

/* ---- layers of the MNIST / CIFAR-shaped configs -------------------------------------- */
/* TConnectedLayer.forward (source/nconnectedlayer.pas:157-184): y[b][o] = sum_i x[b][i] *
 * w[o][i] (gemm NoTrans, Trans) + bias[o], then activation. w is the reference layout
 * [outputs][inputs] packed by tb_conv_pack_weights of a 1x1 conv with channels = inputs. */
int tb_fc_fwd(tb_ctx* ctx, int64_t batch, int64_t inputs, int64_t outputs, const float* x,
              const float* packed_w, const float* bias, int64_t activation, float* y);
/* TSoftmaxLayer.forward -> softmaxBatch (source/nsoftmaxlayer.pas:83-167). */
int tb_softmax_fwd(tb_ctx* ctx, int64_t batch, int64_t inputs, int64_t groups, float temperature,
                   const float* x, float* y);
/* TAvgPoolLayer.forward (source/navgpoollayer.pas:60-84): y[b][c] = mean over h*w. */
int tb_avgpool_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t h, int64_t w,
                   const float* x, float* y);

/* ---- TNNCuda method shims --------------------------------------------------------------
 * One function per TNNCuda<single> method the forward layers call, with that method's argument
 * list in the same order (source/nncuda.pas:100-151), preceded by the context that stands in
 * for the global `cuda` object: SizeInt -> int64_t, single -> float, boolean / longint ->
 * int32_t, TCUMem -> device pointer.  A Pascal TNNCuda replacement forwards each method with a
 * one-line call.  Results follow the reference's CPU routines (the library's parity target):
 * the GEMMs keep cblas_sgemm's orders (s_nn / s_tn: C = beta*C then one FMA of alpha*a per k
 * ascending; s_nt: sdot_avx2's eight lanes; s_tt: sequential sum of (alpha*a)*b).  The GEMM
 * shims are correctness shims (one thread per output); tb_conv2d_fwd is the fast conv path.
 * Training-direction calls (upSample with isForward = 0) return TB_ERR_UNSUPPORTED. */
/* createDeviceBuffer(N bytes) / freeDeviceBuffer (source/nncuda.pas:103-104, 488-497). */
int tbcompat_createDeviceBuffer(tb_ctx* ctx, int64_t N, void** mem);
int tbcompat_freeDeviceBuffer(tb_ctx* ctx, void* mem);
/* readBuffer / writeBuffer (source/nncuda.pas:105-106): blocking copies of bufferSize bytes. */
int tbcompat_readBuffer(tb_ctx* ctx, const void* mem, int64_t bufferSize, void* buffer);
int tbcompat_writeBuffer(tb_ctx* ctx, void* mem, int64_t bufferSize, const void* buffer);
/* finish (source/nncuda.pas:153, 1575-1584). */
int tbcompat_finish(tb_ctx* ctx);
/* ActivateArray(N, x, offset, activation) (source/nncuda.pas:108, 524-580). */
int tbcompat_ActivateArray(tb_ctx* ctx, int64_t N, float* x, int64_t offset, int32_t activation);
/* forwardBias(dstSize, dst, offset, srcSize, src, incb, batch) (source/nncuda.pas:111, 582-600):
 * dst[offset + i] += src[((i / block) % srcSize) * incb], block = dstSize / (srcSize*batch). */
int tbcompat_forwardBias(tb_ctx* ctx, int64_t dstSize, float* dst, int64_t offset, int64_t srcSize,
                         const float* src, int64_t incb, int64_t batch);
/* forwardScale(dstSize, dst, offset, scaleSize, scale, incb, batch) (source/nncuda.pas:145,
 * 1468-1488): dst[offset + i] *= scale[f]. */
int tbcompat_forwardScale(tb_ctx* ctx, int64_t dstSize, float* dst, int64_t offset, int64_t scaleSize,
                          const float* scale, int64_t incb, int64_t batch);
/* forwardScaleAdd(dstSize, dst, offset, scaleSize, scales, biases, incb, batch) (source/
 * nncuda.pas:146, 1490-1508): dst = dst*scales[f] + biases[f], two roundings. */
int tbcompat_forwardScaleAdd(tb_ctx* ctx, int64_t dstSize, float* dst, int64_t offset, int64_t scaleSize,
                             const float* scales, const float* biases, int64_t incb, int64_t batch);
/* normalize(srcSize, dstSize, groups, means, meansStride, vars, varsStride, dst, dstOffset)
 * (source/nncuda.pas:141, 1371-1393): dst[g][i][j] = (dst - means[i*meansStride]) /
 * max(sqrt(vars[i*varsStride]), 1e-6) as blockNormalize (source/ntensors.pas:8693-8718). */
int tbcompat_normalize(tb_ctx* ctx, int64_t srcSize, int64_t dstSize, int64_t groups, const float* means,
                       int64_t meansStride, const float* vars, int64_t varsStride, float* dst, int64_t dstOffset);
/* gemm(transA, transB, M, N, K, ALPHA, A, aOffset, lda, B, bOffset, ldb, BETA, C, cOffset, ldc)
 * (source/nncuda.pas:112, 624-808): row-major C = ALPHA*op(A)*op(B) + BETA*C. */
int tbcompat_gemm(tb_ctx* ctx, int32_t transA, int32_t transB, int64_t M, int64_t N, int64_t K, float ALPHA,
                  const float* A, int64_t aOffset, int64_t lda, const float* B, int64_t bOffset, int64_t ldb,
                  float BETA, float* C, int64_t cOffset, int64_t ldc);
/* gemmStridedBatched(..., strideA, ..., strideB, ..., strideC, batchCount) (source/nncuda.pas:
 * 119, 809-896): batchCount GEMMs, matrices strideA / strideB / strideC elements apart. */
int tbcompat_gemmStridedBatched(tb_ctx* ctx, int32_t transA, int32_t transB, int64_t M, int64_t N, int64_t K,
                                float ALPHA, const float* A, int64_t aOffset, int64_t lda, int64_t strideA,
                                const float* B, int64_t bOffset, int64_t ldb, int64_t strideB, float BETA, float* C,
                                int64_t cOffset, int64_t ldc, int64_t strideC, int64_t batchCount);
/* addvv (source/nncuda.pas:120, 897-915). */
int tbcompat_addvv(tb_ctx* ctx, int64_t N, const float* src1, int64_t src1Offset, int64_t inca, const float* src2,
                   int64_t src2Offset, int64_t incb, float* dst, int64_t dstOffset, int64_t incc);
/* fill (source/nncuda.pas:128, 1017-1035). */
int tbcompat_fill(tb_ctx* ctx, int64_t N, float* x, int64_t offset, float val, int64_t stride);
/* copy (source/nncuda.pas:129, 1037-1054). */
int tbcompat_copy(tb_ctx* ctx, int64_t N, const float* src, int64_t srcOffset, int64_t inca, float* dst,
                  int64_t dstOffset, int64_t incb);
/* fmavss(N, src, offset, scalar, bias, dst) (source/nncuda.pas:137, 1288-1305): dst = src*scalar + bias. */
int tbcompat_fmavss(tb_ctx* ctx, int64_t N, float* src, int64_t offset, float scalar, float bias, float* dst);
/* softmaxBatch(N, input, iOffset, batch, batch_size, groups, group_size, stride, temp, output,
 * oOffset) (source/nncuda.pas:130, 1056-1086). */
int tbcompat_softmaxBatch(tb_ctx* ctx, int64_t N, const float* input, int64_t iOffset, int64_t batch,
                          int64_t batch_size, int64_t groups, int64_t group_size, int64_t stride, float temp,
                          float* output, int64_t oOffset);
/* forwardMaxPool(aBatch, outC, outH, outW, input, c, h, w, stride_x, stride_y, padding,
 * kernelSize, indexes, output) (source/nncuda.pas:132, 1088-1142); indexes are int64. */
int tbcompat_forwardMaxPool(tb_ctx* ctx, int64_t aBatch, int64_t outC, int64_t outH, int64_t outW,
                            const float* input, int64_t c, int64_t h, int64_t w, int64_t stride_x, int64_t stride_y,
                            int64_t padding, int64_t kernelSize, int64_t* indexes, float* output);
/* im2col(aChannels, aHeight, aWidth, kernelHeight, kernelWidth, padHeight, padWidth, strideY,
 * strideX, dilationY, dilationX, im, imOffset, col, colOffset) (source/nncuda.pas:134,
 * 1144-1190): col[(c*kh + r)*kw + s][oy*ow + ox], the CPU sim2Col layout. */
int tbcompat_im2col(tb_ctx* ctx, int64_t aChannels, int64_t aHeight, int64_t aWidth, int64_t kernelHeight,
                    int64_t kernelWidth, int64_t padHeight, int64_t padWidth, int64_t strideY, int64_t strideX,
                    int64_t dilationY, int64_t dilationX, const float* im, int64_t imOffset, float* col,
                    int64_t colOffset);
/* upSample(aBatch, aChannels, outHeight, outWidth, in, stride, isForward, scale, out, zeroIn)
 * (source/nncuda.pas:136, 1267-1286); outHeight / outWidth are the INPUT's size, as the
 * reference passes them. */
int tbcompat_upSample(tb_ctx* ctx, int64_t aBatch, int64_t aChannels, int64_t outHeight, int64_t outWidth,
                      const float* in, int64_t stride, int32_t isForward, float scale, float* out, int32_t zeroIn);

/* Unfused batchnorm layer (TBaseLayer.batchNorm inference, source/nbaselayer.pas:336-370, the
 * cuda.normalize -> forwardScale -> forwardBias sequence of :620-643) in one pass over
 * [batch][channels][spatial]: y = ((x - mean)/max(sqrt(var), 1e-6))*scale + bias, three
 * roundings. scales / biases may be NULL (1 / 0). y may equal x. */
int tb_bn_fwd(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t spatial, const float* x, const float* mean,
              const float* variance, const float* scales, const float* biases, float* y);

/* ---- multi-GPU group (NCCL) ------------------------------------------------------------
 * Inference shards by image: each GPU runs the whole network on its slice of the batch, and the
 * only exchange is the final gather of per-GPU results (detection records, counts, logits) to
 * rank 0. The reference has no multi-GPU path (source/nConvolutionLayer.pas:472 marks it as
 * future work); these entry points are new. NCCL (libnccl.so.2) is loaded on first use. */
typedef struct tb_group tb_group;
/* NCCL loads; *nccl_version = its version code (may be NULL). TB_ERR_UNSUPPORTED without NCCL. */
int tb_group_available(int64_t* nccl_version);
/* One process drives ngpu GPUs: a context per device (tb_group_context) and NCCL communicators
 * over them (ncclCommInitAll). Ranks follow `devices`. */
int tb_group_init(int64_t ngpu, const int64_t* devices, tb_group** out);
/* One process per GPU: rank 0 makes the 128-byte id, the caller hands it to every rank. */
int tb_group_unique_id(void* id_out);
/* This process's rank over ctx's GPU. Non-blocking NCCL initialisation with a deadline of
 * timeout_ms: if a rank never joins, every waiting rank aborts its communicator and returns
 * TB_ERR_TIMEOUT (the same deadline bounds every later tb_group_gather). */
int tb_group_init_rank(tb_ctx* ctx, int64_t nranks, int64_t rank, const void* id, int64_t timeout_ms,
                       tb_group** out);
/* Group size, global rank of this process's first GPU, GPUs this process drives. */
int tb_group_size(tb_group* g, int64_t* nranks, int64_t* first_local_rank, int64_t* local_gpus);
/* Context of local GPU `local` (tb_group_init groups own them; do not shut them down). */
int tb_group_context(tb_group* g, int64_t local, tb_ctx** ctx);
/* Gather to rank 0: rank r sends bytes_per_rank[r] bytes (every rank passes the whole array)
 * from its device buffer send_local[i] (i = local GPU index), and rank 0 receives them back to
 * back in rank order at recv_root (device memory of rank 0's GPU; ignored on other ranks).
 * Blocks until this process's part is complete, within the group's deadline (then the
 * communicators are aborted and TB_ERR_TIMEOUT returned; the group is unusable afterwards). */
int tb_group_gather(tb_group* g, const void* const* send_local, const int64_t* bytes_per_rank, void* recv_root);
/* tb_group_gather split in two: enqueue the transfers on the local contexts' streams and return
 * (they run in stream order after the work already queued), then wait, within the deadline, for
 * the local streams to drain. */
int tb_group_gather_async(tb_group* g, const void* const* send_local, const int64_t* bytes_per_rank,
                          void* recv_root);
int tb_group_wait(tb_group* g);
int tb_group_destroy(tb_group* g);

/* ---- whole-network executor (TNNet.forward / predict, source/nnet.pas:275-317,452-472) --- */
typedef struct tb_net tb_net;
#define TB_LAYER_CONV      1
#define TB_LAYER_SHORTCUT  2
#define TB_LAYER_ROUTE     3
#define TB_LAYER_UPSAMPLE  4
#define TB_LAYER_YOLO      5
#define TB_LAYER_MAXPOOL   6
#define TB_LAYER_CONNECTED 7
#define TB_LAYER_SOFTMAX   8
#define TB_LAYER_AVGPOOL   9

int tb_net_create(tb_ctx* ctx, int64_t batch, int64_t channels, int64_t height, int64_t width,
                  tb_net** out);
int tb_net_destroy(tb_net* net);
/* Each add returns the new layer's index (>= 0) or a negative TB_ERR_*. Weights are host
 * arrays in the reference layout; they are copied (and uploaded at finalize). BN arrays may be
 * NULL when batch_normalize == 0. */
int tb_net_add_conv(tb_net* net, int64_t filters, int64_t ksize, int64_t stride, int64_t pad,
                    int64_t activation, int64_t batch_normalize, const float* weights_host,
                    const float* biases_host, const float* scales_host,
                    const float* rolling_mean_host, const float* rolling_variance_host);
int tb_net_add_shortcut(tb_net* net, int64_t from, int64_t activation);
int tb_net_add_route(tb_net* net, int64_t n, const int64_t* layers);
int tb_net_add_upsample(tb_net* net, int64_t stride, float scale);
int tb_net_add_yolo(tb_net* net, int64_t classes, int64_t n, const int64_t* mask,
                    int64_t total_anchors, const float* anchors, float scale_xy);
int tb_net_add_maxpool(tb_net* net, int64_t ksize, int64_t stride, int64_t padding);
int tb_net_add_connected(tb_net* net, int64_t outputs, int64_t activation,
                         const float* weights_host, const float* biases_host);
int tb_net_add_softmax(tb_net* net, int64_t groups, float temperature);
int tb_net_add_avgpool(tb_net* net);
/* Fusion planning switch (default on). With fusion off every layer output is materialised and
 * every layer runs its own kernel, which lets tests compare each layer with the reference. */
int tb_net_set_fusion(tb_net* net, int64_t enable);
/* TNNet.fuseBatchNorm (source/nnet.pas:268-273). */
int tb_net_fuse_batchnorm(tb_net* net);
/* Plan fusions (shortcut into conv epilogue, zero-copy route slices, yolo activation into the
 * head conv), allocate activations and upload packed weights. math_mode: TB_MATH_*. */
int tb_net_finalize(tb_net* net, int64_t math_mode);
/* Run the whole network on x (device, [batch][c][h][w]); use_graph != 0 replays a CUDA graph
 * captured on first use (per input pointer). The graph runs on the context's own stream, ordered
 * after prior work on the launch stream and before later work on it (event fork / join), so it
 * behaves like an eager forward on the launch stream. Asynchronous. */
int tb_net_forward(tb_net* net, const float* x, int64_t use_graph);
/* Device pointer / element count of a layer's output (per batch) and its batch stride. */
int tb_net_layer_output(tb_net* net, int64_t layer, const float** ptr, int64_t* count_per_image,
                        int64_t* batch_stride);
/* Layout of a layer's output: *pixel_stride = 0 for NCHW ([batch][c][h][w], batch stride as
 * tb_net_layer_output reports); > 0 for NHWC ([batch][h][w][pixel_stride], the layer's channels
 * first in each pixel). A TF32 network of convs, shortcuts, routes, upsamples and fused yolo
 * heads keeps its activations NHWC (its yolo outputs stay NCHW); set TB_NET_NHWC=0 before
 * tb_net_finalize to keep every activation NCHW. */
int tb_net_layer_layout(tb_net* net, int64_t layer, int64_t* pixel_stride);
int tb_net_layer_count(tb_net* net, int64_t* count);
/* Device launches the last tb_net_forward issued (graph replay counts its kernel nodes). */
int tb_net_launch_count(tb_net* net, int64_t* count);
/* Conv FLOPs (2*M*N*K summed over conv / connected layers) of one forward at this batch. */
int tb_net_flops(tb_net* net, double* flops);
/* Per-layer timing (replaces the reference's TMetrics / USE_TELEMETRY per-layer clock,
 * source/nbaselayer.pas:129-178, which synchronises after every op): runs one eager forward
 * with a CUDA event between layers and writes each layer's device milliseconds to ms_out
 * (layer_count entries; 0 for layers fused into their neighbour). Blocks. */
int tb_net_profile(tb_net* net, const float* x, double* ms_out);

/* Network shape as created: batch and the per-image input shape. */
int tb_net_input_shape(tb_net* net, int64_t* batch, int64_t* channels, int64_t* height,
                       int64_t* width);
/* One layer's description (host-side; valid before and after finalize). Fields that do not apply
 * to the layer's type are 0. */
typedef struct tb_layer_info {
    int64_t type;                      /* TB_LAYER_* */
    int64_t c, h, w;                   /* input shape per image */
    int64_t out_c, out_h, out_w;       /* output shape per image */
    int64_t filters, ksize, stride, pad, activation, batch_normalize;  /* conv / connected / maxpool */
    int64_t from;                      /* shortcut: absolute source layer */
    int64_t n_inputs;                  /* route: number of inputs (TB_PARAM_ROUTE_INPUTS) */
    int64_t classes, n, total_anchors; /* yolo */
    int64_t groups;                    /* softmax */
    float scale;                       /* upsample scale, yolo scale_x_y, softmax temperature */
    float reserved;
    int64_t weights_count;             /* floats in TB_PARAM_WEIGHTS */
} tb_layer_info;
int tb_net_layer_info(tb_net* net, int64_t layer, tb_layer_info* out);
/* Copy a layer's host-side parameter array into dst (float, or int64 for the two index arrays).
 * dst == NULL only reports the element count. BN arrays are empty once batchnorm is folded. */
#define TB_PARAM_WEIGHTS       0
#define TB_PARAM_BIASES        1
#define TB_PARAM_SCALES        2
#define TB_PARAM_ROLLING_MEAN  3
#define TB_PARAM_ROLLING_VAR   4
#define TB_PARAM_ROUTE_INPUTS  5   /* int64, absolute layer indices */
#define TB_PARAM_YOLO_MASK     6   /* int64 */
#define TB_PARAM_YOLO_ANCHORS  7   /* float, 2 per anchor */
int tb_net_layer_param(tb_net* net, int64_t layer, int64_t which, void* dst, int64_t capacity,
                       int64_t* count);

/* ---- input pipeline (TImageData, source/ntypes.pas) ---------------------------------------- */
/* A decoded 8-bit image in device memory: rows of width pixels, row_stride bytes apart, each
 * pixel bytes_per_pixel bytes (1: gray, 3: RGB / BGR, 4: RGBA / BGRA; alpha is ignored). */
typedef struct tb_image {
    const uint8_t* pixels;
    int64_t width, height, row_stride, bytes_per_pixel;
    int64_t bgr;                /* 1: bytes in B, G, R order */
} tb_image;
/* Byte-to-float scale of the pixel values. TB_PIXEL_FPC: v * 257 / 65280, what the FPC build's
 * TImageData.loadFromFile gives (FPImage widens a byte to 16 bits as v * 257, the reference
 * divides by $ff00; source/ntypes.pas:684-690). TB_PIXEL_255: v / 255 (the Delphi build, :713-719). */
#define TB_PIXEL_FPC 0
#define TB_PIXEL_255 1
/* TImageData.loadFromFile + resize or letterBoxEx + toTensor for a batch of images
 * (source/ntypes.pas:651-657, 669-694, 837-897, 922-943), on the device, bit-exact with the
 * reference's single-precision arithmetic: image i becomes planes [3][out_h][out_w] at
 * out + i * out_batch_stride (0 = 3 * out_h * out_w), ready to be the network's input.
 * keep_aspect = 0: resize to out_w x out_h (the YOLO sample's img.resize); 1: letterBoxEx
 * (aspect kept, centred, border 0.5). ratio_out (n floats) and placement_out (n x 4 int64: resized
 * width, height, x offset, y offset) are host arrays, may be NULL. Resized sides must be >= 2.
 * Asynchronous on the context stream. */
int tb_images_to_tensor(tb_ctx* ctx, int64_t n, const tb_image* images_host, int64_t out_w,
                        int64_t out_h, int64_t keep_aspect, int64_t pixel_scale, float* out,
                        int64_t out_batch_stride, float* ratio_out, int64_t* placement_out);

/* ---- darknet model files (TDarknetParser, source/nparser.pas) ------------------------------ */
/* TDarknetParser.Create + loadWeights (source/nparser.pas:782-940, 1275-1340): parse a darknet
 * .cfg file into a new, unfinalized tb_net and, when weights_path is not NULL, read a darknet
 * .weights file into it (cutoff > 0: only the first cutoff layers, as loadWeights' cutoff).
 * batch > 0 overrides the [net] batch the way TDarknetParser.Create does (it applies when
 * batch / subdivisions * subdivisions of the cfg differs from it). ctx may be NULL for a
 * host-only net. Supported sections: [net], [convolutional], [connected] (batchnorm folded on
 * load), [maxpool], [avgpool], [softmax], [route], [shortcut], [upsample], [yolo], [dropout]
 * (identity at inference, kept as a one-input route so layer indices match the cfg); any other
 * section or option value outside the executor's scope returns TB_ERR_UNSUPPORTED naming it.
 * Layers past the end of the weights file keep zero weights (the reference stops at EOF); a
 * file that ends inside a layer's arrays is TB_ERR_INVALID. */
int tb_darknet_load(tb_ctx* ctx, const char* cfg_path, const char* weights_path, int64_t batch,
                    int64_t cutoff, tb_net** out);
/* TDarknetParser.saveWeights (source/nparser.pas:1394-1440): header major 0, minor 2, revision 5,
 * 64-bit seen, then per conv layer biases, [scales, rolling mean, rolling variance when its
 * batchnorm is not folded], weights; per connected layer biases, weights. */
int tb_darknet_save_weights(tb_net* net, const char* weights_path, int64_t seen);

/* ---- diagnostics -------------------------------------------------------------------------- */
/* FP32 FFMA throughput of this GPU (TFLOP/s) from a register-resident FMA loop on every SM;
 * the roofline denominator of the FP32 CUDA-core conv path (no reference counterpart). Blocks. */
int tb_diag_fp32_fma_tflops(tb_ctx* ctx, double* tflops);
/* Integer-pipe rate of the XNOR conv's inner step (xor + popcount + add of 32-bit words, in
 * registers, on every SM) in Tbit-MAC/s (32 per popcount): the roofline denominator of
 * tb_xnor_conv_fwd (no reference counterpart). Blocks. */
int tb_diag_popc_tbitmac(tb_ctx* ctx, double* tbitmac);
/* tcgen05.mma kind::tf32 issue rate with operands resident in shared memory (M 128, N 256,
 * K 8, one CTA per SM): cycles per MMA and the implied TFLOP/s at 1965 MHz, for MN-major
 * (kmajor = 0, the conv kernel's layout) or K-major (kmajor = 1) operands (no reference
 * counterpart). Blocks. */
int tb_diag_tc_mma_rate(tb_ctx* ctx, int64_t kmajor, double* tflops, double* cycles_per_mma);
/* One launch of the TF32 tensor-core conv on this geometry (bias, batchnorm and residual off)
 * with per-CTA cycle counters; out12 = averages over CTAs of: producer total cycles, producer
 * cycles waiting for a free stage, MMA-issuer total, MMA waiting for loaded stages, MMA waiting
 * for a free accumulator, epilogue total, epilogue waiting for a finished accumulator, tiles
 * per CTA, epilogue cycles in TMEM loads, epilogue cycles in the per-value work and stores,
 * 0, 0 (no reference counterpart). Blocks. */
int tb_diag_conv_tc_phases(tb_ctx* ctx, const tb_conv_desc* d, const float* x, const float* packed_w, float* y,
                           double* out12);
/* The same counters for one launch of the NHWC tensor-core conv (tb_conv2d_fwd_nhwc's kernel;
 * entry 8 = epilogue cycles in TMEM loads or split-K partial sums, entry 9 = all per-tile
 * epilogue work, entry 10 = the launch's span from the first CTA's start to the last CTA's end
 * and entry 11 = the longest CTA, both in ns of the GPU's global timer). Blocks. */
int tb_diag_conv_nhwc_phases(tb_ctx* ctx, const tb_conv_desc* d, const float* x, int64_t x_pixel_stride,
                             const float* packed_w, float* y, int64_t y_pixel_stride, double* out12);

#ifdef __cplusplus
}
#endif
#endif /* TENSORIUM_B200_H */
