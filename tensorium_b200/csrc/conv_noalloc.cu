// conv_noalloc.cu -- tb_conv2d_fwd_noalloc: the fused conv forward for callers that must not
// allocate device memory.
//
// Some hosts cannot call cudaMalloc at the point where they run a layer: a process whose
// device memory is handed out up front by a framework's arena, code running while another
// component holds the allocator, or a real-time loop where an allocation's latency (or
// failure) is not acceptable.  tb_conv2d_fwd with TB_MATH_FP32_TILED may grow the context's
// workspace for split-K partial sums; this variant runs the same tiled kernels but keeps that
// scratch (partial sums and the per-tile arrival counters) in one fixed array in device memory
// that is part of the library image.  (The default FP32 path, TB_MATH_FP32, needs no scratch.)
// The array's device address is cached per device index for the life of the process; the
// library does not support cudaDeviceReset of a device it has run this entry point on.
#include "conv.cuh"

#include <mutex>

namespace {

// Scratch capacity: 16 MiB of split-K partial sums plus 64 KiB of arrival counters.  Every GPU
// that loads the library holds this array until the process exits.
constexpr int64_t NOALLOC_PARTIAL_FLOATS = (int64_t)4 << 20;
constexpr int64_t NOALLOC_COUNTERS = 16384;
constexpr int64_t NOALLOC_BYTES = NOALLOC_PARTIAL_FLOATS * 4 + NOALLOC_COUNTERS * 4;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

// The array's name in host code is only a host-side stand-in; kernels need its device address,
// looked up once per device (with that device current) and cached here.
std::mutex g_mu;
void* g_scratch_addr[64] = {nullptr};

int scratch_address(int device, unsigned char** out) {
    if (device < 0 || device >= 64) return tbi::fail(TB_ERR_UNSUPPORTED, "noalloc conv: device index %d >= 64", device);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_addr[device]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) return tbi::cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
        g_scratch_addr[device] = ptr;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[device]);
    return TB_OK;
}

}  // namespace

using namespace tbi;

extern "C" int tb_conv2d_fwd_noalloc(tb_ctx* ctx, const tb_conv_desc* d, const float* x,
                                     const float* packed_w, const float* bias, const float* bn_scale,
                                     const float* bn_mean, const float* bn_variance,
                                     const float* residual, float* y) {
    TB_ENTER(ctx);
    ConvGeom g;
    int r = conv_geom(d, &g);
    if (r != TB_OK) return r;
    if (g.B == 0) return TB_OK;
    if (!x || !packed_w || !y) return fail(TB_ERR_INVALID, "noalloc conv: null x, weights or y");
    if (bn_mean && !bn_variance) return fail(TB_ERR_INVALID, "noalloc conv: bn_mean given without bn_variance");
    if (!aligned16(packed_w)) return fail(TB_ERR_INVALID, "noalloc conv: packed weights must be 16-byte aligned");
    if (!act_supported(d->activation))
        return fail(TB_ERR_UNSUPPORTED, "noalloc conv: activation %lld not supported", (long long)d->activation);
    // the tile's K split is lowered until its partial sums fit the static scratch (split 1 needs
    // none); only a split pinned through the TB_CONV_FORCE test hook can still exceed it
    const int64_t need = conv_fp32_ws_floats_fit(ctx, g, x, NOALLOC_PARTIAL_FLOATS, NOALLOC_COUNTERS);
    if (need > NOALLOC_PARTIAL_FLOATS)
        return fail(TB_ERR_INVALID,
                    "noalloc conv: the pinned split needs %lld bytes of split-K scratch; the static scratch holds "
                    "%lld bytes",
                    (long long)need * 4, (long long)NOALLOC_PARTIAL_FLOATS * 4);
    unsigned char* base = nullptr;
    r = scratch_address(ctx->device, &base);
    if (r != TB_OK) return r;
    float* partials = reinterpret_cast<float*>(base);
    int* counters = reinterpret_cast<int*>(base + NOALLOC_PARTIAL_FLOATS * 4);
    if (need > 0) {
        // the counters must start at zero; a previous call may have been cut short
        TB_CHECK_CUDA(cudaMemsetAsync(counters, 0, NOALLOC_COUNTERS * sizeof(int), ctx->stream));
    }
    return conv_fp32_launch(ctx, g, x, packed_w, bias, bn_scale, bn_mean, bn_variance, residual, y,
                            (int)d->activation, 0, partials, NOALLOC_PARTIAL_FLOATS, nullptr, counters,
                            NOALLOC_COUNTERS, false);
}
