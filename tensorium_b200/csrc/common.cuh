// common.cuh -- shared plumbing of the tensorium_b200 C-ABI library: context, error reporting,
// launch helpers and the device-side activation functions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string>
#include <cstdio>
#include <cstdarg>
#include <utility>

#include "../../include/tensorium_b200.h"

struct tb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;      // current launch stream
    cudaStream_t own_stream = nullptr;  // stream created by tb_init
    void* ws = nullptr;                 // split-K / scratch workspace
    size_t ws_bytes = 0;
    int* d_status = nullptr;            // device status word (kernels report errors here)
    int64_t math_mode = TB_MATH_FP32;
    int sm_count = 148;
    int max_smem_optin = 0;
    cudaEvent_t fork = nullptr, join = nullptr;  // order own_stream work with `stream`
    int* tile_cnt = nullptr;                      // split-K arrival counters (zeroed, self-resetting)
    int64_t tile_cnt_len = 0;
    int pdl = 0;  // launches through tbi::launch may overlap the previous kernel's tail (set while
                  // a network forward is captured)
};

namespace tbi {

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
// Make ctx's device current on this thread; returns TB_OK or an error code.
int enter(tb_ctx* ctx);
// Ensure the workspace holds at least `bytes` (may allocate; not capture-safe).
int ensure_workspace(tb_ctx* ctx, size_t bytes);
// Check the last launch.
int check_launch(const char* what);
// Keep the stream busy for about `us` microseconds (a bounded sleep on the GPU timer), so that the
// launches a timing loop enqueues behind it start back to back: autotuners time device work, not
// the host's launch overhead.
void stream_delay_us(tb_ctx* ctx, int us);

// Programmatic dependent launch. A kernel launched through `launch` while ctx->pdl is set may
// start while the previous kernel on the stream is still running; it must execute
// TB_GRID_DEP_ENTRY() before touching global memory that earlier kernels write or read: that waits
// until every earlier kernel has completed and its writes are visible, then lets the next kernel
// be scheduled. Outside such a launch the two instructions return at once.
#define TB_GRID_DEP_ENTRY()                                                      \
    do {                                                                         \
        asm volatile("griddepcontrol.wait;\n" ::: "memory");                     \
        asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");        \
    } while (0)

template <typename... KArgs, typename... Args>
int launch(tb_ctx* ctx, const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
           Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    if (ctx->pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, what);
    return check_launch(what);
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid-stride launch size for n work items of `per_thread` items each.
inline unsigned grid_for(int64_t n, int threads, int sm_count, int per_thread = 1) {
    int64_t blocks = ceil_div(ceil_div(n, per_thread), threads);
    int64_t cap = (int64_t)sm_count * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

bool act_supported(int64_t act);

}  // namespace tbi

#define TB_CHECK_CUDA(call)                                              \
    do {                                                                  \
        cudaError_t _e = (call);                                          \
        if (_e != cudaSuccess) return tbi::cuda_fail(_e, #call);          \
    } while (0)

#define TB_ENTER(ctx)                                                    \
    do {                                                                  \
        if (!(ctx)) return tbi::fail(TB_ERR_INVALID, "null context");     \
        int _r = tbi::enter(ctx);                                         \
        if (_r != TB_OK) return _r;                                       \
    } while (0)

// ---------------------------------------------------------------------------------------
// Device activations: the scalar forms of activate_array (source/nactivation.pas:272-401,
// 508-621).  Untyped Pascal real constants and System.exp are evaluated in double and
// rounded to single, so the arithmetic here is done in double where the reference does.
// ---------------------------------------------------------------------------------------
static __device__ __noinline__ float tb_logistic(float x) {
    return (float)(1.0 / (1.0 + exp(-(double)x)));
}

static __device__ __noinline__ float tb_activate_slow(float x, int a);

// Activation formats of the tensor-core networks (NHWC plan). TF32: each value an fp32 rounded to
// nearest TF32 (what kind::tf32 reads). BF16 pair: each 32-bit slot holds two bf16, hi =
// bf16(v) in the low half and lo = bf16(v - hi) in the high half, so a 32-channel fp32 row is a
// 64-element bf16 row whose even / odd entries are the hi / lo parts (kind::f16 reads it as is).
__device__ __forceinline__ float tb_tf32_rna(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
    return __uint_as_float(u);
}
__device__ __forceinline__ uint32_t tb_bf16_rn_bits(float x) {  // round to nearest even, finite x
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) == 0x7f800000u) return u >> 16;
    return (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ float tb_pair_encode(float v) {
    const uint32_t h = tb_bf16_rn_bits(v);
    const float r = __fsub_rn(v, __uint_as_float(h << 16));
    return __uint_as_float(h | (tb_bf16_rn_bits(r) << 16));
}
__device__ __forceinline__ float tb_pair_decode(float s) {
    const uint32_t u = __float_as_uint(s);
    return __fadd_rn(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
// store / load one activation in the network's format (pair = 0: TF32 rounding)
__device__ __forceinline__ float tb_fmt_store(float v, int pair) { return pair ? tb_pair_encode(v) : tb_tf32_rna(v); }
__device__ __forceinline__ float tb_fmt_load(float s, int pair) { return pair ? tb_pair_decode(s) : s; }

// Common activations inline, the rest out of line (keeps the unrolled conv epilogues small).
__device__ __forceinline__ float tb_activate_dev(float x, int a) {
    if (a == TB_ACT_LEAKY || a == TB_ACT_REVLEAKY) return x < 0.f ? __fmul_rn(x, 0.1f) : x;
    if (a == TB_ACT_LINEAR) return x;
    if (a == TB_ACT_RELU) return x > 0.f ? x : x * 0.0f;
    return tb_activate_slow(x, a);
}

// Full activate_array switch; defined in every translation unit that includes this header
// (static linkage keeps the per-object copies private).
static __device__ __noinline__ float tb_activate_slow(float x, int a) {
    switch (a) {
    case TB_ACT_LOGISTIC: return tb_logistic(x);
    case TB_ACT_RELU: return x > 0.f ? x : x * 0.0f;
    case TB_ACT_RELU6: return (x > 0.f && x <= 6.f) ? x : x * 0.0f;
    case TB_ACT_RELIE: return x > 0.f ? x : (float)(0.01 * (double)x);
    case TB_ACT_LINEAR: return x;
    case TB_ACT_RAMP: return (float)((double)(x > 0.f ? x : x * 0.0f) + 0.1 * (double)x);
    case TB_ACT_TANH: {
        float px = (float)exp((double)x), nx = (float)exp(-(double)x);
        return __fdiv_rn(px - nx, px + nx);
    }
    case TB_ACT_PLSE:
        if (x < -4.f) return (float)(0.01 * ((double)x + 4.0));
        if (x > 4.f) return (float)(0.01 * ((double)x - 4.0) + 1.0);
        return (float)(0.125 * (double)x + 0.5);
    case TB_ACT_REVLEAKY:
    case TB_ACT_LEAKY: return x < 0.f ? __fmul_rn(x, 0.1f) : x;  // leaky_array: single multiply by 0.1f
    case TB_ACT_ELU:
        return (float)((x >= 0.f ? (double)x : 0.0) + (x < 0.f ? exp((double)x) - 1.0 : 0.0));
    case TB_ACT_LOGGY: return (float)(2.0 / (1.0 + exp(-(double)x)) - 1.0);
    case TB_ACT_HARDTAN: return x < -1.f ? -1.f : (x > 1.f ? 1.f : x);
    case TB_ACT_LHTAN:
        if (x < 0.f) return (float)(0.001 * (double)x);
        if (x > 1.f) return (float)(0.001 * ((double)x - 1.0) + 1.0);
        return x;
    case TB_ACT_SELU:
        return (float)((x >= 0.f ? 1.0507 * (double)x : 0.0) +
                       (x < 0.f ? 1.0507 * 1.6732 * (exp((double)x) - 1.0) : 0.0));
    default: return x;
    }
}
