// conv_tc.cuh -- tcgen05 (5th-gen tensor core) TF32 implicit-GEMM convolution: device helpers.
//
// Shared-memory operand tiles use the one canonical MN-major layout that tcgen05 accepts for
// 32-bit (TF32) operands, "128-byte swizzle with 32-byte atomicity" (descriptor layout type 1,
// the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B): rows of 128 bytes (32 fp32
// along M or N) hold one K index each; inside a group of 4 rows the 32-byte chunk index is XORed
// with the row index (byte-address bits [5,7) ^= bits [7,9)).  A TMA box of 32 (M or N) x 32 (K)
// fills 4 KB: 8 K-groups of 512 bytes (the descriptor's stride byte offset); boxes along M or N
// are 4 KB apart (leading byte offset).  One K=8 MMA spans two K-groups, so the k-th MMA of a
// 32-deep stage starts 1024*k bytes into each box.  Tiles start on 1024-byte boundaries.
#pragma once
#include "conv.cuh"

#include <cuda.h>

namespace tbi {
namespace tc {

// --- mbarrier ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(a), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(a) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
    unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(a), "r"(bytes) : "memory");
}

// Waits for the phase with this parity, the thread suspended in hardware for up to ~1 us per try.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    unsigned ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after ~2^32 SM clock cycles (about 2 s), or at once when another role
// has aborted; on timeout sets *abort and the device status word.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, volatile int* abort,
                                                  int* status, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > (1ll << 32)) break;
    }
    *abort = 1;
    if (status) atomicExch(status, code);
    return false;
}

// Wait with a poll limit only (used to drain copies already in flight after an abort).
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, unsigned parity) {
    const long long t0 = clock64();
    while (clock64() - t0 < (1ll << 31))
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// --- TMA (tensor copies global -> shared of this CTA only, completion counted on an mbarrier) ---
__device__ __forceinline__ void tma_load_2d(unsigned dst, const void* tmap, uint64_t* bar, int x, int y) {
    unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(b), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(unsigned dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
    unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(b), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(unsigned dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                            int w) {
    unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(b), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// fp32 -> tf32 (10-bit mantissa), round to nearest with ties away from zero: add half of the
// tf32 unit in the last place (bit 12) to the magnitude bits and clear the 13 low bits (a carry
// into the exponent is the correct rounding up, to infinity past the largest finite value);
// infinities and NaNs pass unchanged.  The tensor core itself drops those bits (truncation),
// which biases every product toward zero; operands rounded here carry an unbiased error.
__device__ __forceinline__ float to_tf32_rna(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
    return __uint_as_float(u);
}

// --- tcgen05 -----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    unsigned a = (unsigned)__cvta_generic_to_shared(dst_smem);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(a), "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, one CTA
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// kind::f16 with BF16 A and B (both operands of one MMA the same type), FP32 accumulate
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// arrive on `bar` once every tcgen05 op issued so far by this thread has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(a)
                 : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// tmem_ld16 split in two: the load is issued, and the registers are valid only after
// tmem_wait16 on the same array (the wait takes them as operands, so no use can move above it)
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait16(uint32_t* r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// shared-memory matrix descriptor: MN-major, 128-byte swizzle with 32-byte atoms (layout type 1),
// version 1
__device__ __forceinline__ uint64_t smem_desc_mn_sw128_32b(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // version (Blackwell)
    d |= (uint64_t)1 << 61;  // SWIZZLE_128B_BASE32B
    return d;
}

// instruction descriptor: F32 accumulate, TF32 A and B, both MN-major, shape M x N
__host__ __device__ constexpr uint32_t idesc_tf32_mn(int M, int N) {
    return (1u << 4)                       // c_format F32
           | (2u << 7) | (2u << 10)        // a_format, b_format TF32
           | (1u << 15) | (1u << 16)       // a_major, b_major = MN
           | ((uint32_t)(N >> 3) << 17)    // n_dim
           | ((uint32_t)(M >> 4) << 24);   // m_dim
}


// --- the 8 epilogue warps (256 threads) of the conv kernel: named barrier 1 ---------------
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 256;\n" ::: "memory"); }

// barrier of the epilogue warps that also tells every thread whether any thread passed `v`
__device__ __forceinline__ bool epi_any(bool v) {
    unsigned r;
    asm volatile(
        "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, 1, 256, p;\nselp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((unsigned)v)
        : "memory");
    return r != 0;
}

// --- CTA pairs (cta_group::2): a cluster of 2 CTAs on two SMs computes one M = 256 tile -----
// the GPU's global nanosecond timer
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// arrive on the mbarrier at the same shared offset in CTA `rank` of the cluster
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, unsigned rank) {
    unsigned a = (unsigned)__cvta_generic_to_shared(bar), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(ra) : "memory");
}

template <int CTAS>
__device__ __forceinline__ void tmem_alloc_g(uint32_t* dst_smem, uint32_t ncols) {
    unsigned a = (unsigned)__cvta_generic_to_shared(dst_smem);
    if constexpr (CTAS == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(a), "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    } else {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(a), "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::);
    }
}

template <int CTAS>
__device__ __forceinline__ void tmem_dealloc_g(uint32_t taddr, uint32_t ncols) {
    if constexpr (CTAS == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
    else
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}

// D (+)= A * B; with CTAS == 2, issued by the pair's even CTA: A rows and B columns are read
// half from each CTA's shared memory at the same offsets, D rows half into each CTA's TMEM.
template <int CTAS>
__device__ __forceinline__ void mma_tf32_g(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                           uint32_t accumulate) {
    if constexpr (CTAS == 1)
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
            "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
    else
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
            "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// kind::f16 (BF16 A and B) for one CTA or the pair, as mma_tf32_g
template <int CTAS>
__device__ __forceinline__ void mma_bf16_g(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                           uint32_t accumulate) {
    if constexpr (CTAS == 1)
        mma_bf16(tmem_d, desc_a, desc_b, idesc, accumulate);
    else
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
            "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

// arrive on `bar` (in both CTAs of the pair when CTAS == 2: one commit to each CTA's barrier,
// the peer's addressed through its shared::cluster window) once every tcgen05 op issued so far
// by this thread has completed
template <int CTAS>
__device__ __forceinline__ void mma_commit_g(uint64_t* bar) {
    unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    if constexpr (CTAS == 1) {
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(a)
                     : "memory");
    } else {
        unsigned peer;
        asm volatile("mapa.shared::cluster.u32 %0, %1, 1;\n" : "=r"(peer) : "r"(a));
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(a)
                     : "memory");
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(peer)
                     : "memory");
    }
}

// TMA loads into this CTA's shared memory; with CTAS == 2 the completed bytes are counted on the
// mbarrier of the pair's even CTA (the one whose MMA thread waits for both halves)
template <int CTAS>
__device__ __forceinline__ unsigned tma_bar(uint64_t* bar) {
    unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    return CTAS == 1 ? b : (b & 0xFEFFFFFFu);
}

template <int CTAS>
__device__ __forceinline__ void tma_load_2d_g(unsigned dst, const void* tmap, uint64_t* bar, int x, int y) {
    if constexpr (CTAS == 1)
        tma_load_2d(dst, tmap, bar, x, y);
    else
        asm volatile(
            "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(tmap)), "r"(tma_bar<2>(bar)), "r"(x), "r"(y)
            : "memory");
}

template <int CTAS>
__device__ __forceinline__ void tma_load_3d_g(unsigned dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
    if constexpr (CTAS == 1)
        tma_load_3d(dst, tmap, bar, x, y, z);
    else
        asm volatile(
            "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];\n" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(tmap)), "r"(tma_bar<2>(bar)), "r"(x), "r"(y), "r"(z)
            : "memory");
}

template <int CTAS>
__device__ __forceinline__ void tma_load_4d_g(unsigned dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                              int w) {
    if constexpr (CTAS == 1)
        tma_load_4d(dst, tmap, bar, x, y, z, w);
    else
        asm volatile(
            "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];\n" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(tmap)), "r"(tma_bar<2>(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
            : "memory");
}

}  // namespace tc

// ---- A-operand planning shared by the TF32 kernel and the FP32 TMA kernel (conv_tc.cu) ----
constexpr int TC_MAX_KH = 8;
// How the A operand is laid out for one geometry.
enum TcMode {
    TC_TAPS = 0,     // tap replicas P[s][ph][b][c][Hrep][Wp] (channels % 32 == 0)
    TC_INPLACE = 1,  // 1x1 stride-1 unpadded, H*W % 4 == 0: x itself on a flat pixel grid
    TC_IM2COL = 2,   // any other channel count: P[b][k][OH][Wp], one row per packed weight row
};

struct TcPlan {
    int mode;
    int64_t Wp, NPH, pad_top, Hrep, Lp, PS;  // PS: replica plane stride (elements)
    int64_t Cr;                              // channels of the GEMM view (k rows per tap)
    int rowoff[TC_MAX_KH], phase[TC_MAX_KH];
};

void tc_plan(const ConvGeom& g, TcPlan* pl, int cmul);
// replica floats of a plan, rounded up to 64
int64_t replica_floats(const ConvGeom& g, const TcPlan& pl);
// fp32 tensor map (swizzle `sw`, zero fill out of bounds)
int encode_map(CUtensorMap* m, const float* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
               const uint32_t* box, CUtensorMapSwizzle sw);
int tc_prepare_a(tb_ctx* ctx, const ConvGeom& g, const float* x, float* scratch, bool round, int box_k, int cmul,
                 CUtensorMapSwizzle sw, CUtensorMap* a4, CUtensorMap* a1, CUtensorMap* tail, TcPlan* plo,
                 int* kmaps_o, int* g_full_o, int64_t* launches);
}  // namespace tbi
