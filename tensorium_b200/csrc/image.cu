// image.cu -- the input pipeline in front of the network: decoded 8-bit images to the network's
// planar fp32 input batch, with the reference's resize or letterbox, in one kernel.
//
// The reference does this on the CPU per image (TImageData.loadFromFile, resize, letterBoxEx,
// toTensor: source/ntypes.pas:651-657, 669-694, 837-943; the YOLO sample calls resize or
// letterBoxEx before predict, Samples/FPC/MSCOCO_Yolo/MSCOCOYolo.pas:348-350,454). Here the
// pixels stay 8-bit until they are on the GPU (a quarter of the fp32 bytes cross PCIe), and one
// thread makes one output pixel of one image: it reads the (up to) 2x2 source pixels the
// reference's two separable passes would combine and repeats their single-precision operations
// in the same order (`__fmul_rn` / `__fadd_rn`, never contracted), so the result is the
// reference's bit for bit without the intermediate column-resized image.
#include "common.cuh"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

using namespace tbi;

namespace {

constexpr int kJobsPerLaunch = 64;
constexpr int64_t kRowsSmemMax = 64 * 1024;  // rows wider than ~31 KB take the direct kernel

// TB_IMAGES_DIRECT=1 forces the direct (unstaged) kernel (the tests compare both forms)
bool t_images_direct() {
    const char* e = getenv("TB_IMAGES_DIRECT");
    return e && e[0] == '1';
}

struct ImageJob {
    const uint8_t* px;
    int64_t row_stride;
    int64_t out_off;       // first float of this image's [3][out_h][out_w] block
    int32_t w, h, bpp, bgr;
    int32_t new_w, new_h;  // size of the resized image
    int32_t dx, dy;        // where it sits in the output (letterbox offsets)
    float w_scale, h_scale;
};

struct ImageLaunch {
    ImageJob job[kJobsPerLaunch];
    int32_t out_w, out_h;
    int64_t plane;         // out_w * out_h
    int32_t pixel_scale;   // TB_PIXEL_*
};

// Byte -> float, the correctly rounded quotient the reference stores (v * 257 / 65280 or v / 255,
// computed there in double and rounded to single). In registers instead of a table (a shared-memory
// table costs bank conflicts on every tap): for v * 257 / 65280 one float multiply by
// fl(257 / 65280) is already correctly rounded for all 256 bytes; for v / 255 the multiply by
// fl(1 / 255) is corrected with one residual step (two explicit FMAs). scale_ok() checks both
// identities on every byte on the host before the first launch.
constexpr float kFpcScale = (float)(257.0 / 65280.0);
constexpr float kInv255 = (float)(1.0 / 255.0);

__host__ __device__ __forceinline__ float byte_value(unsigned v, int mode) {
#ifdef __CUDA_ARCH__
    const float x = (float)v;
    if (mode == TB_PIXEL_FPC) return __fmul_rn(x, kFpcScale);
    const float q = __fmul_rn(x, kInv255);
    const float e = __fmaf_rn(-q, 255.0f, x);
    return __fmaf_rn(e, kInv255, q);
#else
    const float x = (float)v;
    if (mode == TB_PIXEL_FPC) { volatile float p = x * kFpcScale; return p; }
    volatile float q = x * kInv255;
    const float e = std::fma(-(float)q, 255.0f, x);
    return std::fma(e, kInv255, (float)q);
#endif
}

bool scale_ok() {
    static const bool ok = [] {
        for (unsigned v = 0; v < 256; ++v) {
            if (byte_value(v, TB_PIXEL_FPC) != (float)((double)(v * 257) / 65280.0)) return false;
            if (byte_value(v, TB_PIXEL_255) != (float)((double)v / 255.0)) return false;
        }
        return true;
    }();
    return ok;
}

__device__ __forceinline__ float px_at(const ImageJob& j, int mode, int x, int y, int ch) {
    const uint8_t* p = j.px + (int64_t)y * j.row_stride + (int64_t)x * j.bpp;
    const int k = j.bpp == 1 ? 0 : (j.bgr ? 2 - ch : ch);
    return byte_value(p[k], mode);
}

// TImageData.resize's first pass at (column xr, source row y): linear between two source columns,
// the last column taken as is.
__device__ __forceinline__ float column_pass(const ImageJob& j, int mode, bool edge, int ix,
                                             float fx, int y, int ch) {
    if (edge) return px_at(j, mode, j.w - 1, y, ch);
    const float a = __fmul_rn(__fsub_rn(1.0f, fx), px_at(j, mode, ix, y, ch));
    const float b = __fmul_rn(fx, px_at(j, mode, ix + 1, y, ch));
    return __fadd_rn(a, b);
}

__global__ void __launch_bounds__(128) k_images_to_tensor(const __grid_constant__ ImageLaunch L, float* __restrict__ out) {
    const ImageJob& j = L.job[blockIdx.z];
    const int mode = L.pixel_scale;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    if (x >= L.out_w) return;
    float* o = out + j.out_off + (int64_t)y * L.out_w + x;
    const int xr = x - j.dx, yr = y - j.dy;
    if (xr < 0 || yr < 0 || xr >= j.new_w || yr >= j.new_h) {  // letterbox border
        o[0] = 0.5f; o[L.plane] = 0.5f; o[2 * L.plane] = 0.5f;
        return;
    }
    // columns (first pass)
    const bool edge = xr == j.new_w - 1 || j.w == 1;
    int ix = 0;
    float fx = 0.0f;
    if (!edge) {
        const float sx = __fmul_rn((float)xr, j.w_scale);
        ix = (int)sx;
        fx = __fsub_rn(sx, (float)ix);
    }
    // rows (second pass): (1 - dy) * part[iy], plus dy * part[iy + 1] except on the last row
    const float sy = __fmul_rn((float)yr, j.h_scale);
    const int iy = (int)sy;
    const float fy = __fsub_rn(sy, (float)iy);
    const bool last = yr == j.new_h - 1 || j.h == 1;
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        float v = __fmul_rn(__fsub_rn(1.0f, fy), column_pass(j, mode, edge, ix, fx, iy, ch));
        if (!last) v = __fadd_rn(v, __fmul_rn(fy, column_pass(j, mode, edge, ix, fx, iy + 1, ch)));
        o[ch * L.plane] = v;
    }
}

struct RowArgs {
    const unsigned char* r0;  // staged source row iy (shared memory)
    const unsigned char* r1;  // staged source row iy + 1 (unused on the last row)
    float* o;                 // output row, plane 0
    int plane, out_w, dx, new_w, w;
    float w_scale, fy;
    bool last;
};

// Every output pixel of one row from the staged source rows (the arithmetic of column_pass and
// the row pass above), specialised on the pixel layout and byte scale.
template <int BPP, int BGR, int MODE>
__device__ __forceinline__ void row_pixels(const RowArgs& a) {
    const float gy = __fsub_rn(1.0f, a.fy);
    for (int x = threadIdx.x; x < a.out_w; x += blockDim.x) {
        const int xr = x - a.dx;
        float v[3];
        if (xr < 0 || xr >= a.new_w) {
            v[0] = v[1] = v[2] = 0.5f;
        } else {
            const bool edge = xr == a.new_w - 1 || a.w == 1;
            int c0 = a.w - 1;
            float fx = 0.0f;
            if (!edge) {
                const float sx = __fmul_rn((float)xr, a.w_scale);
                c0 = (int)sx;
                fx = __fsub_rn(sx, (float)c0);
            }
            const float gx = __fsub_rn(1.0f, fx);
            const unsigned char* p0 = a.r0 + c0 * BPP;
            const unsigned char* p1 = a.r1 + c0 * BPP;
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                const int k = BPP == 1 ? 0 : (BGR ? 2 - ch : ch);
                float q0 = byte_value(p0[k], MODE);
                if (!edge) q0 = __fadd_rn(__fmul_rn(gx, q0), __fmul_rn(fx, byte_value(p0[BPP + k], MODE)));
                float t = __fmul_rn(gy, q0);
                if (!a.last) {
                    float q1 = byte_value(p1[k], MODE);
                    if (!edge) q1 = __fadd_rn(__fmul_rn(gx, q1), __fmul_rn(fx, byte_value(p1[BPP + k], MODE)));
                    t = __fadd_rn(t, __fmul_rn(a.fy, q1));
                }
                v[ch] = t;
            }
        }
        a.o[x] = v[0];
        a.o[a.plane + x] = v[1];
        a.o[2 * a.plane + x] = v[2];
    }
}

// Row-staged form: one block per output row of one image. The (at most) two source rows the row
// pass reads are staged in shared memory with coalesced 16-byte loads (the rows' sectors are all
// touched anyway when the image is downscaled), then every output pixel of the row is made from
// shared memory with the same arithmetic as above.
__global__ void __launch_bounds__(128) k_images_rows(const __grid_constant__ ImageLaunch L, float* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int mode = L.pixel_scale;
    const ImageJob& j = L.job[blockIdx.y];
    const int y = blockIdx.x;
    float* o = out + j.out_off + (int64_t)y * L.out_w;
    const int yr = y - j.dy;
    if (yr < 0 || yr >= j.new_h) {  // letterbox border row
        for (int x = threadIdx.x; x < L.out_w; x += blockDim.x) {
            o[x] = 0.5f; o[L.plane + x] = 0.5f; o[2 * L.plane + x] = 0.5f;
        }
        return;
    }
    const float sy = __fmul_rn((float)yr, j.h_scale);
    const int iy = (int)sy;
    const float fy = __fsub_rn(sy, (float)iy);
    const bool last = yr == j.new_h - 1 || j.h == 1;
    // stage rows iy (and iy + 1): the 16-byte words that cover each row's bytes, loaded as uint4
    // inside the row and byte by byte in the partial words at its two ends
    const int64_t row_bytes = (int64_t)j.w * j.bpp;
    const int nrows = last ? 1 : 2;
    const uint8_t* row[2] = {j.px + (int64_t)iy * j.row_stride, j.px + (int64_t)(iy + 1) * j.row_stride};
    int head[2], nv[2];
    for (int r = 0; r < 2; ++r) {
        head[r] = (int)(reinterpret_cast<uintptr_t>(row[r]) & 15u);
        nv[r] = (int)((head[r] + row_bytes + 15) >> 4);
    }
    const int vecs = nv[0] > nv[1] ? nv[0] : nv[1];  // smem row pitch in uint4
    uint4* rows = reinterpret_cast<uint4*>(smem);
    for (int t = threadIdx.x; t < nrows * vecs; t += blockDim.x) {
        const int r = t >= vecs ? 1 : 0;
        const int i = t - r * vecs;
        if (i >= nv[r]) continue;
        const int64_t b0 = 16 * (int64_t)i - head[r];  // row byte of the word's first byte
        if (b0 >= 0 && b0 + 16 <= row_bytes) {
            rows[t] = __ldg(reinterpret_cast<const uint4*>(row[r] + b0));
        } else {
            unsigned char* d = reinterpret_cast<unsigned char*>(rows + t);
            for (int q = 0; q < 16; ++q)
                d[q] = (b0 + q >= 0 && b0 + q < row_bytes) ? __ldg(row[r] + b0 + q) : (unsigned char)0;
        }
    }
    __syncthreads();
    const unsigned char* r0 = reinterpret_cast<const unsigned char*>(rows) + head[0];
    const unsigned char* r1 = reinterpret_cast<const unsigned char*>(rows + vecs) + head[1];
    RowArgs a{r0, r1, o, (int)L.plane, L.out_w, j.dx, j.new_w, j.w, j.w_scale, fy, last};
    if (mode == TB_PIXEL_FPC) {
        if (j.bpp == 3) j.bgr ? row_pixels<3, 1, TB_PIXEL_FPC>(a) : row_pixels<3, 0, TB_PIXEL_FPC>(a);
        else if (j.bpp == 4) j.bgr ? row_pixels<4, 1, TB_PIXEL_FPC>(a) : row_pixels<4, 0, TB_PIXEL_FPC>(a);
        else row_pixels<1, 0, TB_PIXEL_FPC>(a);
    } else {
        if (j.bpp == 3) j.bgr ? row_pixels<3, 1, TB_PIXEL_255>(a) : row_pixels<3, 0, TB_PIXEL_255>(a);
        else if (j.bpp == 4) j.bgr ? row_pixels<4, 1, TB_PIXEL_255>(a) : row_pixels<4, 0, TB_PIXEL_255>(a);
        else row_pixels<1, 0, TB_PIXEL_255>(a);
    }
}

}  // namespace

extern "C" {

int tb_images_to_tensor(tb_ctx* ctx, int64_t n, const tb_image* images, int64_t out_w, int64_t out_h,
                        int64_t keep_aspect, int64_t pixel_scale, float* out, int64_t out_batch_stride,
                        float* ratio_out, int64_t* placement_out) {
    TB_ENTER(ctx);
    if (n < 0 || (n > 0 && (!images || !out)) || out_w < 2 || out_h < 2 || out_w > (1 << 20) || out_h > 65535)
        return fail(TB_ERR_INVALID, "tb_images_to_tensor: bad arguments");
    if (pixel_scale != TB_PIXEL_FPC && pixel_scale != TB_PIXEL_255)
        return fail(TB_ERR_INVALID, "tb_images_to_tensor: unknown pixel scale %lld", (long long)pixel_scale);
    const int64_t plane = out_w * out_h;
    if (out_batch_stride == 0) out_batch_stride = 3 * plane;
    if (out_batch_stride < 3 * plane) return fail(TB_ERR_INVALID, "tb_images_to_tensor: batch stride too small");
    if (!scale_ok()) return fail(TB_ERR_STATE, "tb_images_to_tensor: byte scale identity does not hold");
    ImageLaunch L;
    L.pixel_scale = (int32_t)pixel_scale;
    L.out_w = (int32_t)out_w;
    L.out_h = (int32_t)out_h;
    L.plane = plane;
    for (int64_t base = 0; base < n; base += kJobsPerLaunch) {
        const int64_t cnt = std::min<int64_t>(kJobsPerLaunch, n - base);
        for (int64_t q = 0; q < cnt; ++q) {
            const tb_image& im = images[base + q];
            const int64_t i = base + q;
            if (!im.pixels || im.width <= 0 || im.height <= 0 || im.width > (1 << 20) || im.height > (1 << 20) ||
                (im.bytes_per_pixel != 1 && im.bytes_per_pixel != 3 && im.bytes_per_pixel != 4) ||
                im.row_stride < im.width * im.bytes_per_pixel)
                return fail(TB_ERR_INVALID, "tb_images_to_tensor: image %lld: bad description", (long long)i);
            ImageJob& j = L.job[q];
            j.px = im.pixels;
            j.row_stride = im.row_stride;
            j.out_off = i * out_batch_stride;
            j.w = (int32_t)im.width; j.h = (int32_t)im.height;
            j.bpp = (int32_t)im.bytes_per_pixel; j.bgr = im.bgr ? 1 : 0;
            int64_t nw = out_w, nh = out_h;
            float ratio = 1.0f;
            if (keep_aspect) {
                // letterBoxEx (source/ntypes.pas:922-943): out_w / w < out_h / h, compared exactly
                if (out_w * im.height < out_h * im.width) {
                    nw = out_w; nh = im.height * out_w / im.width;
                    ratio = (float)((double)out_w / (double)im.width);
                } else {
                    nh = out_h; nw = im.width * out_h / im.height;
                    ratio = (float)((double)out_h / (double)im.height);
                }
                if (nw < 2 || nh < 2)
                    return fail(TB_ERR_UNSUPPORTED, "tb_images_to_tensor: image %lld: aspect ratio leaves a "
                                "resized side below 2 pixels", (long long)i);
            }
            j.new_w = (int32_t)nw; j.new_h = (int32_t)nh;
            j.dx = (int32_t)((out_w - nw) / 2); j.dy = (int32_t)((out_h - nh) / 2);
            // resize (:837-845): integer quotients stored to single (correctly rounded)
            j.w_scale = (float)((double)(im.width - 1) / (double)(nw - 1));
            j.h_scale = (float)((double)(im.height - 1) / (double)(nh - 1));
            if (ratio_out) ratio_out[i] = ratio;
            if (placement_out) {
                placement_out[4 * i + 0] = nw; placement_out[4 * i + 1] = nh;
                placement_out[4 * i + 2] = j.dx; placement_out[4 * i + 3] = j.dy;
            }
        }
        // staged rows: two source rows of the widest image (+ 4-byte heads) in shared memory
        int64_t row_vecs = 0;
        for (int64_t q = 0; q < cnt; ++q)
            row_vecs = std::max<int64_t>(row_vecs, (L.job[q].w * (int64_t)L.job[q].bpp + 15 + 15) / 16);
        const int64_t smem = 2 * row_vecs * 16;
        int r;
        if (smem <= kRowsSmemMax && 3 * plane < INT32_MAX && !t_images_direct()) {
            static bool attr_set = false;
            if (!attr_set) {
                TB_CHECK_CUDA(cudaFuncSetAttribute(k_images_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)kRowsSmemMax));
                attr_set = true;
            }
            dim3 grid((unsigned)out_h, (unsigned)cnt);
            k_images_rows<<<grid, 128, (size_t)smem, ctx->stream>>>(L, out);
            r = check_launch("k_images_rows");
        } else {
            dim3 grid((unsigned)ceil_div(out_w, 128), (unsigned)out_h, (unsigned)cnt);
            k_images_to_tensor<<<grid, 128, 0, ctx->stream>>>(L, out);
            r = check_launch("k_images_to_tensor");
        }
        if (r != TB_OK) return r;
    }
    return TB_OK;
}

}  // extern "C"
