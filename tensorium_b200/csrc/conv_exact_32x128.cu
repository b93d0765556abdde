// conv_exact_32x128.cu -- instantiation of the order-exact FP32 conv for the 32 x 128 CTA tile
// (thread tile 4 x 8).
#include "conv_exact.cuh"

namespace tbi {
int exact_launch_32x128(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var) {
    return exact_launch_modes<32, 128, 4, 8>(ctx, p, grid, mode, fma, var);
}
}  // namespace tbi
