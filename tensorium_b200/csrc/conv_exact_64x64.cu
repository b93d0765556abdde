// conv_exact_64x64.cu -- instantiation of the order-exact FP32 conv for the 64 x 64 CTA tile
// (thread tile 8 x 8).
#include "conv_exact.cuh"

namespace tbi {
int exact_launch_64x64(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var) {
    return exact_launch_modes<64, 64, 8, 8>(ctx, p, grid, mode, fma, var);
}
}  // namespace tbi
