// conv_exact_128x64.cu -- instantiation of the order-exact FP32 conv for the 128 x 64 CTA tile
// (thread tile 8 x 8).
#include "conv_exact.cuh"

namespace tbi {
int exact_launch_128x64(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var) {
    return exact_launch_modes<128, 64, 8, 8>(ctx, p, grid, mode, fma, var);
}
}  // namespace tbi
