// conv_tile_64x64.cu -- instantiation of the FP32 conv kernel for the 64 x 64 CTA tile
// (thread tile 8 x 8, 4-stage cp.async ring).
#include "conv_fp32_kernel.cuh"

namespace tbi {
int conv_launch_64x64(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode) {
    if (grid.x == 0) return conv_occupancy_modes<64, 64, 8, 8, 4>(ctx, mode);
    return conv_launch_modes<64, 64, 8, 8, 4>(ctx, p, grid, mode);
}
}  // namespace tbi
