// conv_tile_32x256.cu -- instantiation of the FP32 conv kernel for the 32 x 256 CTA tile
// (thread tile 4 x 8, 4-stage cp.async ring).
#include "conv_fp32_kernel.cuh"

namespace tbi {
int conv_launch_32x256(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode) {
    if (grid.x == 0) return conv_occupancy_modes<32, 256, 4, 8, 4>(ctx, mode);
    return conv_launch_modes<32, 256, 4, 8, 4>(ctx, p, grid, mode);
}
}  // namespace tbi
