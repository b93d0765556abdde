// conv_tile_128x128.cu -- instantiation of the FP32 conv kernel for the 128 x 128 CTA tile
// (thread tile 8 x 8, 4-stage cp.async ring).
#include "conv_fp32_kernel.cuh"

namespace tbi {
int conv_launch_128x128(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode) {
    if (grid.x == 0) return conv_occupancy_modes<128, 128, 8, 8, 4>(ctx, mode);
    return conv_launch_modes<128, 128, 8, 8, 4>(ctx, p, grid, mode);
}
}  // namespace tbi
