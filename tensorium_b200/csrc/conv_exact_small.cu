// conv_exact_small.cu -- instantiations of the order-exact FP32 conv with 32 outputs per thread
// (8 filters x 4 pixels on a 64 x 64 tile, 4 x 8 on a 64 x 128 tile): twice the warps of the 8 x 8
// tiles for the same CTA tile, for the layers whose whole output is too small to give every SM
// enough 8 x 8 warps (YOLOv3's 13 x 13 and 26 x 26 convs at small batches).
#include "conv_exact.cuh"

namespace tbi {
int exact_launch_64x64n4(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var) {
    return exact_launch_modes<64, 64, 8, 4>(ctx, p, grid, mode, fma, var);
}
int exact_launch_64x128m4(tb_ctx* ctx, const ConvParams& p, dim3 grid, int mode, bool fma, int var) {
    return exact_launch_modes<64, 128, 4, 8>(ctx, p, grid, mode, fma, var);
}
}  // namespace tbi
