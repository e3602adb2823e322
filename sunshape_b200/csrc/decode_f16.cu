// Explicit instantiations of the fused decode kernel for f16 values (split out for parallel builds).
#include "decode.cuh"
namespace sunshape {
template void launch_decode_t<4, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<4, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<4, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<8, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<8, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<8, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<16, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<16, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
}  // namespace sunshape
