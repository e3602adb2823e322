// Explicit instantiations of the fused decode kernel for f32 values (split out for parallel builds).
#include "decode.cuh"
namespace sunshape {
template void launch_decode_t<4, 64, float, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<4, 128, float, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<4, 256, float, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<8, 64, float, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<8, 128, float, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<8, 256, float, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<16, 64, float, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<16, 128, float, false>(const DecodeLaunch&, cudaStream_t);
}  // namespace sunshape
