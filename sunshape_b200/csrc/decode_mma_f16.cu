// Explicit instantiations of the tensor-core decode kernel for f16 values.
#include "decode_mma.cuh"
namespace sunshape {
template void launch_decode_mma_t<4, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<4, 64, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<4, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<4, 128, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<4, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<4, 256, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<8, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<8, 64, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<8, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<8, 128, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<8, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<8, 256, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<16, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<16, 64, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<16, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<16, 128, __half, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<16, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_mma_t<16, 256, __half, true>(const DecodeLaunch&, cudaStream_t);
}  // namespace sunshape
