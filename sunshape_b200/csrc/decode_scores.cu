// Explicit instantiations of the score-only variant of the decode kernel.
#include "decode.cuh"
namespace sunshape {
template void launch_decode_t<4, 64, float, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<8, 64, float, true>(const DecodeLaunch&, cudaStream_t);
template void launch_decode_t<16, 64, float, true>(const DecodeLaunch&, cudaStream_t);
}  // namespace sunshape
