// Streaming small-M dequant-GEMM, f16 activations.
#include "ee_stream.cuh"

namespace ee {
template int launch_stream<__half>(const GemmArgs&, int*, cudaStream_t, bool*);
}  // namespace ee
