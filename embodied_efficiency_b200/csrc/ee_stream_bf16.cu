// Streaming small-M dequant-GEMM, bf16 activations.
#include "ee_stream.cuh"

namespace ee {
template int launch_stream<__nv_bfloat16>(const GemmArgs&, int*, cudaStream_t, bool*);
}  // namespace ee
