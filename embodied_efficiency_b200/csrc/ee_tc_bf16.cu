// Tensor-core (tcgen05) dequant-GEMM, bf16 activations.
#include "ee_tc.cuh"

namespace ee {
template int launch_tc<__nv_bfloat16>(const GemmArgs&, int*, cudaStream_t, bool*);
}  // namespace ee
