// Tensor-core (tcgen05) dequant-GEMM, f16 activations.
#include "ee_tc.cuh"

namespace ee {
template int launch_tc<__half>(const GemmArgs&, int*, cudaStream_t, bool*);
}  // namespace ee
