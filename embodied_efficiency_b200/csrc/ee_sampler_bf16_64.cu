// ee_sampler_bf16_64.cu -- sampler kernel instantiation: bf16 activations, head size 64.
#include "ee_sampler.cuh"

namespace ee {
template int launch_sampler<__nv_bfloat16, 64>(const Ctx&, cudaStream_t);
}  // namespace ee
