// ee_sampler_bf16_64.cu -- sampler kernel instantiation: bf16 activations, head size 64.
#include "ee_sampler.cuh"

namespace ee {
template int launch_sampler<__nv_bfloat16, 64>(Ctx, cudaStream_t);
template int sampler_geometry<__nv_bfloat16, 64>(const Ctx&, int*, int*, size_t*);
}  // namespace ee
