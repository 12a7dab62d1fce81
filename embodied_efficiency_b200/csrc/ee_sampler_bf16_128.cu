// ee_sampler_bf16_128.cu -- sampler kernel instantiation: bf16 activations, head size 128.
#include "ee_sampler.cuh"

namespace ee {
template int launch_sampler<__nv_bfloat16, 128>(Ctx, cudaStream_t);
template int sampler_geometry<__nv_bfloat16, 128>(const Ctx&, int*, int*, size_t*);
}  // namespace ee
