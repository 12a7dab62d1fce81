// ee_sampler_f16_64.cu -- sampler kernel instantiation: f16 activations, head size 64.
#include "ee_sampler.cuh"

namespace ee {
template int launch_sampler<__half, 64>(Ctx, cudaStream_t);
template int sampler_geometry<__half, 64>(const Ctx&, int*, int*, size_t*);
}  // namespace ee
