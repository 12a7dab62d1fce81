// ee_sampler_f16_128.cu -- sampler kernel instantiation: f16 activations, head size 128.
#include "ee_sampler.cuh"

namespace ee {
template int launch_sampler<__half, 128>(Ctx, cudaStream_t);
template int sampler_geometry<__half, 128>(const Ctx&, int*, int*, size_t*);
}  // namespace ee
