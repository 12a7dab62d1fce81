// ee_norm.cu -- C ABI: LayerNorm over the last dimension of a [rows, cols]
// activation matrix (the nn.LayerNorm of kernel/flow_expert.py's blocks), for
// the layer-by-layer path that large request batches take.
//
// One warp per row; a lane holds its 16-byte chunks (8 values each) of the
// row in registers (cols <= 2048). fp32 statistics in two passes (mean, then
// the biased variance), rstd = rsqrtf(var + eps), and
// y = ((x - mean) * rstd) * w + b in fp32 with one rounding to the activation
// type -- nn.LayerNorm's formula and order of operations.
#include "ee_gemm.cuh"
#include "ee_host.h"

namespace ee {

constexpr int kNormMaxChunks = 8;  // per lane: cols <= 8 chunks x 8 values x 32 lanes

template <typename T>
__global__ void __launch_bounds__(256) layer_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                         const T* __restrict__ b, T* __restrict__ y, long long rows,
                                                         int cols, long long ldx, long long ldy, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nch = cols >> 3;  // 16-byte chunks per row
  const T* xr = x + row * ldx;
  uint4 q[kNormMaxChunks];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxChunks; ++i) {
    const int c = lane + 32 * i;
    q[i] = c < nch ? *reinterpret_cast<const uint4*>(xr + 8 * c) : make_uint4(0, 0, 0, 0);
    if (c < nch) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Act<T>::unpack2(comp(q[i], e));
        sum += f.x + f.y;
      }
    }
  }
  const float mean = warp_sum(sum) / (float)cols;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxChunks; ++i) {
    if (lane + 32 * i < nch) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Act<T>::unpack2(comp(q[i], e));
        const float d0 = f.x - mean, d1 = f.y - mean;
        ss += d0 * d0 + d1 * d1;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / (float)cols + eps);
  T* yr = y + row * ldy;
#pragma unroll
  for (int i = 0; i < kNormMaxChunks; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) {
      const uint4 wq = w ? __ldg(reinterpret_cast<const uint4*>(w + 8 * c)) : make_uint4(0, 0, 0, 0);
      const uint4 bq = b ? __ldg(reinterpret_cast<const uint4*>(b + 8 * c)) : make_uint4(0, 0, 0, 0);
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Act<T>::unpack2(comp(q[i], e));
        const float2 wf = w ? Act<T>::unpack2(comp(wq, e)) : make_float2(1.f, 1.f);
        const float2 bf = b ? Act<T>::unpack2(comp(bq, e)) : make_float2(0.f, 0.f);
        o[e] = Act<T>::pack2((f.x - mean) * rstd * wf.x + bf.x, (f.y - mean) * rstd * wf.y + bf.y);
      }
      *reinterpret_cast<uint4*>(yr + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

}  // namespace ee

using namespace ee;

extern "C" int ee_layer_norm(const void* x, const void* weight, const void* bias, void* y, int64_t rows, int64_t cols,
                             int64_t ldx, int64_t ldy, float eps, int32_t act_dtype, ee_stream_t stream) {
  if (!x || !y || rows < 0) return EE_ERR_ARG;
  if (rows == 0) return EE_OK;
  if (cols < 8 || (cols % 8) != 0 || cols > 8 * 32 * kNormMaxChunks) return EE_ERR_SHAPE;
  if (ldx < cols || ldy < cols || (ldx % 8) != 0 || (ldy % 8) != 0) return EE_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(y) || (weight && !aligned16(weight)) || (bias && !aligned16(bias)))
    return EE_ERR_ALIGN;
  if (act_dtype != EE_BF16 && act_dtype != EE_F16) return EE_ERR_DTYPE;
  const int rc = check_device();
  if (rc) return rc;
  const long long blocks = (rows + 7) / 8;  // 8 rows (warps) per CTA
  if (blocks > 0x7fffffffLL) return EE_ERR_SHAPE;
  cudaStream_t s = (cudaStream_t)stream;
  if (act_dtype == EE_BF16)
    layer_norm_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(weight),
        reinterpret_cast<const __nv_bfloat16*>(bias), reinterpret_cast<__nv_bfloat16*>(y), rows, (int)cols, ldx, ldy,
        eps);
  else
    layer_norm_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(
        reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(weight),
        reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(y), rows, (int)cols, ldx, ldy, eps);
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}
