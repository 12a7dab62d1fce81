// ee_dequant.cu -- C ABI: a packed weight dequantised into the activation
// dtype, [n][k] row-major, with the arithmetic of the GEMM kernels' dequant
// step: the exact integer times the scale rounded to the activation type,
// one rounding (kernel/triton_gemm.py:91-94 and :127-134); for the
// zero-point int4 form, (v - zero) rounded, then times the scale.
//
// The layer-by-layer path dequantises each weight once into a cached dense
// copy for GEMMs with so many tokens that the tensor cores bound them: there,
// dequantising a weight tile again for every token tile costs more time than
// the packed weight saves in bytes.
#include "ee_gemm.cuh"
#include "ee_host.h"

namespace ee {

// one thread per 16-byte chunk of packed weights (16 int8 or 32 int4 values)
template <typename T, int KIND>
__global__ void __launch_bounds__(256) dequant_weight_kernel(const ee_linear L, T* __restrict__ out) {
  constexpr int kVals = KIND == EE_W_INT8 ? 16 : 32;
  const long long cpr = L.k / kVals;  // chunks per row
  const long long total = (long long)L.n * cpr;
  const int ng = L.k / L.group;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / cpr;
    const int k0 = (int)(i - n * cpr) * kVals;
    const size_t si = (size_t)n * ng + k0 / L.group;
    const float scv = L.scale_dtype == EE_F32 ? reinterpret_cast<const float*>(L.scales)[si]
                                              : __half2float(reinterpret_cast<const __half*>(L.scales)[si]);
    const uint32_t s2 = Act<T>::pack2(scv, scv);
    // rows are k (int8) or k / 2 (int4) bytes, multiples of 16: chunk i starts at byte 16 i
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(L.weight) + i);
    uint4* dst = reinterpret_cast<uint4*>(out + n * L.k + k0);
    if (KIND == EE_W_INT8) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t w0 = comp(raw, 2 * u) ^ 0x80808080u, w1 = comp(raw, 2 * u + 1) ^ 0x80808080u;
        dst[u] = make_uint4(hmul2<T>(int8_pair<T>(w0, 0, 1), s2), hmul2<T>(int8_pair<T>(w0, 2, 3), s2),
                            hmul2<T>(int8_pair<T>(w1, 0, 1), s2), hmul2<T>(int8_pair<T>(w1, 2, 3), s2));
      }
    } else {
      const float zcv = KIND == EE_W_UINT4Z ? __half2float(reinterpret_cast<const __half*>(L.zeros)[si]) : 0.f;
      const float zoff = KIND == EE_W_INT4 ? 8.0f : zcv;
      const uint32_t xor8 = KIND == EE_W_INT4 ? 0x00080008u : 0u;
      const uint32_t nego = Act<T>::neg_offset2(Act<T>::kInt4Base + zoff);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t w = comp(raw, u), w4 = w >> 4;
        uint32_t o[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) o[p] = hmul2<T>(fma2<T>(nib_pair<T>(w, w4, p, xor8), Act<T>::kOne2, nego), s2);
        dst[u] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

template <typename T, int KIND>
static int launch_dequant(const ee_linear& L, void* out, cudaStream_t s) {
  const DevProps* dp = device_props();
  if (!dp) return EE_ERR_DEVICE;
  const long long total = (long long)L.n * (L.k / (KIND == EE_W_INT8 ? 16 : 32));
  const long long want = (total + 255) / 256, cap = (long long)dp->sms * 8;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  dequant_weight_kernel<T, KIND><<<grid, 256, 0, s>>>(L, reinterpret_cast<T*>(out));
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

template <typename T>
static int dispatch_dequant(const ee_linear& L, void* out, cudaStream_t s) {
  switch (L.wkind) {
    case EE_W_INT8: return launch_dequant<T, EE_W_INT8>(L, out, s);
    case EE_W_INT4: return launch_dequant<T, EE_W_INT4>(L, out, s);
    default: return launch_dequant<T, EE_W_UINT4Z>(L, out, s);
  }
}

}  // namespace ee

using namespace ee;

extern "C" int ee_dequant_weight(const void* weight, const void* scales, const void* zeros, void* out, int64_t n,
                                 int64_t k, int32_t wkind, int32_t group, int32_t act_dtype, int32_t scale_dtype,
                                 ee_stream_t stream) {
  if (!weight || !out) return EE_ERR_ARG;
  if (act_dtype != EE_BF16 && act_dtype != EE_F16) return EE_ERR_DTYPE;
  if (wkind != EE_W_INT8 && wkind != EE_W_INT4 && wkind != EE_W_UINT4Z) return EE_ERR_ARG;
  if (n < 1 || n > 0x7fffffff || k > 0x7fffffff) return EE_ERR_SHAPE;
  ee_linear L{};
  L.weight = weight;
  L.scales = scales;
  L.zeros = zeros;
  L.n = (int32_t)n;
  L.k = (int32_t)k;
  L.wkind = wkind;
  L.group = group;
  L.scale_dtype = scale_dtype;
  int rc = validate_linear(L, (int32_t)n, (int32_t)k);
  if (rc) return rc;
  if (!aligned16(out)) return EE_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  return act_dtype == EE_BF16 ? dispatch_dequant<__nv_bfloat16>(L, out, s) : dispatch_dequant<__half>(L, out, s);
}
