// ee_attn_op.cu -- C ABI: softmax(Q K^T / sqrt(hd)) V for batch x heads
// independent (batch element, head) units, the attention of the
// layer-by-layer path (kernel/flow_expert.py:86, :91,
// F.scaled_dot_product_attention, non-causal). Each unit is the sampler's
// attention unit (ee_attn.cuh) on one CTA; q / k / v are read in place from
// the projections' row-major outputs (head h at column h * hd of a row) and
// the output is written merged ([rows][heads * hd]), so no split / merge
// copies are needed.
#include <atomic>

#include "ee_attn.cuh"
#include "ee_host.h"

namespace ee {

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads) attention_kernel(const __grid_constant__ AttnArgs a, int units) {
  extern __shared__ __align__(128) char smem[];
  for (int u = blockIdx.x; u < units; u += gridDim.x) Attn<T, HD>::unit(a, u / a.n_heads, u % a.n_heads, smem);
}

template <typename T, int HD>
static int launch_attention(const AttnArgs& a, int units, cudaStream_t s) {
  auto fn = attention_kernel<T, HD>;
  static std::atomic<int> smem_set[64];
  allow_max_smem(fn, smem_set);
  const DevProps* dp = device_props();
  if (!dp) return EE_ERR_DEVICE;
  if ((int)AttnSmem<HD>::kTotal > dp->smem_optin) return EE_ERR_UNSUPPORTED;
  int per_sm = dp->smem_optin / (int)AttnSmem<HD>::kTotal;
  per_sm = per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm);
  const long long cap = (long long)dp->sms * per_sm;
  const int grid = (int)(units < cap ? units : cap);
  fn<<<grid, kThreads, AttnSmem<HD>::kTotal, s>>>(a, units);
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

}  // namespace ee

using namespace ee;

extern "C" int ee_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                            void* out, int64_t ldo, int32_t batch, int32_t n_heads, int32_t head_dim, int32_t n_q,
                            int32_t n_k, int64_t q_rows_per_b, int64_t k_rows_per_b, int32_t act_dtype,
                            ee_stream_t stream) {
  if (!q || !k || !v || !out) return EE_ERR_ARG;
  if (batch < 0 || n_heads < 1 || n_k < 1 || n_q < 0) return EE_ERR_SHAPE;
  if (batch == 0 || n_q == 0) return EE_OK;
  if (head_dim != 64 && head_dim != 128) return EE_ERR_UNSUPPORTED;
  if (n_q > 64) return EE_ERR_UNSUPPORTED;
  const int64_t hw = (int64_t)n_heads * head_dim;
  if (ldq < hw || ldk < hw || ldv < hw || ldo < hw || (ldq % 8) || (ldk % 8) || (ldv % 8) || (ldo % 2))
    return EE_ERR_SHAPE;
  if (q_rows_per_b < n_q || k_rows_per_b < n_k) return EE_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (reinterpret_cast<uintptr_t>(out) & 3)) return EE_ERR_ALIGN;
  if (act_dtype != EE_BF16 && act_dtype != EE_F16) return EE_ERR_DTYPE;
  const int rc = check_device();
  if (rc) return rc;
  const long long units = (long long)batch * n_heads;
  if (units > 0x7fffffffLL) return EE_ERR_SHAPE;
  AttnArgs a{};
  a.q = q; a.ldq = ldq;
  a.k = k; a.ldk = ldk;
  a.v = v; a.ldv = ldv;
  a.out = out; a.ldo = ldo;
  a.n_q = n_q;
  a.n_k = n_k;
  a.q_rows_per_b = (int)q_rows_per_b;
  a.k_rows_per_b = (int)k_rows_per_b;
  a.n_heads = n_heads;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  cudaStream_t s = (cudaStream_t)stream;
  if (act_dtype == EE_BF16)
    return head_dim == 64 ? launch_attention<__nv_bfloat16, 64>(a, (int)units, s)
                          : launch_attention<__nv_bfloat16, 128>(a, (int)units, s);
  return head_dim == 64 ? launch_attention<__half, 64>(a, (int)units, s)
                        : launch_attention<__half, 128>(a, (int)units, s);
}
