// ee_attn_op.cu -- C ABI: softmax(Q K^T / sqrt(hd)) V for batch x heads
// independent (batch element, head) units, the attention of the
// layer-by-layer path (kernel/flow_expert.py:86, :91,
// F.scaled_dot_product_attention, non-causal). A unit is computed as in the
// sampler's attention unit (ee_attn.cuh: 8 warps = 4 query tiles x 2 key
// groups, 64-key blocks in pairs); q / k / v are read in place from the
// projections' row-major outputs (head h at column h * hd of a row) and the
// output is written merged ([rows][heads * hd]), so no split / merge copies
// are needed.
//
// Keys in one 64-key block (self-attention over the action chunk): a CTA
// takes units blockIdx.x, + gridDim.x, ... two at a time, one per key group
// (each group finishes its unit without a merge), and runs them as one
// double-buffered pipeline, so the next two units' Q / K / V tiles are in
// flight while the current two are computed; the second Q tiles live in the
// merge area, which that form does not use. With more key blocks (the
// cross-attention to the prefix) each unit is the sampler's unit, one after
// another: there the unit's own second pair already overlaps its first, and
// running the pairs of consecutive units as one pipeline measured slower
// (117 vs 107 us for 256 requests x 256 prefix keys).

#include <atomic>

#include "ee_attn.cuh"
#include "ee_host.h"

namespace ee {

template <int HD>
struct StreamSmem {
  using S = AttnSmem<HD>;
  static constexpr int kQ2 = (S::kTotal + 127) & ~127;  // key group 0's Q tile of odd items (even: S::kQ)
  static constexpr int kTotal = kQ2 + S::kTile;
  static_assert(2 * S::kTile <= S::kMergeBytes, "two-unit items keep their second Q tiles in the merge area");
};

// any number of keys: the sampler's unit, one unit after another
template <typename T, int HD>
__global__ void __launch_bounds__(kThreads) attention_kernel(const __grid_constant__ AttnArgs a, int units) {
  extern __shared__ __align__(128) char smem[];
  pdl_entry();
  for (int u = blockIdx.x; u < units; u += gridDim.x) Attn<T, HD>::unit(a, u / a.n_heads, u % a.n_heads, smem);
}

// keys in one 64-key block: two units per item, streamed
template <typename T, int HD>
__global__ void __launch_bounds__(kThreads) attention_pair_kernel(const __grid_constant__ AttnArgs a, int units) {
  extern __shared__ __align__(128) char smem[];
  pdl_entry();
  using U = Attn<T, HD>;
  using S = AttnSmem<HD>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = warp & 3, kg = warp >> 2;
  const uint32_t sbase = smem_u32(smem);
  const int my_units = (int)blockIdx.x < units ? (units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const long long items = (my_units + 1) / 2;  // item = two units, one per key group
  // Q tile of item parity p for key group g
  auto q_buf = [&](int p, int g) {
    return sbase + (g ? S::kMerge + p * S::kTile : (p ? StreamSmem<HD>::kQ2 : S::kQ));
  };
  auto sK = [&](int st, int g) { return sbase + S::kKV + ((st * 2 + g) * 2 + 0) * S::kTile; };
  auto sV = [&](int st, int g) { return sbase + S::kKV + ((st * 2 + g) * 2 + 1) * S::kTile; };
  auto unit_of = [&](int j) { return (int)blockIdx.x + j * (int)gridDim.x; };
  // cp.async copies of item i's Q / K / V tiles into stage i & 1
  auto issue = [&](long long i) {
    const int st = (int)(i & 1);
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int j = (int)(2 * i) + g;
      if (j < my_units) {
        const int u = unit_of(j);
        const int b = u / a.n_heads, h = u - b * a.n_heads;
        const long long col = (long long)h * HD, kr0 = (long long)b * a.k_rows_per_b;
        U::load_tile(q_buf(st, g), a.q, a.ldq, col, (long long)b * a.q_rows_per_b, a.n_q);
        U::load_tile(sK(st, g), a.k, a.ldk, col, kr0, a.n_k);
        U::load_tile(sV(st, g), a.v, a.ldv, col, kr0, a.n_k);
      }
    }
  };
  typename U::State sw;
  if (items > 0) issue(0);
  cp_async_commit();
  for (long long i = 0; i < items; ++i) {
    // stage (i + 1) & 1 was last read before the previous iteration's closing __syncthreads
    if (i + 1 < items) issue(i + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int st = (int)(i & 1);
    const int j = (int)(2 * i) + kg;
    if (j < my_units) {
      const int u = unit_of(j);
      const int b = u / a.n_heads, h = u - b * a.n_heads;
      U::reset(sw);
      U::load_q(sw, q_buf(st, kg), qt, lane);
      U::block(sw, a, sK(st, kg), sV(st, kg), 0, lane);
      U::store_solo(sw, a, (long long)b * a.q_rows_per_b, (long long)h * HD, qt, lane);
    }
    __syncthreads();
  }
  cp_async_wait<0>();
}

template <typename T, int HD>
static int launch_attention(const AttnArgs& a, int units, cudaStream_t s) {
  const bool pair = a.n_k <= 64;
  auto fn = pair ? attention_pair_kernel<T, HD> : attention_kernel<T, HD>;
  static std::atomic<int> smem_set[2][64];
  allow_max_smem(fn, smem_set[pair ? 1 : 0]);
  const DevProps* dp = device_props();
  if (!dp) return EE_ERR_DEVICE;
  // the streaming form needs one more Q tile than the unit loop
  const int smem = pair ? StreamSmem<HD>::kTotal : AttnSmem<HD>::kTotal;
  if (smem > dp->smem_optin) return EE_ERR_UNSUPPORTED;
  int per_sm = dp->smem_optin / smem;
  per_sm = per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm);
  const long long cap = (long long)dp->sms * per_sm;
  const int grid = (int)(units < cap ? units : cap);
  return launch_pdl(fn, dim3(grid), dim3(kThreads), (size_t)smem, s, a, units) == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
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
  // the units index rows with 32-bit row counts per batch item
  if (q_rows_per_b > 0x7fffffffLL || k_rows_per_b > 0x7fffffffLL) return EE_ERR_SHAPE;
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
