// ee_rows.cu -- C ABI: the row-wise head and tail operations of the
// layer-by-layer sampler path (large request batches), so that every
// operation of that path runs on this library's kernels:
//
//   ee_time_embed   kernel/flow_expert.py:38-48 timestep_embedding, rounded to
//                   the activation type (the .to(x.dtype) of :120)
//   ee_expert_head  kernel/flow_expert.py:119-121: x = in_proj(x_act) +
//                   t_proj(temb)[:, None] -- the in_proj dot products (K =
//                   action_dim), its bias and the broadcast add of the
//                   already projected time embedding, in one pass
//   ee_euler_step   kernel/flow_expert.py:133-136: x = x + v * dt and
//                   t = t + dt in the activation type
//
// The arithmetic and its roundings are the fused sampler's row phase
// (ee_sampler.cuh) and torch's eager ops: fp32 dot product in k order,
// round(acc + bias), then round(. + temb); round(x + round(v * dt)) with dt
// as an fp32 scalar; t advanced as round(t + dt).
#include <atomic>

#include "ee_gemm.cuh"
#include "ee_host.h"

namespace ee {

constexpr int kRowThreads = 256;
constexpr int kHeadMaxA = 64;  // action_dim bound of ee_expert_head

// emb[b][i] = cos((t_b * f_i) * 1000), emb[b][half + i] = sin(...), fp32 then
// one rounding; one thread per (b, i)
template <typename T>
__global__ void __launch_bounds__(kRowThreads) time_embed_kernel(const T* __restrict__ t, const float* __restrict__ freqs,
                                                                  T* __restrict__ emb, int batch, int half) {
  const long long total = (long long)batch * half;
  for (long long idx = (long long)blockIdx.x * kRowThreads + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * kRowThreads) {
    const int b = (int)(idx / half), i = (int)(idx - (long long)b * half);
    const float arg = (Act<T>::to_f(t[b]) * __ldg(freqs + i)) * 1000.0f;
    emb[(size_t)b * 2 * half + i] = Act<T>::from_f(cosf(arg));
    emb[(size_t)b * 2 * half + half + i] = Act<T>::from_f(sinf(arg));
  }
}

// x[m][n] = round(round(sum_k x_act[m][k] * W[n][k] + bias[n]) + temb[m / rows_per_b][n]).
// CTA (x, y) keeps the in_proj weight rows of column slice y, [y * nc, + nc),
// in shared memory ([nc][A], at most 64 KB) and walks token rows m =
// blockIdx.x, + gridDim.x, ...; thread j computes columns j, j + 256, ... of
// the slice.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) expert_head_kernel(const T* __restrict__ xa, const T* __restrict__ w,
                                                                   const T* __restrict__ bias, const T* __restrict__ temb,
                                                                   T* __restrict__ out, long long rows, int A, int d, int nc,
                                                                   long long rows_per_b, long long ld_temb) {
  extern __shared__ __align__(16) char smem[];
  const int c0 = blockIdx.y * nc, cn = min(nc, d - c0);
  T* ws = reinterpret_cast<T*>(smem);                                                          // [cn][A]
  float* xs = reinterpret_cast<float*>(smem + (((size_t)nc * A * 2 + 15) & ~(size_t)15));  // [A]
  const int chunks = cn * A / 8;
  const uint4* wsrc = reinterpret_cast<const uint4*>(w + (size_t)c0 * A);
  for (int i = threadIdx.x; i < chunks; i += kRowThreads) reinterpret_cast<uint4*>(ws)[i] = __ldg(wsrc + i);
  for (long long m = blockIdx.x; m < rows; m += gridDim.x) {
    __syncthreads();  // the weights are staged; the previous row's xs is no longer read
    if (threadIdx.x < A) xs[threadIdx.x] = Act<T>::to_f(xa[m * A + threadIdx.x]);
    __syncthreads();
    const T* tr = temb + (m / rows_per_b) * ld_temb;
    T* orow = out + m * d;
    for (int j = threadIdx.x; j < cn; j += kRowThreads) {
      const int n = c0 + j;
      const T* wr = ws + (size_t)j * A;
      float acc = 0.f;
      for (int k = 0; k < A; k += 2) {
        const float2 f = Act<T>::unpack2(*reinterpret_cast<const uint32_t*>(wr + k));
        acc = fmaf(xs[k], f.x, acc);
        acc = fmaf(xs[k + 1], f.y, acc);
      }
      acc += bias ? ld_param(bias + n) : 0.f;
      orow[n] = Act<T>::from_f(Act<T>::round(Act<T>::round(acc) + ld_param(tr + n)));
    }
  }
}

// x[i] = round(x[i] + round(v[i] * dt)); t[b] = round(t[b] + dt)
template <typename T>
__global__ void __launch_bounds__(kRowThreads) euler_step_kernel(T* __restrict__ x, const T* __restrict__ v, T* __restrict__ t,
                                                                  long long count, int batch, float dt) {
  for (long long i = (long long)blockIdx.x * kRowThreads + threadIdx.x; i < count;
       i += (long long)gridDim.x * kRowThreads)
    x[i] = Act<T>::from_f(Act<T>::round(Act<T>::to_f(x[i]) + Act<T>::round(Act<T>::to_f(v[i]) * dt)));
  if (t && blockIdx.x == 0)
    for (int b = threadIdx.x; b < batch; b += kRowThreads) t[b] = Act<T>::from_f(Act<T>::to_f(t[b]) + dt);
}

static unsigned grid_for(long long work, int per_cta) {
  const DevProps* dp = device_props();
  const long long cap = (long long)(dp ? dp->sms : 148) * 8;
  long long g = (work + per_cta - 1) / per_cta;
  if (g < 1) g = 1;
  return (unsigned)(g < cap ? g : cap);
}

}  // namespace ee

using namespace ee;

extern "C" {

int ee_time_embed(const void* t, const float* freqs, void* emb, int32_t batch, int32_t dim, int32_t act_dtype,
                  ee_stream_t stream) {
  if (!t || !freqs || !emb || batch < 0) return EE_ERR_ARG;
  if (batch == 0) return EE_OK;
  if (dim < 2 || (dim % 2) != 0) return EE_ERR_SHAPE;
  if (act_dtype != EE_BF16 && act_dtype != EE_F16) return EE_ERR_DTYPE;
  const int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int half = dim / 2;
  const unsigned grid = grid_for((long long)batch * half, kRowThreads);
  if (act_dtype == EE_BF16)
    time_embed_kernel<__nv_bfloat16><<<grid, kRowThreads, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(t), freqs, reinterpret_cast<__nv_bfloat16*>(emb), batch, half);
  else
    time_embed_kernel<__half><<<grid, kRowThreads, 0, s>>>(reinterpret_cast<const __half*>(t), freqs,
                                                           reinterpret_cast<__half*>(emb), batch, half);
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

int ee_expert_head(const void* x_act, const void* w_in, const void* b_in, const void* temb, void* x, int64_t rows,
                   int32_t action_dim, int32_t d_model, int64_t rows_per_b, int64_t ld_temb, int32_t act_dtype,
                   ee_stream_t stream) {
  if (!x_act || !w_in || !temb || !x || rows < 0) return EE_ERR_ARG;
  if (rows == 0) return EE_OK;
  if (action_dim < 2 || (action_dim % 8) != 0 || action_dim > kHeadMaxA) return EE_ERR_SHAPE;
  if (d_model < 8 || rows_per_b < 1 || ld_temb < d_model) return EE_ERR_SHAPE;
  if (!aligned16(w_in)) return EE_ERR_ALIGN;
  if (act_dtype != EE_BF16 && act_dtype != EE_F16) return EE_ERR_DTYPE;
  // column slices of at most 64 KB of weights (a multiple of 256 columns)
  int nc = (int)((65536 / (action_dim * 2)) / kRowThreads * kRowThreads);
  if (nc > d_model) nc = d_model;
  const int slices = (d_model + nc - 1) / nc;
  const size_t smem = (((size_t)nc * action_dim * 2 + 15) & ~(size_t)15) + (size_t)kHeadMaxA * 4;
  const int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  unsigned gx = grid_for(rows, 8);
  gx = gx / (unsigned)slices > 0 ? gx / (unsigned)slices : 1;
  const dim3 grid(gx, (unsigned)slices);
  if (act_dtype == EE_BF16) {
    auto fn = expert_head_kernel<__nv_bfloat16>;
    static std::atomic<int> set[64];
    allow_max_smem(fn, set);
    fn<<<grid, kRowThreads, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(x_act),
                                       reinterpret_cast<const __nv_bfloat16*>(w_in),
                                       reinterpret_cast<const __nv_bfloat16*>(b_in),
                                       reinterpret_cast<const __nv_bfloat16*>(temb),
                                       reinterpret_cast<__nv_bfloat16*>(x), rows, action_dim, d_model, nc, rows_per_b,
                                       ld_temb);
  } else {
    auto fn = expert_head_kernel<__half>;
    static std::atomic<int> set[64];
    allow_max_smem(fn, set);
    fn<<<grid, kRowThreads, smem, s>>>(reinterpret_cast<const __half*>(x_act), reinterpret_cast<const __half*>(w_in),
                                       reinterpret_cast<const __half*>(b_in), reinterpret_cast<const __half*>(temb),
                                       reinterpret_cast<__half*>(x), rows, action_dim, d_model, nc, rows_per_b, ld_temb);
  }
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

int ee_euler_step(void* x, const void* v, void* t, int64_t count, int32_t batch, float dt, int32_t act_dtype,
                  ee_stream_t stream) {
  if (!x || !v || count < 0 || batch < 0) return EE_ERR_ARG;
  if (count == 0 && (!t || batch == 0)) return EE_OK;
  if (act_dtype != EE_BF16 && act_dtype != EE_F16) return EE_ERR_DTYPE;
  const int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned grid = grid_for(count, kRowThreads * 4);
  if (act_dtype == EE_BF16)
    euler_step_kernel<__nv_bfloat16><<<grid, kRowThreads, 0, s>>>(
        reinterpret_cast<__nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(v),
        reinterpret_cast<__nv_bfloat16*>(t), count, batch, dt);
  else
    euler_step_kernel<__half><<<grid, kRowThreads, 0, s>>>(reinterpret_cast<__half*>(x), reinterpret_cast<const __half*>(v),
                                                           reinterpret_cast<__half*>(t), count, batch, dt);
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

}  // extern "C"
