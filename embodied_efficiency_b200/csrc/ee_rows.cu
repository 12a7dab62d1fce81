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
  pdl_entry();
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
// Thread = one output column n (CTA y covers columns [256 y, 256 y + 256)),
// its AK in_proj weights held in fp32 registers for the whole kernel; the CTA
// walks batches of kHeadRows token rows (m0 = blockIdx.x * kHeadRows, +
// gridDim.x * kHeadRows, ...), the batch's activations in shared memory read
// as broadcast float4s, one fp32 dot product per (row, column) in k order.
constexpr int kHeadRows = 8;
template <typename T, int AK>
__global__ void __launch_bounds__(kRowThreads, 2) expert_head_kernel(const T* __restrict__ xa, const T* __restrict__ w,
                                                                      const T* __restrict__ bias, const T* __restrict__ temb,
                                                                      T* __restrict__ out, long long rows, int d,
                                                                      long long rows_per_b, long long ld_temb) {
  pdl_entry();
  __shared__ __align__(16) float xs[kHeadRows][AK];
  __shared__ const T* trow[kHeadRows];  // the batch rows' projected time-embedding rows
  const int n = blockIdx.y * kRowThreads + threadIdx.x;
  const bool live = n < d;
  float wr[AK];
#pragma unroll
  for (int c = 0; c < AK / 8; ++c) {
    const uint4 v = live ? __ldg(reinterpret_cast<const uint4*>(w + (size_t)n * AK) + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Act<T>::unpack2(comp(v, e));
      wr[8 * c + 2 * e] = f.x;
      wr[8 * c + 2 * e + 1] = f.y;
    }
  }
  const float bv = (live && bias) ? ld_param(bias + n) : 0.f;
  for (long long m0 = (long long)blockIdx.x * kHeadRows; m0 < rows; m0 += (long long)gridDim.x * kHeadRows) {
    __syncthreads();  // the previous batch's activations are no longer read
    for (int i = threadIdx.x; i < kHeadRows * AK; i += kRowThreads) {
      const int r = i / AK, k = i - r * AK;
      xs[r][k] = m0 + r < rows ? Act<T>::to_f(xa[(m0 + r) * AK + k]) : 0.f;
    }
    if (threadIdx.x < kHeadRows) trow[threadIdx.x] = temb + ((m0 + threadIdx.x) / rows_per_b) * ld_temb;
    __syncthreads();
#pragma unroll 1
    for (int r = 0; r < kHeadRows; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int k4 = 0; k4 < AK / 4; ++k4) {
        const float4 xv = *reinterpret_cast<const float4*>(&xs[r][4 * k4]);
        acc = fmaf(xv.x, wr[4 * k4], acc);
        acc = fmaf(xv.y, wr[4 * k4 + 1], acc);
        acc = fmaf(xv.z, wr[4 * k4 + 2], acc);
        acc = fmaf(xv.w, wr[4 * k4 + 3], acc);
      }
      const long long m = m0 + r;
      if (live && m < rows)
        out[m * d + n] = Act<T>::from_f(Act<T>::round(Act<T>::round(acc + bv) + ld_param(trow[r] + n)));
    }
  }
}

template <typename T, int AK>
static int launch_head(const void* xa, const void* w, const void* b, const void* temb, void* x, long long rows, int d,
                       long long rows_per_b, long long ld_temb, cudaStream_t s) {
  const DevProps* dp = device_props();
  const int slices = (d + kRowThreads - 1) / kRowThreads;
  const long long batches = (rows + kHeadRows - 1) / kHeadRows;
  long long gx = (long long)(dp ? dp->sms : 148) * 4 / slices;  // about four CTAs per SM in all
  if (gx < 1) gx = 1;
  if (gx > batches) gx = batches;
  return launch_pdl(expert_head_kernel<T, AK>, dim3((unsigned)gx, (unsigned)slices), dim3(kRowThreads), 0, s,
                    reinterpret_cast<const T*>(xa), reinterpret_cast<const T*>(w), reinterpret_cast<const T*>(b),
                    reinterpret_cast<const T*>(temb), reinterpret_cast<T*>(x), rows, d, rows_per_b, ld_temb) == cudaSuccess
             ? EE_OK
             : EE_ERR_LAUNCH;
}

template <typename T>
static int dispatch_head(const void* xa, const void* w, const void* b, const void* temb, void* x, long long rows, int A,
                         int d, long long rows_per_b, long long ld_temb, cudaStream_t s) {
  switch (A) {
    case 8: return launch_head<T, 8>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
    case 16: return launch_head<T, 16>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
    case 24: return launch_head<T, 24>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
    case 32: return launch_head<T, 32>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
    case 40: return launch_head<T, 40>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
    case 48: return launch_head<T, 48>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
    case 56: return launch_head<T, 56>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
    case 64: return launch_head<T, 64>(xa, w, b, temb, x, rows, d, rows_per_b, ld_temb, s);
  }
  return EE_ERR_SHAPE;
}

// x[i] = round(x[i] + round(v[i] * dt)); t[b] = round(t[b] + dt)
template <typename T>
__global__ void __launch_bounds__(kRowThreads) euler_step_kernel(T* __restrict__ x, const T* __restrict__ v, T* __restrict__ t,
                                                                  long long count, int batch, float dt) {
  pdl_entry();
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
  const cudaError_t e =
      act_dtype == EE_BF16
          ? launch_pdl(time_embed_kernel<__nv_bfloat16>, dim3(grid), dim3(kRowThreads), 0, s,
                       reinterpret_cast<const __nv_bfloat16*>(t), freqs, reinterpret_cast<__nv_bfloat16*>(emb), batch, half)
          : launch_pdl(time_embed_kernel<__half>, dim3(grid), dim3(kRowThreads), 0, s, reinterpret_cast<const __half*>(t),
                       freqs, reinterpret_cast<__half*>(emb), batch, half);
  return e == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
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
  const int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (act_dtype == EE_BF16)
    return dispatch_head<__nv_bfloat16>(x_act, w_in, b_in, temb, x, rows, action_dim, d_model, rows_per_b, ld_temb, s);
  return dispatch_head<__half>(x_act, w_in, b_in, temb, x, rows, action_dim, d_model, rows_per_b, ld_temb, s);
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
  const cudaError_t e =
      act_dtype == EE_BF16
          ? launch_pdl(euler_step_kernel<__nv_bfloat16>, dim3(grid), dim3(kRowThreads), 0, s,
                       reinterpret_cast<__nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(v),
                       reinterpret_cast<__nv_bfloat16*>(t), count, batch, dt)
          : launch_pdl(euler_step_kernel<__half>, dim3(grid), dim3(kRowThreads), 0, s, reinterpret_cast<__half*>(x),
                       reinterpret_cast<const __half*>(v), reinterpret_cast<__half*>(t), count, batch, dt);
  return e == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

}  // extern "C"
