// ee_norm.cu -- C ABI: LayerNorm over the last dimension of a [rows, cols]
// activation matrix (the nn.LayerNorm of kernel/flow_expert.py's blocks), for
// the layer-by-layer path that large request batches take.
//
// One warp per row at a time; a lane holds its 16-byte chunks (8 values
// each) of the row in registers (cols <= 2048). fp32 statistics in two passes (mean, then
// the biased variance), rstd = rsqrtf(var + eps), and
// y = ((x - mean) * rstd) * w + b in fp32 with one rounding to the activation
// type -- nn.LayerNorm's formula and order of operations.
#include <atomic>

#include "ee_gemm.cuh"
#include "ee_host.h"

namespace ee {

constexpr int kNormMaxChunks = 8;  // per lane: cols <= 8 chunks x 8 values x 32 lanes
constexpr int kNormWarps = 8;      // rows in flight per CTA

// Persistent warps: warp w of the grid normalises rows w, w + W, w + 2W, ...
// (W = warps in the grid) and issues the loads of its next row before the
// arithmetic of the current one, so each warp keeps two rows in flight and
// the grid has no tail wave. NCH = 16-byte chunks per lane (cols <= 256 NCH).
template <typename T, int NCH>
__global__ void __launch_bounds__(kNormWarps * 32) layer_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                      const T* __restrict__ b, T* __restrict__ y,
                                                                      long long rows, int cols, long long ldx,
                                                                      long long ldy, float eps) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const long long stride = (long long)gridDim.x * kNormWarps;
  long long row = (long long)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nch = cols >> 3;  // 16-byte chunks per row
  auto load_row = [&](uint4 (&q)[NCH], long long r) {
    const T* xr = x + r * ldx;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = lane + 32 * i;
      q[i] = c < nch ? *reinterpret_cast<const uint4*>(xr + 8 * c) : make_uint4(0, 0, 0, 0);
    }
  };
  uint4 q[NCH], qn[NCH];
  load_row(q, row);
  for (; row < rows; row += stride) {
    if (row + stride < rows) load_row(qn, row + stride);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      if (lane + 32 * i < nch) {
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
    for (int i = 0; i < NCH; ++i) {
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
    for (int i = 0; i < NCH; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) {
        // the parameters are re-read per row (L1 hits) to keep registers for the rows in flight
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
#pragma unroll
    for (int i = 0; i < NCH; ++i) q[i] = qn[i];
  }
}

template <typename T, int NCH>
static int launch_norm(const T* x, const T* w, const T* b, T* y, long long rows, int cols, long long ldx,
                       long long ldy, float eps, cudaStream_t s) {
  static std::atomic<int> occ_cache[64];
  const DevProps* dp = device_props();
  if (!dp) return EE_ERR_DEVICE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return EE_ERR_DEVICE;
  int per_sm = occ_cache[dev].load();
  if (per_sm <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, layer_norm_kernel<T, NCH>, kNormWarps * 32, 0) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    occ_cache[dev].store(per_sm);
  }
  const long long need = (rows + kNormWarps - 1) / kNormWarps;
  const long long cap = (long long)dp->sms * per_sm;
  const unsigned grid = (unsigned)(need < cap ? need : cap);
  return launch_pdl(layer_norm_kernel<T, NCH>, dim3(grid), dim3(kNormWarps * 32), 0, s, x, w, b, y, rows, cols, ldx, ldy,
                    eps) == cudaSuccess
             ? EE_OK
             : EE_ERR_LAUNCH;
}

template <typename T>
static int dispatch_norm(const void* x, const void* w, const void* b, void* y, long long rows, int cols,
                         long long ldx, long long ldy, float eps, cudaStream_t s) {
  const T* xt = reinterpret_cast<const T*>(x);
  const T* wt = reinterpret_cast<const T*>(w);
  const T* bt = reinterpret_cast<const T*>(b);
  T* yt = reinterpret_cast<T*>(y);
  const int lanes_chunks = (cols / 8 + 31) / 32;  // 16-byte chunks per lane
  if (lanes_chunks <= 1) return launch_norm<T, 1>(xt, wt, bt, yt, rows, cols, ldx, ldy, eps, s);
  if (lanes_chunks <= 2) return launch_norm<T, 2>(xt, wt, bt, yt, rows, cols, ldx, ldy, eps, s);
  if (lanes_chunks <= 4) return launch_norm<T, 4>(xt, wt, bt, yt, rows, cols, ldx, ldy, eps, s);
  return launch_norm<T, kNormMaxChunks>(xt, wt, bt, yt, rows, cols, ldx, ldy, eps, s);
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
  cudaStream_t s = (cudaStream_t)stream;
  if (act_dtype == EE_BF16)
    return dispatch_norm<__nv_bfloat16>(x, weight, bias, y, rows, (int)cols, ldx, ldy, eps, s);
  return dispatch_norm<__half>(x, weight, bias, y, rows, (int)cols, ldx, ldy, eps, s);
}
