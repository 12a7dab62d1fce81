// ee_ops.cu -- C ABI: int4 pack / unpack and the standalone dequant-GEMM.
#include <atomic>
#include <mutex>

#include "ee_gemm.cuh"
#include "ee_host.h"

namespace ee {

// ---------------------------------------------------------------------------
// int4 packing (kernel/triton_gemm.py:37-48), one thread per output byte
// ---------------------------------------------------------------------------
__global__ void pack_int4_kernel(const int8_t* __restrict__ q, uint8_t* __restrict__ packed,
                                 long long nbytes) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nbytes;
       i += (long long)gridDim.x * blockDim.x) {
    const uint32_t lo = (uint32_t)(uint8_t)q[2 * i] & 0xFu;
    const uint32_t hi = (uint32_t)(uint8_t)q[2 * i + 1] & 0xFu;
    packed[i] = (uint8_t)((hi << 4) | lo);
  }
}

__global__ void unpack_int4_kernel(const uint8_t* __restrict__ packed, int8_t* __restrict__ q,
                                   long long nbytes) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nbytes;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = packed[i];
    const int lo = b & 0xF, hi = b >> 4;
    q[2 * i] = (int8_t)(lo >= 8 ? lo - 16 : lo);
    q[2 * i + 1] = (int8_t)(hi >= 8 ? hi - 16 : hi);
  }
}

// ---------------------------------------------------------------------------
// standalone dequant-GEMM: one cluster per unit (128 rows x 64 tokens)
// ---------------------------------------------------------------------------
template <typename T, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    wq_gemm_kernel(const __grid_constant__ GemmArgs a, GemmSmem sm) {
  extern __shared__ __align__(128) char smem[];
  pdl_entry();
  Gemm<T, KIND>::run(a, smem, sm, nullptr);
}

// largest cluster (<= 8) whose K slices are whole 128-wide k-blocks
static int gemm_cluster(int k) {
  const int kb = k / kKBlock;
  int cl = 8;
  while (cl > 1 && (kb % cl) != 0) cl >>= 1;
  return cl;
}

template <typename T, int KIND>
static int launch_gemm_k(GemmArgs a, cudaStream_t s) {
  const int cl = gemm_cluster(a.w.k);
  a.split = cl;
  a.lsplit = cl == 8 ? 3 : (cl == 4 ? 2 : (cl == 2 ? 1 : 0));
  const int n_tiles = (a.w.n + kRU - 1) / kRU;
  const int m_tiles = (a.M + kMTile - 1) / kMTile;
  const long long units = (long long)n_tiles * m_tiles;
  if (units > 0x7fffffffLL) return EE_ERR_SHAPE;
  const int rows8 = a.M >= kMTile ? kMTile : ((a.M + 7) / 8) * 8;
  size_t x = (size_t)rows8 * (a.w.k / cl) * 2;
  const size_t e = (size_t)rows8 * (kRU / cl + 1) * 4;
  if (e > x) x = e;
  x = (x + 127) & ~(size_t)127;
  GemmSmem sm{};
  sm.x = 0;
  sm.p = (uint32_t)x;
  sm.aux = (uint32_t)(x + 2 * kPBytes);
  sm.pre = (uint32_t)(sm.aux + kAuxBytes);
  const DevProps* dp = device_props();
  if (!dp || (size_t)sm.pre + 1024 > (size_t)dp->smem_optin) return EE_ERR_UNSUPPORTED;
  // stage the unit's weights with cp.async: as many whole k-blocks as fit (at most 64 KB)
  size_t room = (size_t)dp->smem_optin - 1024 - sm.pre;
  if (room > 65536) room = 65536;
  const size_t kbs = (size_t)(a.w.k / cl / kKBlock) * pre_kb_bytes(KIND);
  sm.pre_bytes = (uint32_t)(kbs < room ? kbs : (room / pre_kb_bytes(KIND)) * pre_kb_bytes(KIND));
  const size_t smem = sm.pre + sm.pre_bytes;
  auto fn = wq_gemm_kernel<T, KIND>;
  static std::atomic<int> smem_set[64];
  allow_max_smem(fn, smem_set);
  // one cluster per unit, at most 2^18 clusters (rounds beyond that)
  const long long max_clusters = 1LL << 18;
  const long long nclus = units < max_clusters ? units : max_clusters;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(nclus * cl));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, fn, a, sm);
  return err == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

// Streaming small-M path (ee_stream.cuh, instantiated in ee_stream_*.cu) and
// the tensor-core path (ee_tc.cuh, instantiated in ee_tc_*.cu).
template <typename T> int launch_stream(const GemmArgs& g, int* status, cudaStream_t st, bool* used);
template <typename T> int launch_tc(const GemmArgs& g, int* status, cudaStream_t st, bool* used);

// Token count up to which the warp-MMA streaming kernel is used; above it
// the tcgen05 kernel.
#ifndef EE_STREAM_MAX_M
#define EE_STREAM_MAX_M 32
#endif
constexpr int kStreamMaxM = EE_STREAM_MAX_M;

// Status word of the GEMM kernels (first error since the last reset).
static __device__ int g_gemm_status;

static int* gemm_status_ptr() {
  static std::mutex mu;
  static int* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_status) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<int*>(p);
  }
  return addr[dev];
}

template <typename T>
int launch_gemm_d(const GemmArgs& a, cudaStream_t s) {
  bool used = false;
  int* status = gemm_status_ptr();
  int rc = EE_OK;
  if (a.M <= kStreamMaxM) {
    rc = launch_stream<T>(a, status, s, &used);
    if (used || rc != EE_OK) return rc;
  }
  rc = launch_tc<T>(a, status, s, &used);
  if (used || rc != EE_OK) return rc;
  switch (a.w.wkind) {
    case EE_W_DENSE: return launch_gemm_k<T, EE_W_DENSE>(a, s);
    case EE_W_INT8: return launch_gemm_k<T, EE_W_INT8>(a, s);
    case EE_W_INT4: return launch_gemm_k<T, EE_W_INT4>(a, s);
    case EE_W_UINT4Z: return launch_gemm_k<T, EE_W_UINT4Z>(a, s);
  }
  return EE_ERR_ARG;
}

}  // namespace ee

using namespace ee;

extern "C" {

int ee_pack_int4(const int8_t* q, uint8_t* packed, int64_t n, int64_t k, ee_stream_t stream) {
  if (n < 0 || k < 0 || (k & 1)) return EE_ERR_SHAPE;
  const long long nbytes = (long long)n * (k / 2);
  if (nbytes == 0) return EE_OK;
  if (!q || !packed) return EE_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  const int grid = (int)((nbytes + 255) / 256 < 65536 ? (nbytes + 255) / 256 : 65536);
  pack_int4_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(q, packed, nbytes);
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

int ee_unpack_int4(const uint8_t* packed, int8_t* q, int64_t n, int64_t k, ee_stream_t stream) {
  if (n < 0 || k < 0 || (k & 1)) return EE_ERR_SHAPE;
  const long long nbytes = (long long)n * (k / 2);
  if (nbytes == 0) return EE_OK;
  if (!q || !packed) return EE_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  const int grid = (int)((nbytes + 255) / 256 < 65536 ? (nbytes + 255) / 256 : 65536);
  unpack_int4_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(packed, q, nbytes);
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

int ee_wq_gemm(const void* x, const void* weight, const void* scales, const void* zeros,
               const void* bias, const void* residual, void* y, int64_t m, int64_t n, int64_t k,
               int32_t wkind, int32_t group, int32_t act_dtype, int32_t scale_dtype,
               int32_t epilogue, ee_stream_t stream) {
  if (!x || !weight || !y) return EE_ERR_ARG;
  if (act_dtype != EE_BF16 && act_dtype != EE_F16) return EE_ERR_DTYPE;
  if (wkind < EE_W_DENSE || wkind > EE_W_UINT4Z) return EE_ERR_ARG;
  if ((epilogue & ~(EE_EPI_BIAS | EE_EPI_GELU | EE_EPI_RESIDUAL)) != 0) return EE_ERR_ARG;
  if ((epilogue & EE_EPI_GELU) && (epilogue & EE_EPI_RESIDUAL)) return EE_ERR_ARG;
  if ((epilogue & EE_EPI_BIAS) && !bias) return EE_ERR_ARG;
  if ((epilogue & EE_EPI_RESIDUAL) && !residual) return EE_ERR_ARG;
  if ((epilogue & EE_EPI_RESIDUAL) && (n % 8) != 0) return EE_ERR_SHAPE;
  if (m < 1 || n < 1 || k < kKBlock || (k % kKBlock) != 0) return EE_ERR_SHAPE;
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return EE_ERR_SHAPE;
  ee_linear L{};
  L.weight = weight;
  L.scales = scales;
  L.zeros = zeros;
  L.bias = bias;
  L.n = (int32_t)n;
  L.k = (int32_t)k;
  L.wkind = wkind;
  L.group = group;
  L.scale_dtype = scale_dtype;
  int rc = validate_linear(L, (int32_t)n, (int32_t)k);
  if (rc) return rc;
  if (!aligned16(x) || (residual && !aligned16(residual)) || !aligned16(y)) return EE_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;

  GemmArgs a{};
  a.x = x;
  a.ldx = k;
  a.w = L;
  a.M = (int)m;
  a.epi = (epilogue & EE_EPI_GELU) ? EPI_GELU : ((epilogue & EE_EPI_RESIDUAL) ? EPI_RESID : EPI_STORE);
  a.out = y;
  a.ldo = n;
  a.resid = residual;
  a.ldr = n;
  a.has_bias = (epilogue & EE_EPI_BIAS) ? 1 : 0;
  cudaStream_t s = (cudaStream_t)stream;
  return act_dtype == EE_BF16 ? launch_gemm_d<__nv_bfloat16>(a, s) : launch_gemm_d<__half>(a, s);
}

int ee_wq_gemm_status(int32_t* status, int32_t reset) {
  if (!status) return EE_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return EE_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int)) != cudaSuccess) return EE_ERR_LAUNCH;
  *status = v;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int)) != cudaSuccess) return EE_ERR_LAUNCH;
  }
  return EE_OK;
}

}  // extern "C"
