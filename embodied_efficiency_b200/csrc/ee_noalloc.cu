// ee_noalloc.cu -- the fused sampler for callers that cannot allocate device
// memory.
//
// Some callers cannot call cudaMalloc at all: a hard-real-time control loop
// must not (an allocation can synchronise the device and take an unbounded
// time in the middle of a control period), and a host that binds this
// library through a foreign-function interface often owns all device memory
// through its own allocator and has no buffer to lend us. For them
// ee_flow_sample_noalloc runs the same single-launch sampler as
// ee_flow_sample, with its workspace in a fixed-size array that is part of
// this library's device image: every GPU that loads the library holds
// kStaticScratchBytes for it until the process exits.
#include <atomic>
#include <mutex>

#include "ee_host.h"

namespace ee {

// Maximum workspace of a no-allocation sampler call (4 MiB: a batch-1 call of
// an expert up to d_model 2048 / 18 blocks / MLP 8192 needs about 2.8 MiB).
constexpr size_t kStaticScratchBytes = 4u << 20;

static __device__ __align__(256) unsigned char g_sampler_scratch[kStaticScratchBytes];

// Identity of the CUDA context current on this thread (0 when the driver
// cannot tell): cuCtxGetCurrent + cuCtxGetId, looked up from the driver once
// (no libcuda link).
typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);
static unsigned long long current_context_id() {
  static std::once_flag once;
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    cudaGetLastError();
  });
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
  return id;
}

// Device address of g_sampler_scratch on the current device, looked up once
// per device and context (the symbol's host-side name is not a device
// address). A device whose context was destroyed and made again
// (cudaDeviceReset) reloads the library's device image, possibly at another
// address, so the lookup is repeated for the new context.
static void* scratch_address(int* rc) {
  static std::mutex mu;
  static void* addr[64] = {};
  static unsigned long long ctx_of[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *rc = EE_ERR_DEVICE;
    return nullptr;
  }
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev] || ctx != ctx_of[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sampler_scratch) != cudaSuccess || !p) {
      *rc = EE_ERR_LAUNCH;
      return nullptr;
    }
    addr[dev] = p;
    ctx_of[dev] = ctx;
  }
  *rc = EE_OK;
  return addr[dev];
}

}  // namespace ee

extern "C" {

int ee_flow_sample_noalloc(const ee_expert* ex, const void* x_in, const void* t0, void* x_out,
                           int32_t n_steps, int32_t mode, ee_stream_t stream) {
  if (!ex || !x_in || !x_out) return EE_ERR_ARG;
  const size_t need = ee_flow_sample_workspace_bytes(ex, n_steps);
  if (need == 0) return EE_ERR_ARG;
  if (need > ee::kStaticScratchBytes) return EE_ERR_WORKSPACE;
  int rc = ee::check_device();
  if (rc) return rc;
  void* ws = ee::scratch_address(&rc);
  if (rc) return rc;
  // ee_flow_sample clears the parts of the workspace that must start at zero
  // (barrier counter, status word, row statistics) on the stream before its
  // launch, and allocates nothing.
  return ee_flow_sample(ex, x_in, t0, x_out, n_steps, mode, ws, ee::kStaticScratchBytes, stream);
}

}  // extern "C"
