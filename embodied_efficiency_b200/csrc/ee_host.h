// ee_host.h -- host-side helpers shared by the C ABI translation units:
// argument validation and a read-only per-device properties cache.
#pragma once

#include <atomic>
#include <stdint.h>

#include <cuda_runtime.h>

#include "../../include/ee_b200.h"

// Programmatic dependent launch of the standalone kernels (GEMMs, norm,
// attention, row operations): each is launched with programmatic stream
// serialization and, first thing, waits for its predecessors
// (griddepcontrol.wait) and then lets its successor launch
// (griddepcontrol.launch_dependents), so a successor's launch and CTA
// scheduling overlap this kernel's run while its memory accesses still come
// after this kernel completes. The fused sampler is launched without it.
#ifndef EE_PDL
#define EE_PDL 1
#endif

namespace ee {

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// append the programmatic-serialization attribute (with EE_PDL) to a launch's list
inline void add_pdl_attr(cudaLaunchAttribute* attrs, unsigned int& n) {
  if (EE_PDL) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
}

// a plain launch (no cluster) with the programmatic-serialization attribute
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  unsigned int n = 0;
  add_pdl_attr(attr, n);
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, fn, args...);
}

struct DevProps {
  int sms;        // multiprocessor count
  int major;      // compute capability
  int minor;
  int smem_optin; // max shared memory per block (opt-in), bytes
};

// Properties of the current device, read once per device and then cached.
inline const DevProps* device_props() {
  static std::atomic<int> ready[64];
  static DevProps props[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (ready[dev].load(std::memory_order_acquire) == 0) {
    DevProps p{};
    if (cudaDeviceGetAttribute(&p.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&p.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&p.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&p.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess)
      return nullptr;
    props[dev] = p;  // identical values if two threads race here
    ready[dev].store(1, std::memory_order_release);
  }
  return &props[dev];
}

inline int device_sms() {
  const DevProps* p = device_props();
  return p ? p->sms : 148;
}

// Allow `fn` the largest dynamic shared memory the device permits next to its
// static shared memory (once per device and kernel).
template <typename F>
inline void allow_max_smem(F fn, std::atomic<int>* done /* [64] */) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  if (done[dev].load(std::memory_order_acquire)) return;
  const DevProps* p = device_props();
  cudaFuncAttributes fa{};
  if (!p || cudaFuncGetAttributes(&fa, fn) != cudaSuccess) return;
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       p->smem_optin - (int)fa.sharedSizeBytes);
  done[dev].store(1, std::memory_order_release);
}

// The kernels are built for sm_100a only.
inline int check_device() {
  const DevProps* p = device_props();
  if (!p) return EE_ERR_DEVICE;
  if (p->major != 10) return EE_ERR_DEVICE;
  return EE_OK;
}

// Shape / format checks for one linear layer with expected [n, k].
inline int validate_linear(const ee_linear& L, int32_t n, int32_t k) {
  if (!L.weight) return EE_ERR_ARG;
  if (L.n != n || L.k != k) return EE_ERR_SHAPE;
  if (L.wkind < EE_W_DENSE || L.wkind > EE_W_UINT4Z) return EE_ERR_ARG;
  if (k < 128 || (k % 128) != 0) return EE_ERR_SHAPE;
  if (!aligned16(L.weight)) return EE_ERR_ALIGN;
  if (L.wkind != EE_W_DENSE) {
    if (!L.scales) return EE_ERR_ARG;
    if (L.scale_dtype != EE_F32 && L.scale_dtype != EE_F16) return EE_ERR_DTYPE;
    if (L.group <= 0 || (k % L.group) != 0) return EE_ERR_SHAPE;
    if (L.group != k && (L.group % 128) != 0) return EE_ERR_SHAPE;
    if (L.wkind == EE_W_UINT4Z && !L.zeros) return EE_ERR_ARG;
  }
  return EE_OK;
}

}  // namespace ee
