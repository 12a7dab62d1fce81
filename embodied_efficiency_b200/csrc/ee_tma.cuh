// ee_tma.cuh -- tensor-memory-accelerator (TMA) tile loads and shared-memory
// mbarriers for sm_100a, plus the host-side tensor-map encoder.
//
// Loads are plain (single-CTA destination) `cp.async.bulk.tensor` copies that
// signal an mbarrier with the number of bytes they deliver; no load here uses
// cluster multicast. Every wait is bounded by %globaltimer so a broken
// pipeline ends with an error status instead of a hang.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "ee_common.cuh"

namespace ee {

// ---------------------------------------------------------------------------
// device side
// ---------------------------------------------------------------------------
EE_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// make the initialised barriers visible to the async (TMA) proxy and the cluster
EE_DEV void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
EE_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
EE_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
EE_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the warp is parked in hardware (issuing
// nothing) until the phase completes or about `hint_ns` pass.
EE_DEV bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Wait for the phase of `bar` with the given parity to complete; gives up
// after `timeout_ns` and returns false. Waiting warps are suspended rather
// than spinning, so they take no issue slots from the warps doing work.
EE_DEV bool mbar_wait(uint32_t bar, uint32_t parity, unsigned long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, 200000u)) {
    if (globaltimer() - t0 > timeout_ns) return false;
  }
  return true;
}

// 2-D tiled TMA load of box (x, y) of `map` into shared memory at `dst`,
// completing `bytes` on `bar`. x counts elements of the innermost dimension.
EE_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Pull a tensor map (kernel parameter) into the descriptor cache early.
EE_DEV void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Named barrier over the first `threads` threads of the CTA (id 1..15).
EE_DEV void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Physical byte offset of 16-byte chunk `c` of 128-byte line `line` in a tile
// written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (tile base 1024-aligned):
// the chunk index is XORed with the line index modulo 8.
EE_DEV uint32_t sw128(int line, int c) { return (uint32_t)(line * 128 + ((c ^ (line & 7)) << 4)); }

}  // namespace ee

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
#ifndef __CUDACC_RTC__
#include <mutex>

namespace ee {

// cuTensorMapEncodeTiled from the driver, looked up once (no libcuda link).
inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major 2-D tensor [rows][cols] of `esize`-byte elements with a row
// stride of `stride_bytes`, read in boxes of box_cols x box_rows. Returns
// false if the driver rejects the description (alignment, sizes).
inline bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize,
                         uint64_t cols, uint64_t rows, uint64_t stride_bytes, uint32_t box_cols,
                         uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  auto enc = tmap_encoder();
  if (!enc) return false;
  if (((uintptr_t)base & 15) || (stride_bytes & 15) || ((box_cols * esize) & 15)) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {stride_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace ee
#endif
