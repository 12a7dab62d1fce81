// ee_common.cuh -- shared device primitives for the sm_100a kernels:
// activation-type traits, global loads with explicit cache behaviour,
// warp-level bf16/f16 MMA, in-register int4/int8 -> bf16/f16 dequantisation
// and the bounded grid barrier used by the persistent sampler.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ee_b200.h"

#define EE_DEV __device__ __forceinline__

namespace ee {

constexpr int kWarps = 8;             // warps per CTA in every kernel here
constexpr int kThreads = kWarps * 32;
constexpr int kKBlock = 128;          // K handled by one warp per k-block
constexpr int kMTile = 64;            // tokens per GEMM unit (8 mma n8 tiles)

// ---------------------------------------------------------------------------
// activation traits
// ---------------------------------------------------------------------------
template <typename T> struct Act;

template <> struct Act<__nv_bfloat16> {
  static EE_DEV float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static EE_DEV __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static EE_DEV float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  // two halves of a packed 32-bit word -> floats
  static EE_DEV float2 unpack2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  }
  static EE_DEV uint32_t pack2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  // bit patterns for the magic-number dequantisation
  static constexpr uint32_t kInt4Or = 0x43004300u;   // bf16 128.0 in both halves
  static constexpr uint32_t kOne2 = 0x3F803F80u;     // 1.0, 1.0
  static EE_DEV uint32_t neg_offset2(float off) {    // -(off) in both halves
    return pack2(-off, -off);
  }
  static constexpr float kInt4Base = 128.0f;
};

template <> struct Act<__half> {
  static EE_DEV float to_f(__half v) { return __half2float(v); }
  static EE_DEV __half from_f(float v) { return __float2half_rn(v); }
  static EE_DEV float round(float v) { return __half2float(__float2half_rn(v)); }
  static EE_DEV float2 unpack2(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  static EE_DEV uint32_t pack2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr uint32_t kInt4Or = 0x64006400u;   // f16 1024.0 in both halves
  static constexpr uint32_t kOne2 = 0x3C003C00u;
  static EE_DEV uint32_t neg_offset2(float off) { return pack2(-off, -off); }
  static constexpr float kInt4Base = 1024.0f;
};

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------
// Read-only data that is never written while a kernel runs (weights, scales):
// non-coherent path, no L1 allocation (each CTA streams its tile once).
EE_DEV uint4 ld_weight16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// Data produced earlier in the same launch by other CTAs: L2 only (cg), and a
// memory clobber so the compiler never moves it across a barrier.
EE_DEV uint4 ld_act16(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");
  return r;
}
EE_DEV uint16_t ld_act2(const void* p) {
  uint16_t r;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(r) : "l"(p) : "memory");
  return r;
}
EE_DEV uint32_t ld_act4(const void* p) {
  uint32_t r;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}

EE_DEV float ld_act_f32(const float* p) {
  float r;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(r) : "l"(p) : "memory");
  return r;
}
EE_DEV float2 ld_act_f2(const float* p) {
  float2 r;
  asm volatile("ld.global.cg.v2.f32 {%0,%1}, [%2];" : "=f"(r.x), "=f"(r.y) : "l"(p) : "memory");
  return r;
}
template <typename T> EE_DEV float ld_act_scalar(const T* p) {
  uint16_t b = ld_act2(p);
  return Act<T>::to_f(*reinterpret_cast<T*>(&b));
}
template <typename T> EE_DEV float ld_param(const T* p) {  // read-only params
  return Act<T>::to_f(__ldg(p));
}

// ---------------------------------------------------------------------------
// warp MMA m16n8k16, fp32 accumulate
// ---------------------------------------------------------------------------
template <typename T> EE_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1);
template <> EE_DEV void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                uint32_t a2, uint32_t a3, uint32_t b0,
                                                uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <> EE_DEV void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// bit helpers
// ---------------------------------------------------------------------------
EE_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// (a & b) ^ c
EE_DEV uint32_t and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
template <typename T> EE_DEV uint32_t fma2(uint32_t a, uint32_t b, uint32_t c);
template <> EE_DEV uint32_t fma2<__nv_bfloat16>(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
template <> EE_DEV uint32_t fma2<__half>(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// ---------------------------------------------------------------------------
// dequantisation into MMA operand registers
//
// Nibble -> value: OR the nibble into the mantissa of 128.0 (bf16) / 1024.0
// (f16), which gives base + u exactly, then one packed FMA subtracts
// (base + zero). Symmetric int4 stores two's-complement nibbles; XOR with 8
// maps them to u = q + 8, i.e. zero point 8.
// ---------------------------------------------------------------------------
// byte p (0..3) of w -> {lo nibble, hi nibble} as two packed values u + base
template <typename T> EE_DEV uint32_t nib_pair(uint32_t w, uint32_t w_shr4, int p, uint32_t xor8) {
  uint32_t sel = (uint32_t)p | ((uint32_t)(4 + p) << 8);
  uint32_t r = prmt(w, w_shr4, sel);
  return and_xor(r, 0x000F000Fu, Act<T>::kInt4Or ^ xor8);
}

// int8: bytes (i, j) of w (already XORed with 0x80808080) -> packed {q_i, q_j}
template <typename T> EE_DEV uint32_t int8_pair(uint32_t wx, int i, int j);
template <> EE_DEV uint32_t int8_pair<__nv_bfloat16>(uint32_t wx, int i, int j) {
  // fp32 magic 2^23 + u, subtract 2^23 + 128 -> exact q, then pack to bf16x2 (exact)
  float fi = __uint_as_float(prmt(wx, 0x4Bu, 0x4550u | (uint32_t)i)) - 8388736.0f;
  float fj = __uint_as_float(prmt(wx, 0x4Bu, 0x4550u | (uint32_t)j)) - 8388736.0f;
  return Act<__nv_bfloat16>::pack2(fi, fj);
}
template <> EE_DEV uint32_t int8_pair<__half>(uint32_t wx, int i, int j) {
  // f16 magic 1024 + u in each half, subtract 1152 -> exact q
  uint32_t r = prmt(wx, 0x64u, (uint32_t)i | (4u << 4) | ((uint32_t)j << 8) | (4u << 12));
  return fma2<__half>(r, 0x3C003C00u, 0xE480E480u);
}

// ---------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------
EE_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
EE_DEV unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
EE_DEV int ld_volatile_i32(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

EE_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
EE_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// cluster helpers (a launch without a cluster is a cluster of one CTA)
EE_DEV uint32_t cl_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
EE_DEV uint32_t cl_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
EE_DEV uint32_t cl_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
EE_DEV uint32_t cl_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
#ifndef EE_PDL
#define EE_PDL 1
#endif
// Kernel entry under programmatic dependent launch (see ee_host.h): wait for
// the predecessor grids (complete, memory visible), then allow the successor
// to launch. A no-op for kernels launched without the attribute.
EE_DEV void pdl_entry() {
#if EE_PDL
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}
EE_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
EE_DEV uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
EE_DEV float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr) : "memory");
  return v;
}
EE_DEV void st_dsmem_f2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
EE_DEV void st_dsmem_f4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
// Remote store into a cluster peer's shared memory that completes 16 bytes
// on the peer's mbarrier `bar` (both shared::cluster addresses from mapa).
EE_DEV void st_async_f4(uint32_t addr, float a, float b, float c, float d, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
               : "memory");
}
EE_DEV float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
EE_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
EE_DEV void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
EE_DEV void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
EE_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> EE_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
EE_DEV uint4 lds16(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}

EE_DEV float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

}  // namespace ee
