// ee_stream.cuh -- standalone weight-only dequant-GEMM for few tokens
// (M <= 64): a TMA-fed streaming kernel.
//
// With M <= 64 the GEMM reads each weight byte once and does little math per
// byte, so its speed is set by how many weight bytes each SM keeps in flight
// from HBM. The kernel is built around that:
//
//  * a unit is 128 weight rows over all of K, computed by one thread-block
//    cluster of S CTAs; CTA rank r owns the K slice of k-blocks
//    [r*kbc, (r+1)*kbc) (a k-block is 128 k), and the grid holds one
//    cluster per unit, so every CTA streams its slice exactly once;
//  * one producer warp issues 2-D TMA tile loads (weights [128 rows x one
//    k-block] in the reference layout, plus the matching activation tile
//    [8*JT tokens x 128 k]) into a ring of `nst` shared-memory stages, each
//    stage guarded by a "full" mbarrier (TMA transaction bytes) and an
//    "empty" mbarrier (the consuming warps), so up to nst k-blocks are in
//    flight per SM;
//  * 8 x kStreamKG consumer warps: warp = (row group rw: 16 rows, k group
//    kg), the k groups taking every kStreamKG-th k-block (several warps per
//    scheduler, so one warp's dependency stalls are covered by the others). Each warp
//    dequantises its 16 rows in registers (nibble / byte -> exact bf16/f16 integers, see
//    ee_gemm.cuh) and runs m16n8k16 MMAs with the weights as the A operand
//    and the tokens as B; the fp32 per-(row, group) scale multiplies each
//    k-block's partial sum;
//  * the kStreamKG*S partial tiles of a unit (S CTAs x kStreamKG k groups) are pushed over
//    distributed shared memory to the CTA that owns their rows (128/S rows
//    per CTA), summed there in a fixed order (deterministic), and the owner
//    applies bias / GELU / residual and stores 16-byte chunks.
//
// Shared-memory tiles come from TMA with the 128-byte swizzle for 128-byte
// lines (int8 weights, bf16 weights in two half-k-block boxes, activations
// in two 64-k boxes); int4 rows are 64 bytes per k-block and are read
// conflict-free without a swizzle.
#pragma once

#include <atomic>

#include "ee_gemm.cuh"
#include "ee_host.h"
#include "ee_tma.cuh"

namespace ee {

#ifndef EE_STREAM_KG
#define EE_STREAM_KG 2
#endif
constexpr int kStreamKG = EE_STREAM_KG;            // k groups: consumer warp sets taking every kStreamKG-th k-block
constexpr int kStreamCWarps = 8 * kStreamKG;       // consumer warps: 8 row groups x kStreamKG k groups
constexpr int kStreamCThreads = kStreamCWarps * 32;
constexpr int kStreamWarps = kStreamCWarps + 1;  // + 1 producer warp
constexpr int kStreamThreads = kStreamWarps * 32;
constexpr int kStreamMaxTokens = 64;
#ifndef EE_STREAM_MAX_STAGES
#define EE_STREAM_MAX_STAGES 24
#endif
constexpr int kStreamMaxStages = EE_STREAM_MAX_STAGES;  // ring depth cap

struct StreamArgs {
  ee_linear w;
  int M;
  int epi;
  int has_bias;
  void* out;
  long long ldo;
  const void* resid;
  long long ldr;
  int lsplit;          // log2(S), S = CTAs per cluster along K
  int kbc;             // k-blocks per CTA
  int nst;             // ring stages
  int ps;              // floats per row of a partial tile (8*JT + 4)
  uint32_t stage_bytes;
  uint32_t off_bar, off_scal, off_recv, off_res, off_bias;  // from the 1024-aligned base
  // activations resident for the CTA's whole K slice (few tokens): copied
  // once at the start into [kbc][2 boxes][8*JT rows][128 B] (128-byte
  // swizzle), so the ring carries weights only
  int xres;
  uint32_t off_x;
  const void* x;
  long long ldx;
  int* status;         // device status word (EE_ERR_TIMEOUT / EE_ERR_LAUNCH)
  unsigned long long timeout_ns;
};

template <int KIND> __host__ __device__ constexpr uint32_t stream_wbytes() {
  return KIND == EE_W_DENSE ? 32768u : (KIND == EE_W_INT8 ? 16384u : 8192u);
}

template <typename T, int KIND, int JT>
__global__ void __launch_bounds__(kStreamThreads, 1)
    wq_stream_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                     const __grid_constant__ StreamArgs a) {
  constexpr int WPR = words_per_row(KIND);
  constexpr uint32_t WB = stream_wbytes<KIND>();
  constexpr uint32_t XB = 2048u * JT;  // two boxes of [8*JT tokens][64 k]
  extern __shared__ __align__(1024) char smem_raw[];
  const uint32_t base0 = smem_u32(smem_raw);
  const uint32_t sb = (base0 + 1023u) & ~1023u;
  char* smem = smem_raw + (sb - base0);
  pdl_entry();

  const int S = 1 << a.lsplit;
  if ((int)cl_size() != S) {  // launched without the planned cluster: no work
    if (threadIdx.x == 0) atomicCAS(a.status, 0, (int)EE_ERR_LAUNCH);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rank = (int)cl_rank();
  const int n0 = (int)cl_id() * 128;
  const int RS = 128 >> a.lsplit;  // rows reduced and stored by this CTA
  const int kb_first = rank * a.kbc;
  const ee_linear& L = a.w;
  const uint32_t bar_full = sb + a.off_bar, bar_empty = bar_full + 8u * a.nst;

  if (warp == kStreamCWarps && lane == 0) {
    tma_prefetch_map(&tw);
    if (!a.xres) tma_prefetch_map(&tx);
    for (int s = 0; s < a.nst; ++s) {
      mbar_init(bar_full + 8u * s, 1);
      mbar_init(bar_empty + 8u * s, 8);  // the 8 row-group warps of the k group that consumes the stage
    }
    mbar_fence_init();
  }
  // consumers: the scale / zero point of (row r, k-block kb) is entry
  // kb * 128 + r; the first 4 per thread are requested now (in flight while
  // the producer starts its copies), the rest after the CTA barrier below
  float sv[4], zv[4];
  auto load_scale = [&](int i, float& sc, float& zp) {
    sc = zp = 0.f;
    if (i < a.kbc * 128) {
      const int kb = i >> 7, r = i & 127;
      const int n = min(n0 + r, L.n - 1);
      const size_t si = (size_t)n * (L.k / L.group) + ((size_t)(kb_first + kb) * kKBlock) / L.group;
      sc = L.scale_dtype == EE_F32 ? __ldg(reinterpret_cast<const float*>(L.scales) + si)
                                   : __half2float(__ldg(reinterpret_cast<const __half*>(L.scales) + si));
      if (KIND == EE_W_UINT4Z) zp = __half2float(__ldg(reinterpret_cast<const __half*>(L.zeros) + si));
    }
  };
  if (KIND != EE_W_DENSE && warp < kStreamCWarps) {
#pragma unroll
    for (int u = 0; u < 4; ++u) load_scale(threadIdx.x + kStreamCThreads * u, sv[u], zv[u]);
  }

  __syncthreads();

  if (warp == kStreamCWarps) {
    // ---------------- producer: TMA loads into the ring ----------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      int s = 0, sph = 0;
      for (int kb = 0; kb < a.kbc; ++kb) {
        if (kb >= a.nst && !mbar_wait(bar_empty + 8u * s, (uint32_t)(sph ^ 1), a.timeout_ns)) {
          ok = false;
          break;
        }
        const uint32_t st = sb + (uint32_t)s * a.stage_bytes, fb = bar_full + 8u * s;
        mbar_arrive_expect_tx(fb, a.xres ? WB : WB + XB);
        const int kabs = kb_first + kb;
        if (KIND == EE_W_DENSE) {
          tma_load_2d(st, &tw, kabs * 256, n0, fb);
          tma_load_2d(st + 16384u, &tw, kabs * 256 + 128, n0, fb);
        } else {
          tma_load_2d(st, &tw, kabs * (KIND == EE_W_INT8 ? 128 : 64), n0, fb);
        }
        if (!a.xres) {
          tma_load_2d(st + WB, &tx, kabs * 128, 0, fb);
          tma_load_2d(st + WB + XB / 2, &tx, kabs * 128 + 64, 0, fb);
        }
        ++issued;
        if (++s == a.nst) {
          s = 0;
          sph ^= 1;
        }
      }
      if (!ok) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
      // every issued copy has landed before this CTA can leave
      for (int kb = issued > a.nst ? issued - a.nst : 0; kb < issued; ++kb)
        if (!mbar_wait(bar_full + 8u * (kb % a.nst), (kb / a.nst) & 1, a.timeout_ns))
          atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    float* scal = reinterpret_cast<float*>(smem + a.off_scal);  // [kbc][128]
    float* zero = scal + a.kbc * 128;                            // [kbc][128] (zero points)
    float* sbias = reinterpret_cast<float*>(smem + a.off_bias);  // [RS]
    const int nbase = n0 + rank * RS;
    if (KIND != EE_W_DENSE) {
      for (int base = 0; base < a.kbc * 128; base += 4 * kStreamCThreads) {
        if (base > 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u) load_scale(base + threadIdx.x + kStreamCThreads * u, sv[u], zv[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = base + threadIdx.x + kStreamCThreads * u;
          if (i < a.kbc * 128) {
            scal[i] = sv[u];
            if (KIND == EE_W_UINT4Z) zero[i] = zv[u];
          }
        }
      }
    }
    if (threadIdx.x < RS) {
      const int n = nbase + threadIdx.x;
      sbias[threadIdx.x] = (a.has_bias && n < L.n) ? ld_param(reinterpret_cast<const T*>(L.bias) + n) : 0.f;
    }
    if (a.xres) {
      // the CTA's activation slice, in the layout TMA would have produced
      const char* xb = reinterpret_cast<const char*>(a.x);
      const int per_kb = 2 * 8 * JT * 8;  // 16-byte chunks per k-block
      for (int i = threadIdx.x; i < a.kbc * per_kb; i += kStreamCThreads) {
        const int kb = i / per_kb, rem = i - kb * per_kb;
        const int box = rem / (8 * JT * 8), rem2 = rem - box * (8 * JT * 8);
        const int row = rem2 >> 3, cc = rem2 & 7;
        const bool ok = row < a.M;
        const char* src = xb + ((size_t)(ok ? row : 0) * a.ldx + (size_t)(kb_first + kb) * kKBlock + box * 64 + cc * 8) * 2;
        cp_async16(sb + a.off_x + (uint32_t)(kb * 2 + box) * (XB / 2) + sw128(row, cc), src, ok);
      }
    }
    if (a.epi == EPI_RESID) {
      const int rcpr = RS / 8;
      const char* rb = reinterpret_cast<const char*>(a.resid);
      for (int i = threadIdx.x; i < a.M * rcpr; i += kStreamCThreads) {
        const int row = i / rcpr, c = i - row * rcpr;
        const bool ok = nbase + c * 8 + 8 <= L.n;
        const char* src = rb + ((size_t)row * a.ldr + (ok ? nbase + c * 8 : 0)) * 2;
        cp_async16(sb + a.off_res + (uint32_t)((row * RS + c * 8) * 2), src, ok);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    named_sync(1, kStreamCThreads);

    const int rw = warp & 7, kg = warp >> 3;
    const int jt = min(JT, (a.M + 7) >> 3);  // active 8-token tiles
    float acc[1][JT][4];
#pragma unroll
    for (int j = 0; j < JT; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[0][j][c] = 0.f;

    int s = kg % a.nst, sph = (kg / a.nst) & 1;  // ring position of k-block kb (advanced below)
    for (int kb = kg; kb < a.kbc; kb += kStreamKG) {
      if (!mbar_wait(bar_full + 8u * s, (uint32_t)sph, a.timeout_ns)) {
        if (lane == 0) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
        break;
      }
      const uint32_t st = sb + (uint32_t)s * a.stage_bytes;
      uint32_t A[1][8][4];
      float sc[1][2];
#pragma unroll
      for (int mi = 0; mi < 1; ++mi) {
        uint4 w[2][WPR];
        float z[2] = {0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = 16 * rw + g + 8 * h;
          if (KIND == EE_W_DENSE) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[h][i] = lds16(st + (uint32_t)(t >> 1) * 16384u + sw128(r, (4 * t + i) & 7));
            sc[mi][h] = 1.f;
          } else if (KIND == EE_W_INT8) {
#pragma unroll
            for (int i = 0; i < 2; ++i) w[h][i] = lds16(st + sw128(r, 2 * t + i));
            sc[mi][h] = scal[kb * 128 + r];
          } else {
            w[h][0] = lds16(st + (uint32_t)(r * 64 + t * 16));
            sc[mi][h] = scal[kb * 128 + r];
            if (KIND == EE_W_UINT4Z) z[h] = zero[kb * 128 + r];
          }
        }
        Gemm<T, KIND>::dequant(w, z, A[mi]);
      }
      const uint32_t xs = (a.xres ? sb + a.off_x + (uint32_t)kb * XB : st + WB) + (uint32_t)(t >> 1) * (XB / 2);
#pragma unroll
      for (int j = 0; j < JT; ++j) {
        if (j < jt) {
          const int row = 8 * j + g;
          uint4 xq[4];
#pragma unroll
          for (int s2 = 0; s2 < 4; ++s2) xq[s2] = lds16(xs + sw128(row, (4 * t + s2) & 7));
#pragma unroll
          for (int mi = 0; mi < 1; ++mi) {
            // four chains of two MMAs (chain c: steps 2c, 2c+1 = the k of xq[c])
            float pc[4][4];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
#pragma unroll
              for (int e = 0; e < 4; ++e) pc[cc][e] = 0.f;
#pragma unroll
            for (int hs = 0; hs < 2; ++hs)
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) {
                const int s = 2 * cc + hs;
                mma16816<T>(pc[cc], A[mi][s][0], A[mi][s][1], A[mi][s][2], A[mi][s][3], comp(xq[cc], 2 * hs),
                            comp(xq[cc], 2 * hs + 1));
              }
            acc[mi][j][0] += sc[mi][0] * ((pc[0][0] + pc[1][0]) + (pc[2][0] + pc[3][0]));
            acc[mi][j][1] += sc[mi][0] * ((pc[0][1] + pc[1][1]) + (pc[2][1] + pc[3][1]));
            acc[mi][j][2] += sc[mi][1] * ((pc[0][2] + pc[1][2]) + (pc[2][2] + pc[3][2]));
            acc[mi][j][3] += sc[mi][1] * ((pc[0][3] + pc[1][3]) + (pc[2][3] + pc[3][3]));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8u * s);
      s += kStreamKG;
      while (s >= a.nst) {
        s -= a.nst;
        sph ^= 1;
      }
    }

    // push this warp's partial tile: rows of rank o go to rank o's receive area
    const uint32_t recv = sb + a.off_recv;
    const int qslot = rank * kStreamKG + kg;
    const int rshift = 7 - a.lsplit;
#pragma unroll
    for (int mi = 0; mi < 1; ++mi)
#pragma unroll
      for (int j = 0; j < JT; ++j)
        if (j < jt) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = 16 * rw + g + 8 * h;
            const int owner = row >> rshift, lrow = row & (RS - 1);
            const uint32_t off = (uint32_t)(((qslot * RS + lrow) * a.ps + 8 * j + 2 * t) * 4);
            st_dsmem_f2(mapa(recv + off, (uint32_t)owner), acc[mi][j][2 * h], acc[mi][j][2 * h + 1]);
          }
        }
  }
  cluster_sync();  // every partial of the unit has arrived; the ring is idle

  if (warp < kStreamCWarps) {
    // sum the kStreamKG*S partials of this CTA's RS rows in slot order
    const int ntok = min(JT, (a.M + 7) >> 3) * 8;
    const float* R = reinterpret_cast<const float*>(smem + a.off_recv);
    float* E = reinterpret_cast<float*>(smem);  // [ntok][RS], reuses the ring
    const int nq = kStreamKG * S;
    for (int i = threadIdx.x; i < RS * (ntok >> 2); i += kStreamCThreads) {
      const int row = i % RS, c4 = i / RS;
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < nq; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(R + (q * RS + row) * a.ps + 4 * c4);
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      E[(4 * c4 + 0) * RS + row] = sum.x;
      E[(4 * c4 + 1) * RS + row] = sum.y;
      E[(4 * c4 + 2) * RS + row] = sum.z;
      E[(4 * c4 + 3) * RS + row] = sum.w;
    }
    named_sync(1, kStreamCThreads);

    // epilogue on 8-column chunks: bias, round, GELU / residual, 16-byte stores
    const ee_linear& Lw = a.w;
    const T* sres = reinterpret_cast<const T*>(smem + a.off_res);
    const float* sbias = reinterpret_cast<const float*>(smem + a.off_bias);
    T* out = reinterpret_cast<T*>(a.out);
    const int nbase = n0 + rank * RS;
    const int cpt = RS / 8;
    const bool vec = (a.ldo % 8) == 0;
    for (int i = threadIdx.x; i < a.M * cpt; i += kStreamCThreads) {
      const int tok = i / cpt, ch = i - tok * cpt;
      const int nc = nbase + 8 * ch;
      if (nc >= Lw.n) continue;
      uint4 rq = make_uint4(0, 0, 0, 0);
      if (a.epi == EPI_RESID) rq = *reinterpret_cast<const uint4*>(sres + tok * RS + 8 * ch);
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float y = Act<T>::round(E[tok * RS + 8 * ch + e] + sbias[8 * ch + e]);
        if (a.epi == EPI_GELU) {
          y = Act<T>::round(gelu_erf(y));
        } else if (a.epi == EPI_RESID) {
          const float2 rf = Act<T>::unpack2(comp(rq, e >> 1));
          y = Act<T>::round(((e & 1) ? rf.y : rf.x) + y);
        }
        v[e] = y;
      }
      T* dst = out + (size_t)tok * a.ldo + nc;
      if (vec && nc + 8 <= Lw.n) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(Act<T>::pack2(v[0], v[1]), Act<T>::pack2(v[2], v[3]),
                                                    Act<T>::pack2(v[4], v[5]), Act<T>::pack2(v[6], v[7]));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (nc + e < Lw.n) dst[e] = Act<T>::from_f(v[e]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// Launch one streaming GEMM; *used = false (and nothing launched) when the
// request is outside this kernel's domain (the caller takes another path).
template <typename T, int KIND, int JT>
int stream_launch_k(const GemmArgs& g, int* status, cudaStream_t st, bool* used) {
  *used = false;
  const DevProps* dp = device_props();
  if (!dp) return EE_ERR_DEVICE;
  const int N = g.w.n, K = g.w.k, M = g.M;
  const long long U = (N + 127) / 128;
  if (U > 0x7fffffffLL / 8) return EE_OK;
  // at most 4 CTAs per cluster: 8-CTA splits measured slower on every shape
  // that allows them (2048 x 8192 int4, M = 1: 13.7 vs 11.4 us with 4)
  int S = 4;
  while (S > 1 && ((K % (kKBlock * S)) != 0 || U * S > dp->sms)) S >>= 1;
  const int lsplit = S == 8 ? 3 : (S == 4 ? 2 : (S == 2 ? 1 : 0));
  const int kbc = K / (kKBlock * S), RS = 128 / S;
  // few tokens: the activation slice stays resident (<= 64 KB)
  const uint32_t xres_bytes = (uint32_t)kbc * 2048u * JT;
  const int xres = (JT <= 4 && xres_bytes <= 65536u) ? 1 : 0;
  const uint32_t stage = align_up(stream_wbytes<KIND>() + (xres ? 0u : 2048u * JT), 1024u);
  const int ps = 8 * JT + 4;
  const uint32_t scal = KIND == EE_W_DENSE ? 0u : (uint32_t)kbc * 128u * 4u * (KIND == EE_W_UINT4Z ? 2u : 1u);
  const uint32_t recv = (uint32_t)kStreamKG * 128u * ps * 4u;
  const uint32_t res = g.epi == EPI_RESID ? (uint32_t)(8 * JT * RS * 2) : 0u;
  const uint32_t fixed = 16u * (uint32_t)kStreamMaxStages + 16u + scal + 16u + recv + 16u + res + 16u + (uint32_t)RS * 4u + 1024u +
                         (xres ? xres_bytes + 1024u : 0u);
  if ((uint32_t)dp->smem_optin <= fixed + stage) return EE_OK;
  // as many k-blocks in flight as shared memory holds (up to kStreamMaxStages):
  // with one CTA per SM the ring depth is what keeps HBM busy
  int nst = (int)(((uint32_t)dp->smem_optin - fixed) / stage);
  nst = nst < kStreamMaxStages ? nst : kStreamMaxStages;
  nst = nst < kbc ? nst : kbc;
  // a stage that is reused must always be consumed by the same k group
  // (k-block kb lands in stage kb % nst and is consumed by group kb % kStreamKG):
  // a waiter of another group could otherwise be two barrier phases ahead
  if (nst < kbc) nst -= nst % kStreamKG;
  if (nst < 1) return EE_OK;

  StreamArgs a{};
  a.w = g.w;
  a.M = M;
  a.epi = g.epi;
  a.has_bias = g.has_bias;
  a.out = g.out;
  a.ldo = g.ldo;
  a.resid = g.resid;
  a.ldr = g.ldr;
  a.lsplit = lsplit;
  a.kbc = kbc;
  a.nst = nst;
  a.ps = ps;
  a.stage_bytes = stage;
  uint32_t ring = (uint32_t)nst * stage;
  const uint32_t ebytes = (uint32_t)(8 * JT * RS * 4);
  if (ring < ebytes) ring = ebytes;
  a.off_bar = ring;
  a.off_scal = align_up(a.off_bar + 16u * nst, 16u);
  a.off_recv = align_up(a.off_scal + scal, 16u);
  a.off_res = align_up(a.off_recv + recv, 16u);
  a.off_bias = align_up(a.off_res + res, 16u);
  a.xres = xres;
  a.x = g.x;
  a.ldx = g.ldx;
  a.off_x = align_up(a.off_bias + (uint32_t)RS * 4u, 1024u);
  const size_t smem = (size_t)a.off_x + (xres ? xres_bytes : 0u) + 1024;
  if (smem > (size_t)dp->smem_optin) return EE_OK;
  a.status = status;
  a.timeout_ns = 1000000000ull;

  CUtensorMap tw, tx;
  const uint64_t rowbytes = KIND == EE_W_DENSE ? 2ull * K : (KIND == EE_W_INT8 ? (uint64_t)K : (uint64_t)K / 2);
  const bool int4 = KIND == EE_W_INT4 || KIND == EE_W_UINT4Z;
  if (!make_tmap_2d(&tw, g.w.weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rowbytes, (uint64_t)N, rowbytes,
                    int4 ? 64u : 128u, 128u, int4 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B))
    return EE_OK;
  if (!make_tmap_2d(&tx, g.x, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)K, (uint64_t)M,
                    (uint64_t)g.ldx * 2u, 64u, 8u * JT, CU_TENSOR_MAP_SWIZZLE_128B))
    return EE_OK;

  auto fn = wq_stream_kernel<T, KIND, JT>;
  static std::atomic<int> smem_set[64];
  allow_max_smem(fn, smem_set);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(U * S));
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  unsigned int nattr = 1;
  add_pdl_attr(attr, nattr);
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  *used = true;
  return cudaLaunchKernelEx(&cfg, fn, tw, tx, a) == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

template <typename T, int KIND>
int stream_launch_j(const GemmArgs& g, int* status, cudaStream_t st, bool* used) {
  if (g.M <= 8) return stream_launch_k<T, KIND, 1>(g, status, st, used);
  if (g.M <= 16) return stream_launch_k<T, KIND, 2>(g, status, st, used);
  if (g.M <= 32) return stream_launch_k<T, KIND, 4>(g, status, st, used);
  return stream_launch_k<T, KIND, 8>(g, status, st, used);
}

// Streaming path for M <= 64 with TMA-compatible operands (16-byte aligned
// activations and row strides); *used says whether it applied.
template <typename T>
int launch_stream(const GemmArgs& g, int* status, cudaStream_t st, bool* used) {
  *used = false;
  if (g.M < 1 || g.M > kStreamMaxTokens || !status) return EE_OK;
  if (((uintptr_t)g.x & 15) || ((g.ldx * 2) & 15)) return EE_OK;
  switch (g.w.wkind) {
    case EE_W_DENSE: return stream_launch_j<T, EE_W_DENSE>(g, status, st, used);
    case EE_W_INT8: return stream_launch_j<T, EE_W_INT8>(g, status, st, used);
    case EE_W_INT4: return stream_launch_j<T, EE_W_INT4>(g, status, st, used);
    case EE_W_UINT4Z: return stream_launch_j<T, EE_W_UINT4Z>(g, status, st, used);
  }
  return EE_OK;
}

}  // namespace ee
