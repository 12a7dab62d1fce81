// ee_tc.cuh -- weight-only dequant-GEMM on the 5th-generation tensor cores
// (tcgen05.mma with TMEM accumulators), for any number of tokens.
//
// Tile: 128 weight rows (the MMA's M) x NT tokens (the MMA's N, 16..256)
// over a K range, accumulated in fp32 in tensor memory. Roles inside a CTA
// of 18 warps:
//   warp 16     TMA producer: per k-block (128 k) one tile of raw weights in
//               the reference layout (int4 [128 rows x 64 B], 64-byte swizzle;
//               int8 [128 x 128 B] and dense 16-bit [128 x 2 x 128 B],
//               128-byte swizzle) and the activation tile [NT x 128 k]
//               (two 64-k boxes, 128-byte swizzle) into a ring of `ns` stages;
//   warps 0-15  dequantisers (four per scheduler, so one warp's dependency
//               stalls are covered by the others): raw weights -> q * scale in the activation
//               dtype (the reference kernel's order: exact integer, times the
//               scale rounded to the activation type, kernel/triton_gemm.py:
//               91-94 and :127-134), written into a ring of `na` A tiles in
//               the MMA's K-major 128-byte-swizzled layout; dense weights skip
//               this step (TMA writes the A tile directly);
//   warp 17     TMEM allocator and MMA issuer: one thread issues the eight
//               M128 x N x K16 MMAs of each k-block and commits their
//               completion to the barriers that free the stage and the A tile;
//   warps 0-15  epilogue: TMEM -> registers (each warp its 32-lane quarter,
//               a quarter of the columns), then either the final bias / GELU /
//               residual and the store, or -- when K is split over the S CTAs
//               of a cluster -- a push of the fp32 partial tile to the CTA
//               owning those rows, a fixed-order sum there and the epilogue.
// Every wait is bounded (%globaltimer); a timeout records EE_ERR_TIMEOUT in
// the status word and the CTA still drains its copies, releases TMEM and
// joins every cluster barrier.
#pragma once

#include <atomic>

#include "ee_gemm.cuh"
#include "ee_host.h"
#include "ee_tma.cuh"
#include "ee_umma.cuh"

namespace ee {

constexpr int kTcDqWarps = 16;  // dequantising / epilogue warps
constexpr int kTcDqThreads = kTcDqWarps * 32;
constexpr int kTcProdWarp = kTcDqWarps, kTcMmaWarp = kTcDqWarps + 1;
constexpr int kTcWarps = kTcDqWarps + 2;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcpEpiWarps = 8;  // epilogue warps of the persistent form (ee_tcp.cuh)
// With dense weights the persistent form's 16 dequantising warps have no
// work and join its epilogue (six warps per TMEM lane quarter).
template <int KIND>
constexpr int tcp_epi_warps() { return KIND == EE_W_DENSE ? kTcpEpiWarps + kTcDqWarps : kTcpEpiWarps; }
// per epilogue warp a [16 tokens][32 rows] staging tile of 16-bit values
template <int KIND>
constexpr uint32_t tcp_epi_bytes() { return (uint32_t)tcp_epi_warps<KIND>() * 16u * 32u * 2u; }

struct TcArgs {
  ee_linear w;
  int M;
  int epi;
  int has_bias;
  void* out;
  long long ldo;
  const void* resid;
  long long ldr;
  int lsplit;        // log2(S): CTAs of a cluster sharing one tile's K range
  int kbc;           // k-blocks per CTA
  int ns;            // TMA stages
  int na;            // dequantised A stages
  int ps;            // floats per row of a pushed partial tile (NT + 4)
  int n_units;       // 128-row weight tiles
  uint32_t stage_bytes;
  uint32_t off_a, off_bar, off_recv, off_tm;
  uint32_t off_sc;   // scale / zero-point ring [3 slots][2][256 threads][ITEMS] 4-byte words
  uint32_t off_ep;   // persistent form: per epilogue warp a [16 tokens][32 rows] staging tile
  int* status;
  unsigned long long timeout_ns;
};

template <int KIND> __host__ __device__ constexpr uint32_t tc_wbytes() {
  return KIND == EE_W_DENSE ? 32768u : (KIND == EE_W_INT8 ? 16384u : 8192u);
}
__host__ __device__ constexpr uint32_t tc_tmem_cols(int nt) { return nt < 32 ? 32u : (uint32_t)nt; }

template <typename T, int KIND>
struct TcDequant {
  // Scale (and zero point) element index of weight row n for group g is
  // n * ng + g. The dequantising threads keep their rows' n * ng and find g
  // from the absolute k-block without a division in the common cases.
  struct Groups {
    int ng;      // groups per row
    int kpg;     // k-blocks per group
    int shift;   // log2(kpg) when kpg is a power of two, else -1
  };
  static EE_DEV Groups groups(const ee_linear& L) {
    Groups gp;
    gp.ng = L.k / L.group;
    gp.kpg = L.group / kKBlock;
    gp.shift = (gp.kpg & (gp.kpg - 1)) == 0 ? __ffs(gp.kpg) - 1 : -1;
    return gp;
  }
  static EE_DEV int group_of(const Groups& gp, int kb) {
    return gp.ng == 1 ? 0 : (gp.shift >= 0 ? kb >> gp.shift : kb / gp.kpg);
  }
  // Asynchronously copy the 4-byte word holding element `si` of the scales
  // (and zero points) to shared memory (dst, dst + zoff). 16-bit values are
  // fetched as their aligned 4-byte word.
  static EE_DEV void stage_sz(const ee_linear& L, size_t si, uint32_t dst, uint32_t zoff) {
    if (L.scale_dtype == EE_F32)
      cp_async4(dst, reinterpret_cast<const float*>(L.scales) + si);
    else
      cp_async4(dst, reinterpret_cast<const char*>(L.scales) + ((si * 2) & ~(size_t)3));
    if (KIND == EE_W_UINT4Z) cp_async4(dst + zoff, reinterpret_cast<const char*>(L.zeros) + ((si * 2) & ~(size_t)3));
  }
  static EE_DEV float read_half(uint32_t word, bool hi) {
    return __half2float(__ushort_as_half((unsigned short)(hi ? (word >> 16) : (word & 0xFFFFu))));
  }
  static EE_DEV void read_sz(const ee_linear& L, size_t si, uint32_t src, uint32_t zoff, float& s, float& z) {
    uint32_t w;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w) : "r"(src));
    s = L.scale_dtype == EE_F32 ? __uint_as_float(w) : read_half(w, (si & 1) != 0);
    z = 0.f;
    if (KIND == EE_W_UINT4Z) {
      uint32_t wz;
      asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wz) : "r"(src + zoff));
      z = read_half(wz, (si & 1) != 0);
    }
  }
  // store 16 bytes = 8 values of chunk c (0..15) of A-tile row `row`
  static EE_DEV void st_a(uint32_t abase, int row, int c, uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3) {
    const uint32_t addr = abase + (uint32_t)(c >> 3) * 16384u + sw128(row, c & 7);
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v0), "r"(v1), "r"(v2), "r"(v3)
                 : "memory");
  }
  // One dequantising item: the raw 16-byte chunk `ch` of weight row `row`
  // in the TMA stage `st` -> q * scale (scale rounded to the activation type)
  // into the A tile `ab`.
  static EE_DEV void item(uint32_t st, uint32_t ab, int row, int ch, float scv, float zcv) {
    const uint32_t s2 = Act<T>::pack2(scv, scv);
    if (KIND == EE_W_INT8) {
      const uint4 raw = lds16(st + sw128(row, ch));
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t w0 = comp(raw, 2 * u) ^ 0x80808080u, w1 = comp(raw, 2 * u + 1) ^ 0x80808080u;
        st_a(ab, row, 2 * ch + u, hmul2<T>(int8_pair<T>(w0, 0, 1), s2), hmul2<T>(int8_pair<T>(w0, 2, 3), s2),
             hmul2<T>(int8_pair<T>(w1, 0, 1), s2), hmul2<T>(int8_pair<T>(w1, 2, 3), s2));
      }
    } else {
      // 64-byte swizzle: chunk index XOR bits [7,9) of the row offset
      const uint4 raw = lds16(st + (uint32_t)(row * 64 + ((ch ^ ((row >> 1) & 3)) << 4)));
      const float zoff = KIND == EE_W_INT4 ? 8.0f : zcv;
      const uint32_t xor8 = KIND == EE_W_INT4 ? 0x00080008u : 0u;
      const uint32_t nego = Act<T>::neg_offset2(Act<T>::kInt4Base + zoff);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t w = comp(raw, u), w4 = w >> 4;
        uint32_t o[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) o[p] = hmul2<T>(fma2<T>(nib_pair<T>(w, w4, p, xor8), Act<T>::kOne2, nego), s2);
        st_a(ab, row, 4 * ch + u, o[0], o[1], o[2], o[3]);
      }
    }
  }
};

template <typename T, int KIND, int NT>
__global__ void __launch_bounds__(kTcThreads, 1)
    wq_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                 const __grid_constant__ TcArgs a) {
  constexpr bool DQ = KIND != EE_W_DENSE;
  constexpr uint32_t WB = tc_wbytes<KIND>();
  constexpr uint32_t XB = (uint32_t)NT * 256u;  // two boxes [NT rows][64 k]
  constexpr uint32_t TMC = tc_tmem_cols(NT);
  constexpr int ITEMS = KIND == EE_W_INT8 ? 2 : 1;  // dequant items per thread per k-block
  extern __shared__ __align__(1024) char smem_raw[];
  const uint32_t base0 = smem_u32(smem_raw);
  const uint32_t sb = (base0 + 1023u) & ~1023u;
  char* smem = smem_raw + (sb - base0);
  pdl_entry();

  const int S = 1 << a.lsplit;
  if ((int)cl_size() != S) {
    if (threadIdx.x == 0) atomicCAS(a.status, 0, (int)EE_ERR_LAUNCH);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cl_rank();
  const int cid = (int)cl_id();
  const int unit = cid % a.n_units, tt = cid / a.n_units;
  const int n0 = unit * 128, m0 = tt * NT;
  const int kb_first = rank * a.kbc;
  const ee_linear& L = a.w;
  const uint32_t bar_full = sb + a.off_bar;
  const uint32_t bar_empty = bar_full + 8u * a.ns;
  const uint32_t bar_afull = bar_empty + 8u * a.ns;
  const uint32_t bar_aempty = bar_afull + 8u * a.na;
  const uint32_t bar_acc = bar_aempty + 8u * a.na;

  if (warp == kTcProdWarp && lane == 0) {
    tma_prefetch_map(&tw);
    tma_prefetch_map(&tx);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.ns; ++s) {
      mbar_init(bar_full + 8u * s, 1);
      mbar_init(bar_empty + 8u * s, DQ ? kTcDqWarps + 1 : 1);  // dequant warps + the MMA commit
    }
    for (int s = 0; s < a.na; ++s) {
      mbar_init(bar_afull + 8u * s, kTcDqWarps);
      mbar_init(bar_aempty + 8u * s, 1);
    }
    mbar_init(bar_acc, 1);
    mbar_fence_init();
  }
  if (warp == kTcMmaWarp) {
    tmem_alloc(sb + a.off_tm, TMC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + a.off_tm);

  if (warp == kTcProdWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      int s = 0, sph = 0;
      for (int kb = 0; kb < a.kbc; ++kb) {
        if (kb >= a.ns && !mbar_wait(bar_empty + 8u * s, (uint32_t)(sph ^ 1), a.timeout_ns)) {
          ok = false;
          break;
        }
        const uint32_t st = sb + (uint32_t)s * a.stage_bytes, fb = bar_full + 8u * s;
        mbar_arrive_expect_tx(fb, WB + XB);
        const int kabs = kb_first + kb;
        if (KIND == EE_W_DENSE) {
          tma_load_2d(st, &tw, kabs * 256, n0, fb);
          tma_load_2d(st + 16384u, &tw, kabs * 256 + 128, n0, fb);
        } else {
          tma_load_2d(st, &tw, kabs * (KIND == EE_W_INT8 ? 128 : 64), n0, fb);
        }
        tma_load_2d(st + WB, &tx, kabs * 128, m0, fb);
        tma_load_2d(st + WB + XB / 2, &tx, kabs * 128 + 64, m0, fb);
        ++issued;
        if (++s == a.ns) { s = 0; sph ^= 1; }
      }
      if (!ok) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
      for (int kb = issued > a.ns ? issued - a.ns : 0; kb < issued; ++kb)
        if (!mbar_wait(bar_full + 8u * (kb % a.ns), (kb / a.ns) & 1, a.timeout_ns))
          atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == kTcMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc<T>(128, NT);
      bool ok = true;
      int s = 0, sph = 0, as = 0, aph = 0;
      for (int kb = 0; kb < a.kbc; ++kb) {
        if (!mbar_wait(bar_full + 8u * s, (uint32_t)sph, a.timeout_ns)) {
          ok = false;
          break;
        }
        if (DQ && !mbar_wait(bar_afull + 8u * as, (uint32_t)aph, a.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = sb + (uint32_t)s * a.stage_bytes;
        const uint32_t abase = DQ ? sb + a.off_a + (uint32_t)as * 32768u : st;
        const uint32_t bbase = st + WB;
        const uint64_t ad0 = umma_desc_sw128(abase), bd0 = umma_desc_sw128(bbase);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // advance the start-address field (16-byte units) inside the tile
          const uint64_t ad = ad0 + (uint64_t)(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
          const uint64_t bd = bd0 + (uint64_t)(((kk >> 2) * (int)(XB / 2) + (kk & 3) * 32) >> 4);
          umma_f16(tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        umma_commit(bar_empty + 8u * s);
        if (DQ) umma_commit(bar_aempty + 8u * as);
        if (++s == a.ns) { s = 0; sph ^= 1; }
        if (++as == a.na) { as = 0; aph ^= 1; }
      }
      if (!ok) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
      umma_commit(bar_acc);  // fires once every MMA issued above has completed
    }
    __syncwarp();
  } else {
    // ---------------- dequantisers (warps 0-15) ----------------
    if (DQ) {
      const int tid = threadIdx.x;
      int rows[ITEMS], chs[ITEMS];
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const int q = tid + kTcDqThreads * i;
        if (KIND == EE_W_INT8) {
          rows[i] = (q & 7) + 8 * (q >> 6);
          chs[i] = (q >> 3) & 7;
        } else {
          rows[i] = (q & 7) + 8 * (q >> 5);
          chs[i] = (q >> 3) & 3;
        }
      }
      // scales (and zero points) staged two k-blocks ahead with cp.async into
      // a 3-slot ring of this thread's own words: [slot][item][thread]
      const uint32_t scr = sb + a.off_sc + (uint32_t)tid * 4u;
      constexpr uint32_t kSlot = (uint32_t)ITEMS * kTcDqThreads * 4u, kZoff = 3u * kSlot;
      const typename TcDequant<T, KIND>::Groups gp = TcDequant<T, KIND>::groups(L);
      size_t rowsi[ITEMS];  // n * groups-per-row of each item's row
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) rowsi[i] = (size_t)min(n0 + rows[i], L.n - 1) * gp.ng;
#pragma unroll
      for (int d = 0; d < 2; ++d) {
        if (d < a.kbc) {
          const int g = TcDequant<T, KIND>::group_of(gp, kb_first + d);
#pragma unroll
          for (int i = 0; i < ITEMS; ++i)
            TcDequant<T, KIND>::stage_sz(L, rowsi[i] + g, scr + (uint32_t)d * kSlot + (uint32_t)i * (kTcDqThreads * 4u), kZoff);
        }
        cp_async_commit();
      }
      // ring positions advance by counters (no divisions in the loop)
      int s = 0, sph = 0, as = 0, aph = 0, r3 = 0, r3n = 2;
      for (int kb = 0; kb < a.kbc; ++kb) {
        if (kb + 2 < a.kbc) {
          const int g = TcDequant<T, KIND>::group_of(gp, kb_first + kb + 2);
#pragma unroll
          for (int i = 0; i < ITEMS; ++i)
            TcDequant<T, KIND>::stage_sz(L, rowsi[i] + g, scr + (uint32_t)r3n * kSlot + (uint32_t)i * (kTcDqThreads * 4u), kZoff);
        }
        cp_async_commit();
        bool ok = mbar_wait(bar_full + 8u * s, (uint32_t)sph, a.timeout_ns);
        if (ok && kb >= a.na) ok = mbar_wait(bar_aempty + 8u * as, (uint32_t)(aph ^ 1), a.timeout_ns);
        if (!ok) {
          if (lane == 0) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
          break;
        }
        const uint32_t st = sb + (uint32_t)s * a.stage_bytes;
        const uint32_t ab = sb + a.off_a + (uint32_t)as * 32768u;
        cp_async_wait<2>();  // this k-block's scale words have landed
        const int gcur = TcDequant<T, KIND>::group_of(gp, kb_first + kb);
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
          const int row = rows[i], ch = chs[i];
          float scv, zcv;
          TcDequant<T, KIND>::read_sz(L, rowsi[i] + gcur, scr + (uint32_t)r3 * kSlot + (uint32_t)i * (kTcDqThreads * 4u), kZoff,
                                      scv, zcv);
          TcDequant<T, KIND>::item(st, ab, row, ch, scv, zcv);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_afull + 8u * as);
          mbar_arrive(bar_empty + 8u * s);
        }
        if (++s == a.ns) { s = 0; sph ^= 1; }
        if (++as == a.na) { as = 0; aph ^= 1; }
        r3 = r3 == 2 ? 0 : r3 + 1;
        r3n = r3n == 2 ? 0 : r3n + 1;
      }
      cp_async_wait<0>();
    }

    // ---------------- epilogue part 1: TMEM -> registers ----------------
    const int q4 = warp & 3, quarter = warp >> 2;
    const int r = 32 * q4 + lane;  // weight row of the tile
    const int n = n0 + r;
    // columns split over the four warps of each lane quarter, 16 at a time
    constexpr int NCH = NT / 16;                       // 16-column chunks
    constexpr int CPQ = NCH >= 4 ? NCH / 4 : 1;        // chunks per warp
    const int c_beg = quarter * CPQ * 16;
    const int c_end = quarter < NCH ? c_beg + CPQ * 16 : c_beg;
    const int RS = 128 >> a.lsplit;
    // residual values of this thread's outputs, requested before the wait for
    // the accumulators so that they arrive while the last MMAs complete
    T resv[CPQ * 16];
    if (S == 1 && a.epi == EPI_RESID && n < L.n) {
      const T* res = reinterpret_cast<const T*>(a.resid);
#pragma unroll
      for (int i = 0; i < CPQ * 16; ++i) {
        const int tok = m0 + c_beg + i;
        if (c_beg + i < c_end && tok < a.M) resv[i] = res[(size_t)tok * a.ldr + n];
      }
    }
    if (!mbar_wait(bar_acc, 0, a.timeout_ns) && lane == 0) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
    tc_fence_after();
    if (S == 1) {
      const float bias = (a.has_bias && n < L.n) ? ld_param(reinterpret_cast<const T*>(L.bias) + n) : 0.f;
      T* out = reinterpret_cast<T*>(a.out);
#pragma unroll
      for (int cc = 0; cc < CPQ; ++cc) {
        const int c0 = c_beg + 16 * cc;
        if (c0 >= c_end) break;
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)c0, v);
        tmem_wait_ld();
        if (n < L.n) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int tok = m0 + c0 + e;
            if (tok < a.M) {
              float y = Act<T>::round(__uint_as_float(v[e]) + bias);
              if (a.epi == EPI_GELU) {
                y = Act<T>::round(gelu_erf(y));
              } else if (a.epi == EPI_RESID) {
                y = Act<T>::round(Act<T>::to_f(resv[16 * cc + e]) + y);
              }
              out[(size_t)tok * a.ldo + n] = Act<T>::from_f(y);
            }
          }
        }
      }
    } else {
      // push the fp32 partial rows to their owner's receive area
      const uint32_t recv = sb + a.off_recv;
      const int owner = r >> (7 - a.lsplit), lrow = r & (RS - 1);
      for (int c0 = c_beg; c0 < c_end; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)c0, v);
        tmem_wait_ld();
        const uint32_t off = (uint32_t)(((rank * RS + lrow) * a.ps + c0) * 4);
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          st_dsmem_f2(mapa(recv + off + 4u * e, (uint32_t)owner), __uint_as_float(v[e]), __uint_as_float(v[e + 1]));
      }
    }
  }
  tc_fence_before();
  cluster_sync();  // partials delivered; MMAs, copies and TMEM reads finished
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, TMC);
  }
  if (S > 1 && warp < kTcDqWarps) {
    // ---------------- epilogue part 2: owner sums the S partials ----------------
    const int RS = 128 >> a.lsplit;
    const int ntok = min(NT, a.M - m0);
    const int ntok4 = (ntok + 3) & ~3;
    const float* R = reinterpret_cast<const float*>(smem + a.off_recv);
    float* E = reinterpret_cast<float*>(smem);  // [ntok4][RS], reuses the stage ring
    for (int i = threadIdx.x; i < RS * (ntok4 >> 2); i += kTcDqThreads) {
      const int row = i % RS, c4 = i / RS;
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < S; ++q) {
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
    named_sync(1, kTcDqThreads);
    const int nbase = n0 + rank * RS;
    const int cpt = RS / 8;
    const bool vec = (a.ldo % 8) == 0;
    T* out = reinterpret_cast<T*>(a.out);
    const T* res = reinterpret_cast<const T*>(a.resid);
    for (int i = threadIdx.x; i < ntok * cpt; i += kTcDqThreads) {
      const int tok = i / cpt, ch = i - tok * cpt;
      const int nc = nbase + 8 * ch;
      if (nc >= L.n) continue;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int nn = nc + e < L.n ? nc + e : L.n - 1;
        const float bias = a.has_bias ? ld_param(reinterpret_cast<const T*>(L.bias) + nn) : 0.f;
        float y = Act<T>::round(E[tok * RS + 8 * ch + e] + bias);
        if (a.epi == EPI_GELU) {
          y = Act<T>::round(gelu_erf(y));
        } else if (a.epi == EPI_RESID) {
          y = Act<T>::round(ld_param(res + (size_t)(m0 + tok) * a.ldr + nn) + y);
        }
        v[e] = y;
      }
      T* dst = out + (size_t)(m0 + tok) * a.ldo + nc;
      if (vec && nc + 8 <= L.n) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(Act<T>::pack2(v[0], v[1]), Act<T>::pack2(v[2], v[3]),
                                                    Act<T>::pack2(v[4], v[5]), Act<T>::pack2(v[6], v[7]));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (nc + e < L.n) dst[e] = Act<T>::from_f(v[e]);
      }
    }
  }
}

}  // namespace ee

#include "ee_tcp.cuh"

namespace ee {

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
inline uint32_t tc_align(uint32_t v, uint32_t al) { return (v + al - 1) / al * al; }

struct TcShape {
  int nt = 0;   // tokens per tile (16, 32, 64, 128, 256)
  int S = 1;    // split of K over a cluster
  long long tiles = 0;
};

// Tile shape: fewest estimated cycles over the (tokens per tile, split)
// candidates, counting waves of one CTA per SM and a per-k-block cost that is
// the larger of the dequantisation (~600 cycles, int weights) and the MMAs
// (~4.3 cycles per token column).
inline TcShape tc_pick_shape(int M, int N, int K, int kind, int sms) {
  TcShape best;
  double best_cost = 0;
  const long long U = (N + 127) / 128;
  const int nts[5] = {16, 32, 64, 128, 256};
  for (int ni = 0; ni < 5; ++ni) {
    const int nt = nts[ni];
    if (ni > 0 && nts[ni - 1] >= M) break;  // a smaller tile already holds every token
    const long long T = (M + nt - 1) / nt;
    for (int S = 1; S <= 4; S <<= 1) {  // 8-CTA splits measured slower (2048 x 8192, M = 50: 28.3 vs 19.5 us)
      if (S > 1 && nt > 64) break;
      if (K % (kKBlock * S) != 0) break;
      const int kbc = K / (kKBlock * S);
      const long long ctas = U * T * S;
      const long long waves = (ctas + sms - 1) / sms;
      const double per_kb = (kind == EE_W_DENSE ? 150.0 : 600.0) > 4.3 * nt ? (kind == EE_W_DENSE ? 150.0 : 600.0)
                                                                              : 4.3 * nt;
      const double cost = (double)waves * (kbc * per_kb + 2500.0 + (S > 1 ? 1500.0 : 0.0));
      if (best.nt == 0 || cost < best_cost) {
        best_cost = cost;
        best.nt = nt;
        best.S = S;
        best.tiles = U * T;
      }
    }
  }
  return best;
}

template <typename T, int KIND, int NT>
int tc_launch_k(const GemmArgs& g, const TcShape& sh, int* status, cudaStream_t st, bool* used) {
  *used = false;
  const DevProps* dp = device_props();
  if (!dp) return EE_ERR_DEVICE;
  const int N = g.w.n, K = g.w.k, M = g.M;
  const int S = sh.S;
  const int lsplit = S == 8 ? 3 : (S == 4 ? 2 : (S == 2 ? 1 : 0));
  const int kbc = K / (kKBlock * S), RS = 128 / S;
  const bool dq = KIND != EE_W_DENSE;
  const uint32_t stage = tc_align(tc_wbytes<KIND>() + (uint32_t)NT * 256u, 1024u);
  const int ps = NT + 4;
  const uint32_t recv = S > 1 ? (uint32_t)(S * RS * ps * 4) : 0u;
  const int na = dq ? 2 : 0;
  constexpr uint32_t items = KIND == EE_W_INT8 ? 2u : 1u;
  const uint32_t scbytes = dq ? 3u * items * kTcDqThreads * 4u * (KIND == EE_W_UINT4Z ? 2u : 1u) : 0u;
  const uint32_t ebytes = (uint32_t)(((NT + 3) & ~3) * RS * 4);  // owner's summed tile (reuses the ring)
  // shared memory of a launch with ns stages: the layout below, computed the same way
  auto smem_for = [&](int ns_) -> size_t {
    uint32_t ring_end = (uint32_t)ns_ * stage + (uint32_t)na * 32768u;
    if (ring_end < ebytes) ring_end = ebytes;
    const uint32_t off_bar = tc_align(ring_end, 16u);
    const uint32_t off_tm = off_bar + 8u * (2u * (uint32_t)ns_ + 2u * (uint32_t)(dq ? na : 1) + 4u);
    const uint32_t off_recv = tc_align(off_tm + 4u, 16u);
    const uint32_t off_sc = tc_align(off_recv + recv, 16u);
    return (size_t)tc_align(off_sc + scbytes, 16u) + tcp_epi_bytes<KIND>() + 1024;
  };
  // as many stages as fit (at most 8, at most the k-blocks)
  int ns = kbc < 8 ? kbc : 8;
  while (ns > 0 && smem_for(ns) > (size_t)dp->smem_optin) --ns;
  if (ns < 1) return EE_OK;

  TcArgs a{};
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
  a.ns = ns;
  a.na = dq ? na : 1;
  a.ps = ps;
  a.n_units = (N + 127) / 128;
  a.stage_bytes = stage;
  a.off_a = (uint32_t)ns * stage;
  uint32_t ring_end = a.off_a + (uint32_t)na * 32768u;
  // the owner's summed tile reuses the ring
  if (ring_end < ebytes) ring_end = ebytes;
  a.off_bar = tc_align(ring_end, 16u);
  // stage / A-tile barriers, then the accumulator barrier(s): one for
  // wq_tc_kernel, two full + two drained for wq_tcp_kernel
  a.off_tm = a.off_bar + 8u * (2u * ns + 2u * (uint32_t)a.na + 4u);
  a.off_recv = tc_align(a.off_tm + 4u, 16u);
  a.off_sc = tc_align(a.off_recv + recv, 16u);
  a.off_ep = tc_align(a.off_sc + scbytes, 16u);
  const size_t smem = (size_t)a.off_ep + tcp_epi_bytes<KIND>() + 1024;
  if (smem > (size_t)dp->smem_optin) return EE_OK;
  a.status = status;
  a.timeout_ns = 1000000000ull;

  CUtensorMap tw, tx;
  const uint64_t rowbytes = KIND == EE_W_DENSE ? 2ull * K : (KIND == EE_W_INT8 ? (uint64_t)K : (uint64_t)K / 2);
  const bool int4 = KIND == EE_W_INT4 || KIND == EE_W_UINT4Z;
  if (!make_tmap_2d(&tw, g.w.weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rowbytes, (uint64_t)N, rowbytes,
                    int4 ? 64u : 128u, 128u, int4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B))
    return EE_OK;
  if (!make_tmap_2d(&tx, g.x, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)K, (uint64_t)M,
                    (uint64_t)g.ldx * 2u, 64u, (uint32_t)NT, CU_TENSOR_MAP_SWIZZLE_128B))
    return EE_OK;

  if (S == 1 && sh.tiles > (long long)dp->sms) {
    // more tiles than SMs: the persistent form, one CTA per SM looping over
    // tiles with the epilogue of one tile overlapping the next
    auto fnp = wq_tcp_kernel<T, KIND, NT>;
    static std::atomic<int> smem_set_p[64];
    allow_max_smem(fnp, smem_set_p);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)dp->sms);
    cfg.blockDim = dim3(kTcpThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute pattr[1];
    unsigned int npattr = 0;
    add_pdl_attr(pattr, npattr);
    cfg.attrs = pattr;
    cfg.numAttrs = npattr;
    *used = true;
    return cudaLaunchKernelEx(&cfg, fnp, tw, tx, a) == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
  }
  auto fn = wq_tc_kernel<T, KIND, NT>;
  static std::atomic<int> smem_set[64];
  allow_max_smem(fn, smem_set);
  const long long grid = sh.tiles * S;
  if (grid > 0x7fffffffLL) return EE_OK;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kTcThreads);
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
int tc_launch_n(const GemmArgs& g, int* status, cudaStream_t st, bool* used) {
  const DevProps* dp = device_props();
  const TcShape sh = tc_pick_shape(g.M, g.w.n, g.w.k, KIND, dp ? dp->sms : 148);
  switch (sh.nt) {
    case 16: return tc_launch_k<T, KIND, 16>(g, sh, status, st, used);
    case 32: return tc_launch_k<T, KIND, 32>(g, sh, status, st, used);
    case 64: return tc_launch_k<T, KIND, 64>(g, sh, status, st, used);
    case 128: return tc_launch_k<T, KIND, 128>(g, sh, status, st, used);
    case 256: return tc_launch_k<T, KIND, 256>(g, sh, status, st, used);
  }
  *used = false;
  return EE_OK;
}

// Tensor-core path; *used says whether it applied (TMA-compatible operands).
template <typename T>
int launch_tc(const GemmArgs& g, int* status, cudaStream_t st, bool* used) {
  *used = false;
  if (g.M < 1 || !status) return EE_OK;
  if (((uintptr_t)g.x & 15) || ((g.ldx * 2) & 15)) return EE_OK;
  switch (g.w.wkind) {
    case EE_W_DENSE: return tc_launch_n<T, EE_W_DENSE>(g, status, st, used);
    case EE_W_INT8: return tc_launch_n<T, EE_W_INT8>(g, status, st, used);
    case EE_W_INT4: return tc_launch_n<T, EE_W_INT4>(g, status, st, used);
    case EE_W_UINT4Z: return tc_launch_n<T, EE_W_UINT4Z>(g, status, st, used);
  }
  return EE_OK;
}

}  // namespace ee
