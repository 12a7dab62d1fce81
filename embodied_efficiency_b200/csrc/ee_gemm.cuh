// ee_gemm.cuh -- weight-only dequant-GEMM work unit, cluster split-K form.
//
// A unit is 128 weight rows x up to 64 tokens over all of K, computed by one
// thread-block cluster of CL CTAs: CTA rank r owns the K slice
// [r*K/CL, (r+1)*K/CL). Each CTA stages only its slice of the activations in
// shared memory (so a CTA reads M*K/CL activation bytes, not M*K), its 8
// warps each own one 16-row tile, and the CL partial tiles are summed over
// distributed shared memory: rank r reduces rows [r*128/CL, (r+1)*128/CL)
// and applies the epilogue to them.
//
// MMA formulation ("swap AB"): weights are the m16n8k16 A operand (16 weight
// rows), activations the B operand (8 tokens), fp32 accumulation. Inside a
// 128-wide k-block the k order seen by the MMA is permuted: thread
// (g = lane/4, t = lane%4) owns k in [32t, 32t+32) of the block for both
// operands and step s (0..7) consumes its k = 32t+4s .. 32t+4s+3. A dot
// product is invariant under one permutation applied to both operands; with
// this one every thread reads its weights with contiguous 16-byte loads
// straight from the reference layout (row n contiguous in k; int4 two per
// byte, even k in the low nibble) -- no re-layout of the packed weights.
//
// Dequantisation happens in registers: nibble / byte -> exact bf16/f16
// integers (magic-number OR + one packed FMA, or an fp32 magic for int8 with
// bf16), MMA over the k-block, then the fp32 per-(row, group) scale
// multiplies the k-block partial sum.
#pragma once

#include "ee_common.cuh"
#include "ee_tma.cuh"
#include "ee_umma.cuh"

namespace ee {

enum { EPI_STORE = 0, EPI_GELU = 1, EPI_RESID = 2 };

constexpr int kRU = 128;   // weight rows per unit (8 warps x 16)
constexpr int kPS = 72;    // floats per row of the partial tile (64 tokens + pad)

struct GemmArgs {
  const void* x;       // [M, K] activations, row stride ldx elements
  long long ldx;
  ee_linear w;         // weights, scales, zeros, bias, N, K, kind, group
  int M;
  int epi;             // EPI_*
  void* out;           // [M, N] output, row stride ldo
  long long ldo;
  const void* resid;   // [M, N] residual input (EPI_RESID), row stride ldr
  long long ldr;
  int has_bias;
  int split;           // CTAs of a cluster per unit (a power of two dividing the cluster)
  int lsplit;          // log2(split)
  // Row statistics are kept as partial (sum, sum of squares) per
  // (1 << stat_shift)-column slice of the row (16, or 8 when a unit's CTAs
  // reduce only 8 rows): [M][stat_slots][2], summed in slot order
  // (deterministic).
  int stat_slots;
  int stat_shift;
  // input normalisation: when in_stats is set, every staged activation row is
  // normalised with its statistics over K and the weight / bias in_w / in_b
  // (LayerNorm) or in_w only (RMSNorm) before the MMAs
  const float* in_stats;  // [M][stat_slots][2]
  const void* in_w;
  const void* in_b;
  int in_norm;            // EE_NORM_*
  float in_eps;
  // output statistics: when out_stats is set, each CTA writes the (sum, sum
  // of squares) of its output columns of every token row to the slot of its
  // first columns, and zeros to the slots of its other column slices
  float* out_stats;       // [M][stat_slots][2]
  // tcgen05 form: where a wait for MMA completion that runs out of time
  // records EE_ERR_TIMEOUT, and its limit
  int* status;
  unsigned long long timeout_ns;
  // built with EE_TRACE_DETAIL only: globaltimer stamps of this CTA's first
  // unit at its serial steps (entry, staged, normalised, MMAs done, partials
  // pushed, partials received, reduced, stored, statistics), or null
  unsigned long long* dtr;
};

#ifdef EE_TRACE_DETAIL
#define EE_STAMP(a, i)                                                  \
  do {                                                                  \
    if ((a).dtr && threadIdx.x == 0) (a).dtr[i] = globaltimer();        \
  } while (0)
#else
#define EE_STAMP(a, i) \
  do {                 \
  } while (0)
#endif

// Shared memory of a GEMM unit (byte offsets from the dynamic base).
//   x    activation slice [64 tok][KS] (16-byte chunks swizzled, see
//        x_chunk); after the MMAs it holds the reduced tile E[64][128/S + 1]
//   p    two receive buffers (alternating by round) for the partial tiles the
//        sub-cluster's CTAs push here: [S][128/S rows][kPS] fp32 each
//   aux  norm weight/bias slice, row statistics, bias, staged scales and the
//        residual tile of the unit
//   pre  weight words of the first unit, copied in before a grid barrier
//   tc   (tcgen05 form) kTcStages mbarriers (MMA completion of each A
//        stage) at +kTcBar, the TMEM base address at +kTcTmem and the parity
//        of every barrier's commit count (bit s) at +kTcMask, the two
//        mbarriers of the partial-tile receive buffers at +kTcPBar and the
//        parity of their next phases (bit p) at +kTcPPar; the kernel
//        initialises it and allocates TMEM
struct GemmSmem {
  uint32_t x, p, aux, pre;
  uint32_t pre_bytes;  // size of the pre area (0: no prefetch)
  uint32_t tc;
};
// TMEM columns of the tcgen05 form: kTcStages accumulator slots of 64 fp32
// columns (one k-block each, scaled into registers when drained), then
// kTcStages A stages of 64 columns (128 rows x 128 k of 16-bit weights);
// k-block kb uses slot and stage kb % kTcStages
constexpr int kTcStages = 4;
constexpr uint32_t kTcACol = kTcStages * 64;
constexpr uint32_t kTcCols = 512;  // allocation: kTcStages * 128 columns
constexpr uint32_t kTcBar = 0, kTcTmem = 8 * kTcStages, kTcMask = kTcTmem + 4, kTcPBar = kTcMask + 4,
                   kTcPPar = kTcPBar + 16, kTcStateBytes = 64;
constexpr uint32_t kAuxGB = 0;                 // [2][2048] act: norm weight, bias slice
constexpr uint32_t kAuxRow = 8192;             // [64][2] float: mean, rstd
constexpr uint32_t kAuxBias = kAuxRow + 512;   // [128] act: bias slice
constexpr uint32_t kAuxRes = kAuxBias + 512;   // [64][128] act: residual tile
constexpr uint32_t kAuxScale = kAuxRes + 64 * 128 * 2;  // [kMaxKB][2][8 warps][8 g] float
constexpr int kMaxKB = 16;                     // k-blocks per CTA with staged scales
constexpr uint32_t kAuxBytes = kAuxScale + kMaxKB * 2 * 64 * 4;
constexpr int kMaxNormSlice = 2048;            // K/S limit of a normalised input
__host__ __device__ constexpr size_t gemm_x_bytes(int ks) { return (size_t)kMTile * ks * 2; }
constexpr size_t kPBytes = (size_t)kRU * kPS * 4;
__host__ __device__ constexpr size_t pre_kb_bytes(int kind) {  // prefetch bytes per k-block
  return (size_t)kThreads * 2 * (kind == EE_W_DENSE ? 4 : (kind == EE_W_INT8 ? 2 : 1)) * 16;
}

// split policy: CTAs per unit S (a power of two dividing the cluster, K/S a
// multiple of 128 and at most ks_cap) with the fewest rounds over the
// cluster slots; ties go to the larger S (less work per CTA)
__host__ __device__ inline int pick_split(int n, int k, int m, int nclusters, int cl, int ks_cap) {
  const long long units = (long long)((n + kRU - 1) / kRU) * ((m + kMTile - 1) / kMTile);
  int best = 0;
  long long best_rounds = 0;
  for (int sp = cl; sp >= 1; sp >>= 1) {
    if ((k % (sp * kKBlock)) != 0 || k / sp > ks_cap) continue;
    const long long slots = (long long)nclusters * (cl / sp);
    const long long rounds = (units + slots - 1) / slots;
    if (best == 0 || rounds < best_rounds) {
      best = sp;
      best_rounds = rounds;
    }
  }
  return best;
}

__host__ __device__ constexpr int words_per_row(int kind) {
  return kind == EE_W_DENSE ? 4 : (kind == EE_W_INT8 ? 2 : 1);
}
__host__ __device__ constexpr int bytes_per_k2(int kind) {  // bytes per 2 k values
  return kind == EE_W_DENSE ? 4 : (kind == EE_W_INT8 ? 2 : 1);
}

EE_DEV uint32_t comp(const uint4& v, int c) {
  return c == 0 ? v.x : (c == 1 ? v.y : (c == 2 ? v.z : v.w));
}

// physical 16-byte chunk of logical chunk c (0..15 inside a k-block) of token
// row `row`: spreads the 8 threads of a quarter-warp over all bank groups
EE_DEV int x_chunk(int row, int c) { return c ^ (((c >> 3) & 1) << 1) ^ (row & 1); }

// scales / zero points of the prefetched first k-block, kept in registers
struct PreRegs {
  float s[2];
  float z[2];
  int aux;  // the unit's constant operands (norm slice, scales, bias) are staged too
};

template <typename T, int KIND, bool TC = false>
struct Gemm {
  static constexpr int WPR = words_per_row(KIND);
  static constexpr int CPT = 2 * WPR;  // tcgen05 form: 16-byte weight chunks per thread per k-block

  // k-block kb (absolute, in 128s) of row n, this thread's 32 k; n clamped to N
  static EE_DEV const char* row_ptr(const ee_linear& L, int n, int kb) {
    const int t = threadIdx.x & 3;
    n = n < L.n ? n : L.n - 1;
    const size_t row_bytes = (size_t)L.k * bytes_per_k2(KIND) / 2;
    return reinterpret_cast<const char*>(L.weight) + (size_t)n * row_bytes +
           (size_t)kb * (kKBlock * bytes_per_k2(KIND) / 2) + t * (32 * bytes_per_k2(KIND) / 2);
  }
  // tcgen05 form: chunk j of k-block kb for this thread, which dequantises
  // row 32*(warp%4) + lane of the tile, k half warp/4 (64 k of the block)
  static EE_DEV const char* tc_src(const ee_linear& L, int nt, int kb, int j) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int n = nt * kRU + 32 * (warp & 3) + lane;
    n = n < L.n ? n : L.n - 1;
    const size_t row_bytes = (size_t)L.k * bytes_per_k2(KIND) / 2;
    return reinterpret_cast<const char*>(L.weight) + (size_t)n * row_bytes +
           (size_t)kb * (kKBlock * bytes_per_k2(KIND) / 2) + (warp >> 2) * (CPT * 16) + j * 16;
  }
  static EE_DEV float scale_of(const ee_linear& L, int n, int kb) {
    n = n < L.n ? n : L.n - 1;
    const size_t si = (size_t)n * (L.k / L.group) + (kb * kKBlock) / L.group;
    return L.scale_dtype == EE_F32 ? __ldg(reinterpret_cast<const float*>(L.scales) + si)
                                   : __half2float(__ldg(reinterpret_cast<const __half*>(L.scales) + si));
  }
  static EE_DEV float zero_of(const ee_linear& L, int n, int kb) {
    n = n < L.n ? n : L.n - 1;
    return __half2float(__ldg(reinterpret_cast<const __half*>(L.zeros) + (size_t)n * (L.k / L.group) +
                              (kb * kKBlock) / L.group));
  }
  static EE_DEV void load_scales(const ee_linear& L, int n, int kb, float& s, float& z) {
    if (KIND == EE_W_DENSE) return;
    s = scale_of(L, n, kb);
    if (KIND == EE_W_UINT4Z) z = zero_of(L, n, kb);
  }
  static EE_DEV void load_raw(const ee_linear& L, int nw, int kb, uint4 (&w)[2][WPR], float (&s)[2],
                              float (&z)[2]) {
    const int g = (threadIdx.x & 31) >> 2;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const char* p = row_ptr(L, nw + g + 8 * h, kb);
#pragma unroll
      for (int i = 0; i < WPR; ++i) w[h][i] = ld_weight16(p + 16 * i);
      load_scales(L, nw + g + 8 * h, kb, s[h], z[h]);
    }
  }
  static EE_DEV uint32_t pre_addr(uint32_t spre, int kb, int h, int i) {
    return spre + (uint32_t)((((kb * 2 + h) * WPR + i) * kThreads + threadIdx.x) * 16);
  }
  static EE_DEV uint32_t pre_addr_tc(uint32_t spre, int kb, int j) {
    return spre + (uint32_t)(((kb * CPT + j) * kThreads + threadIdx.x) * 16);
  }
  // byte offset of logical 16-byte chunk c (8 k) of token row `row` in the
  // staged activation slice. tcgen05 form: the K-major 128-byte-swizzled
  // operand layout, [KS/64 slabs][64 rows][128 bytes] with the chunk index
  // XORed with row % 8; mma.sync form: rows of KS, chunks spread by x_chunk.
  static EE_DEV uint32_t xoff(int row, int c, int KS) {
    if (TC) return (uint32_t)((c >> 3) * (kMTile * 128) + row * 128 + (((c & 7) ^ (row & 7)) << 4));
    return (uint32_t)(row * KS * 2 + ((c >> 4) * 16 + x_chunk(row, c & 15)) * 16);
  }

  // raw words -> A-operand registers A[s][0..3] for the 8 mma steps
  static EE_DEV void dequant(const uint4 (&w)[2][WPR], const float (&z)[2], uint32_t (&A)[8][4]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t lo[8], hi[8];  // per step: k pair (4s, 4s+1) and (4s+2, 4s+3)
      if (KIND == EE_W_DENSE) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          lo[s] = comp(w[h][s >> 1], 2 * (s & 1));
          hi[s] = comp(w[h][s >> 1], 2 * (s & 1) + 1);
        }
      } else if (KIND == EE_W_INT8) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t wx = comp(w[h][s >> 2], s & 3) ^ 0x80808080u;
          lo[s] = int8_pair<T>(wx, 0, 1);
          hi[s] = int8_pair<T>(wx, 2, 3);
        }
      } else {
        const float zoff = KIND == EE_W_INT4 ? 8.0f : z[h];
        const uint32_t xor8 = KIND == EE_W_INT4 ? 0x00080008u : 0u;
        const uint32_t nego = Act<T>::neg_offset2(Act<T>::kInt4Base + zoff);
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const uint32_t ww = comp(w[h][0], wi);
          const uint32_t w4 = ww >> 4;
#pragma unroll
          for (int p = 0; p < 4; p += 2) {
            const int s = 2 * wi + (p >> 1);
            lo[s] = fma2<T>(nib_pair<T>(ww, w4, p, xor8), Act<T>::kOne2, nego);
            hi[s] = fma2<T>(nib_pair<T>(ww, w4, p + 1, xor8), Act<T>::kOne2, nego);
          }
        }
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        A[s][h] = lo[s];      // a0 (row g) / a1 (row g+8): k pair 4s, 4s+1
        A[s][2 + h] = hi[s];  // a2 / a3: k pair 4s+2, 4s+3
      }
    }
  }

  // tcgen05 form: this thread's 64 k of one weight row -> 32 packed 16-bit
  // pairs in k order (exact integers q, or q - zero, for the quantised kinds)
  static EE_DEV void dequant_tc(const uint4 (&w)[CPT], float z, uint32_t (&o)[32]) {
    if (KIND == EE_W_DENSE) {
#pragma unroll
      for (int j = 0; j < CPT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[4 * j + e] = comp(w[j], e);
    } else if (KIND == EE_W_INT8) {
#pragma unroll
      for (int j = 0; j < CPT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t wx = comp(w[j], e) ^ 0x80808080u;
          o[8 * j + 2 * e] = int8_pair<T>(wx, 0, 1);
          o[8 * j + 2 * e + 1] = int8_pair<T>(wx, 2, 3);
        }
    } else {
      const float zoff = KIND == EE_W_INT4 ? 8.0f : z;
      const uint32_t xor8 = KIND == EE_W_INT4 ? 0x00080008u : 0u;
      const uint32_t nego = Act<T>::neg_offset2(Act<T>::kInt4Base + zoff);
#pragma unroll
      for (int j = 0; j < CPT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t ww = comp(w[j], e), w4 = ww >> 4;
#pragma unroll
          for (int p = 0; p < 4; ++p) o[16 * j + 4 * e + p] = fma2<T>(nib_pair<T>(ww, w4, p, xor8), Act<T>::kOne2, nego);
        }
    }
  }

  // Start copying this CTA's first k-blocks of n-tile `nt` into the pre area
  // (one cp.async group); scales of the first k-block go to pr.
  static EE_DEV void prefetch(const GemmArgs& a, int nt, const GemmSmem& sm, char* smem, PreRegs& pr) {
    const uint32_t sbase = smem_u32(smem);
    const int rank = (int)cl_rank();
    const int KB = (a.w.k >> a.lsplit) / kKBlock, kb0 = (rank & (a.split - 1)) * KB;
    const int fit = (int)(sm.pre_bytes / pre_kb_bytes(KIND));
    const int npre = KB < fit ? KB : fit;
    if (TC) {
      for (int kb = 0; kb < npre; ++kb)
#pragma unroll
        for (int j = 0; j < CPT; ++j) cp_async16(pre_addr_tc(sbase + sm.pre, kb, j), tc_src(a.w, nt, kb0 + kb, j), true);
    } else {
      const int nw = nt * kRU + 16 * (threadIdx.x >> 5), g = (threadIdx.x & 31) >> 2;
      for (int kb = 0; kb < npre; ++kb)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const char* p = row_ptr(a.w, nw + g + 8 * h, kb0 + kb);
#pragma unroll
          for (int i = 0; i < WPR; ++i) cp_async16(pre_addr(sbase + sm.pre, kb, h, i), p + 16 * i, true);
        }
#pragma unroll
      for (int h = 0; h < 2; ++h) load_scales(a.w, nw + g + 8 * h, kb0, pr.s[h], pr.z[h]);
    }
    stage_const(a, nt, sm, smem);
    cp_async_commit();
    pr.aux = 1;
  }

  // The unit's operands that no other CTA produces -- the norm weight / bias
  // slice, the fp32 scales of every k-block, the bias slice -- into the aux
  // area, all with cp.async (committed by the caller): when this runs between
  // a CTA's grid-barrier arrive and wait nothing in it blocks.
  static EE_DEV void stage_const(const GemmArgs& a, int nt, const GemmSmem& sm, char* smem) {
    const uint32_t sbase = smem_u32(smem);
    const ee_linear& L = a.w;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int rank = (int)cl_rank(), r = rank & (a.split - 1);
    const int KS = L.k >> a.lsplit, KB = KS / kKBlock, kb0 = r * KB;
    const int RPR = kRU >> a.lsplit;
    const int nw = nt * kRU + 16 * warp, nbase = nt * kRU + r * RPR;
    if (a.in_stats) {
      const int cpr = KS / 8;
      const uint32_t sg = sbase + sm.aux + kAuxGB;
      for (int i = threadIdx.x; i < 2 * cpr; i += kThreads) {
        const int which = i / cpr, c = i - which * cpr;
        const void* vec = which == 0 ? a.in_w : a.in_b;
        const bool ok = vec != nullptr;
        const char* src = reinterpret_cast<const char*>(ok ? vec : a.in_w) + ((size_t)kb0 * kKBlock + c * 8) * 2;
        cp_async16(sg + (uint32_t)((which * kMaxNormSlice + c * 8) * 2), src, ok);
      }
    }
    const bool smem_scales = KIND != EE_W_DENSE && L.scale_dtype == EE_F32 && KB <= kMaxKB;
    const int ng = L.k / L.group;
    const float* sp = reinterpret_cast<const float*>(L.scales);
    if (TC) {
      // [kb][128 rows]: thread i < 128 stages row i's scales
      if (smem_scales && threadIdx.x < kRU) {
        int n = nt * kRU + threadIdx.x;
        n = n < L.n ? n : L.n - 1;
        for (int kb = 0; kb < KB; ++kb)
          cp_async4(sbase + sm.aux + kAuxScale + (uint32_t)((kb * kRU + threadIdx.x) * 4),
                    sp + (size_t)n * ng + ((kb0 + kb) * kKBlock) / L.group);
      }
    } else if (smem_scales && t == 0) {
      for (int kb = 0; kb < KB; ++kb)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int n = nw + g + 8 * h;
          n = n < L.n ? n : L.n - 1;
          cp_async4(sbase + sm.aux + kAuxScale + (uint32_t)((((kb * 2 + h) * kWarps + warp) * 8 + g) * 4),
                    sp + (size_t)n * ng + ((kb0 + kb) * kKBlock) / L.group);
        }
    }
    // bias slice: RPR/8 chunks of 8 values; copied with cp.async where N is a
    // multiple of 8 and the bias 16-byte aligned (the sampler's layers), else
    // loaded and stored (zeros without a bias or past N)
    const int bt = threadIdx.x - (kThreads - RPR / 8);
    if (bt >= 0) {
      const int n = nbase + 8 * bt;
      const T* bp = reinterpret_cast<const T*>(L.bias);
      T* sb = reinterpret_cast<T*>(smem + sm.aux + kAuxBias) + 8 * bt;
      if (a.has_bias && (L.n % 8) == 0 && (reinterpret_cast<uintptr_t>(bp) & 15) == 0) {
        const bool ok = n + 8 <= L.n;
        cp_async16(sbase + sm.aux + kAuxBias + (uint32_t)(bt * 16), ok ? bp + n : bp, ok);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) sb[e] = Act<T>::from_f((a.has_bias && n + e < L.n) ? ld_param(bp + n + e) : 0.f);
      }
    }
  }

  // tcgen05 form of the MMAs: this CTA's KB k-blocks of the 128-row tile
  // `nt` against the staged activations (NP token rows, a multiple of 16).
  // k-blocks go in groups of up to kTcStages: the 256 threads dequantise the
  // group's weights into A stages 0.. in TMEM (thread: row 32*(warp%4) +
  // lane, k half warp/4), one CTA barrier, then thread 0 issues the group's
  // 128 x NP x 16 MMAs back to back (eight per k-block, into accumulator slot
  // kb % kTcStages) and commits each k-block to its stage's mbarrier. Issuing
  // whole groups keeps the tensor pipe busy: an MMA of N <= 64 costs about
  // the same as one of N = 64, and the pipe's start-up is paid once per
  // group instead of once per k-block. A later group reuses a stage and slot
  // after their MMAs completed and the slot was drained. Slots are drained
  // into registers with the block's fp32 scale (acc += scale * partial, in
  // k-block order), so the arithmetic matches the mma.sync form: exact
  // integer weights, fp32 sums, fp32 scale per k-block. Returns acc[i] = row
  // 32*(warp%4) + lane, token 32*(warp/4) + i.
  static EE_DEV void mma_tc(const GemmArgs& a, int nt, int kb0, int KB, int npre, int NP, uint32_t sx,
                            char* smem, const GemmSmem& sm, float (&acc)[32]) {
    const ee_linear& L = a.w;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, kh = warp >> 2;
    const int row = 32 * (warp & 3) + lane, n = nt * kRU + row;
    const uint32_t sbase = smem_u32(smem), bar = sbase + sm.tc + kTcBar;
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + sm.tc + kTcTmem);
    uint32_t* mask_s = reinterpret_cast<uint32_t*>(smem + sm.tc + kTcMask);
    uint32_t mask = *mask_s;  // bit s: parity of the commits issued so far to stage s's barrier
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t idesc = umma_idesc<T>(128, NP);
    const bool smem_scales = KIND != EE_W_DENSE && L.scale_dtype == EE_F32 && KB <= kMaxKB;
    const float* ssc = reinterpret_cast<const float*>(smem + sm.aux + kAuxScale);
    const bool tok_live = 32 * kh < NP;  // warp-uniform
    bool ok = true;
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;

    auto wait_stage = [&](int s) {  // the last commit to stage s has completed
      if (!mbar_wait(bar + 8 * s, ((mask >> s) & 1u) ^ 1u, a.timeout_ns)) ok = false;
    };
    auto drain = [&](int kbd) {  // slot of k-block kbd -> acc (its MMAs have completed)
      if (!tok_live) return;
      uint32_t v[32];
      tmem_ld32(tmem + lane_off + (uint32_t)(64 * (kbd % kTcStages) + 32 * kh), v);
      tmem_wait_ld();
      const float sc = KIND == EE_W_DENSE ? 1.f : (smem_scales ? ssc[kbd * kRU + row] : scale_of(L, n, kb0 + kbd));
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = fmaf(sc, __uint_as_float(v[i]), acc[i]);
    };
    auto fetch = [&](int kb, uint4 (&w)[CPT]) {
      if (kb < npre) {
#pragma unroll
        for (int j = 0; j < CPT; ++j) w[j] = lds16(pre_addr_tc(sbase + sm.pre, kb, j));
      } else {
#pragma unroll
        for (int j = 0; j < CPT; ++j) w[j] = ld_weight16(tc_src(L, nt, kb0 + kb, j));
      }
    };

    uint4 raw[CPT];
    fetch(0, raw);
    for (int g0 = 0; g0 < KB; g0 += kTcStages) {
      const int gn = KB - g0 < kTcStages ? KB - g0 : kTcStages;
      for (int i = 0; i < gn; ++i) {
        const int kb = g0 + i;
        uint4 cur[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) cur[j] = raw[j];
        if (kb + 1 < KB) fetch(kb + 1, raw);
        const float z = KIND == EE_W_UINT4Z ? zero_of(L, n, kb0 + kb) : 0.f;
        if (g0 > 0) {
          wait_stage(i);  // k-block kb - kTcStages (stage i, slot i) is done
          tc_fence_after();
          drain(kb - kTcStages);
        }
        uint32_t o[32];
        dequant_tc(cur, z, o);
        tmem_st32(tmem + lane_off + kTcACol + (uint32_t)(64 * i + 32 * kh), o);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncthreads();
      if (threadIdx.x == 0) {
        tc_fence_after();
        for (int i = 0; i < gn; ++i) {
          const int kb = g0 + i;
          const uint32_t d = tmem + (uint32_t)(64 * i);
          const uint32_t at = tmem + kTcACol + (uint32_t)(64 * i);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_f16_ts(d, at + 8 * ks,
                        umma_desc_sw128(sx + (uint32_t)((2 * kb + (ks >> 2)) * (kMTile * 128) + (ks & 3) * 32)),
                        idesc, ks > 0 ? 1u : 0u);
          umma_commit(bar + 8 * i);
        }
      }
      for (int i = 0; i < gn; ++i) mask ^= 1u << i;
    }
    // every MMA of the unit has completed once each used stage's last commit has
    for (int s = 0; s < kTcStages && s < KB; ++s) wait_stage(s);
    tc_fence_after();
    for (int kbd = KB > kTcStages ? KB - kTcStages : 0; kbd < KB; ++kbd) drain(kbd);
    if (!ok && threadIdx.x == 0 && a.status) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
    if (threadIdx.x == 0) *mask_s = mask;
  }

  // One unit: rows nt*128 .. +127 x tokens m0 .. m0+63 over all of K, by the S
  // CTAs of sub-cluster rank/S. Every CTA of the cluster calls this the same
  // number of times (inactive CTAs only join the cluster barriers).
  static EE_DEV void unit(const GemmArgs& a, bool active, int nt, int m0, int parity, char* smem,
                          const GemmSmem& sm, const PreRegs* pre) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const ee_linear& L = a.w;
    const int S = a.split, rank = (int)cl_rank();
    const int sub0 = rank & ~(S - 1), r = rank - sub0;
    const int KS = L.k >> a.lsplit, KB = KS / kKBlock, kb0 = r * KB;
    const int RPR = kRU >> a.lsplit;  // rows this CTA reduces and stores
    const int mrows = active ? min(kMTile, a.M - m0) : 0;
    const int JT = (mrows + 7) >> 3;
    // token rows the MMAs read (tcgen05 N: a multiple of 16; rows past mrows are zero)
    const int NP = TC ? ((mrows + 15) & ~15) : JT * 8;
    const int nw = nt * kRU + 16 * warp;
    const int nbase = nt * kRU + r * RPR;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sx = sbase + sm.x;
    char* aux = smem + sm.aux;
    float* rowst = reinterpret_cast<float*>(aux + kAuxRow);
    const T* sbias = reinterpret_cast<const T*>(aux + kAuxBias);
    T* sres = reinterpret_cast<T*>(aux + kAuxRes);

    // tcgen05 form: partials arrive by st.async on this CTA's receive barrier
    // for buffer `parity`; it expects S senders x RPR rows x the 4-token
    // groups that hold real tokens (what the senders push)
    const uint32_t pbar = sbase + sm.tc + kTcPBar + 8u * (uint32_t)parity;
    const uint32_t ppar = TC ? ((*reinterpret_cast<volatile uint32_t*>(smem + sm.tc + kTcPPar) >> parity) & 1u) : 0u;
    if (TC && active && threadIdx.x == 0) {
      const int q0 = (min(32, mrows) + 3) >> 2, q1 = mrows > 32 ? (mrows - 32 + 3) >> 2 : 0;
      mbar_arrive_expect_tx(pbar, (uint32_t)(S * RPR * (q0 + q1) * 16));
    }
    // weights: prefetched before the grid barrier, or requested now
    PreRegs pr_local;
    const PreRegs* prw = pre;
    if (active && !pre && sm.pre_bytes >= pre_kb_bytes(KIND)) {
      prefetch(a, nt, sm, smem, pr_local);
      prw = &pr_local;
    }
    const int fit = (int)(sm.pre_bytes / pre_kb_bytes(KIND));
    const int npre = prw ? (KB < fit ? KB : fit) : 0;

    EE_STAMP(a, 0);
    if (active) {
      // 1. activation slice, norm weight / bias slice, residual tile -> smem
      const int cpr = KS / 8;  // 16-byte chunks per token row
      const char* xb = reinterpret_cast<const char*>(a.x);
      if (kThreads % cpr == 0) {
        // each thread keeps one chunk column and steps over rows: no per-chunk division
        const int c = threadIdx.x % cpr, rstep = kThreads / cpr;
        const char* src = xb + ((size_t)m0 * a.ldx + (size_t)kb0 * kKBlock + c * 8) * 2;
        const size_t sstep = (size_t)a.ldx * 2;
        for (int row = threadIdx.x / cpr; row < NP; row += rstep) {
          const bool ok = row < mrows;
          cp_async16(sx + xoff(row, c, KS), ok ? src + (size_t)row * sstep : src, ok);
        }
      } else {
        for (int i = threadIdx.x; i < NP * cpr; i += kThreads) {
          const int row = i / cpr, c = i - row * cpr;
          const bool ok = row < mrows;
          const char* src = xb + ((size_t)(m0 + (ok ? row : 0)) * a.ldx + (size_t)kb0 * kKBlock + c * 8) * 2;
          cp_async16(sx + xoff(row, c, KS), src, ok);
        }
      }
      if (!(prw && prw->aux)) stage_const(a, nt, sm, smem);  // else staged before the barrier
      if (a.epi == EPI_RESID) {
        const int rcpr = RPR / 8;  // 16-byte chunks of a residual row segment
        const char* rb = reinterpret_cast<const char*>(a.resid);
        for (int i = threadIdx.x; i < mrows * rcpr; i += kThreads) {
          const int row = i / rcpr, c = i - row * rcpr;
          const bool ok = nbase + c * 8 + 8 <= L.n;
          const char* src = rb + ((size_t)(m0 + row) * a.ldr + (ok ? nbase + c * 8 : 0)) * 2;
          cp_async16(sbase + sm.aux + kAuxRes + (uint32_t)((row * RPR + c * 8) * 2), src, ok);
        }
      }
      cp_async_commit();
      if (a.in_stats) {
        // 4 threads per token row, each summing every 4th slot in order; the
        // four partials are combined in a fixed tree order (deterministic)
        const int tok = threadIdx.x >> 2, part = threadIdx.x & 3;
        float sx = 0.f, sxx = 0.f;
        if (tok < mrows) {
          const float* sp = a.in_stats + 2 * (size_t)(m0 + tok) * a.stat_slots;
          float2 v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int q = part + 4 * i;
            v[i] = q < a.stat_slots ? ld_act_f2(sp + 2 * q) : make_float2(0.f, 0.f);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            sx += v[i].x;
            sxx += v[i].y;
          }
          // more than 128 slots (d_model 2048 with 8-column slots): the rest, in order
          for (int q = part + 128; q < a.stat_slots; q += 4) {
            const float2 w = ld_act_f2(sp + 2 * q);
            sx += w.x;
            sxx += w.y;
          }
        }
        sx += __shfl_xor_sync(0xffffffffu, sx, 1);
        sxx += __shfl_xor_sync(0xffffffffu, sxx, 1);
        sx += __shfl_xor_sync(0xffffffffu, sx, 2);
        sxx += __shfl_xor_sync(0xffffffffu, sxx, 2);
        if (part == 0 && tok < mrows) {
          const float inv_k = 1.0f / (float)L.k;
          float mean = 0.f, rstd;
          if (a.in_norm == EE_NORM_RMS) {
            rstd = 1.0f / sqrtf(sxx * inv_k + a.in_eps);
          } else {
            mean = sx * inv_k;
            const float var = fmaxf(sxx * inv_k - mean * mean, 0.f);
            rstd = 1.0f / sqrtf(var + a.in_eps);
          }
          rowst[2 * tok] = mean;
          rowst[2 * tok + 1] = rstd;
        }
      }
    }
    // 2. weights of the first k-block (mma.sync form: from the pre area, or loaded now)
    uint4 w[2][WPR];
    float sc[2] = {1.f, 1.f}, zr[2] = {0.f, 0.f};
    if (active) {
      cp_async_wait<0>();
      if (!TC) {
        if (prw) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int i = 0; i < WPR; ++i) w[h][i] = lds16(pre_addr(sbase + sm.pre, 0, h, i));
            sc[h] = prw->s[h];
            zr[h] = prw->z[h];
          }
        } else {
          load_raw(L, nw, kb0, w, sc, zr);
        }
      }
    }
    __syncthreads();
    EE_STAMP(a, 1);

    float acc[8][4];  // mma.sync form: token tile j, fragment c
    float acct[32];   // tcgen05 form: row 32*(warp%4)+lane, tokens 32*(warp/4)+i
    if (active) {
      // 3. normalise the staged activations in place
      if (a.in_stats) {
        const int cpr = KS / 8;
        const T* sgw = reinterpret_cast<const T*>(aux + kAuxGB);
        const T* sgb = sgw + kMaxNormSlice;
        const bool rms = a.in_norm == EE_NORM_RMS;
        auto norm_chunk = [&](int row, int c, const float2 (&wf)[4], const float2 (&bf)[4]) {
          uint4* q = reinterpret_cast<uint4*>(smem + sm.x + xoff(row, c, KS));
          const uint4 v = *q;
          const float mean = rowst[2 * row], rstd = rowst[2 * row + 1];
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 xv = Act<T>::unpack2(comp(v, e));
            if (rms) {
              o[e] = Act<T>::pack2(Act<T>::round(xv.x * rstd) * wf[e].x, Act<T>::round(xv.y * rstd) * wf[e].y);
            } else {
              o[e] = Act<T>::pack2((xv.x - mean) * rstd * wf[e].x + bf[e].x, (xv.y - mean) * rstd * wf[e].y + bf[e].y);
            }
          }
          *q = make_uint4(o[0], o[1], o[2], o[3]);
        };
        auto load_wb = [&](int c, float2 (&wf)[4], float2 (&bf)[4]) {
          const uint4 wv = *reinterpret_cast<const uint4*>(sgw + c * 8);
          const uint4 bv = *reinterpret_cast<const uint4*>(sgb + c * 8);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            wf[e] = Act<T>::unpack2(comp(wv, e));
            bf[e] = Act<T>::unpack2(comp(bv, e));
          }
        };
        if (kThreads % cpr == 0) {
          // one chunk column per thread: its norm weight / bias loaded once
          const int c = threadIdx.x % cpr, rstep = kThreads / cpr;
          float2 wf[4], bf[4];
          load_wb(c, wf, bf);
#pragma unroll 4
          for (int row = threadIdx.x / cpr; row < mrows; row += rstep) norm_chunk(row, c, wf, bf);
        } else {
          for (int i = threadIdx.x; i < mrows * cpr; i += kThreads) {
            const int row = i / cpr, c = i - row * cpr;
            float2 wf[4], bf[4];
            load_wb(c, wf, bf);
            norm_chunk(row, c, wf, bf);
          }
        }
        if (!TC) __syncthreads();  // the tcgen05 form syncs before its first MMA
      }
      EE_STAMP(a, 2);

      if (TC) {
        // 4. tcgen05 MMAs (activations written by this thread -> async proxy first)
        fence_proxy_async_smem();
        mma_tc(a, nt, kb0, KB, npre, NP, sx, smem, sm, acct);
        EE_STAMP(a, 3);
      } else {
        // 4. mma.sync MMAs over this CTA's k-blocks (first pre_kb from the pre area)
        const bool smem_scales = KIND != EE_W_DENSE && L.scale_dtype == EE_F32 && KB <= kMaxKB;
        const float* ssc = reinterpret_cast<const float*>(aux + kAuxScale);  // [kb][h][warp][g]
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[j][c] = 0.f;
        for (int kb = 0; kb < KB; ++kb) {
          uint32_t A[8][4];
          dequant(w, zr, A);
          const float s0 = sc[0], s1 = sc[1];
          if (kb + 1 < KB) {
            if (kb + 1 < npre) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
#pragma unroll
                for (int i = 0; i < WPR; ++i) w[h][i] = lds16(pre_addr(sbase + sm.pre, kb + 1, h, i));
                if (smem_scales) {
                  sc[h] = ssc[(((kb + 1) * 2 + h) * kWarps + warp) * 8 + g];
                  if (KIND == EE_W_UINT4Z) zr[h] = zero_of(L, nw + g + 8 * h, kb0 + kb + 1);
                } else {
                  load_scales(L, nw + g + 8 * h, kb0 + kb + 1, sc[h], zr[h]);
                }
              }
            } else {
              load_raw(L, nw, kb0 + kb + 1, w, sc, zr);
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j < JT) {
              const int row = 8 * j + g;
              uint4 xq[4];
#pragma unroll
              for (int s2 = 0; s2 < 4; ++s2) xq[s2] = lds16(sx + xoff(row, kb * 16 + 4 * t + s2, KS));
              // four independent accumulation chains of two MMAs each (chain c
              // takes steps 2c and 2c+1, i.e. the k of xq[c]), so an MMA's
              // latency is exposed twice per token tile, not eight times
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
                  mma16816<T>(pc[cc], A[s][0], A[s][1], A[s][2], A[s][3], comp(xq[cc], 2 * hs), comp(xq[cc], 2 * hs + 1));
                }
              const float f0 = KIND == EE_W_DENSE ? 1.f : s0, f1 = KIND == EE_W_DENSE ? 1.f : s1;
              acc[j][0] += f0 * ((pc[0][0] + pc[1][0]) + (pc[2][0] + pc[3][0]));
              acc[j][1] += f0 * ((pc[0][1] + pc[1][1]) + (pc[2][1] + pc[3][1]));
              acc[j][2] += f1 * ((pc[0][2] + pc[1][2]) + (pc[2][2] + pc[3][2]));
              acc[j][3] += f1 * ((pc[0][3] + pc[1][3]) + (pc[2][3] + pc[3][3]));
            }
          }
        }
      }

      // 5. push the partial tile: rows of rank q go to rank q's receive buffer
      const uint32_t rbuf = sbase + sm.p + (uint32_t)(parity * kPBytes);
      const int rshift = 7 - a.lsplit;  // log2(RPR)
      if (TC) {
        const int row = 32 * (warp & 3) + lane, t0 = 32 * (warp >> 2);
        const int owner = row >> rshift, lrow = row & (RPR - 1);
        const uint32_t dst = mapa(rbuf + (uint32_t)(((r * RPR + lrow) * kPS + t0) * 4), (uint32_t)(sub0 + owner));
        const uint32_t dbar = mapa(pbar, (uint32_t)(sub0 + owner));
        const int nq = t0 < mrows ? (min(32, mrows - t0) + 3) >> 2 : 0;  // 4-token groups to send
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < nq) st_async_f4(dst + 16 * q, acct[4 * q], acct[4 * q + 1], acct[4 * q + 2], acct[4 * q + 3], dbar);
        EE_STAMP(a, 4);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < JT) {
            const int c0 = 8 * j + 2 * t;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int row = 16 * warp + g + 8 * h;
              const int owner = row >> rshift, lrow = row & (RPR - 1);
              const uint32_t off = (uint32_t)(((r * RPR + lrow) * kPS + c0) * 4);
              st_dsmem_f2(mapa(rbuf + off, (uint32_t)(sub0 + owner)), acc[j][2 * h], acc[j][2 * h + 1]);
            }
          }
      }
    }
    if (TC) {
      // every partial of this round has arrived once the receive barrier's
      // byte count has; the barrier chain also orders buffer reuse two
      // rounds later (a sender pushes round rd+2 only after this CTA pushed
      // round rd+1, i.e. after it summed round rd)
      if (active) {
        if (!mbar_wait(pbar, ppar, a.timeout_ns) && a.status) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
        if (threadIdx.x == 0)
          *reinterpret_cast<volatile uint32_t*>(smem + sm.tc + kTcPPar) ^= 1u << parity;
        EE_STAMP(a, 5);
      }
    } else {
      cluster_sync();  // every partial of this round has arrived
    }

    // 6. sum the S partials of this CTA's RPR rows (local, source order)
    const int ES = RPR + 1;  // row stride of E (odd: the transposing writes below are conflict-free)
    float* E = reinterpret_cast<float*>(smem + sm.x);  // [64][ES], reuses the X slice
    if (active) {
      const float* R = reinterpret_cast<const float*>(smem + sm.p + parity * kPBytes);
      const int nc4 = (mrows + 3) >> 2;  // 4-token groups holding real tokens
      for (int i = threadIdx.x; i < RPR * 16; i += kThreads) {
        const int row = i >> 4, c4 = i & 15;
        if (c4 < nc4) {
          float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int q = 0; q < S; ++q) {
            const float4 v = *reinterpret_cast<const float4*>(R + (q * RPR + row) * kPS + 4 * c4);
            sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
          }
          E[(4 * c4 + 0) * ES + row] = sum.x;
          E[(4 * c4 + 1) * ES + row] = sum.y;
          E[(4 * c4 + 2) * ES + row] = sum.z;
          E[(4 * c4 + 3) * ES + row] = sum.w;
        }
      }
      __syncthreads();
      EE_STAMP(a, 6);

      // 7. epilogue on 8-column chunks: bias, round, GELU / residual, one
      //    16-byte store per chunk (scalar stores for a ragged end)
      T* out = reinterpret_cast<T*>(a.out);
      const int cpt = RPR / 8;  // chunks per token row
      const bool vec = (a.ldo % 8) == 0;
      for (int i = threadIdx.x; i < mrows * cpt; i += kThreads) {
        const int tok = i / cpt, ch = i - tok * cpt;
        const int n0 = nbase + 8 * ch;
        float v[8];
        uint4 rq = make_uint4(0, 0, 0, 0);
        if (a.epi == EPI_RESID) rq = *reinterpret_cast<const uint4*>(sres + tok * RPR + 8 * ch);
        const uint4 bq = *reinterpret_cast<const uint4*>(sbias + 8 * ch);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float2 bf = Act<T>::unpack2(comp(bq, e >> 1));
          float y = Act<T>::round(E[tok * ES + 8 * ch + e] + ((e & 1) ? bf.y : bf.x));
          if (a.epi == EPI_GELU) {
            y = Act<T>::round(gelu_erf(y));
          } else if (a.epi == EPI_RESID) {
            const float2 rf = Act<T>::unpack2(comp(rq, e >> 1));
            y = Act<T>::round(((e & 1) ? rf.y : rf.x) + y);
          }
          v[e] = n0 + e < L.n ? y : 0.f;
          if (a.out_stats) E[tok * ES + 8 * ch + e] = v[e];  // final values for the row statistics
        }
        T* dst = out + (size_t)(m0 + tok) * a.ldo + n0;
        if (vec && n0 + 8 <= L.n) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(Act<T>::pack2(v[0], v[1]), Act<T>::pack2(v[2], v[3]),
                                                      Act<T>::pack2(v[4], v[5]), Act<T>::pack2(v[6], v[7]));
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (n0 + e < L.n) dst[e] = Act<T>::from_f(v[e]);
        }
      }
      EE_STAMP(a, 7);
      // 8. row statistics of this CTA's columns (column order), one slot each
      if (a.out_stats) {
        __syncthreads();
        if (threadIdx.x < mrows) {
          float sx = 0.f, sxx = 0.f;
          for (int col = 0; col < RPR; ++col) {
            const float y = E[threadIdx.x * ES + col];
            sx += y;
            sxx += y * y;
          }
          float* st = a.out_stats + 2 * ((size_t)(m0 + threadIdx.x) * a.stat_slots + (nbase >> a.stat_shift));
          st[0] = sx;
          st[1] = sxx;
          for (int q = 1; q < (RPR >> a.stat_shift); ++q) {
            st[2 * q] = 0.f;
            st[2 * q + 1] = 0.f;
          }
        }
      }
    }
    __syncthreads();  // shared memory reuse by the next unit
    EE_STAMP(a, 8);
  }

  // All units of a GEMM in rounds over the cluster slots; `pre` applies to
  // this CTA's first unit.
  static EE_DEV void run(const GemmArgs& a, char* smem, const GemmSmem& sm, const PreRegs* pre) {
    if ((int)cl_size() < a.split) return;  // launched without the planned cluster: no work
    const int n_tiles = (a.w.n + kRU - 1) / kRU;
    const int units = n_tiles * ((a.M + kMTile - 1) / kMTile);
    const int per_cluster = (int)cl_size() >> a.lsplit;
    const int slots = (int)cl_count() * per_cluster;
    const int slot = (int)cl_id() * per_cluster + ((int)cl_rank() >> a.lsplit);
    const int rounds = (units + slots - 1) / slots;
    GemmArgs ar = a;
    EE_STAMP(a, 12);
    for (int rd = 0; rd < rounds; ++rd) {
      const int u = rd * slots + slot;
      const bool act = u < units;
      unit(ar, act, act ? u % n_tiles : 0, act ? (u / n_tiles) * kMTile : 0, rd & 1, smem, sm,
           (rd == 0 && act) ? pre : nullptr);
      ar.dtr = nullptr;  // stamps describe the first round only
    }
  }
  // Start the prefetch of this CTA's first unit; returns whether it has one.
  static EE_DEV bool start_prefetch(const GemmArgs& a, const GemmSmem& sm, char* smem, PreRegs& pr) {
    if ((int)cl_size() < a.split) return false;
    const int n_tiles = (a.w.n + kRU - 1) / kRU;
    const int units = n_tiles * ((a.M + kMTile - 1) / kMTile);
    const int per_cluster = (int)cl_size() >> a.lsplit;
    const int slot = (int)cl_id() * per_cluster + ((int)cl_rank() >> a.lsplit);
    if (slot >= units || sm.pre_bytes < pre_kb_bytes(KIND)) return false;
    prefetch(a, slot % n_tiles, sm, smem, pr);
    return true;
  }
};

}  // namespace ee
