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
  // optional normalisation of finished rows (sampler residual phases)
  const void* ln_w;
  const void* ln_b;
  void* ln_out;        // [M, N] normalised rows; NULL = none
  unsigned* ln_cnt;    // one arrival counter per 64-token tile
  int norm_kind;
  float eps;
};

// Shared memory of a GEMM unit. X holds the activation slice [64 tok][KS]
// (16-byte chunks swizzled, see x_chunk); after the MMAs the same bytes hold
// the reduced tile E[64][128/CL] and the row buffers of the norm. P is this
// CTA's partial tile [128 rows][kPS]. PRE holds weight words prefetched
// before a grid barrier.
struct GemmSmem {
  uint32_t x, p, pre;  // byte offsets
};
__host__ __device__ constexpr size_t gemm_x_bytes(int ks) { return (size_t)kMTile * ks * 2; }
constexpr size_t kPBytes = (size_t)kRU * kPS * 4;
constexpr size_t kPreBytes = (size_t)kThreads * 2 * 4 * 16;  // 2 rows x 4 words x 16 B

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

// Normalise `rows` token rows of x (row stride ldx, width d) into out:
// LayerNorm (two-pass fp32 statistics, as torch's CPU kernel) or RMSNorm
// (x * rsqrt(mean(x^2) + eps) rounded, times weight). One warp per row, the
// row staged in `buf` (d floats per warp, shared memory).
template <typename T>
EE_DEV void norm_rows(const T* x, long long ldx, int row0, int rows, int d, const T* w,
                      const T* b, int kind, float eps, T* out, long long ldo, float* buf) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* rb = buf + (size_t)warp * d;
  const float inv_d = 1.0f / (float)d;
  for (int r = warp; r < rows; r += kWarps) {
    const T* xr = x + (size_t)(row0 + r) * ldx;
    float s = 0.f;
    for (int c = lane; c < d / 8; c += 32) {
      const uint4 q = ld_act16(xr + c * 8);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Act<T>::unpack2(comp(q, e));
        rb[c * 8 + 2 * e] = f.x;
        rb[c * 8 + 2 * e + 1] = f.y;
        s += kind == EE_NORM_RMS ? f.x * f.x + f.y * f.y : f.x + f.y;
      }
    }
    __syncwarp();
    s = warp_sum(s);
    float mean = 0.f, rstd;
    if (kind == EE_NORM_RMS) {
      rstd = 1.0f / sqrtf(s * inv_d + eps);
    } else {
      mean = s * inv_d;
      float q = 0.f;
      for (int i = lane; i < d; i += 32) q += (rb[i] - mean) * (rb[i] - mean);
      rstd = 1.0f / sqrtf(warp_sum(q) * inv_d + eps);
    }
    __syncwarp();
    T* orow = out + (size_t)(row0 + r) * ldo;
    for (int c = lane; c < d / 8; c += 32) {
      const uint4 wq = __ldg(reinterpret_cast<const uint4*>(w + c * 8));
      const uint4 bq = b ? __ldg(reinterpret_cast<const uint4*>(b + c * 8)) : make_uint4(0, 0, 0, 0);
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 wf = Act<T>::unpack2(comp(wq, e));
        const float2 bf = Act<T>::unpack2(comp(bq, e));
        const float v0 = rb[c * 8 + 2 * e], v1 = rb[c * 8 + 2 * e + 1];
        float y0, y1;
        if (kind == EE_NORM_RMS) {
          y0 = Act<T>::round(v0 * rstd) * wf.x;
          y1 = Act<T>::round(v1 * rstd) * wf.y;
        } else {
          y0 = (v0 - mean) * rstd * wf.x + bf.x;
          y1 = (v1 - mean) * rstd * wf.y + bf.y;
        }
        o[e] = Act<T>::pack2(y0, y1);
      }
      *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncwarp();
  }
}

// scales / zero points of a prefetched first k-block, kept in registers
struct PreRegs {
  float s[2];
  float z[2];
};

template <typename T, int KIND>
struct Gemm {
  static constexpr int WPR = words_per_row(KIND);

  // k-block kb (absolute, in 128s) of rows n (warp's g) and n+8, clamped to N
  static EE_DEV const char* row_ptr(const ee_linear& L, int n, int kb) {
    const int t = threadIdx.x & 3;
    n = n < L.n ? n : L.n - 1;
    const size_t row_bytes = (size_t)L.k * bytes_per_k2(KIND) / 2;
    return reinterpret_cast<const char*>(L.weight) + (size_t)n * row_bytes +
           (size_t)kb * (kKBlock * bytes_per_k2(KIND) / 2) + t * (32 * bytes_per_k2(KIND) / 2);
  }
  static EE_DEV void load_scales(const ee_linear& L, int n, int kb, float& s, float& z) {
    if (KIND == EE_W_DENSE) return;
    n = n < L.n ? n : L.n - 1;
    const int ng = L.k / L.group;
    const size_t si = (size_t)n * ng + (kb * kKBlock) / L.group;
    s = L.scale_dtype == EE_F32 ? __ldg(reinterpret_cast<const float*>(L.scales) + si)
                                : __half2float(__ldg(reinterpret_cast<const __half*>(L.scales) + si));
    if (KIND == EE_W_UINT4Z) z = __half2float(__ldg(reinterpret_cast<const __half*>(L.zeros) + si));
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
  // cp.async the words of k-block kb into the prefetch area; scales to regs
  static EE_DEV void prefetch(const ee_linear& L, int nw, int kb, uint32_t spre, PreRegs& pr) {
    const int g = (threadIdx.x & 31) >> 2;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const char* p = row_ptr(L, nw + g + 8 * h, kb);
#pragma unroll
      for (int i = 0; i < WPR; ++i)
        cp_async16(spre + ((h * 4 + i) * kThreads + threadIdx.x) * 16, p + 16 * i, true);
      load_scales(L, nw + g + 8 * h, kb, pr.s[h], pr.z[h]);
    }
    cp_async_commit();
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

  // Rows nt*128 .. +127 x tokens m0 .. m0+63 over all of K by this cluster.
  // pre != nullptr: this CTA's first k-block was prefetched into sm.pre.
  static EE_DEV void unit(const GemmArgs& a, int nt, int m0, char* smem, const GemmSmem& sm,
                          const PreRegs* pre) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const ee_linear& L = a.w;
    const int CL = (int)cl_size(), rank = (int)cl_rank();
    const int KS = L.k / CL, KB = KS / kKBlock, kb0 = rank * KB;
    const int mrows = min(kMTile, a.M - m0);
    const int JT = (mrows + 7) >> 3;
    const int nw = nt * kRU + 16 * warp;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sx = sbase + sm.x;

    // 1. this CTA's activation slice -> shared memory (rows >= mrows zeroed)
    {
      const int cpr = KS / 8;  // 16-byte chunks per token row
      const char* xb = reinterpret_cast<const char*>(a.x);
      for (int i = threadIdx.x; i < JT * 8 * cpr; i += kThreads) {
        const int row = i / cpr, c = i - row * cpr;
        const bool ok = row < mrows;
        const char* src = xb + ((size_t)(m0 + (ok ? row : 0)) * a.ldx + (size_t)kb0 * kKBlock + c * 8) * 2;
        const uint32_t dst = sx + (uint32_t)(row * KS * 2 + ((c >> 4) * 16 + x_chunk(row, c & 15)) * 16);
        cp_async16(dst, src, ok);
      }
      cp_async_commit();
    }
    // 2. first k-block of weights
    uint4 w[2][WPR];
    float sc[2] = {1.f, 1.f}, zr[2] = {0.f, 0.f};
    if (pre) {
      cp_async_wait<1>();  // the prefetch group (issued before the X group)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int i = 0; i < WPR; ++i)
          w[h][i] = lds16(sbase + sm.pre + ((h * 4 + i) * kThreads + threadIdx.x) * 16);
        sc[h] = pre->s[h];
        zr[h] = pre->z[h];
      }
    } else {
      load_raw(L, nw, kb0, w, sc, zr);
    }
    cp_async_wait<0>();
    __syncthreads();

    // 3. MMAs over this CTA's k-blocks
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[j][c] = 0.f;
    for (int kb = 0; kb < KB; ++kb) {
      uint32_t A[8][4];
      dequant(w, zr, A);
      const float s0 = sc[0], s1 = sc[1];
      if (kb + 1 < KB) load_raw(L, nw, kb0 + kb + 1, w, sc, zr);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < JT) {
          const int row = 8 * j + g;
          const uint32_t rbase = sx + (uint32_t)(row * KS * 2 + kb * 256);
          uint4 xq[4];
#pragma unroll
          for (int s2 = 0; s2 < 4; ++s2) xq[s2] = lds16(rbase + x_chunk(row, 4 * t + s2) * 16);
          if (KIND == EE_W_DENSE) {
#pragma unroll
            for (int s = 0; s < 8; ++s)
              mma16816<T>(acc[j], A[s][0], A[s][1], A[s][2], A[s][3], comp(xq[s >> 1], 2 * (s & 1)),
                          comp(xq[s >> 1], 2 * (s & 1) + 1));
          } else {
            float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s = 0; s < 8; ++s)
              mma16816<T>(p, A[s][0], A[s][1], A[s][2], A[s][3], comp(xq[s >> 1], 2 * (s & 1)),
                          comp(xq[s >> 1], 2 * (s & 1) + 1));
            acc[j][0] += s0 * p[0];
            acc[j][1] += s0 * p[1];
            acc[j][2] += s1 * p[2];
            acc[j][3] += s1 * p[3];
          }
        }
      }
    }

    // 4. partial tile -> P, then cluster-wide reduction over DSMEM
    float* P = reinterpret_cast<float*>(smem + sm.p);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < JT) {
        const int r0 = 16 * warp + g, c0 = 8 * j + 2 * t;
        *reinterpret_cast<float2*>(P + r0 * kPS + c0) = make_float2(acc[j][0], acc[j][1]);
        *reinterpret_cast<float2*>(P + (r0 + 8) * kPS + c0) = make_float2(acc[j][2], acc[j][3]);
      }
    cluster_sync();
    const int RPR = kRU / CL;  // rows reduced by this rank
    float* E = reinterpret_cast<float*>(smem + sm.x);  // [64][RPR], reuses the X slice
    const uint32_t pbase = sbase + sm.p;
    for (int i = threadIdx.x; i < RPR * 16; i += kThreads) {
      const int row = i >> 4, c4 = i & 15;
      if (4 * c4 < JT * 8) {
        const uint32_t off = (uint32_t)(((rank * RPR + row) * kPS + 4 * c4) * 4);
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < CL; ++r) {
          const float4 v = ld_dsmem_f4(mapa(pbase + off, (uint32_t)r));
          sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
        }
        E[(4 * c4 + 0) * RPR + row] = sum.x;
        E[(4 * c4 + 1) * RPR + row] = sum.y;
        E[(4 * c4 + 2) * RPR + row] = sum.z;
        E[(4 * c4 + 3) * RPR + row] = sum.w;
      }
    }
    cluster_sync();  // peers done with this CTA's P; E complete in this CTA

    // 5. epilogue: bias, round, GELU / residual, store
    T* out = reinterpret_cast<T*>(a.out);
    const T* bias = a.has_bias ? reinterpret_cast<const T*>(L.bias) : nullptr;
    const int nbase = nt * kRU + rank * RPR;
    for (int i = threadIdx.x; i < mrows * RPR; i += kThreads) {
      const int tok = i / RPR, row = i - tok * RPR;
      const int n = nbase + row;
      if (n < L.n) {
        float v = E[tok * RPR + row];
        if (bias) v += ld_param(bias + n);
        v = Act<T>::round(v);
        const size_t m = (size_t)(m0 + tok);
        if (a.epi == EPI_GELU) {
          v = gelu_erf(v);
        } else if (a.epi == EPI_RESID) {
          v = ld_act_scalar(reinterpret_cast<const T*>(a.resid) + m * a.ldr + n) + v;
        }
        out[m * a.ldo + n] = Act<T>::from_f(v);
      }
    }

    // 6. the last CTA to finish a token tile normalises its rows
    if (a.ln_out != nullptr) {
      __shared__ int s_last;
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        const int n_tiles = (L.n + kRU - 1) / kRU;
        const unsigned prev = atomicAdd(a.ln_cnt + m0 / kMTile, 1u);
        s_last = (prev == (unsigned)(n_tiles * CL - 1));
        if (s_last) {
          __threadfence();
          a.ln_cnt[m0 / kMTile] = 0u;
        }
      }
      __syncthreads();
      if (s_last)
        norm_rows<T>(reinterpret_cast<const T*>(a.out), a.ldo, m0, mrows, L.n,
                     reinterpret_cast<const T*>(a.ln_w), reinterpret_cast<const T*>(a.ln_b),
                     a.norm_kind, a.eps, reinterpret_cast<T*>(a.ln_out), a.ldo,
                     reinterpret_cast<float*>(smem + sm.x));
    }
    __syncthreads();  // shared memory reuse by the next unit
  }

  // Issue the prefetch of this CTA's first k-block of unit (cluster id) `u`.
  static EE_DEV void prefetch_unit(const GemmArgs& a, int u, char* smem, const GemmSmem& sm,
                                   PreRegs& pr) {
    const int n_tiles = (a.w.n + kRU - 1) / kRU;
    const int nt = u % n_tiles;
    const int CL = (int)cl_size(), rank = (int)cl_rank();
    const int KB = a.w.k / CL / kKBlock;
    prefetch(a.w, nt * kRU + 16 * (threadIdx.x >> 5), rank * KB, smem_u32(smem) + sm.pre, pr);
  }
};

}  // namespace ee
