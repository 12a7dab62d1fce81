// ee_attn.cuh -- one (batch, head) attention unit for the sampler:
// softmax(Q K^T / sqrt(hd)) V with up to 64 queries (the action chunk) and
// any number of keys (the 50 action tokens for self-attention, the cached
// prefix for cross-attention). Non-causal, as F.scaled_dot_product_attention
// is called in kernel/flow_expert.py:86,91.
//
// 8 warps = 4 query tiles of 16 rows x 2 key groups. Key blocks of 64 are
// staged through shared memory (double buffered, 16-byte chunks XOR-swizzled
// by row -- the 128-byte swizzle -- so ldmatrix is conflict free): with
// cp.async, or, for keys / values no thread of the kernel writes (the cached
// prefix of cross-attention, head size 64) and a tensor map of them, with
// two TMA box loads per key block issued by one thread. Key group kg takes
// blocks kg, kg+2, ... with an online softmax in fp32, and the two groups'
// partial (max, sum, O) are merged through shared memory.
#pragma once

#include "ee_common.cuh"
#include "ee_tma.cuh"

namespace ee {

struct AttnArgs {
  const void* q;  long long ldq;   // rows = tokens; q of head h at column h*hd
  const void* k;  long long ldk;   // rows = keys
  const void* v;  long long ldv;
  void* out;      long long ldo;   // merged-head output, column h*hd
  int n_q;        // queries per batch element (<= 64)
  int n_k;        // keys per batch element
  int q_rows_per_b, k_rows_per_b;  // row offsets between batch elements
  int n_heads;
  float scale_log2;                // log2(e) / sqrt(hd)
  // optional: tensor map of k / v ([rows][2 * n_heads * hd], 64 x 64 boxes,
  // 128-byte swizzle; v at column n_heads * hd), for data not written while
  // the kernel runs; waits give up after timeout_ns with EE_ERR_TIMEOUT in status
  const CUtensorMap* kv_map;
  int* status;
  unsigned long long timeout_ns;
};

template <int HD>
struct AttnSmem {
  static constexpr int kRowBytes = HD * 2;
  static constexpr int kTile = 64 * kRowBytes;          // one 64-row tile
  static constexpr int kQ = 0;
  static constexpr int kKV = kQ + kTile;                // [stage][blk][K|V]
  static constexpr int kMerge = kKV + 2 * 2 * 2 * kTile;
  static constexpr int kMergeBytes = 4 * 16 * (HD + 2) * 4;
  static constexpr int kBar = kMerge + kMergeBytes;     // two mbarriers (TMA loads of each stage)
  static constexpr int kTotal = kBar + 16;
};

EE_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
EE_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

template <typename T, int HD>
struct Attn {
  using S = AttnSmem<HD>;
  static constexpr int kCh = HD / 8;  // 16-byte chunks per row

  static EE_DEV int off(int row, int ch) { return row * S::kRowBytes + ((ch ^ (row & 7)) << 4); }

  // 64 rows starting at global row r0 (rows >= nvalid are zero-filled)
  static EE_DEV void load_tile(uint32_t sdst, const void* base, long long ld, long long col,
                               long long r0, int nvalid) {
    const char* b = reinterpret_cast<const char*>(base);
    for (int i = threadIdx.x; i < 64 * kCh; i += kThreads) {
      const int row = i / kCh, ch = i - row * kCh;
      const bool ok = row < nvalid;
      const long long gr = r0 + (ok ? row : 0);
      cp_async16(sdst + off(row, ch), b + (gr * ld + col + ch * 8) * 2, ok);
    }
  }

  // Running state of one warp over a unit: its 16 query rows of the output
  // (fp32, unnormalised), the running max / sum of the two rows a lane holds,
  // and the Q fragments.
  struct State {
    float o[HD / 8][4];
    float mrow[2], lrow[2];
    uint32_t qf[HD / 16][4];
  };

  static EE_DEV void reset(State& sw) {
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) sw.o[i][c] = 0.f;
    sw.mrow[0] = sw.mrow[1] = -INFINITY;
    sw.lrow[0] = sw.lrow[1] = 0.f;
  }

  // Q fragments of query tile qt (rows 16 qt ..) from the swizzled Q tile
  static EE_DEV void load_q(State& sw, uint32_t sQ, int qt, int lane) {
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int mi = lane >> 3;
      const int row = qt * 16 + (mi & 1) * 8 + (lane & 7);
      ldsm_x4(sQ + off(row, 2 * ks + (mi >> 1)), sw.qf[ks][0], sw.qf[ks][1], sw.qf[ks][2], sw.qf[ks][3]);
    }
  }

  // one block of 64 keys (keys 64 kb ..; those past n_k are masked) from the
  // swizzled K / V tiles at kt / vt: S = Q K^T, online softmax, O += P V
  static EE_DEV void block(State& sw, const AttnArgs& a, uint32_t kt, uint32_t vt, int kb, int lane) {
    const int t = lane & 3;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[j][c] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int mi = lane >> 3;
        const int key = 16 * np + (mi >> 1) * 8 + (lane & 7);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(kt + off(key, 2 * ks + (mi & 1)), r0, r1, r2, r3);
        mma16816<T>(s[2 * np], sw.qf[ks][0], sw.qf[ks][1], sw.qf[ks][2], sw.qf[ks][3], r0, r1);
        mma16816<T>(s[2 * np + 1], sw.qf[ks][0], sw.qf[ks][1], sw.qf[ks][2], sw.qf[ks][3], r2, r3);
      }
    }
    // scale to log2 domain, mask keys past n_k, online softmax
    const int kbase = kb * 64;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int key = kbase + 8 * j + 2 * t + (c & 1);
        const float vv = key < a.n_k ? s[j][c] * a.scale_log2 : -INFINITY;
        s[j][c] = vv;
        mx[c >> 1] = fmaxf(mx[c >> 1], vv);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float mnew[2], corr[2], ls[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(sw.mrow[r], mx[r]);
      corr[r] = exp2f(sw.mrow[r] - mnew[r]);
      sw.mrow[r] = mnew[r];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float p = exp2f(s[j][c] - mnew[c >> 1]);
        s[j][c] = p;
        ls[c >> 1] += p;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
      ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
      sw.lrow[r] = sw.lrow[r] * corr[r] + ls[r];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      sw.o[i][0] *= corr[0];
      sw.o[i][1] *= corr[0];
      sw.o[i][2] *= corr[1];
      sw.o[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa0 = Act<T>::pack2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t pa1 = Act<T>::pack2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t pa2 = Act<T>::pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t pa3 = Act<T>::pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int nn = 0; nn < HD / 16; ++nn) {
        const int mi = lane >> 3;
        const int key = 16 * kk + (mi & 1) * 8 + (lane & 7);
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vt + off(key, 2 * nn + (mi >> 1)), r0, r1, r2, r3);
        mma16816<T>(sw.o[2 * nn], pa0, pa1, pa2, pa3, r0, r1);
        mma16816<T>(sw.o[2 * nn + 1], pa0, pa1, pa2, pa3, r2, r3);
      }
    }
  }

  // Merge the two key groups (warps 4-7 publish (max, sum, O) through the
  // merge area, warps 0-3 combine) and store the unit's rows: queries at
  // rows qr0 .., columns col .. of the output. Contains one __syncthreads;
  // the merge area is free again after the caller's next one.
  static EE_DEV void finish(const State& sw, const AttnArgs& a, char* merge, long long qr0, long long col, int warp,
                            int lane) {
    const int qt = warp & 3, kg = warp >> 2, g = lane >> 2, t = lane & 3;
    float* mg = reinterpret_cast<float*>(merge) + (size_t)qt * 16 * (HD + 2);
    if (kg == 1) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = g + 8 * r;
        if (t == 0) {
          mg[row * (HD + 2) + HD] = sw.mrow[r];
          mg[row * (HD + 2) + HD + 1] = sw.lrow[r];
        }
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          mg[row * (HD + 2) + 8 * i + 2 * t] = sw.o[i][2 * r];
          mg[row * (HD + 2) + 8 * i + 2 * t + 1] = sw.o[i][2 * r + 1];
        }
      }
    }
    __syncthreads();
    if (kg == 0) {
      T* out = reinterpret_cast<T*>(a.out);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = g + 8 * r;
        const float m1 = mg[row * (HD + 2) + HD], l1 = mg[row * (HD + 2) + HD + 1];
        const float m = fmaxf(sw.mrow[r], m1);
        const float c0 = exp2f(sw.mrow[r] - m), c1 = exp2f(m1 - m);
        const float inv = 1.0f / (sw.lrow[r] * c0 + l1 * c1);
        const int qi = qt * 16 + row;
        if (qi < a.n_q) {
          T* orow = out + (qr0 + qi) * a.ldo + col;
#pragma unroll
          for (int i = 0; i < HD / 8; ++i) {
            const float y0 = (sw.o[i][2 * r] * c0 + mg[row * (HD + 2) + 8 * i + 2 * t] * c1) * inv;
            const float y1 = (sw.o[i][2 * r + 1] * c0 + mg[row * (HD + 2) + 8 * i + 2 * t + 1] * c1) * inv;
            *reinterpret_cast<uint32_t*>(orow + 8 * i + 2 * t) = Act<T>::pack2(y0, y1);
          }
        }
      }
    }
  }

  // Store a unit computed by one key group alone (every key block in this
  // warp's state): rows qr0 .., columns col .. of the output.
  static EE_DEV void store_solo(const State& sw, const AttnArgs& a, long long qr0, long long col, int qt, int lane) {
    const int g = lane >> 2, t = lane & 3;
    T* out = reinterpret_cast<T*>(a.out);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int qi = qt * 16 + g + 8 * r;
      const float inv = 1.0f / sw.lrow[r];
      if (qi < a.n_q) {
        T* orow = out + (qr0 + qi) * a.ldo + col;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i)
          *reinterpret_cast<uint32_t*>(orow + 8 * i + 2 * t) =
              Act<T>::pack2(sw.o[i][2 * r] * inv, sw.o[i][2 * r + 1] * inv);
      }
    }
  }

  static EE_DEV void unit(const AttnArgs& a, int b, int h, char* smem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = warp & 3, kg = warp >> 2;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sQ = sbase + S::kQ;
    auto sK = [&](int st, int blk) { return sbase + S::kKV + ((st * 2 + blk) * 2 + 0) * S::kTile; };
    auto sV = [&](int st, int blk) { return sbase + S::kKV + ((st * 2 + blk) * 2 + 1) * S::kTile; };

    const long long qr0 = (long long)b * a.q_rows_per_b;
    const long long kr0 = (long long)b * a.k_rows_per_b;
    const long long col = (long long)h * HD;
    const int nkb = (a.n_k + 63) >> 6;
    const int npairs = (nkb + 1) >> 1;

    const bool tma = HD == 64 && a.kv_map != nullptr;
    const uint32_t bar = sbase + S::kBar;
    auto load_pair = [&](int pi, int st) {
      if (tma) {
        if (threadIdx.x == 0) {
          const int nb = min(2, nkb - 2 * pi);
          mbar_arrive_expect_tx(bar + 8 * st, (uint32_t)(nb * 2 * S::kTile));
          for (int blk = 0; blk < nb; ++blk) {
            const int row = (int)kr0 + (2 * pi + blk) * 64;  // keys past n_k read as zeros
            tma_load_2d(sK(st, blk), a.kv_map, (int)col, row, bar + 8 * st);
            tma_load_2d(sV(st, blk), a.kv_map, a.n_heads * HD + (int)col, row, bar + 8 * st);
          }
        }
        return;
      }
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const int kb = 2 * pi + blk;
        if (kb < nkb) {
          const int nv = min(64, a.n_k - kb * 64);
          load_tile(sK(st, blk), a.k, a.ldk, col, kr0 + kb * 64, nv);
          load_tile(sV(st, blk), a.v, a.ldv, col, kr0 + kb * 64, nv);
        }
      }
    };

    if (tma) {
      // the barriers live in memory other phases reuse: initialise per unit
      if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        mbar_init(bar + 8, 1);
        mbar_fence_init();
      }
      __syncthreads();
    }
    load_tile(sQ, a.q, a.ldq, col, qr0, a.n_q);
    load_pair(0, 0);
    cp_async_commit();

    State sw;
    reset(sw);
    for (int pi = 0; pi < npairs; ++pi) {
      const int st = pi & 1;
      if (pi + 1 < npairs) load_pair(pi + 1, st ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
      if (tma && !mbar_wait(bar + 8 * st, (uint32_t)((pi >> 1) & 1), a.timeout_ns) && a.status)
        atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
      __syncthreads();
      if (pi == 0) load_q(sw, sQ, qt, lane);
      const int kb = 2 * pi + kg;
      if (kb < nkb) block(sw, a, sK(st, kg), sV(st, kg), kb, lane);
      __syncthreads();  // buffer st is refilled by the next iteration's prefetch
    }
    cp_async_wait<0>();
    finish(sw, a, smem + S::kMerge, qr0, col, warp, lane);
    __syncthreads();  // smem reuse by the next unit / phase
  }
};

}  // namespace ee
