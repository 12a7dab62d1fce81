// ee_sampler.cuh -- the fused flow-matching sampler: one persistent launch per
// sampler call (kernel/flow_expert.py:127-137 flow_sample over
// ActionExpert.forward :117-124 and Block.forward :83-95).
//
// One CTA per SM in clusters of CL CTAs, the grid sized to the clusters
// that can be resident at once (cudaOccupancyMaxActiveClusters), launched as a
// plain cluster launch (the same launch eagerly and inside a CUDA graph). A
// call is a fixed sequence of phases separated by a bounded grid barrier:
//   EMB      time embedding of every step's t (t advanced in the act dtype)
//   TPROJ    t_proj over all steps' embeddings at once (t does not depend on x)
//   HEAD     step-0 in_proj + t_proj add (one CTA per token)
//   per step, per block:
//            qkv (first norm on load) | self-attn | proj + residual |
//            q_c (norm on load) | cross-attn | out_c + residual |
//            mlp0 (norm on load) + GELU | mlp2 + residual
//   TAILHEAD out_norm + out_proj + Euler update of step k, then in_proj + t add
//            of step k+1 (one CTA per token)
//   TAIL     the last step's out_norm + out_proj + Euler update
// GEMM phases are cluster split-K units (ee_gemm.cuh). The norms in front of
// qkv / q_c / mlp0 are applied while those GEMMs stage their activation
// slices, from per-token (sum, sum of squares) partials that the producing
// residual phase writes in its epilogue, one slot per 16 output columns,
// summed by the consumer in a fixed order (deterministic). Before each barrier a CTA
// starts copying the weights of its first unit of the next GEMM phase into
// shared memory, so weight latency overlaps the barrier.
#pragma once

#include <atomic>
#include <mutex>

#include "ee_attn.cuh"
#include "ee_gemm.cuh"
#include "ee_host.h"

namespace ee {

enum { PH_EMB = 0, PH_TPROJ, PH_HEAD, PH_GEMM, PH_ATTN_SELF, PH_ATTN_CROSS, PH_TAILHEAD, PH_TAIL };

// globaltimer stamps per (phase, CTA) in the optional trace: work done and
// barrier left; a build with EE_TRACE_DETAIL adds the GEMM units' step stamps
// (slots 2..10)
#ifdef EE_TRACE_DETAIL
constexpr int kTraceSlots = 16;
#else
constexpr int kTraceSlots = 2;
#endif

struct Ctx {
  ee_expert ex;
  const void* x_in;
  const void* t0;
  void* x_out;
  int n_steps, mode, M, Rt, nbt;
  float dtf;
  unsigned long long timeout_ns;
  unsigned* bar;
  int* abort_flag;
  int* status;
  float* stats;  // [2][M][n_slots][2] row (sum, sum of squares) of the norm inputs,
                 // alternating between the two halves by norm sequence number
  int n_inst;    // norms per step (3 per block, 2 without self-attention)
  int n_slots;   // partial-statistics slots per row: (1 << stat_shift)-column slices of d
  int stat_shift;
  uint32_t desc; // shared-memory copy of the block table (byte offset)
  int ks_cap;    // largest K slice a GEMM unit may stage
  int lsplit[7]; // log2 CTAs per unit of t_proj, qkv, proj, q_c, out_c, mlp0, mlp2
  int cluster;   // cluster size and grid the splits were planned for
  int grid;
  void *x, *qkv, *att, *qb, *hid, *emb, *temb;
  GemmSmem sm;
  size_t smem_bytes;
  unsigned long long* trace;  // optional [n_phases][grid][2] globaltimer stamps
};

struct Phase {
  int type, step, layer, sub;  // sub: canonical block sub-phase 0..7
};

EE_DEV int phases_per_block(const Ctx& c) { return c.ex.self_attn ? 8 : 5; }
EE_DEV int num_phases(const Ctx& c) {
  return 3 + c.n_steps * (c.ex.n_layers * phases_per_block(c) + 1);
}
EE_DEV Phase decode(const Ctx& c, int p) {
  Phase ph{0, 0, 0, 0};
  if (p < 3) {
    ph.type = p == 0 ? PH_EMB : (p == 1 ? PH_TPROJ : PH_HEAD);
    return ph;
  }
  const int nb = phases_per_block(c);
  const int per = c.ex.n_layers * nb + 1;
  const int q = p - 3;
  ph.step = q / per;
  const int r = q - ph.step * per;
  if (r == c.ex.n_layers * nb) {
    ph.type = (ph.step + 1 < c.n_steps && c.mode == EE_MODE_EULER) ? PH_TAILHEAD : PH_TAIL;
    return ph;
  }
  ph.layer = r / nb;
  ph.sub = r - ph.layer * nb + (c.ex.self_attn ? 0 : 3);
  ph.type = ph.sub == 1 ? PH_ATTN_SELF : (ph.sub == 4 ? PH_ATTN_CROSS : PH_GEMM);
  return ph;
}

// norm instances of a step: first norm of layer l, nx of l, n2 of l
EE_DEV int inst_first(const Ctx& c, int l) { return l * (c.ex.self_attn ? 3 : 2); }
EE_DEV int inst_x(const Ctx& c, int l) { return c.ex.self_attn ? 3 * l + 1 : 2 * l; }
EE_DEV int inst_2(const Ctx& c, int l) { return c.ex.self_attn ? 3 * l + 2 : 2 * l + 1; }
EE_DEV float* stats_of(const Ctx& c, int step, int inst) {
  return c.stats + (size_t)((step * c.n_inst + inst) & 1) * c.M * c.n_slots * 2;
}

EE_DEV GemmArgs make_gemm(const Ctx& c, const Phase& ph, const char* smem) {
  GemmArgs a{};
  const int d = c.ex.d_model;
  a.M = c.M;
  a.stat_slots = c.n_slots;
  a.stat_shift = c.stat_shift;
  a.in_norm = c.ex.norm_kind;
  a.in_eps = c.ex.eps;
  if (ph.type == PH_TPROJ) {
    a.x = c.emb; a.ldx = d;
    a.w = c.ex.t_proj;
    a.M = c.Rt;
    a.epi = EPI_STORE;
    a.out = c.temb; a.ldo = d;
  } else {
    const ee_block* blk = reinterpret_cast<const ee_block*>(smem + c.desc) + ph.layer;
    const int l = ph.layer;
    switch (ph.sub) {
      case 0:
        a.x = c.x; a.ldx = d; a.w = blk->qkv; a.epi = EPI_STORE; a.out = c.qkv; a.ldo = 3 * d;
        a.in_stats = stats_of(c, ph.step, inst_first(c, l));
        a.in_w = blk->n1.weight; a.in_b = blk->n1.bias;
        break;
      case 2:
        a.x = c.att; a.ldx = d; a.w = blk->proj; a.epi = EPI_RESID; a.out = c.x; a.ldo = d;
        a.out_stats = stats_of(c, ph.step, inst_x(c, l));
        break;
      case 3:
        a.x = c.x; a.ldx = d; a.w = blk->q_c; a.epi = EPI_STORE; a.out = c.qb; a.ldo = d;
        a.in_stats = stats_of(c, ph.step, inst_x(c, l));
        a.in_w = blk->nx.weight; a.in_b = blk->nx.bias;
        break;
      case 5:
        a.x = c.att; a.ldx = d; a.w = blk->out_c; a.epi = EPI_RESID; a.out = c.x; a.ldo = d;
        a.out_stats = stats_of(c, ph.step, inst_2(c, l));
        break;
      case 6:
        a.x = c.x; a.ldx = d; a.w = blk->mlp0; a.epi = EPI_GELU; a.out = c.hid; a.ldo = c.ex.hidden;
        a.in_stats = stats_of(c, ph.step, inst_2(c, l));
        a.in_w = blk->n2.weight; a.in_b = blk->n2.bias;
        break;
      default:  // 7
        a.x = c.hid; a.ldx = c.ex.hidden; a.w = blk->mlp2; a.epi = EPI_RESID; a.out = c.x; a.ldo = d;
        if (l + 1 < c.ex.n_layers) a.out_stats = stats_of(c, ph.step, inst_first(c, l + 1));
    }
    if (a.epi == EPI_RESID) { a.resid = c.x; a.ldr = d; }
  }
  a.has_bias = a.w.bias != nullptr;
  a.status = c.status;
  a.timeout_ns = c.timeout_ns;
  const int gi = ph.type == PH_TPROJ ? 0 : (ph.sub == 0 ? 1 : ph.sub == 2 ? 2 : ph.sub == 3 ? 3 : ph.sub == 5 ? 4 : ph.sub == 6 ? 5 : 6);
  a.lsplit = c.lsplit[gi];
  a.split = 1 << a.lsplit;
  return a;
}

// run a GEMM phase, or (prefetch) start copying this CTA's first unit's
// weights and return whether one was started
template <typename T>
EE_DEV bool gemm_dispatch(const GemmArgs& a, char* smem, const GemmSmem& sm, const PreRegs* pre,
                          bool prefetch, PreRegs* pr_out) {
  switch (a.w.wkind) {
    case EE_W_DENSE:
      if (prefetch) return Gemm<T, EE_W_DENSE, true>::start_prefetch(a, sm, smem, *pr_out);
      Gemm<T, EE_W_DENSE, true>::run(a, smem, sm, pre);
      break;
    case EE_W_INT8:
      if (prefetch) return Gemm<T, EE_W_INT8, true>::start_prefetch(a, sm, smem, *pr_out);
      Gemm<T, EE_W_INT8, true>::run(a, smem, sm, pre);
      break;
    case EE_W_INT4:
      if (prefetch) return Gemm<T, EE_W_INT4, true>::start_prefetch(a, sm, smem, *pr_out);
      Gemm<T, EE_W_INT4, true>::run(a, smem, sm, pre);
      break;
    default:
      if (prefetch) return Gemm<T, EE_W_UINT4Z, true>::start_prefetch(a, sm, smem, *pr_out);
      Gemm<T, EE_W_UINT4Z, true>::run(a, smem, sm, pre);
  }
  return false;
}

// ---------------------------------------------------------------------------
// row-local phases: one CTA per token row
// ---------------------------------------------------------------------------
EE_DEV float block_sum(float v, float* scratch /* [kWarps] */) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) r += scratch[i];
  __syncthreads();
  return r;
}

// Two sums over the CTA at once (one pair of __syncthreads).
EE_DEV float2 block_sum2(float a, float b, float* scratch /* [2 * kWarps] */) {
  a = warp_sum(a);
  b = warp_sum(b);
  if ((threadIdx.x & 31) == 0) {
    scratch[threadIdx.x >> 5] = a;
    scratch[kWarps + (threadIdx.x >> 5)] = b;
  }
  __syncthreads();
  float ra = 0.f, rb = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) {
    ra += scratch[i];
    rb += scratch[kWarps + i];
  }
  __syncthreads();
  return make_float2(ra, rb);
}

// Token row m at `step`: (tail) out_norm + out_proj + Euler update or
// velocity store, then (head) x = in_proj(x_act) + b + temb(next step) with
// its row statistics for the next first norm. Every load that does not
// depend on this phase's arithmetic (the x row, the out_norm parameters, the
// out_proj weights -- copied into the idle partial-tile buffers --, the
// in_proj weights -- copied into the rest of the x region and the idle
// prefetch area -- and the Euler source values) is issued at entry.
// Shared memory: d + 128 floats in the x region, out_proj in the p region,
// in_proj rows [0, wi_split) after them in the x region, the others in the
// pre area.
template <typename T>
EE_DEV void row_phase(const Ctx& c, int m, int step, bool do_tail, bool do_head, char* smem) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int d = c.ex.d_model, A = c.ex.action_dim, nch = d / 8;
  float* hrow = reinterpret_cast<float*>(smem + c.sm.x);  // [d]
  float* xa = hrow + d;                                    // [32] action row after the update
  float* xs = xa + 32;                                     // [32] Euler source values
  float* red = xs + 32;                                    // [2 * kWarps]
  const int head_step = do_tail ? step + 1 : 0;

  // ---- 1. loads that do not depend on this phase's arithmetic ----
  uint4 xq = make_uint4(0, 0, 0, 0), wq = xq, bq = xq;
  const T* Wo = reinterpret_cast<const T*>(c.ex.out_proj.weight);
  const bool wo_smem = do_tail && (size_t)A * d * 2 <= 2 * kPBytes;
  const uint32_t wo_s = smem_u32(smem) + c.sm.p;
  // in_proj weights [d][A] (A * 2 bytes per row) into shared memory when they fit
  const T* Wi = reinterpret_cast<const T*>(c.ex.in_proj.weight);
  const uint32_t rowb = (uint32_t)A * 2u;
  const uint32_t wi_a = smem_u32(smem) + c.sm.x + (uint32_t)(d + 128) * 4u;  // after hrow / xa / xs / red
  const uint32_t wi_a_cap = (c.sm.p - c.sm.x) - (uint32_t)(d + 128) * 4u;
  const int wi_split = (int)(wi_a_cap / rowb) < d ? (int)(wi_a_cap / rowb) : d;
  const uint32_t wi_b = smem_u32(smem) + c.sm.pre;
  const bool wi_smem = do_head && (size_t)(d - wi_split) * rowb <= c.sm.pre_bytes && (A % 8) == 0;
  auto wi_addr = [&](int n) { return n < wi_split ? wi_a + (uint32_t)n * rowb : wi_b + (uint32_t)(n - wi_split) * rowb; };
  if (do_tail) {
    if (tid < nch) {
      xq = ld_act16(reinterpret_cast<const T*>(c.x) + (size_t)m * d + tid * 8);
      wq = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(c.ex.out_norm.weight) + tid * 8));
      if (c.ex.out_norm.bias)
        bq = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(c.ex.out_norm.bias) + tid * 8));
    }
    if (wo_smem) {
      for (int i = tid; i < A * nch; i += kThreads) cp_async16(wo_s + (uint32_t)i * 16u, Wo + (size_t)i * 8, true);
      cp_async_commit();
    }
    if (tid < A && c.mode != EE_MODE_VELOCITY) {
      const T* src = step == 0 ? reinterpret_cast<const T*>(c.x_in) : reinterpret_cast<const T*>(c.x_out);
      xs[tid] = Act<T>::to_f(*reinterpret_cast<const T*>(reinterpret_cast<const char*>(src) +
                                                           ((size_t)m * A + tid) * sizeof(T)));
    }
  }
  if (wi_smem) {  // after the out_proj copies: the tail waits for those alone
    const int cpr = A / 8;  // 16-byte chunks per row
    for (int i = tid; i < d * cpr; i += kThreads) {
      const int n = i / cpr, q = i - n * cpr;
      cp_async16(wi_addr(n) + (uint32_t)q * 16u, Wi + (size_t)n * A + 8 * q, true);
    }
    cp_async_commit();
  }
  const int bb = m / c.ex.horizon;
  const int trow = head_step * c.nbt + (c.nbt > 1 ? bb : 0);
  const T* bi = reinterpret_cast<const T*>(c.ex.in_proj.bias);
  const T* temb = reinterpret_cast<const T*>(c.temb) + (size_t)trow * d;

  if (do_tail) {
    // ---- 2. out_norm of x[m] (one fused sum / sum-of-squares reduction) ----
    float v[8];
    float s1 = 0.f, s2 = 0.f;
    if (tid < nch) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Act<T>::unpack2(comp(xq, e));
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s1 += v[e];
        s2 += v[e] * v[e];
      }
    }
    const float2 tot = block_sum2(s1, s2, red);
    const float inv_d = 1.0f / (float)d;
    float mean = 0.f, rstd;
    if (c.ex.norm_kind == EE_NORM_RMS) {
      rstd = 1.0f / sqrtf(tot.y * inv_d + c.ex.eps);
    } else {
      mean = tot.x * inv_d;
      rstd = 1.0f / sqrtf(fmaxf(tot.y * inv_d - mean * mean, 0.f) + c.ex.eps);
    }
    if (tid < nch) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 wf = Act<T>::unpack2(comp(wq, e));
        const float2 bf = Act<T>::unpack2(comp(bq, e));
        float y0, y1;
        if (c.ex.norm_kind == EE_NORM_RMS) {
          y0 = Act<T>::round(v[2 * e] * rstd) * wf.x;
          y1 = Act<T>::round(v[2 * e + 1] * rstd) * wf.y;
        } else {
          y0 = (v[2 * e] - mean) * rstd * wf.x + bf.x;
          y1 = (v[2 * e + 1] - mean) * rstd * wf.y + bf.y;
        }
        hrow[tid * 8 + 2 * e] = Act<T>::round(y0);
        hrow[tid * 8 + 2 * e + 1] = Act<T>::round(y1);
      }
    }
    if (wo_smem) {
      if (wi_smem) cp_async_wait<1>();
      else cp_async_wait<0>();
    }
    __syncthreads();
    // ---- 3. out_proj: warp w computes outputs a = w, w+8, w+16, w+24,
    //         the four dot products interleaved (one hrow read for all) ----
    const T* ob = reinterpret_cast<const T*>(c.ex.out_proj.bias);
    float accs[4] = {0.f, 0.f, 0.f, 0.f};
    for (int ch = lane; ch < nch; ch += 32) {
      float hv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) hv[e] = hrow[ch * 8 + e];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int a = warp + kWarps * j;
        if (a < A) {
          const uint4 wv = wo_smem ? lds16(wo_s + (uint32_t)(a * nch + ch) * 16u) : ld_weight16(Wo + (size_t)a * d + ch * 8);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Act<T>::unpack2(comp(wv, e));
            accs[j] = fmaf(hv[2 * e], f.x, accs[j]);
            accs[j] = fmaf(hv[2 * e + 1], f.y, accs[j]);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < 4; ++j) accs[j] += __shfl_xor_sync(0xffffffffu, accs[j], o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int a = warp + kWarps * j;
      if (a < A) {
        const float acc = accs[j];
        if (lane == 0) {
          const float vel = Act<T>::round(acc + (ob ? ld_param(ob + a) : 0.f));
          T* xo = reinterpret_cast<T*>(c.x_out) + (size_t)m * A + a;
          if (c.mode == EE_MODE_VELOCITY) {
            *xo = Act<T>::from_f(vel);
          } else {
            const float xnew = Act<T>::round(xs[a] + Act<T>::round(vel * c.dtf));
            *xo = Act<T>::from_f(xnew);
            xa[a] = xnew;
          }
        }
      }
    }
  } else if (tid < A) {
    xa[tid] = Act<T>::to_f(reinterpret_cast<const T*>(c.x_in)[(size_t)m * A + tid]);
  }
  if (!do_head) return;
  if (wi_smem) cp_async_wait<0>();
  __syncthreads();
  // ---- 4. in_proj + bias + t_proj(temb) for the head step; row statistics ----
  T* xr = reinterpret_cast<T*>(c.x) + (size_t)m * d;
  float s = 0.f, ss = 0.f;
  auto one = [&](int n, const uint4 (&w4)[4], float bias, float tv) {
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (q * 8 < A) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = Act<T>::unpack2(comp(w4[q], e));
          acc = fmaf(xa[8 * q + 2 * e], f.x, acc);
          acc = fmaf(xa[8 * q + 2 * e + 1], f.y, acc);
        }
      }
    }
    acc += bias;
    const float y = Act<T>::round(Act<T>::round(acc) + tv);
    xr[n] = Act<T>::from_f(y);
    s += y;
    ss += y * y;
  };
  for (int n = tid; n < d; n += kThreads) {
    uint4 w4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      w4[q] = q * 8 < A ? (wi_smem ? lds16(wi_addr(n) + (uint32_t)q * 16u) : ld_weight16(Wi + (size_t)n * A + 8 * q))
                        : make_uint4(0, 0, 0, 0);
    one(n, w4, bi ? ld_param(bi + n) : 0.f, ld_act_scalar(temb + n));
  }
  const float2 tot = block_sum2(s, ss, red);
  // slot 0 holds the whole row, the other slots are zero
  float* st = stats_of(c, head_step, 0) + 2 * (size_t)m * c.n_slots;
  if (tid < c.n_slots) {
    st[2 * tid] = tid == 0 ? tot.x : 0.f;
    st[2 * tid + 1] = tid == 0 ? tot.y : 0.f;
  }
}

// ---------------------------------------------------------------------------
// bounded grid barrier: every wait gives up after timeout_ns, records
// EE_ERR_TIMEOUT in the status word and raises the abort flag, so no CTA can
// spin forever; CTAs that see the flag return.
// ---------------------------------------------------------------------------
EE_DEV bool grid_barrier(unsigned* bar, int* abort_flag, int* status, unsigned long long timeout_ns,
                         unsigned target) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    // arrive with release semantics (orders this CTA's writes, made visible to
    // thread 0 by the __syncthreads above, before the count); the polling
    // loads below acquire, so no separate fences are needed
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(bar), "r"(1u) : "memory");
    const unsigned long long t0 = globaltimer();
    unsigned spins = 0;
    while (ld_acquire_gpu(bar) < target) {
      if ((++spins & 63u) == 0) {
        if (ld_volatile_i32(abort_flag)) {
          ok = 0;
          break;
        }
        if (globaltimer() - t0 > timeout_ns) {
          atomicCAS(status, 0, (int)EE_ERR_TIMEOUT);
          atomicExch(abort_flag, 1);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}
EE_DEV bool grid_barrier(const Ctx& c, unsigned target) {
  return grid_barrier(c.bar, c.abort_flag, c.status, c.timeout_ns, target);
}

// Split form of the barrier: arrive (after a __syncthreads that ends the
// phase), do work that needs no other CTA's results, then wait.
EE_DEV void grid_arrive(const Ctx& c) {
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(c.bar), "r"(1u) : "memory");
}
EE_DEV bool grid_wait(const Ctx& c, unsigned target) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long t0 = globaltimer();
    unsigned spins = 0;
    while (ld_acquire_gpu(c.bar) < target) {
      if ((++spins & 63u) == 0) {
        if (ld_volatile_i32(c.abort_flag)) {
          ok = 0;
          break;
        }
        if (globaltimer() - t0 > c.timeout_ns) {
          atomicCAS(c.status, 0, (int)EE_ERR_TIMEOUT);
          atomicExch(c.abort_flag, 1);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads, 1) sampler_kernel(const __grid_constant__ Ctx c) {
  extern __shared__ __align__(128) char smem_raw[];
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  PreRegs pre;
  bool have_pre = false;
  const int P = num_phases(c);
  const int d = c.ex.d_model;
  unsigned target = 0;
  // The work split was planned for this launch shape; any other shape (a
  // launch path that dropped the cluster dimension, say) does no work.
  if ((int)cl_size() != c.cluster || (int)gridDim.x != c.grid) {
    if (threadIdx.x == 0) atomicCAS(c.status, 0, (int)EE_ERR_LAUNCH);
    return;
  }
  {  // block table -> shared memory (read by every GEMM phase)
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(c.ex.blocks);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(smem + c.desc);
    const int n = c.ex.n_layers * (int)(sizeof(ee_block) / 8);
    for (int i = threadIdx.x; i < n; i += kThreads) dst[i] = src[i];
  }
  // tcgen05 state: the two stage mbarriers and the TMEM columns the GEMM
  // units use for the whole call (one CTA per SM, so the allocation is free)
  const uint32_t tc_state = smem_u32(smem) + c.sm.tc;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) mbar_init(tc_state + kTcBar + 8 * s, 1);
    *reinterpret_cast<uint32_t*>(smem + c.sm.tc + kTcMask) = 0;
    mbar_init(tc_state + kTcPBar, 1);
    mbar_init(tc_state + kTcPBar + 8, 1);
    *reinterpret_cast<uint32_t*>(smem + c.sm.tc + kTcPPar) = 0;
    mbar_fence_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(tc_state + kTcTmem, kTcCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  auto release_tmem = [&]() {  // every tcgen05 operation of this CTA has completed
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
      tc_fence_after();
      tmem_dealloc(*reinterpret_cast<volatile uint32_t*>(smem + c.sm.tc + kTcTmem), kTcCols);
    }
  };

  for (int p = 0; p < P; ++p) {
    const Phase ph = decode(c, p);
#ifdef EE_TRACE_DETAIL
    if (c.trace && threadIdx.x == 0) c.trace[((size_t)p * gridDim.x + blockIdx.x) * kTraceSlots + 12] = globaltimer();
#endif
    switch (ph.type) {
      case PH_EMB: {
        const int half = d / 2;
        const long long total = (long long)c.Rt * half;
        const float* fr = c.ex.freqs;
        T* emb = reinterpret_cast<T*>(c.emb);
        for (long long idx = (long long)blockIdx.x * kThreads + threadIdx.x; idx < total;
             idx += (long long)gridDim.x * kThreads) {
          const int row = (int)(idx / half), i = (int)(idx - (long long)row * half);
          const int k = row / c.nbt, bb = row - k * c.nbt;
          float tt = c.t0 ? Act<T>::to_f(reinterpret_cast<const T*>(c.t0)[bb]) : 0.f;
          for (int s = 0; s < k; ++s) tt = Act<T>::round(tt + c.dtf);
          const float arg = (tt * __ldg(fr + i)) * 1000.0f;
          emb[(size_t)row * d + i] = Act<T>::from_f(cosf(arg));
          emb[(size_t)row * d + half + i] = Act<T>::from_f(sinf(arg));
        }
        break;
      }
      case PH_TPROJ:
      case PH_GEMM: {
        GemmArgs ga = make_gemm(c, ph, smem);
#ifdef EE_TRACE_DETAIL
        if (c.trace) ga.dtr = c.trace + ((size_t)p * gridDim.x + blockIdx.x) * kTraceSlots + 2;
        if (c.trace && threadIdx.x == 0) c.trace[((size_t)p * gridDim.x + blockIdx.x) * kTraceSlots + 13] = globaltimer();
#endif
        gemm_dispatch<T>(ga, smem, c.sm, have_pre ? &pre : nullptr, false, nullptr);
        break;
      }
      case PH_ATTN_SELF:
      case PH_ATTN_CROSS: {
        AttnArgs at{};
        const ee_block* blk = reinterpret_cast<const ee_block*>(smem + c.desc) + ph.layer;
        if (ph.type == PH_ATTN_SELF) {
          const T* qkv = reinterpret_cast<const T*>(c.qkv);
          at.q = qkv; at.ldq = 3 * d;
          at.k = qkv + d; at.ldk = 3 * d;
          at.v = qkv + 2 * d; at.ldv = 3 * d;
          at.n_k = c.ex.horizon;
          at.k_rows_per_b = c.ex.horizon;
        } else {
          const T* kv = reinterpret_cast<const T*>(blk->kv);
          at.q = c.qb; at.ldq = d;
          at.k = kv; at.ldk = 2 * d;
          at.v = kv + d; at.ldv = 2 * d;
          at.n_k = c.ex.prefix_len;
          at.k_rows_per_b = c.ex.prefix_len;
          if (c.ex.kv_maps) at.kv_map = reinterpret_cast<const CUtensorMap*>(c.ex.kv_maps) + ph.layer;
        }
        at.status = c.status;
        at.timeout_ns = c.timeout_ns;
        at.out = c.att; at.ldo = d;
        at.n_q = c.ex.horizon;
        at.q_rows_per_b = c.ex.horizon;
        at.n_heads = c.ex.n_heads;
        at.scale_log2 = 1.4426950408889634f / sqrtf((float)HD);
        const int units = c.ex.batch * c.ex.n_heads;
        for (int u = blockIdx.x; u < units; u += gridDim.x)
          Attn<T, HD>::unit(at, u / c.ex.n_heads, u % c.ex.n_heads, smem);
        break;
      }
      case PH_HEAD:
        for (int m = blockIdx.x; m < c.M; m += gridDim.x) {
          row_phase<T>(c, m, 0, false, true, smem);
          __syncthreads();
        }
        break;
      default:  // PH_TAILHEAD, PH_TAIL
        for (int m = blockIdx.x; m < c.M; m += gridDim.x) {
          row_phase<T>(c, m, ph.step, true, ph.type == PH_TAILHEAD, smem);
          __syncthreads();
        }
        break;
    }
    have_pre = false;
    __syncthreads();  // this CTA is done with phase p (and its shared memory)
    if (c.trace && threadIdx.x == 0)
      c.trace[((size_t)p * gridDim.x + blockIdx.x) * kTraceSlots] = globaltimer();
    if (p + 1 < P) {
      // arrive first, then start the next GEMM phase's weight copies while
      // the other CTAs finish (the copies read only constant weights)
      grid_arrive(c);
      target += gridDim.x;
      const Phase nx = decode(c, p + 1);
      if (nx.type == PH_GEMM || nx.type == PH_TPROJ)
        have_pre = gemm_dispatch<T>(make_gemm(c, nx, smem), smem, c.sm, nullptr, true, &pre);
#ifdef EE_TRACE_DETAIL
      if (c.trace && threadIdx.x == 0) c.trace[((size_t)p * gridDim.x + blockIdx.x) * kTraceSlots + 11] = globaltimer();
#endif
      if (!grid_wait(c, target)) {
        cp_async_wait<0>();
        release_tmem();
        return;
      }
    }
    if (c.trace && threadIdx.x == 0)
      c.trace[((size_t)p * gridDim.x + blockIdx.x) * kTraceSlots + 1] = globaltimer();
  }
  release_tmem();
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Layout {
  size_t sync, stats, x, qkv, att, qb, hid, emb, temb, total;
  int M, n_inst, n_slots, Rt_max;
};

inline size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

inline Layout layout_for(const ee_expert& ex, int n_steps) {
  Layout L{};
  const size_t e = 2;  // bytes per act element
  const size_t d = (size_t)ex.d_model;
  L.M = ex.batch * ex.horizon;
  L.n_inst = ex.n_layers * (ex.self_attn ? 3 : 2);
  L.Rt_max = n_steps * ex.batch;
  size_t off = 0;
  L.sync = off; off += 256;
  L.n_slots = (ex.d_model + 7) / 8;  // room for 8-column slots
  L.stats = off; off += al256((size_t)2 * L.M * L.n_slots * 2 * sizeof(float));
  L.x = off; off += al256((size_t)L.M * d * e);
  L.qkv = off; off += ex.self_attn ? al256((size_t)L.M * 3 * d * e) : 0;
  L.att = off; off += al256((size_t)L.M * d * e);
  L.qb = off; off += al256((size_t)L.M * d * e);
  L.hid = off; off += al256((size_t)L.M * ex.hidden * e);
  L.emb = off; off += al256((size_t)L.Rt_max * d * e);
  L.temb = off; off += al256((size_t)L.Rt_max * d * e);
  L.total = off;
  return L;
}

// portable cluster size of the sampler: the model width must split into
// 128-wide k-blocks across the cluster (K = d_model is the smallest GEMM K).
// Where it is 8, a cluster of 16 (non-portable; units of K = d_model then
// take half a cluster) is also considered.
inline int sampler_cluster(const ee_expert& ex) {
  const int kb = ex.d_model / 128;
  int cl = 8;
  while (cl > 1 && (kb % cl) != 0) cl >>= 1;
  return cl;
}

// largest K slice a unit stages: what the widest GEMM (K = max(d, hidden))
// needs with the whole cluster splitting it, at least 512. Where an 8-CTA
// cluster would leave a wider slice (an MLP of 8192 at d_model 2048) and the
// width splits into 16 k-block slices, the plan is for 16-CTA clusters
// (non-portable; the launch geometry then rejects 8-CTA plans, whose split
// would exceed this cap), keeping the staged slice at 512.
inline int sampler_ks_cap(const ee_expert& ex) {
  const int kmax = ex.hidden > ex.d_model ? ex.hidden : ex.d_model;
  int need = kmax / sampler_cluster(ex);
  if (need > 512 && sampler_cluster(ex) == 8 && (ex.d_model / 128) % 16 == 0) need = kmax / 16;
  return need > 512 ? need : 512;
}

struct SamplerSmem {
  GemmSmem g;
  uint32_t desc;   // block table copy
  size_t total;    // dynamic shared memory of the launch
};

inline SamplerSmem sampler_smem_map(const ee_expert& ex, int smem_optin) {
  size_t x = gemm_x_bytes(sampler_ks_cap(ex));
  if (x < (size_t)kMTile * (kRU + 1) * 4) x = (size_t)kMTile * (kRU + 1) * 4;  // reduced tile E
  const size_t rows = ((size_t)ex.d_model + 128) * 4;               // row phases
  if (rows > x) x = rows;
  x = (x + 127) & ~(size_t)127;
  SamplerSmem sm;
  sm.g.x = 0;
  sm.g.p = (uint32_t)x;
  sm.g.aux = (uint32_t)(x + 2 * kPBytes);
  // the block table must survive the attention phases, which use [0, attn)
  const size_t hd = ex.n_heads > 0 ? ex.d_model / ex.n_heads : 64;
  const size_t attn = hd == 128 ? AttnSmem<128>::kTotal : AttnSmem<64>::kTotal;
  size_t desc = sm.g.aux + kAuxBytes;
  if (desc < attn) desc = attn;
  desc = (desc + 127) & ~(size_t)127;
  sm.desc = (uint32_t)desc;
  // tcgen05 state (mbarriers, TMEM address, commit counts) after the block table
  sm.g.tc = (uint32_t)((desc + (size_t)ex.n_layers * sizeof(ee_block) + 15) & ~(size_t)15);
  const size_t pre = (sm.g.tc + kTcStateBytes + 127) & ~(size_t)127;
  sm.g.pre = (uint32_t)pre;
  // 1 KB static reserve, 1 KB to align the dynamic base to 1024 bytes (the
  // 128-byte-swizzled operand tiles start on 1024-byte boundaries)
  const long long room = (long long)smem_optin - 2048 - (long long)pre;
  sm.g.pre_bytes = room > 0 ? (uint32_t)(room < 128 * 1024 ? room : 128 * 1024) : 0;
  sm.total = pre + sm.g.pre_bytes + 1024;
  return sm;
}

inline int validate_expert(const ee_expert& ex, int n_steps, int mode) {
  if (ex.act_dtype != EE_BF16 && ex.act_dtype != EE_F16) return EE_ERR_DTYPE;
  if (ex.n_layers < 1 || ex.n_heads < 1 || ex.batch < 1 || ex.horizon < 1) return EE_ERR_SHAPE;
  if (ex.d_model < 256 || ex.d_model > 2048 || (ex.d_model % 256) != 0) return EE_ERR_SHAPE;
  if (ex.d_model % ex.n_heads) return EE_ERR_SHAPE;
  const int hd = ex.d_model / ex.n_heads;
  if (hd != 64 && hd != 128) return EE_ERR_UNSUPPORTED;
  if (ex.horizon > 64) return EE_ERR_UNSUPPORTED;
  if (ex.action_dim < 8 || ex.action_dim > 32 || (ex.action_dim % 8)) return EE_ERR_UNSUPPORTED;
  if (ex.prefix_len < 1) return EE_ERR_SHAPE;
  if (ex.hidden < 128 || (ex.hidden % 128) || ex.hidden > 16384) return EE_ERR_SHAPE;
  if (ex.norm_kind != EE_NORM_LAYER && ex.norm_kind != EE_NORM_RMS) return EE_ERR_ARG;
  if (n_steps < 1 || n_steps > 1024) return EE_ERR_SHAPE;
  if (mode != EE_MODE_EULER && mode != EE_MODE_VELOCITY) return EE_ERR_ARG;
  if (mode == EE_MODE_VELOCITY && n_steps != 1) return EE_ERR_ARG;
  if (!ex.freqs || !ex.blocks || !ex.out_norm.weight) return EE_ERR_ARG;
  if (ex.norm_kind == EE_NORM_LAYER && !ex.out_norm.bias) return EE_ERR_ARG;
  if (!ex.in_proj.weight || ex.in_proj.wkind != EE_W_DENSE || ex.in_proj.n != ex.d_model ||
      ex.in_proj.k != ex.action_dim)
    return EE_ERR_SHAPE;
  if (!ex.out_proj.weight || ex.out_proj.wkind != EE_W_DENSE || ex.out_proj.n != ex.action_dim ||
      ex.out_proj.k != ex.d_model)
    return EE_ERR_SHAPE;
  if (!aligned16(ex.in_proj.weight) || !aligned16(ex.out_proj.weight) ||
      !aligned16(ex.out_norm.weight) || (ex.out_norm.bias && !aligned16(ex.out_norm.bias)))
    return EE_ERR_ALIGN;
  // shared memory must hold the widest GEMM slice next to the fixed regions
  const SamplerSmem sm = sampler_smem_map(ex, 232448);
  if ((size_t)sm.g.pre + 2048 > 232448) return EE_ERR_UNSUPPORTED;
  return validate_linear(ex.t_proj, ex.d_model, ex.d_model);
}

inline int validate_blocks(const ee_expert& ex, const ee_block* hb) {
  int rc = EE_OK;
  const int d = ex.d_model;
  for (int l = 0; rc == EE_OK && l < ex.n_layers; ++l) {
    const ee_block& b = hb[l];
    auto norm_ok = [&](const ee_norm& nrm) {
      if (!nrm.weight || !aligned16(nrm.weight)) return false;
      if (ex.norm_kind == EE_NORM_LAYER && (!nrm.bias || !aligned16(nrm.bias))) return false;
      return true;
    };
    if (ex.self_attn) {
      if (!norm_ok(b.n1)) rc = EE_ERR_ARG;
      if (!rc) rc = validate_linear(b.qkv, 3 * d, d);
      if (!rc) rc = validate_linear(b.proj, d, d);
    }
    if (!rc && (!norm_ok(b.nx) || !norm_ok(b.n2))) rc = EE_ERR_ARG;
    if (!rc) rc = validate_linear(b.q_c, d, d);
    if (!rc) rc = validate_linear(b.out_c, d, d);
    if (!rc) rc = validate_linear(b.mlp0, ex.hidden, d);
    if (!rc) rc = validate_linear(b.mlp2, d, ex.hidden);
    if (!rc && (!b.kv || !aligned16(b.kv))) rc = EE_ERR_ARG;
  }
  return rc;
}

template <typename T, int HD>
constexpr auto fn_of() { return sampler_kernel<T, HD>; }

// Launch geometry of the sampler kernel: clusters of `cl` CTAs, as many as
// can be resident at once (at most one CTA per SM).
// GEMM shapes of a step (n, k, tokens): t_proj, qkv, proj, q_c, out_c, mlp0, mlp2
inline void step_shapes(const Ctx& c, int (&shapes)[7][3]) {
  const ee_expert& ex = c.ex;
  const int d = ex.d_model, M = c.M;
  const int sh[7][3] = {{d, d, c.Rt}, {3 * d, d, M}, {d, d, M}, {d, d, M},
                        {d, d, M}, {ex.hidden, d, M}, {d, ex.hidden, M}};
  for (int i = 0; i < 7; ++i)
    for (int j = 0; j < 3; ++j) shapes[i][j] = sh[i][j];
}

// Serial work of a CTA over one step's GEMMs with `grid` CTAs in clusters of
// `cl`: sum of rounds x k-blocks per unit under pick_split (-1: no split fits).
inline long long plan_cost(const Ctx& c, int grid, int cl) {
  int shapes[7][3];
  step_shapes(c, shapes);
  long long cost = 0;
  for (int i = 1; i < 7; ++i) {
    const int sp = pick_split(shapes[i][0], shapes[i][1], shapes[i][2], grid / cl, cl, c.ks_cap);
    if (sp <= 0) return -1;
    const long long units = (long long)((shapes[i][0] + kRU - 1) / kRU) * ((shapes[i][2] + kMTile - 1) / kMTile);
    const long long slots = (long long)(grid / cl) * (cl / sp);
    cost += ((units + slots - 1) / slots) * (shapes[i][1] / sp / kKBlock);
  }
  return cost;
}

// Launch geometry of the sampler kernel: clusters of `cl` CTAs, as many as
// can be resident at once (at most one CTA per SM); of the candidate cluster
// sizes the one whose GEMM plan has the least serial work per CTA (ties: the
// portable size).
template <typename T, int HD>
int sampler_geometry(const Ctx& c, int* grid, int* cl_out, size_t* smem_out) {
  auto fn = sampler_kernel<T, HD>;
  const int cl0 = sampler_cluster(c.ex);
  const size_t smem = c.smem_bytes;
  static std::atomic<int> smem_set[64];
  allow_max_smem(fn, smem_set);
  const int cands[2] = {cl0, cl0 == 8 ? 16 : 0};
  // the occupancy queries are costly: remember the resident grid of each
  // candidate per device (0: the candidate cannot launch)
  static std::mutex mu;
  static struct { int cl0; size_t smem; int grids[2]; bool valid; } memo[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return EE_ERR_DEVICE;
  int grids[2] = {0, 0};
  bool have = false;
  {
    std::lock_guard<std::mutex> g(mu);
    if (memo[dev].valid && memo[dev].cl0 == cl0 && memo[dev].smem == smem) {
      grids[0] = memo[dev].grids[0];
      grids[1] = memo[dev].grids[1];
      have = true;
    }
  }
  if (!have) {
    const int max_ctas = device_sms();
    for (int ci = 0; ci < 2; ++ci) {
      const int cl = cands[ci];
      if (cl <= 0) continue;
      if (cl > 8 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        continue;
      }
      cudaLaunchConfig_t cfg{};
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = cl;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cfg.gridDim = dim3(cl);
      int nclusters = 0;
      if (cudaOccupancyMaxActiveClusters(&nclusters, fn, &cfg) != cudaSuccess || nclusters < 1) {
        cudaGetLastError();
        continue;
      }
      if (nclusters * cl > max_ctas) nclusters = max_ctas / cl;
      grids[ci] = nclusters * cl;
    }
    std::lock_guard<std::mutex> g(mu);
    memo[dev].cl0 = cl0;
    memo[dev].smem = smem;
    memo[dev].grids[0] = grids[0];
    memo[dev].grids[1] = grids[1];
    memo[dev].valid = true;
  }
  int best_grid = 0, best_cl = 0;
  long long best_cost = -1;
  for (int ci = 0; ci < 2; ++ci) {
    if (grids[ci] <= 0) continue;
    const long long cost = plan_cost(c, grids[ci], cands[ci]);
    if (cost < 0) continue;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_grid = grids[ci];
      best_cl = cands[ci];
    }
  }
  if (best_grid <= 0) return EE_ERR_LAUNCH;
  *grid = best_grid;
  *cl_out = best_cl;
  *smem_out = smem;
  return EE_OK;
}

// CTAs per unit of every GEMM of the step (host-side, from the grid
// geometry), and the width of the row-statistics slots: 16 columns, or the
// smallest row slice a statistics-producing GEMM (proj, out_c, mlp2) reduces
inline int plan_splits(Ctx& c, int grid, int cl) {
  int shapes[7][3];
  step_shapes(c, shapes);
  int min_rows = kRU;
  for (int i = 0; i < 7; ++i) {
    const int sp = pick_split(shapes[i][0], shapes[i][1], shapes[i][2], grid / cl, cl, c.ks_cap);
    if (sp <= 0) return EE_ERR_UNSUPPORTED;
    int l = 0;
    while ((1 << l) < sp) ++l;
    c.lsplit[i] = l;
    if ((i == 2 || i == 4 || i == 6) && (kRU >> l) < min_rows) min_rows = kRU >> l;
  }
  c.stat_shift = min_rows >= 16 ? 4 : 3;
  if (min_rows < 8) return EE_ERR_UNSUPPORTED;
  c.n_slots = (c.ex.d_model + (1 << c.stat_shift) - 1) >> c.stat_shift;
  return EE_OK;
}

template <typename T, int HD>
int launch_sampler(Ctx c, cudaStream_t s) {
  int grid = 0, cl = 0;
  size_t smem = 0;
  int rc = sampler_geometry<T, HD>(c, &grid, &cl, &smem);
  if (rc) return rc;
  rc = plan_splits(c, grid, cl);
  if (rc) return rc;
  c.cluster = cl;
  c.grid = grid;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  // The grid never exceeds the clusters that fit on the device at once, so
  // on a GPU not shared with concurrent kernels every CTA is resident; if one
  // is not (another process holding SMs), the grid barrier's bounded wait
  // ends the call with EE_ERR_TIMEOUT in the status word instead of hanging.
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn_of<T, HD>(), c);
  return e == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

}  // namespace ee
