// ee_sampler.cuh -- the fused flow-matching sampler: one persistent launch per
// sampler call (kernel/flow_expert.py:127-137 flow_sample over
// ActionExpert.forward :117-124 and Block.forward :83-95).
//
// One CTA per SM in clusters of CL CTAs, cooperative launch. A call is a
// fixed sequence of phases separated by a bounded grid barrier:
//   EMB      time embedding of every step's t (t advanced in the act dtype)
//   TPROJ    t_proj over all steps' embeddings at once (t does not depend on x)
//   HEAD     step-0 in_proj + t_proj add + first norm (row-local, warp/token)
//   per step, per block: qkv | self-attn | proj+residual(+norm) | q_c |
//            cross-attn | out_c+residual(+norm) | mlp0+GELU | mlp2+residual(+norm)
//   TAILHEAD out_norm + out_proj + Euler update of step k, then in_proj + t add
//            + first norm of step k+1 (all row-local: one warp per token)
//   TAIL     the last step's out_norm + out_proj + Euler update
// GEMM phases are cluster split-K units (ee_gemm.cuh). Before each barrier a
// CTA starts copying the weights of its first unit of the next GEMM phase
// into shared memory, so weight latency overlaps the barrier. The norm after
// a residual update is done by the last CTA to finish each 64-token tile.
#pragma once

#include <atomic>

#include "ee_attn.cuh"
#include "ee_gemm.cuh"
#include "ee_host.h"

namespace ee {

enum { PH_EMB = 0, PH_TPROJ, PH_HEAD, PH_GEMM, PH_ATTN_SELF, PH_ATTN_CROSS, PH_TAILHEAD, PH_TAIL };

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
  unsigned* ln_cnt;
  void *x, *h, *qkv, *att, *qb, *hid, *emb, *temb;
  GemmSmem sm;
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

// first norm of a block: n1, or nx when the block has no self-attention
EE_DEV ee_norm first_norm(const Ctx& c, const ee_block* blk) {
  return c.ex.self_attn ? blk->n1 : blk->nx;
}

EE_DEV GemmArgs make_gemm(const Ctx& c, const Phase& ph) {
  GemmArgs a{};
  const int d = c.ex.d_model;
  a.norm_kind = c.ex.norm_kind;
  a.eps = c.ex.eps;
  a.ln_cnt = c.ln_cnt;
  a.M = c.M;
  if (ph.type == PH_TPROJ) {
    a.x = c.emb; a.ldx = d;
    a.w = c.ex.t_proj;
    a.M = c.Rt;
    a.epi = EPI_STORE;
    a.out = c.temb; a.ldo = d;
  } else {
    const ee_block* blk = c.ex.blocks + ph.layer;
    switch (ph.sub) {
      case 0:
        a.x = c.h; a.ldx = d; a.w = blk->qkv; a.epi = EPI_STORE; a.out = c.qkv; a.ldo = 3 * d;
        break;
      case 2:
        a.x = c.att; a.ldx = d; a.w = blk->proj; a.epi = EPI_RESID; a.out = c.x; a.ldo = d;
        a.ln_w = blk->nx.weight; a.ln_b = blk->nx.bias; a.ln_out = c.h;
        break;
      case 3:
        a.x = c.h; a.ldx = d; a.w = blk->q_c; a.epi = EPI_STORE; a.out = c.qb; a.ldo = d;
        break;
      case 5:
        a.x = c.att; a.ldx = d; a.w = blk->out_c; a.epi = EPI_RESID; a.out = c.x; a.ldo = d;
        a.ln_w = blk->n2.weight; a.ln_b = blk->n2.bias; a.ln_out = c.h;
        break;
      case 6:
        a.x = c.h; a.ldx = d; a.w = blk->mlp0; a.epi = EPI_GELU; a.out = c.hid; a.ldo = c.ex.hidden;
        break;
      default: {  // 7
        a.x = c.hid; a.ldx = c.ex.hidden; a.w = blk->mlp2; a.epi = EPI_RESID; a.out = c.x; a.ldo = d;
        if (ph.layer + 1 < c.ex.n_layers) {
          const ee_norm nn = first_norm(c, blk + 1);
          a.ln_w = nn.weight; a.ln_b = nn.bias; a.ln_out = c.h;
        }
      }
    }
    if (a.epi == EPI_RESID) { a.resid = c.x; a.ldr = d; }
  }
  a.has_bias = a.w.bias != nullptr;
  return a;
}

EE_DEV int gemm_units(const GemmArgs& a) {
  return ((a.w.n + kRU - 1) / kRU) * ((a.M + kMTile - 1) / kMTile);
}

template <typename T, int KIND>
EE_DEV void gemm_phase_t(const GemmArgs& a, char* smem, const GemmSmem& sm, const PreRegs* pre,
                         bool prefetch, PreRegs* pr_out) {
  const int units = gemm_units(a);
  const int n_tiles = (a.w.n + kRU - 1) / kRU;
  if (prefetch) {
    if ((int)cl_id() < units) Gemm<T, KIND>::prefetch_unit(a, cl_id(), smem, sm, *pr_out);
    return;
  }
  const PreRegs* p = pre;
  for (int u = cl_id(); u < units; u += cl_count()) {
    Gemm<T, KIND>::unit(a, u % n_tiles, (u / n_tiles) * kMTile, smem, sm, p);
    p = nullptr;
  }
}

// run a GEMM phase (prefetch == false) or start the prefetch of this CTA's
// first unit (prefetch == true; returns whether one was started)
template <typename T>
EE_DEV bool gemm_dispatch(const GemmArgs& a, char* smem, const GemmSmem& sm, const PreRegs* pre,
                          bool prefetch, PreRegs* pr_out) {
  switch (a.w.wkind) {
    case EE_W_DENSE: gemm_phase_t<T, EE_W_DENSE>(a, smem, sm, pre, prefetch, pr_out); break;
    case EE_W_INT8: gemm_phase_t<T, EE_W_INT8>(a, smem, sm, pre, prefetch, pr_out); break;
    case EE_W_INT4: gemm_phase_t<T, EE_W_INT4>(a, smem, sm, pre, prefetch, pr_out); break;
    default: gemm_phase_t<T, EE_W_UINT4Z>(a, smem, sm, pre, prefetch, pr_out); break;
  }
  return prefetch && (int)cl_id() < gemm_units(a);
}

// ---------------------------------------------------------------------------
// row-local phases: one warp per token row, row staged in rb (d floats)
// ---------------------------------------------------------------------------
// norm of the row in rb; result stored to orow (T) when given, else written
// back into rb rounded to the act dtype
template <typename T>
EE_DEV void norm_buf(float* rb, int d, const ee_norm& nrm, int kind, float eps, T* orow) {
  const int lane = threadIdx.x & 31;
  const float inv_d = 1.0f / (float)d;
  const T* w = reinterpret_cast<const T*>(nrm.weight);
  const T* b = reinterpret_cast<const T*>(nrm.bias);
  __syncwarp();
  float s = 0.f;
  for (int i = lane; i < d; i += 32) s += kind == EE_NORM_RMS ? rb[i] * rb[i] : rb[i];
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
  for (int c = lane; c < d / 8; c += 32) {
    const uint4 wq = __ldg(reinterpret_cast<const uint4*>(w + c * 8));
    const uint4 bq = b ? __ldg(reinterpret_cast<const uint4*>(b + c * 8)) : make_uint4(0, 0, 0, 0);
    float y[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 wf = Act<T>::unpack2(comp(wq, e));
      const float2 bf = Act<T>::unpack2(comp(bq, e));
      const float v0 = rb[c * 8 + 2 * e], v1 = rb[c * 8 + 2 * e + 1];
      if (kind == EE_NORM_RMS) {
        y[2 * e] = Act<T>::round(v0 * rstd) * wf.x;
        y[2 * e + 1] = Act<T>::round(v1 * rstd) * wf.y;
      } else {
        y[2 * e] = (v0 - mean) * rstd * wf.x + bf.x;
        y[2 * e + 1] = (v1 - mean) * rstd * wf.y + bf.y;
      }
    }
    if (orow) {
      *reinterpret_cast<uint4*>(orow + c * 8) =
          make_uint4(Act<T>::pack2(y[0], y[1]), Act<T>::pack2(y[2], y[3]),
                     Act<T>::pack2(y[4], y[5]), Act<T>::pack2(y[6], y[7]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) rb[c * 8 + e] = Act<T>::round(y[e]);
    }
  }
  __syncwarp();
}

// x[m] = in_proj(x_act[m]) + b + temb(step); h[m] = first_norm(x[m]).
// xa_lane: lane a (< action_dim) holds x_act[m][a].
template <typename T>
EE_DEV void head_row(const Ctx& c, int m, int step, float xa_lane, float* rb) {
  const int lane = threadIdx.x & 31;
  const int d = c.ex.d_model, A = c.ex.action_dim;
  float xa[32];
#pragma unroll
  for (int a = 0; a < 32; ++a) xa[a] = __shfl_sync(0xffffffffu, xa_lane, a);
  const int bb = m / c.ex.horizon;
  const int trow = step * c.nbt + (c.nbt > 1 ? bb : 0);
  const T* W = reinterpret_cast<const T*>(c.ex.in_proj.weight);
  const T* bias = reinterpret_cast<const T*>(c.ex.in_proj.bias);
  const T* temb = reinterpret_cast<const T*>(c.temb) + (size_t)trow * d;
  T* xr = reinterpret_cast<T*>(c.x) + (size_t)m * d;
  for (int ch = lane; ch < d / 8; ch += 32) {
    const uint4 tq = ld_act16(temb + ch * 8);
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int n = ch * 8 + e;
      const T* wr = W + (size_t)n * A;
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q * 8 < A) {
          const uint4 w = ld_weight16(wr + 8 * q);
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const float2 f = Act<T>::unpack2(comp(w, cc));
            acc = fmaf(xa[8 * q + 2 * cc], f.x, acc);
            acc = fmaf(xa[8 * q + 2 * cc + 1], f.y, acc);
          }
        }
      }
      if (bias) acc += ld_param(bias + n);
      const float2 tf = Act<T>::unpack2(comp(tq, e >> 1));
      y[e] = Act<T>::round(Act<T>::round(acc) + ((e & 1) ? tf.y : tf.x));
      rb[n] = y[e];
    }
    *reinterpret_cast<uint4*>(xr + ch * 8) =
        make_uint4(Act<T>::pack2(y[0], y[1]), Act<T>::pack2(y[2], y[3]),
                   Act<T>::pack2(y[4], y[5]), Act<T>::pack2(y[6], y[7]));
  }
  norm_buf<T>(rb, d, first_norm(c, c.ex.blocks), c.ex.norm_kind, c.ex.eps,
              reinterpret_cast<T*>(c.h) + (size_t)m * d);
}

// out_norm + out_proj + Euler update (or velocity store) of token row m at
// `step`; returns the new x_act value held by lane a (< action_dim).
template <typename T>
EE_DEV float tail_row(const Ctx& c, int m, int step, float* rb) {
  const int lane = threadIdx.x & 31;
  const int d = c.ex.d_model, A = c.ex.action_dim;
  const T* xr = reinterpret_cast<const T*>(c.x) + (size_t)m * d;
  for (int ch = lane; ch < d / 8; ch += 32) {
    const uint4 q = ld_act16(xr + ch * 8);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Act<T>::unpack2(comp(q, e));
      rb[ch * 8 + 2 * e] = f.x;
      rb[ch * 8 + 2 * e + 1] = f.y;
    }
  }
  norm_buf<T>(rb, d, c.ex.out_norm, c.ex.norm_kind, c.ex.eps, nullptr);
  // out_proj partial dots of this lane's chunks for every output a
  const T* W = reinterpret_cast<const T*>(c.ex.out_proj.weight);
  float part[32];
#pragma unroll
  for (int a = 0; a < 32; ++a) part[a] = 0.f;
  for (int ch = lane; ch < d / 8; ch += 32) {
    float hv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) hv[e] = rb[ch * 8 + e];
#pragma unroll
    for (int a = 0; a < 32; ++a) {
      if (a < A) {
        const uint4 w = ld_weight16(W + (size_t)a * d + ch * 8);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const float2 f = Act<T>::unpack2(comp(w, cc));
          part[a] = fmaf(hv[2 * cc], f.x, part[a]);
          part[a] = fmaf(hv[2 * cc + 1], f.y, part[a]);
        }
      }
    }
  }
  // transpose-reduce: afterwards lane a holds the full sum of output a
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? part[i] : part[i + o];
      const float keep = upper ? part[i + o] : part[i];
      part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float xa_new = 0.f;
  if (lane < A) {
    const T* ob = reinterpret_cast<const T*>(c.ex.out_proj.bias);
    const float vel = Act<T>::round(part[0] + (ob ? ld_param(ob + lane) : 0.f));
    T* xo = reinterpret_cast<T*>(c.x_out) + (size_t)m * A + lane;
    if (c.mode == EE_MODE_VELOCITY) {
      *xo = Act<T>::from_f(vel);
      xa_new = vel;
    } else {
      const T* src = step == 0 ? reinterpret_cast<const T*>(c.x_in) + (size_t)m * A + lane : xo;
      const float xa_old = Act<T>::to_f(*src);
      xa_new = Act<T>::round(xa_old + Act<T>::round(vel * c.dtf));
      *xo = Act<T>::from_f(xa_new);
    }
  }
  return xa_new;
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
    __threadfence();
    atomicAdd(bar, 1u);
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
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}
EE_DEV bool grid_barrier(const Ctx& c, unsigned target) {
  return grid_barrier(c.bar, c.abort_flag, c.status, c.timeout_ns, target);
}

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads, 1) sampler_kernel(const __grid_constant__ Ctx c) {
  extern __shared__ __align__(128) char smem[];
  PreRegs pre;
  bool have_pre = false;
  const int P = num_phases(c);
  const int gwarp = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * kWarps;
  const int lane = threadIdx.x & 31;
  const int d = c.ex.d_model;
  float* rb = reinterpret_cast<float*>(smem + c.sm.x) + (size_t)(threadIdx.x >> 5) * d;
  unsigned target = 0;

  for (int p = 0; p < P; ++p) {
    const Phase ph = decode(c, p);
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
      case PH_GEMM:
        gemm_dispatch<T>(make_gemm(c, ph), smem, c.sm, have_pre ? &pre : nullptr, false, nullptr);
        break;
      case PH_ATTN_SELF:
      case PH_ATTN_CROSS: {
        AttnArgs at{};
        const ee_block* blk = c.ex.blocks + ph.layer;
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
        }
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
      case PH_HEAD: {
        for (int m = gwarp; m < c.M; m += nwarps) {
          const float xa =
              lane < c.ex.action_dim
                  ? Act<T>::to_f(reinterpret_cast<const T*>(c.x_in)[(size_t)m * c.ex.action_dim + lane])
                  : 0.f;
          head_row<T>(c, m, 0, xa, rb);
        }
        break;
      }
      default: {  // PH_TAILHEAD, PH_TAIL
        for (int m = gwarp; m < c.M; m += nwarps) {
          const float xa = tail_row<T>(c, m, ph.step, rb);
          if (ph.type == PH_TAILHEAD) head_row<T>(c, m, ph.step + 1, xa, rb);
        }
        break;
      }
    }
    have_pre = false;
    if (p + 1 < P) {
      const Phase nx = decode(c, p + 1);
      __syncthreads();  // this CTA is done with its shared memory for phase p
      if (nx.type == PH_GEMM || nx.type == PH_TPROJ)
        have_pre = gemm_dispatch<T>(make_gemm(c, nx), smem, c.sm, nullptr, true, &pre);
      target += gridDim.x;
      if (!grid_barrier(c, target)) {
        cp_async_wait<0>();
        return;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Layout {
  size_t sync, lncnt, x, h, qkv, att, qb, hid, emb, temb, total;
  int M, m_tiles, Rt_max;
};

inline size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

inline Layout layout_for(const ee_expert& ex, int n_steps) {
  Layout L{};
  const size_t e = 2;  // bytes per act element
  const size_t d = (size_t)ex.d_model;
  L.M = ex.batch * ex.horizon;
  L.m_tiles = (L.M + kMTile - 1) / kMTile;
  L.Rt_max = n_steps * ex.batch;
  size_t off = 0;
  L.sync = off; off += 256;
  L.lncnt = off; off += al256((size_t)L.m_tiles * 4);
  L.x = off; off += al256((size_t)L.M * d * e);
  L.h = off; off += al256((size_t)L.M * d * e);
  L.qkv = off; off += ex.self_attn ? al256((size_t)L.M * 3 * d * e) : 0;
  L.att = off; off += al256((size_t)L.M * d * e);
  L.qb = off; off += al256((size_t)L.M * d * e);
  L.hid = off; off += al256((size_t)L.M * ex.hidden * e);
  L.emb = off; off += al256((size_t)L.Rt_max * d * e);
  L.temb = off; off += al256((size_t)L.Rt_max * d * e);
  L.total = off;
  return L;
}

// cluster size of the sampler: every GEMM K (d and hidden) must split into
// 128-wide slices
inline int sampler_cluster(const ee_expert& ex) {
  const int kb = ex.d_model / 128;
  int cl = 8;
  while (cl > 1 && (kb % cl) != 0) cl >>= 1;
  return cl;
}

inline GemmSmem sampler_smem_map(const ee_expert& ex, int cl) {
  const int kmax = ex.hidden > ex.d_model ? ex.hidden : ex.d_model;
  size_t x = gemm_x_bytes(kmax / cl);
  const size_t e = (size_t)kMTile * (kRU / cl) * 4;
  const size_t rows = (size_t)kWarps * ex.d_model * 4;
  if (e > x) x = e;
  if (rows > x) x = rows;
  x = (x + 127) & ~(size_t)127;
  GemmSmem sm;
  sm.x = 0;
  sm.p = (uint32_t)x;
  sm.pre = (uint32_t)(x + kPBytes);
  return sm;
}

template <int HD>
inline size_t sampler_smem_bytes(const GemmSmem& sm) {
  const size_t g = (size_t)sm.pre + kPreBytes;
  return g > (size_t)AttnSmem<HD>::kTotal ? g : (size_t)AttnSmem<HD>::kTotal;
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
  // shared memory must hold the largest GEMM slice
  const int cl = sampler_cluster(ex);
  const GemmSmem sm = sampler_smem_map(ex, cl);
  if ((size_t)sm.pre + kPreBytes > 227 * 1024) return EE_ERR_UNSUPPORTED;
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
int launch_sampler(const Ctx& c, cudaStream_t s) {
  auto fn = sampler_kernel<T, HD>;
  const int cl = sampler_cluster(c.ex);
  const size_t smem = sampler_smem_bytes<HD>(c.sm);
  static std::atomic<int> smem_set[64];
  allow_max_smem(fn, smem_set);
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // as many whole clusters as can be resident at once (one CTA per SM)
  cfg.gridDim = dim3(cl);
  int nclusters = 0;
  if (cudaOccupancyMaxActiveClusters(&nclusters, fn, &cfg) != cudaSuccess || nclusters < 1)
    return EE_ERR_LAUNCH;
  const int max_ctas = device_sms();
  if (nclusters * cl > max_ctas) nclusters = max_ctas / cl;
  cfg.gridDim = dim3(nclusters * cl);
  // Cooperative launch guarantees that every CTA is resident. Inside a stream
  // capture the plain cluster launch is used: the grid is sized to what can be
  // resident at once, and every barrier wait is bounded either way.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) return EE_ERR_LAUNCH;
  cfg.numAttrs = cap == cudaStreamCaptureStatusNone ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, c);
  return e == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

}  // namespace ee
