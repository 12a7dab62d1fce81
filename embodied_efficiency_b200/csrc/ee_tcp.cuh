// ee_tcp.cuh -- persistent form of the tcgen05 dequant-GEMM (ee_tc.cuh) for
// calls with more tiles than SMs and no split of K: one CTA per SM loops over
// tiles (tile = blockIdx.x,
// blockIdx.x + gridDim.x, ...), and the epilogue of a tile overlaps the next
// tile's loads, dequantisation and MMAs.
//
// Roles (26 warps):
//   warps 0-15   dequantisers, as in ee_tc.cuh; their k-block sequence runs
//                on across tiles
//   warp 16      TMA producer: raw weights and activations of every k-block
//                of every tile into the ring of `ns` stages
//   warp 17      TMEM allocator and MMA issuer: tile i accumulates into TMEM
//                buffer i % 2 (two buffers of TMC columns) once the epilogue
//                has drained that buffer's previous tile
//   warps 18-25  epilogue: two warps per 32-lane quarter of TMEM, half of
//                the NT columns each, in 16-token chunks: bias (and GELU) per lane, the
//                chunk staged through shared memory as [16 tokens][32 rows],
//                then per lane 16-byte residual loads (one chunk ahead) and
//                16-byte stores; the buffer is then released to the MMA issuer.
//                With dense weights (nothing to dequantise) warps 0-15 join
//                them: six warps per quarter, taking its 16-token chunks in
//                turn (the GELU of a large-batch MLP is issue-bound with two)
// The weight and activation tiles, the dequantised A layout, the MMA and the
// epilogue arithmetic are those of wq_tc_kernel, so the two give identical
// outputs. Every wait is bounded (%globaltimer); a timeout records
// EE_ERR_TIMEOUT in the status word.
#pragma once

namespace ee {

constexpr int kTcpEpiWarp0 = kTcDqWarps + 2;  // first epilogue warp
constexpr int kTcpWarps = kTcDqWarps + 2 + kTcpEpiWarps;
constexpr int kTcpThreads = kTcpWarps * 32;

template <typename T, int KIND, int NT>
__global__ void __launch_bounds__(kTcpThreads, 1)
    wq_tcp_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                  const __grid_constant__ TcArgs a) {
  constexpr bool DQ = KIND != EE_W_DENSE;
  constexpr uint32_t WB = tc_wbytes<KIND>();
  constexpr uint32_t XB = (uint32_t)NT * 256u;  // two boxes [NT rows][64 k]
  constexpr uint32_t TMC = tc_tmem_cols(NT);     // columns of one accumulator buffer
  constexpr uint32_t TMA2 = 2 * TMC;             // allocation (a power of two)
  constexpr int ITEMS = KIND == EE_W_INT8 ? 2 : 1;
  extern __shared__ __align__(1024) char smem_raw[];
  const uint32_t base0 = smem_u32(smem_raw);
  const uint32_t sb = (base0 + 1023u) & ~1023u;
  char* smem = smem_raw + (sb - base0);
  pdl_entry();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = a.n_units * ((a.M + NT - 1) / NT);
  const int my_tiles = blockIdx.x < (unsigned)n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const ee_linear& L = a.w;
  const uint32_t bar_full = sb + a.off_bar;
  const uint32_t bar_empty = bar_full + 8u * a.ns;
  const uint32_t bar_afull = bar_empty + 8u * a.ns;
  const uint32_t bar_aempty = bar_afull + 8u * a.na;
  const uint32_t bar_accf = bar_aempty + 8u * a.na;  // [2] accumulator buffer full (MMA commit)
  const uint32_t bar_acce = bar_accf + 16u;          // [2] accumulator buffer drained (epilogue warps)
  auto tile_of = [&](int i, int& n0, int& m0) {
    const int t = (int)blockIdx.x + i * (int)gridDim.x;
    n0 = (t % a.n_units) * 128;
    m0 = (t / a.n_units) * NT;
  };

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
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accf + 8u * b, 1);
      mbar_init(bar_acce + 8u * b, tcp_epi_warps<KIND>());  // the epilogue warps
    }
    mbar_fence_init();
  }
  if (warp == kTcMmaWarp) {
    tmem_alloc(sb + a.off_tm, TMA2);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + a.off_tm);

  if (warp == kTcProdWarp) {
    // ---------------- TMA producer: every k-block of every tile ----------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      int s = 0, sph = 0;
      for (int i = 0; i < my_tiles && ok; ++i) {
        int n0, m0;
        tile_of(i, n0, m0);
        for (int kb = 0; kb < a.kbc; ++kb) {
          if (issued >= a.ns && !mbar_wait(bar_empty + 8u * s, (uint32_t)(sph ^ 1), a.timeout_ns)) {
            ok = false;
            break;
          }
          const uint32_t st = sb + (uint32_t)s * a.stage_bytes, fb = bar_full + 8u * s;
          mbar_arrive_expect_tx(fb, WB + XB);
          if (KIND == EE_W_DENSE) {
            tma_load_2d(st, &tw, kb * 256, n0, fb);
            tma_load_2d(st + 16384u, &tw, kb * 256 + 128, n0, fb);
          } else {
            tma_load_2d(st, &tw, kb * (KIND == EE_W_INT8 ? 128 : 64), n0, fb);
          }
          tma_load_2d(st + WB, &tx, kb * 128, m0, fb);
          tma_load_2d(st + WB + XB / 2, &tx, kb * 128 + 64, m0, fb);
          ++issued;
          if (++s == a.ns) { s = 0; sph ^= 1; }
        }
      }
      if (!ok) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
      // the copies still in flight land before the CTA may exit
      for (int g = issued > a.ns ? issued - a.ns : 0; g < issued; ++g)
        if (!mbar_wait(bar_full + 8u * (g % a.ns), (uint32_t)((g / a.ns) & 1), a.timeout_ns))
          atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == kTcMmaWarp) {
    // ---------------- MMA issuer: tile i into accumulator buffer i % 2 ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc<T>(128, NT);
      bool ok = true;
      int s = 0, sph = 0, as = 0, aph = 0;
      for (int i = 0; i < my_tiles && ok; ++i) {
        const int buf = i & 1;
        // the epilogue has drained this buffer's previous tile (i - 2)
        if (i >= 2 && !mbar_wait(bar_acce + 8u * buf, (uint32_t)(((i >> 1) - 1) & 1), a.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)buf * TMC;
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
            const uint64_t ad = ad0 + (uint64_t)(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
            const uint64_t bd = bd0 + (uint64_t)(((kk >> 2) * (int)(XB / 2) + (kk & 3) * 32) >> 4);
            umma_f16(acc, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(bar_empty + 8u * s);
          if (DQ) umma_commit(bar_aempty + 8u * as);
          if (++s == a.ns) { s = 0; sph ^= 1; }
          if (++as == a.na) { as = 0; aph ^= 1; }
        }
        if (ok) umma_commit(bar_accf + 8u * buf);  // fires when the tile's MMAs have completed
      }
      if (!ok) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp >= kTcpEpiWarp0 || !DQ) {
    // ---------------- epilogue: two (dense weights: six) warps per 32-lane quarter of TMEM ----------------
    // A warp reads TMEM lanes 32 (warp % 4) ..: warps 18-25 cover quarters
    // 2, 3, 0, 1, 2, 3, 0, 1 and warps 0-15 quarters 0, 1, 2, 3, 0, ...
    const int q4 = warp & 3;
    const int ew = warp >= kTcpEpiWarp0 ? warp - kTcpEpiWarp0 : kTcpEpiWarps + warp;  // epilogue warp index
    const int jq = ew >> 2;                                  // index among the quarter's warps
    constexpr int WQ = tcp_epi_warps<KIND>() / 4;            // warps per quarter
    // 16-token chunks: with two warps per quarter, each takes a contiguous
    // half of the NT columns; with six, chunks jq, jq + 6, ...
    constexpr int HC = NT >= 32 ? NT / 2 : NT;
    const int cbeg = DQ ? jq * HC : 16 * jq;
    const int cend = DQ ? (NT >= 32 ? cbeg + HC : (jq == 0 ? NT : 0)) : NT;
    const int cstep = DQ ? 16 : 16 * WQ;
    const int r = 32 * q4 + lane;
    bool ok = true;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int buf = i & 1;
      int n0, m0;
      tile_of(i, n0, m0);
      const int n = n0 + r;
      const float bias = (a.has_bias && n < L.n) ? ld_param(reinterpret_cast<const T*>(L.bias) + n) : 0.f;
      // per 16-token chunk: bias / GELU in registers (lane = weight row),
      // staged as [16 tokens][32 rows] 16-bit values, then each lane handles
      // 8 consecutive rows of one token twice: residual added, 16-byte store
      T* out = reinterpret_cast<T*>(a.out);
      const T* res = reinterpret_cast<const T*>(a.resid);
      const uint32_t stg = sb + a.off_ep + (uint32_t)ew * (16u * 32u * 2u);
      const bool vec = (a.ldo % 8) == 0 && (L.n % 8) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                       (a.epi != EPI_RESID || ((a.ldr % 8) == 0 && (reinterpret_cast<uintptr_t>(a.resid) & 15) == 0));
      const bool vres = vec && a.epi == EPI_RESID;
      // residual pieces of a chunk (this lane's two [token][8 rows] pieces),
      // requested one chunk ahead -- the first before the accumulator wait
      auto load_res = [&](int c0, uint4 (&r)[2]) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int idx = lane + 32 * h2, e = idx >> 2, rg = idx & 3;
          const int tok = m0 + c0 + e, nn = n0 + 32 * q4 + 8 * rg;
          r[h2] = (tok < a.M && nn < L.n) ? *reinterpret_cast<const uint4*>(res + (size_t)tok * a.ldr + nn)
                                          : make_uint4(0, 0, 0, 0);
        }
      };
      uint4 rq_cur[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)}, rq_nxt[2] = {rq_cur[0], rq_cur[1]};
      if (vres && cbeg < cend) load_res(cbeg, rq_cur);
      if (!mbar_wait(bar_accf + 8u * buf, (uint32_t)((i >> 1) & 1), a.timeout_ns)) {
        if (lane == 0) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
        ok = false;
        break;
      }
      tc_fence_after();
      for (int c0 = cbeg; c0 < cend; c0 += cstep) {
        if (vres && c0 + cstep < cend) load_res(c0 + cstep, rq_nxt);
        uint32_t v[16];
        tmem_ld16(tmem + (uint32_t)buf * TMC + ((uint32_t)(32 * q4) << 16) + (uint32_t)c0, v);
        tmem_wait_ld();
        float y[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          y[e] = Act<T>::round(__uint_as_float(v[e]) + bias);
          if (a.epi == EPI_GELU) y[e] = Act<T>::round(gelu_erf(y[e]));
        }
        if (vec) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const T h = Act<T>::from_f(y[e]);
            asm volatile("st.shared.u16 [%0], %1;" ::"r"(stg + (uint32_t)((e * 32 + lane) * 2)),
                         "h"(*reinterpret_cast<const unsigned short*>(&h))
                         : "memory");
          }
          __syncwarp();
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int idx = lane + 32 * h2;  // 64 pieces: 16 tokens x 4 groups of 8 rows
            const int e = idx >> 2, rg = idx & 3;
            const int tok = m0 + c0 + e, nn = n0 + 32 * q4 + 8 * rg;
            if (tok < a.M && nn < L.n) {
              const uint4 q = lds16(stg + (uint32_t)((e * 32 + 8 * rg) * 2));
              uint4 o = q;
              if (a.epi == EPI_RESID) {
                const uint4 rq = rq_cur[h2];
                uint32_t w[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const float2 fy = Act<T>::unpack2(comp(q, c)), fr = Act<T>::unpack2(comp(rq, c));
                  w[c] = Act<T>::pack2(Act<T>::round(fr.x + fy.x), Act<T>::round(fr.y + fy.y));
                }
                o = make_uint4(w[0], w[1], w[2], w[3]);
              }
              *reinterpret_cast<uint4*>(out + (size_t)tok * a.ldo + nn) = o;
            }
          }
          __syncwarp();
          rq_cur[0] = rq_nxt[0];
          rq_cur[1] = rq_nxt[1];
        } else if (n < L.n) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int tok = m0 + c0 + e;
            if (tok < a.M) {
              float yy = y[e];
              if (a.epi == EPI_RESID) yy = Act<T>::round(ld_param(res + (size_t)tok * a.ldr + n) + yy);
              out[(size_t)tok * a.ldo + n] = Act<T>::from_f(yy);
            }
          }
        }
      }
      // this warp's reads of the buffer are done: release it to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acce + 8u * buf);
    }
  } else {
    // ---------------- dequantisers (warps 0-15): every k-block of every tile ----------------
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
      // a 3-slot ring of this thread's own words, restarted per tile
      const uint32_t scr = sb + a.off_sc + (uint32_t)tid * 4u;
      constexpr uint32_t kSlot = (uint32_t)ITEMS * kTcDqThreads * 4u, kZoff = 3u * kSlot;
      const typename TcDequant<T, KIND>::Groups gp = TcDequant<T, KIND>::groups(L);
      int s = 0, sph = 0, as = 0, aph = 0, done = 0;
      bool ok = true;
      for (int ti = 0; ti < my_tiles && ok; ++ti) {
        int n0, m0;
        tile_of(ti, n0, m0);
        size_t rowsi[ITEMS];  // n * groups-per-row of each item's row
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) rowsi[i] = (size_t)min(n0 + rows[i], L.n - 1) * gp.ng;
#pragma unroll
        for (int d = 0; d < 2; ++d) {
          if (d < a.kbc) {
            const int g = TcDequant<T, KIND>::group_of(gp, d);
#pragma unroll
            for (int i = 0; i < ITEMS; ++i)
              TcDequant<T, KIND>::stage_sz(L, rowsi[i] + g, scr + (uint32_t)d * kSlot + (uint32_t)i * (kTcDqThreads * 4u), kZoff);
          }
          cp_async_commit();
        }
        int r3 = 0, r3n = 2;
        for (int kb = 0; kb < a.kbc; ++kb) {
          if (kb + 2 < a.kbc) {
            const int g = TcDequant<T, KIND>::group_of(gp, kb + 2);
#pragma unroll
            for (int i = 0; i < ITEMS; ++i)
              TcDequant<T, KIND>::stage_sz(L, rowsi[i] + g, scr + (uint32_t)r3n * kSlot + (uint32_t)i * (kTcDqThreads * 4u), kZoff);
          }
          cp_async_commit();
          ok = mbar_wait(bar_full + 8u * s, (uint32_t)sph, a.timeout_ns);
          if (ok && done >= a.na) ok = mbar_wait(bar_aempty + 8u * as, (uint32_t)(aph ^ 1), a.timeout_ns);
          if (!ok) {
            if (lane == 0) atomicCAS(a.status, 0, (int)EE_ERR_TIMEOUT);
            break;
          }
          const uint32_t st = sb + (uint32_t)s * a.stage_bytes;
          const uint32_t ab = sb + a.off_a + (uint32_t)as * 32768u;
          cp_async_wait<2>();  // this k-block's scale words have landed
          const int gcur = TcDequant<T, KIND>::group_of(gp, kb);
#pragma unroll
          for (int i = 0; i < ITEMS; ++i) {
            float scv, zcv;
            TcDequant<T, KIND>::read_sz(L, rowsi[i] + gcur, scr + (uint32_t)r3 * kSlot + (uint32_t)i * (kTcDqThreads * 4u),
                                        kZoff, scv, zcv);
            TcDequant<T, KIND>::item(st, ab, rows[i], chs[i], scv, zcv);
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
          ++done;
        }
        cp_async_wait<0>();
      }
    }
  }
  tc_fence_before();
  __syncthreads();  // every MMA completed (the epilogue waited for each tile) and every TMEM read is done
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, TMA2);
  }
}

}  // namespace ee
