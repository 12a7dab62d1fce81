/*
 * ee_b200.h -- C ABI of the B200 (sm_100a) weight-only dequant-GEMM and
 * flow-matching sampler library (libee_b200.so).
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as an opaque pointer), returns EE_OK (0) or an error code and never
 * aborts the process. Nothing here allocates device memory: scratch space is
 * a caller-owned workspace, so the launch entry points can be captured into a
 * CUDA graph. All device pointers must be 16-byte aligned.
 *
 * Reference interfaces replaced (LaelaZorana/embodied-efficiency):
 *   ee_pack_int4          kernel/triton_gemm.py:37-39   _pack_int4
 *   ee_unpack_int4        kernel/triton_gemm.py:42-48   _unpack_int4
 *   ee_wq_gemm            kernel/triton_gemm.py:141-164 wq_linear
 *                         (+ the Triton kernels at :75-138 it launches)
 *   ee_wq_gemm_status     device status word of the dequant-GEMM (new)
 *   ee_dequant_weight     kernel/quant.py:33-35 dequantize_weight, with the
 *                         GEMM's rounding (kernel/triton_gemm.py:91-94, :127-134)
 *   ee_layer_norm         kernel/flow_expert.py:51-95 the blocks' nn.LayerNorm
 *   ee_attention          kernel/flow_expert.py:86, :91 scaled_dot_product_attention
 *   ee_time_embed         kernel/flow_expert.py:38-48 timestep_embedding (+ the .to(dtype) of :120)
 *   ee_expert_head        kernel/flow_expert.py:119-121 in_proj(x) + t_proj(temb)[:, None]
 *   ee_euler_step         kernel/flow_expert.py:133-136 x = x + v * dt; t = t + dt
 *   ee_flow_sample        kernel/flow_expert.py:127-137 flow_sample, run as
 *                         one fused launch over kernel/flow_expert.py:117-124
 *                         ActionExpert.forward and :83-95 Block.forward
 *                         (mode EE_MODE_VELOCITY = one ActionExpert.forward)
 *   ee_flow_sample_workspace_bytes   sizing helper for ee_flow_sample (new)
 *   ee_check_expert       one-time validation of an expert description (new)
 *   ee_flow_sample_geometry   launch geometry of the fused sampler (new)
 *   ee_flow_sample_traced / ee_flow_sample_phases   per-phase device timeline (new)
 *   ee_read_status        device status word of a sampler workspace (new)
 *   ee_encode_kv_maps     TMA descriptors of the cached prefix K/V (new)
 *   ee_barrier_selftest   bounded-wait self-test of the grid barrier (new)
 *   ee_strerror / ee_version / ee_struct_size   (new)
 */
#ifndef EE_B200_H
#define EE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* ee_stream_t; /* a cudaStream_t; NULL = legacy default stream */

/* ---- status codes ------------------------------------------------------ */
enum {
  EE_OK = 0,
  EE_ERR_ARG = 1,         /* null pointer / bad enum value                 */
  EE_ERR_SHAPE = 2,       /* unsupported or inconsistent sizes             */
  EE_ERR_ALIGN = 3,       /* pointer not 16-byte aligned                   */
  EE_ERR_DTYPE = 4,       /* unsupported dtype combination                 */
  EE_ERR_WORKSPACE = 5,   /* workspace missing or too small                */
  EE_ERR_LAUNCH = 6,      /* CUDA launch / runtime error                   */
  EE_ERR_TIMEOUT = 7,     /* a device-side wait gave up (status word)      */
  EE_ERR_DEVICE = 8,      /* no device / not an sm_100 device              */
  EE_ERR_UNSUPPORTED = 9  /* valid request this build does not implement   */
};

/* ---- dtype / weight-format enums --------------------------------------- */
enum { EE_BF16 = 0, EE_F16 = 1, EE_F32 = 2 };

/* weight formats (bits argument of ee_wq_gemm, wkind of ee_linear):
 *  EE_W_DENSE  weight is [N,K] in the activation dtype (the "bf16" rows)
 *  EE_W_INT8   int8 [N,K], symmetric, scale per (row, group)
 *  EE_W_INT4   uint8 [N,K/2], two's-complement nibbles, even k in the low
 *              nibble (kernel/triton_gemm.py:37-39), symmetric
 *  EE_W_UINT4Z uint8 [N,K/2] unsigned nibbles with a zero point per group
 *              (asymmetric int4; no counterpart in the reference)            */
enum { EE_W_DENSE = 0, EE_W_INT8 = 1, EE_W_INT4 = 2, EE_W_UINT4Z = 3 };

/* epilogue flags of ee_wq_gemm */
enum { EE_EPI_BIAS = 1, EE_EPI_GELU = 2, EE_EPI_RESIDUAL = 4 };

/* sampler modes */
enum { EE_MODE_EULER = 0, EE_MODE_VELOCITY = 1 };

/* norm kinds */
enum { EE_NORM_LAYER = 0, EE_NORM_RMS = 1 };

const char* ee_strerror(int code);
int ee_version(void);
/* sizeof of the ABI records, for binding checks: 0 ee_linear, 1 ee_norm,
 * 2 ee_block, 3 ee_expert; 0 for any other value. */
size_t ee_struct_size(int32_t which);

/* ---- int4 packing (bit-exact with the reference) ----------------------- */
/* q: int8 [n,k] (values in -8..7), packed: uint8 [n,k/2]; k even.           */
int ee_pack_int4(const int8_t* q, uint8_t* packed, int64_t n, int64_t k, ee_stream_t stream);
int ee_unpack_int4(const uint8_t* packed, int8_t* q, int64_t n, int64_t k, ee_stream_t stream);

/* ---- fused weight-only dequant-GEMM ------------------------------------ */
/*
 * y[m,n] = epi( sum_k x[m,k] * dequant(W)[n,k] )   with x, y row-major.
 *   x        [m,k] act dtype (EE_BF16 or EE_F16)
 *   weight   see EE_W_* (reference layout, row n contiguous in k)
 *   scales   [n, k/group] EE_F32 or EE_F16 (scale_dtype); NULL for dense
 *   zeros    [n, k/group] fp16 integer-valued zero points (EE_W_UINT4Z only)
 *   bias     [n] act dtype, used when epilogue has EE_EPI_BIAS
 *   residual [m,n] act dtype, used when epilogue has EE_EPI_RESIDUAL
 *   y        [m,n] act dtype (may alias residual)
 * epi applies, in order: +bias, round to act dtype, then GELU(erf) or
 * residual + value, each rounded to the act dtype (the reference's
 * op-by-op rounding). Requires k % 128 == 0 and group % 128 == 0 (or
 * group == k); m, n arbitrary >= 1.
 */
int ee_wq_gemm(const void* x, const void* weight, const void* scales, const void* zeros,
               const void* bias, const void* residual, void* y,
               int64_t m, int64_t n, int64_t k, int32_t wkind, int32_t group,
               int32_t act_dtype, int32_t scale_dtype, int32_t epilogue, ee_stream_t stream);

/* Status word of the dequant-GEMM kernels on the current device: 0, or the
 * first error a launch recorded since the last reset (EE_ERR_TIMEOUT: a
 * bounded wait of the TMA pipeline gave up; EE_ERR_LAUNCH: a kernel found
 * itself launched without its planned cluster shape and did no work).
 * Synchronises the device; reset != 0 clears the word afterwards. (new) */
int ee_wq_gemm_status(int32_t* status, int32_t reset);

/* A packed weight dequantised into the activation dtype (kernel/quant.py:33-35
 * dequantize_weight; the values are those the dequant-GEMM kernels multiply:
 * the exact integer times the scale rounded to the activation type, one
 * rounding, as kernel/triton_gemm.py:91-94 and :127-134 compute them):
 *   weight  [n, k] int8 (EE_W_INT8) or [n, k/2] packed int4 (EE_W_INT4,
 *           EE_W_UINT4Z), 16-byte aligned
 *   scales / zeros / group / scale_dtype as for ee_wq_gemm
 *   out     [n, k] act dtype, 16-byte aligned
 * k % 128 == 0, group % 128 == 0 or group == k. Used to cache a dense copy of
 * a weight for GEMMs with many tokens, where the tensor cores bound the GEMM. */
int ee_dequant_weight(const void* weight, const void* scales, const void* zeros, void* out, int64_t n, int64_t k,
                      int32_t wkind, int32_t group, int32_t act_dtype, int32_t scale_dtype, ee_stream_t stream);

/* LayerNorm over the last dimension (kernel/flow_expert.py:51-95, the blocks'
 * nn.LayerNorm; used by the layer-by-layer path): y[r] = (x[r] - mean) *
 * rsqrt(var + eps) * weight + bias for rows r < rows of `cols` act-dtype
 * values (row strides ldx / ldy elements), fp32 statistics, one rounding.
 * weight / bias may be NULL (1 / 0). cols % 8 == 0 and cols <= 2048;
 * 16-byte aligned pointers and strides. */
int ee_layer_norm(const void* x, const void* weight, const void* bias, void* y, int64_t rows, int64_t cols,
                  int64_t ldx, int64_t ldy, float eps, int32_t act_dtype, ee_stream_t stream);

/* Attention of the layer-by-layer path (kernel/flow_expert.py:86, :91,
 * F.scaled_dot_product_attention, non-causal): for every batch element b and
 * head h, out[b rows][h*hd ..] = softmax(q k^T / sqrt(hd)) v with q rows
 * b * q_rows_per_b .. + n_q (n_q <= 64) and key rows b * k_rows_per_b .. + n_k
 * of row-major q / k / v (head h at column h * hd; row strides in elements),
 * output merged [rows][n_heads * hd]. hd 64 or 128; act dtype. */
int ee_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* out,
                 int64_t ldo, int32_t batch, int32_t n_heads, int32_t head_dim, int32_t n_q, int32_t n_k,
                 int64_t q_rows_per_b, int64_t k_rows_per_b, int32_t act_dtype, ee_stream_t stream);

/* Row operations of the layer-by-layer sampler path (act dtype throughout).
 * ee_time_embed: emb[b] = [cos(t_b * f * 1000), sin(t_b * f * 1000)] for the
 * dim / 2 fp32 frequencies f (kernel/flow_expert.py:41-43), one rounding to the
 * act dtype; emb is [batch][dim].
 * ee_expert_head: x[m] = round(round(x_act[m] . w_in^T + b_in) +
 * temb[m / rows_per_b]) for rows m < rows: x_act [rows][action_dim]
 * (action_dim % 8 == 0, <= 64), w_in [d_model][action_dim] (16-byte aligned),
 * b_in [d_model] or NULL, temb rows of ld_temb elements, x [rows][d_model].
 * ee_euler_step: x[i] = round(x[i] + round(v[i] * dt)) for i < count and, when
 * t is not NULL, t[b] = round(t[b] + dt) for b < batch. */
int ee_time_embed(const void* t, const float* freqs, void* emb, int32_t batch, int32_t dim, int32_t act_dtype,
                  ee_stream_t stream);
int ee_expert_head(const void* x_act, const void* w_in, const void* b_in, const void* temb, void* x, int64_t rows,
                   int32_t action_dim, int32_t d_model, int64_t rows_per_b, int64_t ld_temb, int32_t act_dtype,
                   ee_stream_t stream);
int ee_euler_step(void* x, const void* v, void* t, int64_t count, int32_t batch, float dt, int32_t act_dtype,
                  ee_stream_t stream);

/* ---- fused flow-matching sampler --------------------------------------- */
typedef struct ee_linear {
  const void* weight; /* see EE_W_*                                       */
  const void* scales; /* [n, k/group] (NULL for dense)                    */
  const void* zeros;  /* [n, k/group] fp16 (EE_W_UINT4Z only, else NULL) */
  const void* bias;   /* [n] act dtype or NULL                            */
  int32_t n, k, wkind, group, scale_dtype, reserved;
} ee_linear;

typedef struct ee_norm {
  const void* weight; /* [d] act dtype                  */
  const void* bias;   /* [d] act dtype or NULL (RMSNorm) */
} ee_norm;

typedef struct ee_block {
  ee_norm n1, nx, n2;
  ee_linear qkv, proj, q_c, out_c, mlp0, mlp2;
  const void* kv; /* prefix K/V cache: kv_c(prefix) output, [batch, prefix_len, 2*d] */
} ee_block;

typedef struct ee_expert {
  int32_t d_model, n_layers, n_heads, horizon, action_dim, prefix_len, hidden, batch;
  int32_t act_dtype, norm_kind, self_attn, reserved;
  float eps, reserved_f;
  const float* freqs; /* [d/2] fp32 time-embedding frequencies (kernel/flow_expert.py:41-43) */
  ee_linear in_proj, t_proj, out_proj;
  ee_norm out_norm;
  const ee_block* blocks; /* DEVICE pointer to n_layers ee_block records */
  /* Optional DEVICE pointer to n_layers 128-byte tensor maps (64-byte
   * aligned) of the blocks' cached prefix K/V, written by ee_encode_kv_maps;
   * with them the cross-attention loads K/V with TMA, without (NULL) it
   * copies them with cp.async. */
  const void* kv_maps;
} ee_expert;

/* Encode the tensor maps of every block's cached prefix K/V ([batch *
 * prefix_len][2 d] of the act dtype, as ee_block.kv points to) into the
 * device buffer `maps` (n_layers * 128 bytes, 64-byte aligned), copied on
 * `stream`. Head size 64 only (EE_ERR_UNSUPPORTED otherwise). `host_blocks`
 * is a HOST copy of the block table, as for ee_check_expert. New: no
 * counterpart in the reference. */
int ee_encode_kv_maps(const ee_expert* ex, const ee_block* host_blocks, void* maps, size_t maps_bytes,
                      ee_stream_t stream);

/* Tracing variant of ee_flow_sample: when `trace` is not NULL, thread 0 of
 * every CTA writes two %globaltimer stamps (ns) per phase p:
 * trace[(p * grid + cta) * 2 + 0] when the CTA finished phase p's work and
 * trace[(p * grid + cta) * 2 + 1] when it left the barrier that follows.
 * `trace` holds ee_flow_sample_phases() * grid * 2 entries (grid from
 * ee_flow_sample_geometry). */
int ee_flow_sample_traced(const ee_expert* ex, const void* x_in, const void* t0, void* x_out,
                          int32_t n_steps, int32_t mode, void* workspace, size_t workspace_bytes,
                          uint64_t* trace, ee_stream_t stream);
/* Number of phases of one ee_flow_sample launch (0 for invalid arguments). */
int32_t ee_flow_sample_phases(const ee_expert* ex, int32_t n_steps);

/* Full validation of an expert description: every scalar field, and every
 * block record from a HOST copy of the table that ex->blocks points to on
 * the device. ee_flow_sample re-checks only the scalar fields (it never reads
 * the device table on the host), so call this once when the table is built. */
int ee_check_expert(const ee_expert* ex, const ee_block* host_blocks, int32_t n_steps, int32_t mode);

/* Workspace bytes ee_flow_sample needs for this expert and step count. */
size_t ee_flow_sample_workspace_bytes(const ee_expert* ex, int32_t n_steps);

/*
 * One sampler call as a single persistent launch (one CTA per SM, phases
 * separated by bounded grid barriers).
 *   x_in  [batch, horizon, action_dim] act dtype
 *   t0    [batch] act dtype start times, or NULL for t = 0
 *   x_out [batch, horizon, action_dim]: EE_MODE_EULER -> x after n_steps
 *         Euler steps (dt = 1/n_steps, t and x kept in the act dtype);
 *         EE_MODE_VELOCITY -> the velocity at (x_in, t0), n_steps must be 1.
 * A device-side wait that exceeds its limit aborts the launch and leaves
 * EE_ERR_TIMEOUT in the workspace status word (see ee_read_status).
 */
int ee_flow_sample(const ee_expert* ex, const void* x_in, const void* t0, void* x_out,
                   int32_t n_steps, int32_t mode, void* workspace, size_t workspace_bytes,
                   ee_stream_t stream);

/* Self-test of the bounded device-side wait: launches one CTA that waits at a
 * grid barrier no other CTA reaches, so the wait ends only by its limit
 * (timeout_ns, at most 2 s) and leaves EE_ERR_TIMEOUT in the status word of
 * `workspace` (>= 256 bytes, read it with ee_read_status). */
int ee_barrier_selftest(void* workspace, uint64_t timeout_ns, ee_stream_t stream);

/* Launch geometry ee_flow_sample uses for this expert on the current device:
 * CTAs in the grid (one per SM at most), CTAs per cluster, dynamic shared
 * memory per CTA. */
int ee_flow_sample_geometry(const ee_expert* ex, int32_t* grid_ctas, int32_t* cluster,
                            size_t* smem_bytes);

/*
 * ee_flow_sample without a caller workspace, for callers that cannot allocate
 * device memory: a hard-real-time control loop must not call cudaMalloc (it
 * can synchronise the device and take an unbounded time mid-period), and a
 * host binding this library through an FFI may own all device memory through
 * its own allocator. No counterpart in the reference.
 *   - The workspace is a fixed 4 MiB array in the library's device image
 *     (held on every GPU that loads the library until the process exits);
 *     calls whose ee_flow_sample_workspace_bytes() exceed it return
 *     EE_ERR_WORKSPACE and launch nothing.
 *   - Allocates nothing: no cudaMalloc / cudaFree, no allocating library call.
 *   - The first call on a device looks up the array's device address; make
 *     that first call before any stream capture on that device. The lookup
 *     is repeated when the device's context has been destroyed and made
 *     again (cudaDeviceReset): make the first call after a reset before any
 *     stream capture too.
 *   - All calls on a device share the one array, which keeps the last call's
 *     contents; each call clears the parts that must start at zero (barrier
 *     counter, status word, row statistics) before its launch. Calls that
 *     overlap on the GPU (other streams, other threads) race on the array:
 *     serialise them.
 *   - Launch errors come back as return codes; the device-side status word
 *     lives in the array, out of the caller's reach (use ee_flow_sample with
 *     a workspace of your own where that word is needed).
 */
int ee_flow_sample_noalloc(const ee_expert* ex, const void* x_in, const void* t0, void* x_out,
                           int32_t n_steps, int32_t mode, ee_stream_t stream);

/* Synchronises `stream` and copies the workspace status word to *status. */
int ee_read_status(const void* workspace, int32_t* status, ee_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* EE_B200_H */
