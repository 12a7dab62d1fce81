// ee_sampler.cu -- C ABI of the fused sampler (kernels in ee_sampler.cuh,
// instantiated per activation dtype / head size in ee_sampler_<dtype>_<hd>.cu).
#include <vector>

#include "ee_sampler.cuh"

namespace ee {
extern template int launch_sampler<__nv_bfloat16, 64>(Ctx, cudaStream_t);
extern template int launch_sampler<__nv_bfloat16, 128>(Ctx, cudaStream_t);
extern template int launch_sampler<__half, 64>(Ctx, cudaStream_t);
extern template int launch_sampler<__half, 128>(Ctx, cudaStream_t);
extern template int sampler_geometry<__nv_bfloat16, 64>(const Ctx&, int*, int*, size_t*);
extern template int sampler_geometry<__nv_bfloat16, 128>(const Ctx&, int*, int*, size_t*);
extern template int sampler_geometry<__half, 64>(const Ctx&, int*, int*, size_t*);
extern template int sampler_geometry<__half, 128>(const Ctx&, int*, int*, size_t*);

// Self-test of the bounded grid barrier: CTA 1 leaves without arriving, so
// CTA 0's wait can only end by its time limit.
__global__ void barrier_selftest_kernel(unsigned* bar, int* abort_flag, int* status,
                                        unsigned long long timeout_ns) {
  if (blockIdx.x != 0) return;
  grid_barrier(bar, abort_flag, status, timeout_ns, 2u);
}

}  // namespace ee

using namespace ee;

extern "C" {

int ee_check_expert(const ee_expert* ex, const ee_block* host_blocks, int32_t n_steps, int32_t mode) {
  if (!ex || !host_blocks) return EE_ERR_ARG;
  int rc = validate_expert(*ex, n_steps, mode);
  if (rc) return rc;
  return validate_blocks(*ex, host_blocks);
}

int ee_encode_kv_maps(const ee_expert* ex, const ee_block* host_blocks, void* maps, size_t maps_bytes,
                      ee_stream_t stream) {
  if (!ex || !host_blocks || !maps) return EE_ERR_ARG;
  if (ex->n_layers < 1 || ex->n_heads < 1 || ex->batch < 1 || ex->prefix_len < 1) return EE_ERR_SHAPE;
  if (ex->d_model % ex->n_heads || ex->d_model / ex->n_heads != 64) return EE_ERR_UNSUPPORTED;
  if (maps_bytes < (size_t)ex->n_layers * sizeof(CUtensorMap)) return EE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(maps) & 63) return EE_ERR_ALIGN;
  int rc = check_device();
  if (rc) return rc;
  std::vector<CUtensorMap> h((size_t)ex->n_layers);
  const uint64_t cols = 2 * (uint64_t)ex->d_model, rows = (uint64_t)ex->batch * ex->prefix_len;
  for (int l = 0; l < ex->n_layers; ++l) {
    if (!host_blocks[l].kv) return EE_ERR_ARG;
    if (!make_tmap_2d(&h[l], host_blocks[l].kv, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, cols, rows, cols * 2, 64, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return EE_ERR_ALIGN;
  }
  if (cudaMemcpyAsync(maps, h.data(), h.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice,
                      (cudaStream_t)stream) != cudaSuccess)
    return EE_ERR_LAUNCH;
  // pageable source: the copy has been staged when the call returns
  return EE_OK;
}

size_t ee_flow_sample_workspace_bytes(const ee_expert* ex, int32_t n_steps) {
  if (!ex || n_steps < 1) return 0;
  return layout_for(*ex, n_steps).total;
}

int ee_flow_sample(const ee_expert* exp, const void* x_in, const void* t0, void* x_out,
                   int32_t n_steps, int32_t mode, void* workspace, size_t workspace_bytes,
                   ee_stream_t stream) {
  return ee_flow_sample_traced(exp, x_in, t0, x_out, n_steps, mode, workspace, workspace_bytes,
                               nullptr, stream);
}

int32_t ee_flow_sample_phases(const ee_expert* ex, int32_t n_steps) {
  if (!ex || n_steps < 1 || ex->n_layers < 1) return 0;
  return 3 + n_steps * (ex->n_layers * (ex->self_attn ? 8 : 5) + 1);
}

int ee_flow_sample_traced(const ee_expert* exp, const void* x_in, const void* t0, void* x_out,
                          int32_t n_steps, int32_t mode, void* workspace, size_t workspace_bytes,
                          uint64_t* trace, ee_stream_t stream) {
  if (!exp || !x_in || !x_out) return EE_ERR_ARG;
  const ee_expert& ex = *exp;
  int rc = validate_expert(ex, n_steps, mode);
  if (rc) return rc;
  if (!aligned16(x_in) || !aligned16(x_out) || (t0 && !aligned16(t0))) return EE_ERR_ALIGN;
  const Layout L = layout_for(ex, n_steps);
  if (!workspace || workspace_bytes < L.total) return EE_ERR_WORKSPACE;
  if (!aligned16(workspace)) return EE_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;

  char* ws = reinterpret_cast<char*>(workspace);
  Ctx c{};
  c.ex = ex;
  c.x_in = x_in;
  c.t0 = t0;
  c.x_out = x_out;
  c.n_steps = n_steps;
  c.mode = mode;
  c.M = L.M;
  c.nbt = t0 ? ex.batch : 1;
  c.Rt = n_steps * c.nbt;
  c.dtf = (float)(1.0 / (double)n_steps);
  c.timeout_ns = 1000000000ull;  // 1 s per barrier wait
  c.bar = reinterpret_cast<unsigned*>(ws + L.sync);
  c.abort_flag = reinterpret_cast<int*>(ws + L.sync + 4);
  c.status = reinterpret_cast<int*>(ws + L.sync + 8);
  c.stats = reinterpret_cast<float*>(ws + L.stats);
  c.n_inst = L.n_inst;
  c.n_slots = L.n_slots;
  c.ks_cap = sampler_ks_cap(ex);
  c.x = ws + L.x;
  c.qkv = ws + L.qkv;
  c.att = ws + L.att;
  c.qb = ws + L.qb;
  c.hid = ws + L.hid;
  c.emb = ws + L.emb;
  c.temb = ws + L.temb;
  {
    const SamplerSmem sm = sampler_smem_map(ex, device_props()->smem_optin);
    c.sm = sm.g;
    c.desc = sm.desc;
    c.smem_bytes = sm.total;
  }
  c.trace = reinterpret_cast<unsigned long long*>(trace);

  cudaStream_t s = (cudaStream_t)stream;
  if (cudaMemsetAsync(ws, 0, L.x, s) != cudaSuccess) return EE_ERR_LAUNCH;
  const int hd = ex.d_model / ex.n_heads;
  if (ex.act_dtype == EE_BF16)
    return hd == 64 ? launch_sampler<__nv_bfloat16, 64>(c, s) : launch_sampler<__nv_bfloat16, 128>(c, s);
  return hd == 64 ? launch_sampler<__half, 64>(c, s) : launch_sampler<__half, 128>(c, s);
}

int ee_flow_sample_geometry(const ee_expert* exp, int32_t* grid_ctas, int32_t* cluster,
                            size_t* smem_bytes) {
  if (!exp || !grid_ctas || !cluster || !smem_bytes) return EE_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  Ctx c{};
  c.ex = *exp;
  c.M = c.ex.batch * c.ex.horizon;
  c.Rt = c.ex.batch;
  c.ks_cap = sampler_ks_cap(c.ex);
  {
    const SamplerSmem sm = sampler_smem_map(c.ex, device_props()->smem_optin);
    c.sm = sm.g;
    c.desc = sm.desc;
    c.smem_bytes = sm.total;
  }
  int g = 0, cl = 0;
  size_t sm = 0;
  const int hd = c.ex.d_model / (c.ex.n_heads > 0 ? c.ex.n_heads : 1);
  if (c.ex.act_dtype == EE_BF16)
    rc = hd == 64 ? sampler_geometry<__nv_bfloat16, 64>(c, &g, &cl, &sm)
                  : sampler_geometry<__nv_bfloat16, 128>(c, &g, &cl, &sm);
  else
    rc = hd == 64 ? sampler_geometry<__half, 64>(c, &g, &cl, &sm)
                  : sampler_geometry<__half, 128>(c, &g, &cl, &sm);
  *grid_ctas = g;
  *cluster = cl;
  *smem_bytes = sm;
  return rc;
}

int ee_read_status(const void* workspace, int32_t* status, ee_stream_t stream) {
  if (!workspace || !status) return EE_ERR_ARG;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return EE_ERR_LAUNCH;
  int32_t v = 0;
  if (cudaMemcpy(&v, reinterpret_cast<const char*>(workspace) + 8, 4, cudaMemcpyDeviceToHost) !=
      cudaSuccess)
    return EE_ERR_LAUNCH;
  *status = v;
  return EE_OK;
}

const char* ee_strerror(int code) {
  switch (code) {
    case EE_OK: return "ok";
    case EE_ERR_ARG: return "invalid argument (null pointer or bad enum)";
    case EE_ERR_SHAPE: return "unsupported or inconsistent shape";
    case EE_ERR_ALIGN: return "pointer not 16-byte aligned";
    case EE_ERR_DTYPE: return "unsupported dtype";
    case EE_ERR_WORKSPACE: return "workspace missing or too small";
    case EE_ERR_LAUNCH: return "CUDA launch or runtime error";
    case EE_ERR_TIMEOUT: return "device-side wait timed out";
    case EE_ERR_DEVICE: return "no sm_100 CUDA device";
    case EE_ERR_UNSUPPORTED: return "configuration not supported by this build";
  }
  return "unknown error";
}

int ee_version(void) { return 1; }

int ee_barrier_selftest(void* workspace, uint64_t timeout_ns, ee_stream_t stream) {
  if (!workspace) return EE_ERR_ARG;
  if (timeout_ns == 0 || timeout_ns > 2000000000ull) return EE_ERR_ARG;
  int rc = check_device();
  if (rc) return rc;
  char* ws = reinterpret_cast<char*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  if (cudaMemsetAsync(ws, 0, 16, s) != cudaSuccess) return EE_ERR_LAUNCH;
  barrier_selftest_kernel<<<2, kThreads, 0, s>>>(reinterpret_cast<unsigned*>(ws), reinterpret_cast<int*>(ws + 4),
                                                 reinterpret_cast<int*>(ws + 8), timeout_ns);
  return cudaGetLastError() == cudaSuccess ? EE_OK : EE_ERR_LAUNCH;
}

size_t ee_struct_size(int32_t which) {
  switch (which) {
    case 0: return sizeof(ee_linear);
    case 1: return sizeof(ee_norm);
    case 2: return sizeof(ee_block);
    case 3: return sizeof(ee_expert);
  }
  return 0;
}

}  // extern "C"
