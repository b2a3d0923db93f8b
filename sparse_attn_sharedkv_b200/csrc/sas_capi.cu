// C ABI of libsas.so: argument validation, planning, workspace layout and
// kernel launches.  The library never allocates device memory: the caller
// passes outputs and a workspace sized by sas_fwd_workspace_size.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <cstring>
#include <vector>

#include "sas.h"
#include "sas_internal.h"
#include "sas_kernels.h"

namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct WorkspaceLayout {
  size_t plan_off, plan_bytes;
  size_t opart_off, opart_bytes;
  size_t lpart_off, lpart_bytes;
  size_t total;
};

WorkspaceLayout layout_for(const SasPlanInfo& info, int32_t num_heads, int32_t head_dim_v) {
  WorkspaceLayout w{};
  w.plan_off = 0;
  w.plan_bytes = align_up((size_t)info.plan_ints * sizeof(int32_t));
  w.opart_off = w.plan_off + w.plan_bytes;
  w.opart_bytes = align_up((size_t)info.num_partials * num_heads * head_dim_v * sizeof(float));
  w.lpart_off = w.opart_off + w.opart_bytes;
  w.lpart_bytes = align_up((size_t)info.num_partials * num_heads * sizeof(float));
  w.total = w.lpart_off + w.lpart_bytes;
  return w;
}

int resolve_sms(int32_t requested) {
  if (requested > 0) return requested;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate(const SasProblem& p, const SasFwdParams& f) {
  if (!f.q || !f.ori_kv || !f.ori_block_table || !f.sinks || !f.out || !f.lse)
    return SAS_ERR_INVALID;
  if (f.head_dim != 512 && f.head_dim != 576) return SAS_ERR_UNSUPPORTED;
  if (f.head_dim_v != 512) return SAS_ERR_UNSUPPORTED;
  if (f.dtype != SAS_DTYPE_BF16 && f.dtype != SAS_DTYPE_FP16) return SAS_ERR_UNSUPPORTED;
  if (p.num_heads < 1 || p.num_heads > sas::kHeadsPerCta * sas::kMaxHeadGroups)
    return SAS_ERR_UNSUPPORTED;
  if (f.ori_block_size <= 0 || f.ori_num_blocks <= 0 || f.ori_table_len <= 0)
    return SAS_ERR_INVALID;
  if (!aligned16(f.q) || !aligned16(f.ori_kv) || !aligned16(f.out)) return SAS_ERR_INVALID;
  if (p.scenario >= SAS_SCENARIO_CFA) {
    if (!f.cmp_kv || !f.cmp_block_table || f.cmp_block_size <= 0 || f.cmp_num_blocks <= 0 ||
        f.cmp_table_len <= 0 || !aligned16(f.cmp_kv))
      return SAS_ERR_INVALID;
  }
  if (p.scenario == SAS_SCENARIO_SCFA && (!f.cmp_indices || p.topk <= 0)) return SAS_ERR_INVALID;
  if (!(f.softmax_scale == f.softmax_scale)) return SAS_ERR_INVALID;  // NaN
  return SAS_OK;
}

}  // namespace

extern "C" int sas_fwd_workspace_size(const SasProblem* prob, int32_t num_sms, size_t* bytes) {
  if (!prob || !bytes) return SAS_ERR_INVALID;
  const int sms = resolve_sms(num_sms);
  if (sms <= 0) return SAS_ERR_CUDA;
  SasPlanInfo info;
  int rc = sas_plan_size(prob, sms, &info);
  if (rc != SAS_OK) return rc;
  *bytes = layout_for(info, prob->num_heads, 512).total;
  return SAS_OK;
}

extern "C" int sas_fwd_prepare(const SasProblem* prob, const SasFwdParams* params,
                               void* workspace, size_t workspace_bytes, void* stream_ptr,
                               SasPlanInfo* info_out) {
  if (!prob || !params || !info_out) return SAS_ERR_INVALID;
  int rc = validate(*prob, *params);
  if (rc != SAS_OK) return rc;
  const int sms = resolve_sms(params->num_sms);
  if (sms <= 0) return SAS_ERR_CUDA;
  std::vector<int32_t> plan;
  SasPlanInfo info;
  rc = sas::plan_build(*prob, sms, &plan, &info);
  if (rc != SAS_OK) return rc;
  *info_out = info;
  if (info.num_rows == 0) return SAS_OK;
  const WorkspaceLayout wl = layout_for(info, prob->num_heads, params->head_dim_v);
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0 ||
      workspace_bytes < wl.total)
    return SAS_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  if (cudaMemcpyAsync(ws + wl.plan_off, plan.data(), plan.size() * sizeof(int32_t),
                      cudaMemcpyHostToDevice,
                      reinterpret_cast<cudaStream_t>(stream_ptr)) != cudaSuccess)
    return SAS_ERR_CUDA;
  return SAS_OK;
}

extern "C" int sas_fwd_workspace_size_device(const SasProblem* prob, int32_t num_sms,
                                             size_t* bytes) {
  if (!prob || !bytes) return SAS_ERR_INVALID;
  const int sms = resolve_sms(num_sms);
  if (sms <= 0) return SAS_ERR_CUDA;
  SasPlanInfo info;
  int rc = sas::plan_dev_info(*prob, sms, &info);
  if (rc != SAS_OK) return rc;
  *bytes = layout_for(info, prob->num_heads, 512).total;
  return SAS_OK;
}

extern "C" int sas_fwd_prepare_device(const SasProblem* prob, const SasFwdParams* params,
                                      void* workspace, size_t workspace_bytes,
                                      void* stream_ptr, SasPlanInfo* info_out) {
  if (!prob || !params || !info_out) return SAS_ERR_INVALID;
  int rc = validate(*prob, *params);
  if (rc != SAS_OK) return rc;
  if (!prob->q_start || !prob->q_len || !prob->kv_len) return SAS_ERR_INVALID;
  const int sms = resolve_sms(params->num_sms);
  if (sms <= 0) return SAS_ERR_CUDA;
  SasPlanInfo info;
  rc = sas::plan_dev_info(*prob, sms, &info);
  if (rc != SAS_OK) return rc;
  *info_out = info;
  if (info.num_rows == 0) return SAS_OK;
  const WorkspaceLayout wl = layout_for(info, prob->num_heads, params->head_dim_v);
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0 ||
      workspace_bytes < wl.total)
    return SAS_ERR_WORKSPACE;
  return sas::plan_dev_launch(*prob, info,
                              reinterpret_cast<int32_t*>(static_cast<char*>(workspace) +
                                                         wl.plan_off),
                              params->err, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" int sas_fwd_execute(const SasProblem* prob, const SasFwdParams* params,
                               const SasPlanInfo* info_ptr, void* workspace,
                               size_t workspace_bytes, void* stream_ptr, int32_t phases) {
  if (!prob || !params || !info_ptr) return SAS_ERR_INVALID;
  const SasProblem& p = *prob;
  const SasFwdParams& f = *params;
  const SasPlanInfo& info = *info_ptr;
  if (info.num_rows == 0) return SAS_OK;
  const WorkspaceLayout wl = layout_for(info, p.num_heads, f.head_dim_v);
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0 ||
      workspace_bytes < wl.total)
    return SAS_ERR_WORKSPACE;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  char* ws = static_cast<char*>(workspace);
  const int32_t* dplan = reinterpret_cast<const int32_t*>(ws + wl.plan_off);

  sas::FwdArgs a{};
  a.q = f.q;
  a.ori_kv = f.ori_kv;
  a.ori_block_table = f.ori_block_table;
  a.cmp_kv = f.cmp_kv;
  a.cmp_block_table = f.cmp_block_table;
  a.cmp_indices = f.cmp_indices;
  a.sinks = f.sinks;
  a.out = f.out;
  a.lse = f.lse;
  a.err = f.err;
  a.trace = reinterpret_cast<long long*>(f.trace);
  a.trace_cta = 0;
  if (f.trace != nullptr) {
    const char* e = getenv("SAS_TRACE_CTA");
    a.trace_cta = e != nullptr ? atoi(e) : 0;
  }
  a.plan = dplan;
  a.q_len = dplan + info.actq_off;
  a.kv_len = dplan + info.actkv_off;
  a.o_partial = reinterpret_cast<float*>(ws + wl.opart_off);
  a.lse_partial = reinterpret_cast<float*>(ws + wl.lpart_off);
  a.num_heads = p.num_heads;
  a.head_dim = f.head_dim;
  a.head_dim_v = f.head_dim_v;
  a.dtype = f.dtype;
  a.softmax_scale = f.softmax_scale;
  a.scenario = p.scenario;
  a.ori_win_left = p.ori_win_left;
  a.cmp_ratio = p.cmp_ratio;
  a.topk = p.topk;
  a.ori_block_size = f.ori_block_size;
  a.ori_num_blocks = f.ori_num_blocks;
  a.ori_table_len = f.ori_table_len;
  a.cmp_block_size = f.cmp_block_size > 0 ? f.cmp_block_size : 1;
  a.cmp_num_blocks = f.cmp_num_blocks;
  a.cmp_table_len = f.cmp_table_len;
  a.head_groups = info.head_groups;
  a.total_tokens = p.total_tokens;
  a.ori_rows = f.ori_num_blocks * f.ori_block_size;
  a.cmp_rows = f.cmp_kv ? f.cmp_num_blocks * a.cmp_block_size : 0;
  {
    // Key-row gather engine: TMA tile::gather4 from the four producer warps
    // (default) or cp.async 16 B (SAS_GATHER=lsu), read at each call.
    const char* e = getenv("SAS_GATHER");
    a.gather = (e != nullptr && strcmp(e, "lsu") == 0) ? 0 : 1;
  }
  a.slot_dump = f.slot_dump;
  a.slot_dump_cap = f.slot_dump != nullptr ? f.slot_dump_cap : 0;
  int rc = SAS_OK;
  if (phases & SAS_PHASE_ATTN) {
    // Two head groups (65..128 heads) run on CTA pairs issuing cta_group::2
    // MMAs over 128-key tiles, or on one CTA per 64-head group with
    // SAS_FWD_KERNEL=single or in the cp.async gather mode (read at each
    // call).
    const char* ek = getenv("SAS_FWD_KERNEL");
    const bool single = (ek != nullptr && strcmp(ek, "single") == 0) || a.gather == 0;
    if (info.head_groups == 2 && !single)
      rc = sas::launch_fwd_pair(a, info.num_workers, stream);
    else
      rc = sas::launch_fwd(a, info.num_workers * info.head_groups, stream);
    if (rc != SAS_OK) return rc;
  }
  if ((phases & SAS_PHASE_COMBINE) && info.num_split_rows > 0) {
    const int32_t* split = dplan + info.split_off;
    rc = sas::launch_combine(split, split + 1, split + 2, 4, info.num_split_rows, a.o_partial,
                             a.lse_partial, p.num_heads, f.head_dim_v, f.dtype, f.out, f.lse,
                             stream);
  }
  return rc;
}

extern "C" int sas_fwd(const SasProblem* prob, const SasFwdParams* params, void* workspace,
                       size_t workspace_bytes, void* stream) {
  SasPlanInfo info;
  int rc = sas_fwd_prepare(prob, params, workspace, workspace_bytes, stream, &info);
  if (rc != SAS_OK) return rc;
  return sas_fwd_execute(prob, params, &info, workspace, workspace_bytes, stream, SAS_PHASE_ALL);
}

extern "C" int sas_combine(const int32_t* row_token, const int32_t* row_pieces,
                           const int32_t* partial_base, int32_t num_rows, const float* o_partial,
                           const float* lse_partial, int32_t num_heads, int32_t head_dim_v,
                           int32_t dtype, void* out, float* lse, void* stream) {
  if (num_rows < 0 || num_heads <= 0) return SAS_ERR_INVALID;
  if (num_rows == 0) return SAS_OK;
  if (!row_token || !row_pieces || !partial_base || !o_partial || !lse_partial || !out || !lse)
    return SAS_ERR_INVALID;
  if (dtype != SAS_DTYPE_BF16 && dtype != SAS_DTYPE_FP16) return SAS_ERR_UNSUPPORTED;
  return sas::launch_combine(row_token, row_pieces, partial_base, 1, num_rows, o_partial,
                             lse_partial, num_heads, head_dim_v, dtype, out, lse,
                             reinterpret_cast<cudaStream_t>(stream));
}

extern "C" const char* sas_error_string(int code) {
  switch (code) {
    case SAS_OK: return "ok";
    case SAS_ERR_INVALID: return "invalid argument";
    case SAS_ERR_UNSUPPORTED: return "unsupported configuration";
    case SAS_ERR_CUDA: return "CUDA runtime error";
    case SAS_ERR_SCHEDULE: return "scheduler did not converge";
    case SAS_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case SAS_ERR_DEVICE: return "device-side check failed";
    default: return "unknown error";
  }
}

extern "C" const char* sas_version(void) { return "sparse_attn_sharedkv_b200 0.1 sm_100a"; }

extern "C" int32_t sas_device_sm_count(void) { return resolve_sms(0); }
