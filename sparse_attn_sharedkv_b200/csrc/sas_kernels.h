// Kernel-side argument blocks and launchers (internal to libsas.so).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "sas.h"

namespace sas {

struct FwdArgs {
  const void* q;
  const void* ori_kv;
  const int32_t* ori_block_table;
  const void* cmp_kv;
  const int32_t* cmp_block_table;
  const int32_t* cmp_indices;
  const float* sinks;
  void* out;
  float* lse;
  int32_t* err;
  long long* trace;         // optional clock trace of one CTA (diagnostics)
  int32_t trace_cta;        // CTA traced (SAS_TRACE_CTA, default 0)
  const int32_t* plan;      // device copy of the serialised plan
  const int32_t* q_len;     // [B] device (act_q per batch)
  const int32_t* kv_len;    // [B] device (seqused_kv)
  float* o_partial;         // [partials, H, d_v] fp32
  float* lse_partial;       // [partials, H] fp32
  int32_t num_heads, head_dim, head_dim_v, dtype;
  float softmax_scale;
  int32_t scenario, ori_win_left, cmp_ratio, topk;
  int32_t ori_block_size, ori_num_blocks, ori_table_len;
  int32_t cmp_block_size, cmp_num_blocks, cmp_table_len;
  int32_t head_groups;
  int32_t total_tokens;     // rows of q (for the Q tensor map)
  int32_t ori_rows;         // ori_num_blocks * ori_block_size (out-of-range row = zero fill)
  int32_t cmp_rows;         // cmp_num_blocks * cmp_block_size
  int32_t gather;           // key-row gather: 0 = cp.async (LSU), 1 = TMA gather4 (default)
  int32_t* slot_dump;       // optional [total_tokens, slot_dump_cap] resolved key sources
  int32_t slot_dump_cap;
};

int launch_fwd(const FwdArgs& args, int grid, cudaStream_t stream);
int launch_fwd_pair(const FwdArgs& args, int workers, cudaStream_t stream);

int launch_combine(const int32_t* row_token, const int32_t* row_pieces, const int32_t* row_base,
                   int stride, int n, const float* o_partial, const float* lse_partial, int num_heads,
                   int head_dim_v, int dtype, void* out, float* lse, cudaStream_t stream);

int plan_dev_info(const SasProblem& p, int32_t num_sms, SasPlanInfo* info);
int plan_dev_launch(const SasProblem& p, const SasPlanInfo& info, int32_t* dplan, int32_t* err,
                    cudaStream_t stream);
int plan_build(const SasProblem& p, int32_t num_sms, std::vector<int32_t>* plan,
               SasPlanInfo* info);

}  // namespace sas
