/*
 * sas.h -- C ABI of the B200 (sm_100a) sparse shared-KV attention library
 * (libsas.so).  Plain pointers and sizes only; no framework types.
 *
 * Reference interfaces each entry point replaces (file:line in the reference
 * project yangqiang2018/sparse_attn_sharedkv):
 *
 *   sas_fwd / sas_fwd_workspace_size
 *       the device call api.py:372-384 (the TileLang jit function built by
 *       kernel.py:73-183 with the 11-tensor signature kernel.py:356-382) and
 *       its twin sparse_flash_mla/sparse_flash_mla_api.py:231-242; the
 *       runtime-owned workspaces of the reference (workspace_idx) become a
 *       caller-owned buffer sized by sas_fwd_workspace_size.
 *   sas_combine
 *       the split-KV (flash-decode) reduction that the reference plans in
 *       metadata.py:795-827, 925-954 (fdMetadata) but never runs.
 *   sas_metadata
 *       metadata.py:1018-1086 (sparse_attn_sharedkv_metadata), the port of the
 *       aicpu SparseAttnSharedkvMetadata scheduler; bit-exact int32[1024].
 *   sas_plan_size / sas_plan
 *       the B200 work split that takes the place of the 24/36-core metadata
 *       table for 148 SMs (split-KV pieces + combine bookkeeping).
 *   sas_fwd_workspace_size_device / sas_fwd_prepare_device
 *       the same plan built on the GPU from device-resident lengths, in place
 *       of the host reads api.py:210, 260, 336 (no host sync, graph-capturable).
 *   sas_kv_append
 *       the paged-cache writer that precedes the path: appends new key rows
 *       into a [blocks, block_size, 1, D] pool through its block table, in the
 *       layout of the reference's generators golden.py:315-360 (the inverse of
 *       unpack_paged_kv, golden.py:247-268).  The reference has no device
 *       writer: its tests build the caches on the host.
 *   sas_error_string / sas_version
 *       error reporting in place of the reference's Python asserts
 *       (api.py:187-191, 279-282).
 *
 * Conventions: every function returns SAS_OK (0) or a positive SAS_ERR_*
 * code.  Device pointers are marked [device]; everything else is host memory.
 * Streams are passed as `void*` (a cudaStream_t; NULL = legacy default).
 * The library allocates no device memory: outputs and workspace belong to
 * the caller.
 */
#ifndef SAS_H_
#define SAS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
enum {
  SAS_OK = 0,
  SAS_ERR_INVALID = 1,      /* bad argument: shape, mode, null pointer, size   */
  SAS_ERR_UNSUPPORTED = 2,  /* valid in the reference API but not built here   */
  SAS_ERR_CUDA = 3,         /* a CUDA runtime call or kernel launch failed      */
  SAS_ERR_SCHEDULE = 4,     /* the scheduler could not finish (see sas_metadata)*/
  SAS_ERR_WORKSPACE = 5,    /* workspace missing, misaligned or too small       */
  SAS_ERR_DEVICE = 6        /* a device-side check fired (see SasFwdParams.err) */
};

/* ---- layouts / modes / dtypes (values of the reference's string enums) ---- */
enum { SAS_LAYOUT_BSND = 0, SAS_LAYOUT_TND = 1, SAS_LAYOUT_BSH = 2, SAS_LAYOUT_BNSD = 3,
       SAS_LAYOUT_PA_ND = 4 };
enum { SAS_DTYPE_BF16 = 0, SAS_DTYPE_FP16 = 1 };
/* Scenario (api.py:196-202): 1 = SWA, 2 = CFA (dense compressed), 3 = SCFA (top-k). */
enum { SAS_SCENARIO_SWA = 1, SAS_SCENARIO_CFA = 2, SAS_SCENARIO_SCFA = 3 };

/* ---- reference metadata table geometry (metadata.py:38-60) ---- */
#define SAS_META_SIZE 1024
#define SAS_AIC_CORE_NUM 36
#define SAS_AIV_CORE_NUM 72
#define SAS_FA_METADATA_SIZE 8
#define SAS_FD_METADATA_SIZE 8

/* Parameters of sas_metadata: the keyword arguments of
 * sparse_attn_sharedkv_metadata (metadata.py:1018-1045).  Optional tensors are
 * (pointer, length) pairs; length 0 means "None / empty". */
typedef struct SasMetaParams {
  int64_t num_heads_q, num_heads_kv, head_dim;
  const int64_t* cu_seqlens_q;      int64_t n_cu_seqlens_q;
  const int64_t* cu_seqlens_ori_kv; int64_t n_cu_seqlens_ori_kv;
  const int64_t* cu_seqlens_cmp_kv; int64_t n_cu_seqlens_cmp_kv;
  const int64_t* seqused_q;         int64_t n_seqused_q;
  const int64_t* seqused_kv;        int64_t n_seqused_kv;
  int64_t batch_size, max_seqlen_q, max_seqlen_kv;
  int64_t ori_topk, cmp_topk, cmp_ratio;
  int32_t ori_mask_mode, cmp_mask_mode;
  int64_t ori_win_left, ori_win_right;
  int32_t layout_q, layout_kv;      /* SAS_LAYOUT_* */
  int32_t has_ori_kv, has_cmp_kv;
  int64_t aic_core_num, aiv_core_num;
} SasMetaParams;

/* Reference-exact scheduler (host).  Writes SAS_META_SIZE int32 to `out`.
 * Replaces metadata.py:1018-1086. */
int sas_metadata(const SasMetaParams* params, int32_t* out, size_t out_len);

/* ---- forward ---- */

/* Problem description shared by the planner and the forward.  Host arrays. */
typedef struct SasProblem {
  int32_t batch;            /* B                                               */
  int32_t layout_q;         /* SAS_LAYOUT_TND or SAS_LAYOUT_BSND                */
  int32_t max_q_len;        /* S (BSND row stride in tokens); ignored for TND   */
  int32_t total_tokens;     /* rows of q: T (TND) or B*S (BSND)                 */
  const int32_t* q_start;   /* [B] flat token offset of batch b (q_prefix)       */
  const int32_t* q_len;     /* [B] valid query tokens of batch b (act_q)         */
  const int32_t* kv_len;    /* [B] seqused_kv                                    */
  int32_t num_heads;        /* N1 (1..128), one KV head                         */
  int32_t scenario;         /* SAS_SCENARIO_*                                   */
  int32_t ori_win_left;     /* window is [s_g - left, s_g]; -1 = empty window   */
  int32_t cmp_ratio;        /* compression ratio (>= 1) for scenarios 2, 3      */
  int32_t topk;             /* K of cmp_indices (scenario 3)                    */
} SasProblem;

/* Device-side buffers and remaining shapes of one forward call. */
typedef struct SasFwdParams {
  const void* q;                   /* [device] [total_tokens, H, d_qk] dtype      */
  const void* ori_kv;              /* [device] [ori_blocks, ori_bs, 1, d_qk]      */
  const int32_t* ori_block_table;  /* [device] [B, ori_table_len]                 */
  const void* cmp_kv;              /* [device] or NULL (scenario 1)               */
  const int32_t* cmp_block_table;  /* [device] [B, cmp_table_len] or NULL         */
  const int32_t* cmp_indices;      /* [device] [total_tokens, topk] or NULL       */
  const float* sinks;              /* [device] [H] fp32                           */
  void* out;                       /* [device] [total_tokens, H, d_v] dtype       */
  float* lse;                      /* [device] [total_tokens, H] fp32             */
  int32_t* err;                    /* [device] optional int32[4] error record     */
  int32_t head_dim;                /* d_qk: 512 or 576                            */
  int32_t head_dim_v;              /* d_v: 512                                    */
  int32_t dtype;                   /* SAS_DTYPE_*                                 */
  float softmax_scale;
  int32_t ori_block_size, ori_num_blocks, ori_table_len;
  int32_t cmp_block_size, cmp_num_blocks, cmp_table_len;
  int32_t num_sms;                 /* persistent workers (0 = all SMs)            */
  int64_t* trace;                  /* [device] optional int64[4 * 8192] clock trace
                                      of CTA 0 (diagnostics; NULL = off)           */
  int32_t* slot_dump;              /* [device] optional int32[total_tokens,
                                      slot_dump_cap]: the key source each slot of a
                                      query row resolved to (diagnostics; NULL =
                                      off): 2 * pool_row + cache (0 window, 1
                                      compressed), -2 - cache for an attended
                                      position whose page is unmapped (zero row),
                                      -1 for a masked slot; entries not written are
                                      left as they are.  Slot order is window keys
                                      then compressed keys (golden.py tile order);
                                      a ring row (one head group, a 65..128-key
                                      window) uses its ring order instead.        */
  int32_t slot_dump_cap;           /* row stride of slot_dump (slots per token)    */
} SasFwdParams;

/* Plan summary returned by sas_plan (sizes in elements). */
typedef struct SasPlanInfo {
  int32_t num_rows;          /* work rows (query tokens incl. padded BSND rows) */
  int32_t num_workers;       /* persistent workers (CTA groups)                 */
  int32_t head_groups;       /* CTAs per worker = ceil(H / 64)                  */
  int32_t num_split_rows;    /* rows whose keys were split across workers       */
  int32_t num_partials;      /* partial slots used by split rows                */
  int64_t total_tiles;       /* 64-key tiles over all rows                      */
  int64_t plan_ints;         /* int32 entries of the serialised plan            */
  int64_t split_off;         /* plan offset of the split-row section            */
  int64_t actq_off;          /* plan offset of act_q[B]                         */
  int64_t actkv_off;         /* plan offset of act_kv[B]                        */
} SasPlanInfo;

/* Bytes of device workspace a forward call needs (plan + split-KV partials).
 * Host-only; deterministic in (problem, num_sms). */
int sas_fwd_workspace_size(const SasProblem* prob, int32_t num_sms, size_t* bytes);

/* Full forward on `stream`: plans on the host, uploads the plan into the
 * workspace (cudaMemcpyAsync), runs the attention kernel and, when a query
 * row was split across SMs, the LSE-combine kernel.  Replaces api.py:372-384.
 * `workspace` must be 256-byte aligned and at least sas_fwd_workspace_size. */
int sas_fwd(const SasProblem* prob, const SasFwdParams* params, void* workspace,
            size_t workspace_bytes, void* stream);

/* Two-phase form of sas_fwd, for callers that reuse one plan or time the
 * kernels alone.  sas_fwd_prepare plans on the host and uploads the plan into
 * the workspace (stream-ordered); sas_fwd_execute launches, on a prepared
 * workspace, the attention kernel (phases & SAS_PHASE_ATTN) and/or the
 * combine kernel (phases & SAS_PHASE_COMBINE).  sas_fwd = prepare + execute
 * of both phases. */
enum { SAS_PHASE_ATTN = 1, SAS_PHASE_COMBINE = 2, SAS_PHASE_ALL = 3 };
int sas_fwd_prepare(const SasProblem* prob, const SasFwdParams* params, void* workspace,
                    size_t workspace_bytes, void* stream, SasPlanInfo* info);
int sas_fwd_execute(const SasProblem* prob, const SasFwdParams* params, const SasPlanInfo* info,
                    void* workspace, size_t workspace_bytes, void* stream, int32_t phases);

/* Device-planned forward: the same as sas_fwd_prepare, except that
 * prob->q_start, q_len and kv_len are DEVICE pointers ([device] int32[B]) and
 * the work plan is built on the GPU by one small kernel, so the call reads no
 * length on the host (the reference syncs on them, api.py:210, 260, 336) and
 * the prepare + execute launches can be recorded in a CUDA graph and replayed
 * with new lengths of the same shapes.  q_start must be the prefix sums of
 * q_len (TND) or b * max_q_len (BSND).  The plan is the host planner's
 * (same rows, workers, split rows); its sections are sized for the worst
 * case (info->num_split_rows / num_partials are upper bounds), so the
 * workspace comes from sas_fwd_workspace_size_device.  Invalid lengths are
 * reported in params->err (site 60) and leave the call without work.
 * Then sas_fwd_execute as usual. */
int sas_fwd_workspace_size_device(const SasProblem* prob, int32_t num_sms, size_t* bytes);
int sas_fwd_prepare_device(const SasProblem* prob, const SasFwdParams* params, void* workspace,
                           size_t workspace_bytes, void* stream, SasPlanInfo* info);

/* Forward without a caller workspace, for callers that cannot allocate
 * device memory (an arena planned ahead of time, an allocator frozen during a
 * step, a host that forbids allocation after start-up).  No counterpart in
 * the reference: its jit runtime always owns the workspaces.
 * The plan and split-KV partials live in a file-scope device array of
 * SAS_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * exit; a problem needing more returns SAS_ERR_WORKSPACE (fewer workers via
 * params->num_sms shrink the partials).  The array's device address is set
 * up on a device's first call: make that call before any stream capture.
 * Each call builds its work plan on the host and copies it into the array
 * with a stream-ordered copy from host memory before launching the kernels.
 * All calls on a device share the array (it keeps the last call's contents;
 * nothing in it needs to start at zero), so calls that overlap on the GPU
 * race: serialise them.  Makes no device allocation. */
#define SAS_NOALLOC_SCRATCH_BYTES (16u << 20)
int sas_fwd_noalloc(const SasProblem* prob, const SasFwdParams* params, void* stream);

/* LSE-combine of split-KV partials (normally called by sas_fwd).  For each of
 * `num_rows` split rows, piece i of row r is partial slot `partial_base[r]+i`:
 * o_partial [slots, H, d_v] fp32 (normalised), lse_partial [slots, H] fp32.
 * Writes out [token, H, d_v] dtype and lse [token, H].  All pointers device. */
int sas_combine(const int32_t* row_token, const int32_t* row_pieces,
                const int32_t* partial_base, int32_t num_rows, const float* o_partial,
                const float* lse_partial, int32_t num_heads, int32_t head_dim_v, int32_t dtype,
                void* out, float* lse, void* stream);

/* ---- paged-cache writer ---- */

/* Append new key rows into a paged cache, in place: batch b writes its rows
 * rows[cu_new[b] .. cu_new[b+1]) at logical positions start_pos[b] + i, i.e.
 * at pool[block_table[b, p / block_size], p % block_size].  pool [device]
 * [num_blocks, block_size, 1, row_bytes / 2]; rows [device] [total_new,
 * row_bytes / 2] (any 16-bit dtype: the writer copies bytes); block_table
 * [device] [batch, table_len] int32; cu_new [device] [batch + 1] int32;
 * start_pos [device] [batch] int32 (usually the lengths before the append).
 * row_bytes a multiple of 16, pool and rows 16-byte aligned.  A row whose
 * position is past the table or whose page is -1 / outside the pool is
 * skipped and recorded in the optional err word [device] int32[4] (site 50,
 * detail = row index).  Stream-ordered, no allocation. */
int sas_kv_append(void* pool, int32_t num_blocks, int32_t block_size, int32_t row_bytes,
                  const int32_t* block_table, int32_t table_len, const void* rows,
                  const int32_t* cu_new, const int32_t* start_pos, int32_t batch,
                  int32_t total_new, int32_t* err, void* stream);

/* ---- B200 work plan (host) ---- */


/* Size the plan (host). */
int sas_plan_size(const SasProblem* prob, int32_t num_sms, SasPlanInfo* info);
/* Build the plan into `plan` (host int32[info.plan_ints]). */
int sas_plan(const SasProblem* prob, int32_t num_sms, int32_t* plan, int64_t plan_len,
             SasPlanInfo* info);

/* ---- misc ---- */
const char* sas_error_string(int code);
const char* sas_version(void);
/* Number of SMs of the current device (0 if no device). */
int32_t sas_device_sm_count(void);

#ifdef __cplusplus
}
#endif

#endif /* SAS_H_ */
