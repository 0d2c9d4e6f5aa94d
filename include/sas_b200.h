/*
 * C ABI of the B200 (sm_100a) sparse_attn_sharedkv library (libsas_b200.so).
 *
 * Plain pointers and sizes only. All tensor pointers are DEVICE pointers on
 * the current CUDA device; `stream` is a cudaStream_t passed as void*. The
 * library never allocates: every call that needs scratch takes a caller-owned
 * `workspace` whose size the matching *_workspace_bytes() function returns.
 * Calls keep no state between them (apart from the process-wide options of
 * sas_fwd_set_option and the fixed scratch of sas_metadata_noalloc); all work
 * is enqueued on `stream` and no call synchronises the host with the device.
 *
 * Return values are host-side argument/launch checks (SAS_OK or an SAS_ERR_*
 * code). Conditions only the device can see (a scheduler overrun, a bounded
 * wait that ran out) are written to the caller's device `status` word, which
 * must be zeroed before the call and is read back whenever convenient.
 */
#ifndef SAS_B200_H_
#define SAS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SAS_OK 0
#define SAS_ERR_INVALID_ARG 1    /* shape / value outside the documented contract */
#define SAS_ERR_UNSUPPORTED 2    /* valid for the reference API, not implemented here */
#define SAS_ERR_CUDA 3           /* a CUDA runtime call or launch failed */
#define SAS_ERR_WORKSPACE 4      /* workspace missing or smaller than required */
#define SAS_ERR_SCHED_OVERRUN 5  /* device status: scheduler row scan hit its cap */
#define SAS_ERR_NOALLOC_LIMIT 6  /* request exceeds the fixed scratch of sas_metadata_noalloc */
#define SAS_ERR_BAD_BLOCK_ENTRY 7 /* device status, non-fatal: a block-table column past the table's width
                                     (seqused_kv longer than the table) or an entry >= the pool's block
                                     count was met; those rows were dropped like -1 entries */
#define SAS_ERR_TIMEOUT_BASE 16  /* device status: 16 + id of the bounded wait that ran out */

#define SAS_META_SIZE 1024
#define SAS_AIC_CORE_NUM 36

/* layout codes (layout_q / layout_kv) */
#define SAS_LAYOUT_BSND 0
#define SAS_LAYOUT_TND 1
#define SAS_LAYOUT_BSH 2
#define SAS_LAYOUT_PA_ND 0

/* dtype codes */
#define SAS_DTYPE_BF16 0
#define SAS_DTYPE_FP16 1

/* stage_mask bits of sas_sparse_attn_sharedkv_fwd (SAS_STAGE_ALL for a normal call) */
#define SAS_STAGE_PLAN 1
#define SAS_STAGE_ATTENTION 2
#define SAS_STAGE_COMBINE 4 /* the split-KV merge runs inside the attention launch; kept for callers, no launch */
#define SAS_STAGE_ALL 7
/* Flag for stage_mask: the kernel enqueued just before this call on the same
 * stream is sas_metadata for the same arguments. The attention launch may then
 * start before that kernel ends (it reads the metadata only when it writes a
 * token's output), overlapping the scheduler with the attention work. Never
 * set it when another kernel may run in between (for example the producer of
 * q): the attention kernel would read its inputs too early. The two calls
 * must use separate workspaces, since they may run at the same time. */
#define SAS_FLAG_AFTER_METADATA 8

/* Library version, for a loader to check it got the build it expects. */
int sas_version(void);

/* ------------------------------------------------------------------------
 * Scheduler: SparseAttnSharedkvMetadata.
 * Replaces sparse_attn_sharedkv_tilelang/metadata.py:1018-1086
 * (sparse_attn_sharedkv_metadata, the Python port of the AICPU kernel) with a
 * single-CTA GPU kernel whose int32[1024] output is bit-identical:
 * faMetadata[36][8] = (enable, bn2_start, m_start, s2_start, bn2_end, m_end,
 * s2_end, first_fd_workspace_idx) followed by fdMetadata[72][8] (all zero,
 * as supportFd is false in the reference, metadata.py:323-325).
 * Optional arrays are passed as NULL with count 0, matching the reference's
 * "empty tensor" convention (metadata.py:331-341, 345-357, 393-407).
 * ---------------------------------------------------------------------- */
size_t sas_metadata_workspace_bytes(int32_t batch_size, int32_t aic_core_num);

int sas_metadata(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q,
                 const int32_t* cu_seqlens_ori_kv, int32_t n_cu_seqlens_ori_kv,
                 const int32_t* seqused_q, int32_t n_seqused_q,
                 const int32_t* seqused_kv, int32_t n_seqused_kv,
                 int32_t batch_size, int32_t max_seqlen_q, int32_t max_seqlen_kv,
                 int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                 int32_t cmp_topk, int32_t cmp_ratio, int32_t ori_mask_mode, int32_t ori_win_left,
                 int32_t layout_q, int32_t layout_kv, int32_t has_cmp_kv, int32_t aic_core_num,
                 int32_t* metadata_out, int32_t* status,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Flash-decode schedule: the same scheduler with the reference's supportFd
 * switch on (sparse_attn_sharedkv_tilelang/metadata.py:323-325, which the
 * reference declares and leaves False). Replaces the supportFd branches of
 * metadata.py:777-870 (a core may end inside a row, AssignByBlock /
 * ForceAssign; rows cut between cores become flash-decode heads) and
 * 925-954 (the heads spread over aiv_core_num vector cores). fdMetadata[72][8]
 * = (enable, bn2_idx, m_idx, workspace_idx, workspace_num, m_start, m_num, 0)
 * per vector core. Same arguments, workspace and bit-exact contract as
 * sas_metadata plus aiv_core_num (metadata.py:1043, default 48); the forward
 * kernel accepts either schedule (it reads the per-core (bn2, m) windows). */
int sas_metadata_fd(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q,
                    const int32_t* cu_seqlens_ori_kv, int32_t n_cu_seqlens_ori_kv,
                    const int32_t* seqused_q, int32_t n_seqused_q,
                    const int32_t* seqused_kv, int32_t n_seqused_kv,
                    int32_t batch_size, int32_t max_seqlen_q, int32_t max_seqlen_kv,
                    int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                    int32_t cmp_topk, int32_t cmp_ratio, int32_t ori_mask_mode, int32_t ori_win_left,
                    int32_t layout_q, int32_t layout_kv, int32_t has_cmp_kv, int32_t aic_core_num,
                    int32_t aiv_core_num, int32_t* metadata_out, int32_t* status,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of sas_metadata. No counterpart in the reference.
 * For callers that cannot allocate device memory when they need a schedule
 * (code running inside an allocator or teardown path, plugins whose host owns
 * all device memory, loops that must not synchronise): the scheduler's
 * scratch is a fixed device array inside this library (296,704 bytes, held by
 * every GPU that loads the library until the process exits), so no workspace
 * is passed and nothing is allocated. Limits: batch <= 4096 requests and
 * aic_core_num <= 64; larger requests return SAS_ERR_NOALLOC_LIMIT. The first
 * call on a device looks up the array's device address; make that first call
 * before any stream capture. All calls share the one array, so calls whose
 * executions overlap on the GPU (different streams, or different host threads)
 * race and must be serialised by the caller. Same arguments and output as
 * sas_metadata otherwise. */
int sas_metadata_noalloc(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q,
                         const int32_t* cu_seqlens_ori_kv, int32_t n_cu_seqlens_ori_kv,
                         const int32_t* seqused_q, int32_t n_seqused_q,
                         const int32_t* seqused_kv, int32_t n_seqused_kv,
                         int32_t batch_size, int32_t max_seqlen_q, int32_t max_seqlen_kv,
                         int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                         int32_t cmp_topk, int32_t cmp_ratio, int32_t ori_mask_mode, int32_t ori_win_left,
                         int32_t layout_q, int32_t layout_kv, int32_t has_cmp_kv, int32_t aic_core_num,
                         int32_t* metadata_out, int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Forward: the fused sparse shared-KV attention.
 * Replaces the device half of sparse_attn_sharedkv_tilelang/api.py:129-397
 * (the JIT kernel of kernel.py:56-1745 and its launch at api.py:372-384):
 * one or two launches on `stream`. Above 512 query tokens a single-CTA plan
 * kernel first walks the metadata's per-core (bn2, m) windows
 * (kernel.py:254-278) and lays out every token's softmax tiles; at or below
 * 512 tokens every attention CTA builds that plan in its own shared memory and
 * applies the metadata's coverage when it writes a token. The second launch
 * is the fused gather + tcgen05 attention kernel. Tokens are never split
 * across CTAs by default; with SAS_OPT_SPLIT_TOKENS the split-KV merge of a
 * cut token runs inside the attention launch (no combine kernel).
 *
 *   q            [num_tokens, num_heads, 512] (TND) or [batch, S, num_heads, 512]
 *                (BSND, num_tokens = batch*S), bf16 or fp16, contiguous
 *   ori_kv       paged raw cache [ori_num_blocks, ori_block_size, 1, 512]
 *   ori_block_table [batch, ori_table_stride] int32
 *   cmp_kv / cmp_block_table: compressed cache, NULL for SWA (scenario 1)
 *   cmp_sparse_indices [num_tokens, 1, topk] int32, NULL unless SCFA (scenario 3)
 *   cu_seqlens_q [batch+1] (required for TND, optional for BSND)
 *   seqused_kv   [batch]
 *   sinks        [num_heads] fp32
 *   metadata     int32[1024] from sas_metadata (or any producer of the contract)
 *   out          same shape/dtype as q;  lse [num_tokens, num_heads] fp32 (may be NULL)
 * scenario: 1 = SWA, 2 = CFA (dense compressed rows), 3 = SCFA (top-k).
 * stage_mask: which launches to enqueue (SAS_STAGE_PLAN, SAS_STAGE_ATTENTION;
 * the attention launch also merges split tokens). The stages communicate
 * through `workspace`, so a split call sequence must pass the same arguments
 * to every stage. SAS_STAGE_ALL is the normal call. The workspace must be
 * zero-filled before its first use (its split-token counters start at zero;
 * every launch leaves them zero).
 * ---------------------------------------------------------------------- */
size_t sas_fwd_workspace_bytes(int32_t num_tokens, int32_t num_heads, int32_t num_sms);

int sas_sparse_attn_sharedkv_fwd(
    const void* q, int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t dtype,
    int32_t layout_q, int32_t batch, int32_t max_seqlen_q, const int32_t* cu_seqlens_q,
    const int32_t* seqused_kv,
    const void* ori_kv, int64_t ori_num_blocks, int32_t ori_block_size,
    const int32_t* ori_block_table, int32_t ori_table_stride,
    const void* cmp_kv, int64_t cmp_num_blocks, int32_t cmp_block_size,
    const int32_t* cmp_block_table, int32_t cmp_table_stride,
    const int32_t* cmp_sparse_indices, int32_t topk,
    const float* sinks, const int32_t* metadata,
    float softmax_scale, int32_t cmp_ratio, int32_t ori_win_left, int32_t scenario,
    void* out, float* lse,
    int32_t num_sms, int32_t stage_mask, int32_t* status, void* workspace, size_t workspace_bytes,
    void* stream);

/* Head-sharded forward for one rank of n (no counterpart in the reference,
 * whose op runs on one device): the call computes heads [out_head_offset,
 * out_head_offset + num_heads) of q (passed as this rank's slice) and writes
 * every output and LSE value straight into all n buffers outs[k] / lses[k],
 * each [num_tokens, out_heads_total, 512] / [num_tokens, out_heads_total] -
 * the rank's own and its peers', as device pointers into peer-accessible
 * (symmetric) memory over NVLink. The all-gather of the head-sharded mode is
 * thereby done by the attention kernel's own stores, overlapped with its
 * compute; the caller fences the ranks before and after the call (a buffer
 * must not be read by its owner while peers write it). n <= 8, lses may be
 * NULL, SAS_FLAG_AFTER_METADATA and SAS_OPT_SPLIT_TOKENS are not accepted.
 * Other arguments as sas_sparse_attn_sharedkv_fwd. */
int sas_sparse_attn_sharedkv_fwd_gather(
    const void* q, int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t dtype,
    int32_t layout_q, int32_t batch, int32_t max_seqlen_q, const int32_t* cu_seqlens_q,
    const int32_t* seqused_kv,
    const void* ori_kv, int64_t ori_num_blocks, int32_t ori_block_size,
    const int32_t* ori_block_table, int32_t ori_table_stride,
    const void* cmp_kv, int64_t cmp_num_blocks, int32_t cmp_block_size,
    const int32_t* cmp_block_table, int32_t cmp_table_stride,
    const int32_t* cmp_sparse_indices, int32_t topk,
    const float* sinks, const int32_t* metadata,
    float softmax_scale, int32_t cmp_ratio, int32_t ori_win_left, int32_t scenario,
    void* const* outs, float* const* lses, int32_t n_out, int32_t out_heads_total, int32_t out_head_offset,
    int32_t num_sms, int32_t stage_mask, int32_t* status, void* workspace, size_t workspace_bytes,
    void* stream);

/* ------------------------------------------------------------------------
 * Backward, consuming the forward's LSE. The reference documents the LSE as
 * the input of a FlashAttention-2 style backward
 * (sparse_attn_sharedkv_tilelang/api.py:32-35, 176-184) and ships none; this
 * is the gradient of the forward's math (golden.py:69-204, exact softmax with
 * the sink in the denominator) for every query token:
 *   dq [num_tokens, num_heads, 512] (q's type), written;
 *   d_ori_kv / d_cmp_kv fp32, shaped like the pools, ACCUMULATED into (zero
 *     them first; K = V, so a row gets its key and value gradients);
 *   d_sinks fp32 [num_heads], accumulated into.
 * dout, q and out are [num_tokens, num_heads, 512] in the I/O type, lse fp32
 * [num_tokens, num_heads] as the forward returned it. The other arguments
 * are the forward's. sas_bwd_cast converts n fp32 values to the I/O type
 * (dtype code), e.g. a pool gradient.
 * ---------------------------------------------------------------------- */
int sas_sparse_attn_sharedkv_bwd(
    const void* dout, const void* q, const void* out, const float* lse, int32_t num_tokens, int32_t num_heads,
    int32_t head_dim, int32_t dtype, int32_t layout_q, int32_t batch, int32_t max_seqlen_q,
    const int32_t* cu_seqlens_q, const int32_t* seqused_kv, const void* ori_kv, int64_t ori_num_blocks,
    int32_t ori_block_size, const int32_t* ori_block_table, int32_t ori_table_stride, const void* cmp_kv,
    int64_t cmp_num_blocks, int32_t cmp_block_size, const int32_t* cmp_block_table, int32_t cmp_table_stride,
    const int32_t* cmp_sparse_indices, int32_t topk, const float* sinks, float softmax_scale, int32_t cmp_ratio,
    int32_t ori_win_left, int32_t scenario, void* dq, float* d_ori_kv, float* d_cmp_kv, float* d_sinks,
    int32_t* status, void* stream);
int sas_bwd_cast(const float* src, void* dst, int64_t n, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * Process-wide options of the forward kernel (no counterpart in the
 * reference, whose knobs are compile-time JIT parameters, api.py:59-126).
 *   SAS_OPT_RESCALE_THRESHOLD (value): the online softmax keeps a per-head
 *     running max m, raised once per 512-row tile with the tile's exact max,
 *     so P is rounded at the same points as golden.py. With value > 0 the max
 *     (and the accumulator) is only moved when a tile's max exceeds m by more
 *     than `value` (log2 units). Default 0: exact.
 *   SAS_OPT_TRACE_BUFFER (ptr, value = its size in bytes): device buffer of
 *     46 uint64 per CTA (30 per-role
 *     cycle counters for every CTA, then 16 event timestamps per CTA) that
 *     receives the diagnostics of the next launches (NULL = off).
 *   SAS_OPT_SPLIT_TOKENS (value): by default a token is never split across
 *     CTAs, as the reference keeps every token on one core. With value >= 0, a
 *     token longer than a range plus `value` tiles is split at range
 *     boundaries and its pieces are merged in fp32 (split-KV). Faster for a
 *     few very long tokens, but a piece other than the first rounds P against
 *     its own running max, so such tokens meet the accuracy bounds and not the
 *     reference's rounding points. value < 0 restores the default.
 *   SAS_OPT_WAIT_LIMIT_NS (value): limit, in ns, of every bounded wait of
 *     the attention kernel for the next launches (0 restores the default of
 *     2 s). A wait that runs out records SAS_ERR_TIMEOUT_BASE + its id in the
 *     status word; the CTA drains the copies and MMAs it has in flight, frees
 *     its TMEM and returns, so the context stays usable. Small values exist to
 *     exercise that path.
 *   SAS_OPT_SCHED_SCAN_CAP (value): rows the scheduler's greedy walk may scan
 *     for one core before it stops and records SAS_ERR_SCHED_OVERRUN (0
 *     restores the default of 2^24).
 * These options are process-wide and not synchronised: set them while no
 * other host thread is launching through this library. The trace buffer is
 * one pointer for every device; it must hold 46 uint64 per CTA of the grid.
 * ---------------------------------------------------------------------- */
#define SAS_OPT_RESCALE_THRESHOLD 1
#define SAS_OPT_TRACE_BUFFER 2
#define SAS_OPT_SPLIT_TOKENS 3
#define SAS_OPT_WAIT_LIMIT_NS 4
#define SAS_OPT_SCHED_SCAN_CAP 5
int sas_fwd_set_option(int32_t option, double value, void* ptr);

#ifdef __cplusplus
}
#endif
#endif /* SAS_B200_H_ */
