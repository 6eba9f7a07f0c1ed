/* cra.h -- C ABI of libcra, the B200 (sm_100a) implementation of Cron Root
 * Attention's causal 3-phase sqrt(N) sparse attention.
 *
 * Every entry point takes raw device pointers, sizes and element strides,
 * enqueues work on the given CUDA stream (a cudaStream_t passed as void*;
 * NULL = legacy default stream) and returns a status code.  Nothing here
 * allocates device memory, synchronizes the host, or aborts the process.
 * The caller owns every buffer, including the backward workspace.
 *
 * Tensor layout: q, o, d_o, dq are [batch, heads, seq_len, head_dim]; k, v,
 * dk, dv are [batch, kv_heads, seq_len, head_dim].  A tensor is described by
 * its base pointer and `strides[3]` = element strides of (batch, head, seq);
 * the head_dim stride must be 1.  Base pointers must be 16-byte aligned and
 * strides multiples of 8 elements (TMA requirements).
 * Supported: dtype CRA_F16 / CRA_BF16, head_dim 64 or 128, 1 <= top_k <= 4,
 * heads % kv_heads == 0.
 *
 * The packed global-row list ("G") holds, per (batch, kv_head) and per
 * W-block r, R = 1 + top_k rows (R = 1 without the relay): the strided key
 * k[r*W], then the top_k relay tokens of block r.  g_k / g_v are contiguous
 * [batch, kv_heads, cra_global_rows(), head_dim] in the input dtype; g_src is
 * contiguous int32 [batch, kv_heads, NB, top_k] with NB = ceil(seq_len / W).
 */
#ifndef CRA_H_
#define CRA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

enum cra_status {
  CRA_OK = 0,
  CRA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, heads % kv_heads != 0 */
  CRA_ERR_UNSUPPORTED = 2,      /* dtype / head_dim / top_k outside the supported set */
  CRA_ERR_MISALIGNED = 3,       /* pointer or stride violates the TMA alignment rules */
  CRA_ERR_WORKSPACE = 4,        /* backward workspace smaller than cra_bwd_workspace_bytes() */
  CRA_ERR_CUDA = 5,             /* a CUDA runtime call or kernel launch failed */
  CRA_ERR_DRIVER = 6            /* the driver entry point for tensor maps is unavailable */
};

enum cra_dtype { CRA_F16 = 0, CRA_BF16 = 1 };

/* Device-side error codes written to `*dev_error` (when non-null).  Set only
 * when a kernel gave up on a bounded wait; the kernel then exits cleanly. */
enum cra_device_error { CRA_DEV_OK = 0, CRA_DEV_WAIT_TIMEOUT = 1 };

/* Human-readable text for a cra_status value. */
const char* cra_status_string(int status);

/* Detail text for the last non-zero status returned on the calling thread
 * (which tensor or size was rejected, or which CUDA call failed). */
const char* cra_last_error_message(void);

/* Library version, major * 10000 + minor * 100 + patch. */
int cra_version(void);

/* W = ceil(sqrt(seq_len)): block size, stride and local window length.
 * Replaces `SQRT_N = int(math.ceil(math.sqrt(S)))`, core.py:3479. */
int cra_window(int64_t seq_len);

/* 1 if the relay phase is used at this length (seq_len > 2048), else 0.
 * Replaces `skip_relay = S <= RELAY_THRESHOLD`, core.py:2832,3507. */
int cra_relay_active(int64_t seq_len);

/* Rows per (batch, kv_head) of the packed global list: NB * (1 + top_k)
 * with the relay, NB without. */
int64_t cra_global_rows(int64_t seq_len, int use_relay, int top_k);

/* Builds the packed global list G from k / v: strided rows always, and with
 * use_relay the top_k rows of largest ||k||^2 per W-block (ties to the lower
 * index), scaled by exp(relay_log_scale[h]) when that pointer is non-null
 * (fp32 [kv_heads]).  g_src may be NULL when the backward is not needed.
 * Replaces the relay launch _relay_precompute_topk[(B*H_kv, NB)](...),
 * core.py:3516-3534 (kernel core.py:2630-2748), and the relay scale,
 * core.py:3541-3544. */
int cra_relay_build(const void* k, const void* v, const int64_t* k_strides, const int64_t* v_strides, int batch,
                    int kv_heads, int seq_len, int head_dim, int dtype, int use_relay, int top_k,
                    const float* relay_log_scale, void* g_k, void* g_v, int32_t* g_src, void* stream);

/* Forward: o = softmax over (local band + visible prefix of G) and the
 * natural-log row log-sum-exp lse (fp32, contiguous [batch, heads, seq_len]).
 * softmax_scale is normally 1/sqrt(head_dim).
 * Replaces the forward launch _cron_root_attn_fwd_v14_tiled[(B, H, tiles)],
 * core.py:3591-3610 (kernel core.py:907-1158). */
int cra_fwd(const void* q, const void* k, const void* v, const void* g_k, const void* g_v, const int64_t* q_strides,
            const int64_t* k_strides, const int64_t* v_strides, int batch, int heads, int kv_heads, int seq_len,
            int head_dim, int dtype, int use_relay, int top_k, float softmax_scale, void* o, const int64_t* o_strides,
            float* lse, int* dev_error, void* stream);

/* Sequence split across GPUs.  One GPU's shard of a single long sequence
 * owns the W-block-aligned query range [q_begin, q_begin + q_len) of a
 * sequence of seq_len tokens.
 *
 * cra_relay_build_shard: G rows of the blocks inside rows [row_begin,
 * row_begin + rows) (row_begin a multiple of W = cra_window(seq_len); only
 * the sequence's last shard may end inside a block), from this GPU's k / v
 * rows (local row 0 = absolute position row_begin).  g_k / g_v receive
 * [batch, kv_heads, nblocks_local * R, head_dim]; g_src absolute positions.
 * The full list is the concatenation over shards in order (an all-gather).
 *
 * cra_fwd_shard: forward for the shard's queries.  q / o / lse hold q_len
 * rows (lse contiguous [batch, heads, q_len]); g_k / g_v are the FULL global
 * list of the sequence.  K / V, either way:
 *   - without an edge copy (k_edge = v_edge = NULL): k / v hold kv_len rows
 *     starting at absolute position kv_begin <= max(q_begin - (W - 1), 0),
 *     i.e. the local-window halo from the previous shard in front;
 *   - with an edge copy: k / v are the shard's own rows (kv_begin = q_begin)
 *     and k_edge / v_edge hold edge_len rows from absolute position
 *     edge_begin, covering [max(q_begin - (W - 1), 0), min(q_begin + W + 255,
 *     q_begin + q_len)): the halo plus the shard's first rows, a few thousand rows
 *     in all, read by the query tiles whose window reaches into the halo.
 *     No copy of the whole shard is needed.
 * Same numerics as cra_fwd on the whole sequence.
 * Replaces nothing in the reference (single-GPU only there); used for the
 * sequence-split configuration. */
int cra_relay_build_shard(const void* k, const void* v, const int64_t* k_strides, const int64_t* v_strides,
                          int batch, int kv_heads, int64_t seq_len, int64_t row_begin, int rows, int head_dim,
                          int dtype, int use_relay, int top_k, const float* relay_log_scale, void* g_k, void* g_v,
                          int32_t* g_src, void* stream);
int cra_fwd_shard(const void* q, const void* k, const void* v, const void* g_k, const void* g_v,
                  const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int batch, int heads,
                  int kv_heads, int64_t seq_len, int64_t q_begin, int q_len, int64_t kv_begin, int kv_len,
                  const void* k_edge, const void* v_edge, const int64_t* ke_strides, const int64_t* ve_strides,
                  int64_t edge_begin, int edge_len, int head_dim, int dtype, int use_relay, int top_k,
                  float softmax_scale, void* o, const int64_t* o_strides, float* lse, int* dev_error, void* stream);

/* Packed variable-length batches (documents of different lengths
 * concatenated along the sequence dimension; every document attends only to
 * itself, with its own W = ceil(sqrt(len)) and relay switch).  cu_seqlens is
 * a HOST array of n_docs + 1 increasing offsets starting at 0; the packed
 * length is cu_seqlens[n_docs].
 *   cra_varlen_plan writes the device document table (caller-allocated,
 *   cra_varlen_table_bytes(n_docs) bytes) on `stream`;
 *   cra_relay_build_varlen builds every document's global rows into one
 *   packed list g_k / g_v [batch, kv_heads, cra_varlen_global_rows(), D]
 *   (document d's rows after document d - 1's) and g_src [batch, kv_heads,
 *   cra_varlen_blocks(), top_k] (positions local to the document) -- one
 *   launch for all documents;
 *   cra_fwd_varlen computes every document's forward -- one launch over
 *   (document, query-tile pair, head); lse is [batch, heads, packed length].
 * Replaces the per-document loop of cron_root_attention_varlen, core.py:
 * 3837-3954 (each document there is a separate cron_root_attention_v14
 * call). */
size_t cra_varlen_table_bytes(int n_docs);
int64_t cra_varlen_global_rows(const int64_t* cu_seqlens, int n_docs, int top_k);
int64_t cra_varlen_blocks(const int64_t* cu_seqlens, int n_docs);
int cra_varlen_plan(const int64_t* cu_seqlens, int n_docs, int top_k, void* table, void* stream);
int cra_relay_build_varlen(const void* k, const void* v, const int64_t* k_strides, const int64_t* v_strides,
                           int batch, int kv_heads, const int64_t* cu_seqlens, int n_docs, const void* table,
                           int head_dim, int dtype, int top_k, const float* relay_log_scale, void* g_k, void* g_v,
                           int32_t* g_src, void* stream);
int cra_fwd_varlen(const void* q, const void* k, const void* v, const void* g_k, const void* g_v,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int batch, int heads,
                   int kv_heads, const int64_t* cu_seqlens, int n_docs, const void* table, int head_dim, int dtype,
                   int top_k, float softmax_scale, void* o, const int64_t* o_strides, float* lse, int* dev_error,
                   void* stream);

/* Backward of one GPU's shard of a sequence split across GPUs, in two
 * phases around a cross-GPU sum (no counterpart in the reference, which is
 * single-GPU).  The shard owns queries and keys [q_begin, q_begin + q_len)
 * (q_begin a multiple of W); q / o / d_o / lse / dq / k / v / dk / dv hold
 * those rows; g_k / g_v / g_src are the FULL global-row list of the
 * sequence (as the forward gathered it; g_src absolute positions).
 *   cra_bwd_shard_global: dG_k / dG_v (fp32 [batch, kv_heads, NG, D],
 *     overwritten) of every global row from this shard's queries.  The
 *     caller then sums dg_k / dg_v over all shards (an all-reduce).
 *   cra_bwd_shard_local (same workspace, after the sum): dq of the shard's
 *     queries; dk / dv of its keys from its own queries plus the summed dG of
 *     its blocks' global rows; and dk_halo / dv_halo: the contributions of
 *     this shard's queries to the previous shard's last W - 1 keys (rows
 *     from max(q_begin - (W - 1), 0)), which the caller sends to the previous
 *     shard and adds to its dk / dv.  k_edge / v_edge (edge_len rows from
 *     absolute position edge_begin) must cover [max(q_begin - (W - 1), 0),
 *     min(q_begin + 128, q_begin + q_len)): the halo keys plus the shard's
 *     first rows.  Not needed for the first shard (q_begin = 0).
 *     d_relay_log_scale (nullable) receives the scale gradient of the summed
 *     dG: the same on every shard, so exactly one shard should report it.
 * Workspace: cra_bwd_shard_workspace_bytes() bytes, 256-byte aligned, the
 * same buffer for both phases. */
size_t cra_bwd_shard_workspace_bytes(int batch, int heads, int kv_heads, int64_t seq_len, int q_len, int head_dim,
                                     int use_relay, int top_k);
int cra_bwd_shard_global(const void* q, const void* o, const void* d_o, const float* lse, const void* g_k,
                         const void* g_v, const int64_t* q_strides, const int64_t* o_strides,
                         const int64_t* do_strides, int batch, int heads, int kv_heads, int64_t seq_len,
                         int64_t q_begin, int q_len, int head_dim, int dtype, int use_relay, int top_k,
                         float softmax_scale, float* dg_k, float* dg_v, void* workspace, size_t workspace_bytes,
                         int* dev_error, void* stream);
int cra_bwd_shard_local(const void* q, const void* k, const void* v, const void* d_o, const void* g_k,
                        const void* g_v, const int32_t* g_src, const int64_t* q_strides, const int64_t* k_strides,
                        const int64_t* v_strides, const int64_t* do_strides, const void* k_edge, const void* v_edge,
                        const int64_t* ke_strides, const int64_t* ve_strides, int64_t edge_begin, int edge_len,
                        int batch, int heads, int kv_heads, int64_t seq_len, int64_t q_begin, int q_len,
                        int head_dim, int dtype, int use_relay, int top_k, float softmax_scale,
                        const float* relay_log_scale, const float* dg_k, const float* dg_v, void* dq, void* dk,
                        void* dv, void* dk_halo, void* dv_halo, const int64_t* dq_strides, const int64_t* dk_strides,
                        const int64_t* dv_strides, const int64_t* dkh_strides, const int64_t* dvh_strides,
                        float* d_relay_log_scale, void* workspace, size_t workspace_bytes, int* dev_error,
                        void* stream);

/* Bytes of device workspace cra_bwd needs for these sizes (256-byte aligned
 * base required). */
size_t cra_bwd_workspace_bytes(int batch, int heads, int kv_heads, int seq_len, int head_dim, int use_relay,
                               int top_k);

/* Backward: dq, dk, dv (input dtype) from o, d_o and the forward's lse / G.
 * Gradients of the relay rows are summed into dk / dv at their source
 * positions (g_src); with relay_log_scale non-null they are multiplied by
 * exp(relay_log_scale[h]) on the way (chain rule through the scaled rows),
 * and d_relay_log_scale (fp32 [kv_heads], overwritten) receives
 * sum(dG_k * G_k + dG_v * G_v) over the relay rows.
 * Deterministic: no floating-point atomics; every sum has a fixed order.
 * Replaces CronRootAttentionV14Function.backward, core.py:3626-3759, with its
 * kernels core.py:1165-1316 (dQ), 1650-1745 (local dK/dV), 1755-1889
 * (strided dK/dV), 2381-2492 (relay dK/dV), 2767-2815 (relay scatter). */
int cra_bwd(const void* q, const void* k, const void* v, const void* o, const void* d_o, const float* lse,
            const void* g_k, const void* g_v, const int32_t* g_src, const int64_t* q_strides,
            const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
            int batch, int heads, int kv_heads, int seq_len, int head_dim, int dtype, int use_relay, int top_k,
            float softmax_scale, const float* relay_log_scale, void* dq, void* dk, void* dv,
            const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
            float* d_relay_log_scale, void* workspace, size_t workspace_bytes, int* dev_error, void* stream);

/* Backward variant that computes dQ inside the two key-centric passes (a
 * fifth GEMM per 128 x 64 block, dQ^T = K^T dS^T, added into an fp32
 * accumulator in the workspace with atomic adds, then converted), so the
 * scores are recomputed once instead of twice and there is no dQ pass.  dq
 * may differ in the last bits between calls (atomic order); dk, dv are
 * summed in a fixed order.  Same arguments as cra_bwd, with a workspace of
 * cra_bwd_fused_workspace_bytes(); head_dim 64 runs cra_bwd's kernels.
 * Measured on B200 at B1 H16 S64K D128 it is slower than cra_bwd (the
 * accumulator traffic and the longer per-unit chain cost more than the dQ
 * pass saves), so the Python API uses cra_bwd.  No counterpart in the
 * reference beyond the backward it shares with cra_bwd. */
int cra_bwd_fused(const void* q, const void* k, const void* v, const void* o, const void* d_o, const float* lse,
                  const void* g_k, const void* g_v, const int32_t* g_src, const int64_t* q_strides,
                  const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                  const int64_t* do_strides, int batch, int heads, int kv_heads, int seq_len, int head_dim, int dtype,
                  int use_relay, int top_k, float softmax_scale, const float* relay_log_scale, void* dq, void* dk,
                  void* dv, const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                  float* d_relay_log_scale, void* workspace, size_t workspace_bytes, int* dev_error, void* stream);
size_t cra_bwd_fused_workspace_bytes(int batch, int heads, int kv_heads, int seq_len, int head_dim, int use_relay,
                                     int top_k);

/* Measurement helper (no counterpart in the reference): runs cra_bwd with the
 * same arguments, records a CUDA event on `stream` before each of its kernels
 * and after the last, SYNCHRONIZES the stream, and returns each kernel's
 * event-to-event time in kernel_ms[i] (ms) and its name in kernel_names[i]
 * (static strings; may be NULL) for i < *n_kernels <= max_kernels, in launch
 * order; fused != 0 times cra_bwd_fused's kernels instead (workspace of
 * cra_bwd_fused_workspace_bytes()).
 * For benchmarks and profiles only. */
int cra_bwd_kernel_times(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                         const float* lse, const void* g_k, const void* g_v, const int32_t* g_src,
                         const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                         const int64_t* o_strides, const int64_t* do_strides, int batch, int heads, int kv_heads,
                         int seq_len, int head_dim, int dtype, int use_relay, int top_k, float softmax_scale,
                         const float* relay_log_scale, void* dq, void* dk, void* dv, const int64_t* dq_strides,
                         const int64_t* dk_strides, const int64_t* dv_strides, float* d_relay_log_scale,
                         void* workspace, size_t workspace_bytes, int* dev_error, void* stream, float* kernel_ms,
                         const char** kernel_names, int max_kernels, int* n_kernels, int fused);

/* Backward without a caller-provided workspace, for callers that cannot
 * allocate device memory (no access to an allocator, or code that must not
 * allocate at all, such as a plug-in running under a host framework that owns
 * every allocation).  No counterpart in the reference.
 * Same arguments and results as cra_bwd minus the workspace: the scratch
 * lives in a fixed array inside the library, CRA_BWD_NOALLOC_SCRATCH_BYTES
 * (32 MiB) on every GPU that loads the library, held until the process exits.
 * Sizes whose cra_bwd_workspace_bytes() exceeds that return
 * CRA_ERR_WORKSPACE.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current) and keeps it for
 * the rest of the process: the address belongs to the CUDA context current at
 * that first call, so it is stale after cudaDeviceReset.  Make that first
 * call before any stream capture.  Calls share the array: two calls whose
 * work overlaps on the GPU (different streams, or different host threads
 * without ordering) race and corrupt each other's results.  Nothing in the
 * scratch needs to start at zero; every call overwrites what it reads. */
#define CRA_BWD_NOALLOC_SCRATCH_BYTES (32u << 20)
int cra_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* d_o, const float* lse,
                    const void* g_k, const void* g_v, const int32_t* g_src, const int64_t* q_strides,
                    const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                    const int64_t* do_strides, int batch, int heads, int kv_heads, int seq_len, int head_dim,
                    int dtype, int use_relay, int top_k, float softmax_scale, const float* relay_log_scale, void* dq,
                    void* dk, void* dv, const int64_t* dq_strides, const int64_t* dk_strides,
                    const int64_t* dv_strides, float* d_relay_log_scale, int* dev_error, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* CRA_H_ */
