// params.h -- kernel parameter blocks and internal launch entry points.
// Host code (capi.cu) fills these; kernels receive them as __grid_constant__.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cra {

// One document of a packed variable-length batch (device table, built by
// cra_varlen_plan): rows [start, start + len) of the packed sequence, its
// own window W and global rows per block R, the first row of its global
// rows in the packed list, and prefix counts of query-tile pairs and
// W-blocks over the earlier documents.
struct DocInfo {
  int start, len, W, R, g0, pair0, blk0, pad;
};

// Query-centric attention pass (forward, and the dQ pass of the backward).
struct alignas(64) QueryPassParams {
  CUtensorMap tm_q;   // [B, H,   S,  D]
  CUtensorMap tm_k;   // [B, Hkv, S,  D]
  CUtensorMap tm_v;   // [B, Hkv, S,  D]
  CUtensorMap tm_gk;  // [B, Hkv, NG, D]
  CUtensorMap tm_gv;  // [B, Hkv, NG, D]
  CUtensorMap tm_do;  // [B, H,   S,  D]   (backward only)
  // Sequence shard with an edge copy (forward): pairs whose local window
  // starts before kv_begin read their band keys from tm_ke / tm_ve, whose
  // row 0 is absolute position edge_begin (the previous shard's last W - 1
  // rows followed by this shard's first rows).
  CUtensorMap tm_ke;
  CUtensorMap tm_ve;
  int has_edge, edge_begin;
  // Packed variable-length batch (forward): one CTA per query-tile pair of
  // every document; null for a single sequence.
  const DocInfo* docs;
  int n_docs, n_pairs_total;
  int lse_len;        // row stride of lse per (b, h): q_len, or the packed length
  void* out;          // forward: O;  backward: dQ  (element strides below)
  int64_t out_sb, out_sh, out_ss;
  int out_v8;         // every output row starts on a 32-byte boundary: 32-byte stores allowed
  float* lse;         // [B, H, S] fp32, natural log (written by fwd, read by bwd)
  const float* delta; // [B, H, S] fp32, rowsum(O * dO) (backward only)
  int B, H, kv_groups, S, W, R, NG, n_qtiles;
  // Sequence shard (forward): Q / O / lse rows hold absolute positions
  // [q_begin, q_begin + q_len); K / V rows start at absolute position
  // kv_begin.  Whole sequence: q_begin = kv_begin = 0, q_len = S.
  int q_begin, q_len, kv_begin;
  float scale;        // softmax scale
  float scale_log2;   // softmax scale * log2(e)
  int* err;           // device error word, may be null
};

// Key-centric backward pass (dK/dV over the local band, or dG over the
// global rows).
struct alignas(64) KeyPassParams {
  CUtensorMap tm_q;   // [B, H, S, D]
  CUtensorMap tm_do;  // [B, H, S, D]
  CUtensorMap tm_k;   // key rows:   K [B,Hkv,S,D]  or G_k [B,Hkv,NG,D]
  CUtensorMap tm_v;   // value rows: V               or G_v
  const float* lse;   // [B, H, S]
  const float* delta; // [B, H, S]
  // local mode: dK / dV outputs (element strides), plus the reduced global-row
  // gradients to fold in (fp32 [B,Hkv,NG,D]) and the relay sources.
  void* dk; void* dv;
  int64_t dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  int dkv_v8;         // every dK / dV row starts on a 32-byte boundary: 32-byte stores allowed
  const float* dgk; const float* dgv;
  const int32_t* gsrc;     // [B, Hkv, NB, TOP_K]
  const float* relay_scale;// [Hkv] relay_log_scale (alpha) per kv head, or null
  // global mode: fp32 partial outputs [n_split, B, Hkv, NG, D]
  float* part_k; float* part_v;
  // fused backward: fp32 dQ accumulator [B, H, Spad, D] (unscaled), zeroed
  // by the delta kernel; the key passes add dS K into it
  float* dq_acc;
  int B, H, kv_groups, S, W, R, NB, NG, top_k;
  int n_ktiles;       // key tiles per (b, hkv)
  int n_split;        // global mode: query splits per key tile
  // Sequence shard (backward of a sequence split across GPUs).  Positions
  // are absolute; this GPU's queries are [q_lo, q_hi) (Q / dO / lse / delta
  // rows hold them from q_lo, q_pad rows per (b, h) in the padded arrays);
  // local mode walks the keys [k_lo, q_hi) -- the W - 1 halo keys of the
  // previous shard first -- with K / V rows from kv_main in tm_k / tm_v and,
  // with has_edge, rows below kv_main + 128 from the edge copy tm_ke / tm_ve
  // (row 0 = edge_begin); dK / dV of keys below kv_main go to dkh / dvh (row
  // 0 = k_lo, no global-row fold-in: their blocks belong to the previous
  // shard).  Whole sequence: q_lo = k_lo = kv_main = 0, q_hi = S.
  int q_lo, q_hi, q_pad, k_lo, kv_main, has_edge, edge_begin;
  CUtensorMap tm_ke, tm_ve;
  void* dkh; void* dvh;
  int64_t dkh_sb, dkh_sh, dkh_ss, dvh_sb, dvh_sh, dvh_ss;
  float scale, scale_log2;
  int* err;
};

// Everything one backward launch sequence needs (bwd.cu).
struct BwdLaunch {
  QueryPassParams qp;      // dQ pass (lse / delta point at the padded arrays)
  KeyPassParams global;    // dG over global rows -> partials
  KeyPassParams local;     // dK / dV over the local band (+ dG fold-in)
  const void* o;
  const void* d_o;
  int64_t o_st[3], do_st[3];
  const float* lse_in;     // forward lse [B, H, S]
  float* lse2;             // [B, H, Spad] lse * log2(e)
  float* delta;            // [B, H, Spad] rowsum(O * dO)
  float* dgk;              // [B, Hkv, NG, D] reduced global-row gradients
  float* dgv;
  float* d_alpha;          // [Hkv] or null
  const void* gk_rows;     // G_k / G_v (for d_alpha)
  const void* gv_rows;
  // Optional timing: when non-null, events[i] is recorded on the stream just
  // before kernel i and events[n_kernels] after the last one.
  bool fused;              // dQ from the key passes (fp32 atomics), no dQ pass
  int phase;               // 0 all kernels; shard: 1 delta + global-row pass + reduce, 2 the rest
  static constexpr int kMaxKernels = 8;
  cudaEvent_t* events;
  int n_kernels;                // set by launch_bwd: kernels launched (timed)
  int kernel_ids[kMaxKernels];  // set by launch_bwd: which kernel each was
};

// Name of the backward kernel with id `id` (BwdLaunch::kernel_ids).
const char* bwd_kernel_name(int i);

cudaError_t launch_bwd(const BwdLaunch& L, int D, bool bf16, cudaStream_t stream);

// Sets the calling thread's cra_last_error_message text; returns status.
int set_last_error(int status, const char* text);

}  // namespace cra
