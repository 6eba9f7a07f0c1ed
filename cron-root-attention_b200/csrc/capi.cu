// capi.cu -- the extern "C" entry points declared in include/cra.h: argument
// validation, TMA tensor-map construction and kernel launches.  Stateless and
// reentrant: nothing is cached across calls except the driver entry point
// for cuTensorMapEncodeTiled and per-kernel shared-memory attributes.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/cra.h"
#include "geom.cuh"
#include "params.h"

namespace cra {
cudaError_t launch_relay_build(int D, bool bf16, const void* k, const void* v, const int64_t* ks, const int64_t* vs,
                               int B, int Hkv, int S, int W, int top_k, int R, int pos0, const float* log_scale,
                               void* gk, void* gv, int32_t* gsrc, cudaStream_t stream, const DocInfo* docs = nullptr,
                               int n_docs = 0, int NB_total = 0, int NG_total = 0);
cudaError_t launch_fwd(const QueryPassParams& p, int D, bool bf16, cudaStream_t stream);
}  // namespace cra

using namespace cra;

namespace {

constexpr int kVersion = 100;  // 0.1.0

thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Makes the calling thread's current device's primary context current.  A
// thread that has made no CUDA runtime call yet (for example a framework's
// backward worker whose allocations were all served from a cache) has no
// current context, and cuTensorMapEncodeTiled then fails.
int bind_context() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaSetDevice(dev);
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "binding the device context: %s", cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// True when every row of a 16-bit [dim0, dim1, rows, D] tensor starts on a
// 32-byte boundary (base and the strides of every dimension longer than 1),
// so kernels may write its rows with 32-byte stores.
int rows_aligned32(const void* p, const int64_t* st, int dim0, int dim1, int64_t rows) {
  if (reinterpret_cast<uintptr_t>(p) & 31) return 0;
  const int64_t ext[3] = {dim0, dim1, rows};
  for (int i = 0; i < 3; ++i)
    if (ext[i] > 1 && (st[i] * 2) % 32 != 0) return 0;
  return 1;
}

// Checks one [dim0, dim1, rows, D] tensor description.
int check_tensor(const char* name, const void* p, const int64_t* st, int dim0, int dim1) {
  if (!p || !st) return fail(CRA_ERR_INVALID_ARGUMENT, "%s: null pointer or strides", name);
  if (!aligned16(p)) return fail(CRA_ERR_MISALIGNED, "%s: base pointer not 16-byte aligned", name);
  for (int i = 0; i < 3; ++i) {
    if (st[i] < 0) return fail(CRA_ERR_INVALID_ARGUMENT, "%s: negative stride", name);
    if (st[i] % 8 != 0) {
      const int extent = i == 0 ? dim0 : (i == 1 ? dim1 : 2);
      if (extent > 1)  // stride of a size-1 dim is never used
        return fail(CRA_ERR_MISALIGNED, "%s: stride %d (%lld) not a multiple of 8 elements", name, i,
                    static_cast<long long>(st[i]));
    }
  }
  return CRA_OK;
}

// 4-D tensor map over [d1 (outer), d0, rows, D] with box_rows x 64 boxes, 128B swizzle.
int make_tmap(const char* name, CUtensorMap* m, const void* base, bool bf16, int D, int64_t rows, int64_t d0,
              int64_t d1, const int64_t* st, int box_rows = kTile) {
  auto fn = encode_fn();
  if (!fn) return fail(CRA_ERR_DRIVER, "cuTensorMapEncodeTiled not available from the driver");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(d0),
                        static_cast<cuuint64_t>(d1)};
  // byte strides of dims 1..3; a size-1 dim gets a harmless valid stride
  int64_t s_rows = st[2], s_h = st[1], s_b = st[0];
  if (rows <= 1) s_rows = D;
  if (d0 <= 1) s_h = s_rows * rows;
  if (d1 <= 1) s_b = s_h * d0;
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_rows * 2), static_cast<cuuint64_t>(s_h * 2),
                           static_cast<cuuint64_t>(s_b * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(CRA_ERR_INVALID_ARGUMENT,
                "%s: cuTensorMapEncodeTiled failed (CUresult %d), dims [%llu %llu %llu %llu], byte strides "
                "[%llu %llu %llu]",
                name, static_cast<int>(r), (unsigned long long)dims[0], (unsigned long long)dims[1],
                (unsigned long long)dims[2], (unsigned long long)dims[3], (unsigned long long)strides[0],
                (unsigned long long)strides[1], (unsigned long long)strides[2]);
  return CRA_OK;
}

int check_common(int batch, int heads, int kv_heads, int seq_len, int head_dim, int dtype, int top_k) {
  if (batch < 1 || heads < 1 || kv_heads < 1 || seq_len < 1)
    return fail(CRA_ERR_INVALID_ARGUMENT, "sizes must be >= 1 (batch %d heads %d kv_heads %d seq_len %d)", batch,
                heads, kv_heads, seq_len);
  if (heads % kv_heads != 0)
    return fail(CRA_ERR_INVALID_ARGUMENT, "heads (%d) not a multiple of kv_heads (%d)", heads, kv_heads);
  if (batch > 65535 || heads > 65535) return fail(CRA_ERR_INVALID_ARGUMENT, "batch or heads > 65535");
  if (dtype != CRA_F16 && dtype != CRA_BF16) return fail(CRA_ERR_UNSUPPORTED, "dtype %d unsupported", dtype);
  if (head_dim != 64 && head_dim != 128) return fail(CRA_ERR_UNSUPPORTED, "head_dim %d unsupported", head_dim);
  if (top_k < 1 || top_k > 4) return fail(CRA_ERR_UNSUPPORTED, "top_k %d outside 1..4", top_k);
  return CRA_OK;
}

int rows_per_block(int use_relay, int top_k) { return use_relay ? 1 + top_k : 1; }

// Backward workspace layout (all fp32, each region 256-byte aligned):
//   lse2, delta  [B, H, Spad]              Spad = 128 * ceil(S / 128)
//   dgk, dgv     [B, Hkv, NG, D]           reduced global-row gradients
//   part_k/v     [n_split, B, Hkv, NG, D]  per-split partials
//   dq_acc       [B, H, Spad, D]           fused backward only (head_dim 128)
struct BwdLayout {
  int n_split;
  size_t off_lse2, off_delta, off_dgk, off_dgv, off_pk, off_pv, off_dqacc;
  size_t total;        // cra_bwd: no dQ accumulator
  size_t total_fused;  // cra_bwd_fused: adds the fp32 dQ accumulator when head_dim = 128
};

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Query splits per 128-row global tile; a pure function of the sizes so the workspace size is predictable.
int global_splits(int batch, int kv_heads, int seq_len, int NG) {
  const int n_gtiles = (NG + kTile - 1) / kTile;
  const int n_qtiles = (seq_len + kTile - 1) / kTile;
  const long long base = static_cast<long long>(batch) * kv_heads * n_gtiles;
  // about 4 CTAs per SM in all: at the north star 592 CTAs took 0.475 +
  // 0.018 ms (pass + reduce of the partials), 888 took 0.495 + 0.029, 1776
  // took 0.547 + 0.049 (each CTA re-stages its tile and pays a start-up)
  long long s = (592 + base - 1) / base;
  if (s > 32) s = 32;
  if (s > n_qtiles) s = n_qtiles;
  if (s < 1) s = 1;
  return static_cast<int>(s);
}

// q_len: query rows of this GPU (a sequence shard), or the whole sequence (-1).
BwdLayout bwd_layout(int batch, int heads, int kv_heads, int seq_len, int head_dim, int use_relay, int top_k,
                     int q_len = -1) {
  BwdLayout L;
  const int64_t NG = cra_global_rows(seq_len, use_relay, top_k);
  const int64_t Spad = static_cast<int64_t>(((q_len < 0 ? seq_len : q_len) + kTile - 1) / kTile) * kTile;
  L.n_split = global_splits(batch, kv_heads, seq_len, static_cast<int>(NG));
  const size_t rowsz = round256(sizeof(float) * batch * heads * Spad);
  const size_t gsz = round256(sizeof(float) * batch * kv_heads * NG * head_dim);
  L.off_lse2 = 0;
  L.off_delta = L.off_lse2 + rowsz;
  L.off_dgk = L.off_delta + rowsz;
  L.off_dgv = L.off_dgk + gsz;
  L.off_pk = L.off_dgv + gsz;
  L.off_pv = L.off_pk + gsz * L.n_split;
  L.off_dqacc = L.off_pv + gsz * L.n_split;
  L.total = L.off_dqacc;
  L.total_fused = L.off_dqacc + (head_dim == 128 ? round256(sizeof(float) * batch * heads * Spad * head_dim) : 0);
  return L;
}

#define CRA_TRY(x)                \
  do {                            \
    const int _s = (x);           \
    if (_s != CRA_OK) return _s;  \
  } while (0)

}  // namespace

namespace cra {
// Records the detail text returned by cra_last_error_message for the calling
// thread (used by the other C-ABI translation units).
int set_last_error(int status, const char* text) { return fail(status, "%s", text); }
}  // namespace cra

extern "C" {

const char* cra_status_string(int status) {
  switch (status) {
    case CRA_OK: return "ok";
    case CRA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CRA_ERR_UNSUPPORTED: return "unsupported dtype, head_dim or top_k";
    case CRA_ERR_MISALIGNED: return "pointer or stride not aligned for TMA (16-byte base, 8-element strides)";
    case CRA_ERR_WORKSPACE: return "workspace too small";
    case CRA_ERR_CUDA: return "CUDA runtime error";
    case CRA_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable from the driver";
    default: return "unknown status";
  }
}

int cra_version(void) { return kVersion; }

const char* cra_last_error_message(void) { return g_last_error; }

int cra_window(int64_t seq_len) {
  if (seq_len < 1) return 0;
  int w = static_cast<int>(std::ceil(std::sqrt(static_cast<double>(seq_len))));
  // guard the double rounding at perfect squares
  while (static_cast<int64_t>(w - 1) * (w - 1) >= seq_len) --w;
  while (static_cast<int64_t>(w) * w < seq_len) ++w;
  return w;
}

int cra_relay_active(int64_t seq_len) { return seq_len > 2048 ? 1 : 0; }

int64_t cra_global_rows(int64_t seq_len, int use_relay, int top_k) {
  if (seq_len < 1) return 0;
  const int64_t W = cra_window(seq_len);
  const int64_t NB = (seq_len + W - 1) / W;
  return NB * rows_per_block(use_relay, top_k);
}

int cra_relay_build(const void* k, const void* v, const int64_t* k_strides, const int64_t* v_strides, int batch,
                    int kv_heads, int seq_len, int head_dim, int dtype, int use_relay, int top_k,
                    const float* relay_log_scale, void* g_k, void* g_v, int32_t* g_src, void* stream) {
  CRA_TRY(check_common(batch, kv_heads, kv_heads, seq_len, head_dim, dtype, top_k));
  CRA_TRY(check_tensor("k", k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor("v", v, v_strides, batch, kv_heads));
  if (!g_k || !g_v) return fail(CRA_ERR_INVALID_ARGUMENT, "g_k / g_v: null pointer");
  if (!aligned16(g_k) || !aligned16(g_v)) return fail(CRA_ERR_MISALIGNED, "g_k / g_v: not 16-byte aligned");
  const int W = cra_window(seq_len);
  const int R = rows_per_block(use_relay, top_k);
  cudaError_t e = launch_relay_build(head_dim, dtype == CRA_BF16, k, v, k_strides, v_strides, batch, kv_heads,
                                     seq_len, W, top_k, R, 0, use_relay ? relay_log_scale : nullptr, g_k, g_v,
                                     use_relay ? g_src : nullptr, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}

int cra_fwd(const void* q, const void* k, const void* v, const void* g_k, const void* g_v, const int64_t* q_strides,
            const int64_t* k_strides, const int64_t* v_strides, int batch, int heads, int kv_heads, int seq_len,
            int head_dim, int dtype, int use_relay, int top_k, float softmax_scale, void* o, const int64_t* o_strides,
            float* lse, int* dev_error, void* stream) {
  CRA_TRY(check_common(batch, heads, kv_heads, seq_len, head_dim, dtype, top_k));
  CRA_TRY(check_tensor("q", q, q_strides, batch, heads));
  CRA_TRY(check_tensor("k", k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor("v", v, v_strides, batch, kv_heads));
  CRA_TRY(check_tensor("o", o, o_strides, batch, heads));
  if (!g_k || !g_v || !lse) return fail(CRA_ERR_INVALID_ARGUMENT, "g_k / g_v / lse: null pointer");
  if (!aligned16(g_k) || !aligned16(g_v)) return fail(CRA_ERR_MISALIGNED, "g_k / g_v: not 16-byte aligned");
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
    return fail(CRA_ERR_INVALID_ARGUMENT, "softmax_scale must be finite and > 0");
  const bool bf16 = dtype == CRA_BF16;
  const int W = cra_window(seq_len);
  const int R = rows_per_block(use_relay, top_k);
  const int NG = static_cast<int>(cra_global_rows(seq_len, use_relay, top_k));
  const int64_t g_st[3] = {static_cast<int64_t>(kv_heads) * NG * head_dim, static_cast<int64_t>(NG) * head_dim,
                           head_dim};
  CRA_TRY(bind_context());
  QueryPassParams p;
  std::memset(&p, 0, sizeof(p));
  CRA_TRY(make_tmap("q", &p.tm_q, q, bf16, head_dim, seq_len, heads, batch, q_strides));
  CRA_TRY(make_tmap("k", &p.tm_k, k, bf16, head_dim, seq_len, kv_heads, batch, k_strides));
  CRA_TRY(make_tmap("v", &p.tm_v, v, bf16, head_dim, seq_len, kv_heads, batch, v_strides));
  CRA_TRY(make_tmap("gk", &p.tm_gk, g_k, bf16, head_dim, NG, kv_heads, batch, g_st));
  CRA_TRY(make_tmap("gv", &p.tm_gv, g_v, bf16, head_dim, NG, kv_heads, batch, g_st));
  p.tm_do = p.tm_q;
  p.out = o;
  p.out_sb = o_strides[0];
  p.out_sh = o_strides[1];
  p.out_ss = o_strides[2];
  p.out_v8 = rows_aligned32(o, o_strides, batch, heads, seq_len);
  p.lse = lse;
  p.lse_len = seq_len;
  p.delta = nullptr;
  p.B = batch;
  p.H = heads;
  p.kv_groups = heads / kv_heads;
  p.S = seq_len;
  p.W = W;
  p.R = R;
  p.NG = NG;
  p.n_qtiles = (seq_len + kTile - 1) / kTile;
  p.q_begin = 0;
  p.q_len = seq_len;
  p.kv_begin = 0;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = dev_error;
  cudaError_t e = launch_fwd(p, head_dim, bf16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}


size_t cra_bwd_workspace_bytes(int batch, int heads, int kv_heads, int seq_len, int head_dim, int use_relay,
                               int top_k) {
  if (check_common(batch, heads, kv_heads, seq_len, head_dim, CRA_BF16, top_k) != CRA_OK) return 0;
  return bwd_layout(batch, heads, kv_heads, seq_len, head_dim, use_relay, top_k).total;
}

}  // extern "C"

namespace {

// cra_bwd's body; with `events` non-null (BwdLaunch::kMaxKernels + 1 of
// them) an event is recorded before each kernel and after the last.
// One GPU's shard of a sequence split across GPUs (backward).  phase 1:
// delta, global-row pass and reduce (dG of this shard's queries into dg_k /
// dg_v); phase 2: local key pass (with the summed dG folded in) and dQ.
struct ShardSpec {
  int phase;
  int64_t q_begin;
  int q_len;
  const void* k_edge;
  const void* v_edge;
  const int64_t* ke_strides;
  const int64_t* ve_strides;
  int64_t edge_begin;
  int edge_len;
  void* dk_halo;
  void* dv_halo;
  const int64_t* dkh_strides;
  const int64_t* dvh_strides;
  float* dg_k;
  float* dg_v;
};

int bwd_impl(const void* q, const void* k, const void* v, const void* o, const void* d_o, const float* lse,
             const void* g_k, const void* g_v, const int32_t* g_src, const int64_t* q_strides,
             const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
             int batch, int heads, int kv_heads, int seq_len, int head_dim, int dtype, int use_relay, int top_k,
             float softmax_scale, const float* relay_log_scale, void* dq, void* dk, void* dv,
             const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
             float* d_relay_log_scale, void* workspace, size_t workspace_bytes, int* dev_error, void* stream,
             cudaEvent_t* events, int* n_kernels, int* kernel_ids, int fused_req, const ShardSpec* sh = nullptr) {
  const bool fused = fused_req && head_dim == 128 && !sh;
  const int phase = sh ? sh->phase : 0;
  // query rows held by the q / o / d_o / dq / lse tensors, and their first position
  const int q_len = sh ? sh->q_len : seq_len;
  const int q_begin = sh ? static_cast<int>(sh->q_begin) : 0;
  CRA_TRY(check_common(batch, heads, kv_heads, seq_len, head_dim, dtype, top_k));
  CRA_TRY(check_tensor("q", q, q_strides, batch, heads));
  CRA_TRY(check_tensor("d_o", d_o, do_strides, batch, heads));
  if (phase != 2) CRA_TRY(check_tensor("o", o, o_strides, batch, heads));
  if (phase != 1) {
    CRA_TRY(check_tensor("k", k, k_strides, batch, kv_heads));
    CRA_TRY(check_tensor("v", v, v_strides, batch, kv_heads));
    CRA_TRY(check_tensor("dq", dq, dq_strides, batch, heads));
    CRA_TRY(check_tensor("dk", dk, dk_strides, batch, kv_heads));
    CRA_TRY(check_tensor("dv", dv, dv_strides, batch, kv_heads));
  }
  if (!g_k || !g_v) return fail(CRA_ERR_INVALID_ARGUMENT, "g_k / g_v: null pointer");
  if (phase != 2 && !lse) return fail(CRA_ERR_INVALID_ARGUMENT, "lse: null pointer");
  if (phase != 1 && use_relay && !g_src) return fail(CRA_ERR_INVALID_ARGUMENT, "g_src: null with the relay active");
  if (!aligned16(g_k) || !aligned16(g_v)) return fail(CRA_ERR_MISALIGNED, "g_k / g_v: not 16-byte aligned");
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
    return fail(CRA_ERR_INVALID_ARGUMENT, "softmax_scale must be finite and > 0");
  const BwdLayout lay = bwd_layout(batch, heads, kv_heads, seq_len, head_dim, use_relay, top_k, q_len);
  const size_t need = fused ? lay.total_fused : lay.total;
  if (!workspace || workspace_bytes < need)
    return fail(CRA_ERR_WORKSPACE, "workspace: %zu bytes given, %zu needed", workspace_bytes, need);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(CRA_ERR_MISALIGNED, "workspace: base not 256-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const bool bf16 = dtype == CRA_BF16;
  const int W = cra_window(seq_len);
  const int R = rows_per_block(use_relay, top_k);
  const int NG = static_cast<int>(cra_global_rows(seq_len, use_relay, top_k));
  const int NB = (seq_len + W - 1) / W;
  const int64_t g_st[3] = {static_cast<int64_t>(kv_heads) * NG * head_dim, static_cast<int64_t>(NG) * head_dim,
                           head_dim};
  CRA_TRY(bind_context());
  BwdLaunch L;
  std::memset(&L, 0, sizeof(L));
  float* lse2 = reinterpret_cast<float*>(ws + lay.off_lse2);
  float* delta = reinterpret_cast<float*>(ws + lay.off_delta);
  QueryPassParams& qp = L.qp;
  CRA_TRY(make_tmap("q", &qp.tm_q, q, bf16, head_dim, q_len, heads, batch, q_strides));
  CRA_TRY(make_tmap("g_k", &qp.tm_gk, g_k, bf16, head_dim, NG, kv_heads, batch, g_st, kUnit));
  CRA_TRY(make_tmap("g_v", &qp.tm_gv, g_v, bf16, head_dim, NG, kv_heads, batch, g_st, kUnit));
  CRA_TRY(make_tmap("d_o", &qp.tm_do, d_o, bf16, head_dim, q_len, heads, batch, do_strides));
  CUtensorMap tm_q64, tm_do64, tm_k128, tm_v128, tm_gk128, tm_gv128, tm_ke128, tm_ve128;
  CRA_TRY(make_tmap("q", &tm_q64, q, bf16, head_dim, q_len, heads, batch, q_strides, kUnit));
  CRA_TRY(make_tmap("d_o", &tm_do64, d_o, bf16, head_dim, q_len, heads, batch, do_strides, kUnit));
  CRA_TRY(make_tmap("g_k", &tm_gk128, g_k, bf16, head_dim, NG, kv_heads, batch, g_st));
  CRA_TRY(make_tmap("g_v", &tm_gv128, g_v, bf16, head_dim, NG, kv_heads, batch, g_st));
  if (phase != 1) {
    CRA_TRY(make_tmap("k", &qp.tm_k, k, bf16, head_dim, q_len, kv_heads, batch, k_strides, kUnit));
    CRA_TRY(make_tmap("v", &qp.tm_v, v, bf16, head_dim, q_len, kv_heads, batch, v_strides, kUnit));
    CRA_TRY(make_tmap("k", &tm_k128, k, bf16, head_dim, q_len, kv_heads, batch, k_strides));
    CRA_TRY(make_tmap("v", &tm_v128, v, bf16, head_dim, q_len, kv_heads, batch, v_strides));
  }
  const bool edge = sh && sh->k_edge;
  if (edge && phase == 2) {
    CRA_TRY(make_tmap("k_edge", &qp.tm_ke, sh->k_edge, bf16, head_dim, sh->edge_len, kv_heads, batch, sh->ke_strides,
                      kUnit));
    CRA_TRY(make_tmap("v_edge", &qp.tm_ve, sh->v_edge, bf16, head_dim, sh->edge_len, kv_heads, batch, sh->ve_strides,
                      kUnit));
    CRA_TRY(make_tmap("k_edge", &tm_ke128, sh->k_edge, bf16, head_dim, sh->edge_len, kv_heads, batch,
                      sh->ke_strides));
    CRA_TRY(make_tmap("v_edge", &tm_ve128, sh->v_edge, bf16, head_dim, sh->edge_len, kv_heads, batch,
                      sh->ve_strides));
    qp.has_edge = 1;
    qp.edge_begin = static_cast<int>(sh->edge_begin);
  }
  const int k_lo = q_begin - (W - 1) > 0 ? q_begin - (W - 1) : 0;  // first key a shard query sees
  static const int64_t kNoStrides[3] = {0, 0, 0};  // tensors a shard phase does not touch
  if (!dq_strides) dq_strides = kNoStrides;
  if (!dk_strides) dk_strides = kNoStrides;
  if (!dv_strides) dv_strides = kNoStrides;
  if (!o_strides) o_strides = kNoStrides;
  qp.out = dq;
  qp.out_sb = dq_strides[0];
  qp.out_sh = dq_strides[1];
  qp.out_ss = dq_strides[2];
  qp.out_v8 = phase != 1 && rows_aligned32(dq, dq_strides, batch, heads, q_len);
  qp.lse = lse2;
  qp.delta = delta;
  qp.B = batch;
  qp.H = heads;
  qp.kv_groups = heads / kv_heads;
  qp.S = seq_len;
  qp.W = W;
  qp.R = R;
  qp.NG = NG;
  qp.n_qtiles = (q_len + kTile - 1) / kTile;
  qp.q_begin = q_begin;
  qp.q_len = q_len;
  qp.kv_begin = q_begin;
  qp.scale = softmax_scale;
  qp.scale_log2 = softmax_scale * 1.4426950408889634f;
  qp.err = dev_error;
  for (int mode = 0; mode < 2; ++mode) {
    KeyPassParams& kp = mode ? L.local : L.global;
    kp.tm_q = tm_q64;
    kp.tm_do = tm_do64;
    kp.tm_k = mode ? tm_k128 : tm_gk128;
    kp.tm_v = mode ? tm_v128 : tm_gv128;
    kp.q_lo = q_begin;
    kp.q_hi = q_begin + q_len;
    kp.q_pad = qp.n_qtiles * kTile;
    kp.k_lo = sh ? k_lo : 0;
    kp.kv_main = q_begin;
    if (mode && edge) {
      kp.has_edge = 1;
      kp.edge_begin = static_cast<int>(sh->edge_begin);
      kp.tm_ke = tm_ke128;
      kp.tm_ve = tm_ve128;
    }
    if (sh && sh->dk_halo) {
      kp.dkh = sh->dk_halo;
      kp.dvh = sh->dv_halo;
      kp.dkh_sb = sh->dkh_strides[0];
      kp.dkh_sh = sh->dkh_strides[1];
      kp.dkh_ss = sh->dkh_strides[2];
      kp.dvh_sb = sh->dvh_strides[0];
      kp.dvh_sh = sh->dvh_strides[1];
      kp.dvh_ss = sh->dvh_strides[2];
    }
    kp.lse = lse2;
    kp.delta = delta;
    kp.dk = dk;
    kp.dv = dv;
    kp.dk_sb = dk_strides[0];
    kp.dk_sh = dk_strides[1];
    kp.dk_ss = dk_strides[2];
    kp.dv_sb = dv_strides[0];
    kp.dv_sh = dv_strides[1];
    kp.dv_ss = dv_strides[2];
    kp.dkv_v8 = phase != 1 && rows_aligned32(dk, dk_strides, batch, kv_heads, q_len) &&
                rows_aligned32(dv, dv_strides, batch, kv_heads, q_len) &&
                (!sh || !sh->dk_halo ||
                 (rows_aligned32(sh->dk_halo, sh->dkh_strides, batch, kv_heads, W - 1) &&
                  rows_aligned32(sh->dv_halo, sh->dvh_strides, batch, kv_heads, W - 1)));
    kp.dgk = sh ? sh->dg_k : reinterpret_cast<float*>(ws + lay.off_dgk);
    kp.dgv = sh ? sh->dg_v : reinterpret_cast<float*>(ws + lay.off_dgv);
    kp.gsrc = g_src;
    kp.relay_scale = use_relay ? relay_log_scale : nullptr;
    kp.part_k = reinterpret_cast<float*>(ws + lay.off_pk);
    kp.part_v = reinterpret_cast<float*>(ws + lay.off_pv);
    kp.dq_acc = fused ? reinterpret_cast<float*>(ws + lay.off_dqacc) : nullptr;
    kp.B = batch;
    kp.H = heads;
    kp.kv_groups = heads / kv_heads;
    kp.S = seq_len;
    kp.W = W;
    kp.R = R;
    kp.NB = NB;
    kp.NG = NG;
    kp.top_k = top_k;
    kp.n_ktiles = (q_begin + q_len - (sh ? k_lo : 0) + kTile - 1) / kTile;
    kp.n_split = lay.n_split;
    kp.scale = softmax_scale;
    kp.scale_log2 = qp.scale_log2;
    kp.err = dev_error;
  }
  L.o = o;
  L.d_o = d_o;
  for (int i = 0; i < 3; ++i) {
    L.o_st[i] = o_strides[i];
    L.do_st[i] = do_strides[i];
  }
  L.lse_in = lse;
  L.lse2 = lse2;
  L.delta = delta;
  L.dgk = sh ? sh->dg_k : reinterpret_cast<float*>(ws + lay.off_dgk);
  L.dgv = sh ? sh->dg_v : reinterpret_cast<float*>(ws + lay.off_dgv);
  L.phase = phase;
  L.d_alpha = (use_relay && relay_log_scale) ? d_relay_log_scale : nullptr;
  L.gk_rows = g_k;
  L.gv_rows = g_v;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d_relay_log_scale && !L.d_alpha) {
    const cudaError_t me = cudaMemsetAsync(d_relay_log_scale, 0, sizeof(float) * kv_heads, st);
    if (me != cudaSuccess) return fail(CRA_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(me));
  }
  L.events = events;
  L.fused = fused;
  cudaError_t e = launch_bwd(L, head_dim, bf16, st);
  if (n_kernels) *n_kernels = L.n_kernels;
  if (kernel_ids)
    for (int i = 0; i < L.n_kernels; ++i) kernel_ids[i] = L.kernel_ids[i];
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}

}  // namespace

extern "C" {

int cra_bwd(const void* q, const void* k, const void* v, const void* o, const void* d_o, const float* lse,
            const void* g_k, const void* g_v, const int32_t* g_src, const int64_t* q_strides,
            const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
            int batch, int heads, int kv_heads, int seq_len, int head_dim, int dtype, int use_relay, int top_k,
            float softmax_scale, const float* relay_log_scale, void* dq, void* dk, void* dv,
            const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
            float* d_relay_log_scale, void* workspace, size_t workspace_bytes, int* dev_error, void* stream) {
  return bwd_impl(q, k, v, o, d_o, lse, g_k, g_v, g_src, q_strides, k_strides, v_strides, o_strides, do_strides,
                  batch, heads, kv_heads, seq_len, head_dim, dtype, use_relay, top_k, softmax_scale, relay_log_scale,
                  dq, dk, dv, dq_strides, dk_strides, dv_strides, d_relay_log_scale, workspace, workspace_bytes,
                  dev_error, stream, nullptr, nullptr, nullptr, 0);
}

int cra_bwd_fused(const void* q, const void* k, const void* v, const void* o, const void* d_o, const float* lse,
                  const void* g_k, const void* g_v, const int32_t* g_src, const int64_t* q_strides,
                  const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                  const int64_t* do_strides, int batch, int heads, int kv_heads, int seq_len, int head_dim, int dtype,
                  int use_relay, int top_k, float softmax_scale, const float* relay_log_scale, void* dq, void* dk,
                  void* dv, const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                  float* d_relay_log_scale, void* workspace, size_t workspace_bytes, int* dev_error, void* stream) {
  return bwd_impl(q, k, v, o, d_o, lse, g_k, g_v, g_src, q_strides, k_strides, v_strides, o_strides, do_strides,
                  batch, heads, kv_heads, seq_len, head_dim, dtype, use_relay, top_k, softmax_scale, relay_log_scale,
                  dq, dk, dv, dq_strides, dk_strides, dv_strides, d_relay_log_scale, workspace, workspace_bytes,
                  dev_error, stream, nullptr, nullptr, nullptr, 1);
}

size_t cra_bwd_fused_workspace_bytes(int batch, int heads, int kv_heads, int seq_len, int head_dim, int use_relay,
                                     int top_k) {
  if (check_common(batch, heads, kv_heads, seq_len, head_dim, CRA_BF16, top_k) != CRA_OK) return 0;
  return bwd_layout(batch, heads, kv_heads, seq_len, head_dim, use_relay, top_k).total_fused;
}

int cra_bwd_kernel_times(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                         const float* lse, const void* g_k, const void* g_v, const int32_t* g_src,
                         const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                         const int64_t* o_strides, const int64_t* do_strides, int batch, int heads, int kv_heads,
                         int seq_len, int head_dim, int dtype, int use_relay, int top_k, float softmax_scale,
                         const float* relay_log_scale, void* dq, void* dk, void* dv, const int64_t* dq_strides,
                         const int64_t* dk_strides, const int64_t* dv_strides, float* d_relay_log_scale,
                         void* workspace, size_t workspace_bytes, int* dev_error, void* stream, float* kernel_ms,
                         const char** kernel_names, int max_kernels, int* n_kernels, int fused) {
  if (!kernel_ms || !n_kernels) return fail(CRA_ERR_INVALID_ARGUMENT, "kernel_ms / n_kernels: null pointer");
  CRA_TRY(bind_context());
  cudaEvent_t ev[BwdLaunch::kMaxKernels + 1];
  int made = 0;
  cudaError_t e = cudaSuccess;
  for (; made <= BwdLaunch::kMaxKernels && e == cudaSuccess; ++made) e = cudaEventCreate(&ev[made]);
  if (e != cudaSuccess) made -= 1;
  int status = e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "cudaEventCreate: %s", cudaGetErrorString(e));
  int n = 0;
  int ids[BwdLaunch::kMaxKernels] = {};
  if (status == CRA_OK)
    status = bwd_impl(q, k, v, o, d_o, lse, g_k, g_v, g_src, q_strides, k_strides, v_strides, o_strides, do_strides,
                      batch, heads, kv_heads, seq_len, head_dim, dtype, use_relay, top_k, softmax_scale,
                      relay_log_scale, dq, dk, dv, dq_strides, dk_strides, dv_strides, d_relay_log_scale, workspace,
                      workspace_bytes, dev_error, stream, ev, &n, ids, fused);
  if (status == CRA_OK) {
    e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) status = fail(CRA_ERR_CUDA, "cudaStreamSynchronize: %s", cudaGetErrorString(e));
  }
  for (int i = 0; status == CRA_OK && i < n && i < max_kernels; ++i) {
    e = cudaEventElapsedTime(&kernel_ms[i], ev[i], ev[i + 1]);
    if (e != cudaSuccess) status = fail(CRA_ERR_CUDA, "cudaEventElapsedTime: %s", cudaGetErrorString(e));
    if (kernel_names) kernel_names[i] = bwd_kernel_name(ids[i]);
  }
  *n_kernels = status == CRA_OK ? (n < max_kernels ? n : max_kernels) : 0;
  for (int i = 0; i < made; ++i) cudaEventDestroy(ev[i]);
  return status;
}

int cra_relay_build_shard(const void* k, const void* v, const int64_t* k_strides, const int64_t* v_strides,
                          int batch, int kv_heads, int64_t seq_len, int64_t row_begin, int rows, int head_dim,
                          int dtype, int use_relay, int top_k, const float* relay_log_scale, void* g_k, void* g_v,
                          int32_t* g_src, void* stream) {
  CRA_TRY(check_common(batch, kv_heads, kv_heads, rows, head_dim, dtype, top_k));
  if (seq_len < 1 || seq_len > INT32_MAX) return fail(CRA_ERR_INVALID_ARGUMENT, "seq_len out of range");
  const int W = cra_window(seq_len);
  if (row_begin < 0 || row_begin % W != 0 || row_begin + rows > seq_len)
    return fail(CRA_ERR_INVALID_ARGUMENT, "shard [%lld, %lld) must start on a multiple of W = %d inside the sequence",
                static_cast<long long>(row_begin), static_cast<long long>(row_begin + rows), W);
  if (row_begin + rows != seq_len && rows % W != 0)
    return fail(CRA_ERR_INVALID_ARGUMENT, "only the last shard may end inside a W-block");
  CRA_TRY(check_tensor("k", k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor("v", v, v_strides, batch, kv_heads));
  if (!g_k || !g_v) return fail(CRA_ERR_INVALID_ARGUMENT, "g_k / g_v: null pointer");
  if (!aligned16(g_k) || !aligned16(g_v)) return fail(CRA_ERR_MISALIGNED, "g_k / g_v: not 16-byte aligned");
  const int R = rows_per_block(use_relay, top_k);
  cudaError_t e = launch_relay_build(head_dim, dtype == CRA_BF16, k, v, k_strides, v_strides, batch, kv_heads, rows,
                                     W, top_k, R, static_cast<int>(row_begin),
                                     use_relay ? relay_log_scale : nullptr, g_k, g_v, use_relay ? g_src : nullptr,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}

int cra_fwd_shard(const void* q, const void* k, const void* v, const void* g_k, const void* g_v,
                  const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int batch, int heads,
                  int kv_heads, int64_t seq_len, int64_t q_begin, int q_len, int64_t kv_begin, int kv_len,
                  const void* k_edge, const void* v_edge, const int64_t* ke_strides, const int64_t* ve_strides,
                  int64_t edge_begin, int edge_len, int head_dim, int dtype, int use_relay, int top_k,
                  float softmax_scale, void* o, const int64_t* o_strides, float* lse, int* dev_error, void* stream) {
  CRA_TRY(check_common(batch, heads, kv_heads, q_len, head_dim, dtype, top_k));
  if (seq_len < 1 || seq_len > INT32_MAX) return fail(CRA_ERR_INVALID_ARGUMENT, "seq_len out of range");
  const int W = cra_window(seq_len);
  if (q_begin < 0 || q_begin + q_len > seq_len) return fail(CRA_ERR_INVALID_ARGUMENT, "query shard outside the sequence");
  const bool edge = k_edge != nullptr || v_edge != nullptr;
  if (edge) {
    if (!k_edge || !v_edge) return fail(CRA_ERR_INVALID_ARGUMENT, "k_edge / v_edge: give both or neither");
    if (kv_begin != q_begin) return fail(CRA_ERR_INVALID_ARGUMENT, "with an edge copy K/V rows start at q_begin");
    const int64_t need_lo = q_begin - (W - 1) > 0 ? q_begin - (W - 1) : 0;
    const int64_t need_hi = std::min<int64_t>(q_begin + W + 255, q_begin + q_len);
    if (edge_begin < 0 || edge_begin > need_lo || edge_begin + edge_len < need_hi)
      return fail(CRA_ERR_INVALID_ARGUMENT,
                  "edge rows [%lld, %lld) must cover [max(q_begin - (W - 1), 0), min(q_begin + W + 255, q_begin + "
                  "q_len)) = "
                  "[%lld, %lld)",
                  static_cast<long long>(edge_begin), static_cast<long long>(edge_begin + edge_len),
                  static_cast<long long>(need_lo), static_cast<long long>(need_hi));
    CRA_TRY(check_tensor("k_edge", k_edge, ke_strides, batch, kv_heads));
    CRA_TRY(check_tensor("v_edge", v_edge, ve_strides, batch, kv_heads));
  } else if (kv_begin < 0 || kv_len < 1 || kv_begin > q_begin - (W - 1) && kv_begin > 0) {
    return fail(CRA_ERR_INVALID_ARGUMENT, "K/V rows must start at or before q_begin - (W - 1) (the local window)");
  }
  if (kv_begin + kv_len < q_begin + q_len)
    return fail(CRA_ERR_INVALID_ARGUMENT, "K/V rows must reach the last query of the shard");
  CRA_TRY(check_tensor("q", q, q_strides, batch, heads));
  CRA_TRY(check_tensor("k", k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor("v", v, v_strides, batch, kv_heads));
  CRA_TRY(check_tensor("o", o, o_strides, batch, heads));
  if (!g_k || !g_v || !lse) return fail(CRA_ERR_INVALID_ARGUMENT, "g_k / g_v / lse: null pointer");
  if (!aligned16(g_k) || !aligned16(g_v)) return fail(CRA_ERR_MISALIGNED, "g_k / g_v: not 16-byte aligned");
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
    return fail(CRA_ERR_INVALID_ARGUMENT, "softmax_scale must be finite and > 0");
  const bool bf16 = dtype == CRA_BF16;
  const int R = rows_per_block(use_relay, top_k);
  const int NG = static_cast<int>(cra_global_rows(seq_len, use_relay, top_k));
  const int64_t g_st[3] = {static_cast<int64_t>(kv_heads) * NG * head_dim, static_cast<int64_t>(NG) * head_dim,
                           head_dim};
  CRA_TRY(bind_context());
  QueryPassParams p;
  std::memset(&p, 0, sizeof(p));
  CRA_TRY(make_tmap("q", &p.tm_q, q, bf16, head_dim, q_len, heads, batch, q_strides));
  CRA_TRY(make_tmap("k", &p.tm_k, k, bf16, head_dim, kv_len, kv_heads, batch, k_strides));
  CRA_TRY(make_tmap("v", &p.tm_v, v, bf16, head_dim, kv_len, kv_heads, batch, v_strides));
  CRA_TRY(make_tmap("g_k", &p.tm_gk, g_k, bf16, head_dim, NG, kv_heads, batch, g_st));
  CRA_TRY(make_tmap("g_v", &p.tm_gv, g_v, bf16, head_dim, NG, kv_heads, batch, g_st));
  if (edge) {
    CRA_TRY(make_tmap("k_edge", &p.tm_ke, k_edge, bf16, head_dim, edge_len, kv_heads, batch, ke_strides));
    CRA_TRY(make_tmap("v_edge", &p.tm_ve, v_edge, bf16, head_dim, edge_len, kv_heads, batch, ve_strides));
    p.has_edge = 1;
    p.edge_begin = static_cast<int>(edge_begin);
  }
  p.tm_do = p.tm_q;
  p.out = o;
  p.out_sb = o_strides[0];
  p.out_sh = o_strides[1];
  p.out_ss = o_strides[2];
  p.out_v8 = rows_aligned32(o, o_strides, batch, heads, q_len);
  p.lse = lse;
  p.lse_len = q_len;
  p.B = batch;
  p.H = heads;
  p.kv_groups = heads / kv_heads;
  p.S = static_cast<int>(seq_len);
  p.W = W;
  p.R = R;
  p.NG = NG;
  p.n_qtiles = (q_len + kTile - 1) / kTile;
  p.q_begin = static_cast<int>(q_begin);
  p.q_len = q_len;
  p.kv_begin = static_cast<int>(kv_begin);
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = dev_error;
  cudaError_t e = launch_fwd(p, head_dim, bf16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// packed variable-length batches
// ---------------------------------------------------------------------------
namespace {

// Host copy of the document table for cu_seqlens (n_docs + 1 entries);
// returns the packed global-row count and the totals, or -1 on bad input.
int64_t varlen_table(const int64_t* cu, int n_docs, int top_k, DocInfo* out, int* n_pairs, int* n_blocks) {
  if (!cu || n_docs < 1 || cu[0] != 0) return -1;
  int64_t g = 0, pairs = 0, blks = 0;
  for (int d = 0; d < n_docs; ++d) {
    const int64_t len = cu[d + 1] - cu[d];
    if (len < 1 || cu[d + 1] > INT32_MAX) return -1;
    const int W = cra_window(len);
    const int R = rows_per_block(cra_relay_active(len), top_k);
    const int64_t nb = (len + W - 1) / W;
    if (out) out[d] = DocInfo{static_cast<int>(cu[d]), static_cast<int>(len), W, R, static_cast<int>(g),
                              static_cast<int>(pairs), static_cast<int>(blks), 0};
    g += nb * R;
    blks += nb;
    pairs += (len + 2 * kTile - 1) / (2 * kTile);
    if (g > INT32_MAX || pairs > INT32_MAX) return -1;
  }
  if (n_pairs) *n_pairs = static_cast<int>(pairs);
  if (n_blocks) *n_blocks = static_cast<int>(blks);
  return g;
}

}  // namespace

extern "C" {

size_t cra_varlen_table_bytes(int n_docs) { return n_docs > 0 ? sizeof(DocInfo) * n_docs : 0; }

int64_t cra_varlen_global_rows(const int64_t* cu_seqlens, int n_docs, int top_k) {
  if (top_k < 1 || top_k > 4) return -1;
  return varlen_table(cu_seqlens, n_docs, top_k, nullptr, nullptr, nullptr);
}

int64_t cra_varlen_blocks(const int64_t* cu_seqlens, int n_docs) {
  int nb = 0;
  return varlen_table(cu_seqlens, n_docs, 2, nullptr, nullptr, &nb) < 0 ? -1 : nb;
}

int cra_varlen_plan(const int64_t* cu_seqlens, int n_docs, int top_k, void* table, void* stream) {
  if (top_k < 1 || top_k > 4) return fail(CRA_ERR_UNSUPPORTED, "top_k %d outside 1..4", top_k);
  if (!table) return fail(CRA_ERR_INVALID_ARGUMENT, "table: null pointer");
  if (varlen_table(cu_seqlens, n_docs, top_k, nullptr, nullptr, nullptr) < 0)
    return fail(CRA_ERR_INVALID_ARGUMENT, "cu_seqlens must start at 0 and increase strictly (n_docs %d)", n_docs);
  CRA_TRY(bind_context());
  // pageable source: cudaMemcpyAsync stages it before returning, so the
  // temporary may go out of scope
  DocInfo* host = new DocInfo[n_docs];
  varlen_table(cu_seqlens, n_docs, top_k, host, nullptr, nullptr);
  const cudaError_t e = cudaMemcpyAsync(table, host, sizeof(DocInfo) * n_docs, cudaMemcpyHostToDevice,
                                        static_cast<cudaStream_t>(stream));
  delete[] host;
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "cudaMemcpyAsync: %s", cudaGetErrorString(e));
}

int cra_relay_build_varlen(const void* k, const void* v, const int64_t* k_strides, const int64_t* v_strides,
                           int batch, int kv_heads, const int64_t* cu_seqlens, int n_docs, const void* table,
                           int head_dim, int dtype, int top_k, const float* relay_log_scale, void* g_k, void* g_v,
                           int32_t* g_src, void* stream) {
  int nb = 0;
  const int64_t NG = varlen_table(cu_seqlens, n_docs, top_k, nullptr, nullptr, &nb);
  if (NG < 0) return fail(CRA_ERR_INVALID_ARGUMENT, "cu_seqlens must start at 0 and increase strictly");
  const int64_t T = cu_seqlens[n_docs];
  CRA_TRY(check_common(batch, kv_heads, kv_heads, static_cast<int>(T), head_dim, dtype, top_k));
  CRA_TRY(check_tensor("k", k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor("v", v, v_strides, batch, kv_heads));
  if (!g_k || !g_v || !g_src || !table) return fail(CRA_ERR_INVALID_ARGUMENT, "g_k / g_v / g_src / table: null");
  if (!aligned16(g_k) || !aligned16(g_v)) return fail(CRA_ERR_MISALIGNED, "g_k / g_v: not 16-byte aligned");
  cudaError_t e = launch_relay_build(head_dim, dtype == CRA_BF16, k, v, k_strides, v_strides, batch, kv_heads,
                                     static_cast<int>(T), 1, top_k, 1, 0, relay_log_scale, g_k, g_v, g_src,
                                     static_cast<cudaStream_t>(stream), static_cast<const DocInfo*>(table), n_docs, nb,
                                     static_cast<int>(NG));
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}

int cra_fwd_varlen(const void* q, const void* k, const void* v, const void* g_k, const void* g_v,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int batch, int heads,
                   int kv_heads, const int64_t* cu_seqlens, int n_docs, const void* table, int head_dim, int dtype,
                   int top_k, float softmax_scale, void* o, const int64_t* o_strides, float* lse, int* dev_error,
                   void* stream) {
  int n_pairs = 0;
  const int64_t NG = varlen_table(cu_seqlens, n_docs, top_k, nullptr, &n_pairs, nullptr);
  if (NG < 0) return fail(CRA_ERR_INVALID_ARGUMENT, "cu_seqlens must start at 0 and increase strictly");
  const int64_t T = cu_seqlens[n_docs];
  CRA_TRY(check_common(batch, heads, kv_heads, static_cast<int>(T), head_dim, dtype, top_k));
  CRA_TRY(check_tensor("q", q, q_strides, batch, heads));
  CRA_TRY(check_tensor("k", k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor("v", v, v_strides, batch, kv_heads));
  CRA_TRY(check_tensor("o", o, o_strides, batch, heads));
  if (!g_k || !g_v || !lse || !table) return fail(CRA_ERR_INVALID_ARGUMENT, "g_k / g_v / lse / table: null");
  if (!aligned16(g_k) || !aligned16(g_v)) return fail(CRA_ERR_MISALIGNED, "g_k / g_v: not 16-byte aligned");
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
    return fail(CRA_ERR_INVALID_ARGUMENT, "softmax_scale must be finite and > 0");
  const bool bf16 = dtype == CRA_BF16;
  const int64_t g_st[3] = {static_cast<int64_t>(kv_heads) * NG * head_dim, NG * head_dim, head_dim};
  CRA_TRY(bind_context());
  QueryPassParams p;
  std::memset(&p, 0, sizeof(p));
  CRA_TRY(make_tmap("q", &p.tm_q, q, bf16, head_dim, T, heads, batch, q_strides));
  CRA_TRY(make_tmap("k", &p.tm_k, k, bf16, head_dim, T, kv_heads, batch, k_strides));
  CRA_TRY(make_tmap("v", &p.tm_v, v, bf16, head_dim, T, kv_heads, batch, v_strides));
  CRA_TRY(make_tmap("g_k", &p.tm_gk, g_k, bf16, head_dim, NG, kv_heads, batch, g_st));
  CRA_TRY(make_tmap("g_v", &p.tm_gv, g_v, bf16, head_dim, NG, kv_heads, batch, g_st));
  p.tm_do = p.tm_q;
  p.out = o;
  p.out_sb = o_strides[0];
  p.out_sh = o_strides[1];
  p.out_ss = o_strides[2];
  p.out_v8 = rows_aligned32(o, o_strides, batch, heads, T);
  p.lse = lse;
  p.lse_len = static_cast<int>(T);
  p.B = batch;
  p.H = heads;
  p.kv_groups = heads / kv_heads;
  p.S = static_cast<int>(T);
  p.W = 1;
  p.R = 1;
  p.NG = static_cast<int>(NG);
  p.q_len = static_cast<int>(T);
  p.docs = static_cast<const DocInfo*>(table);
  p.n_docs = n_docs;
  p.n_pairs_total = n_pairs;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = dev_error;
  cudaError_t e = launch_fwd(p, head_dim, bf16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CRA_OK : fail(CRA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
}

}  // extern "C"

extern "C" {

size_t cra_bwd_shard_workspace_bytes(int batch, int heads, int kv_heads, int64_t seq_len, int q_len, int head_dim,
                                     int use_relay, int top_k) {
  if (seq_len < 1 || seq_len > INT32_MAX || q_len < 1) return 0;
  if (check_common(batch, heads, kv_heads, static_cast<int>(seq_len), head_dim, CRA_BF16, top_k) != CRA_OK) return 0;
  return bwd_layout(batch, heads, kv_heads, static_cast<int>(seq_len), head_dim, use_relay, top_k, q_len).total;
}

namespace {
int check_shard(int64_t seq_len, int64_t q_begin, int q_len) {
  if (seq_len < 1 || seq_len > INT32_MAX) return fail(CRA_ERR_INVALID_ARGUMENT, "seq_len out of range");
  const int W = cra_window(seq_len);
  if (q_begin < 0 || q_len < 1 || q_begin + q_len > seq_len || q_begin % W != 0)
    return fail(CRA_ERR_INVALID_ARGUMENT, "query shard [%lld, %lld) must start on a multiple of W = %d inside the sequence",
                static_cast<long long>(q_begin), static_cast<long long>(q_begin + q_len), W);
  return CRA_OK;
}
}  // namespace

int cra_bwd_shard_global(const void* q, const void* o, const void* d_o, const float* lse, const void* g_k,
                         const void* g_v, const int64_t* q_strides, const int64_t* o_strides,
                         const int64_t* do_strides, int batch, int heads, int kv_heads, int64_t seq_len,
                         int64_t q_begin, int q_len, int head_dim, int dtype, int use_relay, int top_k,
                         float softmax_scale, float* dg_k, float* dg_v, void* workspace, size_t workspace_bytes,
                         int* dev_error, void* stream) {
  CRA_TRY(check_shard(seq_len, q_begin, q_len));
  if (!dg_k || !dg_v) return fail(CRA_ERR_INVALID_ARGUMENT, "dg_k / dg_v: null pointer");
  ShardSpec sh{};
  sh.phase = 1;
  sh.q_begin = q_begin;
  sh.q_len = q_len;
  sh.dg_k = dg_k;
  sh.dg_v = dg_v;
  return bwd_impl(q, nullptr, nullptr, o, d_o, lse, g_k, g_v, nullptr, q_strides, nullptr, nullptr, o_strides,
                  do_strides, batch, heads, kv_heads, static_cast<int>(seq_len), head_dim, dtype, use_relay, top_k,
                  softmax_scale, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, workspace,
                  workspace_bytes, dev_error, stream, nullptr, nullptr, nullptr, 0, &sh);
}

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
                        void* stream) {
  CRA_TRY(check_shard(seq_len, q_begin, q_len));
  if (!dg_k || !dg_v) return fail(CRA_ERR_INVALID_ARGUMENT, "dg_k / dg_v: null pointer");
  const int W = cra_window(seq_len);
  const int64_t k_lo = q_begin - (W - 1) > 0 ? q_begin - (W - 1) : 0;
  ShardSpec sh{};
  sh.phase = 2;
  sh.q_begin = q_begin;
  sh.q_len = q_len;
  sh.dg_k = const_cast<float*>(dg_k);
  sh.dg_v = const_cast<float*>(dg_v);
  if (q_begin > 0) {
    const int64_t need_hi = std::min<int64_t>(q_begin + kTile, q_begin + q_len);
    if (!k_edge || !v_edge || edge_begin > k_lo || edge_begin + edge_len < need_hi)
      return fail(CRA_ERR_INVALID_ARGUMENT,
                  "k_edge / v_edge must cover keys [%lld, %lld) (the halo and the shard's first 128 rows)",
                  static_cast<long long>(k_lo), static_cast<long long>(need_hi));
    if (!dk_halo || !dv_halo || !dkh_strides || !dvh_strides)
      return fail(CRA_ERR_INVALID_ARGUMENT, "dk_halo / dv_halo: null (the shard has a halo of %lld keys)",
                  static_cast<long long>(q_begin - k_lo));
    CRA_TRY(check_tensor("k_edge", k_edge, ke_strides, batch, kv_heads));
    CRA_TRY(check_tensor("v_edge", v_edge, ve_strides, batch, kv_heads));
    CRA_TRY(check_tensor("dk_halo", dk_halo, dkh_strides, batch, kv_heads));
    CRA_TRY(check_tensor("dv_halo", dv_halo, dvh_strides, batch, kv_heads));
    sh.k_edge = k_edge;
    sh.v_edge = v_edge;
    sh.ke_strides = ke_strides;
    sh.ve_strides = ve_strides;
    sh.edge_begin = edge_begin;
    sh.edge_len = edge_len;
    sh.dk_halo = dk_halo;
    sh.dv_halo = dv_halo;
    sh.dkh_strides = dkh_strides;
    sh.dvh_strides = dvh_strides;
  }
  return bwd_impl(q, k, v, nullptr, d_o, nullptr, g_k, g_v, g_src, q_strides, k_strides, v_strides, nullptr,
                  do_strides, batch, heads, kv_heads, static_cast<int>(seq_len), head_dim, dtype, use_relay, top_k,
                  softmax_scale, relay_log_scale, dq, dk, dv, dq_strides, dk_strides, dv_strides, d_relay_log_scale,
                  workspace, workspace_bytes, dev_error, stream, nullptr, nullptr, nullptr, 0, &sh);
}

}  // extern "C"
