// capi.cu -- the extern "C" entry points declared in include/cra.h: argument
// validation, TMA tensor-map construction and kernel launches.  Stateless and
// reentrant: nothing is cached across calls except the driver entry point
// for cuTensorMapEncodeTiled and per-kernel shared-memory attributes.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "../../include/cra.h"
#include "geom.cuh"
#include "params.h"

namespace cra {
cudaError_t launch_relay_build(int D, bool bf16, const void* k, const void* v, const int64_t* ks, const int64_t* vs,
                               int B, int Hkv, int S, int W, int top_k, int R, const float* log_scale, void* gk,
                               void* gv, int32_t* gsrc, cudaStream_t stream);
cudaError_t launch_fwd(const QueryPassParams& p, int D, bool bf16, cudaStream_t stream);
}  // namespace cra

using namespace cra;

namespace {

constexpr int kVersion = 100;  // 0.1.0

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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Checks one [dim0, dim1, rows, D] tensor description.
int check_tensor(const void* p, const int64_t* st, int dim0, int dim1) {
  if (!p || !st) return CRA_ERR_INVALID_ARGUMENT;
  if (!aligned16(p)) return CRA_ERR_MISALIGNED;
  for (int i = 0; i < 3; ++i) {
    if (st[i] < 0) return CRA_ERR_INVALID_ARGUMENT;
    if (st[i] % 8 != 0) {
      const int extent = i == 0 ? dim0 : (i == 1 ? dim1 : 2);
      if (extent > 1) return CRA_ERR_MISALIGNED;  // stride of a size-1 dim is never used
    }
  }
  return CRA_OK;
}

// 4-D tensor map over [d1 (outer), d0, rows, D] with 128 x 64 boxes, 128B swizzle.
int make_tmap(CUtensorMap* m, const void* base, bool bf16, int D, int64_t rows, int64_t d0, int64_t d1,
              const int64_t* st) {
  auto fn = encode_fn();
  if (!fn) return CRA_ERR_DRIVER;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(d0),
                        static_cast<cuuint64_t>(d1)};
  // byte strides of dims 1..3; a size-1 dim gets a harmless valid stride
  int64_t s_rows = st[2], s_h = st[1], s_b = st[0];
  if (rows <= 1) s_rows = D;
  if (d0 <= 1) s_h = s_rows * rows;
  if (d1 <= 1) s_b = s_h * d0;
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_rows * 2), static_cast<cuuint64_t>(s_h * 2),
                           static_cast<cuuint64_t>(s_b * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(kTile), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CRA_OK : CRA_ERR_INVALID_ARGUMENT;
}

int check_common(int batch, int heads, int kv_heads, int seq_len, int head_dim, int dtype, int top_k) {
  if (batch < 1 || heads < 1 || kv_heads < 1 || seq_len < 1) return CRA_ERR_INVALID_ARGUMENT;
  if (heads % kv_heads != 0) return CRA_ERR_INVALID_ARGUMENT;
  if (batch > 65535 || heads > 65535) return CRA_ERR_INVALID_ARGUMENT;
  if (dtype != CRA_F16 && dtype != CRA_BF16) return CRA_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return CRA_ERR_UNSUPPORTED;
  if (top_k < 1 || top_k > 4) return CRA_ERR_UNSUPPORTED;
  return CRA_OK;
}

int rows_per_block(int use_relay, int top_k) { return use_relay ? 1 + top_k : 1; }

#define CRA_TRY(x)                \
  do {                            \
    const int _s = (x);           \
    if (_s != CRA_OK) return _s;  \
  } while (0)

}  // namespace

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
  CRA_TRY(check_tensor(k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor(v, v_strides, batch, kv_heads));
  if (!g_k || !g_v) return CRA_ERR_INVALID_ARGUMENT;
  if (!aligned16(g_k) || !aligned16(g_v)) return CRA_ERR_MISALIGNED;
  const int W = cra_window(seq_len);
  const int R = rows_per_block(use_relay, top_k);
  cudaError_t e = launch_relay_build(head_dim, dtype == CRA_BF16, k, v, k_strides, v_strides, batch, kv_heads,
                                     seq_len, W, top_k, R, use_relay ? relay_log_scale : nullptr, g_k, g_v,
                                     use_relay ? g_src : nullptr, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CRA_OK : CRA_ERR_CUDA;
}

int cra_fwd(const void* q, const void* k, const void* v, const void* g_k, const void* g_v, const int64_t* q_strides,
            const int64_t* k_strides, const int64_t* v_strides, int batch, int heads, int kv_heads, int seq_len,
            int head_dim, int dtype, int use_relay, int top_k, float softmax_scale, void* o, const int64_t* o_strides,
            float* lse, int* dev_error, void* stream) {
  CRA_TRY(check_common(batch, heads, kv_heads, seq_len, head_dim, dtype, top_k));
  CRA_TRY(check_tensor(q, q_strides, batch, heads));
  CRA_TRY(check_tensor(k, k_strides, batch, kv_heads));
  CRA_TRY(check_tensor(v, v_strides, batch, kv_heads));
  CRA_TRY(check_tensor(o, o_strides, batch, heads));
  if (!g_k || !g_v || !lse) return CRA_ERR_INVALID_ARGUMENT;
  if (!aligned16(g_k) || !aligned16(g_v)) return CRA_ERR_MISALIGNED;
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale)) return CRA_ERR_INVALID_ARGUMENT;
  const bool bf16 = dtype == CRA_BF16;
  const int W = cra_window(seq_len);
  const int R = rows_per_block(use_relay, top_k);
  const int NG = static_cast<int>(cra_global_rows(seq_len, use_relay, top_k));
  const int64_t g_st[3] = {static_cast<int64_t>(kv_heads) * NG * head_dim, static_cast<int64_t>(NG) * head_dim,
                           head_dim};
  QueryPassParams p;
  std::memset(&p, 0, sizeof(p));
  CRA_TRY(make_tmap(&p.tm_q, q, bf16, head_dim, seq_len, heads, batch, q_strides));
  CRA_TRY(make_tmap(&p.tm_k, k, bf16, head_dim, seq_len, kv_heads, batch, k_strides));
  CRA_TRY(make_tmap(&p.tm_v, v, bf16, head_dim, seq_len, kv_heads, batch, v_strides));
  CRA_TRY(make_tmap(&p.tm_gk, g_k, bf16, head_dim, NG, kv_heads, batch, g_st));
  CRA_TRY(make_tmap(&p.tm_gv, g_v, bf16, head_dim, NG, kv_heads, batch, g_st));
  p.tm_do = p.tm_q;
  p.out = o;
  p.out_sb = o_strides[0];
  p.out_sh = o_strides[1];
  p.out_ss = o_strides[2];
  p.lse = lse;
  p.delta = nullptr;
  p.B = batch;
  p.H = heads;
  p.kv_groups = heads / kv_heads;
  p.S = seq_len;
  p.W = W;
  p.R = R;
  p.NG = NG;
  p.n_qtiles = (seq_len + kTile - 1) / kTile;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = dev_error;
  cudaError_t e = launch_fwd(p, head_dim, bf16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CRA_OK : CRA_ERR_CUDA;
}

}  // extern "C"
