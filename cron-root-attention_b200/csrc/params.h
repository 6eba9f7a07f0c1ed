// params.h -- kernel parameter blocks and internal launch entry points.
// Host code (capi.cu) fills these; kernels receive them as __grid_constant__.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cra {

// Query-centric attention pass (forward, and the dQ pass of the backward).
struct alignas(64) QueryPassParams {
  CUtensorMap tm_q;   // [B, H,   S,  D]
  CUtensorMap tm_k;   // [B, Hkv, S,  D]
  CUtensorMap tm_v;   // [B, Hkv, S,  D]
  CUtensorMap tm_gk;  // [B, Hkv, NG, D]
  CUtensorMap tm_gv;  // [B, Hkv, NG, D]
  CUtensorMap tm_do;  // [B, H,   S,  D]   (backward only)
  void* out;          // forward: O;  backward: dQ  (element strides below)
  int64_t out_sb, out_sh, out_ss;
  float* lse;         // [B, H, S] fp32, natural log (written by fwd, read by bwd)
  const float* delta; // [B, H, S] fp32, rowsum(O * dO) (backward only)
  int B, H, kv_groups, S, W, R, NG, n_qtiles;
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
  const float* dgk; const float* dgv;
  const int32_t* gsrc;     // [B, Hkv, NB, TOP_K]
  const float* relay_scale;// [Hkv] exp(alpha) per kv head, or null
  // global mode: fp32 partial outputs [n_split, B, Hkv, NG, D]
  float* part_k; float* part_v;
  int B, H, kv_groups, S, W, R, NB, NG, top_k;
  int n_ktiles;       // key tiles per (b, hkv)
  int n_split;        // global mode: query splits per key tile
  float scale, scale_log2;
  int* err;
};

}  // namespace cra
