// relay.cu -- builds the packed global-row list (strided + relay rows) that
// the attention kernels read as one contiguous matrix per (b, h).
//
// Reference: _relay_precompute_topk, cron_root_attention/core.py:2630-2748,
// and the optional relay scale core.py:3541-3544.
//   * per W-block r: ||k_i||^2 in fp32 over the block's valid rows; keep the
//     TOP_K largest, ties to the lower index (the reference's strict '>'
//     insertion sort, core.py:2685-2703);
//   * relay rows are exact copies of k / v at the chosen positions (best
//     first, core.py:2715-2730), multiplied by exp(relay_log_scale[h])
//     rounded to the element type when a scale is given (the reference does
//     `relay_k * exp(a).to(dtype)`);
//   * the source positions are written as int32 (the reference stores them
//     as float32, exact below 2^24, core.py:2807).
// Rows are indexed locally (0 .. S-1 of the given k / v); pos0 is the
// absolute sequence position of local row 0 (non-zero for one GPU's shard of
// a sequence split across GPUs, always a multiple of W), added to the
// written source positions.
// Here each W-block is also given its strided row k[r*W] (the phase-2 key,
// core.py:1042-1087) so that the attention kernels see one prefix-visible
// list (geom.cuh).
//
// One warp per block, one lane per row: a lane loads its whole row (D/8
// 16-byte loads, all in flight before use), computes the fp32 norm and keeps
// its own top-4; the warp merges the 32 lists with a shuffle tree.  The scan
// is a single pass over K with 8 KB in flight per warp.
#include "geom.cuh"
#include "params.h"
#include "sm100.cuh"

namespace cra {

struct Cand {
  float n;
  int i;
};
__device__ __forceinline__ bool better(const Cand& a, const Cand& b) { return a.n > b.n || (a.n == b.n && a.i < b.i); }

template <int D, bool BF16>
__global__ void __launch_bounds__(128) relay_build_kernel(const void* __restrict__ kp, const void* __restrict__ vp,
                                                          int64_t k_sb, int64_t k_sh, int64_t k_ss, int64_t v_sb,
                                                          int64_t v_sh, int64_t v_ss, int Hkv, int S, int W, int NB,
                                                          int top_k, int R, int pos0, const float* __restrict__ log_scale,
                                                          void* __restrict__ gkp, void* __restrict__ gvp,
                                                          int32_t* __restrict__ gsrc, const DocInfo* __restrict__ docs,
                                                          int n_docs, int NG) {
  using E = Elt<BF16>;
  using T = typename E::T;
  constexpr int LPR = D / 8;          // lanes per row
  constexpr int RPS = 32 / LPR;       // rows per warp step
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int r = blockIdx.x * 4 + warp;
  const int h = blockIdx.y, b = blockIdx.z;
  if (r >= NB) return;
  const T* k = reinterpret_cast<const T*>(kp) + b * k_sb + h * k_sh;
  const T* v = reinterpret_cast<const T*>(vp) + b * v_sb + h * v_sh;
  // output: global rows from g_row, source slot from src_slot
  int64_t g_row = (static_cast<int64_t>(b) * Hkv + h) * static_cast<int64_t>(NB) * R + static_cast<int64_t>(r) * R;
  int64_t src_slot = (static_cast<int64_t>(b) * Hkv + h) * NB + r;
  if (docs) {  // packed variable-length batch: block r of the whole batch -> document, local block
    int lo = 0, hi = n_docs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (docs[mid].blk0 <= r) lo = mid; else hi = mid - 1;
    }
    const DocInfo dc = docs[lo];
    k += static_cast<int64_t>(dc.start) * k_ss;
    v += static_cast<int64_t>(dc.start) * v_ss;
    S = dc.len;
    W = dc.W;
    R = dc.R;
    r -= dc.blk0;
    g_row = (static_cast<int64_t>(b) * Hkv + h) * NG + dc.g0 + static_cast<int64_t>(r) * R;
    // src_slot stays the batch-wide block index; positions are document-local
  }
  const int row_lo = r * W;
  const int row_hi = min(row_lo + W, S);
  const int sub = lane / LPR, part = lane % LPR;

  Cand best[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) best[t] = Cand{-1.f, row_lo};

  if (R > 1) {
    // lane-per-row scan: lane l takes rows row_lo + l, row_lo + l + 32, ...;
    // all D/8 16-byte loads of a row are issued before use (the other half
    // of each 32-byte sector comes from L1 on the lane's next load)
    for (int i0 = row_lo; i0 < row_hi; i0 += 32) {
      const int i = i0 + lane;
      if (i < row_hi) {
        const uint4* rp = reinterpret_cast<const uint4*>(k + static_cast<int64_t>(i) * k_ss);
        uint4 u[D / 8];
#pragma unroll
        for (int q = 0; q < D / 8; ++q) u[q] = rp[q];
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int q = 0; q < D / 8; ++q) {
          const uint32_t w[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack(w[e]);
            a0 = fmaf(f.x, f.x, a0);
            a1 = fmaf(f.y, f.y, a1);
          }
        }
        Cand c{a0 + a1, i};
        // insertion into this lane's sorted top-4 list
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (better(c, best[t])) {
            const Cand tmp = best[t];
            best[t] = c;
            c = tmp;
          }
        }
      }
    }
    // merge the 32 lanes' lists (tree; the selection order is a total order,
    // so the merge order does not matter), result in every lane
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      Cand in[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        in[t].n = __shfl_xor_sync(0xffffffffu, best[t].n, off);
        in[t].i = __shfl_xor_sync(0xffffffffu, best[t].i, off);
      }
#pragma unroll
      for (int t2 = 0; t2 < 4; ++t2) {
        Cand c = in[t2];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (better(c, best[t])) {
            const Cand tmp = best[t];
            best[t] = c;
            c = tmp;
          }
        }
      }
    }
  }

  // Write the block's R global rows: strided row, then top_k relay rows.
  T* gk = reinterpret_cast<T*>(gkp) + g_row * D;
  T* gv = reinterpret_cast<T*>(gvp) + g_row * D;
  float sc = 1.f;
  if (log_scale) sc = E::to_f(E::from_f(expf(log_scale[h])));
  // each row: D/8 16-byte units; the warp covers RPS rows per pass
  for (int t0 = 0; t0 < R; t0 += RPS) {
    const int t = t0 + sub;
    if (t < R) {
      int src;
      if (t == 0) {
        src = row_lo;
      } else {
        src = best[0].i;
#pragma unroll
        for (int q = 1; q < 4; ++q)
          if (t - 1 == q) src = best[q].i;
      }
      uint4 uk = *reinterpret_cast<const uint4*>(k + static_cast<int64_t>(src) * k_ss + part * 8);
      uint4 uv = *reinterpret_cast<const uint4*>(v + static_cast<int64_t>(src) * v_ss + part * 8);
      if (t > 0 && log_scale) {
        uint32_t* wk = reinterpret_cast<uint32_t*>(&uk);
        uint32_t* wv = reinterpret_cast<uint32_t*>(&uv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 fk = E::unpack(wk[e]);
          float2 fv = E::unpack(wv[e]);
          wk[e] = E::pack(fk.x * sc, fk.y * sc);
          wv[e] = E::pack(fv.x * sc, fv.y * sc);
        }
      }
      *reinterpret_cast<uint4*>(gk + t * D + part * 8) = uk;
      *reinterpret_cast<uint4*>(gv + t * D + part * 8) = uv;
      if (t > 0 && part == 0 && gsrc)
        gsrc[src_slot * top_k + (t - 1)] = src + pos0;
    }
  }
}

// host-side launcher (called from capi.cu)
cudaError_t launch_relay_build(int D, bool bf16, const void* k, const void* v, const int64_t* ks, const int64_t* vs,
                               int B, int Hkv, int S, int W, int top_k, int R, int pos0, const float* log_scale,
                               void* gk, void* gv, int32_t* gsrc, cudaStream_t stream, const DocInfo* docs,
                               int n_docs, int NB_total, int NG_total) {
  const int NB = docs ? NB_total : (S + W - 1) / W;
  dim3 grid((NB + 3) / 4, Hkv, B);
#define CRA_RELAY(DD, BB)                                                                                          \
  relay_build_kernel<DD, BB><<<grid, 128, 0, stream>>>(k, v, ks[0], ks[1], ks[2], vs[0], vs[1], vs[2], Hkv, S, W, \
                                                       NB, top_k, R, pos0, log_scale, gk, gv, gsrc, docs, n_docs, NG_total)
  if (D == 128) {
    if (bf16) CRA_RELAY(128, true); else CRA_RELAY(128, false);
  } else {
    if (bf16) CRA_RELAY(64, true); else CRA_RELAY(64, false);
  }
#undef CRA_RELAY
  return cudaGetLastError();
}

}  // namespace cra
