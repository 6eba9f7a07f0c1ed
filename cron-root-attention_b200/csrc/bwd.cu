// bwd.cu -- backward pass of the causal 3-phase sqrt(N) attention on sm_100a.
//
// Math (reference: CronRootAttentionV14Function.backward, core.py:3626-3759;
// kernels core.py:1165-1316, 1650-1745, 1755-1889, 2381-2492, 2767-2815):
//   Di  = sum_d O * dO                              (core.py:1220)
//   P   = exp(s - lse),  dS = P * (dO . v - Di)     (core.py:1242-1246)
//   dQ  = scale * dS K,  dK = scale * dS^T Q,  dV = P^T dO
//   relay-row gradients land on their source tokens (core.py:2811-2815).
//
// Kernels, in launch order:
//   delta_kernel     -Di and -lse*log2(e), padded to whole 128-query tiles;
//                    fused: also zeroes the fp32 dQ accumulator.
//   keyglobal_kernel one CTA per (128 global rows, query split): dG_k / dG_v
//                    over every query that sees the rows; fp32 partials per
//                    split (no atomics).
//   reduce_kernel    sums the splits in a fixed order -> dG (fp32).
//   dalpha_kernel    d(relay_log_scale) = sum over relay rows of dG * G
//                    (only when a relay scale is used).
//   keylocal_kernel  persistent (one CTA per SM) over 128-key tiles: dK / dV
//                    over the local band, then folds in dG of the tile's
//                    strided key and of every relay row whose source lies in
//                    the tile, and stores.
//   then either (cra_bwd_fused, head_dim 128)
//   dq_convert_kernel dQ = scale * accumulator, to the output dtype: the two
//                    key passes have already added dS K of every unit into
//                    the fp32 accumulator (a fifth GEMM per unit, dQ^T = K^T
//                    dS^T, read out of TMEM and added with fp32 atomics), so
//                    the scores are recomputed once instead of twice;
//   or (cra_bwd, the default: every sum in a fixed order)
//   dq_kernel        persistent (one CTA per SM) over 128-query tiles: dQ over
//                    band + global prefix.
// dK, dV and dG always have a fixed summation order; only the fused dQ does
// not (fp32 atomic adds).
//
// The attention kernels use the warp roles of the forward (fwd.cu): warp 0
// TMA producer, warp 1 tcgen05 issuer (whole warp, one elected lane) + TMEM
// owner, warps 2-5 and 6-9 two softmax warpgroups, one row per thread (TMEM
// lane = row); the persistent kernels add an epilogue warpgroup.
#include "geom.cuh"
#include "params.h"
#include "sm100.cuh"

#include <type_traits>

namespace cra {

constexpr float kLog2e = 1.4426950408889634f;

// Bit e set iff column e of a 32-column chunk lies in [lo, hi) (bounds
// relative to the chunk's first column, any range).
__device__ __forceinline__ uint32_t col_mask32(int lo, int hi) {
  const int a = min(max(lo, 0), 32), z = min(max(hi, 0), 32);
  const uint32_t mz = z >= 32 ? 0xffffffffu : ((1u << z) - 1u);
  const uint32_t ma = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
  return mz & ~ma;
}

// Key-centric softmax of one 32-column chunk (columns = queries): P^T =
// 2^(s scale log2e + nlse) and dS^T = P^T (dP^T + ndelta), with the per-query
// nlse = -lse log2e and ndelta = -Di read four at a time from shared memory
// (warp-wide broadcasts) and the arithmetic done two columns per f32x2
// instruction.  Columns outside `m` give 0; a warp whose chunk is entirely
// visible skips the selects.
template <typename E>
__device__ __forceinline__ void key_softmax_chunk(const float (&s)[32], const float (&dp)[32],
                                                  const float* __restrict__ nlse, const float* __restrict__ ndi,
                                                  float sl2, uint32_t m, uint32_t (&ppk)[16], uint32_t (&dpk)[16]) {
  const float2 sl2x2 = make_float2(sl2, sl2);
  auto body = [&](auto masked) {
#pragma unroll
    for (int e4 = 0; e4 < 8; ++e4) {
      const float4 l = reinterpret_cast<const float4*>(nlse)[e4];
      const float4 d = reinterpret_cast<const float4*>(ndi)[e4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e = 4 * e4 + 2 * h;
        const float2 x = fma2(make_float2(s[e], s[e + 1]), sl2x2, h ? make_float2(l.z, l.w) : make_float2(l.x, l.y));
        float p0 = ex2(x.x), p1 = ex2(x.y);
        if constexpr (decltype(masked)::value) {
          p0 = (m >> e) & 1u ? p0 : 0.f;
          p1 = (m >> (e + 1)) & 1u ? p1 : 0.f;
        }
        const float2 ds = mul2(make_float2(p0, p1),
                               add2(make_float2(dp[e], dp[e + 1]), h ? make_float2(d.z, d.w) : make_float2(d.x, d.y)));
        ppk[e / 2] = E::pack(p0, p1);
        dpk[e / 2] = E::pack(ds.x, ds.y);
      }
    }
  };
  if (__all_sync(0xffffffffu, m == 0xffffffffu))
    body(std::false_type{});
  else
    body(std::true_type{});
}

// Fused backward: row r (key) of the unit's dS^T, chunk c (queries [32c,
// 32c+32), 16 packed pairs), into the [128 x 64] 16-bit dS^T buffer in the
// 128-byte swizzled layout of an MN-major UMMA operand (16-byte piece j of
// row r at j ^ (r & 7)).
__device__ __forceinline__ void store_ds_chunk(uint8_t* ds, int r, int c, const uint32_t (&dpk)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int piece = (4 * c + i) ^ (r & 7);
    *reinterpret_cast<uint4*>(ds + r * 128 + piece * 16) =
        make_uint4(dpk[4 * i], dpk[4 * i + 1], dpk[4 * i + 2], dpk[4 * i + 3]);
  }
}

// Fused backward: dQ^T[d, q] = sum_j K[j, d] dS^T[j, q] for one 64-query
// unit into TMEM (lanes = the 128 head dims, 64 columns = queries): A = K^T
// (the key tile in shared memory read MN-major), B = dS^T (MN-major), 8
// K-steps of 16 keys.  Whole warp, one elected lane.
template <bool BF16>
__device__ __forceinline__ void mma_dqt(uint32_t d_tmem, uint32_t k_smem, uint32_t ds_smem) {
  constexpr uint32_t ID = idesc_f16(BF16, 128, kUnit, true, true);
  const uint64_t a = sdesc(k_smem, kTile * 128, 1024), b = sdesc(ds_smem, kTile * 128, 1024);
#pragma unroll
  for (int kk = 0; kk < kTile / 16; ++kk)
    mma_ss_w(d_tmem, a + ((kk * 16 * 128) >> 4), b + ((kk * 16 * 128) >> 4), ID, kk > 0 ? 1u : 0u);
}

// Fused backward: reads dQ^T of a unit out of TMEM (this thread: head dim r,
// 64 queries), frees the slot, then adds it into the fp32 dQ accumulator
// rows q0 .. q0 + 63 (one warp instruction covers 32 consecutive dims of a
// row).  The scale is applied when the accumulator is converted.
__device__ __forceinline__ bool drain_dqt(uint32_t taddr, uint32_t full_bar, uint32_t parity, uint32_t free_bar,
                                          float* acc_row0, int D, const Abort& ab) {
  if (!mbar_wait(full_bar, parity, ab)) return false;
  tc_fence_after();
  float a[32], c[32];
  tmem_ld32(taddr, a);
  tmem_ld32(taddr + 32, c);
  tmem_ld_wait();
  tc_fence_before();
  mbar_arrive(free_bar);
#ifdef CRA_PROBE_NORED  // measurement probe: no accumulation (wrong dQ)
  if (a[0] == 12345.f && c[0] == 54321.f) acc_row0[0] = 1.f;
#else
#pragma unroll
  for (int j = 0; j < 32; ++j) atomicAdd(acc_row0 + static_cast<int64_t>(j) * D, a[j]);
#pragma unroll
  for (int j = 0; j < 32; ++j) atomicAdd(acc_row0 + static_cast<int64_t>(j + 32) * D, c[j]);
#endif
  return true;
}

// ===========================================================================
// delta: ndelta = -rowsum(O * dO);  nlse2 = -lse * log2(e).  Both are stored
// negated so the softmax passes add them with one packed f32x2 instruction
// per two columns.  Rows >= S of the padded arrays are zero (always masked).
// ===========================================================================
template <int D, bool BF16>
__global__ void __launch_bounds__(256) delta_kernel(const void* __restrict__ op, const void* __restrict__ dop,
                                                    int64_t o_sb, int64_t o_sh, int64_t o_ss, int64_t d_sb,
                                                    int64_t d_sh, int64_t d_ss, const float* __restrict__ lse, int H,
                                                    int S, int Spad, float* __restrict__ lse2,
                                                    float* __restrict__ delta, float* __restrict__ dq_acc) {
  using E = Elt<BF16>;
  using T = typename E::T;
  constexpr int LPR = D / 8, RPW = 32 / LPR;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int row = (blockIdx.x * 8 + warp) * RPW + lane / LPR;
  const int part = lane % LPR;
  float acc = 0.f;
  if (row < S) {
    const uint4 uo = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(op) + b * o_sb + h * o_sh +
                                                     static_cast<int64_t>(row) * o_ss + part * 8);
    const uint4 ud = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(dop) + b * d_sb + h * d_sh +
                                                     static_cast<int64_t>(row) * d_ss + part * 8);
    const uint32_t wo[4] = {uo.x, uo.y, uo.z, uo.w}, wd[4] = {ud.x, ud.y, ud.z, ud.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = E::unpack(wo[e]), c = E::unpack(wd[e]);
      acc = fmaf(a.x, c.x, acc);
      acc = fmaf(a.y, c.y, acc);
    }
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (dq_acc && row < Spad) {  // fused backward: the dQ accumulator starts at zero
    float4* z = reinterpret_cast<float4*>(dq_acc + (static_cast<int64_t>(bh) * Spad + row) * D + part * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (part == 0 && row < Spad) {
    const int64_t i = static_cast<int64_t>(bh) * Spad + row;
    delta[i] = row < S ? -acc : 0.f;
    lse2[i] = row < S ? -lse[static_cast<int64_t>(bh) * S + row] * kLog2e : 0.f;
  }
}

// ===========================================================================
// dQ: query-centric, persistent.  One CTA per SM walks query tiles t =
// blockIdx.x, blockIdx.x + gridDim.x, ... (each a 128-query tile of one
// (b, h), longest tiles first) and, per tile, the forward's key tiles (band,
// then global prefix) in 64-key units, skipping halves no row needs.  Per
// unit: S = Q K_u^T and dP = dO V_u^T into TMEM slot u & 1 (TS-form MMAs:
// the tile's Q and dO are copied into TMEM once per tile, so only K_u / V_u
// are read from shared memory); softmax warpgroup u & 1 writes dS = P * (dP -
// Di) (P from the stored lse, 16-bit) back over S; dQ += dS K_u reads dS from
// TMEM (TS-form MMA) into the dQ accumulator, which an epilogue warpgroup
// reads out while the next tile's first scores are computed.  The K/V unit
// stream, the S/dP -> softmax -> dQ pipeline and the epilogue all run across
// tile boundaries, so no per-tile start-up or drain is exposed.
//
// Warps: 0 K / V producer (TMA), 1 MMA issuer, 2-5 / 6-9 softmax (units of
// parity 0 / 1), 10-13 epilogue, 14 Q / dO producer.  TMEM lane = 32 * (warp
// % 4) + lane = query row.
// ===========================================================================
// Optional cycle counters of the dQ pass (build with -DCRA_PROF; read with
// cra_dq_prof): per role, cycles spent waiting on each barrier and working.
// Counters live in registers and are flushed once per warp at exit.
#ifdef CRA_PROF
__device__ unsigned long long g_dq_prof[32];
__device__ unsigned long long g_kl_prof[32];
#define PROF_ARR g_dq_prof
#define PROF_DECL unsigned long long pacc[32] = {};
#define PROF_T(v) const unsigned long long v = clock64()
#define PROF_ADD(k, t0) (pacc[k] += clock64() - (t0))
#define PROF_CNT(k, n) (pacc[k] += static_cast<unsigned long long>(n))
#define PROF_FLUSH()                                                     \
  if ((threadIdx.x & 31) == 0)                                           \
    _Pragma("unroll") for (int k = 0; k < 32; ++k) if (pacc[k]) atomicAdd(&PROF_ARR[k], pacc[k]);
#else
#define PROF_DECL
#define PROF_T(v)
#define PROF_ADD(k, t0)
#define PROF_CNT(k, n)
#define PROF_FLUSH()
#endif

struct DqUnits {
  int m0, nband, ntiles, ls0, qmax, cmax;
  __device__ __forceinline__ DqUnits(int m0_, int S, int W, int R) : m0(m0_) {
    nband = band_tiles(m0, W);
    ntiles = nband + global_tiles(m0, S, W, R);
    ls0 = local_start(m0, W);
    qmax = min(m0 + kTile - 1, S - 1);
    cmax = gcount(qmax, W, R);
  }
  // half hh of key tile j: first key row / global row, and whether any row of
  // the tile needs it
  __device__ __forceinline__ bool get(int j, int hh, int& row0, bool& g) const {
    if (j < nband) {
      g = false;
      row0 = m0 - j * kTile + kUnit * hh;
      return row0 <= qmax && row0 + kUnit > ls0;
    }
    g = true;
    row0 = (j - nband) * kTile + kUnit * hh;
    return row0 < cmax;
  }
};

// Query tile t of the persistent dQ walk: consecutive t are consecutive tiles
// of one (b, h) (their band keys overlap in L2), latest queries first.
struct DqTile {
  int m0, h, b;  // m0: absolute position of the tile's first query (tiles start at q_lo)
  __device__ __forceinline__ DqTile(int t, int n_qtiles, int H, int q_lo) {
    const int qt = n_qtiles - 1 - t % n_qtiles;
    const int bh = t / n_qtiles;
    m0 = q_lo + qt * kTile;
    h = bh % H;
    b = bh / H;
  }
};

template <int D>
struct DqCfg {
  static constexpr int TB = kTile * D * 2;   // Q / dO tile
  static constexpr int UB = kUnit * D * 2;   // one K or V unit
  static constexpr int NSLOT = (D == 128) ? 10 : 20;  // ring entries K_0, V_0, K_1, V_1, ...
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + TB;
  static constexpr int OFF_RING = OFF_DO + TB;
  static constexpr int OFF_BAR = OFF_RING + NSLOT * UB;
  static constexpr int B_QFULL = 0, B_QEMPTY = 1, B_FULL = 2, B_EMPTY = 2 + NSLOT, B_SFULL = 2 + 2 * NSLOT,
                       B_DSFULL = B_SFULL + 2, B_ACCFULL = B_DSFULL + 2, B_ACCFREE = B_ACCFULL + 1,
                       B_QREAD = B_ACCFREE + 1, B_DRAIN = B_QREAD + 1, N_BAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  // TMEM: slot s -> S at 128 s, dP at 128 s + 64 (fp32, 64 columns each; dS
  // overwrites the first 32 columns of S as 16-bit pairs); the tile's Q and
  // dO as 16-bit pairs (the A operands of S and dP) at 256 and 256 + D / 2;
  // the dQ accumulator after them
  static constexpr int COL_Q = 256, COL_DO = COL_Q + D / 2, COL_DQ = 384;
  static constexpr int THREADS = 480;
  static constexpr int Q_WARP = 14;
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(480, 1) dq_kernel(const __grid_constant__ QueryPassParams p) {
  using C = DqCfg<D>;
  using E = Elt<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = p.W, S = p.S, R = p.R;
  const int Spad = p.n_qtiles * kTile;
  const int q_end = p.q_begin + p.q_len;  // queries [q_begin, q_end) (the whole sequence, or a shard)
  (void)S;
  const int n_tiles = p.n_qtiles * p.H * p.B;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR = [&](int i) { return bar0 + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Abort ab{abort_flag, p.err};
  PROF_DECL

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_QFULL), 1);
    mbar_init(BAR(C::B_QEMPTY), 1);
    for (int i = 0; i < C::NSLOT; ++i) {
      mbar_init(BAR(C::B_FULL + i), 1);
      mbar_init(BAR(C::B_EMPTY + i), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR(C::B_SFULL + s), 1);
      mbar_init(BAR(C::B_DSFULL + s), 128);
    }
    mbar_init(BAR(C::B_ACCFULL), 1);
    mbar_init(BAR(C::B_ACCFREE), 128);
    mbar_init(BAR(C::B_QREAD), 1);
    mbar_init(BAR(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int e = 0;  // ring entries issued
      bool ok = true;
      for (int t = blockIdx.x, it = 0; ok && t < n_tiles; t += gridDim.x, ++it) {
        const DqTile tl(t, p.n_qtiles, p.H, p.q_begin);
        const int hk = tl.h / p.kv_groups;
        const DqUnits un(tl.m0, q_end, W, R);
        for (int j = 0; ok && j < un.ntiles; ++j)
          for (int hh = 0; hh < 2 && ok; ++hh) {
            int row0;
            bool g;
            if (!un.get(j, hh, row0, g)) continue;
            for (int kv = 0; kv < 2; ++kv, ++e) {
              const int sl = e % C::NSLOT;
              PROF_T(t0);
              if (e >= C::NSLOT && !mbar_wait(BAR(C::B_EMPTY + sl), ((e / C::NSLOT) - 1) & 1, ab)) {
                ok = false;
                break;
              }
              PROF_ADD(1, t0);
              // band units below this shard's own K / V rows: the halo (edge copy)
              const bool edge = !g && p.has_edge && row0 < p.kv_begin;
              const CUtensorMap* m = g ? (kv ? &p.tm_gv : &p.tm_gk)
                                       : edge ? (kv ? &p.tm_ve : &p.tm_ke) : (kv ? &p.tm_v : &p.tm_k);
              mbar_expect_tx(BAR(C::B_FULL + sl), C::UB);
              for (int c = 0; c < D / 64; ++c)
                tma_load_4d(sbase + C::OFF_RING + sl * C::UB + c * kUnit * 128, m, BAR(C::B_FULL + sl), c * 64,
                            g ? row0 : edge ? row0 - p.edge_begin : row0 - p.kv_begin, hk, tl.b);
            }
          }
      }
      if (*abort_flag)  // let copies in flight land before the CTA exits
        for (int i = (e > C::NSLOT ? e - C::NSLOT : 0); i < e; ++i)
          mbar_wait_bounded(BAR(C::B_FULL + i % C::NSLOT), (i / C::NSLOT) & 1);
    }
    __syncwarp();
  } else if (warp == C::Q_WARP) {
    // ---------------- Q / dO producer ----------------
    // A thread of its own, so that the K / V stream runs on into the next
    // tile while this one waits for the current tile's last scores (the
    // single Q / dO buffer frees only then).
    if (lane == 0) {
      int nq = 0;
      for (int t = blockIdx.x, it = 0; t < n_tiles; t += gridDim.x, ++it) {
        const DqTile tl(t, p.n_qtiles, p.H, p.q_begin);
        PROF_T(t0);
        if (it > 0 && !mbar_wait(BAR(C::B_QEMPTY), (it - 1) & 1, ab)) break;
        PROF_ADD(0, t0);
        mbar_expect_tx(BAR(C::B_QFULL), 2 * C::TB);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(sbase + C::OFF_Q + c * kTile * 128, &p.tm_q, BAR(C::B_QFULL), c * 64, tl.m0 - p.q_begin, tl.h, tl.b);
          tma_load_4d(sbase + C::OFF_DO + c * kTile * 128, &p.tm_do, BAR(C::B_QFULL), c * 64, tl.m0 - p.q_begin, tl.h, tl.b);
        }
        ++nq;
#ifndef CRA_DQ_NO_PREFETCH
        // the next tile's Q / dO into L2, so that its load, which waits for
        // this tile's last scores, comes from L2
        if (t + static_cast<int>(gridDim.x) < n_tiles) {
          const DqTile tn(t + gridDim.x, p.n_qtiles, p.H, p.q_begin);
          for (int c = 0; c < D / 64; ++c) {
            tma_prefetch_l2_4d(&p.tm_q, c * 64, tn.m0 - p.q_begin, tn.h, tn.b);
            tma_prefetch_l2_4d(&p.tm_do, c * 64, tn.m0 - p.q_begin, tn.h, tn.b);
          }
        }
#endif
      }
      if (*abort_flag && nq > 0) mbar_wait_bounded(BAR(C::B_QFULL), (nq - 1) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    {  // whole warp, converged; one elected lane issues
      constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kUnit, false, false);
      constexpr uint32_t ID_Q = idesc_f16(BF16, kTile, D, false, true);
      // shared-memory descriptors: the start-address field (bits 0-13, in 16-byte
      // units) of a base descriptor plus a constant offset never carries, as
      // shared memory ends below 256 KB
      const uint64_t qd = sdesc(sbase + C::OFF_Q, 16, 1024), dd = sdesc(sbase + C::OFF_DO, 16, 1024);
      bool ok = true;
      // dQ += dS K for unit i of tile iteration iti (its K sits in ring entry 2 i)
      auto issue_dq = [&](int i, int iti, bool first, bool last) -> bool {
        const int sl = i & 1, ek = (2 * i) % C::NSLOT;
        PROF_T(t0);
        if (!warp_wait(BAR(C::B_DSFULL + sl), (i >> 1) & 1, ab)) return false;
        PROF_ADD(4, t0);
        PROF_T(t1);
        if (first && iti >= 1 && !warp_wait(BAR(C::B_ACCFREE), (iti - 1) & 1, ab)) return false;
        PROF_ADD(5, t1);
        tc_fence_after();
        const uint64_t kd = sdesc(sbase + C::OFF_RING + ek * C::UB, kUnit * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < kUnit / 16; ++kk)
          mma_ts_w(tmem + C::COL_DQ, tmem + 128 * sl + kk * 8, kd + ((kk * 16 * 128) >> 4), ID_Q,
                 (!first || kk > 0) ? 1u : 0u);
        mma_commit_w(BAR(C::B_EMPTY + ek));
        if (last) mma_commit_w(BAR(C::B_ACCFULL));
        return true;
      };
      PROF_T(tstart);
      int u = 0;                                     // units issued (all tiles)
      int pit = -1;                                  // tile iteration of unit u - 1
      bool pfirst = false;                           // unit u - 1 was its tile's first
      for (int t = blockIdx.x, it = 0; ok && t < n_tiles; t += gridDim.x, ++it) {
        const DqTile tl(t, p.n_qtiles, p.H, p.q_begin);
        const DqUnits un(tl.m0, q_end, W, R);
        PROF_T(tq);
        // Q / dO into TMEM once the previous tile's last S / dP products
        // (which read the TMEM copies) have completed; the copies execute in
        // order before this tile's MMAs, and their commit frees the
        // shared-memory buffer for the next tile's loads
        if (!warp_wait(BAR(C::B_QFULL), it & 1, ab) ||
            (it > 0 && !warp_wait(BAR(C::B_QREAD), (it - 1) & 1, ab))) {
          ok = false;
          break;
        }
        PROF_ADD(6, tq);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qo = ((kk >> 2) * kTile * 128 + (kk & 3) * 32) >> 4;
          tmem_cp_128x256b_w(tmem + C::COL_Q + kk * 8, qd + qo);
          tmem_cp_128x256b_w(tmem + C::COL_DO + kk * 8, dd + qo);
        }
        mma_commit_w(BAR(C::B_QEMPTY));
        bool first = true;
        for (int j = 0; ok && j < un.ntiles; ++j)
          for (int hh = 0; ok && hh < 2; ++hh) {
            int row0;
            bool g;
            if (!un.get(j, hh, row0, g)) continue;
            const int sl = u & 1, ek = 2 * u, ev = 2 * u + 1;
            // Slot sl was last read by dQ(u - 2), issued before this S / dP:
            // MMAs issued by this warp execute in issue order, so no wait is needed
            // (a wait on a commit would also wait for S / dP(u - 1), issued
            // before dQ(u - 2), and drain the tensor pipe every unit).
            PROF_T(t0);
            if (!warp_wait(BAR(C::B_FULL + ek % C::NSLOT), (ek / C::NSLOT) & 1, ab) ||
                !warp_wait(BAR(C::B_FULL + ev % C::NSLOT), (ev / C::NSLOT) & 1, ab)) {
              ok = false;
              break;
            }
            PROF_ADD(7, t0);
            PROF_T(t1);
            tc_fence_after();
            const uint64_t kd = sdesc(sbase + C::OFF_RING + (ek % C::NSLOT) * C::UB, 16, 1024);
            const uint64_t vd = sdesc(sbase + C::OFF_RING + (ev % C::NSLOT) * C::UB, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              // K-step kk: 64-column chunk kk / 4, 32-byte step kk % 4 in its 128-byte rows
              const uint32_t ko = ((kk >> 2) * kUnit * 128 + (kk & 3) * 32) >> 4;
              mma_ts_w(tmem + 128 * sl, tmem + C::COL_Q + kk * 8, kd + ko, ID_S, kk > 0 ? 1u : 0u);
              mma_ts_w(tmem + 128 * sl + 64, tmem + C::COL_DO + kk * 8, vd + ko, ID_S, kk > 0 ? 1u : 0u);
            }
            mma_commit_w(BAR(C::B_SFULL + sl));
            mma_commit_w(BAR(C::B_EMPTY + ev % C::NSLOT));  // V_u is no longer needed
            PROF_ADD(8, t1);
            // dQ of the previous unit (possibly the previous tile's last)
            if (u > 0 && !issue_dq(u - 1, pit, pfirst, pit != it)) { ok = false; break; }
            pit = it;
            pfirst = first;
            first = false;
            ++u;
          }
        if (ok) mma_commit_w(BAR(C::B_QREAD));  // every S / dP of this tile issued
      }
      if (ok && u > 0) ok = issue_dq(u - 1, pit, pfirst, true);
      PROF_ADD(9, tstart);
      PROF_CNT(30, u);
      PROF_CNT(31, 1);
      if (!ok) {
        mma_commit_w(BAR(C::B_DRAIN));
        mbar_wait_bounded(BAR(C::B_DRAIN), 0);
      }
    }
    __syncwarp();
  } else if (warp < 10) {
    // ---------------- softmax: dS = P * (dP - Di) ----------------
    const int w = (warp - 2) >> 2;           // units with (u & 1) == w, TMEM slot w
    const int r = ((warp & 3) << 5) | lane;  // query row within the tile = TMEM lane
    const uint32_t scol = tmem + (static_cast<uint32_t>(r & ~31) << 16) + 128 * w;
    const float sl2 = p.scale_log2;
    bool ok = true;
    int u = 0;
    for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
      const DqTile tl(t, p.n_qtiles, p.H, p.q_begin);
      const DqUnits un(tl.m0, q_end, W, R);
      const int qi = tl.m0 + r;
      const bool row_ok = qi < q_end;
      const int ls = local_start(qi, W);
      const int cnt = gcount(qi, W, R);
      const int64_t rowi = (static_cast<int64_t>(tl.b) * p.H + tl.h) * Spad + (qi - p.q_begin);
      const float nl = p.lse[rowi];    // -lse * log2(e), padded array
      const float nd = p.delta[rowi];  // -Di
      const float2 sl2x2 = make_float2(sl2, sl2), nlx2 = make_float2(nl, nl), ndx2 = make_float2(nd, nd);
      for (int j = 0; ok && j < un.ntiles; ++j)
        for (int hh = 0; hh < 2; ++hh) {
          int row0;
          bool g;
          if (!un.get(j, hh, row0, g)) continue;
          const int uu = u++;
          if ((uu & 1) != w) continue;
          PROF_T(t0);
          if (!mbar_wait(BAR(C::B_SFULL + w), (uu >> 1) & 1, ab)) {
            ok = false;
            break;
          }
          PROF_ADD(12, t0);
          PROF_T(t1);
          tc_fence_after();
          int lo, hi;
          if (!g) {
            lo = ls - row0;
            hi = qi - row0 + 1;
          } else {
            lo = 0;
            hi = cnt - row0;
          }
          if (!row_ok) { lo = 0; hi = 0; }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float s[32], dp[32];
            tmem_ld32(scol + 32 * c, s);
            tmem_ld32(scol + 64 + 32 * c, dp);
            tmem_ld_wait();
            const uint32_t m = col_mask32(lo - 32 * c, hi - 32 * c);
            uint32_t pk[16];
            // dS = P (dP - Di), P = 2^(s scale log2e - lse log2e); masked columns 0
            auto body = [&](auto masked) {
#pragma unroll
              for (int e2 = 0; e2 < 32; e2 += 2) {
                const float2 x = fma2(make_float2(s[e2], s[e2 + 1]), sl2x2, nlx2);
                float p0 = ex2(x.x), p1 = ex2(x.y);
                if constexpr (decltype(masked)::value) {
                  p0 = (m >> e2) & 1u ? p0 : 0.f;
                  p1 = (m >> (e2 + 1)) & 1u ? p1 : 0.f;
                }
                const float2 ds = mul2(make_float2(p0, p1), add2(make_float2(dp[e2], dp[e2 + 1]), ndx2));
                pk[e2 / 2] = E::pack(ds.x, ds.y);
              }
            };
            if (__all_sync(0xffffffffu, m == 0xffffffffu))
              body(std::false_type{});
            else
              body(std::true_type{});
            tmem_st16(scol + 16 * c, pk);  // dS over S columns [16c, 16c+16), already read
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(BAR(C::B_DSFULL + w));
          PROF_ADD(13, t1);
        }
    }
  } else if (warp < C::Q_WARP) {
    // ---------------- epilogue: dQ accumulator -> global ----------------
    const int r = ((warp & 3) << 5) | lane;
    const uint32_t lane_off = static_cast<uint32_t>(r & ~31) << 16;
    for (int t = blockIdx.x, it = 0; t < n_tiles; t += gridDim.x, ++it) {
      const DqTile tl(t, p.n_qtiles, p.H, p.q_begin);
      PROF_T(t0);
      if (!mbar_wait(BAR(C::B_ACCFULL), it & 1, ab)) break;
      PROF_ADD(16, t0);
      tc_fence_after();
      uint32_t pk[D / 2];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_off + C::COL_DQ + 32 * c, o);
        tmem_ld_wait();
#pragma unroll
        for (int e2 = 0; e2 < 32; e2 += 2) pk[16 * c + e2 / 2] = E::pack(o[e2] * p.scale, o[e2 + 1] * p.scale);
      }
      tc_fence_before();
      mbar_arrive(BAR(C::B_ACCFREE));
      const int qi = tl.m0 + r;
      if (qi < q_end) {
        typename E::T* orow = reinterpret_cast<typename E::T*>(p.out) + tl.b * p.out_sb + tl.h * p.out_sh +
                              static_cast<int64_t>(qi - p.q_begin) * p.out_ss;
#pragma unroll
        for (int q = 0; q < D / 16; ++q) {  // 16 columns = one 32-byte sector per store
          uint32_t w8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) w8[e] = pk[8 * q + e];
          st_global_8w(orow + 16 * q, w8, p.out_v8);
        }
      }
    }
  }
  PROF_FLUSH()
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

#ifdef CRA_PROF
extern "C" __attribute__((visibility("default"))) int cra_dq_prof(unsigned long long* out32, int reset) {
  cudaMemcpyFromSymbol(out32, g_dq_prof, sizeof(g_dq_prof));
  if (reset) {
    unsigned long long z[32] = {};
    cudaMemcpyToSymbol(g_dq_prof, z, sizeof(z));
  }
  return 0;
}
extern "C" __attribute__((visibility("default"))) int cra_kl_prof(unsigned long long* out32, int reset) {
  cudaMemcpyFromSymbol(out32, g_kl_prof, sizeof(g_kl_prof));
  if (reset) {
    unsigned long long z[32] = {};
    cudaMemcpyToSymbol(g_kl_prof, z, sizeof(z));
  }
  return 0;
}
#endif

// ===========================================================================
// Key-centric pass over the global rows G (strided + relay keys).  Thread r
// owns global row r of the CTA's 128-row tile.  The queries that see the
// tile (a contiguous range starting at first_query_seeing) are split into
// n_split ranges, one per CTA, walked in 64-query units; per unit:
//   S^T = K Q_u^T, dP^T = V dO_u^T  (one of two TMEM slots),
//   P^T, dS^T (16-bit) written back into the same TMEM slot,
//   dV += P^T dO_u,  dK += dS^T Q_u  (TMEM accumulators; A operands read
//   from TMEM, so only dO_u / Q_u come from shared memory).
// The two softmax warpgroups take alternate units.  A slot is rewritten by
// S^T / dP^T of unit u + 2 only after the dV / dK products of unit u that
// read it were issued; MMAs issued by one warp execute in issue order, so no
// completion wait is needed (one would drain the tensor pipe every unit).
// ===========================================================================
template <int D, bool FUSED>
struct KeyCfg {
  static constexpr int TB = kTile * D * 2;         // K or V tile
  static constexpr int UB = kUnit * D * 2;         // Q or dO unit
  static constexpr int NSQ = FUSED ? 3 : (D == 128) ? 4 : 8;  // Q/dO unit stages
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TB;
  static constexpr int OFF_Q = OFF_V + TB;         // stage s: Q at OFF_Q + 2 s UB, dO after it
  static constexpr int OFF_LSE = OFF_Q + NSQ * 2 * UB;  // stage s: lse2[64], delta[64]
  // fused: dS^T of the units of parity s, [128 keys x 64 queries] 16-bit
  static constexpr int OFF_DS = (OFF_LSE + NSQ * 2 * kUnit * 4 + 1023) / 1024 * 1024;
  static constexpr int DSB = kTile * kUnit * 2;
  static constexpr int OFF_BAR = FUSED ? OFF_DS + 2 * DSB : OFF_LSE + NSQ * 2 * kUnit * 4;
  static constexpr int B_KVFULL = 0, B_QFULL = 1, B_QEMPTY = 1 + NSQ, B_SFULL = 1 + 2 * NSQ, B_PFULL = B_SFULL + 2,
                       B_DONE = B_PFULL + 2, B_DRAIN = B_DONE + 1, B_DQFULL = B_DRAIN + 1, B_DQFREE = B_DQFULL + 2,
                       N_BAR = B_DQFREE + 2;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  // TMEM: slot s -> S^T at 128 s, dP^T at 128 s + 64 (fp32, 64 columns each);
  // the softmax overwrites them with P^T (128 s, 32 columns of 16-bit pairs)
  // and dS^T (128 s + 64), which the dV / dK products read from TMEM.
  // dV at 256, dK at 256 + D.
  static constexpr int COL_DV = 256, COL_DK = 256 + D;
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <int D, bool BF16, bool FUSED>
__global__ void __launch_bounds__(320, 1) keyglobal_kernel(const __grid_constant__ KeyPassParams p) {
  using C = KeyCfg<D, FUSED>;
  using E = Elt<BF16>;
  using T = typename E::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTAs in launch order take the global-row tiles first to last, all heads
  // and splits of a tile together: earlier tiles are seen by more queries,
  // so the longest CTAs start first and the last wave holds the shortest.
  // (The heads' queries then do not stay in L2 between tiles: about twice
  // the DRAM reads of a head-by-head order, which was measured slower.)
  const int lin = static_cast<int>(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
  const int per_tile = static_cast<int>(gridDim.y * gridDim.z) * p.n_split;
  const int gt = lin / per_tile;
  const int rem = lin % per_tile;
  const int split = rem % p.n_split;
  const int hk = (rem / p.n_split) % static_cast<int>(gridDim.y), b = (rem / p.n_split) / static_cast<int>(gridDim.y);
  const int W = p.W, S = p.S, R = p.R;
  const int q_lo = p.q_lo, q_hi = p.q_hi;
  const int n_units = (q_hi - q_lo + kUnit - 1) / kUnit;  // 64-query units from q_lo
  const int Spad = p.q_pad;
  const int groups = p.kv_groups;

  // global-row tile gt and this split's 64-query units [t_lo, t_hi) (per group head)
  const int k0 = gt * kTile;
  const int tmin = min(max(first_query_seeing(k0, S, W, R) - q_lo, 0) / kUnit, n_units);
  const int tot = n_units - tmin;
  const int t_lo = tmin + static_cast<int>((static_cast<int64_t>(tot) * split) / p.n_split);
  const int t_hi = tmin + static_cast<int>((static_cast<int64_t>(tot) * (split + 1)) / p.n_split);
  const int nT = t_hi - t_lo;
  const int nU = nT * groups;

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR = [&](int i) { return bar0 + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Abort ab{abort_flag, p.err};

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_KVFULL), 1);
    for (int i = 0; i < C::NSQ; ++i) {
      mbar_init(BAR(C::B_QFULL + i), 1);
      mbar_init(BAR(C::B_QEMPTY + i), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR(C::B_SFULL + s), 1);
      mbar_init(BAR(C::B_PFULL + s), 128);
    }
    mbar_init(BAR(C::B_DONE), 1);
    for (int q = 0; q < 2; ++q) {
      mbar_init(BAR(C::B_DQFULL + q), 1);
      mbar_init(BAR(C::B_DQFREE + q), 128);
    }
    mbar_init(BAR(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto unit = [&](int u, int& h, int& q0) {  // q0: absolute position of the unit's first query
    h = hk * groups + u / nT;
    q0 = q_lo + (t_lo + u % nT) * kUnit;
  };

  if (warp == 0) {
    if (lane == 0 && nU > 0) {
      mbar_expect_tx(BAR(C::B_KVFULL), 2 * C::TB);
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(sbase + C::OFF_K + c * kTile * 128, &p.tm_k, BAR(C::B_KVFULL), c * 64, k0, hk, b);
        tma_load_4d(sbase + C::OFF_V + c * kTile * 128, &p.tm_v, BAR(C::B_KVFULL), c * 64, k0, hk, b);
      }
      int issued = 0;
      for (int u = 0; u < nU; ++u) {
        const int st = u % C::NSQ;
        if (u >= C::NSQ && !mbar_wait(BAR(C::B_QEMPTY + st), ((u / C::NSQ) - 1) & 1, ab)) break;
        int h, q0;
        unit(u, h, q0);
        const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::UB;
        mbar_expect_tx(BAR(C::B_QFULL + st), 2 * C::UB + 2 * kUnit * 4);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(qd + c * kUnit * 128, &p.tm_q, BAR(C::B_QFULL + st), c * 64, q0 - q_lo, h, b);
          tma_load_4d(qd + C::UB + c * kUnit * 128, &p.tm_do, BAR(C::B_QFULL + st), c * 64, q0 - q_lo, h, b);
        }
        const int64_t li = (static_cast<int64_t>(b) * p.H + h) * Spad + (q0 - q_lo);
        const uint32_t ld = sbase + C::OFF_LSE + st * 2 * kUnit * 4;
        bulk_load(ld, p.lse + li, kUnit * 4, BAR(C::B_QFULL + st));
        bulk_load(ld + kUnit * 4, p.delta + li, kUnit * 4, BAR(C::B_QFULL + st));
        ++issued;
      }
      if (*abort_flag) {
        for (int u = (issued > C::NSQ ? issued - C::NSQ : 0); u < issued; ++u)
          mbar_wait_bounded(BAR(C::B_QFULL + u % C::NSQ), (u / C::NSQ) & 1);
        mbar_wait_bounded(BAR(C::B_KVFULL), 0);  // the K / V tile
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (nU > 0) {  // whole warp, converged; one elected lane issues
      constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kUnit, false, false);
      constexpr uint32_t ID_G = idesc_f16(BF16, kTile, D, false, true);
      const uint32_t ks = sbase + C::OFF_K, vs = sbase + C::OFF_V;
      bool ok = warp_wait(BAR(C::B_KVFULL), 0, ab);
      auto issue_dqt = [&](uint32_t d_tmem, uint32_t k_smem, uint32_t ds_smem) { mma_dqt<BF16>(d_tmem, k_smem, ds_smem); };
      auto issue_kv = [&](int i) -> bool {
        const int st = i % C::NSQ, sl = i & 1;
        if (!warp_wait(BAR(C::B_PFULL + sl), (i >> 1) & 1, ab)) return false;
        tc_fence_after();
        const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::UB;
#pragma unroll
        for (int kk = 0; kk < kUnit / 16; ++kk) {
          const uint32_t boff = kk * 16 * 128;
          mma_ts_w(tmem + C::COL_DV, tmem + 128 * sl + kk * 8, sdesc(qd + C::UB + boff, kUnit * 128, 1024), ID_G,
                 (i > 0 || kk > 0) ? 1u : 0u);
          mma_ts_w(tmem + C::COL_DK, tmem + 128 * sl + 64 + kk * 8, sdesc(qd + boff, kUnit * 128, 1024), ID_G,
                 (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit_w(BAR(C::B_QEMPTY + st));
        if constexpr (FUSED) {  // dQ^T of the unit into its (read) score slot
          issue_dqt(tmem + 128 * sl, ks, sbase + C::OFF_DS + sl * C::DSB);
          mma_commit_w(BAR(C::B_DQFULL + sl));
        }
        return true;
      };
      for (int u = 0; ok && u < nU; ++u) {
        const int st = u % C::NSQ, sl = u & 1;
        // slot sl was last read by the dV / dK products of unit u - 2, issued
        // before this S^T / dP^T (in-order execution); fused, it then held
        // dQ^T of unit u - 2 until the softmax warps read it out
        if (!warp_wait(BAR(C::B_QFULL + st), (u / C::NSQ) & 1, ab) ||
            (FUSED && u >= 2 && !warp_wait(BAR(C::B_DQFREE + sl), ((u >> 1) - 1) & 1, ab))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::UB;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t ko = (kk >> 2) * kTile * 128 + (kk & 3) * 32;
          const uint32_t qo = (kk >> 2) * kUnit * 128 + (kk & 3) * 32;
          mma_ss_w(tmem + 128 * sl, sdesc(ks + ko, 16, 1024), sdesc(qd + qo, 16, 1024), ID_S, kk > 0 ? 1u : 0u);
          mma_ss_w(tmem + 128 * sl + 64, sdesc(vs + ko, 16, 1024), sdesc(qd + C::UB + qo, 16, 1024), ID_S,
                 kk > 0 ? 1u : 0u);
        }
        mma_commit_w(BAR(C::B_SFULL + sl));
        if (u > 0 && !issue_kv(u - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_kv(nU - 1);
      if (ok) mma_commit_w(BAR(C::B_DONE));
      if (!ok) {
        mma_commit_w(BAR(C::B_DRAIN));
        mbar_wait_bounded(BAR(C::B_DRAIN), 0);
      }
    }
    __syncwarp();
  } else {
    const int w = (warp - 2) >> 2;           // softmax warpgroup: units with (u & 1) == w
    const int r = ((warp & 3) << 5) | lane;  // key row = TMEM lane
    const int kj = k0 + r;                   // global row
    const uint32_t lane_off = static_cast<uint32_t>(r & ~31) << 16;
    const float sl2 = p.scale_log2;
    // queries that see this global row: [qa, S)
    const int qa = kj < p.NG ? first_query_seeing(kj, S, W, R) : S, qb = q_hi;
    const uint32_t scol = tmem + lane_off + 128 * w;
    bool ok = true;
    for (int u = w; u < nU; u += 2) {
      const int st = u % C::NSQ;
      int h, q0;
      unit(u, h, q0);
      // SFULL first: it implies this unit's Q/dO stage load has completed, and
      // the stage cannot be refilled before this unit's dV/dK products, so
      // the QFULL parity test below refers to exactly this load (this
      // warpgroup skips every other unit, so waiting on QFULL alone could
      // match an older phase of the stage).  Waiting on QFULL makes the TMA
      // writes of lse / delta visible to this thread.
      if (!mbar_wait(BAR(C::B_SFULL + w), (u >> 1) & 1, ab) ||
          !mbar_wait(BAR(C::B_QFULL + st), (u / C::NSQ) & 1, ab)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int lo = qa - q0, hi = qb - q0;
      const float* sm_lse = reinterpret_cast<const float*>(smem + C::OFF_LSE + st * 2 * kUnit * 4);
      const float* sm_di = sm_lse + kUnit;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float s[32], dp[32];
        tmem_ld32(scol + 32 * c, s);
        tmem_ld32(scol + 64 + 32 * c, dp);
        tmem_ld_wait();
        uint32_t ppk[16], dpk[16];
        key_softmax_chunk<E>(s, dp, sm_lse + 32 * c, sm_di + 32 * c, sl2, col_mask32(lo - 32 * c, hi - 32 * c), ppk,
                             dpk);
        // chunk c of P^T / dS^T overwrites score columns [16c, 16c+16) of
        // S^T / dP^T, already consumed (columns [0, 32c+32) have been read)
        tmem_st16(scol + 16 * c, ppk);
        tmem_st16(scol + 64 + 16 * c, dpk);
        if constexpr (FUSED) store_ds_chunk(smem + C::OFF_DS + w * C::DSB, r, c, dpk);
      }
      tmem_st_wait();
      if constexpr (FUSED) fence_proxy_async();  // dS^T stores -> the dQ^T MMA
      tc_fence_before();
      mbar_arrive(BAR(C::B_PFULL + w));
      if constexpr (FUSED) {
        float* acc = p.dq_acc + ((static_cast<int64_t>(b) * p.H + h) * Spad + (q0 - q_lo)) * D + r;
        if (!drain_dqt(scol, BAR(C::B_DQFULL + w), (u >> 1) & 1, BAR(C::B_DQFREE + w), acc, D, ab)) {
          ok = false;
          break;
        }
      }
    }
    // ------------------------------------------------------------ epilogue
    // warpgroup 0 writes dG_k partials, warpgroup 1 dG_v partials
    const bool have = nU > 0;
    if (ok && (!have || mbar_wait(BAR(C::B_DONE), 0, ab))) {
      tc_fence_after();
      const uint32_t acc = tmem + lane_off + (w == 0 ? C::COL_DK : C::COL_DV);
      const float mul = w == 0 ? p.scale : 1.f;
      const bool row_ok = kj < p.NG;
      float* dst = (w == 0 ? p.part_k : p.part_v) +
                   ((static_cast<int64_t>(split) * p.B + b) * gridDim.y + hk) * static_cast<int64_t>(p.NG) * D +
                   static_cast<int64_t>(kj) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        if (have) {
          tmem_ld32(acc + 32 * c, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0.f;
        }
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(dst + 32 * c + e) =
                make_float4(v[e] * mul, v[e + 1] * mul, v[e + 2] * mul, v[e + 3] * mul);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ===========================================================================
// Local key pass, persistent.  One CTA per SM walks the local key tiles t =
// blockIdx.x, blockIdx.x + gridDim.x, ... (kt fastest, latest keys first).
// Per tile the work is the key-centric pass above, over K / V rows of the
// local band instead of global rows; across tiles
//   * K / V are double-buffered (tile i in buffer i & 1), so the next tile's
//     K / V arrive while the current tile runs;
//   * the Q / dO unit stream, the MMA issue and the two softmax warpgroups
//     run on without a break (one global unit counter);
//   * a dedicated epilogue warpgroup drains dK / dV (plus the dG fold-in) of
//     tile i while tile i + 1 starts; only tile i + 1's first dV / dK product
//     waits for it (ACCFREE).
// Warps: 0 producer, 1 MMA issuer, 2-5 / 6-9 softmax, 10-13 epilogue.
// ===========================================================================
template <int D, bool FUSED>
struct KeyLocalCfg {
  static constexpr int TB = kTile * D * 2;         // K or V tile
  static constexpr int UB = kUnit * D * 2;         // Q or dO unit
  static constexpr int NSQ = FUSED ? 2 : (D == 128) ? 3 : 8;  // Q/dO unit stages
  static constexpr int OFF_KV = 0;                 // buffer b: K at 2 b TB, V at (2 b + 1) TB
  static constexpr int OFF_Q = 4 * TB;             // stage s: Q at OFF_Q + 2 s UB, dO after it
  static constexpr int OFF_LSE = OFF_Q + NSQ * 2 * UB;  // stage s: lse2[64], delta[64]
  static constexpr int OFF_DS = (OFF_LSE + NSQ * 2 * kUnit * 4 + 1023) / 1024 * 1024;  // fused: dS^T, 2 buffers
  static constexpr int DSB = kTile * kUnit * 2;
  static constexpr int OFF_BAR = FUSED ? OFF_DS + 2 * DSB : OFF_LSE + NSQ * 2 * kUnit * 4;
  static constexpr int B_KVFULL = 0, B_KVEMPTY = 2, B_QFULL = 4, B_QEMPTY = 4 + NSQ, B_SFULL = 4 + 2 * NSQ,
                       B_PFULL = B_SFULL + 2, B_ACCFULL = B_PFULL + 2, B_ACCFREE = B_ACCFULL + 1,
                       B_DRAIN = B_ACCFREE + 1, B_DQFULL = B_DRAIN + 1, B_DQFREE = B_DQFULL + 2, N_BAR = B_DQFREE + 2;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr int COL_DV = 256, COL_DK = 256 + D;  // slots at 0 and 128 as in KeyCfg
  static constexpr int THREADS = 448;
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Local key tile t of the persistent walk and the 64-query units it meets.
struct KeyLocalTile {
  int k0, hk, b, t_lo, nT, nU, q_lo;
  // Key tiles start at k_lo (128 keys each); queries [q_lo, q_hi) in 64-query
  // units from q_lo.  Every key of [k_lo, q_hi) has a query in range.
  __device__ __forceinline__ KeyLocalTile(int t, int n_ktiles, int Hkv, int k_lo, int q_lo_, int q_hi, int W,
                                          int groups)
      : q_lo(q_lo_) {
    const int kt = t % n_ktiles;
    hk = (t / n_ktiles) % Hkv;
    b = t / (n_ktiles * Hkv);
    k0 = k_lo + (n_ktiles - 1 - kt) * kTile;
    const int qfirst = max(k0, q_lo), qlast = min(k0 + kTile - 1 + W - 1, q_hi - 1);
    t_lo = (qfirst - q_lo) / kUnit;
    nT = (qlast - q_lo) / kUnit + 1 - t_lo;
    nU = nT * groups;
  }
  // unit ul: head h, absolute position q0 of its first query
  __device__ __forceinline__ void unit(int ul, int groups, int& h, int& q0) const {
    h = hk * groups + ul / nT;
    q0 = q_lo + (t_lo + ul % nT) * kUnit;
  }
};

#ifdef CRA_PROF
#undef PROF_ARR
#define PROF_ARR g_kl_prof
#endif

template <int D, bool BF16, bool FUSED>
__global__ void __launch_bounds__(448, 1) keylocal_kernel(const __grid_constant__ KeyPassParams p) {
  using C = KeyLocalCfg<D, FUSED>;
  using E = Elt<BF16>;
  using T = typename E::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = p.W, S = p.S, R = p.R;
  const int Spad = p.q_pad;
  (void)S;
  const int groups = p.kv_groups;
  const int Hkv = p.H / groups;
  const int n_tiles = p.n_ktiles * Hkv * p.B;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR = [&](int i) { return bar0 + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Abort ab{abort_flag, p.err};
  PROF_DECL

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR(C::B_KVFULL + s), 1);
      mbar_init(BAR(C::B_KVEMPTY + s), 1);
      mbar_init(BAR(C::B_SFULL + s), 1);
      mbar_init(BAR(C::B_PFULL + s), 128);
    }
    for (int i = 0; i < C::NSQ; ++i) {
      mbar_init(BAR(C::B_QFULL + i), 1);
      mbar_init(BAR(C::B_QEMPTY + i), 1);
    }
    mbar_init(BAR(C::B_ACCFULL), 1);
    mbar_init(BAR(C::B_ACCFREE), 128);
    for (int q = 0; q < 2; ++q) {
      mbar_init(BAR(C::B_DQFULL + q), 1);
      mbar_init(BAR(C::B_DQFREE + q), 128);
    }
    mbar_init(BAR(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int e = 0, nkv = 0;  // Q/dO units issued, K/V tiles issued
      bool ok = true;
      for (int t = blockIdx.x, i = 0; ok && t < n_tiles; t += gridDim.x, ++i) {
        const KeyLocalTile tl(t, p.n_ktiles, Hkv, p.k_lo, p.q_lo, p.q_hi, W, groups);
        const int kb = i & 1;
        PROF_T(tk);
        if (i >= 2 && !mbar_wait(BAR(C::B_KVEMPTY + kb), ((i >> 1) - 1) & 1, ab)) break;
        PROF_ADD(0, tk);
        mbar_expect_tx(BAR(C::B_KVFULL + kb), 2 * C::TB);
        const uint32_t kd = sbase + C::OFF_KV + 2 * kb * C::TB;
        // tiles that start below this shard's own K / V rows come from the edge copy
        const bool edge = p.has_edge && tl.k0 < p.kv_main;
        const int krow = edge ? tl.k0 - p.edge_begin : tl.k0 - p.kv_main;
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(kd + c * kTile * 128, edge ? &p.tm_ke : &p.tm_k, BAR(C::B_KVFULL + kb), c * 64, krow, tl.hk,
                      tl.b);
          tma_load_4d(kd + C::TB + c * kTile * 128, edge ? &p.tm_ve : &p.tm_v, BAR(C::B_KVFULL + kb), c * 64, krow,
                      tl.hk, tl.b);
        }
        ++nkv;
        for (int ul = 0; ul < tl.nU; ++ul, ++e) {
          const int st = e % C::NSQ;
          PROF_T(tq);
          if (e >= C::NSQ && !mbar_wait(BAR(C::B_QEMPTY + st), ((e / C::NSQ) - 1) & 1, ab)) { ok = false; break; }
          PROF_ADD(1, tq);
          int h, q0;
          tl.unit(ul, groups, h, q0);
          const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::UB;
          mbar_expect_tx(BAR(C::B_QFULL + st), 2 * C::UB + 2 * kUnit * 4);
          for (int c = 0; c < D / 64; ++c) {
            tma_load_4d(qd + c * kUnit * 128, &p.tm_q, BAR(C::B_QFULL + st), c * 64, q0 - p.q_lo, h, tl.b);
            tma_load_4d(qd + C::UB + c * kUnit * 128, &p.tm_do, BAR(C::B_QFULL + st), c * 64, q0 - p.q_lo, h, tl.b);
          }
          const int64_t li = (static_cast<int64_t>(tl.b) * p.H + h) * Spad + (q0 - p.q_lo);
          const uint32_t ld = sbase + C::OFF_LSE + st * 2 * kUnit * 4;
          bulk_load(ld, p.lse + li, kUnit * 4, BAR(C::B_QFULL + st));
          bulk_load(ld + kUnit * 4, p.delta + li, kUnit * 4, BAR(C::B_QFULL + st));
        }
      }
      if (*abort_flag) {  // let copies in flight land before the CTA exits
        for (int u = (e > C::NSQ ? e - C::NSQ : 0); u < e; ++u)
          mbar_wait_bounded(BAR(C::B_QFULL + u % C::NSQ), (u / C::NSQ) & 1);
        for (int i = (nkv > 2 ? nkv - 2 : 0); i < nkv; ++i) mbar_wait_bounded(BAR(C::B_KVFULL + (i & 1)), (i >> 1) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp, one elected lane) ----------------
    constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kUnit, false, false);
    constexpr uint32_t ID_G = idesc_f16(BF16, kTile, D, false, true);
    bool ok = true;
    // dV += P^T dO, dK += dS^T Q for unit i (of tile iteration iti)
    auto issue_kv = [&](int i, int iti, bool first, bool last) -> bool {
      const int st = i % C::NSQ, sl = i & 1;
      PROF_T(tp);
      if (!warp_wait(BAR(C::B_PFULL + sl), (i >> 1) & 1, ab)) return false;
      PROF_ADD(4, tp);
      PROF_T(ta);
      if (first && iti >= 1 && !warp_wait(BAR(C::B_ACCFREE), (iti - 1) & 1, ab)) return false;
      PROF_ADD(5, ta);
      tc_fence_after();
      const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::UB;
      const uint64_t dod = sdesc(qd + C::UB, kUnit * 128, 1024), qdd = sdesc(qd, kUnit * 128, 1024);
#pragma unroll
      for (int kk = 0; kk < kUnit / 16; ++kk) {
        const uint32_t boff = (kk * 16 * 128) >> 4;
        mma_ts_w(tmem + C::COL_DV, tmem + 128 * sl + kk * 8, dod + boff, ID_G, (!first || kk > 0) ? 1u : 0u);
        mma_ts_w(tmem + C::COL_DK, tmem + 128 * sl + 64 + kk * 8, qdd + boff, ID_G, (!first || kk > 0) ? 1u : 0u);
      }
      mma_commit_w(BAR(C::B_QEMPTY + st));
      if (last) mma_commit_w(BAR(C::B_ACCFULL));
      if constexpr (FUSED) {  // dQ^T of the unit into its (read) score slot; reads the tile's K
        mma_dqt<BF16>(tmem + 128 * sl, sbase + C::OFF_KV + 2 * (iti & 1) * C::TB, sbase + C::OFF_DS + sl * C::DSB);
        mma_commit_w(BAR(C::B_DQFULL + sl));
        if (last) mma_commit_w(BAR(C::B_KVEMPTY + (iti & 1)));  // K / V of the tile: last reader issued
      }
      return true;
    };
    PROF_T(tstart);
    int u = 0, pit = -1;
    bool pfirst = false;
    for (int t = blockIdx.x, i = 0; ok && t < n_tiles; t += gridDim.x, ++i) {
      const KeyLocalTile tl(t, p.n_ktiles, Hkv, p.k_lo, p.q_lo, p.q_hi, W, groups);
      const int kb = i & 1;
      PROF_T(tk);
      if (!warp_wait(BAR(C::B_KVFULL + kb), (i >> 1) & 1, ab)) { ok = false; break; }
      PROF_ADD(6, tk);
      const uint64_t kd = sdesc(sbase + C::OFF_KV + 2 * kb * C::TB, 16, 1024);
      const uint64_t vd = sdesc(sbase + C::OFF_KV + (2 * kb + 1) * C::TB, 16, 1024);
      for (int ul = 0; ul < tl.nU; ++ul, ++u) {
        const int st = u % C::NSQ, sl = u & 1;
        // slot sl was last read by the dV / dK products of unit u - 2, issued
        // before this S^T / dP^T (in-order execution)
        PROF_T(tq);
        if (!warp_wait(BAR(C::B_QFULL + st), (u / C::NSQ) & 1, ab)) { ok = false; break; }
        if (FUSED && u >= 2 && !warp_wait(BAR(C::B_DQFREE + sl), ((u >> 1) - 1) & 1, ab)) { ok = false; break; }
        PROF_ADD(7, tq);
        tc_fence_after();
        const uint32_t qa = sbase + C::OFF_Q + st * 2 * C::UB;
        const uint64_t qd = sdesc(qa, 16, 1024), dd = sdesc(qa + C::UB, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t ko = ((kk >> 2) * kTile * 128 + (kk & 3) * 32) >> 4;
          const uint32_t qo = ((kk >> 2) * kUnit * 128 + (kk & 3) * 32) >> 4;
          mma_ss_w(tmem + 128 * sl, kd + ko, qd + qo, ID_S, kk > 0 ? 1u : 0u);
          mma_ss_w(tmem + 128 * sl + 64, vd + ko, dd + qo, ID_S, kk > 0 ? 1u : 0u);
        }
        mma_commit_w(BAR(C::B_SFULL + sl));
        if (!FUSED && ul == tl.nU - 1) mma_commit_w(BAR(C::B_KVEMPTY + kb));  // K / V of this tile: last reader issued
        if (u > 0 && !issue_kv(u - 1, pit, pfirst, pit != i)) { ok = false; break; }
        pit = i;
        pfirst = ul == 0;
      }
    }
    if (ok && u > 0) ok = issue_kv(u - 1, pit, pfirst, true);
    PROF_ADD(9, tstart);
    PROF_CNT(30, u);
    PROF_CNT(31, 1);
    if (!ok) {
      mma_commit_w(BAR(C::B_DRAIN));
      mbar_wait_bounded(BAR(C::B_DRAIN), 0);
    }
    __syncwarp();
  } else if (warp < 10) {
    // ---------------- softmax: P^T, dS^T ----------------
    const int w = (warp - 2) >> 2;           // units with (u & 1) == w
    const int r = ((warp & 3) << 5) | lane;  // key row = TMEM lane
    const uint32_t scol = tmem + (static_cast<uint32_t>(r & ~31) << 16) + 128 * w;
    const float sl2 = p.scale_log2;
    bool ok = true;
    int u = 0;
    for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
      const KeyLocalTile tl(t, p.n_ktiles, Hkv, p.k_lo, p.q_lo, p.q_hi, W, groups);
      const int kj = tl.k0 + r;
      // queries that see this key row: [qa, qb)
      const int qa = kj, qb = kj < p.q_hi ? min(kj + W, p.q_hi) : kj;
      for (int ul = 0; ul < tl.nU; ++ul) {
        const int uu = u++;
        if ((uu & 1) != w) continue;
        const int st = uu % C::NSQ;
        int h, q0;
        tl.unit(ul, groups, h, q0);
        // SFULL first: it implies this unit's Q/dO stage load has completed,
        // and the stage cannot be refilled before this unit's dV/dK products,
        // so the QFULL parity test refers to exactly this load.  Waiting on
        // QFULL makes the TMA writes of lse / delta visible to this thread.
        PROF_T(ts);
        if (!mbar_wait(BAR(C::B_SFULL + w), (uu >> 1) & 1, ab) ||
            !mbar_wait(BAR(C::B_QFULL + st), (uu / C::NSQ) & 1, ab)) {
          ok = false;
          break;
        }
        PROF_ADD(12, ts);
        PROF_T(tb);
        tc_fence_after();
        const int lo = qa - q0, hi = qb - q0;
        const float* sm_lse = reinterpret_cast<const float*>(smem + C::OFF_LSE + st * 2 * kUnit * 4);
        const float* sm_di = sm_lse + kUnit;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float s[32], dp[32];
          tmem_ld32(scol + 32 * c, s);
          tmem_ld32(scol + 64 + 32 * c, dp);
          tmem_ld_wait();
          uint32_t ppk[16], dpk[16];
          key_softmax_chunk<E>(s, dp, sm_lse + 32 * c, sm_di + 32 * c, sl2, col_mask32(lo - 32 * c, hi - 32 * c),
                               ppk, dpk);
          // chunk c of P^T / dS^T overwrites score columns [16c, 16c+16) of
          // S^T / dP^T, already consumed (columns [0, 32c+32) have been read)
          tmem_st16(scol + 16 * c, ppk);
          tmem_st16(scol + 64 + 16 * c, dpk);
          if constexpr (FUSED) store_ds_chunk(smem + C::OFF_DS + w * C::DSB, r, c, dpk);
        }
        tmem_st_wait();
        if constexpr (FUSED) fence_proxy_async();  // dS^T stores -> the dQ^T MMA
        tc_fence_before();
        mbar_arrive(BAR(C::B_PFULL + w));
        if constexpr (FUSED) {
          float* acc = p.dq_acc + ((static_cast<int64_t>(tl.b) * p.H + h) * Spad + (q0 - p.q_lo)) * D + r;
          if (!drain_dqt(scol, BAR(C::B_DQFULL + w), (uu >> 1) & 1, BAR(C::B_DQFREE + w), acc, D, ab)) {
            ok = false;
            break;
          }
        }
        PROF_ADD(13, tb);
      }
    }
  } else {
    // ---------------- epilogue: dK, dV -> global, then the dG fold-in ----------------
    // The accumulators are read, scaled, rounded and stored first, and
    // released as soon as the last TMEM load has landed: the next tile's
    // first dV / dK product waits for that release, so nothing slow may sit
    // between ACCFULL and ACCFREE.  The global-row gradients that belong to
    // this key position (its strided row and relay rows whose source it is)
    // are added afterwards by a read-add-write of the stored row in the
    // output dtype -- the reference's relay scatter does the same
    // (core.py:2811-2815) -- by the thread that stored it, so program order
    // makes its own stores visible to the re-read.
    const int r = ((warp & 3) << 5) | lane;
    const uint32_t lane_off = static_cast<uint32_t>(r & ~31) << 16;
    for (int t = blockIdx.x, i = 0; t < n_tiles; t += gridDim.x, ++i) {
      const KeyLocalTile tl(t, p.n_ktiles, Hkv, p.k_lo, p.q_lo, p.q_hi, W, groups);
      const int kj = tl.k0 + r;
      const bool row_ok = kj < p.q_hi;
      const bool halo = kj < p.kv_main;  // key of the previous shard: output to dkh / dvh, no fold-in
      // global rows of this key position (looked up before the wait)
      const int blk = kj / W;
      const int64_t gbase = (static_cast<int64_t>(tl.b) * Hkv + tl.hk) * static_cast<int64_t>(p.NG);
      int grow[5];
      float gsc[5];
      int ng = 0;
      if (row_ok && !halo) {
        if (kj == blk * W) {
          grow[ng] = blk * R;
          gsc[ng] = 1.f;
          ++ng;
        }
        if (R > 1) {
          float rs = 1.f;
          if (p.relay_scale) rs = E::to_f(E::from_f(expf(p.relay_scale[tl.hk])));
          const int32_t* src = p.gsrc + ((static_cast<int64_t>(tl.b) * Hkv + tl.hk) * p.NB + blk) * p.top_k;
          for (int q = 0; q < p.top_k; ++q)
            if (src[q] == kj) {
              grow[ng] = blk * R + 1 + q;
              gsc[ng] = rs;
              ++ng;
            }
        }
      }
      T* const dkrow =
          halo ? reinterpret_cast<T*>(p.dkh) + tl.b * p.dkh_sb + tl.hk * p.dkh_sh + static_cast<int64_t>(kj - p.k_lo) * p.dkh_ss
               : reinterpret_cast<T*>(p.dk) + tl.b * p.dk_sb + tl.hk * p.dk_sh +
                     static_cast<int64_t>(kj - p.kv_main) * p.dk_ss;
      T* const dvrow =
          halo ? reinterpret_cast<T*>(p.dvh) + tl.b * p.dvh_sb + tl.hk * p.dvh_sh + static_cast<int64_t>(kj - p.k_lo) * p.dvh_ss
               : reinterpret_cast<T*>(p.dv) + tl.b * p.dv_sb + tl.hk * p.dv_sh +
                     static_cast<int64_t>(kj - p.kv_main) * p.dv_ss;
      PROF_T(te);
      if (!mbar_wait(BAR(C::B_ACCFULL), i & 1, ab)) break;
      PROF_ADD(16, te);
      PROF_T(tb);
      tc_fence_after();
#pragma unroll 1
      for (int g4 = 0; g4 < 2 * (D / 64); ++g4) {  // 64-column groups: dK then dV
        const int which = g4 / (D / 64), c2 = g4 % (D / 64);
        const uint32_t acc = tmem + lane_off + (which == 0 ? C::COL_DK : C::COL_DV) + 64 * c2;
        const float mul = which == 0 ? p.scale : 1.f;
        float v[2][32];
        tmem_ld32(acc, v[0]);
        tmem_ld32(acc + 32, v[1]);
        tmem_ld_wait();
        if (g4 == 2 * (D / 64) - 1) {  // every TMEM read of this tile's dK / dV done
          tc_fence_before();
          mbar_arrive(BAR(C::B_ACCFREE));
        }
        if (row_ok) {
          T* drow = (which == 0 ? dkrow : dvrow) + 64 * c2;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
            for (int q = 0; q < 2; ++q) {  // 16 columns = one 32-byte sector per store
              uint32_t w8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) w8[e] = E::pack(v[h2][16 * q + 2 * e] * mul, v[h2][16 * q + 2 * e + 1] * mul);
              st_global_8w(drow + 32 * h2 + 16 * q, w8, p.dkv_v8);
            }
        }
      }
      // fold-in: d{K,V}[kj] += sum_g gsc_g * dG_{k,v}[g], summed in fp32 onto
      // the stored value.  The few rows that have global rows (about one per
      // 128-key tile) are done by the whole warp, one row at a time, lane l
      // covering D / 32 consecutive columns, so each row costs one round trip
      // to memory instead of D / 8 dependent ones.  __syncwarp orders the
      // owner's stores before the other lanes' reads.
      unsigned fm = __ballot_sync(0xffffffffu, ng > 0);
      if (fm) __syncwarp();
      while (fm) {
        const int src = __ffs(fm) - 1;
        fm &= fm - 1;
        constexpr int CPL = D / 32;  // columns per lane: 4 (D = 128) or 2 (D = 64)
        const int n_s = __shfl_sync(0xffffffffu, ng, src);
        const int kj_s = __shfl_sync(0xffffffffu, kj, src);
        int g_s[5];
        float sc_s[5];
#pragma unroll
        for (int gi = 0; gi < 5; ++gi) {
          g_s[gi] = __shfl_sync(0xffffffffu, gi < ng ? grow[gi] : 0, src);
          sc_s[gi] = __shfl_sync(0xffffffffu, gi < ng ? gsc[gi] : 0.f, src);
        }
        const int c0 = lane * CPL;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const float* dg = which == 0 ? p.dgk : p.dgv;
          T* drow = which == 0 ? reinterpret_cast<T*>(p.dk) + tl.b * p.dk_sb + tl.hk * p.dk_sh +
                                     static_cast<int64_t>(kj_s - p.kv_main) * p.dk_ss
                               : reinterpret_cast<T*>(p.dv) + tl.b * p.dv_sb + tl.hk * p.dv_sh +
                                     static_cast<int64_t>(kj_s - p.kv_main) * p.dv_ss;
          float a[CPL];
          if constexpr (CPL == 4) {
            const uint2 cur = *reinterpret_cast<const uint2*>(drow + c0);
            const float2 f0 = E::unpack(cur.x), f1 = E::unpack(cur.y);
            a[0] = f0.x; a[1] = f0.y; a[2] = f1.x; a[3] = f1.y;
          } else {
            const float2 f0 = E::unpack(*reinterpret_cast<const uint32_t*>(drow + c0));
            a[0] = f0.x; a[1] = f0.y;
          }
#pragma unroll
          for (int gi = 0; gi < 5; ++gi)
            if (gi < n_s) {
              const float* gr = dg + (gbase + g_s[gi]) * D + c0;
              if constexpr (CPL == 4) {
                const float4 x = *reinterpret_cast<const float4*>(gr);
                a[0] += sc_s[gi] * x.x; a[1] += sc_s[gi] * x.y; a[2] += sc_s[gi] * x.z; a[3] += sc_s[gi] * x.w;
              } else {
                const float2 x = *reinterpret_cast<const float2*>(gr);
                a[0] += sc_s[gi] * x.x; a[1] += sc_s[gi] * x.y;
              }
            }
          if constexpr (CPL == 4)
            *reinterpret_cast<uint2*>(drow + c0) = make_uint2(E::pack(a[0], a[1]), E::pack(a[2], a[3]));
          else
            *reinterpret_cast<uint32_t*>(drow + c0) = E::pack(a[0], a[1]);
        }
      }
      PROF_ADD(17, tb);
    }
  }
  PROF_FLUSH()
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ===========================================================================
// dG = sum over splits of the partials (fixed order).
// ===========================================================================
__global__ void __launch_bounds__(256) reduce_kernel(const float4* __restrict__ pk, const float4* __restrict__ pv,
                                                     int64_t n4, int n_split, float4* __restrict__ gk,
                                                     float4* __restrict__ gv) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = pk[i], c = pv[i];
    for (int s = 1; s < n_split; ++s) {
      const float4 x = pk[s * n4 + i], y = pv[s * n4 + i];
      a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
      c.x += y.x; c.y += y.y; c.z += y.z; c.w += y.w;
    }
    gk[i] = a;
    gv[i] = c;
  }
}

// d(relay_log_scale)[hk] = sum_b sum_{relay rows g} sum_d dG_k*G_k + dG_v*G_v.
// One CTA per kv head; fixed summation order.
template <bool BF16>
__global__ void __launch_bounds__(256) dalpha_kernel(const float* __restrict__ dgk, const float* __restrict__ dgv,
                                                     const void* __restrict__ gkp, const void* __restrict__ gvp,
                                                     int B, int Hkv, int NG, int R, int D, float* __restrict__ out) {
  using T = typename Elt<BF16>::T;
  const int hk = blockIdx.x;
  const T* gk = reinterpret_cast<const T*>(gkp);
  const T* gv = reinterpret_cast<const T*>(gvp);
  float acc = 0.f;
  for (int b = 0; b < B; ++b) {
    const int64_t base = (static_cast<int64_t>(b) * Hkv + hk) * NG * D;
    for (int64_t i = threadIdx.x; i < static_cast<int64_t>(NG) * D; i += blockDim.x) {
      const int g = static_cast<int>(i / D);
      if (g % R == 0) continue;
      acc += dgk[base + i] * Elt<BF16>::to_f(gk[base + i]) + dgv[base + i] * Elt<BF16>::to_f(gv[base + i]);
    }
  }
  __shared__ float red[256];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[hk] = red[0];
}

// ===========================================================================
// host side
// ===========================================================================
// SMs of the current device (cached per device).
static int sm_count() {
  static int cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

template <typename K>
static cudaError_t set_smem(K kern, int bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Fused backward: dQ = scale * dQ accumulator, rounded to the output dtype.
// One thread per 8 elements of a row.
template <int D, bool BF16>
__global__ void __launch_bounds__(256) dq_convert_kernel(const float* __restrict__ acc, void* __restrict__ dq,
                                                         int64_t sb, int64_t sh, int64_t ss, int64_t n_rows, int H,
                                                         int S, int Spad, float scale) {
  using E = Elt<BF16>;
  constexpr int PR = D / 8;  // threads per row
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t row = i / PR;  // over B * H * S rows
  if (row >= n_rows) return;
  const int part = static_cast<int>(i % PR);
  const int64_t bh = row / S;
  const int srow = static_cast<int>(row % S);
  const float4* a = reinterpret_cast<const float4*>(acc + (bh * Spad + srow) * D + part * 8);
  const float4 x = a[0], y = a[1];
  const int b = static_cast<int>(bh / H), h = static_cast<int>(bh % H);
  typename E::T* out = reinterpret_cast<typename E::T*>(dq) + b * sb + h * sh + static_cast<int64_t>(srow) * ss +
                       part * 8;
  *reinterpret_cast<uint4*>(out) = make_uint4(E::pack(x.x * scale, x.y * scale), E::pack(x.z * scale, x.w * scale),
                                              E::pack(y.x * scale, y.y * scale), E::pack(y.z * scale, y.w * scale));
}

// Launch order of the backward kernels (dalpha_kernel only with a relay scale).
static const char* const kBwdKernelNames[] = {"delta_kernel", "keyglobal_kernel", "reduce_kernel", "dalpha_kernel",
                                              "keylocal_kernel", "dq_kernel", "dq_convert_kernel"};

// The key passes (and, unfused, the dQ pass; fused, the dQ conversion).
template <int D, bool BF16, bool FUSED, typename Mark, typename Done>
static cudaError_t launch_key_passes(BwdLaunch& L, cudaStream_t st, Mark& mark, Done& done) {
  const QueryPassParams& qp = L.qp;
  const int B = qp.B, H = qp.H, S = qp.S;
  const int Spad = qp.n_qtiles * kTile;
  cudaError_t e;
  const KeyPassParams& gp = L.global;
  const int Hkv = gp.H / gp.kv_groups;
  const int n_gtiles = (gp.NG + kTile - 1) / kTile;
  if (L.phase != 2) {
    using C = KeyCfg<D, FUSED>;
    auto kern = keyglobal_kernel<D, BF16, FUSED>;
    if ((e = set_smem(kern, C::SMEM)) != cudaSuccess) return e;
    if ((e = mark(1)) != cudaSuccess) return e;
    kern<<<dim3(n_gtiles * gp.n_split, Hkv, B), 320, C::SMEM, st>>>(gp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (L.phase != 2) {
    const int64_t n4 = static_cast<int64_t>(B) * Hkv * gp.NG * D / 4;
    const int64_t nb = (n4 + 255) / 256;
    if ((e = mark(2)) != cudaSuccess) return e;
    reduce_kernel<<<static_cast<int>(nb < 4096 ? nb : 4096), 256, 0, st>>>(
        reinterpret_cast<const float4*>(gp.part_k), reinterpret_cast<const float4*>(gp.part_v), n4, gp.n_split,
        reinterpret_cast<float4*>(L.dgk), reinterpret_cast<float4*>(L.dgv));
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (L.phase == 1) return done();  // shard: dG goes through a cross-GPU sum first
  if (L.d_alpha && gp.R > 1) {
    if ((e = mark(3)) != cudaSuccess) return e;
    dalpha_kernel<BF16><<<Hkv, 256, 0, st>>>(L.dgk, L.dgv, L.gk_rows, L.gv_rows, B, Hkv, gp.NG, gp.R, D, L.d_alpha);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const KeyPassParams& lp = L.local;
  {
    using C = KeyLocalCfg<D, FUSED>;
    auto kern = keylocal_kernel<D, BF16, FUSED>;
    if ((e = set_smem(kern, C::SMEM)) != cudaSuccess) return e;
    const int n_tiles = lp.n_ktiles * Hkv * B;
    if ((e = mark(4)) != cudaSuccess) return e;
    kern<<<dim3(n_tiles < sm_count() ? n_tiles : sm_count()), C::THREADS, C::SMEM, st>>>(lp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if constexpr (FUSED) {
    const int64_t n = static_cast<int64_t>(B) * H * S * (D / 8);
    if ((e = mark(6)) != cudaSuccess) return e;
    dq_convert_kernel<D, BF16><<<dim3(static_cast<unsigned>((n + 255) / 256)), 256, 0, st>>>(
        gp.dq_acc, qp.out, qp.out_sb, qp.out_sh, qp.out_ss, static_cast<int64_t>(B) * H * S, H, S, Spad, qp.scale);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  } else {
    auto kern = dq_kernel<D, BF16>;
    if ((e = set_smem(kern, DqCfg<D>::SMEM)) != cudaSuccess) return e;
    const int n_tiles = qp.n_qtiles * H * B;
    if ((e = mark(5)) != cudaSuccess) return e;
    kern<<<dim3(n_tiles < sm_count() ? n_tiles : sm_count()), DqCfg<D>::THREADS, DqCfg<D>::SMEM, st>>>(qp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return done();
}

template <int D, bool BF16>
static cudaError_t launch_bwd_t(const BwdLaunch& L_, cudaStream_t st) {
  BwdLaunch& L = const_cast<BwdLaunch&>(L_);
  const QueryPassParams& qp = L.qp;
  const int B = qp.B, H = qp.H;
  const int Spad = qp.n_qtiles * kTile;
  cudaError_t e;
  int nk = 0;
  L.n_kernels = 0;
  // records the event before kernel `id` (index into kBwdKernelNames)
  auto mark = [&](int id) -> cudaError_t {
    if (!L.events) return cudaSuccess;
    L.kernel_ids[nk] = id;
    return cudaEventRecord(L.events[nk++], st);
  };
  auto done = [&]() -> cudaError_t {
    L.n_kernels = nk;
    return L.events ? cudaEventRecord(L.events[nk], st) : cudaSuccess;
  };
  if (L.phase != 2) {
    constexpr int RPB = 8 * (32 / (D / 8));  // rows per 256-thread block
    dim3 grid((Spad + RPB - 1) / RPB, B * H);
    if ((e = mark(0)) != cudaSuccess) return e;
    delta_kernel<D, BF16><<<grid, 256, 0, st>>>(L.o, L.d_o, L.o_st[0], L.o_st[1], L.o_st[2], L.do_st[0], L.do_st[1],
                                                L.do_st[2], L.lse_in, H, qp.q_len, Spad, L.lse2, L.delta,
                                                L.fused ? L.global.dq_acc : nullptr);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if constexpr (D == 128) {
    if (L.fused) return launch_key_passes<D, BF16, true>(L, st, mark, done);
  }
  return launch_key_passes<D, BF16, false>(L, st, mark, done);
}

const char* bwd_kernel_name(int id) {
  return id >= 0 && id < static_cast<int>(sizeof(kBwdKernelNames) / sizeof(kBwdKernelNames[0])) ? kBwdKernelNames[id]
                                                                                                : "unknown";
}

cudaError_t launch_bwd(const BwdLaunch& L, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_bwd_t<128, true>(L, stream) : launch_bwd_t<128, false>(L, stream);
  return bf16 ? launch_bwd_t<64, true>(L, stream) : launch_bwd_t<64, false>(L, stream);
}

}  // namespace cra
