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
//   delta_kernel     Di and lse*log2(e), padded to whole 128-query tiles.
//   keypass<GLOBAL>  one CTA per (128 global rows, query split): dG_k / dG_v
//                    over every query that sees the rows; fp32 partials per
//                    split (no atomics).
//   reduce_kernel    sums the splits in a fixed order -> dG (fp32).
//   dalpha_kernel    d(relay_log_scale) = sum over relay rows of dG * G
//                    (only when a relay scale is used).
//   keypass<LOCAL>   one CTA per 128-key tile: dK / dV over the local band,
//                    then folds in dG of the tile's strided key and of every
//                    relay row whose source lies in the tile, and stores.
//   dq_kernel        one CTA per 128-query tile: dQ over band + global prefix.
// The result is deterministic: every sum has a fixed order.
//
// Both attention kernels use the warp roles of the forward (fwd.cu): warp 0
// TMA producer, warp 1 single-thread tcgen05 issuer + TMEM owner, warps 4-7
// one row per thread (TMEM lane = row).
#include "geom.cuh"
#include "params.h"
#include "sm100.cuh"

namespace cra {

constexpr float kLog2e = 1.4426950408889634f;

// ===========================================================================
// delta: Di = rowsum(O * dO);  lse2 = lse * log2(e).  Rows >= S of the padded
// arrays are zero (never read unmasked).
// ===========================================================================
template <int D, bool BF16>
__global__ void __launch_bounds__(256) delta_kernel(const void* __restrict__ op, const void* __restrict__ dop,
                                                    int64_t o_sb, int64_t o_sh, int64_t o_ss, int64_t d_sb,
                                                    int64_t d_sh, int64_t d_ss, const float* __restrict__ lse, int H,
                                                    int S, int Spad, float* __restrict__ lse2,
                                                    float* __restrict__ delta) {
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
  if (part == 0 && row < Spad) {
    const int64_t i = static_cast<int64_t>(bh) * Spad + row;
    delta[i] = row < S ? acc : 0.f;
    lse2[i] = row < S ? lse[static_cast<int64_t>(bh) * S + row] * kLog2e : 0.f;
  }
}

// ===========================================================================
// dQ: query-centric, same key-tile sequence as the forward.
// ===========================================================================
template <int D>
struct DqCfg {
  static constexpr int NST = (D == 128) ? 2 : 4;
  static constexpr int TB = kTile * D * 2;  // one [128 x D] tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + TB;
  static constexpr int OFF_K = OFF_DO + TB;
  static constexpr int OFF_V = OFF_K + NST * TB;
  static constexpr int OFF_DS = OFF_V + NST * TB;
  static constexpr int OFF_BAR = OFF_DS + kTile * kTile * 2;
  static constexpr int B_QFULL = 0, B_KFULL = 1, B_VFULL = 1 + NST, B_EMPTY = 1 + 2 * NST;
  static constexpr int B_SFULL = 1 + 3 * NST, B_SFREE = B_SFULL + 1, B_DSFULL = B_SFREE + 1,
                       B_DQDONE = B_DSFULL + 1, B_DRAIN = B_DQDONE + 1, N_BAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr int COL_S = 0, COL_DP = 128, COL_DQ = 256;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(256, 1) dq_kernel(const __grid_constant__ QueryPassParams p) {
  using C = DqCfg<D>;
  using E = Elt<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.n_qtiles - 1 - static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z, hk = h / p.kv_groups;
  const int m0 = qt * kTile;
  const int W = p.W, S = p.S, R = p.R;
  const int Spad = p.n_qtiles * kTile;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR = [&](int i) { return bar0 + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Abort ab{abort_flag, p.err};
  const int nband = band_tiles(m0, W);
  const int ntiles = nband + global_tiles(m0, S, W, R);

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_QFULL), 1);
    for (int i = 0; i < C::NST; ++i) {
      mbar_init(BAR(C::B_KFULL + i), 1);
      mbar_init(BAR(C::B_VFULL + i), 1);
      mbar_init(BAR(C::B_EMPTY + i), 1);
    }
    mbar_init(BAR(C::B_SFULL), 1);
    mbar_init(BAR(C::B_SFREE), 128);
    mbar_init(BAR(C::B_DSFULL), 128);
    mbar_init(BAR(C::B_DQDONE), 1);
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
    if (lane == 0) {
      mbar_expect_tx(BAR(C::B_QFULL), 2 * C::TB);
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(sbase + C::OFF_Q + c * kTile * 128, &p.tm_q, BAR(C::B_QFULL), c * 64, m0, h, b);
        tma_load_4d(sbase + C::OFF_DO + c * kTile * 128, &p.tm_do, BAR(C::B_QFULL), c * 64, m0, h, b);
      }
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % C::NST;
        if (j >= C::NST && !mbar_wait(BAR(C::B_EMPTY + st), ((j / C::NST) - 1) & 1, ab)) break;
        const bool g = j >= nband;
        const int row0 = g ? (j - nband) * kTile : m0 - j * kTile;
        mbar_expect_tx(BAR(C::B_KFULL + st), C::TB);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sbase + C::OFF_K + st * C::TB + c * kTile * 128, g ? &p.tm_gk : &p.tm_k, BAR(C::B_KFULL + st),
                      c * 64, row0, hk, b);
        mbar_expect_tx(BAR(C::B_VFULL + st), C::TB);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sbase + C::OFF_V + st * C::TB + c * kTile * 128, g ? &p.tm_gv : &p.tm_v, BAR(C::B_VFULL + st),
                      c * 64, row0, hk, b);
        ++issued;
      }
      if (*abort_flag)
        for (int j = (issued > C::NST ? issued - C::NST : 0); j < issued; ++j)
          mbar_wait_bounded(BAR(C::B_VFULL + j % C::NST), (j / C::NST) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kTile, false, false);
      constexpr uint32_t ID_Q = idesc_f16(BF16, kTile, D, false, true);
      const uint32_t qs = sbase + C::OFF_Q, dos = sbase + C::OFF_DO, dss = sbase + C::OFF_DS;
      bool ok = mbar_wait(BAR(C::B_QFULL), 0, ab);
      auto issue_dq = [&](int i) -> bool {
        const int st = i % C::NST;
        if (!mbar_wait(BAR(C::B_DSFULL), i & 1, ab)) return false;
        tc_fence_after();
        const uint32_t ks = sbase + C::OFF_K + st * C::TB;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint64_t a = sdesc(dss + (kk >> 2) * kTile * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(ks + kk * 16 * 128, kTile * 128, 1024);
          mma_ss(tmem + C::COL_DQ, a, bd, ID_Q, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(BAR(C::B_DQDONE));
        mma_commit(BAR(C::B_EMPTY + st));
        return true;
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % C::NST;
        if (!mbar_wait(BAR(C::B_KFULL + st), (j / C::NST) & 1, ab)) { ok = false; break; }
        if (!mbar_wait(BAR(C::B_VFULL + st), (j / C::NST) & 1, ab)) { ok = false; break; }
        if (j > 0 && !mbar_wait(BAR(C::B_SFREE), (j - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ks = sbase + C::OFF_K + st * C::TB, vs = sbase + C::OFF_V + st * C::TB;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kTile * 128 + (kk & 3) * 32;
          mma_ss(tmem + C::COL_S, sdesc(qs + off, 16, 1024), sdesc(ks + off, 16, 1024), ID_S, kk > 0 ? 1u : 0u);
          mma_ss(tmem + C::COL_DP, sdesc(dos + off, 16, 1024), sdesc(vs + off, 16, 1024), ID_S, kk > 0 ? 1u : 0u);
        }
        mma_commit(BAR(C::B_SFULL));
        if (j > 0 && !issue_dq(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_dq(ntiles - 1);
      if (!ok) {
        mma_commit(BAR(C::B_DRAIN));
        mbar_wait_bounded(BAR(C::B_DRAIN), 0);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    const int r = threadIdx.x - 128;
    const int qi = m0 + r;
    const bool row_ok = qi < S;
    const int ls = local_start(qi, W);
    const int cnt = gcount(qi, W, R);
    const uint32_t lane_off = static_cast<uint32_t>(r & ~31) << 16;
    const float sl = p.scale_log2;
    const int64_t rowi = (static_cast<int64_t>(b) * p.H + h) * Spad + qi;
    const float lse2 = p.lse[rowi];  // lse * log2(e), padded array
    const float di = p.delta[rowi];
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!mbar_wait(BAR(C::B_SFULL), j & 1, ab)) { ok = false; break; }
      tc_fence_after();
      int lo, hi;
      if (j < nband) {
        const int kb = m0 - j * kTile;
        lo = ls - kb;
        hi = qi - kb + 1;
      } else {
        lo = 0;
        hi = cnt - (j - nband) * kTile;
      }
      if (!row_ok) { lo = 0; hi = 0; }
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float s[32], dp[32];
        tmem_ld32(tmem + lane_off + C::COL_S + 32 * c, s);
        tmem_ld32(tmem + lane_off + C::COL_DP + 32 * c, dp);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int col = 32 * c + e;
          const float p0 = (col >= lo && col < hi) ? ex2(fmaf(s[e], sl, -lse2)) : 0.f;
          const float p1 = (col + 1 >= lo && col + 1 < hi) ? ex2(fmaf(s[e + 1], sl, -lse2)) : 0.f;
          pk[16 * c + e / 2] = E::pack(p0 * (dp[e] - di), p1 * (dp[e + 1] - di));
        }
      }
      tc_fence_before();
      mbar_arrive(BAR(C::B_SFREE));
      if (j > 0 && !mbar_wait(BAR(C::B_DQDONE), (j - 1) & 1, ab)) { ok = false; break; }
      uint8_t* dsrow = smem + C::OFF_DS;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        *reinterpret_cast<uint4*>(dsrow + sw128_off(r, u, kTile)) =
            make_uint4(pk[4 * u + 0], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR(C::B_DSFULL));
    }
    if (ok && mbar_wait(BAR(C::B_DQDONE), (ntiles - 1) & 1, ab)) {
      tc_fence_after();
      typename E::T* orow = reinterpret_cast<typename E::T*>(p.out) + b * p.out_sb + h * p.out_sh +
                            static_cast<int64_t>(qi) * p.out_ss;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_off + C::COL_DQ + 32 * c, o);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 v4;
            v4.x = E::pack(o[8 * u + 0] * p.scale, o[8 * u + 1] * p.scale);
            v4.y = E::pack(o[8 * u + 2] * p.scale, o[8 * u + 3] * p.scale);
            v4.z = E::pack(o[8 * u + 4] * p.scale, o[8 * u + 5] * p.scale);
            v4.w = E::pack(o[8 * u + 6] * p.scale, o[8 * u + 7] * p.scale);
            *reinterpret_cast<uint4*>(orow + 32 * c + 8 * u) = v4;
          }
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
// Key-centric pass.  Thread r owns key row r of the CTA's 128-row key tile
// (K/V rows in LOCAL mode, global rows G in GLOBAL mode).  Per query tile:
//   S^T = K Q^T, dP^T = V dO^T  (TMEM),  P^T, dS^T -> shared memory,
//   dV += P^T dO,  dK += dS^T Q  (TMEM accumulators).
// ===========================================================================
template <int D>
struct KeyCfg {
  static constexpr int NSQ = (D == 128) ? 1 : 2;  // Q/dO stages
  static constexpr int TB = kTile * D * 2;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TB;
  static constexpr int OFF_Q = OFF_V + TB;  // stage s: Q at OFF_Q + s*2*TB, dO after it
  static constexpr int OFF_PT = OFF_Q + NSQ * 2 * TB;
  static constexpr int OFF_DST = OFF_PT + kTile * kTile * 2;
  static constexpr int OFF_LSE = OFF_DST + kTile * kTile * 2;  // stage s: lse2[128], delta[128]
  static constexpr int OFF_BAR = OFF_LSE + NSQ * 2 * kTile * 4;
  static constexpr int B_KVFULL = 0, B_QFULL = 1, B_QEMPTY = 1 + NSQ, B_SFULL = 1 + 2 * NSQ, B_SFREE = B_SFULL + 1,
                       B_PFULL = B_SFREE + 1, B_MMADONE = B_PFULL + 1, B_DRAIN = B_MMADONE + 1,
                       N_BAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr int COL_ST = 0, COL_DPT = 128, COL_DV = 256, COL_DK = 256 + D;
};

template <int D, bool BF16, bool GLOBAL>
__global__ void __launch_bounds__(256, 1) keypass_kernel(const __grid_constant__ KeyPassParams p) {
  using C = KeyCfg<D>;
  using E = Elt<BF16>;
  using T = typename E::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int W = p.W, S = p.S, R = p.R;
  const int n_qtiles = (S + kTile - 1) / kTile;
  const int Spad = n_qtiles * kTile;
  const int groups = p.kv_groups;

  // key tile and the query tiles [t_lo, t_hi) it meets (per group head)
  int k0, split = 0, t_lo, t_hi;
  if (GLOBAL) {
    const int gt = static_cast<int>(blockIdx.x) / p.n_split;
    split = static_cast<int>(blockIdx.x) % p.n_split;
    k0 = gt * kTile;
    const int qmin = first_query_seeing(k0, S, W, R);
    const int tmin = qmin / kTile;
    const int tot = n_qtiles - tmin;
    t_lo = tmin + static_cast<int>((static_cast<int64_t>(tot) * split) / p.n_split);
    t_hi = tmin + static_cast<int>((static_cast<int64_t>(tot) * (split + 1)) / p.n_split);
  } else {
    k0 = (p.n_ktiles - 1 - static_cast<int>(blockIdx.x)) * kTile;
    const int qlast = min(k0 + kTile - 1 + W - 1, S - 1);
    t_lo = k0 / kTile;
    t_hi = qlast / kTile + 1;
  }
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
    mbar_init(BAR(C::B_SFULL), 1);
    mbar_init(BAR(C::B_SFREE), 128);
    mbar_init(BAR(C::B_PFULL), 128);
    mbar_init(BAR(C::B_MMADONE), 1);
    mbar_init(BAR(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto unit = [&](int u, int& h, int& q0) {
    h = hk * groups + u / nT;
    q0 = (t_lo + u % nT) * kTile;
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
        const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::TB;
        mbar_expect_tx(BAR(C::B_QFULL + st), 2 * C::TB + 2 * kTile * 4);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(qd + c * kTile * 128, &p.tm_q, BAR(C::B_QFULL + st), c * 64, q0, h, b);
          tma_load_4d(qd + C::TB + c * kTile * 128, &p.tm_do, BAR(C::B_QFULL + st), c * 64, q0, h, b);
        }
        const int64_t li = (static_cast<int64_t>(b) * p.H + h) * Spad + q0;
        const uint32_t ld = sbase + C::OFF_LSE + st * 2 * kTile * 4;
        bulk_load(ld, p.lse + li, kTile * 4, BAR(C::B_QFULL + st));
        bulk_load(ld + kTile * 4, p.delta + li, kTile * 4, BAR(C::B_QFULL + st));
        ++issued;
      }
      if (*abort_flag)
        for (int u = (issued > C::NSQ ? issued - C::NSQ : 0); u < issued; ++u)
          mbar_wait_bounded(BAR(C::B_QFULL + u % C::NSQ), (u / C::NSQ) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && nU > 0) {
      constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kTile, false, false);
      constexpr uint32_t ID_G = idesc_f16(BF16, kTile, D, false, true);
      const uint32_t ks = sbase + C::OFF_K, vs = sbase + C::OFF_V;
      const uint32_t pts = sbase + C::OFF_PT, dsts = sbase + C::OFF_DST;
      bool ok = mbar_wait(BAR(C::B_KVFULL), 0, ab);
      auto issue_kv = [&](int i) -> bool {
        const int st = i % C::NSQ;
        if (!mbar_wait(BAR(C::B_PFULL), i & 1, ab)) return false;
        tc_fence_after();
        const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::TB;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * kTile * 128 + (kk & 3) * 32;
          const uint32_t boff = kk * 16 * 128;
          mma_ss(tmem + C::COL_DV, sdesc(pts + aoff, 16, 1024), sdesc(qd + C::TB + boff, kTile * 128, 1024), ID_G,
                 (i > 0 || kk > 0) ? 1u : 0u);
          mma_ss(tmem + C::COL_DK, sdesc(dsts + aoff, 16, 1024), sdesc(qd + boff, kTile * 128, 1024), ID_G,
                 (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(BAR(C::B_MMADONE));
        mma_commit(BAR(C::B_QEMPTY + st));
        return true;
      };
      for (int u = 0; ok && u < nU; ++u) {
        const int st = u % C::NSQ;
        // With one Q/dO stage the stage is refilled only after the previous
        // unit's dV/dK MMAs release it, so those must be issued first.
        if (C::NSQ == 1 && u > 0 && !issue_kv(u - 1)) { ok = false; break; }
        if (!mbar_wait(BAR(C::B_QFULL + st), (u / C::NSQ) & 1, ab)) { ok = false; break; }
        if (u > 0 && !mbar_wait(BAR(C::B_SFREE), (u - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qd = sbase + C::OFF_Q + st * 2 * C::TB;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kTile * 128 + (kk & 3) * 32;
          mma_ss(tmem + C::COL_ST, sdesc(ks + off, 16, 1024), sdesc(qd + off, 16, 1024), ID_S, kk > 0 ? 1u : 0u);
          mma_ss(tmem + C::COL_DPT, sdesc(vs + off, 16, 1024), sdesc(qd + C::TB + off, 16, 1024), ID_S,
                 kk > 0 ? 1u : 0u);
        }
        mma_commit(BAR(C::B_SFULL));
        if (C::NSQ > 1 && u > 0 && !issue_kv(u - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_kv(nU - 1);
      if (!ok) {
        mma_commit(BAR(C::B_DRAIN));
        mbar_wait_bounded(BAR(C::B_DRAIN), 0);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    const int r = threadIdx.x - 128;
    const int kj = k0 + r;  // key position (LOCAL) or global row (GLOBAL)
    const uint32_t lane_off = static_cast<uint32_t>(r & ~31) << 16;
    const float sl = p.scale_log2;
    // queries that see this key row: [qa, qb)
    int qa, qb;
    if (GLOBAL) {
      qa = kj < p.NG ? first_query_seeing(kj, S, W, R) : S;
      qb = S;
    } else {
      qa = kj;
      qb = kj < S ? min(kj + W, S) : kj;
    }
    bool ok = true;
    for (int u = 0; u < nU; ++u) {
      const int st = u % C::NSQ;
      int h, q0;
      unit(u, h, q0);
      if (!mbar_wait(BAR(C::B_QFULL + st), (u / C::NSQ) & 1, ab)) { ok = false; break; }
      if (!mbar_wait(BAR(C::B_SFULL), u & 1, ab)) { ok = false; break; }
      tc_fence_after();
      const int lo = qa - q0, hi = qb - q0;
      const float* sm_lse = reinterpret_cast<const float*>(smem + C::OFF_LSE + st * 2 * kTile * 4);
      const float* sm_di = sm_lse + kTile;
      uint32_t ppk[64], dpk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float s[32], dp[32];
        tmem_ld32(tmem + lane_off + C::COL_ST + 32 * c, s);
        tmem_ld32(tmem + lane_off + C::COL_DPT + 32 * c, dp);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int col = 32 * c + e;
          const float p0 = (col >= lo && col < hi) ? ex2(fmaf(s[e], sl, -sm_lse[col])) : 0.f;
          const float p1 = (col + 1 >= lo && col + 1 < hi) ? ex2(fmaf(s[e + 1], sl, -sm_lse[col + 1])) : 0.f;
          ppk[16 * c + e / 2] = E::pack(p0, p1);
          dpk[16 * c + e / 2] = E::pack(p0 * (dp[e] - sm_di[col]), p1 * (dp[e + 1] - sm_di[col + 1]));
        }
      }
      tc_fence_before();
      mbar_arrive(BAR(C::B_SFREE));
      if (u > 0 && !mbar_wait(BAR(C::B_MMADONE), (u - 1) & 1, ab)) { ok = false; break; }
#pragma unroll
      for (int w = 0; w < 16; ++w) {
        const uint32_t off = sw128_off(r, w, kTile);
        *reinterpret_cast<uint4*>(smem + C::OFF_PT + off) =
            make_uint4(ppk[4 * w], ppk[4 * w + 1], ppk[4 * w + 2], ppk[4 * w + 3]);
        *reinterpret_cast<uint4*>(smem + C::OFF_DST + off) =
            make_uint4(dpk[4 * w], dpk[4 * w + 1], dpk[4 * w + 2], dpk[4 * w + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR(C::B_PFULL));
    }
    // ------------------------------------------------------------ epilogue
    const bool have = nU > 0;
    if (ok && (!have || mbar_wait(BAR(C::B_MMADONE), (nU - 1) & 1, ab))) {
      tc_fence_after();
      if (GLOBAL) {
        const bool row_ok = kj < p.NG;
        const int64_t base =
            ((static_cast<int64_t>(split) * p.B + b) * (gridDim.y) + hk) * static_cast<int64_t>(p.NG) * D +
            static_cast<int64_t>(kj) * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float vk[32], vv[32];
          if (have) {
            tmem_ld32(tmem + lane_off + C::COL_DK + 32 * c, vk);
            tmem_ld32(tmem + lane_off + C::COL_DV + 32 * c, vv);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) vk[e] = vv[e] = 0.f;
          }
          if (row_ok) {
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              *reinterpret_cast<float4*>(p.part_k + base + 32 * c + e) =
                  make_float4(vk[e] * p.scale, vk[e + 1] * p.scale, vk[e + 2] * p.scale, vk[e + 3] * p.scale);
              *reinterpret_cast<float4*>(p.part_v + base + 32 * c + e) =
                  make_float4(vv[e], vv[e + 1], vv[e + 2], vv[e + 3]);
            }
          }
        }
      } else {
        const bool row_ok = kj < S;
        // global-row gradients that belong to this key position
        const int blk = kj / W;
        const int64_t gbase = (static_cast<int64_t>(b) * gridDim.y + hk) * static_cast<int64_t>(p.NG);
        int grow[5];
        float gsc[5];
        int ng = 0;
        if (row_ok) {
          if (kj == blk * W) {
            grow[ng] = blk * R;
            gsc[ng] = 1.f;
            ++ng;
          }
          if (R > 1) {
            float rs = 1.f;
            if (p.relay_scale) rs = E::to_f(E::from_f(expf(p.relay_scale[hk])));
            const int32_t* src = p.gsrc + ((static_cast<int64_t>(b) * gridDim.y + hk) * p.NB + blk) * p.top_k;
            for (int t = 0; t < p.top_k; ++t)
              if (src[t] == kj) {
                grow[ng] = blk * R + 1 + t;
                gsc[ng] = rs;
                ++ng;
              }
          }
        }
        T* dkrow = reinterpret_cast<T*>(p.dk) + b * p.dk_sb + hk * p.dk_sh + static_cast<int64_t>(kj) * p.dk_ss;
        T* dvrow = reinterpret_cast<T*>(p.dv) + b * p.dv_sb + hk * p.dv_sh + static_cast<int64_t>(kj) * p.dv_ss;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float vk[32], vv[32];
          tmem_ld32(tmem + lane_off + C::COL_DK + 32 * c, vk);
          tmem_ld32(tmem + lane_off + C::COL_DV + 32 * c, vv);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int e = 0; e < 32; ++e) vk[e] *= p.scale;
            for (int g = 0; g < ng; ++g) {
              const float* gk = p.dgk + (gbase + grow[g]) * D + 32 * c;
              const float* gv = p.dgv + (gbase + grow[g]) * D + 32 * c;
#pragma unroll
              for (int e = 0; e < 32; e += 4) {
                const float4 a = *reinterpret_cast<const float4*>(gk + e);
                const float4 bb = *reinterpret_cast<const float4*>(gv + e);
                vk[e] += gsc[g] * a.x; vk[e + 1] += gsc[g] * a.y; vk[e + 2] += gsc[g] * a.z; vk[e + 3] += gsc[g] * a.w;
                vv[e] += gsc[g] * bb.x; vv[e + 1] += gsc[g] * bb.y; vv[e + 2] += gsc[g] * bb.z; vv[e + 3] += gsc[g] * bb.w;
              }
            }
#pragma unroll
            for (int u4 = 0; u4 < 4; ++u4) {
              uint4 a, bb;
              a.x = E::pack(vk[8 * u4 + 0], vk[8 * u4 + 1]);
              a.y = E::pack(vk[8 * u4 + 2], vk[8 * u4 + 3]);
              a.z = E::pack(vk[8 * u4 + 4], vk[8 * u4 + 5]);
              a.w = E::pack(vk[8 * u4 + 6], vk[8 * u4 + 7]);
              bb.x = E::pack(vv[8 * u4 + 0], vv[8 * u4 + 1]);
              bb.y = E::pack(vv[8 * u4 + 2], vv[8 * u4 + 3]);
              bb.z = E::pack(vv[8 * u4 + 4], vv[8 * u4 + 5]);
              bb.w = E::pack(vv[8 * u4 + 6], vv[8 * u4 + 7]);
              *reinterpret_cast<uint4*>(dkrow + 32 * c + 8 * u4) = a;
              *reinterpret_cast<uint4*>(dvrow + 32 * c + 8 * u4) = bb;
            }
          }
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
template <typename K>
static cudaError_t set_smem(K kern, int bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int D, bool BF16>
static cudaError_t launch_bwd_t(const BwdLaunch& L, cudaStream_t st) {
  const QueryPassParams& qp = L.qp;
  const int B = qp.B, H = qp.H, S = qp.S;
  const int Spad = qp.n_qtiles * kTile;
  cudaError_t e;
  {
    constexpr int RPB = 8 * (32 / (D / 8));  // rows per 256-thread block
    dim3 grid((Spad + RPB - 1) / RPB, B * H);
    delta_kernel<D, BF16><<<grid, 256, 0, st>>>(L.o, L.d_o, L.o_st[0], L.o_st[1], L.o_st[2], L.do_st[0], L.do_st[1],
                                                L.do_st[2], L.lse_in, H, S, Spad, L.lse2, L.delta);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const KeyPassParams& gp = L.global;
  const int Hkv = gp.H / gp.kv_groups;
  const int n_gtiles = (gp.NG + kTile - 1) / kTile;
  {
    auto kern = keypass_kernel<D, BF16, true>;
    if ((e = set_smem(kern, KeyCfg<D>::SMEM)) != cudaSuccess) return e;
    kern<<<dim3(n_gtiles * gp.n_split, Hkv, B), 256, KeyCfg<D>::SMEM, st>>>(gp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  {
    const int64_t n4 = static_cast<int64_t>(B) * Hkv * gp.NG * D / 4;
    const int64_t nb = (n4 + 255) / 256;
    reduce_kernel<<<static_cast<int>(nb < 4096 ? nb : 4096), 256, 0, st>>>(
        reinterpret_cast<const float4*>(gp.part_k), reinterpret_cast<const float4*>(gp.part_v), n4, gp.n_split,
        reinterpret_cast<float4*>(L.dgk), reinterpret_cast<float4*>(L.dgv));
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (L.d_alpha && gp.R > 1) {
    dalpha_kernel<BF16><<<Hkv, 256, 0, st>>>(L.dgk, L.dgv, L.gk_rows, L.gv_rows, B, Hkv, gp.NG, gp.R, D, L.d_alpha);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const KeyPassParams& lp = L.local;
  {
    auto kern = keypass_kernel<D, BF16, false>;
    if ((e = set_smem(kern, KeyCfg<D>::SMEM)) != cudaSuccess) return e;
    kern<<<dim3(lp.n_ktiles, Hkv, B), 256, KeyCfg<D>::SMEM, st>>>(lp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  {
    auto kern = dq_kernel<D, BF16>;
    if ((e = set_smem(kern, DqCfg<D>::SMEM)) != cudaSuccess) return e;
    kern<<<dim3(qp.n_qtiles, H, B), 256, DqCfg<D>::SMEM, st>>>(qp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_bwd(const BwdLaunch& L, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_bwd_t<128, true>(L, stream) : launch_bwd_t<128, false>(L, stream);
  return bf16 ? launch_bwd_t<64, true>(L, stream) : launch_bwd_t<64, false>(L, stream);
}

}  // namespace cra
