// fwd.cu -- forward pass of the causal 3-phase sqrt(N) attention on sm_100a.
//
// One CTA computes TWO consecutive 128-query tiles (A = [m0, m0+128),
// B = [m0+128, m0+256)) of one (b, h).  The keys they need -- the local band
// and a prefix of the (b, h) global-row list (strided + relay rows,
// geom.cuh) -- are streamed ONCE through shared memory and used by both
// tiles (PairSchedule), halving L2 -> SMEM traffic per FLOP compared with one
// tile per CTA.  Each tile runs one online softmax over all its keys, i.e. the
// reference forward's three phases (core.py:907-1158) folded into one loop.
//
// Warp roles (320 threads):
//   warp 0      TMA producer: Q_A, Q_B once, then K_j, V_j, K_j+1, ... into a
//               ring of NSLOT 128-row slots (K and V tiles are separate
//               ring entries).
//   warp 1      tcgen05 issuer (one thread) + TMEM owner.  Per key tile j:
//               S_A = Q_A K_j^T, S_B = Q_B K_j^T (each only if that tile
//               needs K_j), then O_A += P_A V_{j-1}, O_B += P_B V_{j-1}.
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B: a thread owns
//               one query row (TMEM lane = 32 * (warp % 4) + lane).  It loads
//               its score row, masks it with per-row [lo, hi) column bounds,
//               updates the running max / sum and writes P (bf16 / f16,
//               swizzled) to shared memory.  O is rescaled in TMEM only when
//               the running max grows by more than 2^8 (exact either way).
// A CTA may also work on one GPU's shard of a sequence split across GPUs:
// queries [q_begin, q_begin + q_len) with K / V rows from kv_begin (a W - 1
// row halo before the shard) and the full global-row list.
// While one softmax warpgroup works on its scores the tensor core computes
// the other tile's scores and the PV products (ping-pong).
#include "geom.cuh"
#include "params.h"
#include "sm100.cuh"

namespace cra {

template <int D>
struct FwdCfg {
  static constexpr int TB = kTile * D * 2;            // one [128 x D] tile
  static constexpr int NSLOT = (D == 128) ? 3 : 6;    // K/V ring slots
  static constexpr int P_BYTES = kTile * kTile * 2;
  static constexpr int OFF_Q = 0;                      // Q_A, Q_B
  static constexpr int OFF_P = OFF_Q + 2 * TB;         // P_A, P_B
  static constexpr int OFF_RING = OFF_P + 2 * P_BYTES;
  static constexpr int OFF_BAR = OFF_RING + NSLOT * TB;
  static constexpr int B_QFULL = 0;
  static constexpr int B_FULL = 1;                     // [NSLOT]
  static constexpr int B_EMPTY = B_FULL + NSLOT;       // [NSLOT]
  static constexpr int B_SFULL = B_EMPTY + NSLOT;      // [2] per query tile
  static constexpr int B_SFREE = B_SFULL + 2;          // [2]
  static constexpr int B_PFULL = B_SFREE + 2;          // [2]
  static constexpr int B_PVDONE = B_PFULL + 2;         // [2]
  static constexpr int B_DRAIN = B_PVDONE + 2;
  static constexpr int N_BAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;  // tmem slot, abort flag
  static constexpr int SMEM = OFF_MISC + 16 + 1024;     // + alignment slack
  static constexpr int TMEM_COLS = 512;
  // TMEM columns: S_A, S_B (128 each), then O_A, O_B (D each)
  static constexpr int COL_S = 0, COL_O = 256;
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(320, 1) fwd_kernel(const __grid_constant__ QueryPassParams p) {
  using C = FwdCfg<D>;
  using E = Elt<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_pairs = (p.q_len + 2 * kTile - 1) / (2 * kTile);
  const int pr = n_pairs - 1 - static_cast<int>(blockIdx.x);  // longest pairs first
  const int h = blockIdx.y, b = blockIdx.z, hk = h / p.kv_groups;
  const int m0 = p.q_begin + pr * 2 * kTile;  // absolute position of the first query
  const int W = p.W, R = p.R;
  const int q_end = p.q_begin + p.q_len;
  const PairSchedule sch(m0, q_end, W, R);

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR = [&](int i) { return bar0 + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Abort ab{abort_flag, p.err};

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_QFULL), 1);
    for (int i = 0; i < C::NSLOT; ++i) {
      mbar_init(BAR(C::B_FULL + i), 1);
      mbar_init(BAR(C::B_EMPTY + i), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(BAR(C::B_SFULL + x), 1);
      mbar_init(BAR(C::B_SFREE + x), 128);
      mbar_init(BAR(C::B_PFULL + x), 128);
      mbar_init(BAR(C::B_PVDONE + x), 1);
    }
    mbar_init(BAR(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nload = 2 * sch.ntiles;  // ring entries: K_0, V_0, K_1, V_1, ...

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch(&p.tm_q);
      tma_prefetch(&p.tm_k);
      tma_prefetch(&p.tm_v);
      tma_prefetch(&p.tm_gk);
      tma_prefetch(&p.tm_gv);
      const int nq = sch.valid_b ? 2 : 1;
      mbar_expect_tx(BAR(C::B_QFULL), nq * C::TB);
      for (int x = 0; x < nq; ++x)
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sbase + C::OFF_Q + x * C::TB + c * kTile * 128, &p.tm_q, BAR(C::B_QFULL), c * 64,
                      m0 + x * kTile - p.q_begin, h, b);
      int issued = 0;
      for (int i = 0; i < nload; ++i) {
        const int sl = i % C::NSLOT;
        if (i >= C::NSLOT && !mbar_wait(BAR(C::B_EMPTY + sl), ((i / C::NSLOT) - 1) & 1, ab)) break;
        int row0;
        bool g, ua, ub;
        sch.tile(i >> 1, row0, g, ua, ub);
        const bool is_v = i & 1;
        const CUtensorMap* m = g ? (is_v ? &p.tm_gv : &p.tm_gk) : (is_v ? &p.tm_v : &p.tm_k);
        mbar_expect_tx(BAR(C::B_FULL + sl), C::TB);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sbase + C::OFF_RING + sl * C::TB + c * kTile * 128, m, BAR(C::B_FULL + sl), c * 64,
                      g ? row0 : row0 - p.kv_begin, hk, b);
        ++issued;
      }
      // Do not leave while copies into this CTA's shared memory are in
      // flight (only reachable after an abort).
      if (*abort_flag)
        for (int i = (issued > C::NSLOT ? issued - C::NSLOT : 0); i < issued; ++i)
          mbar_wait_bounded(BAR(C::B_FULL + i % C::NSLOT), (i / C::NSLOT) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    {  // whole warp, converged; one elected lane issues
      constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kTile, false, false);
      constexpr uint32_t ID_O = idesc_f16(BF16, kTile, D, false, true);
      bool ok = warp_wait(BAR(C::B_QFULL), 0, ab);
      int ns[2] = {0, 0};   // score tiles issued per query tile
      int npv[2] = {0, 0};  // PV products issued per query tile
      auto issue_pv = [&](int j) -> bool {
        int row0;
        bool g, use[2];
        sch.tile(j, row0, g, use[0], use[1]);
        const int i = 2 * j + 1, sl = i % C::NSLOT;
        if (!warp_wait(BAR(C::B_FULL + sl), (i / C::NSLOT) & 1, ab)) return false;
        const uint32_t vs = sbase + C::OFF_RING + sl * C::TB;
        for (int x = 0; x < 2; ++x) {
          if (!use[x]) continue;
          if (!warp_wait(BAR(C::B_PFULL + x), npv[x] & 1, ab)) return false;
          tc_fence_after();
          const uint32_t ps = sbase + C::OFF_P + x * C::P_BYTES;
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk) {
            const uint64_t a = sdesc(ps + (kk >> 2) * kTile * 128 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc(vs + kk * 16 * 128, kTile * 128, 1024);
            mma_ss_w(tmem + C::COL_O + x * D, a, bd, ID_O, (npv[x] > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit_w(BAR(C::B_PVDONE + x));
          ++npv[x];
        }
        mma_commit_w(BAR(C::B_EMPTY + sl));
        return true;
      };
      for (int j = 0; ok && j < sch.ntiles; ++j) {
        int row0;
        bool g, use[2];
        sch.tile(j, row0, g, use[0], use[1]);
        const int i = 2 * j, sl = i % C::NSLOT;
        if (!warp_wait(BAR(C::B_FULL + sl), (i / C::NSLOT) & 1, ab)) { ok = false; break; }
        const uint32_t ks = sbase + C::OFF_RING + sl * C::TB;
        for (int x = 0; x < 2 && ok; ++x) {
          if (!use[x]) continue;
          if (ns[x] > 0 && !warp_wait(BAR(C::B_SFREE + x), (ns[x] - 1) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          const uint32_t qs = sbase + C::OFF_Q + x * C::TB;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kTile * 128 + (kk & 3) * 32;
            mma_ss_w(tmem + C::COL_S + x * kTile, sdesc(qs + off, 16, 1024), sdesc(ks + off, 16, 1024), ID_S,
                   kk > 0 ? 1u : 0u);
          }
          mma_commit_w(BAR(C::B_SFULL + x));
          ++ns[x];
        }
        if (!ok) break;
        mma_commit_w(BAR(C::B_EMPTY + sl));
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(sch.ntiles - 1);
      if (!ok) {
        // aborting: let every MMA already issued finish before TMEM is freed
        mma_commit_w(BAR(C::B_DRAIN));
        mbar_wait_bounded(BAR(C::B_DRAIN), 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int x = (warp - 2) >> 2;           // 0: tile A, 1: tile B
    const int r = ((warp & 3) << 5) | lane;  // row = TMEM lane
    const int qi = m0 + x * kTile + r;
    const bool tile_ok = (x == 0) || sch.valid_b;
    const bool row_ok = qi < q_end;
    const int ls = local_start(qi, W);
    const int cnt = gcount(qi, W, R);
    const uint32_t lane_off = static_cast<uint32_t>(r & ~31) << 16;
    const uint32_t scol = tmem + lane_off + C::COL_S + x * kTile;
    const uint32_t ocol = tmem + lane_off + C::COL_O + x * D;
    const float sl = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    int n = 0;  // key tiles processed by this query tile
    bool ok = true;
    for (int j = 0; tile_ok && j < sch.ntiles; ++j) {
      int row0;
      bool g, ua, ub;
      sch.tile(j, row0, g, ua, ub);
      if (!(x == 0 ? ua : ub)) continue;
      if (!mbar_wait(BAR(C::B_SFULL + x), n & 1, ab)) { ok = false; break; }
      tc_fence_after();
      float s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(scol + 32 * c, s[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(BAR(C::B_SFREE + x));
      int lo, hi;
      if (!g) {
        lo = ls - row0;
        hi = qi - row0 + 1;
      } else {
        lo = 0;
        hi = cnt - row0;
      }
      if (!row_ok) { lo = 0; hi = 0; }
      lo = max(lo, 0);
      hi = min(hi, kTile);
      float mx = -INFINITY;
      if (lo == 0 && hi == kTile) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) mx = fmaxf(mx, s[c][e]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int col = 32 * c + e;
            s[c][e] = (col >= lo && col < hi) ? s[c][e] : -INFINITY;
            mx = fmaxf(mx, s[c][e]);
          }
      }
      mx *= sl;
      const bool need = mx > m_run + 8.0f;  // false while the row has seen nothing
      const bool any = __any_sync(0xffffffffu, need);
      float factor = 1.f;
      if (any && mx > m_run) {
        factor = ex2(m_run - mx);  // ex2(-inf) = 0 on the first update
        m_run = mx;
      }
      const float mu = (m_run == -INFINITY) ? 0.f : m_run;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          s[c][e] = ex2(fmaf(s[c][e], sl, -mu));
          sum += s[c][e];
        }
      l_run = l_run * factor + sum;
      if (n > 0) {
        if (!mbar_wait(BAR(C::B_PVDONE + x), (n - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        if (any) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            tmem_ld32(ocol + 32 * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= factor;
            tmem_st32(ocol + 32 * c, o);
          }
          tmem_st_wait();
        }
      }
      uint8_t* prow = smem + C::OFF_P + x * C::P_BYTES;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int c = u >> 2, e0 = (u & 3) * 8;
        uint4 pk;
        pk.x = E::pack(s[c][e0 + 0], s[c][e0 + 1]);
        pk.y = E::pack(s[c][e0 + 2], s[c][e0 + 3]);
        pk.z = E::pack(s[c][e0 + 4], s[c][e0 + 5]);
        pk.w = E::pack(s[c][e0 + 6], s[c][e0 + 7]);
        *reinterpret_cast<uint4*>(prow + sw128_off(r, u, kTile)) = pk;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR(C::B_PFULL + x));
      ++n;
    }
    // ---------------------------------------------------------- epilogue
    if (tile_ok && ok && n > 0 && mbar_wait(BAR(C::B_PVDONE + x), (n - 1) & 1, ab)) {
      tc_fence_after();
      const float inv = 1.f / fmaxf(l_run, 1e-6f);
      typename E::T* orow = reinterpret_cast<typename E::T*>(p.out) + b * p.out_sb + h * p.out_sh +
                            static_cast<int64_t>(qi - p.q_begin) * p.out_ss;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(ocol + 32 * c, o);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 pk;
            pk.x = E::pack(o[8 * u + 0] * inv, o[8 * u + 1] * inv);
            pk.y = E::pack(o[8 * u + 2] * inv, o[8 * u + 3] * inv);
            pk.z = E::pack(o[8 * u + 4] * inv, o[8 * u + 5] * inv);
            pk.w = E::pack(o[8 * u + 6] * inv, o[8 * u + 7] * inv);
            *reinterpret_cast<uint4*>(orow + 32 * c + 8 * u) = pk;
          }
        }
      }
      if (row_ok)
        p.lse[(static_cast<int64_t>(b) * p.H + h) * p.q_len + (qi - p.q_begin)] =
            (m_run + log2f(fmaxf(l_run, 1e-6f))) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int D, bool BF16>
static cudaError_t launch_fwd_t(const QueryPassParams& p, cudaStream_t stream) {
  using C = FwdCfg<D>;
  auto kern = fwd_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid((p.q_len + 2 * kTile - 1) / (2 * kTile), p.H, p.B);
  kern<<<grid, 320, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_fwd(const QueryPassParams& p, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_fwd_t<128, true>(p, stream) : launch_fwd_t<128, false>(p, stream);
  return bf16 ? launch_fwd_t<64, true>(p, stream) : launch_fwd_t<64, false>(p, stream);
}

}  // namespace cra
