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
//   warp 1      tcgen05 issuer (whole warp, one elected lane) + TMEM owner.
//               Per key tile j and query tile x in {A, B} that needs it:
//               O_x += P_x V_{j'} for x's previous key tile j', then
//               S_x = Q_x K_j^T.
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B: a thread owns
//               one query row (TMEM lane = 32 * (warp % 4) + lane).  It loads
//               its score row, masks it with per-row [lo, hi) column bounds,
//               updates the running max / sum and writes P (16-bit) back into
//               TMEM over the scores; P V is a TS-form MMA (A from TMEM).  O
//               is rescaled in TMEM only when the running max grows by more
//               than 2^8 (exact either way).
// TMEM holds S/P and O of both tiles (4 x 128 columns for D = 128).  A tile's
// next scores are issued after its PV product, so MMA issue order protects
// P, and the commit that signals "scores ready" also covers every earlier PV
// product: when the softmax sees S_x(n), O_x holds all of P_x V up to n - 1.
// A CTA may also work on one GPU's shard of a sequence split across GPUs:
// queries [q_begin, q_begin + q_len) with K / V rows from kv_begin and the
// full global-row list; the pairs whose window reaches below kv_begin read
// their band from a small edge copy (halo rows of the previous shard + the
// shard's first rows) instead.
// While one softmax warpgroup works on its scores the tensor core computes
// the other tile's scores and the PV products (ping-pong).
#include "geom.cuh"
#include "params.h"
#include "sm100.cuh"

namespace cra {

// Optional cycle counters (build with -DCRA_PROF; read with cra_fwd_prof).
#ifdef CRA_PROF
__device__ unsigned long long g_fwd_prof[32];
#define FPROF_DECL unsigned long long pacc[32] = {};
#define FPROF_T(v) const unsigned long long v = clock64()
#define FPROF_ADD(k, t0) (pacc[k] += clock64() - (t0))
#define FPROF_CNT(k, n) (pacc[k] += static_cast<unsigned long long>(n))
#define FPROF_FLUSH()                                                    \
  if ((threadIdx.x & 31) == 0)                                           \
    _Pragma("unroll") for (int k = 0; k < 32; ++k) if (pacc[k]) atomicAdd(&g_fwd_prof[k], pacc[k]);
#else
#define FPROF_DECL
#define FPROF_T(v)
#define FPROF_ADD(k, t0)
#define FPROF_CNT(k, n)
#define FPROF_FLUSH()
#endif

template <int D>
struct FwdCfg {
  static constexpr int TB = kTile * D * 2;            // one [128 x D] tile
  static constexpr int NSLOT = (D == 128) ? 5 : 12;   // K/V ring slots
  static constexpr int OFF_Q = 0;                      // Q_A, Q_B
  static constexpr int OFF_RING = OFF_Q + 2 * TB;
  static constexpr int OFF_BAR = OFF_RING + NSLOT * TB;
  static constexpr int B_QFULL = 0;
  static constexpr int B_FULL = 1;                     // [NSLOT]
  static constexpr int B_EMPTY = B_FULL + NSLOT;       // [NSLOT]
  static constexpr int B_SFULL = B_EMPTY + NSLOT;      // [2] per query tile
  static constexpr int B_PFULL = B_SFULL + 2;          // [2]
  static constexpr int B_ODONE = B_PFULL + 2;          // [2] all PV products of a tile done
  static constexpr int B_DRAIN = B_ODONE + 2;
  static constexpr int N_BAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;  // tmem slot, abort flag
  static constexpr int SMEM = OFF_MISC + 16 + 1024;     // + alignment slack
  static constexpr int TMEM_COLS = 512;
  // TMEM columns: S_A, S_B (128 each; P over the first 64), then O_A, O_B (D each)
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
  const int h = blockIdx.y, b = blockIdx.z, hk = h / p.kv_groups;
  // Positions below are in the coordinates of one sequence; these offsets
  // map them to tensor rows: Q / O rows (qoff), K / V rows (koff), global
  // rows (goff).  A packed variable-length batch maps each CTA to one
  // document (docs table); a sequence shard offsets by its begin.
  int q_begin = p.q_begin, q_len = p.q_len, W = p.W, R = p.R, pr;
  int qoff = -p.q_begin, koff = -p.kv_begin, goff = 0;
  if (p.docs) {
    int lo = 0, hi = p.n_docs - 1;  // last document whose pair0 <= blockIdx.x
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.docs[mid].pair0 <= static_cast<int>(blockIdx.x)) lo = mid; else hi = mid - 1;
    }
    const DocInfo dc = p.docs[lo];
    q_begin = 0;
    q_len = dc.len;
    W = dc.W;
    R = dc.R;
    qoff = koff = dc.start;
    goff = dc.g0;
    const int np = (dc.len + 2 * kTile - 1) / (2 * kTile);
    pr = np - 1 - (static_cast<int>(blockIdx.x) - dc.pair0);  // longest pairs of the document first
  } else {
    const int n_pairs = (p.q_len + 2 * kTile - 1) / (2 * kTile);
    pr = n_pairs - 1 - static_cast<int>(blockIdx.x);  // longest pairs first
  }
  const int m0 = q_begin + pr * 2 * kTile;  // position of the first query
  const int q_end = q_begin + q_len;
  const PairSchedule sch(m0, q_end, W, R);

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR = [&](int i) { return bar0 + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Abort ab{abort_flag, p.err};
  FPROF_DECL

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_QFULL), 1);
    for (int i = 0; i < C::NSLOT; ++i) {
      mbar_init(BAR(C::B_FULL + i), 1);
      mbar_init(BAR(C::B_EMPTY + i), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(BAR(C::B_SFULL + x), 1);
      mbar_init(BAR(C::B_PFULL + x), 128);
      mbar_init(BAR(C::B_ODONE + x), 1);
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
                      m0 + x * kTile + qoff, h, b);
      // band keys of this pair from the edge copy when its window reaches
      // below this shard's own K / V rows
      const bool use_edge = p.has_edge && local_start(m0, W) < p.kv_begin;
      if (p.has_edge) {
        tma_prefetch(&p.tm_ke);
        tma_prefetch(&p.tm_ve);
      }
      int issued = 0;
      for (int i = 0; i < nload; ++i) {
        const int sl = i % C::NSLOT;
        if (i >= C::NSLOT && !mbar_wait(BAR(C::B_EMPTY + sl), ((i / C::NSLOT) - 1) & 1, ab)) break;
        int row0;
        bool g, ua, ub;
        sch.tile(i >> 1, row0, g, ua, ub);
        const bool is_v = i & 1;
        const CUtensorMap* m = g ? (is_v ? &p.tm_gv : &p.tm_gk)
                                 : use_edge ? (is_v ? &p.tm_ve : &p.tm_ke) : (is_v ? &p.tm_v : &p.tm_k);
        mbar_expect_tx(BAR(C::B_FULL + sl), C::TB);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sbase + C::OFF_RING + sl * C::TB + c * kTile * 128, m, BAR(C::B_FULL + sl), c * 64,
                      g ? row0 + goff : use_edge ? row0 - p.edge_begin : row0 + koff, hk, b);
        ++issued;
      }
      // Do not leave while copies into this CTA's shared memory are in
      // flight (only reachable after an abort).
      if (*abort_flag) {
        for (int i = (issued > C::NSLOT ? issued - C::NSLOT : 0); i < issued; ++i)
          mbar_wait_bounded(BAR(C::B_FULL + i % C::NSLOT), (i / C::NSLOT) & 1);
        mbar_wait_bounded(BAR(C::B_QFULL), 0);  // the Q tiles
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    {  // whole warp, converged; one elected lane issues
      constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kTile, false, false);
      constexpr uint32_t ID_O = idesc_f16(BF16, kTile, D, false, true);
      FPROF_T(tstart);
      bool ok = warp_wait(BAR(C::B_QFULL), 0, ab);
      FPROF_ADD(3, tstart);
      const uint64_t qdesc[2] = {sdesc(sbase + C::OFF_Q, 16, 1024), sdesc(sbase + C::OFF_Q + C::TB, 16, 1024)};
      int ns[2] = {0, 0};      // score tiles issued per query tile
      int pend[2] = {-1, -1};  // key tile whose PV product is still to issue
      auto full = [&](int i) { return warp_wait(BAR(C::B_FULL + i % C::NSLOT), (i / C::NSLOT) & 1, ab); };
      // O_x += P_x V_jp  (P from TMEM over S_x; V_jp is ring entry 2 jp + 1)
      auto issue_pv = [&](int x) -> bool {
        const int jp = pend[x], i = 2 * jp + 1;
        FPROF_T(t0);
        if (!warp_wait(BAR(C::B_PFULL + x), (ns[x] - 1) & 1, ab)) return false;
        FPROF_ADD(1, t0);
        FPROF_T(t1);
        if (!full(i)) return false;
        FPROF_ADD(2, t1);
        tc_fence_after();
        const uint64_t vd = sdesc(sbase + C::OFF_RING + (i % C::NSLOT) * C::TB, kTile * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          mma_ts_w(tmem + C::COL_O + x * D, tmem + C::COL_S + x * kTile + kk * 8, vd + ((kk * 16 * 128) >> 4), ID_O,
                   (ns[x] > 1 || kk > 0) ? 1u : 0u);
        pend[x] = -1;
        return true;
      };
      for (int j = 0; ok && j <= sch.ntiles; ++j) {
        int row0 = 0;
        bool g = false, use[2] = {false, false};
        if (j < sch.ntiles) sch.tile(j, row0, g, use[0], use[1]);
        for (int x = 0; x < 2 && ok; ++x) {
          if (pend[x] >= 0 && !issue_pv(x)) { ok = false; break; }
          if (!use[x]) continue;
          FPROF_T(t0);
          if (!full(2 * j)) { ok = false; break; }
          FPROF_ADD(2, t0);
          tc_fence_after();
          const uint64_t kd = sdesc(sbase + C::OFF_RING + ((2 * j) % C::NSLOT) * C::TB, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * kTile * 128 + (kk & 3) * 32) >> 4;
            mma_ss_w(tmem + C::COL_S + x * kTile, qdesc[x] + off, kd + off, ID_S, kk > 0 ? 1u : 0u);
          }
          mma_commit_w(BAR(C::B_SFULL + x));
          ++ns[x];
          pend[x] = j;
        }
        if (!ok) break;
        if (j > 0) mma_commit_w(BAR(C::B_EMPTY + (2 * j - 1) % C::NSLOT));  // V_{j-1}: both PV products issued
        if (j < sch.ntiles) mma_commit_w(BAR(C::B_EMPTY + (2 * j) % C::NSLOT));  // K_j: both score tiles issued
      }
      if (ok)
        for (int x = 0; x < 2; ++x)
          if (ns[x] > 0) mma_commit_w(BAR(C::B_ODONE + x));
      FPROF_ADD(0, tstart);
      FPROF_CNT(30, ns[0] + ns[1]);
      FPROF_CNT(31, 1);
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
      FPROF_T(tw);
      if (!mbar_wait(BAR(C::B_SFULL + x), n & 1, ab)) { ok = false; break; }
      FPROF_ADD(8, tw);
      FPROF_T(tl);
      tc_fence_after();
      float s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(scol + 32 * c, s[c]);
      tmem_ld_wait();
      FPROF_ADD(9, tl);
      FPROF_T(tc);
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
      if (__any_sync(0xffffffffu, lo != 0 || hi != kTile)) {
        // visible columns [lo, hi) as one 32-bit mask per 32-column chunk
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int a = min(max(lo - 32 * c, 0), 32), z = min(max(hi - 32 * c, 0), 32);
          const uint32_t mz = z >= 32 ? 0xffffffffu : ((1u << z) - 1u);
          const uint32_t ma = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
          const uint32_t m = mz & ~ma;
#pragma unroll
          for (int e = 0; e < 32; ++e) s[c][e] = (m & (1u << e)) ? s[c][e] : -INFINITY;
        }
      }
      // row max with 8 independent partial maxima (short dependency chains)
      float pm0 = s[0][0], pm1 = s[0][1], pm2 = s[0][2], pm3 = s[0][3];
      float pm4 = s[0][4], pm5 = s[0][5], pm6 = s[0][6], pm7 = s[0][7];
#pragma unroll
      for (int k = 1; k < 16; ++k) {
        pm0 = fmaxf(pm0, s[k >> 2][8 * (k & 3) + 0]);
        pm1 = fmaxf(pm1, s[k >> 2][8 * (k & 3) + 1]);
        pm2 = fmaxf(pm2, s[k >> 2][8 * (k & 3) + 2]);
        pm3 = fmaxf(pm3, s[k >> 2][8 * (k & 3) + 3]);
        pm4 = fmaxf(pm4, s[k >> 2][8 * (k & 3) + 4]);
        pm5 = fmaxf(pm5, s[k >> 2][8 * (k & 3) + 5]);
        pm6 = fmaxf(pm6, s[k >> 2][8 * (k & 3) + 6]);
        pm7 = fmaxf(pm7, s[k >> 2][8 * (k & 3) + 7]);
      }
      float mx = fmaxf(fmaxf(fmaxf(pm0, pm1), fmaxf(pm2, pm3)), fmaxf(fmaxf(pm4, pm5), fmaxf(pm6, pm7)));
      mx *= sl;
      const bool need = mx > m_run + 8.0f;  // false while the row has seen nothing
      const bool any = __any_sync(0xffffffffu, need);
      float factor = 1.f;
      if (any && mx > m_run) {
        factor = ex2(m_run - mx);  // ex2(-inf) = 0 on the first update
        m_run = mx;
      }
      const float mu = (m_run == -INFINITY) ? 0.f : m_run;
      FPROF_ADD(10, tc);
      FPROF_T(tp);
      // P = 2^(s * scale_log2 - m), written as 16-bit pairs over score
      // columns [0, 64) of this tile.
      const float nmu = -mu;
      float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;  // partial row sums
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float a0 = s[c][e], a1 = s[c][e + 1];
          ffma2(a0, a1, sl, nmu);
          a0 = ex2(a0);
          a1 = ex2(a1);
          if (e & 2)
            fadd2(q2, q3, a0, a1);
          else
            fadd2(q0, q1, a0, a1);
          pk[e / 2] = E::pack(a0, a1);
        }
        tmem_st16(scol + 16 * c, pk);
      }
      l_run = l_run * factor + ((q0 + q1) + (q2 + q3));
      // Rescale O (after P, when the scores are dead).  O_x already holds
      // every PV product up to key tile n - 1: the commit that signalled
      // these scores also covers them.
      if (n > 0 && any) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(ocol + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= factor;
          tmem_st32(ocol + 32 * c, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(BAR(C::B_PFULL + x));
      FPROF_ADD(11, tp);
      FPROF_CNT(12, any ? 1 : 0);
      ++n;
    }
    // ---------------------------------------------------------- epilogue
    if (tile_ok && ok && n > 0 && mbar_wait(BAR(C::B_ODONE + x), 0, ab)) {
      tc_fence_after();
      const float inv = 1.f / fmaxf(l_run, 1e-6f);
      typename E::T* orow = reinterpret_cast<typename E::T*>(p.out) + b * p.out_sb + h * p.out_sh +
                            static_cast<int64_t>(qi + qoff) * p.out_ss;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(ocol + 32 * c, o);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int u = 0; u < 2; ++u) {  // 16 columns = one 32-byte sector per store
            uint32_t w8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) w8[e] = E::pack(o[16 * u + 2 * e] * inv, o[16 * u + 2 * e + 1] * inv);
            st_global_8w(orow + 32 * c + 16 * u, w8, p.out_v8);
          }
        }
      }
      if (row_ok)
        p.lse[(static_cast<int64_t>(b) * p.H + h) * p.lse_len + (qi + qoff)] =
            (m_run + log2f(fmaxf(l_run, 1e-6f))) * 0.69314718055994531f;
    }
  }

  FPROF_FLUSH()
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

#ifdef CRA_PROF
extern "C" __attribute__((visibility("default"))) int cra_fwd_prof(unsigned long long* out32, int reset) {
  cudaMemcpyFromSymbol(out32, g_fwd_prof, sizeof(g_fwd_prof));
  if (reset) {
    unsigned long long z[32] = {};
    cudaMemcpyToSymbol(g_fwd_prof, z, sizeof(z));
  }
  return 0;
}
#endif

template <int D, bool BF16>
static cudaError_t launch_fwd_t(const QueryPassParams& p, cudaStream_t stream) {
  using C = FwdCfg<D>;
  auto kern = fwd_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.docs ? p.n_pairs_total : (p.q_len + 2 * kTile - 1) / (2 * kTile), p.H, p.B);
  kern<<<grid, 320, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_fwd(const QueryPassParams& p, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_fwd_t<128, true>(p, stream) : launch_fwd_t<128, false>(p, stream);
  return bf16 ? launch_fwd_t<64, true>(p, stream) : launch_fwd_t<64, false>(p, stream);
}

}  // namespace cra
