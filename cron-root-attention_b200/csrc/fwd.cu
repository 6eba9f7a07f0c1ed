// fwd.cu -- forward pass of the causal 3-phase sqrt(N) attention on sm_100a.
//
// One CTA computes one 128-query tile of one (b, h).  The keys it needs are
//   * the local band: 128-key tiles ending at the diagonal (band_tiles()),
//   * a prefix of the (b, h) global-row list (strided + relay rows, geom.cuh),
// and the CTA streams them through ONE online softmax, exactly the reference
// forward's three phases (core.py:907-1158) folded into one loop.
//
// Warp roles (256 threads):
//   warp 0      TMA producer: Q once, then K/V (or G_k/G_v) tiles into an
//               NST-deep ring of shared-memory stages.
//   warp 1      tcgen05 issuer (one thread): S = Q K^T into one of two TMEM
//               score buffers, then O += P V into the TMEM accumulator.
//               Also owns the TMEM allocation.
//   warps 4-7   softmax: thread r owns query row r (= TMEM lane r).  Loads
//               its score row from TMEM, masks it with per-row [lo, hi)
//               column bounds, updates the running max / sum, writes P
//               (bf16/f16, swizzled) to shared memory for the PV MMA.
//               O is rescaled in TMEM only when the running max grows by
//               more than 2^8 (the result is exact either way: p <= 256).
//   warps 2-3   idle.
// Pipelining: S for tile j+1 is issued before PV for tile j, so the tensor
// core works on the next scores while the softmax warps process this tile.
#include "geom.cuh"
#include "params.h"
#include "sm100.cuh"

namespace cra {

template <int D>
struct FwdCfg {
  static constexpr int NST = (D == 128) ? 2 : 4;      // K/V ring depth
  static constexpr int Q_BYTES = kTile * D * 2;
  static constexpr int KV_BYTES = kTile * D * 2;     // one K (or V) tile
  static constexpr int P_BYTES = kTile * kTile * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NST * KV_BYTES;
  static constexpr int OFF_P = OFF_V + NST * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  // barriers: Q_FULL, K_FULL[NST], V_FULL[NST], KV_EMPTY[NST], S_FULL[2],
  // S_FREE[2], P_FULL, PV_DONE
  static constexpr int B_QFULL = 0;
  static constexpr int B_KFULL = 1;
  static constexpr int B_VFULL = B_KFULL + NST;
  static constexpr int B_EMPTY = B_VFULL + NST;
  static constexpr int B_SFULL = B_EMPTY + NST;
  static constexpr int B_SFREE = B_SFULL + 2;
  static constexpr int B_PFULL = B_SFREE + 2;
  static constexpr int B_PVDONE = B_PFULL + 1;
  static constexpr int B_DRAIN = B_PVDONE + 1;
  static constexpr int N_BAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;  // tmem slot, abort flag
  static constexpr int SMEM = OFF_MISC + 16 + 1024;     // + alignment slack
  static constexpr int TMEM_COLS = 512;
  static constexpr int COL_S0 = 0, COL_S1 = 128, COL_O = 256;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(256, 1) fwd_kernel(const __grid_constant__ QueryPassParams p) {
  using C = FwdCfg<D>;
  using E = Elt<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.n_qtiles - 1 - static_cast<int>(blockIdx.x);  // longest tiles first
  const int h = blockIdx.y, b = blockIdx.z, hk = h / p.kv_groups;
  const int m0 = qt * kTile;
  const int W = p.W, S = p.S, R = p.R;

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
    for (int i = 0; i < 2; ++i) {
      mbar_init(BAR(C::B_SFULL + i), 1);
      mbar_init(BAR(C::B_SFREE + i), 128);
    }
    mbar_init(BAR(C::B_PFULL), 128);
    mbar_init(BAR(C::B_PVDONE), 1);
    mbar_init(BAR(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch(&p.tm_q);
      tma_prefetch(&p.tm_k);
      tma_prefetch(&p.tm_v);
      tma_prefetch(&p.tm_gk);
      tma_prefetch(&p.tm_gv);
      mbar_expect_tx(BAR(C::B_QFULL), C::Q_BYTES);
      for (int c = 0; c < D / 64; ++c)
        tma_load_4d(sbase + C::OFF_Q + c * kTile * 128, &p.tm_q, BAR(C::B_QFULL), c * 64, m0, h, b);
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % C::NST;
        if (j >= C::NST && !mbar_wait(BAR(C::B_EMPTY + st), ((j / C::NST) - 1) & 1, ab)) break;
        const bool g = j >= nband;
        const int row0 = g ? (j - nband) * kTile : m0 - j * kTile;
        const CUtensorMap* mk = g ? &p.tm_gk : &p.tm_k;
        const CUtensorMap* mv = g ? &p.tm_gv : &p.tm_v;
        mbar_expect_tx(BAR(C::B_KFULL + st), C::KV_BYTES);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sbase + C::OFF_K + st * C::KV_BYTES + c * kTile * 128, mk, BAR(C::B_KFULL + st), c * 64, row0,
                      hk, b);
        mbar_expect_tx(BAR(C::B_VFULL + st), C::KV_BYTES);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sbase + C::OFF_V + st * C::KV_BYTES + c * kTile * 128, mv, BAR(C::B_VFULL + st), c * 64, row0,
                      hk, b);
        ++issued;
      }
      // Drain: do not leave the CTA while copies into its shared memory are
      // still in flight (only reachable after an abort).
      if (*abort_flag) {
        for (int j = (issued > C::NST ? issued - C::NST : 0); j < issued; ++j) {
          const int st = j % C::NST;
          const uint64_t t0 = globaltimer();
          while (!mbar_try(BAR(C::B_VFULL + st), (j / C::NST) & 1) && globaltimer() - t0 < CRA_WAIT_LIMIT_NS) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_f16(BF16, kTile, kTile, false, false);
      constexpr uint32_t ID_O = idesc_f16(BF16, kTile, D, false, true);
      const uint32_t qs = sbase + C::OFF_Q, ps = sbase + C::OFF_P;
      bool ok = mbar_wait(BAR(C::B_QFULL), 0, ab);
      auto issue_pv = [&](int i) -> bool {
        const int st = i % C::NST;
        if (!mbar_wait(BAR(C::B_PFULL), i & 1, ab)) return false;
        if (!mbar_wait(BAR(C::B_VFULL + st), (i / C::NST) & 1, ab)) return false;
        tc_fence_after();
        const uint32_t vs = sbase + C::OFF_V + st * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint64_t a = sdesc(ps + (kk >> 2) * kTile * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(vs + kk * 16 * 128, kTile * 128, 1024);
          mma_ss(tmem + C::COL_O, a, bd, ID_O, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(BAR(C::B_PVDONE));
        mma_commit(BAR(C::B_EMPTY + st));
        return true;
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % C::NST, sb = j & 1;
        if (!mbar_wait(BAR(C::B_KFULL + st), (j / C::NST) & 1, ab)) { ok = false; break; }
        if (j >= 2 && !mbar_wait(BAR(C::B_SFREE + sb), ((j >> 1) - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ks = sbase + C::OFF_K + st * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = sdesc(qs + (kk >> 2) * kTile * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(ks + (kk >> 2) * kTile * 128 + (kk & 3) * 32, 16, 1024);
          mma_ss(tmem + (sb ? C::COL_S1 : C::COL_S0), a, bd, ID_S, kk > 0 ? 1u : 0u);
        }
        mma_commit(BAR(C::B_SFULL + sb));
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(ntiles - 1);
      if (!ok) {
        // aborting: let every MMA already issued finish before TMEM is freed
        mma_commit(BAR(C::B_DRAIN));
        const uint64_t t0 = globaltimer();
        while (!mbar_try(BAR(C::B_DRAIN), 0) && globaltimer() - t0 < CRA_WAIT_LIMIT_NS) {
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int r = threadIdx.x - 128;
    const int qi = m0 + r;
    const bool row_ok = qi < S;
    const int ls = local_start(qi, W);
    const int cnt = gcount(qi, W, R);
    const uint32_t lane_off = static_cast<uint32_t>(r & ~31) << 16;
    const float sl = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(BAR(C::B_SFULL + sb), (j >> 1) & 1, ab)) { ok = false; break; }
      tc_fence_after();
      float s[4][32];
      const uint32_t scol = tmem + lane_off + (sb ? C::COL_S1 : C::COL_S0);
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(scol + 32 * c, s[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(BAR(C::B_SFREE + sb));
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
      if (j > 0) {
        if (!mbar_wait(BAR(C::B_PVDONE), (j - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
        if (any) {
          const uint32_t ocol = tmem + lane_off + C::COL_O;
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
      // P row -> shared memory, 128B-swizzled, two 64-key chunks
      uint8_t* prow = smem + C::OFF_P;
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
      mbar_arrive(BAR(C::B_PFULL));
    }
    // ---------------------------------------------------------- epilogue
    if (ok && mbar_wait(BAR(C::B_PVDONE), (ntiles - 1) & 1, ab)) {
      tc_fence_after();
      const float inv = 1.f / fmaxf(l_run, 1e-6f);
      const uint32_t ocol = tmem + lane_off + C::COL_O;
      typename E::T* orow = reinterpret_cast<typename E::T*>(p.out) + b * p.out_sb + h * p.out_sh +
                            static_cast<int64_t>(qi) * p.out_ss;
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
        p.lse[(static_cast<int64_t>(b) * p.H + h) * S + qi] = (m_run + log2f(fmaxf(l_run, 1e-6f))) * 0.69314718055994531f;
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
  dim3 grid(p.n_qtiles, p.H, p.B);
  kern<<<grid, 256, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_fwd(const QueryPassParams& p, int D, bool bf16, cudaStream_t stream) {
  if (D == 128) return bf16 ? launch_fwd_t<128, true>(p, stream) : launch_fwd_t<128, false>(p, stream);
  return bf16 ? launch_fwd_t<64, true>(p, stream) : launch_fwd_t<64, false>(p, stream);
}

}  // namespace cra
