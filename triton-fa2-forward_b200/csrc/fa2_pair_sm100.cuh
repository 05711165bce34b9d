// CTA-pair build of the forward kernel (D = 128, fixed lengths, no split-KV): a cluster of two
// CTAs runs every GEMM as one M = 256 tcgen05.mma (cta_group::2) issued by the even CTA.
//
// Why: in the single-CTA kernel each SM streams a whole K and V tile (64 KiB) per K/V step
// from L2 and its tensor core reads Q and K at the full shared-memory bandwidth for QK^T. A
// pair-MMA takes B (K for QK^T, V for PV) half from each CTA, so each SM loads and reads half
// of every K/V tile while both SMs' rows use all of it: per K/V step an SM moves 32 KiB from L2
// instead of 64 and its shared memory serves 160 KiB instead of 256.
//
// Work unit: 512 packed Q rows of one (batch, head block), the pair's four 128-row tiles.
// Tile t of CTA r holds rows row0 + 256 t + 128 r, so pair-tile t (the M = 256 of one MMA) is
// rows [row0 + 256 t, row0 + 256 t + 256). Both CTAs walk the same units (the cluster's
// persistent slots); the K/V loop of a unit covers its last row's causal band.
//
// Roles per CTA are those of the single-CTA kernel (softmax warps 0-7, MMA warp 8, TMA warp 9):
//  * TMA (both CTAs): this CTA's Q rows, the K rows [64 r, 64 r + 64) of each K tile and the V
//    columns [64 r, 64 r + 64) of each V tile, each completing on the even CTA's barrier
//    (which expects both halves); ring slots of 16 KiB, 6 of them.
//  * MMA (even CTA only): the single-CTA schedule with pair instructions; each commit arrives
//    on the barrier of both CTAs (S ready, K/V slot free, Q free, O final, all done).
//  * softmax (both CTAs): unchanged per row; the P hand-offs arrive once per warp on the even
//    CTA's barriers (8 arrivals: 4 warps x 2 CTAs).
// Every wait is bounded as in the single-CTA kernel; both CTAs end with a cluster barrier, so
// neither leaves while the other can still signal it or read its memory.

namespace fa2 {

// ------------------------------------------------------- CTA pairs (cta_group::2)
// A cluster of two CTAs whose MMAs run as one M = 256 instruction on both SMs: the even CTA
// (rank 0) issues every MMA; A (Q or P) comes from each CTA's own rows, B (K or V) is split
// along N between the two CTAs' shared memory, and each CTA's TMEM receives its 128 rows.
// Every tcgen05 alloc / mma / commit of such a kernel uses cta_group::2.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in cluster CTA `rank` (shared::cluster window).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Every thread of both CTAs; orders barrier initialisation and TMEM allocation before any
// cross-CTA use, and at the end keeps both CTAs resident until neither can be signalled.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// One arrival on an mbarrier of a cluster CTA (default semantics: release at CTA scope). The
// data it publishes is TMEM written by tcgen05.st, ordered by tcgen05.wait::st and
// tcgen05.fence::before_thread_sync on this side and fence::after_thread_sync after the wait on
// the other; a cluster-scope release (which also drains this thread's other memory traffic)
// measured ~900 cycles per hand-off.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[smem] * B[smem] over the CTA pair.
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem] over the CTA pair.
__device__ __forceinline__ void mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at shared offset `bar` of both CTAs of the pair when every
// tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(static_cast<uint16_t>(0x3))
      : "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on an mbarrier of
// either CTA of the pair (`cluster_bar`, a shared::cluster address).
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap* m, uint32_t cluster_bar, int c0,
                                                 int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(cluster_bar), "l"(policy)
      : "memory");
}


struct PairCfg {
  static constexpr int D = 128;
  static constexpr int TILE_BYTES = BM * D * 2;          // one CTA's Q tile: 32 KiB
  static constexpr int Q_CHUNK = 128 * 128;              // 128 rows x 128 bytes (64 columns)
  static constexpr int SLOT_BYTES = 16 * 1024;           // half a K tile (64 rows) or V tile (64 cols)
  static constexpr int K_CHUNK = 64 * 128;               // 64 rows x 128 bytes
  static constexpr int STAGES = 6;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = Q_TILES * TILE_BYTES;
  static constexpr int STG_SLOT_BYTES = 32 * 128;        // O staging: 32 rows x 64 columns
  static constexpr int STG_WARP_BYTES = (D / 64) * STG_SLOT_BYTES;
  static constexpr int OFF_STG = OFF_KV + STAGES * SLOT_BYTES;
  static constexpr int OFF_BAR = OFF_STG + SOFTMAX_WARPS * STG_WARP_BYTES;
  static constexpr int B_Q = 0;                      // [2] (even CTA) both CTAs' Q_t landed
  static constexpr int B_KV_FULL = 2;                // [S] (even CTA) both halves of a K/V tile landed
  static constexpr int B_KV_EMPTY = 2 + STAGES;      // [S] slot released by the MMAs
  static constexpr int B_S_FULL = 2 + 2 * STAGES;    // [2] S_t in TMEM
  static constexpr int B_P_FULL = 4 + 2 * STAGES;    // [2] (even CTA) first P chunks of both CTAs
  static constexpr int B_P_LATE = 6 + 2 * STAGES;    // [2] (even CTA) the remaining P chunks
  static constexpr int B_O_FULL = 8 + 2 * STAGES;    // [2] last PV of tile t retired
  static constexpr int B_Q_EMPTY = 10 + 2 * STAGES;  // [2] last QK of tile t retired
  static constexpr int B_MMA_DONE = 12 + 2 * STAGES; // [1] every MMA retired
  static constexpr int NUM_BARS = 13 + 2 * STAGES;
  static constexpr int OFF_TMEM_PTR = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEM_PTR + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
  static constexpr int TMEM_O = 2 * BN;
  static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory budget");
  static_assert(TMEM_O + 2 * D <= TMEM_COLS, "TMEM budget");
};

// Unit slot n of this cluster (512-row blocks); false when the cluster has no n-th slot.
template <bool CAUSAL>
__device__ __forceinline__ bool get_pair_unit(const KArgs& a, int n, Unit& u) {
  const uint32_t G = gridDim.x >> 1, c = blockIdx.x >> 1, nn = static_cast<uint32_t>(n);
  const uint32_t idx = nn * G + ((nn & 1u) ? (G - 1u - c) : c);
  if (idx >= static_cast<uint32_t>(a.num_units)) return false;
  int mb;
  if (CAUSAL || !FA2_HEAD_MAJOR) {
    const uint32_t mi = a.div_xblocks.div(idx);
    u.x = static_cast<int>(idx - mi * a.div_xblocks.d);
    mb = CAUSAL ? a.mblocks - 1 - static_cast<int>(mi) : static_cast<int>(mi);
  } else {
    const uint32_t xs = a.div_mblocks.div(idx);
    u.x = static_cast<int>(xs);
    mb = static_cast<int>(idx - xs * a.div_mblocks.d);
  }
  u.b = static_cast<int>(a.div_hblocks.div(static_cast<uint32_t>(u.x)));
  u.hq0 = (u.x - u.b * a.hblocks) << a.pack_shift;
  u.hkv = static_cast<int>(a.div_group.div(static_cast<uint32_t>(u.hq0)));
  u.row0 = mb * 512;
  u.j0 = 0;
  u.j0b = 0;
  u.q0 = 0;
  u.kv0 = 0;
  u.tb = u.b;
  u.tbkv = u.b;
  u.n_q = a.n_q;
  u.n_kv = a.n_kv;
  u.coff = a.causal_off;
  int kv_end = a.n_kv, kv_end0 = a.n_kv;
  if (CAUSAL) {
    const int last_pos = min((u.row0 + 511) >> a.pack_shift, a.n_q - 1);
    const int last_pos0 = min((u.row0 + 255) >> a.pack_shift, a.n_q - 1);
    kv_end = min(last_pos + 1 + a.causal_off, a.n_kv);
    kv_end0 = min(last_pos0 + 1 + a.causal_off, a.n_kv);
  }
  u.J = max(1, (kv_end + 127) / 128);
  u.J0 = max(1, (kv_end0 + 127) / 128);  // pair-tile 0 stops here (its later tiles are fully masked)
  return true;
}

template <bool CAUSAL, bool BF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
fa2_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const KArgs a) {
  static_assert(HALVES == 1 && !FA2_TWO_ISSUERS, "the pair build uses the 12-warp single-issuer layout");
  constexpr int D = 128;
  using C = PairCfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sraw = smem_u32(smem_raw);
  const uint32_t sbase = (sraw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - sraw);
  auto bar = [&](int i) -> uint32_t { return sbase + C::OFF_BAR + 8u * static_cast<uint32_t>(i); };
  const uint32_t rank = cluster_ctarank();
  const bool lead = (rank == 0);
  // The even CTA's copy of barrier i, as a shared::cluster address.
  auto lbar = [&](int i) -> uint32_t { return mapa_shared(bar(i), 0); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  {
    Unit u0;
    if (!get_pair_unit<CAUSAL>(a, 0, u0)) return;  // both CTAs of the pair alike, before any sync
  }

  if (warp == LOAD_WARP && lane == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(C::B_Q + t), 1);
      mbar_init(bar(C::B_Q_EMPTY + t), 1);
      mbar_init(bar(C::B_S_FULL + t), 1);
      mbar_init(bar(C::B_P_FULL + t), 8);
      mbar_init(bar(C::B_P_LATE + t), 8);
      mbar_init(bar(C::B_O_FULL + t), 1);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::B_KV_FULL + s), 1);
      mbar_init(bar(C::B_KV_EMPTY + s), 1);
    }
    mbar_init(bar(C::B_MMA_DONE), 1);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == MMA_WARP) {
    __syncwarp();
    tmem_alloc_pair(sbase + C::OFF_TMEM_PTR, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + C::OFF_TMEM_PTR);

  bool ok = true;

  if (warp == LOAD_WARP) {
    reg_dealloc<regs_other<D>()>();
    // ------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmO);
      const uint64_t pol_kv = FA2_L2_HINTS ? l2_policy_evict_last() : l2_policy_evict_normal();
      const uint64_t pol_q = FA2_L2_HINTS ? l2_policy_evict_first() : l2_policy_evict_normal();
      int q_loads = 0;
      auto load_q = [&](const Unit& u, int t) {
        const int R = u.row0 + t * 256 + static_cast<int>(rank) * BM;
        const int pos = R >> a.pack_shift;
        const int h = u.hq0 + (R & (a.pack - 1));
        if (lead) mbar_arrive_expect_tx(bar(C::B_Q + t), 2 * C::TILE_BYTES);
        const uint32_t qb = lbar(C::B_Q + t);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d_pair(sbase + C::OFF_Q + t * C::TILE_BYTES + c * C::Q_CHUNK, &tmQ, qb, c * 64, h, u.q0 + pos,
                           u.tb, pol_q);
        }
      };
      if (a.gate != nullptr) ok = flag_wait(a.gate, a.timeout, a.err);
      int i = 0;  // K/V half tiles issued into the ring, over all units
      for (int n = 0; ok; ++n) {
        Unit u;
        if (!get_pair_unit<CAUSAL>(a, n, u)) break;
        if (n > 0 && !mbar_wait(bar(C::B_Q_EMPTY + 0), static_cast<uint32_t>(n - 1) & 1u, a.timeout, a.err)) {
          ok = false;
          break;
        }
        load_q(u, 0);
        for (int k = 0; k < 2 * u.J; ++k) {
          const int st = i % C::STAGES;
          const uint32_t ph = static_cast<uint32_t>(i / C::STAGES) & 1u;
          if (!mbar_wait(bar(C::B_KV_EMPTY + st), ph ^ 1u, a.timeout, a.err)) {
            ok = false;
            break;
          }
          const bool is_v = (k & 1) != 0;
          const int kv_tile = u.j0 + (k >> 1);
          if (lead) mbar_arrive_expect_tx(bar(C::B_KV_FULL + st), 2 * C::SLOT_BYTES);
          const uint32_t kb = lbar(C::B_KV_FULL + st);
          const uint32_t dst = sbase + C::OFF_KV + st * C::SLOT_BYTES;
          if (is_v) {
            // V columns [64 r, 64 r + 64) of the tile's 128 keys.
            tma_load_4d_pair(dst, &tmV, kb, static_cast<int>(rank) * 64, u.kv0 + kv_tile * BN, u.hkv, u.tbkv, pol_kv);
          } else {
            // K rows [64 r, 64 r + 64) of the tile, both 64-column halves of d.
#pragma unroll
            for (int c = 0; c < D / 64; ++c) {
              tma_load_4d_pair(dst + c * C::K_CHUNK, &tmK, kb, c * 64,
                               u.kv0 + kv_tile * BN + static_cast<int>(rank) * 64, u.hkv, u.tbkv, pol_kv);
            }
          }
          ++i;
          if (k == 0) {
            if (n > 0 &&
                !mbar_wait(bar(C::B_Q_EMPTY + 1), static_cast<uint32_t>(n - 1) & 1u, a.timeout, a.err)) {
              ok = false;
              break;
            }
            load_q(u, 1);
          }
        }
        ++q_loads;
      }
      // Drain (even CTA): the phases of its barriers count both CTAs' loads, so once the last
      // ones completed no load of either CTA is in flight. The odd CTA stays resident until
      // the closing cluster barrier, which the even CTA reaches only after this.
      if (lead) {
        for (int d = max(0, i - C::STAGES); d < i; ++d) {
          mbar_wait(bar(C::B_KV_FULL + d % C::STAGES), static_cast<uint32_t>(d / C::STAGES) & 1u, DEFAULT_TIMEOUT,
                    nullptr);
        }
        if (q_loads > 0) {
          for (int t = 0; t < 2; ++t) {
            mbar_wait(bar(C::B_Q + t), static_cast<uint32_t>(q_loads - 1) & 1u, DEFAULT_TIMEOUT, nullptr);
          }
        }
      }
    }
  } else if (warp == MMA_WARP) {
    reg_dealloc<regs_other<D>()>();
    // -------------------------------------------------------------- MMA issuer (even CTA)
    if (lane == 0 && lead) {
      constexpr uint32_t idesc_qk = idesc_f16(BF16, 2 * BM, BN, false);
      constexpr uint32_t idesc_pv = idesc_f16(BF16, 2 * BM, D, true);
      const uint64_t dq_base = sdesc_sw128(sbase + C::OFF_Q, 16, 1024);
      const uint64_t dk_base = sdesc_sw128(sbase + C::OFF_KV, 16, 1024);
      const uint64_t dv_base = sdesc_sw128(sbase + C::OFF_KV, C::SLOT_BYTES, 1024);
      auto issue_qk = [&](int t, int st) {
        const uint64_t qd = dq_base + static_cast<uint64_t>((t * C::TILE_BYTES) >> 4);
        const uint64_t kd = dk_base + static_cast<uint64_t>((st * C::SLOT_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t qo = static_cast<uint64_t>(((kk >> 2) * C::Q_CHUNK + (kk & 3) * 32) >> 4);
          const uint64_t ko = static_cast<uint64_t>(((kk >> 2) * C::K_CHUNK + (kk & 3) * 32) >> 4);
          mma_ss_pair(tmem + t * BN, qd + qo, kd + ko, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int st, bool acc, int kk0, int kk1) {
        const uint64_t vd = dv_base + static_cast<uint64_t>((st * C::SLOT_BYTES) >> 4);
#pragma unroll
        for (int kk = kk0; kk < kk1; ++kk) {
          const int k0 = kk * 16;  // first key (V row) of this k-step
          mma_ts_pair(tmem + C::TMEM_O + t * D, tmem + t * BN + P_OFF + kk * 8,
                      vd + static_cast<uint64_t>((k0 * 128) >> 4), idesc_pv, (acc || k0 > 0) ? 1u : 0u);
        }
      };
      auto mwait = [&](int b_idx, uint32_t parity) -> bool {
        return mbar_wait(bar(b_idx), parity, a.timeout, a.err);
      };
      auto pv_tile = [&](int t, int st, bool acc, uint32_t pph) -> bool {
        if (!mwait(C::B_P_FULL + t, pph)) return false;
        tc_fence_after();
        issue_pv(t, st, acc, 0, 2 * P_SPLIT_W);
        if (!mwait(C::B_P_LATE + t, pph)) return false;
        tc_fence_after();
        issue_pv(t, st, acc, 2 * P_SPLIT_W, BN / 16);
        return true;
      };
      auto kv_wait = [&](int i) -> bool {
        return mwait(C::B_KV_FULL + i % C::STAGES, static_cast<uint32_t>(i / C::STAGES) & 1u);
      };
      Unit u;
      get_pair_unit<CAUSAL>(a, 0, u);
      do {
        if (!mwait(C::B_Q + 0, 0) || !kv_wait(0)) { ok = false; break; }
        tc_fence_after();
        issue_qk(0, 0);
        mma_commit_pair(bar(C::B_S_FULL + 0));
        if (u.J0 == 1) mma_commit_pair(bar(C::B_Q_EMPTY + 0));
        if (!mwait(C::B_Q + 1, 0)) { ok = false; break; }
        tc_fence_after();
        issue_qk(1, 0);
        mma_commit_pair(bar(C::B_S_FULL + 1));
        mma_commit_pair(bar(C::B_KV_EMPTY + 0));
        if (u.J == 1) mma_commit_pair(bar(C::B_Q_EMPTY + 1));
        // Pair-tile 0 (the unit's first 256 rows) runs J0 <= J steps: under a causal mask its
        // tiles past J0 are fully masked, so their GEMMs are skipped, and its phase counts (g0)
        // advance by J0 per unit; pair-tile 1 runs all J (g1). The next unit's first QK of both
        // tiles is issued in this unit's last step, after its K_0 (the next ring entry).
        int n = 0, i = 0, g0 = 0, g1 = 0;
        while (true) {
          Unit nx;
          const bool has_next = get_pair_unit<CAUSAL>(a, n + 1, nx);
          const uint32_t qph_next = static_cast<uint32_t>(n + 1) & 1u;
          for (int j = 0; j < u.J; ++j) {
            const bool last = (j + 1 == u.J);
            const int iv = i + 2 * j + 1, ik = i + 2 * j + 2;
            const int sv = iv % C::STAGES, sk = ik % C::STAGES;
            const bool more = !last || has_next;
            if (!kv_wait(iv)) { ok = false; break; }
            if (j < u.J0) {
              if (!pv_tile(0, sv, j > 0, static_cast<uint32_t>(g0 + j) & 1u)) { ok = false; break; }
              if (j + 1 == u.J0) mma_commit_pair(bar(C::B_O_FULL + 0));
            }
            if (j + 1 < u.J0 || (last && has_next)) {
              // QK(0, j + 1) of this unit, or the next unit's QK(0, 0).
              const bool qk_final0 = last ? (nx.J0 == 1) : (j + 2 == u.J0);
              if ((last && !mwait(C::B_Q + 0, qph_next)) || !kv_wait(ik)) { ok = false; break; }
              tc_fence_after();
              issue_qk(0, sk);
              mma_commit_pair(bar(C::B_S_FULL + 0));
              if (qk_final0) mma_commit_pair(bar(C::B_Q_EMPTY + 0));
            }
            if (!pv_tile(1, sv, j > 0, static_cast<uint32_t>(g1 + j) & 1u)) { ok = false; break; }
            mma_commit_pair(bar(C::B_KV_EMPTY + sv));
            if (last) mma_commit_pair(bar(C::B_O_FULL + 1));
            if (more) {
              const bool qk_final1 = last ? (nx.J == 1) : (j + 2 == u.J);
              if ((last && !mwait(C::B_Q + 1, qph_next)) || !kv_wait(ik)) { ok = false; break; }
              tc_fence_after();
              issue_qk(1, sk);
              mma_commit_pair(bar(C::B_S_FULL + 1));
              mma_commit_pair(bar(C::B_KV_EMPTY + sk));
              if (qk_final1) mma_commit_pair(bar(C::B_Q_EMPTY + 1));
            }
          }
          if (!ok || !has_next) break;
          i += 2 * u.J;
          g0 += u.J0;
          g1 += u.J;
          ++n;
          u = nx;
        }
      } while (false);
      // Both CTAs' MMA_DONE: every issued MMA retired (the odd CTA frees its TMEM after it).
      mma_commit_pair(bar(C::B_MMA_DONE));
      mbar_wait(bar(C::B_MMA_DONE), 0, DEFAULT_TIMEOUT, nullptr);
    }
  } else if (warp < SOFTMAX_WARPS) {
    reg_alloc<regs_softmax<D>()>();
    // ------------------------------------------------------------------ softmax
    const int q = warp & 3;
    const int t = warp >> 2;
    const int r = q * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t tS = tmem + lane_addr + t * BN;
    const uint32_t tP = tS + P_OFF;
    const uint32_t tO = tmem + lane_addr + C::TMEM_O + t * D;
    const float qk_scale = a.qk_scale;
    const uint64_t sc2 = f2_pack(qk_scale, qk_scale);
    const uint32_t so = sbase + C::OFF_STG + warp * C::STG_WARP_BYTES;  // O staging
    const uint32_t p_full = lbar(C::B_P_FULL + t), p_late = lbar(C::B_P_LATE + t);
    // One arrival per warp on the even CTA's barrier, after every lane's P stores completed.
    auto p_arrive = [&](uint32_t cbar) {
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cbar);
    };
    int g = 0;  // steps of the units before
    auto epilogue = [&](const Unit& eu, int en, float el) -> bool {
      const int e_row0 = eu.row0 + t * 256 + static_cast<int>(rank) * BM;
      {
        bool w = mbar_wait(bar(C::B_O_FULL + t), static_cast<uint32_t>(en) & 1u, a.timeout, a.err);
        if (!__all_sync(0xffffffffu, w)) return false;
      }
      tc_fence_after();
      uint32_t o[D / 32][32];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld32(tO + c * 32, o[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) reg_fence32(o[c]);
      const float inv_l = el > 0.0f ? 1.0f / el : 0.0f;
      const uint64_t inv2 = f2_pack(inv_l, inv_l);
      const int R0 = e_row0 + q * 32;
      const int pos0 = R0 >> a.pack_shift;
      const int h0 = eu.hq0 + (R0 & (a.pack - 1));
      if (lane == 0) bulk_wait_read();  // the slot's previous stores have read it
      __syncwarp();
#pragma unroll
      for (int ch = 0; ch < D / 64; ++ch) {
        const uint32_t slot = so + ch * C::STG_SLOT_BYTES;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const uint32_t* src = o[2 * ch + (v >> 2)];
          uint32_t w4[4];
#pragma unroll
          for (int i2 = 0; i2 < 4; ++i2) {
            const int e = (v & 3) * 8 + 2 * i2;
            float x0, x1;
            f2_unpack(f2_mul(f2_pack(__uint_as_float(src[e]), __uint_as_float(src[e + 1])), inv2), x0, x1);
            w4[i2] = cvt_pack2<BF16>(x0, x1);
          }
          st_shared_v4(slot + lane * 128 + ((static_cast<uint32_t>(v) ^ static_cast<uint32_t>(lane & 7)) << 4), w4[0],
                       w4[1], w4[2], w4[3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && pos0 < eu.n_q) {
#pragma unroll
        for (int ch = 0; ch < D / 64; ++ch) {
          tma_store_4d(&tmO, so + ch * C::STG_SLOT_BYTES, ch * 64, h0, eu.q0 + pos0, eu.tb);
        }
        bulk_commit();
      }
      return true;
    };

    Unit u;
    bool have = get_pair_unit<CAUSAL>(a, 0, u);
    for (int n = 0; ok && have; ++n) {
      const int J = (t == 0) ? u.J0 : u.J;  // pair-tile 0 stops after its causal band
      const int tile_row0 = u.row0 + t * 256 + static_cast<int>(rank) * BM;
      const int pos = (tile_row0 + r) >> a.pack_shift;
      const int tile_pos0 = tile_row0 >> a.pack_shift;
      float m_use = -INFINITY;
      float l = 0.0f;
      for (int j = 0; j < J; ++j) {
        bool w = mbar_wait(bar(C::B_S_FULL + t), static_cast<uint32_t>(g + j) & 1u, a.timeout, a.err);
        if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
        tc_fence_after();
        const int col0 = (u.j0 + j) * BN;
        const bool need_causal = CAUSAL && (col0 + BN - 1 > tile_pos0 + u.coff);
        const bool need_pad = (col0 + BN > u.n_kv);
        const bool masked = need_causal || need_pad;
        int lim = u.n_kv - 1 - col0;
        if (CAUSAL) lim = min(lim, pos + u.coff - col0);
        uint32_t s[NCH][32];
#pragma unroll
        for (int c = 0; c < NCH; ++c) tmem_ld32(tS + c * 32, s[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < NCH; ++c) reg_fence32(s[c]);
        if (masked) {
#pragma unroll
          for (int c = 0; c < NCH; ++c) mask_chunk(s[c], c * 32, lim);
        }
        const float m_cand = row_max_chunks(s) * qk_scale;
        const bool bump = m_cand > m_use + RESCALE_TH;
        float alpha = 1.0f;
        if (bump) {
          alpha = ex2_mufu(m_use - m_cand);
          m_use = m_cand;
        }
        if (j > 0 && __any_sync(0xffffffffu, bump)) {
          // PV(t, j-1) has retired: S_t(j) was committed after it.
          rescale_o_cols<D>(tO, alpha);
        }
        const float m_safe = (m_use == -INFINITY) ? 0.0f : m_use;
        const uint64_t nm2 = f2_pack(-m_safe, -m_safe);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          uint32_t pk[16];
          if (masked) {
            make_p32<BF16, 0u>(s[c], sc2, nm2, pk);
          } else {
            make_p32<BF16, emu_pair_mask<D, BF16>()>(s[c], sc2, nm2, pk);
          }
          tmem_st16(tP + c * 16, pk);
          if (c == P_SPLIT_W - 1) p_arrive(p_full);
        }
        p_arrive(p_late);
        uint64_t acc2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
#pragma unroll
          for (int i2 = 0; i2 < 32; i2 += 2) {
            acc2[(i2 >> 1) & 3] =
                f2_add(acc2[(i2 >> 1) & 3], f2_pack(__uint_as_float(s[c][i2]), __uint_as_float(s[c][i2 + 1])));
          }
        }
        const uint64_t acc01 = f2_add(f2_add(acc2[0], acc2[1]), f2_add(acc2[2], acc2[3]));
        float sl0, sl1;
        f2_unpack(acc01, sl0, sl1);
        l = l * alpha + (sl0 + sl1);
      }
      if (!ok) break;
      g += J;
      Unit nu;
      have = get_pair_unit<CAUSAL>(a, n + 1, nu);
      if (!epilogue(u, n, l)) { ok = false; break; }
      u = nu;
    }
    if (lane == 0) bulk_wait_all();
  } else {
    reg_dealloc<regs_other<D>()>();
  }

  if (!ok && a.err != nullptr) atomicCAS(a.err, 0, FA2_ERR_TIMEOUT);

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    // The odd CTA frees its TMEM once the even CTA's last commit says every MMA retired.
    if (!lead && lane == 0) mbar_wait(bar(C::B_MMA_DONE), 0, DEFAULT_TIMEOUT, nullptr);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
  cluster_sync();
}

}  // namespace fa2
