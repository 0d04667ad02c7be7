// SM-pair variant of the persistent prefill GEMM (tcgen05 cta_group::2). Included by
// gemm.cu after gemm_persist.cuh.
//
// A cluster of two CTAs on two SMs computes one tile of 256 weight rows x one 256-row token
// block with M = 256 MMAs issued by the leader CTA (rank 0): CTA r stages weight rows
// [128 r, 128 r + 128) of the tile and token rows [r N/2, (r+1) N/2) of the block, and holds
// the accumulator lanes of its own 128 weight rows for all N tokens. Each SM thus reads
// half of the token operand from its own shared memory per MMA instead of all of it; on
// expert blocks that are not exactly full (most of a prefill batch) the tensor pipe of a
// single-CTA tile is bound by those shared-memory reads.
//
//   SwiGLU (w13): tile = 256 features; per stage each CTA loads its 128 gate rows and its
//     128 up rows, two MMAs per 16-deep K step (gate -> columns [0, 256), up -> [256, 512)).
//   BF16 (w2):    tile = 256 output features; one MMA per K step into 256 columns, and the
//     two accumulator sets are double-buffered so the next tile's MMAs run under the drain.
//
// Token boxes per CTA are 16, 64, 96 or 128 rows (one TMA copy per stage, the smallest
// that holds the CTA's half of the live rows: a ~150-token block moves 96 rows, not 128).
//
// Synchronisation: both CTAs' TMA loads of a stage complete on the LEADER's full barrier
// (cp.async.bulk.tensor .cta_group::2, barrier addressed through the cluster window; no
// multicast), whose expected byte count the leader posts for both. The leader's
// tcgen05.commit (cta_group::2, multicast mask 0b11) frees the stage on both CTAs' empty
// barriers and signals both CTAs' accumulator-full barriers. Each CTA's two epilogue
// groups arrive on the leader's accumulator-empty barrier (count 4). TMEM is allocated and
// freed by warp 1 of both CTAs (cta_group::2); every wait is bounded, and every exit path
// reaches the same cluster barrier before the pair frees TMEM.
//
// Outputs are dense (rows in dispatch order; bf16, or fp32 for FUS_GEMM_OUT_F32) and leave
// through TMA tile stores, as in the single-CTA persistent kernel; the host selects this
// kernel only for such launches.
#pragma once

FUS_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
FUS_DEVICE uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
FUS_DEVICE uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
FUS_DEVICE uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
FUS_DEVICE void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
FUS_DEVICE void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
FUS_DEVICE void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
FUS_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
FUS_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
FUS_DEVICE void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` (same offset) in both CTAs of the pair once the leader's MMAs complete
FUS_DEVICE void tc_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on a barrier of
// either CTA of the pair (`bar` is a shared::cluster address)
FUS_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1,
                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

constexpr int kPairBN = 256;  // token rows per block (both CTAs)

// NA = 128-row weight tiles per CTA and stage, each with its own accumulator and all
// multiplied by the same token tile (SwiGLU: gate + up; BF16: 1, or 2 for 512-row tiles)
template <int EPI, int NA_ = (EPI == FUS_EPI_SWIGLU ? 2 : 1)>
struct PairCfg {
  static constexpr int NA = NA_;
  static constexpr int A_BYTES = NA * kATileBytes;
  static constexpr int B_BYTES = (kPairBN / 2) * kBK * 2;  // this CTA's half of the tokens
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGING_BYTES = 16 * 1024;  // per epilogue group
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int ACC_COLS = NA * kPairBN;
  static constexpr int NBUF = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_BYTES = RING_BYTES + kPEpiGroups * STAGING_BYTES + 256 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static_assert(STAGES >= 2, "pipeline too shallow");
  static_assert(NBUF * ACC_COLS <= TMEM_COLS, "tensor memory");
};

template <int EPI, int NA>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    grouped_gemm_pair(const __grid_constant__ CUtensorMap ta0,
                      const __grid_constant__ CUtensorMap ta1,
                      const __grid_constant__ CUtensorMap tb0,   // token box 128 rows
                      const __grid_constant__ CUtensorMap tb1,
                      const __grid_constant__ CUtensorMap tbs0,  // token box 16 rows
                      const __grid_constant__ CUtensorMap tbs1,
                      const __grid_constant__ CUtensorMap tbm0,  // token box 64 rows
                      const __grid_constant__ CUtensorMap tbm1,
                      const __grid_constant__ CUtensorMap tbw0,  // token box 96 rows
                      const __grid_constant__ CUtensorMap tbw1,
                      const __grid_constant__ CUtensorMap to0,
                      const __grid_constant__ CUtensorMap to1,
                      const __grid_constant__ GemmArgs args) {
  using Cfg = PairCfg<EPI, NA>;
  constexpr int STAGES = Cfg::STAGES;
  static_assert(EPI != FUS_EPI_SWIGLU || NA == 2, "SwiGLU pairs gate and up tiles");
  extern __shared__ uint8_t smem_raw[];
  // the same offsets in both CTAs: the dynamic window starts at the same address in each
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sA = smem_u32(smem);
  const uint32_t sB = sA + STAGES * Cfg::A_BYTES;
  uint8_t* staging_all = smem + Cfg::RING_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging_all + kPEpiGroups * Cfg::STAGING_BYTES);
  const uint32_t bar_full = smem_u32(bars);                        // [STAGES], leader's used
  const uint32_t bar_empty = smem_u32(bars + STAGES);              // [STAGES]
  const uint32_t bar_acc_full = smem_u32(bars + 2 * STAGES);       // [2]
  const uint32_t bar_acc_empty = smem_u32(bars + 2 * STAGES + 2);  // [2], leader's used
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* ep_ok = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [kPEpiGroups]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const long first = cluster_id_x(), stride = cluster_count_x();
  const long total = (long)args.units0 + (long)args.g[1].max_blocks * args.m_tiles;
  const int nk = args.ksteps_total;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full + 8 * b, 1);
      mbar_init(bar_acc_empty + 8 * b, 2 * kPEpiGroups);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&ta0);
    tma_prefetch_desc(&tb0);
    tma_prefetch_desc(&ta1);
    tma_prefetch_desc(&tb1);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // barriers initialised and TMEM allocated in both CTAs before either touches the other
  tc_fence_before();
  cluster_barrier();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    const uint64_t pol_x = policy_evict_last();
    uint32_t c = 0;
    bool stop = false;
    for (long uu = first; uu < total && !stop; uu += stride) {
      Unit un;
      if (!decode_unit(args, (int)uu, kPairBN, un, leader && lane == 0)) continue;
      const GroupDev& G = args.g[un.gi];
      const int pos0 = un.blk * kPairBN;
      const int n_live = live_columns(G, pos0, kPairBN, lane);
      const int half = max(16, (n_live + 15) & ~15) / 2;  // token rows per CTA (multiple of 8)
      // one box per stage, the smallest of 16 / 64 / 96 / 128 rows that holds the half
      const int bx = half <= 16 ? 16 : half <= 64 ? 64 : half <= 96 ? 96 : 128;
      const CUtensorMap* tma_a = un.gi ? &ta1 : &ta0;
      const CUtensorMap* tma_b = bx == 128 ? (un.gi ? &tb1 : &tb0)
                                 : bx == 16 ? (un.gi ? &tbs1 : &tbs0)
                                 : bx == 96 ? (un.gi ? &tbw1 : &tbw0)
                                            : (un.gi ? &tbm1 : &tbm0);
      // both CTAs' bytes land on the leader's barrier
      const uint32_t stage_tx = 2u * (uint32_t)(Cfg::A_BYTES + bx * kBK * 2);
      const uint64_t pol_w = (G.flags & FUS_GEMM_W_STREAM) ? policy_evict_first()
                                                           : policy_evict_normal();
      const int ebase = un.expert * args.w_rows;
      // SwiGLU: gate rows of a 256-feature tile, then the matching up rows; BF16 with two
      // tiles: 256 consecutive rows of a 512-row tile per CTA
      const int a_row0 = EPI == FUS_EPI_SWIGLU || NA == 1
                             ? ebase + un.mt * 256 + 128 * (int)rank
                             : ebase + un.mt * 512 + 256 * (int)rank;
      const int a_row1 = EPI == FUS_EPI_SWIGLU ? a_row0 + (args.w_rows >> 1) : a_row0 + 128;
      const int b_row = pos0 + (int)rank * half;
      for (int i = 0; i < nk; ++i, ++c) {
        const int s = c % STAGES;
        const uint32_t r = c / STAGES;
        if (lane == 0) {
          if (!mbar_wait_bounded(bar_empty + 8 * s, (r & 1u) ^ 1u, abort_flag, args.status)) {
            stop = true;
          } else {
            const uint32_t full_leader = cluster_map(bar_full + 8 * s, 0);
            if (leader) mbar_arrive_expect_tx(bar_full + 8 * s, stage_tx);
            const int kk = i * kBK;
            const uint32_t a_dst = sA + s * Cfg::A_BYTES;
            tma_load_2d_pair(a_dst, tma_a, full_leader, kk, a_row0, pol_w);
            if (NA == 2)
              tma_load_2d_pair(a_dst + kATileBytes, tma_a, full_leader, kk, a_row1, pol_w);
            tma_load_2d_pair(sB + s * Cfg::B_BYTES, tma_b, full_leader, kk % args.K, b_row,
                             pol_x);
          }
        }
        stop = __shfl_sync(0xffffffffu, (int)stop, 0);
        if (stop) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader) {
      uint32_t c = 0, t = 0;
      bool stop = false;
      for (long uu = first; uu < total && !stop; uu += stride) {
        Unit un;
        if (!decode_unit(args, (int)uu, kPairBN, un, false)) continue;
        const int n_live = live_columns(args.g[un.gi], un.blk * kPairBN, kPairBN, lane);
        const int n_mma = max(16, (n_live + 15) & ~15);
        const uint32_t buf = t % Cfg::NBUF, use = t / Cfg::NBUF;
        const uint32_t acc = tmem + buf * Cfg::ACC_COLS;
        if (lane == 0) {
          if (!mbar_wait_bounded(bar_acc_empty + 8 * buf, (use & 1u) ^ 1u, abort_flag,
                                 args.status)) {
            stop = true;
          } else {
            tc_fence_after();
            const uint32_t idesc = idesc_bf16_f32(256, n_mma);
            for (int i = 0; i < nk; ++i, ++c) {
              const int s = c % STAGES;
              const uint32_t r = c / STAGES;
              if (!mbar_wait_bounded(bar_full + 8 * s, r & 1u, abort_flag, args.status)) {
                stop = true;
                break;
              }
              tc_fence_after();
              const uint32_t a_base = sA + s * Cfg::A_BYTES;
              const uint32_t b_base = sB + s * Cfg::B_BYTES;
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                const uint64_t bdesc = sw128_desc(b_base + 32 * k);
                tc_mma_bf16_pair(acc, sw128_desc(a_base + 32 * k), bdesc, idesc, (i | k) != 0);
                if (NA == 2)
                  tc_mma_bf16_pair(acc + kPairBN, sw128_desc(a_base + kATileBytes + 32 * k),
                                   bdesc, idesc, (i | k) != 0);
              }
              tc_commit_pair(bar_empty + 8 * s);
            }
            if (!stop) tc_commit_pair(bar_acc_full + 8 * buf);
          }
        }
        stop = __shfl_sync(0xffffffffu, (int)stop, 0);
        ++t;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9 of both CTAs: two groups of four) ----------
    // Group g takes token chunks g, g + 2, ... of 32 columns (16 for fp32 output); each
    // chunk goes through TMEM -> registers -> an 8 KB half of the group's staging buffer
    // -> one TMA store of 128 features x 32 (16) token rows.
    const int q4 = warp & 3;
    const int m = q4 * 32 + lane;
    const int eg = (threadIdx.x - 64) >> 7;
    const int et = (threadIdx.x - 64) & 127;
    const int bar_id = 1 + eg;
    uint8_t* staging = staging_all + eg * Cfg::STAGING_BYTES;
    volatile int* my_ok = ep_ok + eg;
    uint32_t t = 0, half_sel = 0;
    for (long uu = first; uu < total; uu += stride) {
      Unit un;
      if (!decode_unit(args, (int)uu, kPairBN, un, false)) continue;
      const GroupDev& G = args.g[un.gi];
      const int pos0 = un.blk * kPairBN;
      const int n_live = live_columns(G, pos0, kPairBN, lane);
      const int n_mma = max(16, (n_live + 15) & ~15);
      const uint32_t buf = t % Cfg::NBUF, use = t / Cfg::NBUF;
      const uint32_t lane_base = tmem + buf * Cfg::ACC_COLS + ((uint32_t)(q4 * 32) << 16);
      const bool exact = G.flags & FUS_GEMM_SWIGLU_EXACT;
      const bool out32 = EPI == FUS_EPI_BF16 && (G.flags & FUS_GEMM_OUT_F32);
      const int CH = out32 ? 16 : 32;
      const CUtensorMap* tmo = un.gi ? &to1 : &to0;
      constexpr bool kTwoOut = EPI == FUS_EPI_BF16 && NA == 2;  // two 128-feature outputs
      // this CTA's first output feature
      const int col0 = kTwoOut ? un.mt * 512 + 256 * (int)rank : un.mt * 256 + 128 * (int)rank;
      if (et == 0)
        *my_ok = mbar_wait_bounded(bar_acc_full + 8 * buf, use & 1u, abort_flag, args.status);
      named_bar_sync(bar_id, 128);
      if (!*my_ok) break;
      tc_fence_after();
      for (int c0 = eg * CH; c0 < n_mma; c0 += kPEpiGroups * CH) {
        const bool two = !out32 && c0 + 16 < n_mma;  // second 16 columns (warp-uniform)
        uint8_t* stg = staging + (half_sel & 1u) * (Cfg::STAGING_BYTES / 2);
        if (kTwoOut) {
          // this chunk fills both halves: every earlier store has read its source first
          stg = staging;
          if (et == 0) bulk_wait_read_all();
          named_bar_sync(bar_id, 128);
        }
        uint32_t ra[16], rb[16], rc[16], rd[16];
        tmem_ld16_issue(lane_base + (uint32_t)c0, ra);
        if (two) tmem_ld16_issue(lane_base + (uint32_t)(c0 + 16), rc);
        if (NA == 2) {
          tmem_ld16_issue(lane_base + (uint32_t)(kPairBN + c0), rb);
          if (two) tmem_ld16_issue(lane_base + (uint32_t)(kPairBN + c0 + 16), rd);
        }
        tmem_ld_wait(ra);
        if (two) tmem_ld_wait(rc);
        if (NA == 2) {
          tmem_ld_wait(rb);
          if (two) tmem_ld_wait(rd);
        }
        auto stage16 = [&](int c, const uint32_t* rg, const uint32_t* ru) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v;
            if (EPI == FUS_EPI_SWIGLU) {
              const float g0 = __uint_as_float(rg[j]), u0 = __uint_as_float(ru[j]);
              v = silu_mul(exact ? g0 : round_bf(g0), exact ? u0 : round_bf(u0));
            } else {
              v = __uint_as_float(rg[j]);
            }
            if (out32)
              reinterpret_cast<float*>(stg)[(c + j) * 128 + m] = v;
            else
              reinterpret_cast<__nv_bfloat16*>(stg)[(c + j) * 128 + m] = __float2bfloat16_rn(v);
          }
        };
        stage16(0, ra, rb);
        if (two) stage16(16, rc, rd);
        if (kTwoOut) {  // the second weight tile's features into the other half
          uint8_t* keep = stg;
          stg = staging + Cfg::STAGING_BYTES / 2;
          stage16(0, rb, rb);
          if (two) stage16(16, rd, rd);
          stg = keep;
        }
        // the previous store (other half) must have read its source before anyone passes
        // this barrier into the next chunk, which refills that half. Rows past the map's
        // extent are clipped by the copy engine; rows past n_live inside the block are
        // dispatch pads (their contents are unused).
        fence_proxy_async_smem();
        if (et == 0) bulk_wait_read_all();
        named_bar_sync(bar_id, 128);
        if (et == 0) {
          tma_store_2d(tmo, smem_u32(stg), col0, pos0 + c0);
          if (kTwoOut)
            tma_store_2d(tmo, smem_u32(staging + Cfg::STAGING_BYTES / 2), col0 + 128, pos0 + c0);
          bulk_commit();
        }
        ++half_sel;
      }
      // accumulators read: hand them back to the leader's MMA warp
      tc_fence_before();
      named_bar_sync(bar_id, 128);
      if (et == 0) {
        if (leader)
          mbar_arrive(bar_acc_empty + 8 * buf);
        else
          mbar_arrive_remote(cluster_map(bar_acc_empty + 8 * buf, 0));
      }
      ++t;
    }
    if (et == 0) bulk_wait_all();  // stores complete before the CTA's shared memory goes
  }

  // neither CTA leaves (or frees the pair's TMEM) while the other may still signal its
  // barriers or read its shared memory
  tc_fence_before();
  cluster_barrier();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
}
