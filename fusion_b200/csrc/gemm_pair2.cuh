// SM-pair prefill GEMM with expert-spanning tiles (tcgen05 cta_group::2). Included by
// gemm.cu after gemm_pair.cuh, whose cluster helpers it uses.
//
// A cluster of two CTAs computes M = 256 weight rows (128 per CTA, the accumulator lanes
// of each CTA's TMEM) against the tokens of one expert. TMEM holds two accumulator SLOTS
// of 256 columns; a token block of up to 256 rows occupies one slot. An expert whose
// tokens fill exactly two blocks (at T = 8192 over 256 experts about half of them: 257-311
// tokens, two balanced ~150-row blocks) is ONE tile of two parts: every weight stage is
// loaded once and feeds two MMAs (one per block, into the two slots), so the expert's
// weights cross HBM, L2 and shared memory once and each stage carries 2x the MMA work of
// a lone ~150-row block. Single-block tiles take one slot each and alternate, so the next
// tile's MMAs run while the epilogue drains the previous one.
//
//   BF16 (w2):    CTA r stages weight rows [128 r, 128 r + 128) of a 256-row tile.
//   SwiGLU (w13): CTA r stages 64 gate rows and the 64 matching up rows as one 128-row
//                 operand (gate in TMEM lanes 0-63, up in lanes 64-127): a tile is 128
//                 output features, and its gate and up values meet in the epilogue, where
//                 the warps of TMEM subpartitions 0-1 (gate) and 2-3 (up) exchange half of
//                 each 32-token chunk through shared memory and each computes 16 tokens.
//
// Token operand: CTA r stages rows [r N/2, (r+1) N/2) of each block (N = live rows rounded
// up to 16). A two-part tile uses two ring stages per K step: stage c holds the weight
// rows and block 0's token rows, stage c+1 block 1's token rows. Barriers, TMEM allocation
// and the exit protocol are those of grouped_gemm_pair (every wait bounded; both CTAs meet
// at a cluster barrier before the pair frees TMEM).
#pragma once

constexpr int kP2SlotCols = 256;  // accumulator columns per slot (two slots = 512)

// Optional phase counters (SM clock cycles per CTA), compiled only with FUS_PAIR2_TRACE:
// [0] MMA waiting for a free slot, [1] MMA waiting for staged operands, [2] MMA-warp
// span, [3] tiles, [4] epilogue waiting for a full slot, [5] epilogue draining, [6]
// producer waiting for a free stage, [7] parts.
#ifdef FUS_PAIR2_TRACE
__device__ unsigned long long g_pair2_trace[2][160][8];
__device__ int g_pair2_trace_sel;
#define P2T(...) __VA_ARGS__
#else
#define P2T(...)
#endif

template <int EPI>
struct Pair2Cfg {
  static constexpr int A_BYTES = kATileBytes;               // 128 weight rows per CTA
  static constexpr int B_BYTES = (kPairBN / 2) * kBK * 2;   // this CTA's half of a block
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGING_BYTES = 16 * 1024;  // per epilogue group
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * kP2SlotCols;
  static constexpr int SMEM_BYTES = RING_BYTES + kPEpiGroups * STAGING_BYTES + 256 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static_assert(STAGES >= 4, "a two-part tile takes two stages per K step");
};

// Blocks a unit's tile spans: 2 when `blk` starts an expert's run of exactly two blocks
// (the tile takes both), 0 when it is the second of such a run (its tile is the
// previous unit's), else 1. Blocks past the padded total never match.
__device__ __forceinline__ int pair2_span(const GroupDev& G, int blk) {
  if (!G.expert_ids || (G.flags & FUS_GEMM_PAIR_SPLIT)) return 1;
  const int used = (G.ntp ? __ldg(G.ntp) : G.x_rows) / kPairBN;
  auto eid = [&](int b) { return b >= 0 && b < used ? __ldg(G.expert_ids + b) : -1; };
  const int me = eid(blk);
  const bool prev = eid(blk - 1) == me, next = eid(blk + 1) == me;
  if (next && !prev && eid(blk + 2) != me) return 2;
  if (prev && !next && eid(blk - 2) != me) return 0;
  return 1;
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    grouped_gemm_pair2(const __grid_constant__ CUtensorMap ta0,
                       const __grid_constant__ CUtensorMap ta1,
                       const __grid_constant__ CUtensorMap tb0,   // token box 128 rows
                       const __grid_constant__ CUtensorMap tb1,
                       const __grid_constant__ CUtensorMap tbs0,  // token box 16 rows
                       const __grid_constant__ CUtensorMap tbs1,
                       const __grid_constant__ CUtensorMap tbm0,  // token box 64 rows
                       const __grid_constant__ CUtensorMap tbm1,
                       const __grid_constant__ CUtensorMap to0,
                       const __grid_constant__ CUtensorMap to1,
                       const __grid_constant__ GemmArgs args) {
  using Cfg = Pair2Cfg<EPI>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr bool kSwiglu = EPI == FUS_EPI_SWIGLU;
  extern __shared__ uint8_t smem_raw[];
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
  tc_fence_before();
  cluster_barrier();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    const uint64_t pol_x = policy_evict_last();
    uint32_t c = 0;
    bool stop = false;
    P2T(unsigned long long p_wait = 0; long long tp0 = 0;)
    for (long uu = first; uu < total && !stop; uu += stride) {
      Unit un;
      if (!decode_unit(args, (int)uu, kPairBN, un, leader && lane == 0)) continue;
      const GroupDev& G = args.g[un.gi];
      const int span = pair2_span(G, un.blk);
      if (span == 0) continue;
      const CUtensorMap* tma_a = un.gi ? &ta1 : &ta0;
      // token rows of part p: box, bytes and first row of this CTA's half
      auto part = [&](int p, const CUtensorMap*& tm, uint32_t& bytes, int& row) {
        const int pos0 = (un.blk + p) * kPairBN;
        const int n_live = live_columns(G, pos0, kPairBN, lane);
        const int half = max(16, (n_live + 15) & ~15) / 2;  // token rows per CTA
        const int bx = half <= 16 ? 16 : (half <= 64 ? 64 : 128);
        tm = bx == 128 ? (un.gi ? &tb1 : &tb0) : bx == 16 ? (un.gi ? &tbs1 : &tbs0)
                                                          : (un.gi ? &tbm1 : &tbm0);
        bytes = (uint32_t)bx * kBK * 2;
        row = pos0 + (int)rank * half;
      };
      const CUtensorMap *tb_0, *tb_1;
      uint32_t bb0, bb1 = 0;
      int br0, br1 = 0;
      part(0, tb_0, bb0, br0);
      tb_1 = tb_0;
      if (span == 2) part(1, tb_1, bb1, br1);
      const uint64_t pol_w = (G.flags & FUS_GEMM_W_STREAM) ? policy_evict_first()
                                                           : policy_evict_normal();
      const int ebase = un.expert * args.w_rows;
      // SwiGLU: 64 gate rows and the matching 64 up rows; BF16: 128 rows
      const int a_row0 = kSwiglu ? ebase + un.mt * 128 + 64 * (int)rank
                                 : ebase + un.mt * 256 + 128 * (int)rank;
      const int a_row1 = a_row0 + (args.w_rows >> 1);
      for (int i = 0; i < nk; ++i) {
        const int kk = i * kBK;
        // stage c: weight rows + block 0's tokens; two-block tiles: stage c+1 block 1's
        if (lane == 0) {
          const int s = c % STAGES;
          P2T(tp0 = clock64();)
          if (!mbar_wait_bounded(bar_empty + 8 * s, ((c / STAGES) & 1u) ^ 1u, abort_flag,
                                 args.status)) {
            stop = true;
          } else {
            P2T(p_wait += clock64() - tp0;)
            const uint32_t full_leader = cluster_map(bar_full + 8 * s, 0);
            if (leader) mbar_arrive_expect_tx(bar_full + 8 * s, 2u * (Cfg::A_BYTES + bb0));
            const uint32_t a_dst = sA + s * Cfg::A_BYTES;
            tma_load_2d_pair(a_dst, tma_a, full_leader, kk, a_row0, pol_w);
            if (kSwiglu)
              tma_load_2d_pair(a_dst + kATileBytes / 2, tma_a, full_leader, kk, a_row1, pol_w);
            tma_load_2d_pair(sB + s * Cfg::B_BYTES, tb_0, full_leader, kk % args.K, br0, pol_x);
          }
          if (span == 2 && !stop) {
            const int s1 = (c + 1) % STAGES;
            if (!mbar_wait_bounded(bar_empty + 8 * s1, (((c + 1) / STAGES) & 1u) ^ 1u,
                                   abort_flag, args.status)) {
              stop = true;
            } else {
              const uint32_t full_leader = cluster_map(bar_full + 8 * s1, 0);
              if (leader) mbar_arrive_expect_tx(bar_full + 8 * s1, 2u * bb1);
              tma_load_2d_pair(sB + s1 * Cfg::B_BYTES, tb_1, full_leader, kk % args.K, br1,
                               pol_x);
            }
          }
        }
        c += span;
        stop = __shfl_sync(0xffffffffu, (int)stop, 0);
        if (stop) break;
      }
    }
    P2T(if (lane == 0 && blockIdx.x < 160) g_pair2_trace[g_pair2_trace_sel][blockIdx.x][6] = p_wait;)
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader) {
      uint32_t c = 0, t = 0;
      bool stop = false;
      P2T(unsigned long long w_acc = 0, w_full = 0, n_tiles = 0; const long long t_beg = clock64();)
      for (long uu = first; uu < total && !stop; uu += stride) {
        Unit un;
        if (!decode_unit(args, (int)uu, kPairBN, un, false)) continue;
        const GroupDev& G = args.g[un.gi];
        const int span = pair2_span(G, un.blk);
        if (span == 0) continue;
        uint32_t idesc[2], acc[2];
        idesc[0] = idesc_bf16_f32(256, max(16, (live_columns(G, un.blk * kPairBN, kPairBN,
                                                               lane) + 15) & ~15));
        acc[0] = tmem + (t & 1u) * kP2SlotCols;
        idesc[1] = span == 2 ? idesc_bf16_f32(256, max(16, (live_columns(G, (un.blk + 1) *
                                                         kPairBN, kPairBN, lane) + 15) & ~15))
                             : idesc[0];
        acc[1] = tmem + ((t + 1) & 1u) * kP2SlotCols;
        if (lane == 0) {
          P2T(++n_tiles; long long tw = clock64();)
          for (int p = 0; p < span && !stop; ++p) {
            const uint32_t tp = t + p;
            if (!mbar_wait_bounded(bar_acc_empty + 8 * (tp & 1u), ((tp >> 1) & 1u) ^ 1u,
                                   abort_flag, args.status))
              stop = true;
          }
          P2T(w_acc += clock64() - tw;)
          tc_fence_after();
          if (span == 1 && !stop) {
            for (int i = 0; i < nk; ++i, ++c) {
              const int s = c % STAGES;
              P2T(tw = clock64();)
              if (!mbar_wait_bounded(bar_full + 8 * s, (c / STAGES) & 1u, abort_flag,
                                     args.status)) {
                stop = true;
                break;
              }
              P2T(w_full += clock64() - tw;)
              tc_fence_after();
              const uint32_t a_base = sA + s * Cfg::A_BYTES;
              const uint32_t b_base = sB + s * Cfg::B_BYTES;
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k)
                tc_mma_bf16_pair(acc[0], sw128_desc(a_base + 32 * k), sw128_desc(b_base + 32 * k),
                                 idesc[0], (i | k) != 0);
              tc_commit_pair(bar_empty + 8 * s);
            }
          }
          if (span == 2 && !stop) {
            // two blocks: stage c holds the weight rows and block 0's tokens, stage c+1
            // block 1's tokens; each weight sub-tile feeds both MMAs
            for (int i = 0; i < nk; ++i, c += 2) {
              const int s0 = c % STAGES, s1 = (c + 1) % STAGES;
              P2T(tw = clock64();)
              if (!mbar_wait_bounded(bar_full + 8 * s0, (c / STAGES) & 1u, abort_flag,
                                     args.status) ||
                  !mbar_wait_bounded(bar_full + 8 * s1, ((c + 1) / STAGES) & 1u, abort_flag,
                                     args.status)) {
                stop = true;
                break;
              }
              P2T(w_full += clock64() - tw;)
              tc_fence_after();
              const uint32_t a_base = sA + s0 * Cfg::A_BYTES;
              const uint32_t b0 = sB + s0 * Cfg::B_BYTES, b1 = sB + s1 * Cfg::B_BYTES;
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                const uint64_t adesc = sw128_desc(a_base + 32 * k);
                tc_mma_bf16_pair(acc[0], adesc, sw128_desc(b0 + 32 * k), idesc[0], (i | k) != 0);
                tc_mma_bf16_pair(acc[1], adesc, sw128_desc(b1 + 32 * k), idesc[1], (i | k) != 0);
              }
              tc_commit_pair(bar_empty + 8 * s0);
              tc_commit_pair(bar_empty + 8 * s1);
            }
          }
          if (!stop)
            for (int p = 0; p < span; ++p) tc_commit_pair(bar_acc_full + 8 * ((t + p) & 1u));
        }
        stop = __shfl_sync(0xffffffffu, (int)stop, 0);
        t += span;
      }
      P2T(if (lane == 0 && blockIdx.x < 160) {
        unsigned long long* o = g_pair2_trace[g_pair2_trace_sel][blockIdx.x];
        o[0] = w_acc; o[1] = w_full; o[2] = clock64() - t_beg; o[3] = n_tiles;
      })
    }
  } else {
    // ---------------- epilogue (warps 2..9 of both CTAs: two groups of four) ----------
    // Group g takes the 32-token chunks g, g + 2, ... of each part (16 for fp32 output).
    const int q4 = warp & 3;  // TMEM subpartition this warp may read (lanes 32 q4 ...)
    const int m = q4 * 32 + lane;
    const int eg = (threadIdx.x - 64) >> 7;
    const int et = (threadIdx.x - 64) & 127;
    const int bar_id = 1 + eg;
    uint8_t* staging = staging_all + eg * Cfg::STAGING_BYTES;
    volatile int* my_ok = ep_ok + eg;
    uint32_t t = 0, half_sel = 0;
    bool quit = false;
    P2T(unsigned long long e_wait = 0, e_drain = 0, n_parts = 0; long long te = 0;)
    for (long uu = first; uu < total && !quit; uu += stride) {
      Unit un;
      if (!decode_unit(args, (int)uu, kPairBN, un, false)) continue;
      const GroupDev& G = args.g[un.gi];
      const int span = pair2_span(G, un.blk);
      if (span == 0) continue;
      const bool exact = G.flags & FUS_GEMM_SWIGLU_EXACT;
      const bool out32 = !kSwiglu && (G.flags & FUS_GEMM_OUT_F32);
      const int CH = out32 ? 16 : 32;
      const CUtensorMap* tmo = un.gi ? &to1 : &to0;
      // this CTA's first output feature
      const int col0 = kSwiglu ? un.mt * 128 + 64 * (int)rank : un.mt * 256 + 128 * (int)rank;
      for (int p = 0; p < span; ++p, ++t) {
        const int pos0 = (un.blk + p) * kPairBN;
        const int n_live = live_columns(G, pos0, kPairBN, lane);
        const int n_mma = max(16, (n_live + 15) & ~15);
        const uint32_t slot = t & 1u, use = t >> 1;
        const uint32_t lane_base = tmem + slot * kP2SlotCols + ((uint32_t)(q4 * 32) << 16);
        P2T(te = clock64();)
        if (et == 0)
          *my_ok = mbar_wait_bounded(bar_acc_full + 8 * slot, use & 1u, abort_flag, args.status);
        named_bar_sync(bar_id, 128);
        if (!*my_ok) {
          quit = true;
          break;
        }
        P2T(e_wait += clock64() - te; te = clock64(); ++n_parts;)
        tc_fence_after();
        for (int c0 = eg * CH; c0 < n_mma; c0 += kPEpiGroups * CH) {
          const bool two = !out32 && c0 + 16 < n_mma;  // second 16 columns (warp-uniform)
          uint32_t ra[16], rc[16];
          tmem_ld16_issue(lane_base + (uint32_t)c0, ra);
          if (two) tmem_ld16_issue(lane_base + (uint32_t)(c0 + 16), rc);
          tmem_ld_wait(ra);
          if (two) tmem_ld_wait(rc);
          if (kSwiglu) {
            // staging: out[32 tokens][64 features] bf16 in alternating 4 KB halves, then
            // the exchange buffer xg[2 feature blocks][16][32] (gate) and xu (up), fp32
            uint8_t* stg = staging + (half_sel & 1u) * 4096;
            float* xg = reinterpret_cast<float*>(staging + 8192);
            float* xu = xg + 2 * 16 * 32;
            const int fb = q4 & 1;  // features [32 fb, 32 fb + 32) of this CTA's 64
            const bool gate = q4 < 2;
            if (gate) {
              if (two)
#pragma unroll
                for (int j = 0; j < 16; ++j) xg[(fb * 16 + j) * 32 + lane] = __uint_as_float(rc[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) xu[(fb * 16 + j) * 32 + lane] = __uint_as_float(ra[j]);
            }
            named_bar_sync(bar_id, 128);
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(stg);
            if (gate) {  // tokens c0 .. c0+15: own gate, up from the exchange
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float g0 = __uint_as_float(ra[j]), u0 = xu[(fb * 16 + j) * 32 + lane];
                o[j * 64 + fb * 32 + lane] = __float2bfloat16_rn(
                    silu_mul(exact ? g0 : round_bf(g0), exact ? u0 : round_bf(u0)));
              }
            } else if (two) {  // tokens c0+16 .. c0+31: gate from the exchange, own up
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float g0 = xg[(fb * 16 + j) * 32 + lane], u0 = __uint_as_float(rc[j]);
                o[(16 + j) * 64 + fb * 32 + lane] = __float2bfloat16_rn(
                    silu_mul(exact ? g0 : round_bf(g0), exact ? u0 : round_bf(u0)));
              }
            }
          } else {
            uint8_t* stg = staging + (half_sel & 1u) * (Cfg::STAGING_BYTES / 2);
            auto stage16 = [&](int cc, const uint32_t* rg) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float v = __uint_as_float(rg[j]);
                if (out32)
                  reinterpret_cast<float*>(stg)[(cc + j) * 128 + m] = v;
                else
                  reinterpret_cast<__nv_bfloat16*>(stg)[(cc + j) * 128 + m] =
                      __float2bfloat16_rn(v);
              }
            };
            stage16(0, ra);
            if (two) stage16(16, rc);
          }
          // the previous store (other half) has read its source before anyone passes this
          // barrier into the next chunk, which refills that half. Rows past n_live inside
          // the block are dispatch pads (their contents are unused); rows past the map's
          // extent are clipped by the copy engine.
          fence_proxy_async_smem();
          if (et == 0) bulk_wait_read_all();
          named_bar_sync(bar_id, 128);
          if (et == 0) {
            const uint32_t src = kSwiglu ? smem_u32(staging + (half_sel & 1u) * 4096)
                                         : smem_u32(staging + (half_sel & 1u) *
                                                                  (Cfg::STAGING_BYTES / 2));
            tma_store_2d(tmo, src, col0, pos0 + c0);
            bulk_commit();
          }
          ++half_sel;
        }
        // accumulators read: hand the slot back to the leader's MMA warp
        tc_fence_before();
        named_bar_sync(bar_id, 128);
        P2T(e_drain += clock64() - te;)
        if (et == 0) {
          if (leader)
            mbar_arrive(bar_acc_empty + 8 * slot);
          else
            mbar_arrive_remote(cluster_map(bar_acc_empty + 8 * slot, 0));
        }
      }
    }
    if (et == 0) bulk_wait_all();  // stores complete before the CTA's shared memory goes
    P2T(if (et == 0 && eg == 0 && blockIdx.x < 160) {
      unsigned long long* o = g_pair2_trace[g_pair2_trace_sel][blockIdx.x];
      o[4] = e_wait; o[5] = e_drain; o[7] = n_parts;
    })
  }

  tc_fence_before();
  cluster_barrier();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
}
