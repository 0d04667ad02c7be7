// Persistent variant of the grouped GEMM for prefill (two 128-row weight tiles per CTA,
// FUS_EPI_BF16 / FUS_EPI_SWIGLU, no split-K, no fused merge). Included by gemm.cu.
//
// One CTA per SM walks the same unit list as the one-tile-per-CTA kernel (stride
// gridDim.x). Warp 0 is the TMA producer (weight tiles; token tiles as one box sized to
// the unit's live rows, or gathered four rows per gather4 by all 32 lanes), warp 1
// issues the MMAs, and two groups of four warps drain the accumulators. The producer's
// ring runs continuously across units, so the next unit's tiles stream in while the
// epilogue drains; with block_n <= 128 the two accumulator sets are double-buffered in
// TMEM and the next unit's MMAs run during the drain too (at 256 they fill TMEM and wait).
// Epilogue: TMEM -> registers (SwiGLU / row scale / residual in fp32) -> a 16 KB staging
// buffer per group -> TMA tile stores from alternating 8 KB halves for dense outputs, or
// 16-byte stores through the row map for scattered ones.
#pragma once

// warp 0 TMA, warp 1 MMA, then two epilogue groups of four warps
constexpr int kPEpiGroups = 2;
constexpr int kPThreads = 64 + kPEpiGroups * 128;

template <int BN>
struct PersistCfg {
  static constexpr int A_BYTES = 2 * kATileBytes;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGING_BYTES = 16 * 1024;  // per epilogue group
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  // two accumulator sets (double buffering) when they fit in the 512 TMEM columns
  static constexpr int NBUF = 4 * BN <= 512 ? 2 : 1;
  static constexpr int ACC_COLS = 2 * BN;
  static constexpr int TMEM_COLS = pow2_at_least(NBUF * ACC_COLS < 32 ? 32 : NBUF * ACC_COLS, 32);
  static constexpr int SMEM_BYTES = RING_BYTES + kPEpiGroups * STAGING_BYTES + 256 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static_assert(STAGES >= 2, "pipeline too shallow");
};

struct Unit {
  int gi, mt, blk, expert;
};

// Decodes unit u (same order as the one-tile-per-CTA kernel); false when the unit has
// no live rows.
__device__ __forceinline__ bool decode_unit(const GemmArgs& a, int u, int BN, Unit& out,
                                            bool report) {
  int gi = 0;
  if (u >= a.units0) {
    gi = 1;
    u -= a.units0;
  }
  const GroupDev& G = a.g[gi];
  const int gsz_full = a.group_blocks * a.m_tiles;
  const int grp = u / gsz_full;
  const int rem = u - grp * gsz_full;
  const int gsz = min(a.group_blocks, G.max_blocks - grp * a.group_blocks);
  out.gi = gi;
  out.mt = rem / gsz;
  out.blk = grp * a.group_blocks + rem % gsz;
  const int rows_used = G.ntp ? __ldg(G.ntp) : G.x_rows;
  if (out.blk * BN >= rows_used) return false;
  out.expert = G.expert_ids ? __ldg(G.expert_ids + out.blk) : 0;
  if (out.expert < 0 || out.expert >= G.n_experts) {
    if (report) raise_status(a.status, FUS_ERR_BAD_EXPERT);
    return false;
  }
  return true;
}

// live token columns of a block (warp-wide; every lane gets the count)
__device__ __forceinline__ int live_columns(const GroupDev& G, int pos0, int BN, int lane) {
  int cnt = 0;
  if (G.live_ids) {
    for (int j = lane; j < BN; j += 32) cnt += __ldg(G.live_ids + pos0 + j) < G.live_limit;
  } else if (lane == 0) {
    cnt = min(BN, G.x_rows - pos0);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  return cnt;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kPThreads, 1)
    grouped_gemm_persistent(const __grid_constant__ CUtensorMap ta0,
                            const __grid_constant__ CUtensorMap ta1,
                            const __grid_constant__ CUtensorMap tb0,
                            const __grid_constant__ CUtensorMap tb1,
                            const __grid_constant__ CUtensorMap tbs0,  // token box 32 rows
                            const __grid_constant__ CUtensorMap tbs1,
                            const __grid_constant__ CUtensorMap tbm0,  // token box 128 rows
                            const __grid_constant__ CUtensorMap tbm1,
                            const __grid_constant__ CUtensorMap to0,
                            const __grid_constant__ CUtensorMap to1,
                            const __grid_constant__ GemmArgs args) {
  using Cfg = PersistCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sA = smem_u32(smem);
  const uint32_t sB = sA + STAGES * Cfg::A_BYTES;
  uint8_t* staging_all = smem + Cfg::RING_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging_all + kPEpiGroups * Cfg::STAGING_BYTES);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = smem_u32(bars + STAGES);
  const uint32_t bar_acc_full = smem_u32(bars + 2 * STAGES);       // [NBUF]
  const uint32_t bar_acc_empty = smem_u32(bars + 2 * STAGES + 2);  // [NBUF]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* ep_ok = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [kPEpiGroups]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long total = (long)args.units0 + (long)args.g[1].max_blocks * args.m_tiles;
  const int nk = args.ksteps_total;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < Cfg::NBUF; ++b) {
      mbar_init(bar_acc_full + 8 * b, 1);
      mbar_init(bar_acc_empty + 8 * b, kPEpiGroups);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&ta0);
    tma_prefetch_desc(&tb0);
    tma_prefetch_desc(&ta1);
    tma_prefetch_desc(&tb1);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: one continuous ring over all units ----------------
    // The token box is sized to the block's live rows (32 / 128 / BN): a block that holds
    // the few tokens an expert has beyond a full block moves 4 KB of tokens per stage,
    // not 32 KB of mostly dispatch pads.
    const uint64_t pol_x = policy_evict_last();
    uint32_t c = 0;
    bool stop = false;
    for (long uu = blockIdx.x; uu < total && !stop; uu += gridDim.x) {
      Unit un;
      if (!decode_unit(args, (int)uu, BN, un, lane == 0)) continue;
      const GroupDev& G = args.g[un.gi];
      const int pos0 = un.blk * BN;
      const int n_live = live_columns(G, pos0, BN, lane);
      const CUtensorMap* tma_a = un.gi ? &ta1 : &ta0;
      constexpr int kMid = BN < 128 ? BN : 128;  // the tbm maps' box rows
      const int bx = n_live <= 32 ? 32 : (n_live <= kMid ? kMid : BN);
      const bool gather = G.gather_ids != nullptr;
      const CUtensorMap* tma_b = gather || bx == BN ? (un.gi ? &tb1 : &tb0)
                                 : bx == 32         ? (un.gi ? &tbs1 : &tbs0)
                                                    : (un.gi ? &tbm1 : &tbm0);
      const uint32_t stage_bytes = Cfg::A_BYTES + (uint32_t)bx * kBK * 2;
      const uint64_t pol_w = (G.flags & FUS_GEMM_W_STREAM) ? policy_evict_first()
                                                           : policy_evict_normal();
      const int ebase = un.expert * args.w_rows;
      int a_row0, a_row1;
      if (EPI == FUS_EPI_SWIGLU) {
        a_row0 = ebase + un.mt * 128;
        a_row1 = ebase + (args.w_rows >> 1) + un.mt * 128;
      } else {
        a_row0 = ebase + un.mt * 256;
        a_row1 = a_row0 + 128;
      }
      // gathered token rows (rows of x picked by dispatch position, one TMA gather4 per
      // 4 rows, issued by all lanes): lane l owns 4-row groups l and l + 32 of the box
      int grow[2][4];
#pragma unroll
      for (int gq = 0; gq < 2; ++gq)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int j = (lane + 32 * gq) * 4 + q;
          int row = G.x_rows;  // past the end: zero fill
          if (gather && j < bx) {
            const int id = __ldg(G.gather_ids + pos0 + j);
            if (id < G.live_limit) row = id / G.gather_div;
          }
          grow[gq][q] = row;
        }
      for (int i = 0; i < nk; ++i, ++c) {
        const int s = c % STAGES;
        const uint32_t r = c / STAGES;
        const uint32_t full = bar_full + 8 * s;
        const int kk = i * kBK;
        if (lane == 0) {
          if (!mbar_wait_bounded(bar_empty + 8 * s, (r & 1u) ^ 1u, abort_flag, args.status)) {
            stop = true;
          } else {
            mbar_arrive_expect_tx(full, stage_bytes);
            const uint32_t a_dst = sA + s * Cfg::A_BYTES;
            tma_load_2d(a_dst, tma_a, full, kk, a_row0, pol_w);
            tma_load_2d(a_dst + kATileBytes, tma_a, full, kk, a_row1, pol_w);
            if (!gather) tma_load_2d(sB + s * Cfg::B_BYTES, tma_b, full, kk % args.K, pos0, pol_x);
          }
        }
        if (gather) {
          // the slot is free (lane 0 waited) and its byte count is posted before any
          // gathered row can land
          stop = __shfl_sync(0xffffffffu, (int)stop, 0);
          if (stop) break;
#pragma unroll
          for (int gq = 0; gq < 2; ++gq) {
            const int grp4 = lane + 32 * gq;
            if (grp4 * 4 < bx)
              tma_gather4(sB + s * Cfg::B_BYTES + grp4 * 4 * 128, tma_b, full, kk % args.K,
                          grow[gq][0], grow[gq][1], grow[gq][2], grow[gq][3], pol_x);
          }
        } else if (stop) {
          break;
        }
      }
      stop = __shfl_sync(0xffffffffu, (int)stop, 0);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    uint32_t c = 0, t = 0;
    bool stop = false;
    for (long uu = blockIdx.x; uu < total && !stop; uu += gridDim.x) {
      Unit un;
      if (!decode_unit(args, (int)uu, BN, un, false)) continue;
      const int n_live = live_columns(args.g[un.gi], un.blk * BN, BN, lane);
      const int n_mma = max(16, (n_live + 15) & ~15);
      const uint32_t buf = t % Cfg::NBUF, use = t / Cfg::NBUF;  // accumulator set, its use
      const uint32_t acc = tmem + buf * Cfg::ACC_COLS;
      if (lane == 0) {
        if (!mbar_wait_bounded(bar_acc_empty + 8 * buf, (use & 1u) ^ 1u, abort_flag,
                               args.status)) {
          stop = true;
        } else {
          tc_fence_after();
          const uint32_t idesc = idesc_bf16_f32(128, n_mma);
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
              tc_mma_bf16(acc, sw128_desc(a_base + 32 * k), bdesc, idesc, (i | k) != 0);
              tc_mma_bf16(acc + BN, sw128_desc(a_base + kATileBytes + 32 * k), bdesc, idesc,
                          (i | k) != 0);
            }
            tc_commit(bar_empty + 8 * s);
          }
          tc_commit(bar_acc_full + 8 * buf);
        }
      }
      stop = __shfl_sync(0xffffffffu, (int)stop, 0);
      ++t;
    }
  } else {
    // ---------------- epilogue (warps 2..9: two groups of four) ----------------
    // Each group of four warps covers the 128 TMEM lanes (warp % 4 = lane quadrant). With
    // two passes (bf16/fp32 output) group g drains pass g; with SwiGLU the groups take
    // alternate token chunks. Both arrive on acc_empty before the MMA warp reuses TMEM.
    const int q4 = warp & 3;
    const int m = q4 * 32 + lane;
    const int eg = (threadIdx.x - 64) >> 7;
    const int et = (threadIdx.x - 64) & 127;
    const int bar_id = 1 + eg;
    uint8_t* staging = staging_all + eg * Cfg::STAGING_BYTES;
    volatile int* my_ok = ep_ok + eg;
    // outputs are streamed: keep them from evicting the weight and token tiles that
    // neighbouring units re-read from L2
    const uint64_t pol_out = policy_evict_first();
    uint32_t t = 0, half = 0;
    for (long uu = blockIdx.x; uu < total; uu += gridDim.x) {
      Unit un;
      if (!decode_unit(args, (int)uu, BN, un, false)) continue;
      const GroupDev& G = args.g[un.gi];
      const int pos0 = un.blk * BN;
      const int n_live = live_columns(G, pos0, BN, lane);
      const int n_mma = max(16, (n_live + 15) & ~15);
      const uint32_t buf = t % Cfg::NBUF, use = t / Cfg::NBUF;
      const uint32_t lane_base =
          tmem + buf * Cfg::ACC_COLS + ((uint32_t)(q4 * 32) << 16);
      const bool exact = G.flags & FUS_GEMM_SWIGLU_EXACT;
      const bool out32 = (EPI == FUS_EPI_BF16) && (G.flags & FUS_GEMM_OUT_F32);
      // dense outputs (no row map / scale) leave through TMA tile stores from alternating
      // 8 KB halves of the group's staging buffer (one store drains while the next half
      // fills); scattered rows go through 16-byte stores from the whole 16 KB
      const bool tma_out = G.tma_store;
      const CUtensorMap* tmo = un.gi ? &to1 : &to0;
      const int CH = tma_out ? (out32 ? 16 : 32) : (out32 ? 32 : 64);  // tokens per round
      const int vec_per_row = out32 ? 32 : 16;  // 16-byte vectors per 128 features
      // each group drains one pass: with two passes (bf16/fp32 output) group g takes pass
      // g, with SwiGLU the groups take alternate token chunks
      constexpr int PASSES = (EPI == FUS_EPI_SWIGLU) ? 1 : 2;
      const int pass = PASSES == 2 ? eg : 0;
      const int c_first = PASSES == 2 ? 0 : eg * CH;
      const int c_step = PASSES == 2 ? CH : kPEpiGroups * CH;
      // destination rows of a chunk: store k of this thread is 16-byte vector et + 128 k
      // (CH * vec_per_row / 128 = 8 stores per thread and chunk); -1 = no store. The rows
      // of the first chunk are fetched before the accumulator wait and each next chunk's
      // during the current one, so the index loads never stall the drain.
      auto fetch_rows = [&](int c0, int* rr) {
        const int nrow = min(min(CH, n_mma - c0), n_live - c0);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int j = (et + 128 * k) / vec_per_row;
          int row = -1;
          if (j < nrow) {
            const int pos = pos0 + c0 + j;
            row = G.row_map ? __ldg(G.row_map + pos) : pos;
            if (row >= G.row_limit) row = -1;
          }
          rr[k] = row;
        }
      };
      int rr[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
      if (!tma_out) fetch_rows(c_first, rr);
      if (et == 0)
        *my_ok = mbar_wait_bounded(bar_acc_full + 8 * buf, use & 1u, abort_flag, args.status);
      named_bar_sync(bar_id, 128);
      if (!*my_ok) break;
      tc_fence_after();
      {
        const int col0 = (EPI == FUS_EPI_SWIGLU) ? un.mt * 128 : (un.mt * 2 + pass) * 128;
        for (int c0 = c_first; c0 < n_mma; c0 += c_step) {
          const int cw = min(CH, n_mma - c0);
          uint8_t* stg = tma_out ? staging + (half & 1u) * (Cfg::STAGING_BYTES / 2) : staging;
          int rn[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
          if (!tma_out && c0 + c_step < n_mma) fetch_rows(c0 + c_step, rn);
          // one staging column group: scale (w2 with row_scale), convert, write to smem
          auto stage16 = [&](int c, float* v) {
            if (EPI != FUS_EPI_SWIGLU && G.row_scale) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int pos = pos0 + c0 + c + j;
                const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
                const int si = (G.flags & FUS_GEMM_SCALE_TOKEN) ? row / G.token_div : row;
                v[j] *= row < G.row_limit ? __ldg(G.row_scale + si) : 0.f;
              }
            }
            if (EPI != FUS_EPI_SWIGLU && G.res) {  // residual of feature col0 + m
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int pos = pos0 + c0 + c + j;
                const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
                if (row < G.row_limit)
                  v[j] += __bfloat162float(G.res[(long)row * G.ldr + col0 + m]);
              }
            }
            if (out32) {
              float* st = reinterpret_cast<float*>(stg);
#pragma unroll
              for (int j = 0; j < 16; ++j) st[(c + j) * 128 + m] = v[j];
            } else {
              __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(stg);
#pragma unroll
              for (int j = 0; j < 16; ++j) st[(c + j) * 128 + m] = __float2bfloat16_rn(v[j]);
            }
          };
          auto swiglu16 = [&](const uint32_t* rg, const uint32_t* ru, float* v) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float g0 = __uint_as_float(rg[j]), u0 = __uint_as_float(ru[j]);
              const float g = exact ? g0 : round_bf(g0);
              const float up = exact ? u0 : round_bf(u0);
              v[j] = silu_mul(g, up);
            }
          };
          // TMEM reads in batches of 32 token columns, one wait per batch
          for (int c = 0; c < cw; c += 32) {
            const bool two = c + 16 < cw;  // warp-uniform
            uint32_t ra[16], rb[16], rc[16], rd[16];
            float v[16];
            if (EPI == FUS_EPI_SWIGLU) {
              tmem_ld16_issue(lane_base + (uint32_t)(c0 + c), ra);
              tmem_ld16_issue(lane_base + (uint32_t)(BN + c0 + c), rb);
              if (two) {
                tmem_ld16_issue(lane_base + (uint32_t)(c0 + c + 16), rc);
                tmem_ld16_issue(lane_base + (uint32_t)(BN + c0 + c + 16), rd);
              }
              tmem_ld_wait(ra);
              tmem_ld_wait(rb);
              if (two) {
                tmem_ld_wait(rc);
                tmem_ld_wait(rd);
              }
              swiglu16(ra, rb, v);
              stage16(c, v);
              if (two) {
                swiglu16(rc, rd, v);
                stage16(c + 16, v);
              }
            } else {
              tmem_ld16_issue(lane_base + (uint32_t)(pass * BN + c0 + c), ra);
              if (two) tmem_ld16_issue(lane_base + (uint32_t)(pass * BN + c0 + c + 16), rc);
              tmem_ld_wait(ra);
              if (two) tmem_ld_wait(rc);
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(ra[j]);
              stage16(c, v);
              if (two) {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(rc[j]);
                stage16(c + 16, v);
              }
            }
          }
          if (tma_out) {
            // the previous store (other half) must have read its source before anyone
            // passes this barrier into the next chunk, which refills that half. Rows past
            // the map's extent (row_limit) are clipped by the copy engine; rows past n_live
            // inside the block are dispatch pads (their contents are unused).
            fence_proxy_async_smem();
            if (et == 0) bulk_wait_read_all();
            named_bar_sync(bar_id, 128);
            if (et == 0) {
              tma_store_2d(tmo, smem_u32(stg), col0, pos0 + c0);
              bulk_commit();
            }
            ++half;
            continue;
          }
          named_bar_sync(bar_id, 128);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (rr[k] < 0) continue;
            const int it = et + 128 * k;
            const int j = it / vec_per_row, q = it % vec_per_row;
            if (out32) {
              const uint4 val = reinterpret_cast<const uint4*>(staging)[j * 32 + q];
              st_global_v4_hint(reinterpret_cast<float*>(G.out) + (long)rr[k] * G.ldo + col0 +
                                    q * 4, val, pol_out);
            } else {
              const uint4 val = reinterpret_cast<const uint4*>(staging)[j * 16 + q];
              st_global_v4_hint(reinterpret_cast<__nv_bfloat16*>(G.out) + (long)rr[k] * G.ldo +
                                    col0 + q * 8, val, pol_out);
            }
          }
          named_bar_sync(bar_id, 128);
#pragma unroll
          for (int k = 0; k < 8; ++k) rr[k] = rn[k];
        }
      }
      // accumulators read: hand TMEM back to the MMA warp for the next unit
      tc_fence_before();
      named_bar_sync(bar_id, 128);
      if (et == 0) mbar_arrive(bar_acc_empty + 8 * buf);
      ++t;
    }
    if (et == 0) bulk_wait_all();  // stores complete before the CTA's shared memory goes
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}
