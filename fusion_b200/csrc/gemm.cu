// Grouped expert GEMM on Blackwell tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the Triton grouped GEMMs of the reference:
//   glm52/kernels/moe_gateup.py:34-148  (w13, optional SwiGLU epilogue, FUSE_ACT)
//   glm52/kernels/moe_down_merge.py:66-169 (w2, routed-weight epilogue)
//   glm52/kernels/norm_router.py:87-212 as router_gemm (fp32 logits)
//
// B200 design (not a port): the expert WEIGHT is the MMA's M operand (128 rows per
// tile) and the tokens of one dispatch block are its N operand (block_n = 16..256),
// so a decode block with one token per expert still runs full-width 128xN MMAs
// while streaming the weight through a deep TMA ring; prefill blocks use N up to 256.
// One CTA = one (token block, 128-row weight tile, K split):
//   warp 0  : TMA producer (one elected lane) filling a STAGES-deep smem ring
//   warp 1  : TMEM allocator + MMA issuer (one lane), tcgen05.commit frees stages
//   warps 2-5: epilogue; TMEM -> registers -> smem (token-major) -> 16-byte stores
// Work order puts the weight tiles of one token block next to each other, so a block's
// token rows stay in L2 while the weights stream from HBM exactly once per block.
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace fus {

struct GroupDev {
  const int* expert_ids;
  const int* ntp;
  int x_rows;
  int max_blocks;
  int n_experts;
  int row_limit;
  void* out;
  long ldo;
  const int* row_map;
  const float* row_scale;
  int flags;
  const int* live_ids;
  int live_limit;
  int token_div;
  const int* gather_ids;
  int gather_div;
  int tma_store;  // persistent kernel: dense output written by TMA tile stores
  const __nv_bfloat16* res;  // optional residual (FUS_EPI_BF16), row stride ldr
  long ldr;
};

struct MergeDev {
  int* counters;  // null: no fused merge
  int parts;
  const __nv_bfloat16* y;
  long ld_t, ld_k;
  int topk;
  const float* w;
  long ldw;
  const __nv_bfloat16* res;
  long ldr;
  const float* extra;
  long lde;
  __nv_bfloat16* out;
  long ldo;
};

struct GemmArgs {
  GroupDev g[2];
  int units0;            // CTAs of group 0
  int w_rows;            // weight rows per expert
  int K;                 // token K extent (elements)
  int ksteps_total;      // weight K extent / 64
  int ksteps_per_split;
  int ksplit;
  int m_tiles;           // weight tiles per expert
  int group_blocks;      // token blocks swept together across all weight tiles
  long split_stride;     // FUS_EPI_F32 partial plane stride (elements)
  int* status;
  MergeDev mg;
  int pdl;  // 0 none; 1 wait before any read; 2 prefetch weights, then wait
};

constexpr int kBK = 64;                  // K elements per stage (128 B rows, one swizzle span)
constexpr int kATileBytes = 128 * kBK * 2;  // one 128-row weight tile per stage
constexpr int kThreads = 192;

__host__ __device__ constexpr int pow2_at_least(int v, int p) { return p >= v ? p : pow2_at_least(v, 2 * p); }

// MT = weight tiles (128 rows each) per CTA, all multiplied by the same token tile; each
// has its own TMEM accumulator. MT=2 halves the token-operand bytes per flop, so the same
// shared-memory ring covers twice the MMA time (prefill); MT=1 gives more CTAs (decode).
template <int BN, int MT>
struct GemmCfg {
  static constexpr int A_BYTES = MT * kATileBytes;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // decode tiles (block_n <= 32): ~72 KB so that three CTAs share an SM (a w2 launch of
  // 9 experts x 48 tiles then runs in one wave: 432 CTAs, 444 slots); block_n 64:
  // ~110 KB, two per SM; otherwise ~200 KB. Bytes in flight per SM stay ~200 KB.
  static constexpr int RING_TARGET = (MT == 1 && BN <= 32)   ? 72 * 1024
                                     : (MT == 1 && BN <= 64) ? 112 * 1024
                                                             : 200 * 1024;
  static constexpr int STAGES = RING_TARGET / STAGE_BYTES > 8 ? 8 : RING_TARGET / STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TMEM_COLS = pow2_at_least(MT * BN < 32 ? 32 : MT * BN, 32);
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = RING_BYTES + BAR_BYTES + 1024;  // + alignment slack
  static_assert(RING_BYTES >= BN * 128 * 4 + BN * 4 + 16, "epilogue staging must fit in the ring");
  static_assert(STAGES >= 2, "pipeline too shallow");
  static_assert(TMEM_COLS <= 512, "TMEM holds 512 columns");
};

// Fused expert merge, run by the 128 epilogue threads after this CTA stored its rows.
// Per (token, weight tile) a counter collects the contributions (topk routed rows + the
// shared row); the CTA that lands the last one sums them in a fixed order, adds the
// residual, writes the block output for the tile's features and re-arms the counter.
template <int BN, int MT>
__device__ __noinline__ void fused_merge_tail(const GemmArgs& args, const GroupDev& G,
                                              uint8_t* scratch, int pos0, int n_live, int mt,
                                              int et) {
  const MergeDev& M = args.mg;
  int* list_n = reinterpret_cast<int*>(scratch);
  int* list = list_n + 4;
  __threadfence();  // release: this thread's row stores before its counter update
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (et == 0) *list_n = 0;
  asm volatile("bar.sync 1, 128;" ::: "memory");
  for (int j = et; j < n_live; j += 128) {
    const int pos = pos0 + j;
    const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
    if (row >= G.row_limit) continue;
    const int t = row / G.token_div;
    const int old = atomicAdd(M.counters + (long)t * args.m_tiles + mt, 1);
    if (old == M.parts - 1) list[atomicAdd(list_n, 1)] = t;
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  __threadfence();  // acquire: the other contributions are visible now
  const int n = *list_n;
  constexpr int NF = 128 * MT;  // features of this tile
  constexpr int NV = NF / 8;
  const int f0 = mt * NF;
  for (int it = et; it < n * NV; it += 128) {
    const int t = list[it / NV];
    const int f = f0 + (it % NV) * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int k = 0; k < M.topk; ++k) {
      const float wk = __ldg(M.w + (long)t * M.ldw + k);
      float yv[8];
      unpack8(__ldcg(reinterpret_cast<const uint4*>(M.y + (long)t * M.ld_t + (long)k * M.ld_k + f)),
              yv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += wk * yv[e];
    }
    if (M.res) {
      float r[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(M.res + (long)t * M.ldr + f)), r);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += r[e];
    }
    if (M.extra) {
      const float4* ep = reinterpret_cast<const float4*>(M.extra + (long)t * M.lde + f);
      const float4 a = __ldcg(ep), b = __ldcg(ep + 1);
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    *reinterpret_cast<uint4*>(M.out + (long)t * M.ldo + f) = pack8(acc);
  }
  for (int i = et; i < n; i += 128) M.counters[(long)list[i] * args.m_tiles + mt] = 0;
}

template <int BN, int EPI, int MT>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap ta0,
                        const __grid_constant__ CUtensorMap ta1,
                        const __grid_constant__ CUtensorMap tb0,
                        const __grid_constant__ CUtensorMap tb1,
                        const __grid_constant__ GemmArgs args) {
  using Cfg = GemmCfg<BN, MT>;
  constexpr int STAGES = Cfg::STAGES;

  // ---- which unit of work is this CTA ------------------------------------------------
  int u = blockIdx.x;
  int gi = 0;
  if (u >= args.units0) {
    gi = 1;
    u -= args.units0;
  }
  const GroupDev& G = args.g[gi];
  const int split = u % args.ksplit;
  u /= args.ksplit;
  // `group_blocks` consecutive token blocks visit every weight tile before the next
  // group starts: a group's token rows stay in L2 and same-expert blocks (adjacent in
  // the dispatch layout) read each weight tile back to back.
  const int gsz_full = args.group_blocks * args.m_tiles;
  const int grp = u / gsz_full;
  const int rem = u - grp * gsz_full;
  const int gsz = min(args.group_blocks, G.max_blocks - grp * args.group_blocks);
  const int mt = rem / gsz;
  const int blk = grp * args.group_blocks + rem % gsz;
  if (args.pdl == 1) pdl_wait();  // the dispatch layout comes from the predecessor
  pdl_allow_dependents();
  const int rows_used = G.ntp ? __ldg(G.ntp) : G.x_rows;
  if (blk * BN >= rows_used) return;  // uniform across the CTA: nothing allocated yet
  const int expert = G.expert_ids ? __ldg(G.expert_ids + blk) : 0;
  if (expert < 0 || expert >= G.n_experts) {
    if (threadIdx.x == 0) raise_status(args.status, FUS_ERR_BAD_EXPERT);
    return;
  }
  const int kbeg = split * args.ksteps_per_split;
  const int kend = min(args.ksteps_total, kbeg + args.ksteps_per_split);
  const int nk = kend - kbeg;
  if (nk <= 0) return;

  const CUtensorMap* tma_a = gi ? &ta1 : &ta0;
  const CUtensorMap* tma_b = gi ? &tb1 : &tb0;

  // ---- shared memory ------------------------------------------------------------------
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sA = smem_u32(smem);
  const uint32_t sB = sA + STAGES * Cfg::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::RING_BYTES);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = smem_u32(bars + STAGES);
  const uint32_t bar_accum = smem_u32(bars + 2 * STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* n_live_slot = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pos0 = blk * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(tma_a);
    tma_prefetch_desc(tma_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
    // live token columns of this block: dispatch pads sit at the end of a block
    int cnt = 0;
    if (G.live_ids) {
      for (int j = lane; j < BN; j += 32) cnt += __ldg(G.live_ids + pos0 + j) < G.live_limit;
    } else if (lane == 0) {
      cnt = min(BN, G.x_rows - pos0);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) *n_live_slot = cnt;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_live = *n_live_slot;
  // MMA width: live columns rounded up to the instruction's N granule (16 for M=128)
  const int n_mma = max(16, (n_live + 15) & ~15);

  if (warp == 0) {
    // ---------------- TMA producer (lane 0; all lanes issue row gathers) ----------------
    // weights: evict-first when no other token block reads the tile, else normal
    const uint64_t pol_w = (G.flags & FUS_GEMM_W_STREAM) ? policy_evict_first()
                                                         : policy_evict_normal();
    const uint64_t pol_x = policy_evict_last();  // token rows: re-read by every tile
    // weight rows of the two A sub-tiles (SwiGLU: gate rows, then the matching up rows)
    const int ebase = expert * args.w_rows;
    int a_row0, a_row1;
    if (EPI == FUS_EPI_SWIGLU) {
      const int half = 64 * MT;  // features per tile
      a_row0 = ebase + mt * half;
      a_row1 = ebase + (args.w_rows >> 1) + mt * half;
    } else {
      a_row0 = ebase + mt * 128 * MT;
      a_row1 = a_row0 + 128;
    }
    constexpr uint32_t a_half_bytes = (EPI == FUS_EPI_SWIGLU && MT == 1) ? kATileBytes / 2
                                                                        : kATileBytes;
    const bool two_a = (EPI == FUS_EPI_SWIGLU) || MT == 2;
    // gathered token rows: lane l owns 4-row groups l and l+32 (BN <= 256)
    const bool gather = G.gather_ids != nullptr;
    int grow[2][4];
#pragma unroll
    for (int gq = 0; gq < 2; ++gq)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = (lane + 32 * gq) * 4 + q;
        int row = G.x_rows;  // past the end: zero fill
        if (gather && j < BN) {
          const int id = __ldg(G.gather_ids + pos0 + j);
          if (id < G.live_limit) row = id / G.gather_div;
        }
        grow[gq][q] = row;
      }
    // weight tiles of stage s, k-step i (lane 0; also posts the stage's byte count)
    auto load_a = [&](int s, int i) {
      const uint32_t full = bar_full + 8 * s;
      const int kk = (kbeg + i) * kBK;
      mbar_arrive_expect_tx(full, Cfg::STAGE_BYTES);
      const uint32_t a_dst = sA + s * Cfg::A_BYTES;
      tma_load_2d(a_dst, tma_a, full, kk, a_row0, pol_w);
      if (two_a) tma_load_2d(a_dst + a_half_bytes, tma_a, full, kk, a_row1, pol_w);
    };
    // token rows of stage s, k-step i (whole warp)
    auto load_b = [&](int s, int i) {
      const uint32_t full = bar_full + 8 * s;
      const int kk = (kbeg + i) * kBK;
      if (gather) {
#pragma unroll
        for (int gq = 0; gq < 2; ++gq) {
          const int grp4 = lane + 32 * gq;
          if (grp4 * 4 < BN)
            tma_gather4(sB + s * Cfg::B_BYTES + grp4 * 4 * 128, tma_b, full, kk % args.K,
                        grow[gq][0], grow[gq][1], grow[gq][2], grow[gq][3], pol_x);
        }
      } else if (lane == 0) {
        tma_load_2d(sB + s * Cfg::B_BYTES, tma_b, full, kk % args.K, pos0, pol_x);
      }
    };
    // pdl == 2: the weight tiles of the first ring are requested while the predecessor
    // (which produces the token rows) is still running; token rows follow its completion
    int i0 = 0;
    if (args.pdl == 2) {
      i0 = min(nk, STAGES);
      if (lane == 0) {
        for (int i = 0; i < i0; ++i) load_a(i, i);
        pdl_wait();
      }
      __syncwarp();
      for (int i = 0; i < i0; ++i) load_b(i, i);
    }
    for (int i = i0; i < nk; ++i) {
      const int s = i % STAGES;
      const uint32_t r = (uint32_t)(i / STAGES);
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait_bounded(bar_empty + 8 * s, (r & 1u) ^ 1u, abort_flag, args.status);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (lane == 0) load_a(s, i);
      load_b(s, i);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_bf16_f32(128, n_mma);
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t r = (uint32_t)(i / STAGES);
        if (!mbar_wait_bounded(bar_full + 8 * s, r & 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t a_base = sA + s * Cfg::A_BYTES;
        const uint32_t b_base = sB + s * Cfg::B_BYTES;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          // advance 16 bf16 (32 B) along K inside the 128-byte swizzle span
          const uint64_t bdesc = sw128_desc(b_base + 32 * k);
#pragma unroll
          for (int t = 0; t < MT; ++t)
            tc_mma_bf16(tmem + t * BN, sw128_desc(a_base + t * kATileBytes + 32 * k), bdesc,
                        idesc, (i | k) != 0);
        }
        tc_commit(bar_empty + 8 * s);
      }
      tc_commit(bar_accum);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q4 = warp & 3;  // TMEM lane quarter this warp may access
    const bool ok = mbar_wait_bounded(bar_accum, 0, abort_flag, args.status) && !*abort_flag;
    tc_fence_after();
    const int et = threadIdx.x - 64;  // 0..127
    if (ok) {
      float* S = reinterpret_cast<float*>(smem);  // [BN][128] fp32, token-major
      const int m = q4 * 32 + lane;
      const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
      const bool exact = G.flags & FUS_GEMM_SWIGLU_EXACT;
      // passes: SwiGLU with MT=2 pairs both accumulators in one pass; otherwise one pass
      // per accumulator (128 output features each)
      constexpr int PASSES = (EPI == FUS_EPI_SWIGLU) ? 1 : MT;
#pragma unroll 1
      for (int pass = 0; pass < PASSES; ++pass) {
#pragma unroll 1
        for (int c = 0; c < n_mma; c += 16) {
          float v[16];
          if (EPI == FUS_EPI_SWIGLU && MT == 2) {
            float w[16];
            tmem_ld16(lane_base + (uint32_t)c, v);         // gate feature m
            tmem_ld16(lane_base + (uint32_t)(BN + c), w);  // up feature m
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float g = exact ? v[j] : round_bf(v[j]);
              const float up = exact ? w[j] : round_bf(w[j]);
              v[j] = silu_mul(g, up);
            }
          } else {
            tmem_ld16(lane_base + (uint32_t)(pass * BN + c), v);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) S[(c + j) * 128 + m] = v[j];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");

        if (EPI == FUS_EPI_SWIGLU && MT == 1) {
          // rows 0-63 of the tile are gate features, 64-127 the matching up features
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(G.out);
          for (int it = et; it < n_live * 8; it += 128) {
            const int j = it >> 3, q = it & 7;
            const int pos = pos0 + j;
            const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
            if (row >= G.row_limit) continue;
            const float4* gp = reinterpret_cast<const float4*>(S + j * 128 + q * 8);
            const float4* up = reinterpret_cast<const float4*>(S + j * 128 + 64 + q * 8);
            float g[8], uu[8], o[8];
            *reinterpret_cast<float4*>(g) = gp[0];
            *reinterpret_cast<float4*>(g + 4) = gp[1];
            *reinterpret_cast<float4*>(uu) = up[0];
            *reinterpret_cast<float4*>(uu + 4) = up[1];
            if (!exact) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                g[e] = round_bf(g[e]);
                uu[e] = round_bf(uu[e]);
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = silu_mul(g[e], uu[e]);
            *reinterpret_cast<uint4*>(out + (long)row * G.ldo + mt * 64 + q * 8) = pack8(o);
          }
        } else {
          // 128 finished features per token row: SwiGLU (MT=2) output, or one accumulator
          const int col0 = (EPI == FUS_EPI_SWIGLU) ? mt * 128 : (mt * MT + pass) * 128;
          for (int it = et; it < n_live * 16; it += 128) {
            const int j = it >> 4, q = it & 15;
            const int pos = pos0 + j;
            const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
            if (row >= G.row_limit) continue;
            const float4* sp = reinterpret_cast<const float4*>(S + j * 128 + q * 8);
            float vv[8];
            *reinterpret_cast<float4*>(vv) = sp[0];
            *reinterpret_cast<float4*>(vv + 4) = sp[1];
            if (EPI == FUS_EPI_F32) {
              float* dp = reinterpret_cast<float*>(G.out) + (long)split * args.split_stride +
                          (long)row * G.ldo + col0 + q * 8;
              reinterpret_cast<float4*>(dp)[0] = sp[0];
              reinterpret_cast<float4*>(dp)[1] = sp[1];
              continue;
            }
            if (EPI == FUS_EPI_BF16) {
              const float sc =
                  G.row_scale
                      ? __ldg(G.row_scale + ((G.flags & FUS_GEMM_SCALE_TOKEN) ? row / G.token_div
                                                                              : row))
                      : 1.0f;
#pragma unroll
              for (int e = 0; e < 8; ++e) vv[e] *= sc;
              if (G.res) {
                float rr[8];
                unpack8(__ldg(reinterpret_cast<const uint4*>(G.res + (long)row * G.ldr + col0 +
                                                             q * 8)), rr);
#pragma unroll
                for (int e = 0; e < 8; ++e) vv[e] += rr[e];
              }
              if (G.flags & FUS_GEMM_OUT_F32) {
                float4* dp = reinterpret_cast<float4*>(reinterpret_cast<float*>(G.out) +
                                                       (long)row * G.ldo + col0 + q * 8);
                dp[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
                dp[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
                continue;
              }
            }
            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(G.out) +
                                      (long)row * G.ldo + col0 + q * 8) = pack8(vv);
          }
        }
        if (pass + 1 < PASSES) asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      if (EPI == FUS_EPI_BF16 && (G.flags & FUS_GEMM_MERGE) && args.mg.counters)
        fused_merge_tail<BN, MT>(args, G, smem + Cfg::RING_BYTES - BN * 4 - 16, pos0, n_live, mt,
                                 et);
    }
  }

  // ---- teardown: every tcgen05 op of this CTA is complete or abandoned -------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

#include "gemm_persist.cuh"
#include "gemm_pair.cuh"

// ======================================================================================
// host side
// ======================================================================================
namespace {

template <int BN, int EPI>
int launch_p(const CUtensorMap* maps, const GemmArgs& a, int grid, cudaStream_t st) {
  using Cfg = PersistCfg<BN>;
  if (int rc = ensure_smem_attr((const void*)grouped_gemm_persistent<BN, EPI>, Cfg::SMEM_BYTES,
                                 "grouped_gemm_persistent"))
    return rc;
  grouped_gemm_persistent<BN, EPI><<<grid, kPThreads, Cfg::SMEM_BYTES, st>>>(
      maps[0], maps[1], maps[2], maps[3], maps[6], maps[7], maps[8], maps[9], maps[4], maps[5], a);
  return check_launch("grouped_gemm_persistent");
}

template <int EPI>
int launch_persist(int bn, const CUtensorMap* maps, const GemmArgs& a, int grid,
                   cudaStream_t st) {
  switch (bn) {
    case 64: return launch_p<64, EPI>(maps, a, grid, st);
    case 128: return launch_p<128, EPI>(maps, a, grid, st);
    case 256: return launch_p<256, EPI>(maps, a, grid, st);
  }
  return set_error(FUS_E_UNSUPPORTED, "persistent GEMM: block_n %d", bn);
}

template <int EPI, int NA>
int launch_pair(const CUtensorMap* maps, const GemmArgs& a, long total, cudaStream_t st) {
  using Cfg = PairCfg<EPI, NA>;
  if (int rc = ensure_smem_attr((const void*)grouped_gemm_pair<EPI, NA>, Cfg::SMEM_BYTES,
                                 "grouped_gemm_pair"))
    return rc;
  // co-resident cluster count (same on every B200; computed on the first device used)
  static std::once_flag once;
  static int max_clusters = 0;
  std::call_once(once, [] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    if (cudaOccupancyMaxActiveClusters(&max_clusters, grouped_gemm_pair<EPI, NA>, &cfg) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      max_clusters = 0;
    }
  });
  // one resident cluster per SM pair; clusters beyond the co-resident count would only
  // queue behind the first wave
  long clusters = max_clusters > 0 ? max_clusters : num_sms() / 2;
  if (clusters > total) clusters = total;
  grouped_gemm_pair<EPI, NA><<<(int)(2 * clusters), kPThreads, Cfg::SMEM_BYTES, st>>>(
      maps[0], maps[1], maps[2], maps[3], maps[6], maps[7], maps[8], maps[9], maps[10], maps[11],
      maps[4], maps[5], a);
  return check_launch("grouped_gemm_pair");
}

template <int BN, int EPI, int MT>
int launch_t(const CUtensorMap* maps, const GemmArgs& a, int grid, cudaStream_t st) {
  using Cfg = GemmCfg<BN, MT>;
  if (int rc = ensure_smem_attr((const void*)grouped_gemm_kernel<BN, EPI, MT>, Cfg::SMEM_BYTES,
                                 "grouped_gemm"))
    return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, grouped_gemm_kernel<BN, EPI, MT>, maps[0], maps[1],
                                     maps[2], maps[3], a);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "grouped_gemm: %s", cudaGetErrorString(e));
  return check_launch("grouped_gemm");
}

template <int EPI>
int launch_bn(int bn, int mt2, const CUtensorMap* maps, const GemmArgs& a, int grid,
              cudaStream_t st) {
  if (mt2) {
    switch (bn) {
      case 64: return launch_t<64, EPI, 2>(maps, a, grid, st);
      case 128: return launch_t<128, EPI, 2>(maps, a, grid, st);
      case 256: return launch_t<256, EPI, 2>(maps, a, grid, st);
    }
  } else {
    switch (bn) {
      case 16: return launch_t<16, EPI, 1>(maps, a, grid, st);
      case 32: return launch_t<32, EPI, 1>(maps, a, grid, st);
      case 64: return launch_t<64, EPI, 1>(maps, a, grid, st);
      case 128: return launch_t<128, EPI, 1>(maps, a, grid, st);
      case 256: return launch_t<256, EPI, 1>(maps, a, grid, st);
    }
  }
  return set_error(FUS_E_UNSUPPORTED, "block_n %d not in {16,32,64,128,256}", bn);
}

}  // namespace
}  // namespace fus

using namespace fus;

static int mt2_for(int w_rows, int epilogue, int block_n) {
  // two weight tiles per CTA for wide token tiles (prefill); the router (fp32 partials,
  // split-K) keeps one for parallelism
  return block_n >= 64 && epilogue != FUS_EPI_F32 && w_rows % 256 == 0;
}

static int grouped_gemm_impl(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                             int a_kplanes, int epilogue, int block_n, int ksplit,
                             long split_stride, int group_blocks, const fus_merge_spec* merge,
                             void* stream, int* status, int pdl = 0);

namespace fus {
int grouped_gemm_launch(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                        int a_kplanes, int epilogue, int block_n, int ksplit, long split_stride,
                        int group_blocks, const fus_merge_spec* merge, int pdl, void* stream,
                        int* status) {
  return grouped_gemm_impl(groups, ngroups, w_rows, K, a_kplanes, epilogue, block_n, ksplit,
                           split_stride, group_blocks, merge, stream, status, pdl);
}
}  // namespace fus

extern "C" int fus_grouped_gemm(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                                int a_kplanes, int epilogue, int block_n, int ksplit,
                                long split_stride, void* stream, int* status) {
  return grouped_gemm_impl(groups, ngroups, w_rows, K, a_kplanes, epilogue, block_n, ksplit,
                           split_stride, 0, nullptr, stream, status);
}

extern "C" int fus_grouped_gemm_ex(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                                   int a_kplanes, int epilogue, int block_n, int ksplit,
                                   long split_stride, int group_blocks, void* stream,
                                   int* status) {
  return grouped_gemm_impl(groups, ngroups, w_rows, K, a_kplanes, epilogue, block_n, ksplit,
                           split_stride, group_blocks, nullptr, stream, status);
}

extern "C" int fus_grouped_gemm_tiles(int w_rows, int epilogue, int block_n) {
  if (w_rows <= 0 || w_rows % 128) return 0;
  const int MTv = mt2_for(w_rows, epilogue, block_n) ? 2 : 1;
  return epilogue == FUS_EPI_SWIGLU ? w_rows / 2 / (64 * MTv) : w_rows / (128 * MTv);
}

extern "C" int fus_grouped_gemm_merge(const fus_gemm_group* groups, int ngroups, int w_rows,
                                      int K, int block_n, const fus_merge_spec* merge,
                                      void* stream, int* status) {
  if (!merge || !merge->counters || !merge->y || !merge->w || !merge->out || merge->parts < 1 ||
      merge->topk < 1)
    return set_error(FUS_E_INVALID, "grouped_gemm_merge: incomplete merge spec");
  if (!aligned16(merge->y) || !aligned16(merge->out) || (merge->res && !aligned16(merge->res)) ||
      (merge->extra && !aligned16(merge->extra)) || merge->ld_t % 8 || merge->ld_k % 8 ||
      merge->ldo % 8 || merge->ldr % 8 || merge->lde % 4)
    return set_error(FUS_E_INVALID, "grouped_gemm_merge: rows must be 16-byte aligned");
  for (int g = 0; g < ngroups; ++g)
    if ((groups[g].flags & FUS_GEMM_MERGE) && groups[g].token_div < 1)
      return set_error(FUS_E_INVALID, "grouped_gemm_merge: token_div must be >= 1");
  return grouped_gemm_impl(groups, ngroups, w_rows, K, 1, FUS_EPI_BF16, block_n, 1, 0, 0, merge,
                           stream, status);
}

static int grouped_gemm_impl(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                             int a_kplanes, int epilogue, int block_n, int ksplit,
                             long split_stride, int group_blocks, const fus_merge_spec* merge,
                             void* stream, int* status, int pdl) {
  if (!groups || ngroups < 1 || ngroups > 2)
    return set_error(FUS_E_INVALID, "ngroups must be 1 or 2");
  if (K <= 0 || K % kBK) return set_error(FUS_E_INVALID, "K=%d must be a positive multiple of 64", K);
  if (w_rows <= 0 || w_rows % 128)
    return set_error(FUS_E_INVALID, "w_rows=%d must be a positive multiple of 128", w_rows);
  if (a_kplanes < 1) return set_error(FUS_E_INVALID, "a_kplanes must be >= 1");
  if (epilogue < FUS_EPI_BF16 || epilogue > FUS_EPI_F32)
    return set_error(FUS_E_INVALID, "unknown epilogue %d", epilogue);
  if (ksplit < 1) return set_error(FUS_E_INVALID, "ksplit must be >= 1");
  if (ksplit > 1 && epilogue != FUS_EPI_F32)
    return set_error(FUS_E_INVALID, "split-K needs the fp32 partial epilogue");
  if (group_blocks < 0) return set_error(FUS_E_INVALID, "group_blocks < 0");

  const int mt2 = mt2_for(w_rows, epilogue, block_n);
  const int MTv = mt2 ? 2 : 1;

  GemmArgs a{};
  a.w_rows = w_rows;
  a.K = K;
  a.ksteps_total = a_kplanes * K / kBK;
  a.ksteps_per_split = (a.ksteps_total + ksplit - 1) / ksplit;
  a.ksplit = (a.ksteps_total + a.ksteps_per_split - 1) / a.ksteps_per_split;
  a.m_tiles = w_rows / (128 * MTv);
  a.split_stride = split_stride;
  a.status = status;
  a.pdl = pdl;
  if (merge) {
    a.mg.counters = merge->counters;
    a.mg.parts = merge->parts;
    a.mg.y = reinterpret_cast<const __nv_bfloat16*>(merge->y);
    a.mg.ld_t = merge->ld_t;
    a.mg.ld_k = merge->ld_k;
    a.mg.topk = merge->topk;
    a.mg.w = merge->w;
    a.mg.ldw = merge->ldw;
    a.mg.res = reinterpret_cast<const __nv_bfloat16*>(merge->res);
    a.mg.ldr = merge->ldr;
    a.mg.extra = merge->extra;
    a.mg.lde = merge->lde;
    a.mg.out = reinterpret_cast<__nv_bfloat16*>(merge->out);
    a.mg.ldo = merge->ldo;
  }
  if (group_blocks == 0) {
    // several blocks per expert (or a multi-block dense group): sweep 8 blocks together
    long blocks = 0, experts = 0;
    for (int g = 0; g < ngroups; ++g) {
      blocks += groups[g].max_blocks;
      experts += groups[g].n_experts;
    }
    group_blocks = blocks > 2 * experts ? 8 : 1;
  }
  a.group_blocks = group_blocks;

  CUtensorMap maps[12] = {};
  long units[2] = {0, 0};
  const int a_box_rows = (epilogue == FUS_EPI_SWIGLU && !mt2) ? 64 : 128;
  const int out_cols = epilogue == FUS_EPI_SWIGLU ? w_rows / 2 : w_rows;
  for (int g = 0; g < ngroups; ++g) {
    const fus_gemm_group& G = groups[g];
    if (!G.w || !G.x || !G.out) return set_error(FUS_E_INVALID, "group %d: null pointer", g);
    if (G.n_experts < 1 || G.x_rows < 1 || G.max_blocks < 0)
      return set_error(FUS_E_INVALID, "group %d: bad sizes", g);
    if (G.ldx < K || G.ldx % 8 || ((uintptr_t)G.x % 16) || ((uintptr_t)G.w % 16))
      return set_error(FUS_E_INVALID, "group %d: rows must be 16-byte aligned", g);
    const bool out32 = epilogue == FUS_EPI_F32 ||
                       (epilogue == FUS_EPI_BF16 && (G.flags & FUS_GEMM_OUT_F32));
    if (G.ldo < out_cols || ((uintptr_t)G.out % 16) || (G.ldo % (out32 ? 4 : 8)))
      return set_error(FUS_E_INVALID, "group %d: output rows must be 16-byte aligned", g);
    int rc = make_tmap_bf16_2d(&maps[g], G.w, (uint64_t)a_kplanes * K,
                               (uint64_t)G.n_experts * w_rows, (uint64_t)a_kplanes * K, kBK,
                               a_box_rows);
    if (rc) return rc;
    if (G.gather_ids && !G.live_ids)
      return set_error(FUS_E_INVALID, "group %d: gathered rows need live_ids/live_limit", g);
    rc = make_tmap_bf16_2d(&maps[2 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows, (uint64_t)G.ldx,
                           kBK, G.gather_ids ? 1 : block_n);
    if (rc) return rc;
    GroupDev& D = a.g[g];
    D.expert_ids = G.expert_ids;
    D.ntp = G.ntp;
    D.x_rows = G.x_rows;
    D.max_blocks = G.max_blocks;
    D.n_experts = G.n_experts;
    D.row_limit = G.row_limit;
    D.out = G.out;
    D.ldo = G.ldo;
    D.row_map = G.row_map;
    D.row_scale = G.row_scale;
    D.flags = G.flags;
    D.live_ids = G.live_ids;
    D.live_limit = G.live_limit;
    D.token_div = G.token_div > 0 ? G.token_div : 1;
    D.gather_ids = G.gather_ids;
    D.gather_div = G.gather_div > 0 ? G.gather_div : 1;
    if (G.res && (epilogue != FUS_EPI_BF16 || (G.flags & FUS_GEMM_MERGE) || G.ldr % 8 ||
                  !aligned16(G.res)))
      return set_error(FUS_E_INVALID, "group %d: residual needs FUS_EPI_BF16, 16-byte rows", g);
    D.res = reinterpret_cast<const __nv_bfloat16*>(G.res);
    D.ldr = G.ldr;
    units[g] = (long)G.max_blocks * a.m_tiles * a.ksplit;
  }
  if (ngroups == 1) {
    maps[1] = maps[0];
    maps[3] = maps[2];
  }
  const long total = units[0] + units[1];
  if (total == 0) return FUS_OK;
  if (total > 0x7fffffffL) return set_error(FUS_E_UNSUPPORTED, "grid too large");
  a.units0 = (int)units[0];
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // prefill with many tiles: one persistent CTA per SM (each tile's loads and MMAs
  // overlap the previous tile's epilogue); FUS_GEMM_NO_PERSIST in the first group's
  // flags opts out.
  const int sms = num_sms();
  if (mt2 && epilogue != FUS_EPI_F32 && !merge && pdl == 0 && a.ksplit == 1 &&
      total > 2L * sms &&
      !(groups[0].flags & FUS_GEMM_NO_PERSIST)) {
    // SM pairs (2-CTA clusters, M = 256 tiles) for 256-token blocks with dense outputs
    bool pair = block_n == kPairBN && a_kplanes == 1 && !(groups[0].flags & FUS_GEMM_NO_PAIR) &&
                (epilogue == FUS_EPI_BF16 || w_rows % 512 == 0);
    for (int g = 0; g < ngroups && pair; ++g) {
      const fus_gemm_group& G = groups[g];
      pair = !G.gather_ids && !G.row_map && !G.row_scale && !G.res && G.row_limit >= 1;
    }
    if (pair) {
      // BF16 tiles of 512 rows when the rows divide: two weight tiles per CTA share each
      // staged token tile, so a stage carries twice the MMA work for 1.5x the bytes (on
      // ~150-token blocks the 256-row tile is bound by operand delivery)
      const bool wide = epilogue == FUS_EPI_BF16 && w_rows % 512 == 0 &&
                        !(groups[0].flags & FUS_GEMM_PAIR_NARROW);
      a.m_tiles = (epilogue == FUS_EPI_SWIGLU || wide) ? w_rows / 512 : w_rows / 256;
      long pu[2] = {0, 0};
      for (int g = 0; g < ngroups; ++g) {
        const fus_gemm_group& G = groups[g];
        pu[g] = (long)G.max_blocks * a.m_tiles;
        const bool out32 = epilogue == FUS_EPI_BF16 && (G.flags & FUS_GEMM_OUT_F32);
        int rc = make_tmap_store_2d(&maps[4 + g], G.out, out32, (uint64_t)out_cols,
                                    (uint64_t)G.row_limit, (uint64_t)G.ldo, 128, out32 ? 16 : 32);
        // token maps: boxes of 128 / 16 / 64 rows (one CTA's half of a block)
        if (!rc)
          rc = make_tmap_bf16_2d(&maps[2 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows,
                                 (uint64_t)G.ldx, kBK, kPairBN / 2);
        if (!rc)
          rc = make_tmap_bf16_2d(&maps[6 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows,
                                 (uint64_t)G.ldx, kBK, 16);
        if (!rc)
          rc = make_tmap_bf16_2d(&maps[8 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows,
                                 (uint64_t)G.ldx, kBK, 64);
        if (!rc)
          rc = make_tmap_bf16_2d(&maps[10 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows,
                                 (uint64_t)G.ldx, kBK, 96);
        if (rc) return rc;
        a.g[g].tma_store = 1;
      }
      if (ngroups == 1) {
        maps[3] = maps[2];
        maps[5] = maps[4];
        maps[7] = maps[6];
        maps[9] = maps[8];
        maps[11] = maps[10];
      }
      const long ptotal = pu[0] + pu[1];
      if (ptotal > 0x7fffffffL) return set_error(FUS_E_UNSUPPORTED, "grid too large");
      a.units0 = (int)pu[0];
      if (epilogue == FUS_EPI_SWIGLU) return launch_pair<FUS_EPI_SWIGLU, 2>(maps, a, ptotal, st);
      return wide ? launch_pair<FUS_EPI_BF16, 2>(maps, a, ptotal, st)
                  : launch_pair<FUS_EPI_BF16, 1>(maps, a, ptotal, st);
    }
    const int grid = (int)(total < sms ? total : sms);
    for (int g = 0; g < ngroups; ++g) {
      const fus_gemm_group& G = groups[g];
      a.g[g].tma_store = 0;
      if (G.row_map || G.row_scale || G.row_limit < 1) continue;
      const bool out32 = epilogue == FUS_EPI_BF16 && (G.flags & FUS_GEMM_OUT_F32);
      // one store = half a staging buffer: 128 features x (32 bf16 | 16 fp32) token rows
      int rc = make_tmap_store_2d(&maps[4 + g], G.out, out32, (uint64_t)out_cols,
                                  (uint64_t)G.row_limit, (uint64_t)G.ldo, 128, out32 ? 16 : 32);
      if (rc) return rc;
      a.g[g].tma_store = 1;
    }
    if (ngroups == 1) maps[5] = maps[4];
    // token maps with 32- and 128-row boxes for blocks with few live rows
    for (int g = 0; g < ngroups; ++g) {
      const fus_gemm_group& G = groups[g];
      int rc = make_tmap_bf16_2d(&maps[6 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows,
                                 (uint64_t)G.ldx, kBK, 32);
      if (!rc)
        rc = make_tmap_bf16_2d(&maps[8 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows,
                               (uint64_t)G.ldx, kBK, block_n < 128 ? block_n : 128);
      if (rc) return rc;
    }
    if (ngroups == 1) {
      maps[7] = maps[6];
      maps[9] = maps[8];
    }
    return epilogue == FUS_EPI_SWIGLU ? launch_persist<FUS_EPI_SWIGLU>(block_n, maps, a, grid, st)
                                      : launch_persist<FUS_EPI_BF16>(block_n, maps, a, grid, st);
  }
  switch (epilogue) {
    case FUS_EPI_BF16: return launch_bn<FUS_EPI_BF16>(block_n, mt2, maps, a, (int)total, st);
    case FUS_EPI_SWIGLU: return launch_bn<FUS_EPI_SWIGLU>(block_n, mt2, maps, a, (int)total, st);
    default: return launch_bn<FUS_EPI_F32>(block_n, mt2, maps, a, (int)total, st);
  }
}
