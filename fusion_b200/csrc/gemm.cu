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
  long split_stride;     // FUS_EPI_F32 partial plane stride (elements)
  int* status;
};

constexpr int kBK = 64;                 // K elements per stage (128 B rows, one swizzle span)
constexpr int kATileBytes = 128 * kBK * 2;
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN <= 16 ? 6 : BN <= 32 ? 5 : BN <= 64 ? 4 : BN <= 128 ? 6 : 4;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = kATileBytes + B_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = RING_BYTES + BAR_BYTES + 1024;  // + alignment slack
  static_assert(RING_BYTES >= BN * 128 * 4, "epilogue staging must fit in the ring");
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap ta0,
                        const __grid_constant__ CUtensorMap ta1,
                        const __grid_constant__ CUtensorMap tb0,
                        const __grid_constant__ CUtensorMap tb1,
                        const __grid_constant__ GemmArgs args) {
  using Cfg = GemmCfg<BN>;
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
  const int mt = u % args.m_tiles;
  const int blk = u / args.m_tiles;
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
  const uint32_t sB = sA + STAGES * kATileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::RING_BYTES);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = smem_u32(bars + STAGES);
  const uint32_t bar_accum = smem_u32(bars + 2 * STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

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
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const uint64_t pol_w = policy_evict_first();  // weights: streamed once
      const uint64_t pol_x = policy_evict_last();   // token rows: re-read by every tile
      const int b_row = blk * BN;
      int a_row0, a_row1 = 0;
      if (EPI == FUS_EPI_SWIGLU) {
        a_row0 = expert * args.w_rows + mt * 64;
        a_row1 = expert * args.w_rows + (args.w_rows >> 1) + mt * 64;
      } else {
        a_row0 = expert * args.w_rows + mt * 128;
      }
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t r = (uint32_t)(i / STAGES);
        if (!mbar_wait_bounded(bar_empty + 8 * s, (r & 1u) ^ 1u, abort_flag, args.status)) break;
        const uint32_t full = bar_full + 8 * s;
        mbar_arrive_expect_tx(full, Cfg::STAGE_BYTES);
        const int kk = (kbeg + i) * kBK;
        const uint32_t a_dst = sA + s * kATileBytes;
        if (EPI == FUS_EPI_SWIGLU) {
          tma_load_2d(a_dst, tma_a, full, kk, a_row0, pol_w);
          tma_load_2d(a_dst + kATileBytes / 2, tma_a, full, kk, a_row1, pol_w);
        } else {
          tma_load_2d(a_dst, tma_a, full, kk, a_row0, pol_w);
        }
        tma_load_2d(sB + s * Cfg::B_BYTES, tma_b, full, kk % args.K, b_row, pol_x);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_bf16_f32(128, BN);
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t r = (uint32_t)(i / STAGES);
        if (!mbar_wait_bounded(bar_full + 8 * s, r & 1u, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t a_base = sA + s * kATileBytes;
        const uint32_t b_base = sB + s * Cfg::B_BYTES;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          // advance 16 bf16 (32 B) along K inside the 128-byte swizzle span
          tc_mma_bf16(tmem, sw128_desc(a_base + 32 * k), sw128_desc(b_base + 32 * k), idesc,
                      (i | k) != 0);
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
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) S[(c + j) * 128 + m] = v[j];
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");

      const int pos0 = blk * BN;
      if (EPI == FUS_EPI_SWIGLU) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(G.out);
        for (int it = et; it < BN * 8; it += 128) {
          const int j = it >> 3, q = it & 7;
          const int pos = pos0 + j;
          const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
          if (row >= G.row_limit) continue;
          const float4* gp = reinterpret_cast<const float4*>(S + j * 128 + q * 8);
          const float4* up = reinterpret_cast<const float4*>(S + j * 128 + 64 + q * 8);
          float g[8], u[8], o[8];
          *reinterpret_cast<float4*>(g) = gp[0];
          *reinterpret_cast<float4*>(g + 4) = gp[1];
          *reinterpret_cast<float4*>(u) = up[0];
          *reinterpret_cast<float4*>(u + 4) = up[1];
          if (!(G.flags & FUS_GEMM_SWIGLU_EXACT)) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              g[e] = round_bf(g[e]);
              u[e] = round_bf(u[e]);
            }
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = (g[e] / (1.0f + expf(-g[e]))) * u[e];
          *reinterpret_cast<uint4*>(out + (long)row * G.ldo + mt * 64 + q * 8) = pack8(o);
        }
      } else if (EPI == FUS_EPI_BF16) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(G.out);
        for (int it = et; it < BN * 16; it += 128) {
          const int j = it >> 4, q = it & 15;
          const int pos = pos0 + j;
          const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
          if (row >= G.row_limit) continue;
          const float sc = G.row_scale ? __ldg(G.row_scale + row) : 1.0f;
          const float4* sp = reinterpret_cast<const float4*>(S + j * 128 + q * 8);
          float v[8];
          *reinterpret_cast<float4*>(v) = sp[0];
          *reinterpret_cast<float4*>(v + 4) = sp[1];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] *= sc;
          if (G.flags & FUS_GEMM_OUT_F32) {
            float4* dp = reinterpret_cast<float4*>(reinterpret_cast<float*>(G.out) +
                                                   (long)row * G.ldo + mt * 128 + q * 8);
            dp[0] = make_float4(v[0], v[1], v[2], v[3]);
            dp[1] = make_float4(v[4], v[5], v[6], v[7]);
          } else {
            *reinterpret_cast<uint4*>(out + (long)row * G.ldo + mt * 128 + q * 8) = pack8(v);
          }
        }
      } else {
        float* out = reinterpret_cast<float*>(G.out) + (long)split * args.split_stride;
        for (int it = et; it < BN * 16; it += 128) {
          const int j = it >> 4, q = it & 15;
          const int pos = pos0 + j;
          const int row = G.row_map ? __ldg(G.row_map + pos) : pos;
          if (row >= G.row_limit) continue;
          const float4* sp = reinterpret_cast<const float4*>(S + j * 128 + q * 8);
          float4* dp = reinterpret_cast<float4*>(out + (long)row * G.ldo + mt * 128 + q * 8);
          dp[0] = sp[0];
          dp[1] = sp[1];
        }
      }
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

// ======================================================================================
// host side
// ======================================================================================
namespace {

template <int BN, int EPI>
int launch_t(const CUtensorMap* maps, const GemmArgs& a, int grid, cudaStream_t st) {
  using Cfg = GemmCfg<BN>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(grouped_gemm_kernel<BN, EPI>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return set_error(FUS_E_LAUNCH, "cudaFuncSetAttribute: %s",
                                                cudaGetErrorString(attr_err));
  grouped_gemm_kernel<BN, EPI><<<grid, kThreads, Cfg::SMEM_BYTES, st>>>(maps[0], maps[1], maps[2],
                                                                       maps[3], a);
  return check_launch("grouped_gemm");
}

template <int EPI>
int launch_bn(int bn, const CUtensorMap* maps, const GemmArgs& a, int grid, cudaStream_t st) {
  switch (bn) {
    case 16: return launch_t<16, EPI>(maps, a, grid, st);
    case 32: return launch_t<32, EPI>(maps, a, grid, st);
    case 64: return launch_t<64, EPI>(maps, a, grid, st);
    case 128: return launch_t<128, EPI>(maps, a, grid, st);
    case 256: return launch_t<256, EPI>(maps, a, grid, st);
  }
  return set_error(FUS_E_UNSUPPORTED, "block_n %d not in {16,32,64,128,256}", bn);
}

}  // namespace
}  // namespace fus

using namespace fus;

extern "C" int fus_grouped_gemm(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                                int a_kplanes, int epilogue, int block_n, int ksplit,
                                long split_stride, void* stream, int* status) {
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

  GemmArgs a{};
  a.w_rows = w_rows;
  a.K = K;
  a.ksteps_total = a_kplanes * K / kBK;
  a.ksteps_per_split = (a.ksteps_total + ksplit - 1) / ksplit;
  a.ksplit = (a.ksteps_total + a.ksteps_per_split - 1) / a.ksteps_per_split;
  a.m_tiles = w_rows / 128;
  a.split_stride = split_stride;
  a.status = status;

  CUtensorMap maps[4];
  long units[2] = {0, 0};
  const int a_box_rows = epilogue == FUS_EPI_SWIGLU ? 64 : 128;
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
    rc = make_tmap_bf16_2d(&maps[2 + g], G.x, (uint64_t)K, (uint64_t)G.x_rows, (uint64_t)G.ldx,
                           kBK, block_n);
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
  switch (epilogue) {
    case FUS_EPI_BF16: return launch_bn<FUS_EPI_BF16>(block_n, maps, a, (int)total, st);
    case FUS_EPI_SWIGLU: return launch_bn<FUS_EPI_SWIGLU>(block_n, maps, a, (int)total, st);
    default: return launch_bn<FUS_EPI_F32>(block_n, maps, a, (int)total, st);
  }
}
