// Router of the GLM-5.2 MoE block: fp32 logits on the tensor cores, then sigmoid
// noaux_tc top-k selection.
//
// Reference: glm52/reference.py:46-79 (router), glm52/kernels/norm_router.py:347 and
// :352 (router_gemm / topk_only entry points).
//
// Logits. The router weight is fp32 (moe_router_dtype float32). Every fp32 value is
// exactly the sum of three bf16 values (8+8+8 significand bits), and x2 is bf16, so
// x2 . W == x2 . W_hi + x2 . W_mid + x2 . W_lo with every product exact in fp32. The
// three planes are laid along K ([E, 3H]) and accumulated into one fp32 TMEM
// accumulator by the grouped tcgen05 GEMM, i.e. an fp32-accurate GEMM at bf16
// tensor-core rate. Small T splits K across CTAs into fp32 partial planes that the
// top-k kernel sums in a fixed order, so the result is deterministic.
#include "common.cuh"
#include "host_util.h"

namespace fus {

__global__ void split_weight_kernel(const float* __restrict__ wg, __nv_bfloat16* __restrict__ wa,
                                    int E, int H) {
  const long n = (long)E * H;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    const int e = (int)(i / H), k = (int)(i % H);
    const float w = wg[i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(w);
    const float r1 = w - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(mid);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r2);
    __nv_bfloat16* row = wa + (long)e * 3 * H;
    row[k] = hi;
    row[H + k] = mid;
    row[2 * H + k] = lo;
  }
}

__global__ void transpose_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out,
                                 int R, int C) {  // in [R, C] -> out [C, R]
  __shared__ __nv_bfloat16 tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = in[(long)r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) out[(long)c * R + r] = tile[threadIdx.x][i];
  }
}

// One warp per token. Lane l owns experts [8l, 8l+8).
constexpr int kTopkWarps = 8;

__global__ void __launch_bounds__(kTopkWarps * 32)
    topk_kernel(const float* __restrict__ partial, long split_stride, int nsplit,
                const float* __restrict__ bias, float* __restrict__ logits_out,
                float* __restrict__ topw, int* __restrict__ topi, int T, int E, int topk,
                float scale, int renorm, int n_group, int topk_group) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kTopkWarps + (threadIdx.x >> 5);
  if (t >= T) return;
  const int e0 = lane * 8;
  float l[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) l[j] = 0.f;
  if (e0 < E) {  // E % 8 == 0 (host check) so a lane's 8 experts are all valid or all not
    const float* p = partial + (long)t * E + e0;
    for (int s = 0; s < nsplit; ++s) {
      const float4 a = *reinterpret_cast<const float4*>(p + (long)s * split_stride);
      const float4 b = *reinterpret_cast<const float4*>(p + (long)s * split_stride + 4);
      l[0] += a.x; l[1] += a.y; l[2] += a.z; l[3] += a.w;
      l[4] += b.x; l[5] += b.y; l[6] += b.z; l[7] += b.w;
    }
    if (logits_out) {
      float4* o = reinterpret_cast<float4*>(logits_out + (long)t * E + e0);
      o[0] = make_float4(l[0], l[1], l[2], l[3]);
      o[1] = make_float4(l[4], l[5], l[6], l[7]);
    }
  }
  float sc[8], ch[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = e0 + j;
    if (e < E) {
      sc[j] = 1.0f / (1.0f + expf(-l[j]));
      ch[j] = sc[j] + (bias ? __ldg(bias + e) : 0.f);
    } else {
      sc[j] = 0.f;
      ch[j] = -INFINITY;
    }
  }
  group_mask_choice(ch, lane, E, n_group, topk_group);
  unsigned used = 0;
  float my_w = 0.f;
  int my_id = 0;
  float wsum = 0.f;
  for (int k = 0; k < topk; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (!(used & (1u << j)) && e0 + j < E && (ch[j] > bv || bi == 0x7fffffff)) {
        bv = ch[j];
        bi = e0 + j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    const int owner = bi >> 3;
    float s_win = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane == owner && bi == e0 + j) {
        used |= 1u << j;
        s_win = sc[j];
      }
    s_win = __shfl_sync(0xffffffffu, s_win, owner & 31);
    wsum += s_win;
    if (lane == k) {
      my_w = s_win;
      my_id = bi;
    }
  }
  if (lane < topk) {
    float wv = my_w;
    if (renorm) wv = wv / fmaxf(wsum, 1e-20f);
    wv = wv * scale;
    topw[(long)t * topk + lane] = wv;
    topi[(long)t * topk + lane] = my_id;
  }
}

// CUDA-core fp32 GEMV for small T: CTA = 2 experts x all tokens. Every weight element is
// reassembled exactly from its bf16 planes (hi + mid + lo, each sum exact) and used in
// fp32 FMAs, so the result is an fp32 dot product like the reference's F.linear.
constexpr int kGemvThreads = 256;
constexpr int kGemvExperts = 2;
constexpr int kGemvTokens = 8;
constexpr int kGemvMaxT = 16;

template <int NP>
__global__ void __launch_bounds__(kGemvThreads)
    router_gemv_kernel(const __nv_bfloat16* __restrict__ x2, long ldx,
                       const __nv_bfloat16* __restrict__ wa, float* __restrict__ logits, int T,
                       int H, int E) {
  __shared__ float red[kGemvThreads / 32][kGemvExperts * kGemvTokens];
  const int e0 = blockIdx.x * kGemvExperts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunk = H >> 3;
  for (int t0 = 0; t0 < T; t0 += kGemvTokens) {
    float acc[kGemvExperts][kGemvTokens];
#pragma unroll
    for (int a = 0; a < kGemvExperts; ++a)
#pragma unroll
      for (int b = 0; b < kGemvTokens; ++b) acc[a][b] = 0.f;
    for (int c = threadIdx.x; c < nchunk; c += kGemvThreads) {
      float w[kGemvExperts][8];
#pragma unroll
      for (int a = 0; a < kGemvExperts; ++a) {
        const __nv_bfloat16* row = wa + (long)(e0 + a) * NP * H + c * 8;
        unpack8(__ldg(reinterpret_cast<const uint4*>(row)), w[a]);
#pragma unroll
        for (int p = 1; p < NP; ++p) {
          float q[8];
          unpack8(__ldg(reinterpret_cast<const uint4*>(row + (long)p * H)), q);
#pragma unroll
          for (int i = 0; i < 8; ++i) w[a][i] += q[i];
        }
      }
#pragma unroll
      for (int b = 0; b < kGemvTokens; ++b) {
        if (t0 + b < T) {
          float x[8];
          unpack8(__ldg(reinterpret_cast<const uint4*>(x2 + (long)(t0 + b) * ldx + c * 8)), x);
#pragma unroll
          for (int a = 0; a < kGemvExperts; ++a)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[a][b] = fmaf(x[i], w[a][i], acc[a][b]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < kGemvExperts; ++a)
#pragma unroll
      for (int b = 0; b < kGemvTokens; ++b) {
        const float v = warp_sum(acc[a][b]);
        if (lane == 0) red[warp][a * kGemvTokens + b] = v;
      }
    __syncthreads();
    if (threadIdx.x < kGemvExperts * kGemvTokens) {
      const int a = threadIdx.x / kGemvTokens, b = threadIdx.x % kGemvTokens;
      float v = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kGemvThreads / 32; ++w2) v += red[w2][threadIdx.x];
      if (t0 + b < T) logits[(long)(t0 + b) * E + e0 + a] = v;
    }
    __syncthreads();
  }
}

int router_block_n(int T) {
  return T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
}

}  // namespace fus

using namespace fus;

extern "C" int fus_router_split_weight(const float* wg, void* wa, int E, int H, void* stream) {
  if (!wg || !wa || E <= 0 || H <= 0) return set_error(FUS_E_INVALID, "split_weight: bad args");
  const long n = (long)E * H;
  const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  split_weight_kernel<<<grid, 256, 0, as_stream(stream)>>>(wg, (__nv_bfloat16*)wa, E, H);
  return check_launch("router_split_weight");
}

extern "C" int fus_router_transpose_weight(const void* wgt, void* wa, int H, int E, void* stream) {
  if (!wgt || !wa || E <= 0 || H <= 0) return set_error(FUS_E_INVALID, "transpose_weight: bad args");
  dim3 grid(ceil_div(E, 32), ceil_div(H, 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>((const __nv_bfloat16*)wgt,
                                                                (__nv_bfloat16*)wa, H, E);
  return check_launch("router_transpose_weight");
}

extern "C" int fus_router_nsplit(int T, int H, int E, int nplanes) {
  if (T <= 0 || H <= 0 || E <= 0 || nplanes <= 0 || H % 64 || E % 128) return 1;
  if (T <= kGemvMaxT) return 1;  // CUDA-core GEMV path writes the logits directly
  const int bn = router_block_n(T);
  const long units = (long)(E / 128) * ceil_div(T, bn);
  const int ksteps = nplanes * H / 64;
  if (T < 1024) {
    // weight-streaming regime: as many CTAs as the SMs take, each on its own K range
    long want = (num_sms() + units - 1) / units;
    if (want > ksteps / 4) want = ksteps / 4;
    if (want > 64) want = 64;
    if (want < 1) want = 1;
    const int kps = ceil_div(ksteps, want);
    return ceil_div(ksteps, kps);  // the split count the GEMM will actually use
  }
  // compute regime: K splits s minimising  waves(s) * (tile time / s)  +  partial-plane
  // traffic(s):
  // a tile's full-K time at the tensor peak per SM, waves over the CTA slots of this
  // tile width, and s fp32 planes written and read back by the top-k
  const double slots = (double)num_sms() * (bn <= 32 ? 3 : bn <= 64 ? 2 : 1);
  const double tile_s = 2.0 * bn * 128 * (double)ksteps * 64 / 10.8e12;
  const double plane_s = 2.0 * (double)T * E * 4 / 6.5e12;
  int smax = ksteps / 4;
  if (smax > 64) smax = 64;
  if (smax < 1) smax = 1;
  int best = 1;
  double best_cost = 1e30;
  for (int sp = 1; sp <= smax; ++sp) {
    const int kps = ceil_div(ksteps, sp);
    const int s = ceil_div(ksteps, kps);  // the split count the GEMM will actually use
    const double waves = ceil((double)units * s / slots);
    const double cost = waves * tile_s / s + s * plane_s;
    if (cost < best_cost * (1 - 1e-9)) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

extern "C" int fus_router_logits(const void* x2, long ldx, const void* wa, int nplanes,
                                 float* partial, int T, int H, int E, int nsplit, void* stream,
                                 int* status) {
  if (!x2 || !wa || !partial || T < 0 || nplanes < 1)
    return set_error(FUS_E_INVALID, "router_logits: bad args");
  if (E % 128) return set_error(FUS_E_UNSUPPORTED, "router_logits: E=%d must be a multiple of 128", E);
  if (H % 64) return set_error(FUS_E_UNSUPPORTED, "router_logits: H=%d must be a multiple of 64", H);
  if (T == 0) return FUS_OK;
  if (T <= kGemvMaxT && (nplanes == 1 || nplanes == 3)) {
    if (nsplit != 1) return set_error(FUS_E_INVALID, "router_logits: nsplit must be 1 for T <= 16");
    if (!aligned16(x2) || ldx % 8 || !aligned16(wa))
      return set_error(FUS_E_INVALID, "router_logits: rows must be 16-byte aligned");
    const int grid = E / kGemvExperts;
    if (nplanes == 3)
      router_gemv_kernel<3><<<grid, kGemvThreads, 0, as_stream(stream)>>>(
          (const __nv_bfloat16*)x2, ldx, (const __nv_bfloat16*)wa, partial, T, H, E);
    else
      router_gemv_kernel<1><<<grid, kGemvThreads, 0, as_stream(stream)>>>(
          (const __nv_bfloat16*)x2, ldx, (const __nv_bfloat16*)wa, partial, T, H, E);
    return check_launch("router_gemv");
  }
  const int ksteps = nplanes * H / 64;
  if (nsplit < 1 || nsplit > ksteps || ceil_div(ksteps, ceil_div(ksteps, nsplit)) != nsplit)
    return set_error(FUS_E_INVALID, "router_logits: nsplit=%d not normalised (use fus_router_nsplit)",
                     nsplit);
  const int bn = router_block_n(T);
  fus_gemm_group g{};
  g.w = wa;
  g.n_experts = 1;
  g.x = x2;
  g.ldx = ldx;
  g.x_rows = T;
  g.expert_ids = nullptr;
  g.ntp = nullptr;
  g.max_blocks = ceil_div(T, bn);
  g.out = partial;
  g.ldo = E;
  g.row_map = nullptr;
  g.row_limit = T;
  g.row_scale = nullptr;
  return fus_grouped_gemm(&g, 1, E, H, nplanes, FUS_EPI_F32, bn, nsplit, (long)T * E, stream,
                          status);
}

extern "C" int fus_router_topk_grouped(const float* partial, int nsplit, const float* bias,
                                       float* logits_out, float* topw, int* topi, int T, int E,
                                       int topk, int n_group, int topk_group, float scale,
                                       int renorm, void* stream, int* status) {
  (void)status;
  if (n_group < 1 || topk_group < 1 || topk_group > n_group || E % n_group ||
      (n_group > 1 && ((E / n_group) % 8 || ((E / n_group / 8) & (E / n_group / 8 - 1)) ||
                       n_group > 32 || topk > topk_group * (E / n_group))))
    return set_error(FUS_E_UNSUPPORTED,
                     "router_topk: n_group=%d topk_group=%d E=%d (groups of 8*2^k experts, "
                     "n_group <= 32)", n_group, topk_group, E);
  if (!partial || !topw || !topi || T < 0 || nsplit < 1)
    return set_error(FUS_E_INVALID, "router_topk: bad args");
  if (E <= 0 || E > 256 || E % 8 || topk < 1 || topk > 16 || topk > E)
    return set_error(FUS_E_UNSUPPORTED, "router_topk: E=%d topk=%d unsupported", E, topk);
  if (!aligned16(partial) || (logits_out && !aligned16(logits_out)))
    return set_error(FUS_E_INVALID, "router_topk: logits must be 16-byte aligned");
  if (T == 0) return FUS_OK;
  topk_kernel<<<ceil_div(T, kTopkWarps), kTopkWarps * 32, 0, as_stream(stream)>>>(
      partial, (long)T * E, nsplit, bias, logits_out, topw, topi, T, E, topk, scale, renorm,
      n_group, topk_group);
  return check_launch("router_topk");
}

extern "C" int fus_router_topk(const float* partial, int nsplit, const float* bias,
                               float* logits_out, float* topw, int* topi, int T, int E, int topk,
                               float scale, int renorm, void* stream, int* status) {
  return fus_router_topk_grouped(partial, nsplit, bias, logits_out, topw, topi, T, E, topk, 1, 1,
                                 scale, renorm, stream, status);
}
