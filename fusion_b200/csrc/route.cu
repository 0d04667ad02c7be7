// Decode front end of the MoE block in ONE launch (T <= 16 tokens):
//   add + RMSNorm  ->  fp32 router logits  ->  sigmoid noaux_tc top-k  ->  dispatch layout
//
// At decode sizes each of these steps is a few microseconds of latency and almost no
// work, so as four launches they cost more than the data they move. Here every CTA
// normalises the T rows into shared memory (same rounding as add_rmsnorm_kernel, so h1
// and x2 are bit-identical to the separate kernel) and computes the fp32 logits of one
// expert from the reassembled bf16 weight planes; the last CTA to finish (atomic
// ticket) selects the top-k of every token (same rule as topk_kernel) and builds the
// sglang dispatch layout (same layout as fus_moe_align), then re-arms the ticket.
//
// Reference: glm52/reference.py:22-33 (add_rmsnorm), :46-79 (router), :85-128
// (moe_align_block_size).
#include "common.cuh"
#include "host_util.h"

namespace fus {

constexpr int kRouteThreads = 256;
constexpr int kRouteExperts = 1;
constexpr int kRouteMaxT = 16;

struct RouteArgs {
  const __nv_bfloat16* h;
  const __nv_bfloat16* r;
  const __nv_bfloat16* gamma;
  float eps;
  const __nv_bfloat16* wa;
  int nplanes;
  const float* bias;
  int T, H, E, topk;
  float scale;
  int renorm;
  int n_group, topk_group;
  __nv_bfloat16* h1;
  __nv_bfloat16* x2;
  float* logits;
  float* topw;
  int* topi;
  int block_m;
  int* sorted;
  int sorted_cap;
  int* eids;
  int blocks_cap;
  int* ntp;
  int* done;
  int* zero;
  int zero_n;
  int* status;
};

// Optional phase timestamps (globaltimer ns), compiled only with FUS_ROUTE_TRACE:
// [0] earliest CTA start, [1] latest CTA at the ticket, [2] CTA 0 after the norm,
// [3] CTA 0 after the logits, [4] last CTA after selection, [5] last CTA done.
#ifdef FUS_ROUTE_TRACE
__device__ unsigned long long g_route_trace[8];
#define RT(...) __VA_ARGS__
#else
#define RT(...)
#endif

__global__ void __launch_bounds__(kRouteThreads)
    route_small_kernel(const __grid_constant__ RouteArgs a) {
  RT(if (threadIdx.x == 0) atomicMin(&g_route_trace[0], globaltimer_ns());)
  extern __shared__ __align__(16) uint8_t dsm[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(dsm);  // [T][H]: h1, then x2
  __shared__ float rstd_s[kRouteMaxT];
  __shared__ float part[kRouteThreads / 32][kRouteExperts * kRouteMaxT];
  __shared__ int is_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, H = a.H, E = a.E;
  const int nv = H >> 3;
  const bool writer = blockIdx.x == 0;
  const int e0 = blockIdx.x * kRouteExperts;
  pdl_allow_dependents();  // the w13 GEMM may become resident and set up meanwhile
  // this expert's weight planes for up to 4 chunks per thread are loaded up front (all
  // in flight at once) while the CTA normalises
  constexpr int kMaxChunks = 4;  // H <= 4 * 8 * 256 = 8192
  uint4 wq[kMaxChunks][3];
  uint4 gq[kMaxChunks];  // the norm weight, for step 2
#pragma unroll
  for (int ci = 0; ci < kMaxChunks; ++ci) {
    const int c = tid + ci * kRouteThreads;
#pragma unroll
    for (int p = 0; p < 3; ++p)
      if (c < nv && p < a.nplanes)
        wq[ci][p] = __ldg(reinterpret_cast<const uint4*>(a.wa + (long)e0 * a.nplanes * H +
                                                         (long)p * H + c * 8));
    if (c < nv) gq[ci] = __ldg(reinterpret_cast<const uint4*>(a.gamma) + c);
  }
  // the correction bias of experts lane*8 .. lane*8+7, for the selection (whichever CTA
  // turns out to be the last one needs it; loading it now takes it off the tail)
  float bq[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = lane * 8 + j;
    bq[j] = (a.bias && e < E) ? __ldg(a.bias + e) : 0.f;
  }

  // ---- 1. h1 = bf16(h + r) into shared memory, sum of squares per token ----
  // per-warp partial sums per token (no block barrier between tokens); one reduction
  // across the warps for all T afterwards
  for (int t = 0; t < T; ++t) {
    float ss = 0.f;
#pragma unroll
    for (int ci = 0; ci < kMaxChunks; ++ci) {
      const int c = tid + ci * kRouteThreads;
      if (c < nv) {
        float x[8], rr[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(a.h + (long)t * H) + c), x);
        unpack8(__ldg(reinterpret_cast<const uint4*>(a.r + (long)t * H) + c), rr);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          x[e] = round_bf(x[e] + rr[e]);
          ss += x[e] * x[e];
        }
        const uint4 v = pack8(x);
        reinterpret_cast<uint4*>(xs + (long)t * H)[c] = v;
        if (writer) reinterpret_cast<uint4*>(a.h1 + (long)t * H)[c] = v;
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) part[warp][t] = ss;
  }
  __syncthreads();
  if (tid < T) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kRouteThreads / 32; ++w) v += part[w][tid];
    rstd_s[tid] = 1.0f / sqrtf(v / (float)H + a.eps);
  }
  __syncthreads();
  // ---- 2. x2 = bf16(bf16(h1 * rstd) * gamma), in place ----
  for (int t = 0; t < T; ++t) {
    const float rs = rstd_s[t];
#pragma unroll
    for (int ci = 0; ci < kMaxChunks; ++ci) {
      const int c = tid + ci * kRouteThreads;
      if (c >= nv) break;
      float x[8], g[8];
      unpack8(reinterpret_cast<const uint4*>(xs + (long)t * H)[c], x);
      unpack8(gq[ci], g);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = round_bf(x[e] * rs) * g[e];
      const uint4 v = pack8(x);
      reinterpret_cast<uint4*>(xs + (long)t * H)[c] = v;
      if (writer) reinterpret_cast<uint4*>(a.x2 + (long)t * H)[c] = v;
    }
  }
  __syncthreads();
  RT(if (threadIdx.x == 0 && blockIdx.x == 0) g_route_trace[2] = globaltimer_ns();)
  // ---- 3. logits of expert e0 (fp32 FMAs over the reassembled fp32 weight) ----
  float acc[kRouteExperts][kRouteMaxT];
#pragma unroll
  for (int e = 0; e < kRouteExperts; ++e)
#pragma unroll
    for (int t = 0; t < kRouteMaxT; ++t) acc[e][t] = 0.f;
#pragma unroll
  for (int ci = 0; ci < kMaxChunks; ++ci) {
    const int c = tid + ci * kRouteThreads;
    if (c >= nv) break;
    float w[kRouteExperts][8];
    unpack8(wq[ci][0], w[0]);
#pragma unroll
    for (int p = 1; p < 3; ++p) {
      if (p < a.nplanes) {
        float q[8];
        unpack8(wq[ci][p], q);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[0][i] += q[i];
      }
    }
#pragma unroll
    for (int t = 0; t < kRouteMaxT; ++t) {
      if (t < T) {
        float x[8];
        unpack8(reinterpret_cast<const uint4*>(xs + (long)t * H)[c], x);
#pragma unroll
        for (int e = 0; e < kRouteExperts; ++e)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[e][t] = fmaf(x[i], w[e][i], acc[e][t]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < kRouteExperts; ++e)
#pragma unroll
    for (int t = 0; t < kRouteMaxT; ++t) {
      const float v = warp_sum(acc[e][t]);
      if (lane == 0) part[warp][e * kRouteMaxT + t] = v;
    }
  __syncthreads();
  if (tid < kRouteExperts * kRouteMaxT) {
    const int e = tid / kRouteMaxT, t = tid % kRouteMaxT;
    if (t < T) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kRouteThreads / 32; ++w) v += part[w][tid];
      a.logits[(long)t * E + e0 + e] = v;
    }
  }
  RT(if (threadIdx.x == 0 && blockIdx.x == 0) g_route_trace[3] = globaltimer_ns();)
  // ---- 4. ticket: the last CTA selects and lays out ----
  __threadfence();
  __syncthreads();
  RT(if (threadIdx.x == 0) atomicMax(&g_route_trace[1], globaltimer_ns());)
  if (tid == 0) is_last = atomicAdd(a.done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  int* ids_s = reinterpret_cast<int*>(dsm);  // reuse: [T*topk] chosen experts
  int* cnt = ids_s + kRouteMaxT * 16;         // [E]
  int* start = cnt + 256;                     // [E]
  int* scan = start + 256;                    // [256]
  const int e8 = lane * 8;
  for (int t = warp; t < T; t += kRouteThreads / 32) {
    // lane l holds experts 8l .. 8l+7: unbiased score sc, selection score ch
    float sc[8], ch[8];
    int ix[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e8 + j;
      ix[j] = e;
      if (e < E) {
        const float l = __ldcg(a.logits + (long)t * E + e);
        sc[j] = 1.0f / (1.0f + expf(-l));
        ch[j] = sc[j] + bq[j];
      } else {
        sc[j] = 0.f;
        ch[j] = -INFINITY;
        ix[j] = 0x7fffffff;
      }
    }
    RT(if (lane == 0 && t == 0) g_route_trace[6] = globaltimer_ns();)
    group_mask_choice(ch, lane, E, a.n_group, a.topk_group);
    // order-preserving unsigned keys of the choice values (descending choice, then the
    // lower expert id): each round takes the warp's best with two redux.sync maxima
    // (key, then 0xffff - id among the lanes holding that key), and the winner's lane
    // drops it and re-takes its own best of 8
    uint32_t key[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t u = __float_as_uint(ch[j] + 0.0f);  // -0 (a masked choice) as +0
      key[j] = ix[j] == 0x7fffffff ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
    }
    auto lane_best = [&](uint32_t& bk, int& bj) {
      bk = key[0];
      bj = 0;
#pragma unroll
      for (int j = 1; j < 8; ++j)
        if (key[j] > bk) {  // strict: equal keys keep the lower index (lower expert id)
          bk = key[j];
          bj = j;
        }
    };
    uint32_t bk;
    int bj;
    lane_best(bk, bj);
    RT(if (lane == 0 && t == 0) g_route_trace[7] = globaltimer_ns();)
    float my_w = 0.f, wsum = 0.f;
    int my_id = 0;
    for (int k = 0; k < a.topk; ++k) {
      const uint32_t top = __reduce_max_sync(0xffffffffu, bk);
      const uint32_t lo = __reduce_max_sync(0xffffffffu, bk == top ? 0xffffu - (uint32_t)(e8 + bj) : 0u);
      const int bi = 0xffff - (int)lo;
      const int owner = bi >> 3;
      float s_mine = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j == bj) s_mine = sc[j];
      const float s_win = __shfl_sync(0xffffffffu, s_mine, owner);
      if (lane == owner) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j == bj) key[j] = 0u;
        lane_best(bk, bj);
      }
      wsum += s_win;
      if (lane == k) {
        my_w = s_win;
        my_id = bi;
      }
    }
    if (lane < a.topk) {
      float wv = my_w;
      if (a.renorm) wv = wv / fmaxf(wsum, 1e-20f);
      wv = wv * a.scale;
      a.topw[(long)t * a.topk + lane] = wv;
      a.topi[(long)t * a.topk + lane] = my_id;
      ids_s[t * a.topk + lane] = my_id;
    }
  }
  RT(__syncthreads(); if (threadIdx.x == 0) g_route_trace[4] = globaltimer_ns();)
  if (a.block_m == 0) {  // no layout wanted (the expert-parallel step builds its own)
    for (int i = tid; i < a.zero_n; i += kRouteThreads) a.zero[i] = 0;
    if (tid == 0) *a.done = 0;  // re-arm the ticket
    return;
  }
  // dispatch layout over the T*topk flat indices (stable by flat index)
  const int numel = T * a.topk;
  for (int e = tid; e < 256; e += kRouteThreads) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < numel; i += kRouteThreads) atomicAdd(cnt + ids_s[i], 1);
  __syncthreads();
  const int bm = a.block_m;
  const int padded = tid < E ? (cnt[tid] + bm - 1) / bm * bm : 0;
  // inclusive scan of the padded counts: within each warp by shuffles, then over the
  // eight warp totals
  int incl = padded;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) scan[warp] = incl;
  __syncthreads();
  int total = 0;
#pragma unroll
  for (int w = 0; w < kRouteThreads / 32; ++w) {
    const int v = scan[w];
    if (w < warp) incl += v;
    total += v;
  }
  if (tid < E) start[tid] = incl - padded;
  if (tid == 0) {
    a.ntp[0] = total;
    if (total > a.sorted_cap || total / bm > a.blocks_cap) raise_status(a.status, FUS_ERR_CAPACITY);
  }
  if (tid < E && padded > 0) {
    const int s0 = incl - padded;
    for (int b = s0 / bm; b < (s0 + padded) / bm; ++b)
      if (b < a.blocks_cap) a.eids[b] = tid;
    for (int p = s0 + cnt[tid]; p < s0 + padded; ++p)
      if (p < a.sorted_cap) a.sorted[p] = numel;
  }
  __syncthreads();
  for (int i = tid; i < numel; i += kRouteThreads) {
    const int e = ids_s[i];
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += ids_s[j] == e;
    const int p = start[e] + rank;
    if (p < a.sorted_cap) a.sorted[p] = i;
  }
  for (int i = tid; i < a.zero_n; i += kRouteThreads) a.zero[i] = 0;
  if (tid == 0) *a.done = 0;  // re-arm the ticket
  RT(__syncthreads(); if (threadIdx.x == 0) g_route_trace[5] = globaltimer_ns();)
}

}  // namespace fus

using namespace fus;

namespace fus {
int route_small_check(int T, int H, int E, int topk, int n_group, int topk_group, int block_m,
                      int nplanes) {
  if (n_group < 1) n_group = 1;
  if (topk_group < 1) topk_group = 1;
  if (n_group > 1 && (E % n_group || (E / n_group) % 8 ||
                      ((E / n_group / 8) & (E / n_group / 8 - 1)) || n_group > 32 ||
                      topk_group > n_group || topk > topk_group * (E / n_group)))
    return set_error(FUS_E_UNSUPPORTED, "route_small: n_group=%d topk_group=%d E=%d", n_group,
                     topk_group, E);
  if (T < 1 || T > kRouteMaxT || E < 2 || E > 256 || E % 2 || topk < 1 || topk > 16 ||
      topk > E || T * topk > 256 || H % 8 || H <= 0 || H > 8192 || block_m < 0 ||
      (nplanes != 1 && nplanes != 3))
    return set_error(FUS_E_UNSUPPORTED, "route_small: T=%d E=%d topk=%d H=%d unsupported", T, E,
                     topk, H);
  const size_t smem = (size_t)T * H * 2;
  if (smem > 200 * 1024) return set_error(FUS_E_UNSUPPORTED, "route_small: T*H too large");
  return FUS_OK;
}

int route_small_launch(const void* h, const void* r, const void* gamma, float eps, const void* wa,
                       int nplanes, const float* bias, int T, int H, int E, int topk, float scale,
                       int renorm, int n_group, int topk_group, void* h1, void* x2, float* logits,
                       float* topw, int* topi, int block_m, int* sorted_ids, int sorted_cap,
                       int* expert_ids, int blocks_cap, int* ntp, int* done, int* zero,
                       int zero_n, void* stream, int* status) {
  if (int rc = route_small_check(T, H, E, topk, n_group, topk_group, block_m, nplanes))
    return rc;
  if (n_group < 1) n_group = 1;
  if (topk_group < 1) topk_group = 1;
  if (!h || !r || !gamma || !wa || !h1 || !x2 || !logits || !topw || !topi ||
      (block_m > 0 && (!sorted_ids || !expert_ids || !ntp)) || !done || (zero_n > 0 && !zero))
    return set_error(FUS_E_INVALID, "route_small: null argument");
  if (!aligned16(h) || !aligned16(r) || !aligned16(gamma) || !aligned16(wa) || !aligned16(h1) ||
      !aligned16(x2))
    return set_error(FUS_E_INVALID, "route_small: rows must be 16-byte aligned");
  const size_t smem = (size_t)T * H * 2;
  const size_t smem_min = sizeof(int) * (kRouteMaxT * 16 + 3 * 256);
  const size_t dyn = smem > smem_min ? smem : smem_min;
  if (int rc = ensure_smem_attr((const void*)route_small_kernel, 200 * 1024, "route_small"))
    return rc;
  if (dyn > 200 * 1024) return set_error(FUS_E_UNSUPPORTED, "route_small: T*H too large");
  RouteArgs a{};
  a.h = (const __nv_bfloat16*)h;
  a.r = (const __nv_bfloat16*)r;
  a.gamma = (const __nv_bfloat16*)gamma;
  a.eps = eps;
  a.wa = (const __nv_bfloat16*)wa;
  a.nplanes = nplanes;
  a.bias = bias;
  a.T = T;
  a.H = H;
  a.E = E;
  a.topk = topk;
  a.scale = scale;
  a.renorm = renorm;
  a.n_group = n_group;
  a.topk_group = topk_group;
  a.h1 = (__nv_bfloat16*)h1;
  a.x2 = (__nv_bfloat16*)x2;
  a.logits = logits;
  a.topw = topw;
  a.topi = topi;
  a.block_m = block_m;
  a.sorted = sorted_ids;
  a.sorted_cap = sorted_cap;
  a.eids = expert_ids;
  a.blocks_cap = blocks_cap;
  a.ntp = ntp;
  a.done = done;
  a.zero = zero;
  a.zero_n = zero_n;
  a.status = status;
  route_small_kernel<<<E / kRouteExperts, kRouteThreads, dyn, as_stream(stream)>>>(a);
  return check_launch("route_small");
}
}  // namespace fus

extern "C" int fus_moe_route_small(const void* h, const void* r, const void* gamma, float eps,
                                   const void* wa, int nplanes, const float* bias, int T, int H,
                                   int E, int topk, float scale, int renorm, void* h1, void* x2,
                                   float* logits, float* topw, int* topi, int block_m,
                                   int* sorted_ids, int sorted_cap, int* expert_ids,
                                   int blocks_cap, int* ntp, int* done, int* zero, int zero_n,
                                   void* stream, int* status) {
  return route_small_launch(h, r, gamma, eps, wa, nplanes, bias, T, H, E, topk, scale, renorm, 1,
                            1, h1, x2, logits, topw, topi, block_m, sorted_ids, sorted_cap,
                            expert_ids, blocks_cap, ntp, done, zero, zero_n, stream, status);
}

#ifdef FUS_ROUTE_TRACE
extern "C" int fus_route_trace(int reset, unsigned long long* host) {
  if (reset) {
    unsigned long long init[8] = {~0ull, 0, 0, 0, 0, 0, 0, 0};
    return cudaMemcpyToSymbol(fus::g_route_trace, init, sizeof(init)) != cudaSuccess;
  }
  return cudaMemcpyFromSymbol(host, fus::g_route_trace, sizeof(fus::g_route_trace)) != cudaSuccess;
}
#endif
