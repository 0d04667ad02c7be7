// Memory-bound row kernels of the MoE block: ResAdd+RMSNorm, SwiGLU, expert merge
// (+ residual + shared expert), residual add and accumulator seeding.
//
// All of them stream bf16 rows with 128-bit loads/stores (8 elements per thread per
// access), keep arithmetic in fp32, and reproduce the reference's rounding points
// exactly where the reference rounds (glm52/reference.py:22-40, :159-188).
#include "common.cuh"
#include "host_util.h"

namespace fus {

// ======================================================================================
// ResAdd + RMSNorm   (glm52/kernels/add_rmsnorm.py:50-191; reference.py:22-33)
// One CTA per row; the row stays in registers between the sum of squares and the
// normalisation, so the fused form moves exactly 2 reads + 2 writes per element.
// ======================================================================================
constexpr int kNormThreads = 256;

template <int VPT>
__global__ void __launch_bounds__(kNormThreads)
    add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long ldx,
                       const __nv_bfloat16* __restrict__ res, long ldr,
                       const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ h1,
                       long ldh, __nv_bfloat16* __restrict__ out, long ldo, int N, float eps,
                       int do_add, int do_norm) {
  const int t = blockIdx.x;
  const int nv = N >> 3;
  float h[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int idx = threadIdx.x + v * kNormThreads;
    if (idx < nv) {
      unpack8(ldg_stream(x + (long)t * ldx + idx * 8), h[v]);
      if (do_add) {
        float r[8];
        unpack8(ldg_stream(res + (long)t * ldr + idx * 8), r);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[v][e] = round_bf(h[v][e] + r[e]);  // h1 = bf16(x + r)
        if (h1) *reinterpret_cast<uint4*>(h1 + (long)t * ldh + idx * 8) = pack8(h[v]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += h[v][e] * h[v][e];
    }
  }
  if (!do_norm) return;

  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean = red[0] / (float)N;
  const float rstd = 1.0f / sqrtf(mean + eps);
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int idx = threadIdx.x + v * kNormThreads;
    if (idx < nv) {
      float g[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(w + idx * 8), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = round_bf(h[v][e] * rstd) * g[e];  // (h*rstd).bf16 * w
      *reinterpret_cast<uint4*>(out + (long)t * ldo + idx * 8) = pack8(o);
    }
  }
}

// ======================================================================================
// SwiGLU  (glm52/kernels/moe_gateup.py:154-182; reference.py:36-40)
// ======================================================================================
__global__ void silu_and_mul_kernel(const __nv_bfloat16* __restrict__ x, long ldx,
                                    __nv_bfloat16* __restrict__ y, long ldy, int I) {
  const int m = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= I) return;
  float g[8], u[8], o[8];
  unpack8(ldg_stream(x + (long)m * ldx + c), g);
  unpack8(ldg_stream(x + (long)m * ldx + I + c), u);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = (g[e] / (1.0f + expf(-g[e]))) * u[e];
  *reinterpret_cast<uint4*>(y + (long)m * ldy + c) = pack8(o);
}

// ======================================================================================
// Expert merge (+ residual, + shared expert)
//   (glm52/kernels/merge_resadd.py:59-185, moe_down_merge.py:300-349, reference.py:159-188)
// ======================================================================================
template <int KT>
__global__ void merge_kernel(const __nv_bfloat16* __restrict__ y, long ld_t, long ld_k, int K,
                             const int* __restrict__ pos_of, const float* __restrict__ w, long ldw,
                             const __nv_bfloat16* __restrict__ res, long ldr,
                             const void* __restrict__ extra, long lde, int extra_f32,
                             __nv_bfloat16* __restrict__ out, long ldo, int H, int round_mid,
                             const int* flags, const int* epoch, int W, int* status) {
  // expert-parallel combine: wait until every owner raised flags[w] >= *epoch (their
  // rows are in y); bounded, FUS_ERR_TIMEOUT when it runs out
  if (flags) {
    pdl_wait();
    if ((int)threadIdx.x < W) {
      const int e = *epoch;
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys_i32(flags + threadIdx.x) < e) {
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
          raise_status(status, FUS_ERR_TIMEOUT);
          break;
        }
      }
    }
    __syncthreads();
  }
  const int t = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= H) return;
  const int nk = KT > 0 ? KT : K;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  // row of (t, k): y + t*ld_t + k*ld_k, or y + pos_of[t*K + k]*ld_k (rows stored in
  // dispatch order)
  const __nv_bfloat16* yt = y + (long)t * ld_t + c;
  auto yrow = [&](int k) {
    return pos_of ? y + (long)__ldg(pos_of + (long)t * nk + k) * ld_k + c : yt + (long)k * ld_k;
  };
  if (KT > 0) {
    uint4 yv[KT > 0 ? KT : 1];
#pragma unroll
    for (int k = 0; k < (KT > 0 ? KT : 1); ++k) yv[k] = ldg_stream(yrow(k));
#pragma unroll
    for (int k = 0; k < (KT > 0 ? KT : 1); ++k) {
      const float wk = w ? __ldg(w + (long)t * ldw + k) : 1.0f;
      float f[8];
      unpack8(yv[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += wk * f[e];
    }
  } else {
    for (int k = 0; k < nk; ++k) {
      const float wk = w ? __ldg(w + (long)t * ldw + k) : 1.0f;
      float f[8];
      unpack8(ldg_stream(yrow(k)), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += wk * f[e];
    }
  }
  if (round_mid) {
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = round_bf(acc[e]);
  }
  if (res) {
    float f[8];
    unpack8(ldg_stream(res + (long)t * ldr + c), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += f[e];
  }
  if (extra) {
    float f[8];
    if (extra_f32) {
      const float* ep = reinterpret_cast<const float*>(extra) + (long)t * lde + c;
      *reinterpret_cast<uint4*>(f) = ldg_stream(ep);
      *reinterpret_cast<uint4*>(f + 4) = ldg_stream(ep + 4);
    } else {
      unpack8(ldg_stream(reinterpret_cast<const __nv_bfloat16*>(extra) + (long)t * lde + c), f);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += f[e];
  }
  *reinterpret_cast<uint4*>(out + (long)t * ldo + c) = pack8(acc);
}

// o_proj split-K finish (glm52/kernels/oproj_resadd.py epilogue_kernel; bench_layer.py:355):
//   out = bf16(sum_s part[s] (+ res))          fused: one rounding
//   out = bf16(bf16(sum_s part[s]) + res)      round_mid: the unfused chain's c, then add
// out32 (optional): fp32 result instead, += when accumulate (the reference's atomic acc32)
__global__ void oproj_finish_kernel(const float* __restrict__ part, long plane, int S, long ldp,
                                    const __nv_bfloat16* __restrict__ res, long ldr,
                                    __nv_bfloat16* __restrict__ out, long ldo, int N,
                                    int round_mid, float* __restrict__ out32, int accumulate,
                                    const float* __restrict__ row_scale) {
  const int t = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= N) return;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int s = 0; s < S; ++s) {
    const float* p = part + (long)s * plane + (long)t * ldp + c;
    const uint4 a = ldg_stream(p);
    const uint4 b = ldg_stream(p + 4);
    acc[0] += __uint_as_float(a.x); acc[1] += __uint_as_float(a.y);
    acc[2] += __uint_as_float(a.z); acc[3] += __uint_as_float(a.w);
    acc[4] += __uint_as_float(b.x); acc[5] += __uint_as_float(b.y);
    acc[6] += __uint_as_float(b.z); acc[7] += __uint_as_float(b.w);
  }
  if (row_scale) {  // lazy pre-norm: the row's rstd applied after the contraction
    const float rs = __ldg(row_scale + t);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= rs;
  }
  if (round_mid) {
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = round_bf(acc[e]);
  }
  if (res) {
    float r[8];
    unpack8(ldg_stream(res + (long)t * ldr + c), r);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += r[e];
  }
  if (out32) {
    float4* o = reinterpret_cast<float4*>(out32 + (long)t * ldo + c);
    if (accumulate) {
      const float4 a = o[0], b = o[1];
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    return;
  }
  *reinterpret_cast<uint4*>(out + (long)t * ldo + c) = pack8(acc);
}

// Lazy pre-norm pieces (glm52/kernels/lazy_prenorm.py:347 rstd_kernel, :75-86 fold_weight_*)
// rstd[t] = 1 / sqrt(mean(x[t]^2) + eps), fp32 over the bf16 row; one CTA per row
__global__ void __launch_bounds__(256)
    row_rstd_kernel(const __nv_bfloat16* __restrict__ x, long ldx, int N, float eps,
                    float* __restrict__ rstd) {
  const int t = blockIdx.x;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < N; c += 256 * 8) {
    float v[8];
    unpack8(ldg_stream(x + (long)t * ldx + c), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
  }
  __shared__ float red[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w];
    rstd[t] = 1.0f / sqrtf(s / (float)N + eps);
  }
}

// dst[r, c] = bf16(src[r, c] * (by_row ? w[r] : w[c]))  (the affine norm weight folded
// into a weight's K dimension: rows of a [K, N] weight, columns of an [.., N, K] one)
__global__ void fold_weight_kernel(const __nv_bfloat16* __restrict__ src,
                                   const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ dst, long rows, int cols,
                                   int by_row, long wdiv) {
  const long n = rows * (long)cols;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    const long r = i / cols;
    const int c = (int)(i - r * cols);
    const float s = __bfloat162float(w[by_row ? (r % wdiv) : c]);
    dst[i] = __float2bfloat16_rn(__bfloat162float(src[i]) * s);
  }
}

__global__ void add_kernel(const __nv_bfloat16* __restrict__ a, long lda,
                           const __nv_bfloat16* __restrict__ b, long ldb,
                           __nv_bfloat16* __restrict__ o, long ldo, int N) {
  const int m = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= N) return;
  float fa[8], fb[8];
  unpack8(ldg_stream(a + (long)m * lda + c), fa);
  unpack8(ldg_stream(b + (long)m * ldb + c), fb);
#pragma unroll
  for (int e = 0; e < 8; ++e) fa[e] += fb[e];
  *reinterpret_cast<uint4*>(o + (long)m * ldo + c) = pack8(fa);
}

__global__ void seed_kernel(__nv_bfloat16* __restrict__ o, long ldo,
                            const __nv_bfloat16* __restrict__ s, long lds, int N) {
  const int m = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= N) return;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (s) v = ldg_stream(s + (long)m * lds + c);
  *reinterpret_cast<uint4*>(o + (long)m * ldo + c) = v;
}

}  // namespace fus

using namespace fus;
typedef __nv_bfloat16 bf16;

static bool rows_ok(const void* p, long ld) { return p && aligned16(p) && ld % 8 == 0; }

extern "C" int fus_add_rmsnorm(const void* x, long ldx, const void* res, long ldr, const void* w,
                               void* h1, long ldh, void* out, long ldo, int T, int N, float eps,
                               int do_add, int do_norm, void* stream, int* status) {
  (void)status;
  if (T < 0 || N <= 0 || N % 8) return set_error(FUS_E_INVALID, "add_rmsnorm: N=%d must be a multiple of 8", N);
  if (N > kNormThreads * 8 * 8) return set_error(FUS_E_UNSUPPORTED, "add_rmsnorm: N=%d > 16384", N);
  if (!do_add && !do_norm) return FUS_OK;
  if (!rows_ok(x, ldx)) return set_error(FUS_E_INVALID, "add_rmsnorm: x rows must be 16-byte aligned");
  if (do_add && (!rows_ok(res, ldr) || (h1 && !rows_ok(h1, ldh))))
    return set_error(FUS_E_INVALID, "add_rmsnorm: residual / h1 rows must be 16-byte aligned");
  if (do_add && !do_norm && !h1) return set_error(FUS_E_INVALID, "add_rmsnorm: add_only needs h1");
  if (do_norm && (!rows_ok(out, ldo) || !w || !aligned16(w)))
    return set_error(FUS_E_INVALID, "add_rmsnorm: out / w must be 16-byte aligned");
  if (T == 0) return FUS_OK;
  const int vpt = ceil_div(N / 8, kNormThreads);
  cudaStream_t st = as_stream(stream);
#define FUS_NORM_LAUNCH(V)                                                                     \
  add_rmsnorm_kernel<V><<<T, kNormThreads, 0, st>>>(                                          \
      (const bf16*)x, ldx, (const bf16*)res, ldr, (const bf16*)w, (bf16*)h1, ldh, (bf16*)out, \
      ldo, N, eps, do_add, do_norm)
  switch (vpt) {
    case 1: FUS_NORM_LAUNCH(1); break;
    case 2: FUS_NORM_LAUNCH(2); break;
    case 3: FUS_NORM_LAUNCH(3); break;
    case 4: FUS_NORM_LAUNCH(4); break;
    default: FUS_NORM_LAUNCH(8); break;
  }
#undef FUS_NORM_LAUNCH
  return check_launch("add_rmsnorm");
}

static dim3 row_grid(int M, int N, int threads) { return dim3(ceil_div(N / 8, threads), M); }

extern "C" int fus_silu_and_mul(const void* x, long ldx, void* y, long ldy, int M, int I,
                                void* stream, int* status) {
  (void)status;
  if (M < 0 || I <= 0 || I % 8 || !rows_ok(x, ldx) || !rows_ok(y, ldy))
    return set_error(FUS_E_INVALID, "silu_and_mul: bad shape/alignment");
  if (M == 0) return FUS_OK;
  silu_and_mul_kernel<<<row_grid(M, I, 128), 128, 0, as_stream(stream)>>>(
      (const bf16*)x, ldx, (bf16*)y, ldy, I);
  return check_launch("silu_and_mul");
}

static int merge_launch(const void* y, long ld_t, long ld_k, int K, const int* pos_of,
                        const float* w, long ldw, const void* res, long ldr, const void* extra,
                        long lde, int extra_f32, void* out, long ldo, int T, int H, int round_mid,
                        void* stream, const int* flags = nullptr, const int* epoch = nullptr,
                        int W = 0, int pdl = 0, int* status = nullptr) {
  if (T < 0 || H <= 0 || H % 8 || K < 0) return set_error(FUS_E_INVALID, "merge: bad shape");
  if (K > 0 && (!y || !aligned16(y) || ld_t % 8 || ld_k % 8))
    return set_error(FUS_E_INVALID, "merge: y rows must be 16-byte aligned");
  if ((res && !rows_ok(res, ldr)) || (extra && (!aligned16(extra) || lde % 8)) ||
      !rows_ok(out, ldo))
    return set_error(FUS_E_INVALID, "merge: rows must be 16-byte aligned");
  if (T == 0) return FUS_OK;
  cudaStream_t st = as_stream(stream);
  dim3 grid = row_grid(T, H, 128);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err = cudaLaunchKernelEx(&cfg, K == 8 ? merge_kernel<8> : merge_kernel<0>,
                                       (const bf16*)y, ld_t, ld_k, K, pos_of, w, ldw,
                                       (const bf16*)res, ldr, extra, lde, extra_f32, (bf16*)out,
                                       ldo, H, round_mid, flags, epoch, W, status);
  if (err != cudaSuccess) return set_error(FUS_E_LAUNCH, "merge: %s", cudaGetErrorString(err));
  return check_launch("merge");
}

extern "C" int fus_merge(const void* y, long ld_t, long ld_k, int K, const float* w, long ldw,
                         const void* res, long ldr, const void* extra, long lde, int extra_f32,
                         void* out, long ldo, int T, int H, int round_mid, void* stream,
                         int* status) {
  (void)status;
  return merge_launch(y, ld_t, ld_k, K, nullptr, w, ldw, res, ldr, extra, lde, extra_f32, out, ldo,
                      T, H, round_mid, stream);
}

namespace fus {
int oproj_finish(const float* part, long plane, int S, long ldp, const void* res, long ldr,
                 void* out, long ldo, int T, int N, int round_mid, void* stream, int out_f32,
                 int accumulate, const float* row_scale) {
  if (T == 0) return FUS_OK;
  oproj_finish_kernel<<<row_grid(T, N, 128), 128, 0, as_stream(stream)>>>(
      part, plane, S, ldp, (const bf16*)res, ldr, out_f32 ? nullptr : (bf16*)out, ldo, N,
      round_mid, out_f32 ? (float*)out : nullptr, accumulate, row_scale);
  return check_launch("oproj_finish");
}

int merge_pos_after_flags(const void* y, long ldy, const int* pos_of, int K, const float* w,
                          long ldw, const void* res, long ldr, const void* extra, long lde,
                          int extra_f32, void* out, long ldo, int T, int H, const int* flags,
                          const int* epoch, int W, int pdl, void* stream, int* status) {
  if (!flags || !epoch || W < 1 || W > 128)
    return set_error(FUS_E_INVALID, "merge_after_flags: bad flags");
  return merge_launch(y, 0, ldy, K, pos_of, w, ldw, res, ldr, extra, lde, extra_f32, out, ldo, T,
                      H, 0, stream, flags, epoch, W, pdl, status);
}
}  // namespace fus

extern "C" int fus_merge_pos(const void* y, long ldy, const int* pos_of, int K, const float* w,
                             long ldw, const void* res, long ldr, const void* extra, long lde,
                             int extra_f32, void* out, long ldo, int T, int H, void* stream,
                             int* status) {
  (void)status;
  if (K > 0 && !pos_of) return set_error(FUS_E_INVALID, "merge_pos: pos_of is NULL");
  return merge_launch(y, 0, ldy, K, pos_of, w, ldw, res, ldr, extra, lde, extra_f32, out, ldo, T,
                      H, 0, stream);
}

extern "C" int fus_row_rstd(const void* x, long ldx, int T, int N, float eps, float* rstd,
                            void* stream, int* status) {
  (void)status;
  if (!x || !rstd || T < 0 || N <= 0 || N % 8 || ldx % 8 || !aligned16(x))
    return set_error(FUS_E_INVALID, "row_rstd: bad args");
  if (T == 0) return FUS_OK;
  row_rstd_kernel<<<T, 256, 0, as_stream(stream)>>>((const bf16*)x, ldx, N, eps, rstd);
  return check_launch("row_rstd");
}

extern "C" int fus_fold_weight(const void* src, const void* w, void* dst, long rows, int cols,
                               int by_row, long wdiv, void* stream, int* status) {
  (void)status;
  if (!src || !w || !dst || rows < 0 || cols <= 0 || (by_row && wdiv < 1))
    return set_error(FUS_E_INVALID, "fold_weight: bad args");
  const long n = rows * (long)cols;
  if (n == 0) return FUS_OK;
  long grid = (n + 255) / 256;
  if (grid > 148L * 32) grid = 148L * 32;
  fold_weight_kernel<<<(int)grid, 256, 0, as_stream(stream)>>>((const bf16*)src, (const bf16*)w,
                                                               (bf16*)dst, rows, cols, by_row,
                                                               by_row ? wdiv : 1);
  return check_launch("fold_weight");
}

extern "C" int fus_scale_sum_planes(const float* partial, int nsplit, long plane, int T, int N,
                                    const float* row_scale, float* out, long ldo, void* stream,
                                    int* status) {
  (void)status;
  if (!partial || !out || T < 0 || N <= 0 || N % 8 || nsplit < 1 || ldo % 4)
    return set_error(FUS_E_INVALID, "scale_sum_planes: bad args");
  return oproj_finish(partial, plane, nsplit, N, nullptr, 0, out, ldo, T, N, 0, stream, 1, 0,
                      row_scale);
}

extern "C" int fus_add(const void* a, long lda, const void* b, long ldb, void* o, long ldo, int M,
                       int N, void* stream, int* status) {
  (void)status;
  if (M < 0 || N <= 0 || N % 8 || !rows_ok(a, lda) || !rows_ok(b, ldb) || !rows_ok(o, ldo))
    return set_error(FUS_E_INVALID, "add: bad shape/alignment");
  if (M == 0) return FUS_OK;
  add_kernel<<<row_grid(M, N, 128), 128, 0, as_stream(stream)>>>((const bf16*)a, lda,
                                                                 (const bf16*)b, ldb, (bf16*)o,
                                                                 ldo, N);
  return check_launch("add");
}

extern "C" int fus_seed(void* o, long ldo, const void* src, long lds, int M, int N, int from_src,
                        void* stream, int* status) {
  (void)status;
  if (M < 0 || N <= 0 || N % 8 || !rows_ok(o, ldo) || (from_src && !rows_ok(src, lds)))
    return set_error(FUS_E_INVALID, "seed: bad shape/alignment");
  if (M == 0) return FUS_OK;
  seed_kernel<<<row_grid(M, N, 128), 128, 0, as_stream(stream)>>>(
      (bf16*)o, ldo, from_src ? (const bf16*)src : nullptr, lds, N);
  return check_launch("seed");
}
