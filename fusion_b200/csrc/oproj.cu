// o_proj GEMM + ResAdd1 (glm52/kernels/oproj_resadd.py; the layer chain of
// glm52/bench/bench_layer.py:399-415): h1 = a @ W_o + h_in with the reference's two
// numerics, fused (one bf16 rounding of the fp32 sum, bench_layer.py:355) and unfused
// (c = bf16(a @ W_o), then h1 = bf16(c + h_in): oproj_resadd.py epilogue_kernel).
//
// The weight is K-major here, w [N, K] (the reference's w_o [K, N] transposed once at
// load): its rows are the MMA's M side like the expert weights. Two shapes:
//   decode  (T <= 64): N/128 weight tiles are too few CTAs for K = 32768, so K is split
//           into fp32 partial planes (FUS_EPI_F32) summed in fixed order by one finish
//           kernel that also adds the residual (deterministic; no atomics)
//   prefill (T > 64):  the grouped GEMM on one dense group with the residual added in
//           its epilogue (fused) or a bf16 GEMM then fus_add (unfused)
#include "common.cuh"
#include "host_util.h"

namespace {

int oproj_block_n(int T) {
  return T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
}

// K splits for the decode shape: about two CTAs per SM, at least 8 k-steps each
int oproj_ksplit(int T, int N, int K) {
  if (T > 64) return 1;
  const int tiles = N / 128;
  const int ksteps = K / 64;
  int s = (2 * fus::num_sms() + tiles - 1) / tiles;
  if (s > ksteps / 8) s = ksteps / 8;
  return s < 1 ? 1 : s;
}

}  // namespace

using namespace fus;

extern "C" size_t fus_oproj_workspace(int T, int N, int K, int fuse) {
  if (T <= 0 || N <= 0 || K <= 0) return 0;
  const int S = oproj_ksplit(T, N, K);
  if (S > 1 || T <= 64) return (size_t)S * T * N * 4 + 256;
  return fuse ? 256 : (size_t)T * N * 2 + 256;
}

extern "C" int fus_oproj_resadd(const void* a, long lda, const void* w, int T, int N, int K,
                                const void* res, long ldr, void* out, long ldo, int fuse,
                                void* workspace, size_t ws_bytes, void* stream, int* status) {
  if (!a || !w || !out || T < 0 || N <= 0 || N % 128 || K <= 0 || K % 64 || lda % 8 ||
      ldo % 8 || (res && ldr % 8))
    return set_error(FUS_E_INVALID, "oproj: bad args (N %% 128, K %% 64, 16-byte rows)");
  if (T == 0) return FUS_OK;
  const size_t need = fus_oproj_workspace(T, N, K, fuse);
  if (ws_bytes < need || (need > 256 && !workspace))
    return set_error(FUS_E_INVALID, "oproj: workspace of %zu bytes required", need);
  uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) &
                                           ~uintptr_t(255));
  const int bn = oproj_block_n(T);
  const int S = oproj_ksplit(T, N, K);
  fus_gemm_group g = {};
  g.w = w;
  g.n_experts = 1;
  g.x = a;
  g.ldx = lda;
  g.x_rows = T;
  g.max_blocks = (T + bn - 1) / bn;
  g.row_limit = T;
  g.flags = T <= bn ? FUS_GEMM_W_STREAM : 0;
  int rc;
  if (T <= 64) {
    float* part = reinterpret_cast<float*>(ws);
    g.out = part;
    g.ldo = N;
    if ((rc = fus_grouped_gemm(&g, 1, N, K, 1, FUS_EPI_F32, bn, S, (long)T * N, stream, status)))
      return rc;
    return oproj_finish(part, (long)T * N, S, N, res, ldr, out, ldo, T, N, fuse ? 0 : 1, stream);
  }
  if (fuse) {
    g.out = out;
    g.ldo = ldo;
    g.res = res;
    g.ldr = ldr;
    return fus_grouped_gemm(&g, 1, N, K, 1, FUS_EPI_BF16, bn, 1, 0, stream, status);
  }
  if (!res) {  // no residual: c is the output
    g.out = out;
    g.ldo = ldo;
    return fus_grouped_gemm(&g, 1, N, K, 1, FUS_EPI_BF16, bn, 1, 0, stream, status);
  }
  void* c = ws;  // the unfused chain materialises c = bf16(a @ W_o)
  g.out = c;
  g.ldo = N;
  if ((rc = fus_grouped_gemm(&g, 1, N, K, 1, FUS_EPI_BF16, bn, 1, 0, stream, status))) return rc;
  return fus_add(c, N, res, ldr, out, ldo, T, N, stream, status);
}

extern "C" size_t fus_oproj_f32_workspace(int T, int N, int K) {
  if (T <= 0 || N <= 0 || K <= 0) return 0;
  return (size_t)oproj_ksplit(T, N, K) * T * N * 4 + 256;
}

extern "C" int fus_oproj_gemm_f32(const void* a, long lda, const void* w, int T, int N, int K,
                                  const void* res, long ldr, float* acc32, long ldc,
                                  int accumulate, void* workspace, size_t ws_bytes, void* stream,
                                  int* status) {
  if (!a || !w || !acc32 || T < 0 || N <= 0 || N % 128 || K <= 0 || K % 64 || lda % 8 ||
      ldc % 4 || (res && ldr % 8))
    return set_error(FUS_E_INVALID, "oproj_f32: bad args");
  if (T == 0) return FUS_OK;
  const size_t need = fus_oproj_f32_workspace(T, N, K);
  if (!workspace || ws_bytes < need) return set_error(FUS_E_INVALID, "oproj_f32: workspace of %zu bytes required", need);
  float* part = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) &
                                         ~uintptr_t(255));
  const int bn = oproj_block_n(T);
  const int S = oproj_ksplit(T, N, K);
  fus_gemm_group g = {};
  g.w = w;
  g.n_experts = 1;
  g.x = a;
  g.ldx = lda;
  g.x_rows = T;
  g.max_blocks = (T + bn - 1) / bn;
  g.row_limit = T;
  g.flags = T <= bn ? FUS_GEMM_W_STREAM : 0;
  g.out = part;
  g.ldo = N;
  int rc;
  if ((rc = fus_grouped_gemm(&g, 1, N, K, 1, FUS_EPI_F32, bn, S, (long)T * N, stream, status)))
    return rc;
  return oproj_finish(part, (long)T * N, S, N, res, ldr, acc32, ldc, T, N, 0, stream, 1,
                      accumulate);
}

extern "C" int fus_oproj_finish(const float* acc32, long ldc, const void* res, long ldr,
                                void* out, long ldo, int T, int N, void* stream, int* status) {
  (void)status;
  if (!acc32 || !out || T < 0 || N <= 0 || N % 8 || ldc % 4 || ldo % 8 || (res && ldr % 8))
    return set_error(FUS_E_INVALID, "oproj_finish: bad args");
  return oproj_finish(acc32, 0, 1, ldc, res, ldr, out, ldo, T, N, 0, stream);
}
