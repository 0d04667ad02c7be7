// Seeded synthetic inputs that are bit-identical on the GPU and on the host.
//
// Element i of stream `seed` is  mean + std * z_i  with
//   z_i = (sum of 12 uniform 16-bit draws - 12*65535/2) / 65536
// (Irwin-Hall approximation of a standard normal: mean 0, variance ~1, tails cut at
// +-6). The draws come from three splitmix64 hashes of (seed, 3i+j). Every step is an
// integer operation or a single IEEE-rounded fp32 multiply/add (no fused multiply-add),
// so host and device produce the same bits, and any slice (one expert's weights) can
// be regenerated on its own from its element offset.
#include <string.h>

#include <thread>
#include <vector>

#include "common.cuh"
#include "host_util.h"

namespace fus {

__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ inline int irwin_hall12(uint64_t key, uint64_t i) {
  int sum = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint64_t h = mix64(key + (3 * i + (uint64_t)j) * 0x9E3779B97F4A7C15ull);
    sum += (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) +
           (int)(h >> 48);
  }
  return sum - 393210;  // 12 * 65535 / 2
}

__host__ __device__ inline uint64_t stream_key(uint64_t seed) {
  return mix64(seed + 0x9E3779B97F4A7C15ull);
}

__global__ void synth_kernel(void* dst, int dtype, long n, long offset, uint64_t key, float mean,
                             float stdv) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    const float z = (float)irwin_hall12(key, (uint64_t)(offset + i)) * (1.0f / 65536.0f);
    const float v = __fadd_rn(__fmul_rn(z, stdv), mean);
    if (dtype == 0)
      reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<float*>(dst)[i] = v;
  }
}

static inline uint16_t host_f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);  // round to nearest even (inputs are finite)
  return (uint16_t)(u >> 16);
}

}  // namespace fus

using namespace fus;

extern "C" int fus_synth_fill(void* dst, int dtype, long n, long offset, unsigned long long seed,
                              float mean, float std, void* stream) {
  if (!dst || n < 0 || (dtype != 0 && dtype != 1)) return set_error(FUS_E_INVALID, "synth: bad args");
  if (n == 0) return FUS_OK;
  long grid = (n + 255) / 256;
  const long cap = (long)num_sms() * 16;
  if (grid > cap) grid = cap;
  synth_kernel<<<(int)grid, 256, 0, as_stream(stream)>>>(dst, dtype, n, offset, stream_key(seed),
                                                         mean, std);
  return check_launch("synth_fill");
}

extern "C" void fus_synth_fill_host(void* dst, int dtype, long n, long offset,
                                    unsigned long long seed, float mean, float std) {
  if (!dst || n <= 0) return;
  const uint64_t key = stream_key(seed);
  auto work = [=](long b, long e) {
    for (long i = b; i < e; ++i) {
      volatile float z = (float)irwin_hall12(key, (uint64_t)(offset + i)) * (1.0f / 65536.0f);
      volatile float p = z * std;  // volatile: one rounding per operation, never an FMA
      const float v = p + mean;
      if (dtype == 0)
        reinterpret_cast<uint16_t*>(dst)[i] = host_f2bf(v);
      else
        reinterpret_cast<float*>(dst)[i] = v;
    }
  };
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (n < (1L << 16)) nt = 1;
  if (nt > 64) nt = 64;
  std::vector<std::thread> th;
  const long chunk = (n + nt - 1) / nt;
  for (unsigned t = 0; t < nt; ++t) {
    const long b = t * chunk, e = b + chunk < n ? b + chunk : n;
    if (b >= e) break;
    th.emplace_back(work, b, e);
  }
  for (auto& x : th) x.join();
}
