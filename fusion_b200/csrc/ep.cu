// Expert-parallel dispatch and combine helpers (the exchange itself is NCCL
// all_to_all through torch.distributed).
//
// The reference runs on one GPU (log/LOG-00-plan-and-filter.md:41, "Single GPU, no
// TP/EP"); expert parallelism is new here. Rank g owns experts [g*E_loc, (g+1)*E_loc).
// For every (token, slot) pair of the local top-k:
//   plan   : dest = expert / E_loc, local expert = expert % E_loc, per-rank pair counts
//   pack   : rows[p] = x2[send_ids[p] / div], leid_out[p] = leid[send_ids[p]]
//            (send_ids = the pairs stably sorted by destination rank, fus_moe_align
//             with block_m = 1 over `dest`)
//   unpack : y[send_ids[p]] = rows[p]       (returned expert outputs back to slot order)
#include "common.cuh"
#include "host_util.h"

namespace fus {

constexpr int kEpMaxRanks = 64;

__global__ void __launch_bounds__(1024)
    ep_plan_kernel(const int* __restrict__ topi, int R, int E_loc, int W, int* __restrict__ dest,
                   int* __restrict__ leid, int* __restrict__ counts, int* status) {
  __shared__ int cnt[kEpMaxRanks];
  for (int i = threadIdx.x; i < W; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const int e = topi[i];
    const int d = e / E_loc;
    if (e < 0 || d >= W) {
      raise_status(status, FUS_ERR_BAD_EXPERT);
      dest[i] = 0;
      leid[i] = 0;
      continue;
    }
    dest[i] = d;
    leid[i] = e - d * E_loc;
    atomicAdd(cnt + d, 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < W; i += blockDim.x) counts[i] = cnt[i];
}

// one warp per row
__global__ void ep_pack_kernel(const __nv_bfloat16* __restrict__ x, long ldx, int H,
                               const int* __restrict__ send_ids, int n, int div,
                               const int* __restrict__ leid, __nv_bfloat16* __restrict__ rows,
                               long ldr, int* __restrict__ leid_out) {
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n; p += warps) {
    const int id = __ldg(send_ids + p);
    const uint4* s = reinterpret_cast<const uint4*>(x + (long)(id / div) * ldx);
    uint4* d = reinterpret_cast<uint4*>(rows + (long)p * ldr);
    warp_copy_row(d, s, H >> 3, lane);
    if (lane == 0 && leid) leid_out[p] = __ldg(leid + id);
  }
}

__global__ void ep_unpack_kernel(const __nv_bfloat16* __restrict__ rows, long ldr, int H,
                                 const int* __restrict__ send_ids, int n,
                                 __nv_bfloat16* __restrict__ y, long ldy) {
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n; p += warps) {
    const int id = __ldg(send_ids + p);
    const uint4* s = reinterpret_cast<const uint4*>(rows + (long)p * ldr);
    uint4* d = reinterpret_cast<uint4*>(y + (long)id * ldy);
    warp_copy_row(d, s, H >> 3, lane);
  }
}

// one CTA: slots by a stable rank per destination, then one warp per used slot copies
__global__ void __launch_bounds__(1024)
    ep_dispatch_small_kernel(const __nv_bfloat16* __restrict__ x, long ldx, int H,
                             const int* __restrict__ topi, int R, int topk, int E_loc, int W,
                             int S, __nv_bfloat16* __restrict__ rows, long ldr,
                             int* __restrict__ leid_out, int* __restrict__ slot_of_pair,
                             int* status) {
  __shared__ int dst_s[1024];
  __shared__ int slot_s[1024];
  for (int i = threadIdx.x; i < W * S; i += blockDim.x) leid_out[i] = -1;
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const int e = topi[i];
    int d = e / E_loc;
    if (e < 0 || d >= W) {
      raise_status(status, FUS_ERR_BAD_EXPERT);
      d = -1;
    }
    dst_s[i] = d;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const int d = dst_s[i];
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += dst_s[j] == d;
    const int slot = d < 0 || rank >= S ? -1 : d * S + rank;
    if (d >= 0 && rank >= S) raise_status(status, FUS_ERR_CAPACITY);
    slot_s[i] = slot;
    slot_of_pair[i] = slot < 0 ? 0 : slot;
    if (slot >= 0) leid_out[slot] = topi[i] - d * E_loc;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < R; i += blockDim.x >> 5) {
    const int slot = slot_s[i];
    if (slot < 0) continue;
    const uint4* s = reinterpret_cast<const uint4*>(x + (long)(i / topk) * ldx);
    uint4* d = reinterpret_cast<uint4*>(rows + (long)slot * ldr);
    warp_copy_row(d, s, H >> 3, lane);
  }
}

static int row_grid(int n) {
  int g = ceil_div(n, 8);
  const int cap = num_sms() * 8;
  return g < 1 ? 1 : (g > cap ? cap : g);
}

}  // namespace fus

using namespace fus;

extern "C" int fus_ep_plan(const int* topi, int R, int E_loc, int W, int* dest, int* leid,
                           int* counts, void* stream, int* status) {
  if (!topi || !dest || !leid || !counts || R < 0 || E_loc < 1 || W < 1 || W > kEpMaxRanks)
    return set_error(FUS_E_INVALID, "ep_plan: bad args");
  ep_plan_kernel<<<1, 1024, 0, as_stream(stream)>>>(topi, R, E_loc, W, dest, leid, counts, status);
  return check_launch("ep_plan");
}

extern "C" int fus_ep_pack(const void* x, long ldx, int H, const int* send_ids, int n, int div,
                           const int* leid, void* rows, long ldr, int* leid_out, void* stream,
                           int* status) {
  (void)status;
  if (!x || !send_ids || !rows || n < 0 || div < 1 || H <= 0 || H % 8 || ldx % 8 || ldr % 8 ||
      !aligned16(x) || !aligned16(rows) || (leid && !leid_out))
    return set_error(FUS_E_INVALID, "ep_pack: bad args");
  if (n == 0) return FUS_OK;
  ep_pack_kernel<<<row_grid(n), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)x, ldx, H, send_ids, n, div, leid, (__nv_bfloat16*)rows, ldr, leid_out);
  return check_launch("ep_pack");
}

extern "C" int fus_ep_unpack(const void* rows, long ldr, int H, const int* send_ids, int n,
                             void* y, long ldy, void* stream, int* status) {
  (void)status;
  if (!rows || !send_ids || !y || n < 0 || H <= 0 || H % 8 || ldr % 8 || ldy % 8 ||
      !aligned16(rows) || !aligned16(y))
    return set_error(FUS_E_INVALID, "ep_unpack: bad args");
  if (n == 0) return FUS_OK;
  ep_unpack_kernel<<<row_grid(n), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)rows, ldr, H, send_ids, n, (__nv_bfloat16*)y, ldy);
  return check_launch("ep_unpack");
}

extern "C" int fus_ep_dispatch_small(const void* x, long ldx, int H, const int* topi, int T,
                                     int topk, int E_loc, int W, int S, void* rows, long ldr,
                                     int* leid_out, int* slot_of_pair, void* stream, int* status) {
  const int R = T * topk;
  if (!x || !topi || !rows || !leid_out || !slot_of_pair || T < 0 || topk < 1 || E_loc < 1 ||
      W < 1 || W > kEpMaxRanks || S < R || H <= 0 || H % 8 || ldx % 8 || ldr % 8 ||
      !aligned16(x) || !aligned16(rows))
    return set_error(FUS_E_INVALID, "ep_dispatch_small: bad args");
  if (R > 1024) return set_error(FUS_E_UNSUPPORTED, "ep_dispatch_small: T*topk=%d > 1024", R);
  ep_dispatch_small_kernel<<<1, 1024, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)x, ldx, H, topi, R, topk, E_loc, W, S, (__nv_bfloat16*)rows, ldr,
      leid_out, slot_of_pair, status);
  return check_launch("ep_dispatch_small");
}
