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

// ---- deduplicated dispatch (prefill): one row per (token, destination rank) ----------
// keys[t*W + d] = d when token t has at least one expert on rank d, else -1 (skipped by
// the stable sort that orders the send rows); counts[d] = rows for rank d, counts[W + d] =
// (token, slot) pairs for rank d.
__global__ void ep_plan_dedup_kernel(const int* __restrict__ topi, int T, int K, int E_loc, int W,
                                     int* __restrict__ keys, int* __restrict__ counts,
                                     int* status) {
  __shared__ int cnt[2 * kEpMaxRanks];
  for (int i = threadIdx.x; i < 2 * W; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    uint64_t mask = 0;
    for (int k = 0; k < K; ++k) {
      const int e = __ldg(topi + (long)t * K + k);
      const int d = e / E_loc;
      if (e < 0 || d >= W) {
        raise_status(status, FUS_ERR_BAD_EXPERT);
        continue;
      }
      mask |= 1ull << d;
      atomicAdd(cnt + W + d, 1);
    }
    for (int d = 0; d < W; ++d) {
      const bool on = (mask >> d) & 1ull;
      keys[(long)t * W + d] = on ? d : -1;
      if (on) atomicAdd(cnt + d, 1);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * W; i += blockDim.x)
    if (cnt[i]) atomicAdd(counts + i, cnt[i]);
}

// one warp per send row p = (t, d): the token's row, and per top-k slot k its local
// expert when slot k's expert lives on d (else -1), plus, as requested:
//   ret_out[p*K + k]: where the owner must put slot k's expert row in what it returns to
//     this rank = the pair's index among this rank's pairs for d (pair_pos = each pair's
//     position in the pairs stably sorted by destination, counts[W + d'] = pairs for d')
//   w_out[p*K + k] (weight, 0 off d) and pos[t*K + k] = p for the first slot of t on d,
//     zero_row for its other slots: the partial-sum combine, where a merge over the K
//     positions with unit weights adds each returned partial row exactly once
__global__ void ep_pack_dedup_kernel(const __nv_bfloat16* __restrict__ x, long ldx, int H,
                                     const int* __restrict__ send_ids, int n, int W,
                                     const int* __restrict__ topi, const float* __restrict__ topw,
                                     int K, int E_loc, const int* __restrict__ pair_pos,
                                     const int* __restrict__ counts,
                                     __nv_bfloat16* __restrict__ rows, long ldr,
                                     int* __restrict__ leid_out, int* __restrict__ ret_out,
                                     float* __restrict__ w_out, int* __restrict__ pos,
                                     int zero_row) {
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n; p += warps) {
    const int id = __ldg(send_ids + p);
    const int t = id / W, d = id - t * W;
    const uint4* s = reinterpret_cast<const uint4*>(x + (long)t * ldx);
    warp_copy_row(reinterpret_cast<uint4*>(rows + (long)p * ldr), s, H >> 3, lane);
    const int e = lane < K ? __ldg(topi + (long)t * K + lane) : -1;
    const bool mine = lane < K && e >= 0 && e / E_loc == d;
    const unsigned on = __ballot_sync(0xffffffffu, mine);
    int base = 0;  // pairs this rank sends to ranks before d
    if (ret_out)
      for (int j = lane; j < d; j += 32) base += __ldg(counts + W + j);
    base = __reduce_add_sync(0xffffffffu, base);
    if (lane < K) {
      leid_out[(long)p * K + lane] = mine ? e - d * E_loc : -1;
      if (ret_out) ret_out[(long)p * K + lane] = mine ? __ldg(pair_pos + (long)t * K + lane) - base : -1;
      if (w_out) w_out[(long)p * K + lane] = mine ? __ldg(topw + (long)t * K + lane) : 0.f;
      if (pos && mine) pos[(long)t * K + lane] = (__ffs(on) - 1 == lane) ? p : zero_row;
    }
  }
}

// owner side: the w2 row map that writes every received pair's expert row straight into
// the return buffer. Entry x of the dispatch layout holds flat slot f = i*K + j of
// received row i; row i came from source s (row_prefix[s] <= i < row_prefix[s + 1]) and
// its row goes to pair_prefix[s] + ret_idx[f]. Pads (f >= n*K) stay past every row.
// Only the first *ntp entries (the padded total) of the layout are written by moe_align;
// entries past it are not read and map to the pad row n*K.
__global__ void ep_return_rowmap_kernel(const int* __restrict__ sorted_ids, int cap,
                                        const int* __restrict__ ntp,
                                        const int* __restrict__ ret_idx, int K, int nK,
                                        const int* __restrict__ row_prefix,
                                        const int* __restrict__ pair_prefix, int W,
                                        int* __restrict__ rowmap, int* status) {
  const int used = ntp ? min(cap, __ldg(ntp)) : cap;
  for (int x = blockIdx.x * blockDim.x + threadIdx.x; x < cap; x += gridDim.x * blockDim.x) {
    if (x >= used) {
      rowmap[x] = nK;
      continue;
    }
    const int f = __ldg(sorted_ids + x);
    int out = f < nK ? -1 : f;
    if (f < 0) {
      raise_status(status, FUS_ERR_CAPACITY);
      out = nK;
    } else if (f < nK) {
      const int i = f / K;
      int s = 0;
      while (s + 1 < W && __ldg(row_prefix + s + 1) <= i) ++s;
      const int ri = __ldg(ret_idx + f);
      const int lim = __ldg(pair_prefix + s + 1) - __ldg(pair_prefix + s);
      if (ri < 0 || ri >= lim) {
        raise_status(status, FUS_ERR_CAPACITY);
        out = nK;  // dropped rather than written out of place
      } else {
        out = __ldg(pair_prefix + s) + ri;
      }
    }
    rowmap[x] = out;
  }
}

// out[i] = bf16(sum over slots j with leid[i*K + j] >= 0 of w[i*K + j] * y[i*K + j]),
// fp32 accumulation in slot order (the owner's partial of one (token, source) row)
__global__ void ep_partial_sum_kernel(const __nv_bfloat16* __restrict__ y, long ldy, int H,
                                      const int* __restrict__ leid, const float* __restrict__ w,
                                      int K, __nv_bfloat16* __restrict__ out, long ldo) {
  const int i = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= H) return;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int j = 0; j < K; ++j) {
    if (__ldg(leid + (long)i * K + j) < 0) continue;
    const float wj = __ldg(w + (long)i * K + j);
    float f[8];
    unpack8(ldg_stream(y + ((long)i * K + j) * ldy + c), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += wj * f[e];
  }
  *reinterpret_cast<uint4*>(out + (long)i * ldo + c) = pack8(acc);
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

extern "C" int fus_ep_plan_dedup(const int* topi, int T, int K, int E_loc, int W, int* keys,
                                 int* counts, void* stream, int* status) {
  if (!topi || !keys || !counts || T < 0 || K < 1 || E_loc < 1 || W < 1 || W > kEpMaxRanks)
    return set_error(FUS_E_INVALID, "ep_plan_dedup: bad args");
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(counts, 0, sizeof(int) * 2 * W, st) != cudaSuccess)
    return set_error(FUS_E_LAUNCH, "ep_plan_dedup: memset");
  if (T == 0) return FUS_OK;
  int grid = ceil_div(T, 256);
  if (grid > num_sms()) grid = num_sms();
  ep_plan_dedup_kernel<<<grid, 256, 0, st>>>(topi, T, K, E_loc, W, keys, counts, status);
  return check_launch("ep_plan_dedup");
}

extern "C" int fus_ep_pack_dedup(const void* x, long ldx, int H, const int* send_ids, int n,
                                 int W, const int* topi, const float* topw, int K, int E_loc,
                                 const int* pair_pos, const int* counts, void* rows, long ldr,
                                 int* leid_out, int* ret_out, float* w_out, int* pos,
                                 int zero_row, void* stream, int* status) {
  (void)status;
  if (!x || !send_ids || !topi || !rows || !leid_out || n < 0 || W < 1 || W > kEpMaxRanks ||
      K < 1 || K > 32 || E_loc < 1 || H <= 0 || H % 8 || ldx % 8 || ldr % 8 || !aligned16(x) ||
      !aligned16(rows) || (ret_out && (!pair_pos || !counts)) || (w_out && !topw) ||
      (!w_out != !pos))
    return set_error(FUS_E_INVALID, "ep_pack_dedup: bad args");
  if (n == 0) return FUS_OK;
  ep_pack_dedup_kernel<<<row_grid(n), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)x, ldx, H, send_ids, n, W, topi, topw, K, E_loc, pair_pos, counts,
      (__nv_bfloat16*)rows, ldr, leid_out, ret_out, w_out, pos, zero_row);
  return check_launch("ep_pack_dedup");
}

extern "C" int fus_ep_return_rowmap(const int* sorted_ids, int cap, const int* ntp,
                                    const int* ret_idx, int n,
                                    int K, const int* row_prefix, const int* pair_prefix, int W,
                                    int* rowmap, void* stream, int* status) {
  if (!sorted_ids || !ret_idx || !row_prefix || !pair_prefix || !rowmap || cap < 0 || n < 0 ||
      K < 1 || W < 1 || W > kEpMaxRanks)
    return set_error(FUS_E_INVALID, "ep_return_rowmap: bad args");
  if (cap == 0) return FUS_OK;
  int grid = ceil_div(cap, 256);
  if (grid > 4 * num_sms()) grid = 4 * num_sms();
  ep_return_rowmap_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      sorted_ids, cap, ntp, ret_idx, K, n * K, row_prefix, pair_prefix, W, rowmap, status);
  return check_launch("ep_return_rowmap");
}

extern "C" int fus_ep_partial_sum(const void* y, long ldy, int H, const int* leid, const float* w,
                                  int n, int K, void* out, long ldo, void* stream, int* status) {
  (void)status;
  if (!y || !leid || !w || !out || n < 0 || K < 1 || H <= 0 || H % 8 || ldy % 8 || ldo % 8 ||
      !aligned16(y) || !aligned16(out))
    return set_error(FUS_E_INVALID, "ep_partial_sum: bad args");
  if (n == 0) return FUS_OK;
  if (n > 65535) return set_error(FUS_E_UNSUPPORTED, "ep_partial_sum: %d rows > 65535", n);
  dim3 grid(ceil_div(H / 8, 128), n);
  ep_partial_sum_kernel<<<grid, 128, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)y, ldy, H, leid, w, K, (__nv_bfloat16*)out, ldo);
  return check_launch("ep_partial_sum");
}
