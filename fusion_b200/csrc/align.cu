// Dispatch layout (sglang moe_align_block_size) and row permutation, on the device.
//
// Reference: glm52/reference.py:85-128 (a host loop over experts with .tolist() syncs;
// bench_layer.py:14-17 keeps it out of the timed region). Contract in
// glm52/kernels/REFERENCES.md:41-51:
//   sorted_token_ids : flat (token*topk+k) indices, stably sorted by expert, each
//                      expert's run padded to a multiple of block_m with `numel`
//   expert_ids[b]    : expert owning block b
//   ntp[0]           : padded total
//
// Here it is a counting sort. A stable rank of every element among the elements with
// the same expert and a smaller flat index is built chunk by chunk: inside a warp with
// __match_any_sync (rank = peers below me), across the 32 warps of a chunk with a
// per-expert exclusive scan over warp counts. Then
//   pos(i) = start[expert(i)] + rank(i),
// which reproduces torch.argsort(stable=True) + the padded placement bit for bit.
// Small inputs run in one CTA (one launch); large inputs use three launches
// (per-chunk ranks + histograms, one-CTA scan, scatter) with a global workspace.
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace fus {

constexpr int kAlignThreads = 1024;
constexpr int kAlignWarps = kAlignThreads / 32;
constexpr int kAlignSmallMax = 8192;   // elements handled by the single-CTA path
constexpr int kAlignMaxE = 512;

// Ranks the (up to 1024) elements [base, base+1024) of `ids` against each other and
// against earlier chunks (`cursor[e]` = elements of expert e already ranked).
// wcnt is [32][E] shared scratch. Returns (through rank_out) the stable rank, -1 for
// elements that are out of range, holes (negative ids) or carry an invalid expert.
__device__ void rank_chunk(const int* __restrict__ ids, int base, int numel, int E, int* wcnt,
                           int* cursor, int& my_e, int& my_rank, int* status) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i = base + tid;
  int e = -1;
  if (i < numel) {
    e = ids[i];
    if (e >= E) {
      raise_status(status, FUS_ERR_BAD_EXPERT);
      e = -1;
    } else if (e < 0) {
      e = -1;  // a hole: no pair at this flat index (expert-parallel slot buffers)
    }
  }
  for (int j = tid; j < kAlignWarps * E; j += kAlignThreads) wcnt[j] = 0;
  __syncthreads();
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int wr = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && wr == 0) wcnt[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int x = tid; x < E; x += kAlignThreads) {
    int run = cursor[x];
    for (int w = 0; w < kAlignWarps; ++w) {
      const int c = wcnt[w * E + x];
      wcnt[w * E + x] = run;
      run += c;
    }
    cursor[x] = run;
  }
  __syncthreads();
  my_e = e;
  my_rank = e >= 0 ? wcnt[warp * E + e] + wr : -1;
  __syncthreads();  // wcnt is cleared by the next chunk
}

// Position of an expert's q-th pair (stable order) inside its padded region. Reference
// layout: start + q, pads after the last pair. Balanced layout (FUS_ALIGN_BALANCED):
// the c pairs are spread evenly over the region's nb = ceil(c / block_m) blocks,
// pb = ceil(c / nb) per block with the block's pads after them, so no block holds only
// a few stragglers (each block streams the expert's full weights through the GEMM).
__device__ __forceinline__ int place_pair(int start, int q, int c, int block_m, int balanced) {
  if (!balanced) return start + q;
  const int nb = (c + block_m - 1) / block_m;
  const int pb = (c + nb - 1) / nb;
  return start + (q / pb) * block_m + (q % pb);
}

// Per-expert padded placement from counts (cnt[e]); writes start[e], ntp, expert_ids
// and the pad sentinels. Needs E <= blockDim.x * 1 handled by a strided loop + scan.
__device__ void place_experts(const int* cnt, int* start, int E, int block_m, int numel,
                              int* sorted_ids, int sorted_cap, int* expert_ids, int blocks_cap,
                              int* ntp, int* scan_tmp, int* status, int balanced) {
  const int tid = threadIdx.x;
  // exclusive scan of padded counts (E <= 1024: one element per thread)
  int padded = 0;
  if (tid < E) padded = (cnt[tid] + block_m - 1) / block_m * block_m;
  scan_tmp[tid] = padded;
  __syncthreads();
  for (int off = 1; off < kAlignThreads; off <<= 1) {
    const int v = tid >= off ? scan_tmp[tid - off] : 0;
    __syncthreads();
    scan_tmp[tid] += v;
    __syncthreads();
  }
  const int incl = scan_tmp[tid];
  const int total = scan_tmp[kAlignThreads - 1];
  if (tid < E) start[tid] = incl - padded;
  if (tid == 0) {
    ntp[0] = total;
    if (total > sorted_cap || total / block_m > blocks_cap) raise_status(status, FUS_ERR_CAPACITY);
  }
  if (tid < E && padded > 0) {
    const int s = incl - padded;
    for (int b = s / block_m; b < (s + padded) / block_m; ++b)
      if (b < blocks_cap) expert_ids[b] = tid;
    const int c = cnt[tid];
    if (!balanced) {
      for (int p = s + c; p < s + padded; ++p)
        if (p < sorted_cap) sorted_ids[p] = numel;
    } else {
      const int nb = padded / block_m;
      const int pb = (c + nb - 1) / nb;
      for (int b = 0; b < nb; ++b) {
        const int live = max(0, min(pb, c - b * pb));
        for (int p = s + b * block_m + live; p < s + (b + 1) * block_m; ++p)
          if (p < sorted_cap) sorted_ids[p] = numel;
      }
    }
  }
  __syncthreads();
}

__device__ void align_small_body(const int* __restrict__ ids, int numel, int E, int block_m,
                                 int* __restrict__ sorted_ids, int sorted_cap,
                                 int* __restrict__ expert_ids, int blocks_cap,
                                 int* __restrict__ ntp, int* __restrict__ pos_of, int balanced,
                                 int* status) {
  extern __shared__ int sm[];
  int* wcnt = sm;                            // [32][E]
  int* cursor = wcnt + kAlignWarps * E;      // [E]
  int* start = cursor + E;                   // [E]
  int* scan_tmp = start + E;                 // [1024]
  int* rank = scan_tmp + kAlignThreads;      // [numel] (stable rank)
  int* eid = rank + kAlignSmallMax;          // [numel]
  for (int x = threadIdx.x; x < E; x += kAlignThreads) cursor[x] = 0;
  __syncthreads();
  for (int base = 0; base < numel; base += kAlignThreads) {
    int e, r;
    rank_chunk(ids, base, numel, E, wcnt, cursor, e, r, status);
    if (base + (int)threadIdx.x < numel) {
      rank[base + threadIdx.x] = r;
      eid[base + threadIdx.x] = e;
    }
  }
  __syncthreads();
  place_experts(cursor, start, E, block_m, numel, sorted_ids, sorted_cap, expert_ids, blocks_cap,
                ntp, scan_tmp, status, balanced);
  for (int i = threadIdx.x; i < numel; i += kAlignThreads) {
    const int e = eid[i];
    if (e < 0) continue;
    const int p = place_pair(start[e], rank[i], cursor[e], block_m, balanced);
    if (p < sorted_cap) sorted_ids[p] = i;
    if (pos_of) pos_of[i] = p;
  }
}

__global__ void __launch_bounds__(kAlignThreads)
    align_small_kernel(const int* __restrict__ ids, int numel, int E, int block_m,
                       int* __restrict__ sorted_ids, int sorted_cap, int* __restrict__ expert_ids,
                       int blocks_cap, int* __restrict__ ntp, int* __restrict__ pos_of,
                       int balanced, int* status) {
  align_small_body(ids, numel, E, block_m, sorted_ids, sorted_cap, expert_ids, blocks_cap, ntp,
                   pos_of, balanced, status);
}

// The same after `flags[w] >= *epoch` for every w < W (the expert-parallel receive
// side: ids are the received local expert ids, written by the peers before they raise
// their flag). A wait that runs out sets FUS_ERR_TIMEOUT and the layout is built from
// what arrived.
__global__ void __launch_bounds__(kAlignThreads)
    align_small_after_flags_kernel(const int* flags, const int* epoch, int W,
                                   const int* __restrict__ ids, int numel, int E, int block_m,
                                   int* __restrict__ sorted_ids, int sorted_cap,
                                   int* __restrict__ expert_ids, int blocks_cap,
                                   int* __restrict__ ntp, int* status) {
  pdl_wait();  // the epoch is bumped by the predecessor (the dispatch)
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
  align_small_body(ids, numel, E, block_m, sorted_ids, sorted_cap, expert_ids, blocks_cap, ntp,
                   nullptr, 0, status);
  pdl_allow_dependents();
}

// ---- large inputs: 3 launches ------------------------------------------------------
// chunk c = elements [c*1024, (c+1)*1024): rank within the chunk, hist[c][E]
__global__ void __launch_bounds__(kAlignThreads)
    align_rank_kernel(const int* __restrict__ ids, int numel, int E, int* __restrict__ rank,
                      int* __restrict__ hist, int* status) {
  extern __shared__ int sm[];
  int* wcnt = sm;
  int* cursor = wcnt + kAlignWarps * E;
  for (int x = threadIdx.x; x < E; x += kAlignThreads) cursor[x] = 0;
  __syncthreads();
  const int base = blockIdx.x * kAlignThreads;
  int e, r;
  rank_chunk(ids, base, numel, E, wcnt, cursor, e, r, status);
  if (base + (int)threadIdx.x < numel) rank[base + threadIdx.x] = r;
  for (int x = threadIdx.x; x < E; x += kAlignThreads) hist[(long)blockIdx.x * E + x] = cursor[x];
}

// one CTA: hist[c][e] <- start[e] + sum_{c'<c} hist[c'][e]; placement
__global__ void __launch_bounds__(kAlignThreads)
    align_scan_kernel(int* __restrict__ hist, int nchunks, int E, int block_m, int numel,
                      int* __restrict__ sorted_ids, int sorted_cap, int* __restrict__ expert_ids,
                      int blocks_cap, int* __restrict__ ntp, int* __restrict__ se, int balanced,
                      int* status) {
  __shared__ int cnt[kAlignMaxE];
  __shared__ int start[kAlignMaxE];
  __shared__ int scan_tmp[kAlignThreads];
  for (int x = threadIdx.x; x < E; x += kAlignThreads) {
    int run = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int v = hist[(long)c * E + x];
      hist[(long)c * E + x] = run;
      run += v;
    }
    cnt[x] = run;
  }
  __syncthreads();
  place_experts(cnt, start, E, block_m, numel, sorted_ids, sorted_cap, expert_ids, blocks_cap, ntp,
                scan_tmp, status, balanced);
  // hist[c][e] stays the expert-relative rank of chunk c's first pair; se = (start, count)
  for (int x = threadIdx.x; x < E; x += kAlignThreads) {
    se[2 * x] = start[x];
    se[2 * x + 1] = cnt[x];
  }
}

__global__ void align_scatter_kernel(const int* __restrict__ ids, int numel, int E,
                                     const int* __restrict__ rank, const int* __restrict__ hist,
                                     int* __restrict__ sorted_ids, int sorted_cap,
                                     int* __restrict__ pos_of, const int* __restrict__ se,
                                     int block_m, int balanced) {
  const int i = blockIdx.x * kAlignThreads + threadIdx.x;
  if (i >= numel) return;
  const int e = ids[i];
  const int r = rank[i];
  if (e < 0 || e >= E || r < 0) return;
  const int p = place_pair(__ldg(se + 2 * e), hist[(long)blockIdx.x * E + e] + r,
                          __ldg(se + 2 * e + 1), block_m, balanced);
  if (p < sorted_cap) sorted_ids[p] = i;
  if (pos_of) pos_of[i] = p;
}

// ---- permutation ------------------------------------------------------------------
__global__ void permute_rows_kernel(const __nv_bfloat16* __restrict__ src, long ld_src,
                                    const int* __restrict__ sorted_ids, const int* __restrict__ ntp,
                                    int div, int num_valid, __nv_bfloat16* __restrict__ dst,
                                    long ld_dst, int max_rows, int H) {
  const int rows = min(__ldg(ntp), max_rows);
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int nv = H >> 3;
  for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < rows; p += warps) {
    const int id = __ldg(sorted_ids + p);
    if (id >= num_valid) continue;  // dispatch pad: never multiplied, left as is
    uint4* d = reinterpret_cast<uint4*>(dst + (long)p * ld_dst);
    const uint4* s = reinterpret_cast<const uint4*>(src + (long)(id / div) * ld_src);
    warp_copy_row(d, s, nv, threadIdx.x & 31);
  }
}

size_t small_smem_bytes(int E) {
  return sizeof(int) * ((size_t)kAlignWarps * E + 2 * E + kAlignThreads + 2 * kAlignSmallMax);
}

}  // namespace fus

using namespace fus;

namespace fus {
int moe_align_small_after_flags(const int* flags, const int* epoch, int W, const int* ids,
                                int numel, int E, int block_m, int* sorted_ids, int sorted_cap,
                                int* expert_ids, int blocks_cap, int* ntp, int pdl, void* stream,
                                int* status) {
  if (numel > kAlignSmallMax || E < 1 || E > kAlignMaxE || W > kAlignThreads)
    return set_error(FUS_E_UNSUPPORTED, "moe_align_after_flags: numel=%d E=%d W=%d", numel, E, W);
  if (int rc = ensure_smem_attr((const void*)align_small_after_flags_kernel,
                                 (int)small_smem_bytes(kAlignMaxE), "moe_align_after_flags"))
    return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kAlignThreads);
  cfg.dynamicSmemBytes = small_smem_bytes(E);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, align_small_after_flags_kernel, flags, epoch, W, ids,
                                     numel, E, block_m, sorted_ids, sorted_cap, expert_ids,
                                     blocks_cap, ntp, status);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "moe_align_after_flags: %s", cudaGetErrorString(e));
  return check_launch("moe_align_after_flags");
}
}  // namespace fus

extern "C" size_t fus_moe_align_workspace(int numel, int E) {
  if (numel <= kAlignSmallMax) return 0;
  const size_t nchunks = (size_t)ceil_div(numel, kAlignThreads);
  return sizeof(int) * ((size_t)numel + nchunks * (size_t)E + 2 * (size_t)E) + 256;
}

extern "C" int fus_moe_align_ex(const int* ids, int numel, int E, int block_m, int* sorted_ids,
                                int sorted_cap, int* expert_ids, int blocks_cap, int* ntp,
                                int* pos_of, int flags, void* workspace, size_t ws_bytes,
                                void* stream, int* status) {
  if (!ids || !sorted_ids || !expert_ids || !ntp || numel < 0 || block_m < 1 ||
      (flags & ~FUS_ALIGN_BALANCED))
    return set_error(FUS_E_INVALID, "moe_align: bad args");
  const int balanced = (flags & FUS_ALIGN_BALANCED) ? 1 : 0;
  if (E < 1 || E > kAlignMaxE) return set_error(FUS_E_UNSUPPORTED, "moe_align: E=%d > %d", E, kAlignMaxE);
  cudaStream_t st = as_stream(stream);
  if (numel <= kAlignSmallMax) {
    const size_t sm = small_smem_bytes(E);
    if (int rc = ensure_smem_attr((const void*)align_small_kernel,
                                   (int)small_smem_bytes(kAlignMaxE), "moe_align"))
      return rc;
    align_small_kernel<<<1, kAlignThreads, sm, st>>>(ids, numel, E, block_m, sorted_ids, sorted_cap,
                                                    expert_ids, blocks_cap, ntp, pos_of, balanced,
                                                    status);
    return check_launch("moe_align_small");
  }
  const size_t need = fus_moe_align_workspace(numel, E);
  if (!workspace || ws_bytes < need || !aligned16(workspace))
    return set_error(FUS_E_INVALID, "moe_align: workspace of %zu bytes required", need);
  const int nchunks = ceil_div(numel, kAlignThreads);
  int* rank = reinterpret_cast<int*>(workspace);
  int* hist = rank + numel;
  int* se = hist + (size_t)nchunks * E;
  const size_t sm = sizeof(int) * ((size_t)kAlignWarps * E + E);
  if (int rc = ensure_smem_attr((const void*)align_rank_kernel,
                                 (int)(sizeof(int) * ((size_t)kAlignWarps * kAlignMaxE + kAlignMaxE)),
                                 "moe_align"))
    return rc;
  align_rank_kernel<<<nchunks, kAlignThreads, sm, st>>>(ids, numel, E, rank, hist, status);
  align_scan_kernel<<<1, kAlignThreads, 0, st>>>(hist, nchunks, E, block_m, numel, sorted_ids,
                                                 sorted_cap, expert_ids, blocks_cap, ntp, se,
                                                 balanced, status);
  align_scatter_kernel<<<nchunks, kAlignThreads, 0, st>>>(ids, numel, E, rank, hist, sorted_ids,
                                                          sorted_cap, pos_of, se, block_m,
                                                          balanced);
  return check_launch("moe_align");
}

extern "C" int fus_moe_align(const int* ids, int numel, int E, int block_m, int* sorted_ids,
                             int sorted_cap, int* expert_ids, int blocks_cap, int* ntp,
                             void* workspace, size_t ws_bytes, void* stream, int* status) {
  return fus_moe_align_ex(ids, numel, E, block_m, sorted_ids, sorted_cap, expert_ids, blocks_cap,
                          ntp, nullptr, 0, workspace, ws_bytes, stream, status);
}

extern "C" int fus_permute_rows(const void* src, long ld_src, const int* sorted_ids, const int* ntp,
                                int div, int num_valid, void* dst, long ld_dst, int max_rows, int H,
                                void* stream, int* status) {
  (void)status;
  if (!src || !sorted_ids || !ntp || !dst || div < 1 || H <= 0 || H % 8 || max_rows < 0 ||
      !aligned16(src) || !aligned16(dst) || ld_src % 8 || ld_dst % 8)
    return set_error(FUS_E_INVALID, "permute_rows: bad args");
  if (max_rows == 0) return FUS_OK;
  int grid = ceil_div(max_rows, 8);
  const int cap = num_sms() * 8;
  if (grid > cap) grid = cap;
  permute_rows_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)src, ld_src, sorted_ids, ntp, div, num_valid, (__nv_bfloat16*)dst,
      ld_dst, max_rows, H);
  return check_launch("permute_rows");
}

// ---- variant that allocates nothing ---------------------------------------------------
// Scratch for the multi-launch path (stable ranks + per-chunk histograms) lives in a
// file-scope device array sized for the largest input this variant accepts: numel up to
// 65536 (T = 8192 tokens at top-8) and up to 512 experts, 397,568 bytes. Every GPU that
// loads the library holds it until the process exits.
namespace fus {
constexpr int kAlignNoAllocMaxNumel = 65536;
constexpr size_t kAlignNoAllocBytes =
    sizeof(int) * ((size_t)kAlignNoAllocMaxNumel +
                   (size_t)(kAlignNoAllocMaxNumel / kAlignThreads) * kAlignMaxE + 2 * kAlignMaxE) +
    256;
static __device__ __align__(256) unsigned char g_align_scratch[kAlignNoAllocBytes];

// Host code cannot use g_align_scratch as a device address (on the host the name is only
// a stand-in); its device address is looked up once per device with that device current.
constexpr int kMaxDevices = 64;
static std::mutex g_align_scratch_mu;
static void* g_align_scratch_ptr[kMaxDevices] = {};
}  // namespace fus

extern "C" int fus_moe_align_noalloc(const int* ids, int numel, int E, int block_m,
                                     int* sorted_ids, int sorted_cap, int* expert_ids,
                                     int blocks_cap, int* ntp, void* stream, int* status) {
  if (numel < 0 || numel > kAlignNoAllocMaxNumel)
    return set_error(FUS_E_UNSUPPORTED, "moe_align_noalloc: numel=%d exceeds the built-in "
                     "scratch limit of %d pairs (T*topk)", numel, kAlignNoAllocMaxNumel);
  if (E < 1 || E > kAlignMaxE)
    return set_error(FUS_E_UNSUPPORTED, "moe_align_noalloc: E=%d > %d", E, kAlignMaxE);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "moe_align_noalloc: cudaGetDevice: %s",
                                         cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(FUS_E_UNSUPPORTED, "moe_align_noalloc: device %d out of range", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_align_scratch_mu);
    scratch = g_align_scratch_ptr[dev];
    if (!scratch) {
      e = cudaGetSymbolAddress(&scratch, g_align_scratch);
      if (e != cudaSuccess || !scratch)
        return set_error(FUS_E_LAUNCH, "moe_align_noalloc: cudaGetSymbolAddress: %s",
                         cudaGetErrorString(e));
      g_align_scratch_ptr[dev] = scratch;
    }
  }
  // Every scratch word the kernels read is written earlier in the same call, so the
  // previous call's contents never need clearing.
  return fus_moe_align(ids, numel, E, block_m, sorted_ids, sorted_cap, expert_ids, blocks_cap,
                       ntp, scratch, kAlignNoAllocBytes, stream, status);
}
