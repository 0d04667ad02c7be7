// Expert-parallel row exchange over NVLink peer memory (decode, fixed slots).
//
// The NCCL all_to_all of the fixed-slot exchange moves a few rows per step but costs a
// collective launch and handshake each way. Here every rank exports one buffer
// (CUDA IPC); the others map it and write into it directly with plain stores:
//
//   exchange buffer of rank g (W ranks, S slots per source, H features):
//     recv_rows [W*S][H] bf16   block w = the rows rank w sent to g for its experts
//     recv_leid [W*S]    int32  their local expert ids, -1 = unused slot
//     ret_rows  [W*S][H] bf16   block d = the expert rows rank d sends back to g
//     dflags    [W]      int32  dflags[w] = last step whose dispatch from w is complete
//     cflags    [W]      int32  cflags[d] = last step whose combine from d is complete
//
// One step (epoch e = previous + 1, kept on the device so the step replays from a CUDA
// graph):
//   fus_ep_p2p_dispatch  pair (t, k) with owner d and rank j among this rank's pairs to
//                        d: row x[t] -> recv_rows of d at [rank*S + j], its local expert
//                        -> recv_leid of d (unused slots -1), then dflags[rank] = e at
//                        every d (after a system-scope fence)
//   fus_ep_p2p_wait      until dflags[w] >= e for all w (bounded: FUS_ERR_TIMEOUT)
//   (owner: the routed experts over recv_rows / recv_leid, rows y[W*S][H])
//   fus_ep_p2p_combine   y[w*S + j] of live slots -> ret_rows of w at [rank*S + j], then
//                        cflags[rank] = e at every w
//   fus_ep_p2p_wait      on cflags; the merge reads ret_rows[slot_of_pair[t*K + k]]
//
// One buffer per rank suffices: a rank overwrites a peer's recv area only in the next
// step's dispatch, which follows (in its stream) its wait for that peer's combine, which
// the peer issues after its last read of recv; and a peer overwrites this rank's ret
// area only after this rank's next dispatch reached it, which follows this rank's merge.
// Plain peer stores only (no multicast objects, no TMA from peer memory).
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace fus {

constexpr int kP2PMaxRanks = 64;
constexpr int kP2PMaxSlots = 4096;  // W * S of one exchange buffer

struct P2PPeers {
  const unsigned long long* rows;   // [W] base of each rank's recv_rows (or ret_rows)
  const unsigned long long* leid;   // [W] base of each rank's recv_leid (dispatch only)
  const unsigned long long* flags;  // [W] base of each rank's dflags (or cflags)
};

// one CTA of 1024 threads; R = T*topk <= 1024 pairs
__global__ void __launch_bounds__(1024)
    p2p_dispatch_kernel(const __nv_bfloat16* __restrict__ x, long ldx, int H,
                        const int* __restrict__ topi, int R, int topk, int E_loc, int W, int S,
                        int rank, P2PPeers peers, int* epoch, int* __restrict__ slot_of_pair,
                        int* status) {
  __shared__ int dst_s[1024];
  __shared__ int rank_s[1024];
  __shared__ int e_s;
  pdl_wait();  // x / topi come from the predecessor (when launched as a dependent)
  if (threadIdx.x == 0) e_s = *epoch + 1;
  // unused slots of this rank's block at every peer read -1 (overwritten below for the
  // used ones, ordered by the barrier)
  for (int i = threadIdx.x; i < W * S; i += blockDim.x) {
    int* pl = reinterpret_cast<int*>(peers.leid[i / S]);
    pl[rank * S + i % S] = -1;
  }
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
    int j = 0;
    for (int q = 0; q < i; ++q) j += dst_s[q] == d;
    if (d >= 0 && j >= S) raise_status(status, FUS_ERR_CAPACITY);
    const bool ok = d >= 0 && j < S;
    rank_s[i] = ok ? j : -1;
    slot_of_pair[i] = ok ? d * S + j : 0;
    if (ok) {
      int* pl = reinterpret_cast<int*>(peers.leid[d]);
      pl[rank * S + j] = topi[i] - d * E_loc;
    }
  }
  __syncthreads();
  // all rows as one flat range of 16-byte vectors, four loads in flight per thread
  const int nv = H >> 3;
  const int total = R * nv;
  for (int base = threadIdx.x; base < total; base += 4 * blockDim.x) {
    uint4 v[4];
    uint4* o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = base + u * blockDim.x;
      o[u] = nullptr;
      if (idx < total) {
        const int i = idx / nv, q = idx - i * nv;
        const int j = rank_s[i];
        if (j >= 0) {
          v[u] = __ldg(reinterpret_cast<const uint4*>(x + (long)(i / topk) * ldx) + q);
          o[u] = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers.rows[dst_s[i]]) +
                                          (long)(rank * S + j) * H) + q;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (o[u]) *o[u] = v[u];
  }
  // every thread's peer stores precede the barrier; the signalling thread's system-scope
  // fence then orders them (cumulatively) before its flag stores
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int e = e_s;
    for (int d = 0; d < W; ++d) st_release_sys_i32(reinterpret_cast<int*>(peers.flags[d]) + rank, e);
    *epoch = e;
  }
  pdl_allow_dependents();
}

// one CTA: copies the live rows of every source block back to its rank, then signals
__global__ void __launch_bounds__(1024)
    p2p_combine_kernel(const __nv_bfloat16* __restrict__ y, long ldy, int H,
                       const int* __restrict__ recv_leid, int W, int S, int rank, P2PPeers peers,
                       const int* epoch) {
  __shared__ int live_s[kP2PMaxSlots];  // compacted live slots
  __shared__ int n_live;
  pdl_wait();  // y comes from the predecessor (the down projection)
  if (threadIdx.x == 0) n_live = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < W * S; i += blockDim.x) {
    if (recv_leid[i] >= 0) {
      const int k = atomicAdd(&n_live, 1);
      live_s[k] = i;
    }
  }
  __syncthreads();
  const int nv = H >> 3;
  const int total = n_live * nv;
  for (int base = threadIdx.x; base < total; base += 4 * blockDim.x) {
    uint4 v[4];
    uint4* o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = base + u * blockDim.x;
      o[u] = nullptr;
      if (idx < total) {
        const int k = idx / nv, q = idx - k * nv;
        const int i = live_s[k];
        const int w = i / S, j = i - w * S;
        v[u] = *(reinterpret_cast<const uint4*>(y + (long)i * ldy) + q);
        o[u] = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers.rows[w]) +
                                        (long)(rank * S + j) * H) + q;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (o[u]) *o[u] = v[u];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int e = *epoch;
    for (int w = 0; w < W; ++w) st_release_sys_i32(reinterpret_cast<int*>(peers.flags[w]) + rank, e);
  }
  pdl_allow_dependents();
}

// lane w waits for flags[w] >= epoch; gives up after timeout_ns with FUS_ERR_TIMEOUT
__global__ void p2p_wait_kernel(const int* flags, const int* epoch, int W,
                                unsigned long long timeout_ns, int* status) {
  const int e = *epoch;
  for (int w = threadIdx.x; w < W; w += blockDim.x) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_i32(flags + w) < e) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        raise_status(status, FUS_ERR_TIMEOUT);
        break;
      }
    }
  }
}

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  });
  return fn;
}

// one CTA of 1024 threads, optionally as a programmatic dependent of the previous kernel
template <typename... KArgs, typename... Args>
int launch_1cta(void (*kernel)(KArgs...), int pdl, void* stream, const char* what,
                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(1024);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

// ---- the whole decode step on one rank (workspace layout) ----
struct P2PStepLayout {
  int R, n, l_cap, l_bcap;
  size_t off_x2, off_logits, off_slots, off_ls, off_leids, off_lntp,
      off_act, off_acts, off_y, off_ys, total;
};

static bool p2p_layout(const fus_ep_p2p_desc* d, int T, P2PStepLayout& L) {
  if (!d || !d->blk || T < 1 || d->W < 1 || d->S < 1) return false;
  const fus_moe_block_desc* b = d->blk;
  const int H = b->H, I = b->I, E = b->E, K = b->topk;
  L.R = T * K;
  L.n = d->W * d->S;
  L.l_cap = (L.n + d->E_loc * 15 + 15) / 16 * 16;
  L.l_bcap = L.l_cap / 16;
  size_t o = 256;  // the front end's ticket sits at offset 0 and stays zero
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = (o + bytes + 255) / 256 * 256;
    return at;
  };
  L.off_x2 = take((size_t)T * H * 2);
  L.off_logits = take((size_t)T * E * 4);
  L.off_slots = take((size_t)L.R * 4);
  L.off_ls = take((size_t)L.l_cap * 4);
  L.off_leids = take((size_t)L.l_bcap * 4);
  L.off_lntp = take(16);
  L.off_act = take((size_t)L.l_cap * I * 2);
  L.off_acts = take((size_t)T * I * 2);
  L.off_y = take((size_t)L.n * H * 2);
  L.off_ys = take((size_t)T * H * 4);
  L.total = o + 256;
  return true;
}

}  // namespace fus

using namespace fus;

extern "C" size_t fus_ep_p2p_decode_workspace(const fus_ep_p2p_desc* d, int T) {
  P2PStepLayout L;
  return p2p_layout(d, T, L) ? L.total : 0;
}

extern "C" int fus_ep_p2p_decode_forward(const fus_ep_p2p_desc* d, const void* h, const void* r,
                                         int T, void* out, void* h1, float* topw, int* topi,
                                         void* workspace, size_t ws_bytes, void* stream,
                                         int* status) {
  if (!d || !d->blk || !h || !r || !out || !h1 || !topw || !topi || !workspace)
    return set_error(FUS_E_INVALID, "ep_p2p_decode: null argument");
  if (T == 0) return FUS_OK;
  const fus_moe_block_desc* b = d->blk;
  const int H = b->H, I = b->I, E = b->E, K = b->topk, W = d->W;
  P2PStepLayout L;
  if (!p2p_layout(d, T, L)) return set_error(FUS_E_INVALID, "ep_p2p_decode: bad sizes");
  if (ws_bytes < L.total)
    return set_error(FUS_E_INVALID, "ep_p2p_decode: workspace %zu < %zu", ws_bytes, L.total);
  if (d->E_loc * W != E || d->rank < 0 || d->rank >= W || d->S < L.R ||
      W * d->S > kP2PMaxSlots)
    return set_error(FUS_E_INVALID,
                     "ep_p2p_decode: E_loc*W != E, bad rank, S < T*topk or W*S > 4096");
  if (!(E <= 256 && E % 2 == 0 && L.R <= 256 && (b->nplanes == 1 || b->nplanes == 3)))
    return set_error(FUS_E_UNSUPPORTED, "ep_p2p_decode: needs the fused front end "
                     "(E <= 256, T*topk <= 256)");
  if (!d->peer_rows || !d->peer_leid || !d->peer_dflags || !d->peer_ret || !d->peer_cflags ||
      !d->recv_rows || !d->recv_leid || !d->ret_rows || !d->dflags || !d->cflags || !d->epoch)
    return set_error(FUS_E_INVALID, "ep_p2p_decode: exchange buffers missing");
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) &
                                             ~uintptr_t(255));
  auto at = [&](size_t off) { return base + off; };
  int* done = reinterpret_cast<int*>(base);
  void* x2 = at(L.off_x2);
  int* slots = reinterpret_cast<int*>(at(L.off_slots));
  int* ls = reinterpret_cast<int*>(at(L.off_ls));
  int* leids = reinterpret_cast<int*>(at(L.off_leids));
  int* lntp = reinterpret_cast<int*>(at(L.off_lntp));
  void* act = at(L.off_act);
  void* act_s = at(L.off_acts);
  void* y = at(L.off_y);
  void* ys = at(L.off_ys);
  const bool shared = b->w13s != nullptr;
  int rc;
  // 1 norm + router + top-k (block_m 0: no dispatch layout over all experts; the owners
  // build theirs from what they receive)
  if ((rc = route_small_launch(h, r, b->gamma, b->eps, b->wa, b->nplanes, b->bias, T, H, E, K,
                                b->routed_scale, b->renorm, b->n_group, b->topk_group, h1, x2,
                                reinterpret_cast<float*>(at(L.off_logits)), topw, topi, 0,
                                nullptr, 0, nullptr, 0, nullptr, done, nullptr, 0, stream,
                                status)))
    return rc;
  // 2 rows + local expert ids into the owners' exchange buffers, flags raised
  P2PPeers pd{d->peer_rows, d->peer_leid, d->peer_dflags};
  if ((rc = launch_1cta(p2p_dispatch_kernel, 1, stream, "ep_p2p_dispatch",
                        (const __nv_bfloat16*)x2, (long)H, H, (const int*)topi, L.R, K, d->E_loc,
                        W, d->S, d->rank, pd, d->epoch, slots, status)))
    return rc;
  // 3 once every source's rows are in: layout of the received slots over local experts
  if ((rc = moe_align_small_after_flags(d->dflags, d->epoch, W, d->recv_leid, L.n, d->E_loc, 16,
                                        ls, L.l_cap, leids, L.l_bcap, lntp, 1, stream, status)))
    return rc;
  // 4 w13 + SwiGLU: received rows gathered by dispatch position; shared expert over x2
  const int maxb = (L.n < d->E_loc ? L.n : d->E_loc) + L.n / 16;
  fus_gemm_group g[2] = {};
  g[0].w = b->w13;
  g[0].n_experts = d->E_loc;
  g[0].x = d->recv_rows;
  g[0].ldx = H;
  g[0].x_rows = L.n;
  g[0].expert_ids = leids;
  g[0].ntp = lntp;
  g[0].max_blocks = maxb < L.l_bcap ? maxb : L.l_bcap;
  g[0].out = act;
  g[0].ldo = I;
  g[0].row_limit = L.l_cap;
  g[0].flags = FUS_GEMM_SWIGLU_EXACT | FUS_GEMM_W_STREAM;
  g[0].live_ids = ls;
  g[0].live_limit = L.n;
  g[0].gather_ids = ls;
  g[0].gather_div = 1;
  g[1].w = b->w13s;
  g[1].n_experts = 1;
  g[1].x = x2;
  g[1].ldx = H;
  g[1].x_rows = T;
  g[1].max_blocks = (T + 15) / 16;
  g[1].out = act_s;
  g[1].ldo = I;
  g[1].row_limit = T;
  g[1].flags = FUS_GEMM_SWIGLU_EXACT | FUS_GEMM_W_STREAM;
  if ((rc = grouped_gemm_launch(g, shared ? 2 : 1, 2 * I, H, 1, FUS_EPI_SWIGLU, 16, 1, 0, 0,
                                nullptr, 1, stream, status)))
    return rc;
  // 5 w2: routed rows to y[slot], shared rows to ys (fp32)
  g[0].w = b->w2;
  g[0].x = act;
  g[0].ldx = I;
  g[0].x_rows = L.l_cap;
  g[0].gather_ids = nullptr;
  g[0].out = y;
  g[0].ldo = H;
  g[0].row_map = ls;
  g[0].row_limit = L.n;
  g[0].flags = FUS_GEMM_W_STREAM;
  g[1].w = b->w2s;
  g[1].x = act_s;
  g[1].ldx = I;
  g[1].out = ys;
  g[1].ldo = H;
  g[1].flags = FUS_GEMM_OUT_F32 | FUS_GEMM_W_STREAM;
  if ((rc = grouped_gemm_launch(g, shared ? 2 : 1, H, I, 1, FUS_EPI_BF16, 16, 1, 0, 0, nullptr, 2,
                                stream, status)))
    return rc;
  // 6 expert rows back to their sources, flags raised
  P2PPeers pc{d->peer_ret, nullptr, d->peer_cflags};
  if ((rc = launch_1cta(p2p_combine_kernel, 1, stream, "ep_p2p_combine",
                        (const __nv_bfloat16*)y, (long)H, H, (const int*)d->recv_leid, W, d->S,
                        d->rank, pc, (const int*)d->epoch)))
    return rc;
  // 7 once every owner's rows are back: out = bf16(sum_k w_k y_k + h1 + ys)
  return merge_pos_after_flags(d->ret_rows, H, slots, K, topw, K, h1, H, shared ? ys : nullptr, H,
                               1, out, H, T, H, d->cflags, d->epoch, W, 1, stream, status);
}

extern "C" int fus_ipc_handle(const void* ptr, void* handle_out, size_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return set_error(FUS_E_INVALID, "ipc_handle: null");
  GetAddressRangeFn range = address_range_fn();
  if (!range) return set_error(FUS_E_LAUNCH, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(FUS_E_INVALID, "ipc_handle: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base;
  return FUS_OK;
}

extern "C" int fus_ipc_open(const void* handle, size_t offset, void** ptr_out) {
  if (!handle || !ptr_out) return set_error(FUS_E_INVALID, "ipc_open: null");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr_out = static_cast<char*>(base) + offset;
  return FUS_OK;
}

extern "C" int fus_ipc_close(void* ptr, size_t offset) {
  if (!ptr) return FUS_OK;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return set_error(FUS_E_LAUNCH, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return FUS_OK;
}

extern "C" int fus_ep_p2p_dispatch(const void* x, long ldx, int H, const int* topi, int T, int topk,
                                   int E_loc, int W, int S, int rank,
                                   const unsigned long long* peer_rows,
                                   const unsigned long long* peer_leid,
                                   const unsigned long long* peer_flags, int* epoch,
                                   int* slot_of_pair, void* stream, int* status) {
  const int R = T * topk;
  if (!x || !topi || !peer_rows || !peer_leid || !peer_flags || !epoch || !slot_of_pair ||
      T < 0 || topk < 1 || E_loc < 1 || W < 1 || W > kP2PMaxRanks || rank < 0 || rank >= W ||
      S < R || H <= 0 || H % 8 || ldx % 8 || !aligned16(x))
    return set_error(FUS_E_INVALID, "ep_p2p_dispatch: bad args");
  if (R > 1024) return set_error(FUS_E_UNSUPPORTED, "ep_p2p_dispatch: T*topk=%d > 1024", R);
  P2PPeers p{peer_rows, peer_leid, peer_flags};
  return launch_1cta(p2p_dispatch_kernel, 0, stream, "ep_p2p_dispatch", (const __nv_bfloat16*)x,
                     ldx, H, topi, R, topk, E_loc, W, S, rank, p, epoch, slot_of_pair, status);
}

extern "C" int fus_ep_p2p_combine(const void* y, long ldy, int H, const int* recv_leid, int W,
                                  int S, int rank, const unsigned long long* peer_ret,
                                  const unsigned long long* peer_cflags, const int* epoch,
                                  void* stream, int* status) {
  (void)status;
  if (!y || !recv_leid || !peer_ret || !peer_cflags || !epoch || W < 1 || W > kP2PMaxRanks ||
      rank < 0 || rank >= W || S < 1 || W * S > kP2PMaxSlots || H <= 0 || H % 8 || ldy % 8 ||
      !aligned16(y))
    return set_error(FUS_E_INVALID, "ep_p2p_combine: bad args");
  P2PPeers p{peer_ret, nullptr, peer_cflags};
  return launch_1cta(p2p_combine_kernel, 0, stream, "ep_p2p_combine", (const __nv_bfloat16*)y, ldy,
                     H, recv_leid, W, S, rank, p, epoch);
}

extern "C" int fus_ep_p2p_wait(const int* flags, const int* epoch, int W,
                               unsigned long long timeout_ns, void* stream, int* status) {
  if (!flags || !epoch || W < 1 || W > kP2PMaxRanks)
    return set_error(FUS_E_INVALID, "ep_p2p_wait: bad args");
  if (timeout_ns == 0 || timeout_ns > kWaitBudgetNs) timeout_ns = kWaitBudgetNs;
  p2p_wait_kernel<<<1, 64, 0, as_stream(stream)>>>(flags, epoch, W, timeout_ns, status);
  return check_launch("ep_p2p_wait");
}
