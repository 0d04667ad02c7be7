// The whole GLM-5.2 MoE block as one C-ABI call: the layer-chain driver of
// glm52/bench/bench_layer.py:395-481 (build_chain, without o_proj) with the oracle
// composition of bench_layer.py:365-374, issued as 8 kernel launches on one stream:
//
//   1 add_rmsnorm            h, r            -> h1, x2
//   2 router GEMM (tcgen05)  x2, W_g planes  -> fp32 partial logits
//   3 top-k                  partials, bias  -> topw, topi
//   4 moe_align              topi            -> sorted ids, expert ids, padded total
//   5 permute                x2, sorted ids  -> xs (rows in dispatch order)
//   6 w13 GEMM + SwiGLU      routed (xs) and shared (x2) groups in ONE launch -> act
//   7 w2 GEMM                routed (act) and shared groups in ONE launch     -> y
//   8 merge                  out = bf16(sum_k w_k y_k + h1 + y_shared)
//
// Rounding: only at the tensors the block must store in bf16 (x2, act, y) and at the
// output. Gate/up feed SwiGLU in fp32, the shared output stays fp32 and the routed sum
// is not rounded before the residual add. This is closer to the reference's exact fp32
// path (glm52_h200/reference.py moe_mlp_exact_fp32) than its framework chain, which
// rounds at every kernel boundary; the framework rounding is still available per step
// (FUS_GEMM_* flags, fus_merge round_mid) for the drop-in unfused entry points.
//
// No step needs the host: every data-dependent size (padded total, blocks per expert)
// stays on the device, so the sequence can be captured in a CUDA graph.
#include "common.cuh"
#include "host_util.h"

namespace {

struct BlockLayout {
  int R, cap, blocks_cap, max_blocks, nsplit;
  size_t off_x2, off_partial, off_sorted, off_eids, off_ntp, off_align, off_xs, off_act, off_acts,
      off_y, off_ys, total;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool layout_for(const fus_moe_block_desc* d, int T, int bn, BlockLayout& L) {
  if (!d || T < 1 || bn < 16) return false;
  const int H = d->H, I = d->I, E = d->E, k = d->topk;
  L.R = T * k;
  L.cap = L.R + E * (bn - 1);
  L.cap = (L.cap + bn - 1) / bn * bn;
  L.blocks_cap = L.cap / bn;
  L.max_blocks = (L.R < E ? L.R : E) + L.R / bn;
  if (L.max_blocks > L.blocks_cap) L.max_blocks = L.blocks_cap;
  L.nsplit = fus_router_nsplit(T, H, E, d->nplanes);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.off_x2 = take((size_t)T * H * 2);
  L.off_partial = take((size_t)L.nsplit * T * E * 4);
  L.off_sorted = take((size_t)L.cap * 4);
  L.off_eids = take((size_t)L.blocks_cap * 4);
  L.off_ntp = take(16);
  L.off_align = take(fus_moe_align_workspace(L.R, E));
  L.off_xs = take((size_t)L.cap * H * 2);
  L.off_act = take((size_t)L.cap * I * 2);
  L.off_acts = take((size_t)T * I * 2);
  L.off_y = take((size_t)L.R * H * 2);
  L.off_ys = take((size_t)T * H * 4);  // shared expert output, fp32
  L.total = o + 256;  // base alignment slack
  return true;
}

}  // namespace

using namespace fus;

extern "C" int fus_moe_block_pick_block_n(int T, int E, int topk) {
  const double per_expert = (double)T * topk / (E > 0 ? E : 1);
  if (per_expert <= 16) return 16;
  if (per_expert <= 64) return 32;
  if (per_expert <= 160) return 64;
  return 128;
}

extern "C" size_t fus_moe_block_workspace(const fus_moe_block_desc* d, int T, int block_n) {
  if (!d) return 0;
  if (block_n <= 0) block_n = fus_moe_block_pick_block_n(T, d->E, d->topk);
  BlockLayout L;
  if (!layout_for(d, T, block_n, L)) return 0;
  return L.total;
}

extern "C" int fus_moe_block_forward(const fus_moe_block_desc* d, const void* h, const void* r,
                                     int T, int block_n, void* out, void* h1, float* topw,
                                     int* topi, void* workspace, size_t ws_bytes, void* stream,
                                     int* status) {
  if (!d || !h || !r || !out || !h1 || !topw || !topi || !workspace)
    return set_error(FUS_E_INVALID, "moe_block: null argument");
  if (T < 0) return set_error(FUS_E_INVALID, "moe_block: T < 0");
  if (T == 0) return FUS_OK;
  if (!d->gamma || !d->wa || !d->w13 || !d->w2 || (!d->w13s) != (!d->w2s))
    return set_error(FUS_E_INVALID, "moe_block: missing weights");
  if (block_n <= 0) block_n = fus_moe_block_pick_block_n(T, d->E, d->topk);
  BlockLayout L;
  if (!layout_for(d, T, block_n, L)) return set_error(FUS_E_INVALID, "moe_block: bad sizes");
  if (ws_bytes < L.total) return set_error(FUS_E_INVALID, "moe_block: workspace %zu < %zu", ws_bytes, L.total);
  const int H = d->H, I = d->I, E = d->E, K = d->topk;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  auto at = [&](size_t off) { return base + off; };
  void* x2 = at(L.off_x2);
  float* partial = reinterpret_cast<float*>(at(L.off_partial));
  int* sorted = reinterpret_cast<int*>(at(L.off_sorted));
  int* eids = reinterpret_cast<int*>(at(L.off_eids));
  int* ntp = reinterpret_cast<int*>(at(L.off_ntp));
  void* align_ws = at(L.off_align);
  void* xs = at(L.off_xs);
  void* act = at(L.off_act);
  void* act_s = at(L.off_acts);
  void* y = at(L.off_y);
  void* ys = at(L.off_ys);
  const bool shared = d->w13s != nullptr;

  int rc;
  if ((rc = fus_add_rmsnorm(h, H, r, H, d->gamma, h1, H, x2, H, T, H, d->eps, 1, 1, stream, status)))
    return rc;
  if ((rc = fus_router_logits(x2, H, d->wa, d->nplanes, partial, T, H, E, L.nsplit, stream, status)))
    return rc;
  if ((rc = fus_router_topk(partial, L.nsplit, d->bias, nullptr, topw, topi, T, E, K,
                            d->routed_scale, d->renorm, stream, status)))
    return rc;
  if ((rc = fus_moe_align(topi, L.R, E, block_n, sorted, L.cap, eids, L.blocks_cap, ntp, align_ws,
                          fus_moe_align_workspace(L.R, E), stream, status)))
    return rc;
  if ((rc = fus_permute_rows(x2, H, sorted, ntp, K, L.R, xs, H, L.cap, H, stream, status)))
    return rc;

  fus_gemm_group g[2] = {};
  // ---- w13 + SwiGLU: routed experts over xs, shared expert over x2 ----
  g[0].w = d->w13;
  g[0].n_experts = E;
  g[0].x = xs;
  g[0].ldx = H;
  g[0].x_rows = L.cap;
  g[0].expert_ids = eids;
  g[0].ntp = ntp;
  g[0].max_blocks = L.max_blocks;
  g[0].out = act;
  g[0].ldo = I;
  g[0].row_limit = L.cap;
  g[0].flags = FUS_GEMM_SWIGLU_EXACT;
  g[1].w = d->w13s;
  g[1].n_experts = 1;
  g[1].x = x2;
  g[1].ldx = H;
  g[1].x_rows = T;
  g[1].max_blocks = (T + block_n - 1) / block_n;
  g[1].out = act_s;
  g[1].ldo = I;
  g[1].row_limit = T;
  g[1].flags = FUS_GEMM_SWIGLU_EXACT;
  if ((rc = fus_grouped_gemm(g, shared ? 2 : 1, 2 * I, H, 1, FUS_EPI_SWIGLU, block_n, 1, 0, stream,
                             status)))
    return rc;
  // ---- w2: routed rows scatter to y[flat], shared rows to ys ----
  g[0].w = d->w2;
  g[0].x = act;
  g[0].ldx = I;
  g[0].out = y;
  g[0].ldo = H;
  g[0].row_map = sorted;
  g[0].row_limit = L.R;
  g[0].flags = 0;
  g[1].w = d->w2s;
  g[1].x = act_s;
  g[1].ldx = I;
  g[1].out = ys;
  g[1].ldo = H;
  g[1].flags = FUS_GEMM_OUT_F32;  // reference keeps the shared output in fp32
  if ((rc = fus_grouped_gemm(g, shared ? 2 : 1, H, I, 1, FUS_EPI_BF16, block_n, 1, 0, stream, status)))
    return rc;
  // ---- merge + residual + shared ----
  return fus_merge(y, (long)K * H, H, K, topw, K, h1, H, shared ? ys : nullptr, H, 1, out, H, T,
                   H, /*round_mid=*/0, stream, status);
}
