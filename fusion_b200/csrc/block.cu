// The whole GLM-5.2 MoE block as one C-ABI call: the layer-chain driver of
// glm52/bench/bench_layer.py:395-481 (build_chain, without o_proj) with the oracle
// composition of bench_layer.py:365-374, issued as 8 kernel launches on one stream:
//
//   1 add_rmsnorm            h, r            -> h1, x2
//   2 router GEMM (tcgen05)  x2, W_g planes  -> fp32 partial logits
//   3 top-k                  partials, bias  -> topw, topi
//   4 moe_align              topi            -> sorted ids, expert ids, padded total,
//                                               pos_of (each pair's dispatch position)
//      (T <= 16: steps 1-4 are ONE launch, fus_moe_route_small)
//   5 permute (T > 16)       x2, sorted ids  -> xs (rows in dispatch order)
//   6 w13 GEMM + SwiGLU      routed rows (T <= 16: gathered from x2 by dispatch position
//                            with TMA gather4; else xs) and the shared expert's x2 -> act
//   7 w2 GEMM                routed (act) and shared groups in ONE launch -> y (rows in
//                            dispatch order), y_shared
//   8 merge                  out = bf16(sum_k w_k y[pos_of[t,k]] + h1 + y_shared)
//      (T <= 16: fused into step 7 -- the CTA that lands a token tile's last
//       contribution writes the output for it; y is then in pair order)
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
  int tiles;
  size_t off_x2, off_partial, off_sorted, off_eids, off_ntp, off_align, off_xs, off_act, off_acts,
      off_y, off_ys, off_cnt, off_done, off_pos, total;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// decode path: the fused front end (fus_moe_route_small) and gathered-row GEMMs
bool small_path(const fus_moe_block_desc* d, int T) {
  const int E = d->E, K = d->topk;
  return T <= 16 && E <= 256 && E % 2 == 0 && T * K <= 256 && (d->nplanes == 1 || d->nplanes == 3);
}

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
  // the decode front end's ticket sits first, at the same offset for every T: no other
  // buffer ever overlaps it, so it stays zero between calls of any size
  size_t o = 256;
  L.off_done = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.off_x2 = take((size_t)T * H * 2);
  L.off_partial = take((size_t)(L.nsplit > 1 ? L.nsplit : 1) * T * E * 4);
  L.off_sorted = take((size_t)L.cap * 4);
  L.off_eids = take((size_t)L.blocks_cap * 4);
  L.off_ntp = take(16);
  L.off_align = take(fus_moe_align_workspace(L.R, E));
  const bool small = small_path(d, T);
  L.off_xs = small ? 0 : take((size_t)L.cap * H * 2);  // permuted rows (prefill only)
  L.off_act = take((size_t)L.cap * I * 2);
  L.off_acts = take((size_t)T * I * 2);
  // decode: y[pair] in pair order (fused merge); prefill: the down projection's rows in
  // dispatch order (dense tile stores) in the permuted-row buffer, dead once w13 has
  // read it; the merge gathers them back per token through pos_of
  L.off_y = small ? take((size_t)L.R * H * 2) : L.off_xs;
  L.off_pos = small ? 0 : take((size_t)L.R * 4);
  L.off_ys = take((size_t)T * H * 4);  // shared expert output, fp32
  L.tiles = fus_grouped_gemm_tiles(H, FUS_EPI_BF16, bn);
  L.off_cnt = take((size_t)T * L.tiles * 4);  // fused-merge arrival counters

  L.total = o + 256;  // base alignment slack
  return true;
}

}  // namespace

using namespace fus;

extern "C" int fus_moe_block_pick_block_n(int T, int E, int topk) {
  // token tile vs. average tokens per expert: decode keeps one narrow block per expert
  // (weights streamed once, many CTAs); prefill takes wide tiles with two weight tiles
  // per CTA (block_n >= 64), where padding the last block of each expert costs less
  // than the extra weight passes of narrow tiles (measured on B200).
  const double per_expert = (double)T * topk / (E > 0 ? E : 1);
  if (per_expert <= 12) return 16;
  if (per_expert <= 24) return 32;
  if (per_expert <= 48) return 64;
  if (per_expert <= 96) return 128;
  return 256;
}

extern "C" size_t fus_moe_block_workspace(const fus_moe_block_desc* d, int T, int block_n) {
  if (!d) return 0;
  if (block_n <= 0) block_n = fus_moe_block_pick_block_n(T, d->E, d->topk);
  BlockLayout L;
  if (!layout_for(d, T, block_n, L)) return 0;
  return L.total;
}

extern "C" int fus_moe_block_check(const fus_moe_block_desc* d, int T, int block_n,
                                   size_t ws_bytes) {
  if (!d) return set_error(FUS_E_INVALID, "moe_block: null argument");
  if (T < 0) return set_error(FUS_E_INVALID, "moe_block: T < 0");
  if (T == 0) return FUS_OK;
  if (!d->gamma || !d->wa || !d->w13 || !d->w2 || (!d->w13s) != (!d->w2s))
    return set_error(FUS_E_INVALID, "moe_block: missing weights");
  if (block_n <= 0) block_n = fus_moe_block_pick_block_n(T, d->E, d->topk);
  BlockLayout L;
  if (!layout_for(d, T, block_n, L)) return set_error(FUS_E_INVALID, "moe_block: bad sizes");
  if (ws_bytes < L.total)
    return set_error(FUS_E_INVALID, "moe_block: workspace %zu < %zu", ws_bytes, L.total);
  if (d->flags) return set_error(FUS_E_INVALID, "moe_block: flags must be 0");
  if (small_path(d, T))
    return route_small_check(T, d->H, d->E, d->topk, d->n_group, d->topk_group, block_n,
                             d->nplanes);
  return FUS_OK;
}

extern "C" int fus_moe_block_forward(const fus_moe_block_desc* d, const void* h, const void* r,
                                     int T, int block_n, void* out, void* h1, float* topw,
                                     int* topi, void* workspace, size_t ws_bytes, void* stream,
                                     int* status) {
  if (!d || !h || !r || !out || !h1 || !topw || !topi || !workspace)
    return set_error(FUS_E_INVALID, "moe_block: null argument");
  if (int rc = fus_moe_block_check(d, T, block_n, ws_bytes)) return rc;
  if (T == 0) return FUS_OK;
  if (block_n <= 0) block_n = fus_moe_block_pick_block_n(T, d->E, d->topk);
  BlockLayout L;
  layout_for(d, T, block_n, L);
  const int H = d->H, I = d->I, E = d->E, K = d->topk;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  auto at = [&](size_t off) { return base + off; };
  void* x2 = at(L.off_x2);
  float* partial = reinterpret_cast<float*>(at(L.off_partial));
  int* sorted = reinterpret_cast<int*>(at(L.off_sorted));
  int* eids = reinterpret_cast<int*>(at(L.off_eids));
  int* ntp = reinterpret_cast<int*>(at(L.off_ntp));
  void* align_ws = at(L.off_align);
  void* act = at(L.off_act);
  void* act_s = at(L.off_acts);
  void* y = at(L.off_y);
  void* ys = at(L.off_ys);
  int* counters = reinterpret_cast<int*>(at(L.off_cnt));
  int* done = reinterpret_cast<int*>(at(L.off_done));
  int* pos_of = reinterpret_cast<int*>(at(L.off_pos));
  void* xs = at(L.off_xs);
  const bool shared = d->w13s != nullptr;

  int rc;
  const bool small = small_path(d, T);
  if (small) {
    // decode: norm + router + top-k + layout in one launch; it also clears the merge
    // counters, so the down projection needs no separate reset
    if ((rc = route_small_launch(h, r, d->gamma, d->eps, d->wa, d->nplanes, d->bias, T, H, E, K,
                                 d->routed_scale, d->renorm, d->n_group, d->topk_group, h1, x2,
                                 partial, topw, topi, block_n, sorted, L.cap, eids, L.blocks_cap,
                                 ntp, done, counters, T * L.tiles, stream, status)))
      return rc;
  } else {
    if ((rc = fus_add_rmsnorm(h, H, r, H, d->gamma, h1, H, x2, H, T, H, d->eps, 1, 1, stream,
                              status)))
      return rc;
    if ((rc = fus_router_logits(x2, H, d->wa, d->nplanes, partial, T, H, E, L.nsplit, stream,
                                status)))
      return rc;
    if ((rc = fus_router_topk_grouped(partial, L.nsplit, d->bias, nullptr, topw, topi, T, E, K,
                                      d->n_group > 1 ? d->n_group : 1,
                                      d->topk_group > 1 ? d->topk_group : 1, d->routed_scale,
                                      d->renorm, stream, status)))
      return rc;
    // balanced layout: an expert just over a block fills two even blocks, not a full
    // block plus a few stragglers that stream the same weights again
    if ((rc = fus_moe_align_ex(topi, L.R, E, block_n, sorted, L.cap, eids, L.blocks_cap, ntp,
                               pos_of, FUS_ALIGN_BALANCED, align_ws,
                               fus_moe_align_workspace(L.R, E), stream, status)))
      return rc;
    if ((rc = fus_permute_rows(x2, H, sorted, ntp, K, L.R, xs, H, L.cap, H, stream, status)))
      return rc;
  }

  // weights stream past L2 when a typical expert fills at most one token block
  const int wstream = (double)L.R / E <= block_n ? FUS_GEMM_W_STREAM : 0;
  fus_gemm_group g[2] = {};
  // ---- w13 + SwiGLU: routed experts over xs (prefill) or x2, shared expert over x2 ----
  g[0].w = d->w13;
  g[0].n_experts = E;
  if (small) {
    // decode: a handful of rows per launch, gathered from x2 by dispatch position
    // (TMA gather4) instead of a separate permutation pass
    g[0].x = x2;
    g[0].x_rows = T;
    g[0].gather_ids = sorted;
    g[0].gather_div = K;
  } else {
    // prefill: one permutation pass, then dense box loads (gather4 moves 4 rows per TMA
    // operation: 64 operations per stage at 256 rows overwhelm the copy engine, 2.5x
    // slower than the permuted copy measured at T=2048-8192)
    g[0].x = xs;
    g[0].x_rows = L.cap;
  }
  g[0].ldx = H;
  g[0].expert_ids = eids;
  g[0].ntp = ntp;
  g[0].max_blocks = L.max_blocks;
  g[0].out = act;
  g[0].ldo = I;
  g[0].row_limit = L.cap;
  g[0].flags = FUS_GEMM_SWIGLU_EXACT | wstream;
  g[0].live_ids = sorted;
  g[0].live_limit = L.R;
  g[1].w = d->w13s;
  g[1].n_experts = 1;
  g[1].x = x2;
  g[1].ldx = H;
  g[1].x_rows = T;
  g[1].max_blocks = (T + block_n - 1) / block_n;
  g[1].out = act_s;
  g[1].ldo = I;
  g[1].row_limit = T;
  g[1].flags = FUS_GEMM_SWIGLU_EXACT | (T <= block_n ? FUS_GEMM_W_STREAM : 0);
  // decode: launched early (programmatic dependent launch) behind the front end
  if ((rc = grouped_gemm_launch(g, shared ? 2 : 1, 2 * I, H, 1, FUS_EPI_SWIGLU, block_n, 1, 0, 0,
                                nullptr, small ? 1 : 0, stream, status)))
    return rc;
  // ---- w2: routed rows to y[flat], shared rows to ys (fp32) ----
  g[0].w = d->w2;
  g[0].x = act;
  g[0].ldx = I;
  g[0].x_rows = L.cap;
  g[0].gather_ids = nullptr;
  g[0].out = y;
  g[0].ldo = H;
  g[0].row_map = sorted;
  g[0].row_limit = L.R;
  g[0].flags = wstream;
  g[0].token_div = K;
  g[1].w = d->w2s;
  g[1].x = act_s;
  g[1].ldx = I;
  g[1].out = ys;
  g[1].ldo = H;
  g[1].flags = FUS_GEMM_OUT_F32 | (T <= block_n ? FUS_GEMM_W_STREAM : 0);
  g[1].token_div = 1;
  if (!small) {
    // prefill: rows land in dispatch order (dense tile stores, no scatter); the merge is
    // a bandwidth-bound pass of its own (in GEMM epilogues it would be serialised behind
    // each CTA's MMAs)
    g[0].row_map = nullptr;
    g[0].row_limit = L.cap;
    if ((rc = fus_grouped_gemm(g, shared ? 2 : 1, H, I, 1, FUS_EPI_BF16, block_n, 1, 0, stream,
                               status)))
      return rc;
    return fus_merge_pos(y, H, pos_of, K, topw, K, h1, H, shared ? ys : nullptr, H, 1, out, H, T,
                         H, stream, status);
  }
  // decode: the CTA that lands the last contribution of a (token, tile) writes
  // out = bf16(sum_k w_k y_k + h1 + ys) for it (counters cleared by the front end)
  g[0].flags |= FUS_GEMM_MERGE;
  g[1].flags |= FUS_GEMM_MERGE;
  fus_merge_spec m{};
  m.counters = counters;
  m.parts = K + (shared ? 1 : 0);
  m.y = y;
  m.ld_t = (long)K * H;
  m.ld_k = H;
  m.topk = K;
  m.w = topw;
  m.ldw = K;
  m.res = h1;
  m.ldr = H;
  m.extra = shared ? reinterpret_cast<const float*>(ys) : nullptr;
  m.lde = H;
  m.out = out;
  m.ldo = H;
  // launched early; its weight tiles stream in while the w13 grid drains (expert ids
  // come from the front end, which finished before w13 started)
  return grouped_gemm_launch(g, shared ? 2 : 1, H, I, 1, FUS_EPI_BF16, block_n, 1, 0, 0, &m, 2,
                             stream, status);
}
