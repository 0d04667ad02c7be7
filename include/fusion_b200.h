/*
 * fusion_b200 — C ABI of the B200 (sm_100a) GLM-5.2 MoE-block hot path.
 *
 * Plain pointers, sizes and a CUDA stream; no torch types. Every entry point is
 * destination-passing (the caller allocates every output and workspace), enqueues
 * work on `stream` asynchronously and returns 0 on success or a negative FUS_E_*
 * code when an argument is rejected before anything was launched (the message is
 * available from fus_last_error()). Device-side problems (a pipeline wait that ran
 * out of time, an expert id out of range, a layout larger than its buffer) are
 * reported by OR-ing FUS_ERR_* bits into the optional device word `status`, which
 * the caller reads after synchronising.
 *
 * Reference interfaces (HansonZhang-cuhksz/fusion, glm52/) that each entry point
 * replaces are cited beside it as file:line.
 *
 * Layout conventions (same as the reference, glm52/config.py:61-64):
 *   activations  [T, H] bf16 row-major, row stride `ld*` in elements
 *   w13          [E, 2I, H] bf16  (rows [0,I) gate, [I,2I) up)
 *   w2           [E, H, I]  bf16
 *   router       [E, H] fp32 (nn.Linear); stored on device as bf16 planes
 *   topk ids     [T, topk] int32, weights [T, topk] fp32
 */
#ifndef FUSION_B200_H
#define FUSION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* host return codes */
#define FUS_OK 0
#define FUS_E_INVALID (-1)     /* bad argument (shape, alignment, null pointer) */
#define FUS_E_LAUNCH (-2)      /* CUDA reported an error when launching */
#define FUS_E_UNSUPPORTED (-3) /* shape outside what the kernels implement */

/* device status bits */
#define FUS_ERR_TIMEOUT 0x1    /* a pipeline wait exceeded its time budget */
#define FUS_ERR_BAD_EXPERT 0x2 /* an expert id outside [0, E) was seen */
#define FUS_ERR_CAPACITY 0x4   /* a layout did not fit the buffer it was given */

/* epilogues of fus_grouped_gemm */
#define FUS_EPI_BF16 0   /* out[row, n] = bf16(acc * scale[row]?)                         */
#define FUS_EPI_SWIGLU 1 /* out[row, n] = bf16(silu(acc_gate) * acc_up), w rows paired     */
#define FUS_EPI_F32 2    /* out[row, n] = acc (fp32), optional split-K partial planes      */

/* per-group epilogue flags (fus_gemm_group.flags) */
#define FUS_GEMM_OUT_F32 0x1      /* FUS_EPI_BF16 writes fp32 instead of bf16                */
#define FUS_GEMM_SWIGLU_EXACT 0x2 /* SwiGLU on fp32 gate/up; default rounds them to bf16     */
                                  /* first, as the framework's unfused chain does          */
#define FUS_GEMM_W_STREAM 0x4     /* each weight tile is read by one token block only:      */
                                  /* load it L2 evict-first (decode); default evict-normal */
#define FUS_GEMM_MERGE 0x8        /* this group's rows take part in the fused merge of     */
                                  /* fus_grouped_gemm_merge (token = row / token_div)      */
#define FUS_GEMM_SCALE_TOKEN 0x20 /* row_scale is indexed by token = row / token_div       */
                                  /* (lazy pre-norm: the token's rstd), not by row          */
#define FUS_GEMM_NO_PERSIST 0x10  /* (first group) keep one tile per CTA; by default wide- */
                                  /* tile launches with many tiles run one persistent CTA  */
                                  /* per SM that overlaps each epilogue with the next loads */
#define FUS_GEMM_NO_PAIR 0x40     /* (first group) no SM-pair (2-CTA cluster, M = 256)     */
                                  /* tiles; by default persistent launches with 256-token  */
                                  /* blocks and dense outputs use them                     */
#define FUS_GEMM_PAIR_NARROW 0x80 /* (first group) FUS_EPI_BF16 SM-pair tiles of 256 rows  */
                                  /* (one weight tile per CTA, TMEM double-buffered); by  */
                                  /* default 512-row tiles (two weight tiles per CTA      */
                                  /* share each staged token tile) when w_rows allows     */

int fus_version(void);
const char* fus_last_error(void);
int fus_num_sms(void);

/* ---------------------------------------------------------------------------------
 * ResAdd + RMSNorm (fusion #3).
 * Replaces glm52/kernels/add_rmsnorm.py:234 fused_add_rmsnorm (do_add=1, do_norm=1),
 * :239 add_only (do_norm=0) and :244 norm_only (do_add=0, x is h1).
 *   h1  = bf16(x + res)
 *   out = bf16( bf16(h1 * rsqrt(mean(h1^2) + eps)) * w )      (reference.py:22-33)
 * ------------------------------------------------------------------------------- */
int fus_add_rmsnorm(const void* x, long ldx, const void* res, long ldr, const void* w,
                    void* h1, long ldh, void* out, long ldo, int T, int N, float eps,
                    int do_add, int do_norm, void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * Router weights. The router GEMM runs on the tensor cores in bf16 with fp32
 * accumulation over `nplanes` bf16 planes whose sum is the weight:
 *   fp32 weight  -> 3 planes hi/mid/lo, exact (every fp32 is the sum of 3 bf16)
 *   bf16 weight  -> 1 plane
 * fus_router_split_weight: wg [E,H] fp32 -> wa [E, 3H] bf16 (planes along K).
 * fus_router_transpose_weight: wgt [H,E] bf16 (the layout of
 *   glm52/kernels/norm_router.py:251-255 wgt_from_gate) -> wa [E,H] bf16.
 * ------------------------------------------------------------------------------- */
int fus_router_split_weight(const float* wg, void* wa, int E, int H, void* stream);
int fus_router_transpose_weight(const void* wgt, void* wa, int H, int E, void* stream);

/* Router GEMM (glm52/kernels/norm_router.py:347 router_gemm; reference.py:61):
 * partial[s, t, e] = sum over the s-th K split of x2[t,:] . wa[e, :] (fp32).
 * Summing the nsplit planes (fus_router_topk does, in fixed order) gives
 * logits = x2.float() @ W.float().T. Use fus_router_nsplit() for nsplit. Up to
 * T = 16 tokens it is a CUDA-core fp32 GEMV over the reassembled weight (nsplit 1);
 * above, the tcgen05 grouped GEMM over the planes. */
int fus_router_nsplit(int T, int H, int E, int nplanes);
int fus_router_logits(const void* x2, long ldx, const void* wa, int nplanes, float* partial,
                      int T, int H, int E, int nsplit, void* stream, int* status);

/* Router selection (reference.py:62-79; glm52/kernels/norm_router.py:352 topk_only):
 *   logits = sum_s partial[s]; s = sigmoid(logits); choice = s + bias (bias may be NULL)
 *   ids = top-k of choice, descending (ties: lower expert id first)
 *   w = s[ids]; if renorm: w /= max(sum(w), 1e-20); w *= scale
 * logits_out (optional) receives the summed logits [T, E]. E <= 256, topk <= 16. */
int fus_router_topk(const float* partial, int nsplit, const float* bias, float* logits_out,
                    float* topw, int* topi, int T, int E, int topk, float scale, int renorm,
                    void* stream, int* status);
/* Same with noaux_tc group masking (reference.py:159-166, DeepSeek-V3-style configs):
 * experts form n_group groups of E/n_group consecutive ids; a group's score is the sum
 * of its two largest choice values; experts outside the topk_group best groups (ties:
 * lower group index) get choice * 0 before the top-k. Groups of 8*2^j experts,
 * n_group <= 32. n_group = 1 is fus_router_topk (GLM-5.2). */
int fus_router_topk_grouped(const float* partial, int nsplit, const float* bias,
                            float* logits_out, float* topw, int* topi, int T, int E, int topk,
                            int n_group, int topk_group, float scale, int renorm, void* stream,
                            int* status);

/* ---------------------------------------------------------------------------------
 * Dispatch layout (glm52/reference.py:85-128 moe_align_block_size, sglang layout):
 *   stable sort of the flat (token*topk+k) indices by expert, each expert's run
 *   padded to a multiple of block_m with the sentinel `numel`;
 *   expert_ids[b] = expert of block b; ntp[0] = padded total.
 * Negative ids are holes: their flat index is simply not placed (no error); ids >= E
 * raise FUS_ERR_BAD_EXPERT. The pad sentinel stays `numel`.
 * sorted_cap >= numel + E*(block_m-1) and blocks_cap >= sorted_cap/block_m are
 * always enough. Entries past ntp[0] are left untouched. `workspace` of
 * fus_moe_align_workspace(numel, E) bytes (may be 0 for small numel). E <= 512.
 * ------------------------------------------------------------------------------- */
size_t fus_moe_align_workspace(int numel, int E);
int fus_moe_align(const int* ids, int numel, int E, int block_m, int* sorted_ids, int sorted_cap,
                  int* expert_ids, int blocks_cap, int* ntp, void* workspace, size_t ws_bytes,
                  void* stream, int* status);
/* Same, with options. pos_of (optional, numel entries): each pair's dispatch position,
 * pos_of[i] = p where sorted_ids[p] = i (holes / invalid ids left untouched).
 * flags: FUS_ALIGN_BALANCED spreads each expert's c pairs evenly over its
 * nb = ceil(c / block_m) blocks (ceil(c / nb) per block, each block's pads after its
 * pairs) instead of filling blocks in order; padded sizes, expert_ids and ntp are
 * unchanged. Not the reference's layout: for callers that own the layout (the block). */
#define FUS_ALIGN_BALANCED 0x1
int fus_moe_align_ex(const int* ids, int numel, int E, int block_m, int* sorted_ids,
                     int sorted_cap, int* expert_ids, int blocks_cap, int* ntp, int* pos_of,
                     int flags, void* workspace, size_t ws_bytes, void* stream, int* status);

/* Same result as fus_moe_align, but the call allocates nothing and takes no workspace.
 * No counterpart in the reference. It is for callers that cannot allocate device
 * memory: engines whose memory pool owns nearly all of HBM from start-up (the KV cache
 * takes what is left, so a later cudaMalloc fails), and callers that cannot pay the
 * device-wide synchronisation cudaMalloc / cudaFree imply inside a serving loop.
 * Scratch is a fixed array inside the library (397,568 bytes on every GPU that loads
 * it, held until the process exits), so the limits are numel <= 65536 (T <= 8192 at
 * top-8) and E <= 512; larger inputs are rejected with FUS_E_UNSUPPORTED. The first
 * call on each device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture. All calls on a
 * device share the array: calls that may overlap on the GPU (different streams, no
 * ordering between them) race and corrupt each other's layout. The looked-up address is
 * kept for the life of the process: after cudaDeviceReset on a device it is stale, so do
 * not call this entry again on that device. */
int fus_moe_align_noalloc(const int* ids, int numel, int E, int block_m, int* sorted_ids,
                          int sorted_cap, int* expert_ids, int blocks_cap, int* ntp, void* stream,
                          int* status);

/* Decode front end in one launch (T <= 16): add_rmsnorm + fp32 router + top-k + dispatch
 * layout (replaces fus_add_rmsnorm + fus_router_logits + fus_router_topk +
 * fus_moe_align for small T). Every CTA normalises the T rows into shared memory and
 * computes the logits of one expert; the last CTA to finish selects the top-k and
 * builds the layout (block_m = 0: no layout; sorted_ids, expert_ids and ntp may then be
 * NULL). `done` is an int that must be zero before the first call (each call leaves it
 * zero); `zero`/`zero_n` optionally names an int buffer the call clears (the fused
 * merge's counters). Requires E <= 256, E % 2 == 0, T*topk <= 256. */
int fus_moe_route_small(const void* h, const void* r, const void* gamma, float eps, const void* wa,
                        int nplanes, const float* bias, int T, int H, int E, int topk,
                        float scale, int renorm, void* h1, void* x2, float* logits, float* topw,
                        int* topi, int block_m, int* sorted_ids, int sorted_cap, int* expert_ids,
                        int blocks_cap, int* ntp, int* done, int* zero, int zero_n, void* stream,
                        int* status);

/* Row permutation into dispatch order (the A gather `offs_token // top_k` of
 * glm52/kernels/moe_gateup.py:96-99, done once up front so the GEMM reads dense rows):
 *   dst[p] = src[sorted_ids[p] / div]  if sorted_ids[p] < num_valid,
 * for p < min(ntp[0], max_rows); pad rows are left untouched (the GEMMs do not
 * multiply dispatch pads). H % 8 == 0, 16-byte aligned rows. */
int fus_permute_rows(const void* src, long ld_src, const int* sorted_ids, const int* ntp, int div,
                     int num_valid, void* dst, long ld_dst, int max_rows, int H, void* stream,
                     int* status);

/* ---------------------------------------------------------------------------------
 * Grouped expert GEMM on tcgen05 tensor cores (replaces the Triton grouped GEMMs
 * glm52/kernels/moe_gateup.py:199 launch_gateup and
 * glm52/kernels/moe_down_merge.py:427 launch_down).
 *
 * Each group is one weight stack and one set of token rows. Token rows are cut into
 * blocks of `block_n`; block b belongs to expert expert_ids[b]. For every block and
 * every 128-row weight tile the kernel computes
 *     acc[n, j] = sum_k w[e, n, k] * x[b*block_n + j, k]
 * (the weight is the MMA's M side, tokens its N side), then the epilogue writes
 * output row  r = row_map ? row_map[b*block_n + j] : b*block_n + j  (skipped if
 * r >= row_limit) with:
 *   FUS_EPI_BF16   out[r, n]           = bf16(acc * (row_scale ? row_scale[r] : 1))
 *                  (fp32 with FUS_GEMM_OUT_F32)
 *   FUS_EPI_SWIGLU out[r, n]  n < w_rows/2 = bf16(silu(g) * u),  g = bf16(acc[n]),
 *                  u = bf16(acc[n + w_rows/2])  (unrounded with FUS_GEMM_SWIGLU_EXACT)
 *   FUS_EPI_F32    out[s][r, n]        = acc over the s-th of `ksplit` K ranges
 * The weight's K extent may be `a_kplanes` times the token K (bf16 planes of one
 * fp32 weight): token columns wrap, so all planes accumulate against the same x.
 * Requirements: K % 64 == 0, w_rows % 128 == 0, 16-byte aligned rows,
 * block_n in {16, 32, 64, 128, 256}.
 * ------------------------------------------------------------------------------- */
typedef struct fus_gemm_group {
  const void* w;          /* [n_experts, w_rows, a_kplanes*K] bf16                        */
  int n_experts;
  const void* x;          /* token rows [x_rows, K] bf16, row stride ldx elements          */
  long ldx;
  int x_rows;
  const int* expert_ids;  /* per block; NULL: every block uses expert 0                    */
  const int* ntp;         /* device int, rows of x in use; NULL: x_rows                    */
  int max_blocks;         /* blocks launched for this group (extra blocks exit at once)    */
  void* out;              /* output, row stride ldo elements                               */
  long ldo;
  const int* row_map;     /* NULL: identity                                                */
  int row_limit;
  const float* row_scale; /* optional, FUS_EPI_BF16 only                                   */
  int flags;              /* FUS_GEMM_* bits                                               */
  const int* live_ids;    /* optional: column j of block b is live iff                     */
  int live_limit;         /*   live_ids[b*block_n + j] < live_limit; dead columns sit at   */
                          /*   the end of a block (dispatch pads) and are not multiplied   */
                          /*   (the MMA N shrinks); with row_map NULL their output rows    */
                          /*   (< row_limit) may receive unspecified values                */
  int token_div;          /* FUS_GEMM_MERGE: token of output row r is r / token_div        */
  const int* gather_ids;  /* optional: token rows are gathered, not read densely: row j of */
  int gather_div;         /*   block b is x[gather_ids[b*block_n+j] / gather_div] when that */
                          /*   id is live (< live_limit), zeros otherwise (TMA gather4)     */
  const void* res;        /* optional, FUS_EPI_BF16: bf16 residual added before the output */
  long ldr;               /*   rounding, out[r, n] = bf16(acc + res[r, n]) (o_proj+ResAdd)  */
} fus_gemm_group;

int fus_grouped_gemm(const fus_gemm_group* groups, int ngroups, int w_rows, int K, int a_kplanes,
                     int epilogue, int block_n, int ksplit, long split_stride, void* stream,
                     int* status);
/* Same, with `group_blocks` consecutive token blocks swept across all weight tiles before
 * the next group of blocks starts (0 = pick from block counts): blocks of one expert then
 * share each weight tile through L2 while their token rows stay resident. */
int fus_grouped_gemm_ex(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                        int a_kplanes, int epilogue, int block_n, int ksplit, long split_stride,
                        int group_blocks, void* stream, int* status);

/* Down projection with the expert merge fused into its epilogue (replaces
 * glm52/kernels/moe_down_merge.py:427 launch_down + :504 launch_moe_sum / the F10
 * merge, reference.py:159-188). Groups flagged FUS_GEMM_MERGE write their rows as
 * fus_grouped_gemm does (epilogue FUS_EPI_BF16; fp32 rows with FUS_GEMM_OUT_F32), then
 * count, per (token, weight tile), how many of the `parts` contributions have landed.
 * The CTA that lands the last one computes, in a fixed order (deterministic),
 *   out[t, f] = bf16( sum_k w[t,k] * y[t,k,f] + res[t,f] + extra[t,f] )
 * for that tile's features and resets the counter. `counters` ([T * tiles] ints, tiles
 * = fus_grouped_gemm_tiles()) must be zero before the first call; every call leaves
 * them zero. */
typedef struct fus_merge_spec {
  int* counters;
  int parts;            /* contributions per token: topk (+1 with a shared expert)        */
  const void* y;        /* bf16 routed rows, row (t, k) at y + t*ld_t + k*ld_k            */
  long ld_t, ld_k;
  int topk;
  const float* w;       /* [T, topk] routing weights, row stride ldw                      */
  long ldw;
  const void* res;      /* bf16 [T, H] residual (h1) or NULL                              */
  long ldr;
  const float* extra;   /* fp32 [T, H] shared-expert output or NULL                       */
  long lde;
  void* out;            /* bf16 [T, H]                                                     */
  long ldo;
} fus_merge_spec;

int fus_grouped_gemm_tiles(int w_rows, int epilogue, int block_n);
int fus_grouped_gemm_merge(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                           int block_n, const fus_merge_spec* merge, void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * o_proj GEMM + ResAdd1 (glm52/kernels/oproj_resadd.py:144 gemm_launch / :181
 * epilogue_launch / :199 make_fused_chain / :216 make_unfused_chain;
 * glm52/bench/bench_layer.py:399-415):
 *   fuse = 1: out = bf16(a @ W + res)            (fp32 sum, one rounding)
 *   fuse = 0: out = bf16(bf16(a @ W) + res)      (the unfused chain's c, then the add)
 * a [T, K] bf16 (row stride lda), W K-major [N, K] bf16 (the reference's w_o [K, N]
 * transposed once), res [T, N] bf16 or NULL. N % 128 == 0, K % 64 == 0. T <= 64 splits K
 * into fp32 partial planes summed in fixed order (deterministic). The workspace size
 * comes from fus_oproj_workspace. */
size_t fus_oproj_workspace(int T, int N, int K, int fuse);
int fus_oproj_resadd(const void* a, long lda, const void* w, int T, int N, int K, const void* res,
                     long ldr, void* out, long ldo, int fuse, void* workspace, size_t ws_bytes,
                     void* stream, int* status);
/* The reference's split-K form with an fp32 accumulator (gemm_launch atomic_out=True and
 * epilogue_launch over acc32): fus_oproj_gemm_f32: acc32 (+)= a @ W (+ res) (+= when
 * accumulate); fus_oproj_finish: out = bf16(acc32 (+ res)). */
size_t fus_oproj_f32_workspace(int T, int N, int K);
int fus_oproj_gemm_f32(const void* a, long lda, const void* w, int T, int N, int K,
                       const void* res, long ldr, float* acc32, long ldc, int accumulate,
                       void* workspace, size_t ws_bytes, void* stream, int* status);
int fus_oproj_finish(const float* acc32, long ldc, const void* res, long ldr, void* out, long ldo,
                     int T, int N, void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * Lazy pre-norm, half fused (F11b', glm52/kernels/lazy_prenorm.py): the affine RMSNorm
 * weight w is folded into the next GEMM's K dimension once at load, the GEMM reads the
 * un-normalised h1 and its output rows are scaled by rstd afterwards.
 * fus_row_rstd: rstd[t] = 1/sqrt(mean_k x[t,k]^2 + eps)          (lazy_prenorm.py:347)
 * fus_fold_weight: dst = bf16(src * w) along K: by_row = 1 scales row r of a [K, N]
 *   weight by w[r % wdiv] (fold_weight_rowmajor), by_row = 0 scales column c of an
 *   [.., N, K] weight by w[c] (fold_weight_nk)                      (lazy_prenorm.py:75-86)
 * fus_scale_sum_planes: out[t, n] = row_scale[t] * sum_s partial[s, t, n] (fp32; the
 *   router GEMM's partial planes with the rstd epilogue; row_scale may be NULL)
 * The grouped GEMM applies a token's rstd with row_scale + FUS_GEMM_SCALE_TOKEN. */
int fus_row_rstd(const void* x, long ldx, int T, int N, float eps, float* rstd, void* stream,
                 int* status);
int fus_fold_weight(const void* src, const void* w, void* dst, long rows, int cols, int by_row,
                    long wdiv, void* stream, int* status);
int fus_scale_sum_planes(const float* partial, int nsplit, long plane, int T, int N,
                         const float* row_scale, float* out, long ldo, void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * Checkpoint ingest: FP8 (e4m3) weights with one fp32 scale per br x bc block (the
 * `weight_scale_inv` of block-quantised MoE checkpoints), dequantised to bf16 at load:
 *   dst[r, c] = bf16(fp8(src[r, c]) * scale[(r / br) * scale_ld + c / bc])
 * rows x cols row-major, cols % 8 == 0, bc % 8 == 0. */
int fus_fp8_block_dequant(const void* src, const float* scale, long scale_ld, void* dst, long rows,
                          int cols, int br, int bc, void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * Element-wise / merge kernels
 * ------------------------------------------------------------------------------- */
/* glm52/kernels/moe_gateup.py:251 launch_silu_and_mul; reference.py:36-40:
 *   y[m, i] = bf16(silu(x[m, i]) * x[m, I + i]) */
int fus_silu_and_mul(const void* x, long ldx, void* y, long ldy, int M, int I, void* stream,
                     int* status);

/* Merge (glm52/kernels/merge_resadd.py:243-255, moe_down_merge.py:504 launch_moe_sum,
 * reference.py:159-188 expert_merge):
 *   m   = sum_k (w ? w[t,k] : 1) * y[t,k,:]                  (fp32, k in order)
 *   if round_mid: m = bf16(m)
 *   out = bf16(m + res[t] + extra[t])      (res / extra optional, fp32 sum)
 * y rows: y + t*ld_t + k*ld_k. `extra` is bf16, or fp32 when extra_f32 != 0 (the
 * shared expert's unrounded output, glm52_h200/reference.py:294-311). */
int fus_merge(const void* y, long ld_t, long ld_k, int K, const float* w, long ldw,
              const void* res, long ldr, const void* extra, long lde, int extra_f32, void* out,
              long ldo, int T, int H, int round_mid, void* stream, int* status);
/* fus_merge over expert rows stored in dispatch order: row (t, k) is
 * y + pos_of[t*K + k]*ldy (round_mid = 0); pos_of as written by fus_moe_align_ex. */
int fus_merge_pos(const void* y, long ldy, const int* pos_of, int K, const float* w, long ldw,
                  const void* res, long ldr, const void* extra, long lde, int extra_f32,
                  void* out, long ldo, int T, int H, void* stream, int* status);

/* moe_down_merge.py:532 launch_resadd / merge_resadd.py:253 resadd_only:
 *   o = bf16(a + b) */
int fus_add(const void* a, long lda, const void* b, long ldb, void* o, long ldo, int M, int N,
            void* stream, int* status);

/* moe_down_merge.py:551 launch_seed: o = from_src ? src : 0 */
int fus_seed(void* o, long ldo, const void* src, long lds, int M, int N, int from_src,
             void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * Whole MoE block (glm52/bench/bench_layer.py:395-481 build_chain without o_proj,
 * oracle composition bench_layer.py:365-374):
 *   h1, x2  = add_rmsnorm(h, r, gamma)
 *   ids, w  = router(x2, W_g, bias)                   (sigmoid, noaux_tc, top-k)
 *   layout  = moe_align(ids, block_n)
 *   act     = silu(x2 W13_gate^T) * (x2 W13_up^T)     per routed expert + shared
 *   y       = act W2^T
 *   out     = bf16( sum_k w_k y_k + h1 + y_shared )   (fp32 sum; x2, act, y stored bf16)
 * block_n = 0 picks the token tile from T. The workspace holds every intermediate and
 * two sets of counters; it must be all zero before its first use (every call leaves
 * the counters zero again).
 * ------------------------------------------------------------------------------- */
typedef struct fus_moe_block_desc {
  int H, I, E, topk;
  float eps, routed_scale;
  int renorm;
  const void* gamma;  /* [H] bf16                                 */
  const void* wa;     /* router planes [E, nplanes*H] bf16        */
  int nplanes;        /* 3 for an fp32 router weight, 1 for bf16  */
  const float* bias;  /* [E] fp32 e_score_correction_bias or NULL */
  const void* w13;    /* [E, 2I, H] bf16                          */
  const void* w2;     /* [E, H, I] bf16                           */
  const void* w13s;   /* shared expert [2I, H] bf16 or NULL       */
  const void* w2s;    /* shared expert [H, I] bf16 or NULL        */
  int n_group;        /* noaux_tc groups (0 or 1: none; GLM-5.2)  */
  int topk_group;     /* groups kept when n_group > 1             */
  int flags;          /* reserved, must be 0                      */
} fus_moe_block_desc;

int fus_moe_block_pick_block_n(int T, int E, int topk);
size_t fus_moe_block_workspace(const fus_moe_block_desc* d, int T, int block_n);
/* Every argument check fus_moe_block_forward makes before its first launch, on the host
 * only (no device access; weight pointers are only compared with NULL and 16-byte
 * alignment): FUS_OK exactly when forward would reach its kernels with these sizes. */
int fus_moe_block_check(const fus_moe_block_desc* d, int T, int block_n, size_t ws_bytes);
int fus_moe_block_forward(const fus_moe_block_desc* d, const void* h, const void* r, int T,
                          int block_n, void* out, void* h1, float* topw, int* topi,
                          void* workspace, size_t ws_bytes, void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * Expert parallelism (no reference counterpart: the reference is single-GPU,
 * log/LOG-00-plan-and-filter.md:41). Rank g owns experts [g*E_loc, (g+1)*E_loc); the
 * row exchange is NCCL all_to_all (torch.distributed) between these steps.
 * fus_ep_plan  : for each of the R (token, slot) pairs: dest rank = topi / E_loc,
 *                leid = topi % E_loc, counts[W] = pairs per destination. W <= 64.
 * fus_ep_pack  : rows[p] = x[send_ids[p] / div]; leid_out[p] = leid[send_ids[p]]
 *                (leid may be NULL). send_ids = pairs stably sorted by dest, e.g.
 *                fus_moe_align(dest, R, W, 1, ...).
 * fus_ep_unpack: y[send_ids[p]] = rows[p]  (returned expert rows back to slot order)
 * ------------------------------------------------------------------------------- */
int fus_ep_plan(const int* topi, int R, int E_loc, int W, int* dest, int* leid, int* counts,
                void* stream, int* status);
/* Fixed-slot dispatch for small batches (T*topk <= 1024), no host synchronisation: the
 * send buffer has W blocks of S slots (S >= T*topk); pair i = (t, k) with destination d
 * takes slot d*S + (its stable rank among the pairs to d). Writes rows[slot] =
 * x[t], leid_out[slot] = local expert (-1 in unused slots), slot_of_pair[i]. */
int fus_ep_dispatch_small(const void* x, long ldx, int H, const int* topi, int T, int topk,
                          int E_loc, int W, int S, void* rows, long ldr, int* leid_out,
                          int* slot_of_pair, void* stream, int* status);
int fus_ep_pack(const void* x, long ldx, int H, const int* send_ids, int n, int div,
                const int* leid, void* rows, long ldr, int* leid_out, void* stream, int* status);
int fus_ep_unpack(const void* rows, long ldr, int H, const int* send_ids, int n, void* y, long ldy,
                  void* stream, int* status);
/* Deduplicated dispatch (prefill): a token's row travels once to each rank that owns at
 * least one of its experts (not once per (token, slot) pair).
 * fus_ep_plan_dedup : keys[t*W + d] = d if token t has an expert on rank d, else -1;
 *                     counts[2W] = rows, then (token, slot) pairs, per destination
 *                     (zeroed here). Sorting keys stably (fus_moe_align(keys, T*W, W, 1,
 *                     ...)) gives send_ids = t*W + d.
 * fus_ep_pack_dedup : row p (id = send_ids[p] = t*W + d): rows[p] = x[t]; for k < K:
 *                     leid_out[p*K + k] = local expert of slot k if its expert is on d,
 *                     else -1 (K <= 32). Optional outputs:
 *                     ret_out[p*K + k] = the pair's index among this rank's pairs for d
 *                       (pair_pos: each pair's position in the pairs stably sorted by
 *                       destination, counts as above; -1 off d);
 *                     w_out / pos (together): slot weight (0 off d); pos[t*K + k] = p for
 *                       the first slot of t on d, zero_row for its other slots on d.
 * fus_ep_return_rowmap: owner side, the w2 row map that writes each received pair's
 *                     expert row at its place in the return buffer: layout entry x with
 *                     slot f = sorted_ids[x] < n*K of row i = f / K from source s
 *                     (row_prefix[s] <= i < row_prefix[s+1]) -> pair_prefix[s] +
 *                     ret_idx[f]; pads stay >= n*K. row_prefix / pair_prefix: W+1 ints.
 *                     ntp: the layout's padded total (moe_align's ntp; entries from it on
 *                     are never read and map to n*K) or NULL when all cap entries are set.
 * fus_ep_partial_sum: owner side, out[i] = bf16(sum_{j: leid[i*K+j] >= 0} w[i*K+j] *
 *                     y[i*K+j]) in fp32, slot order (y: expert rows in slot order).
 * Pair combine (exact): the owner returns one expert row per pair, the source merges
 * with fus_merge_pos(ret, pair_pos, K, topw, h1, shared), as on one GPU. Partial-sum
 * combine (fewer bytes, the partial is rounded to bf16 before the final sum): one row
 * per (token, rank) returns and fus_merge_pos(ret, pos, K, w = NULL, h1, shared) with
 * ret row zero_row zero. */
int fus_ep_plan_dedup(const int* topi, int T, int K, int E_loc, int W, int* keys, int* counts,
                      void* stream, int* status);
int fus_ep_pack_dedup(const void* x, long ldx, int H, const int* send_ids, int n, int W,
                      const int* topi, const float* topw, int K, int E_loc, const int* pair_pos,
                      const int* counts, void* rows, long ldr, int* leid_out, int* ret_out,
                      float* w_out, int* pos, int zero_row, void* stream, int* status);
int fus_ep_return_rowmap(const int* sorted_ids, int cap, const int* ntp, const int* ret_idx,
                         int n, int K,
                         const int* row_prefix, const int* pair_prefix, int W, int* rowmap,
                         void* stream, int* status);
int fus_ep_partial_sum(const void* y, long ldy, int H, const int* leid, const float* w, int n,
                       int K, void* out, long ldo, void* stream, int* status);

/* Row exchange over NVLink peer memory for the fixed-slot (decode) step, replacing the
 * three all_to_alls with direct peer stores and flag waits. Every rank exports one
 * exchange buffer through CUDA IPC and maps the others':
 *   recv_rows [W*S][H] bf16 (block w: rows from rank w), recv_leid [W*S] int32 (-1 =
 *   unused slot), ret_rows [W*S][H] bf16 (block d: expert rows returned by rank d),
 *   dflags [W], cflags [W] int32 (zero before the first step), epoch (int, zero).
 * peer_* arguments are device arrays of W addresses (rank w's buffer at index w, this
 * rank's own included).
 * fus_ep_p2p_dispatch: epoch += 1; pair (t, k) whose owner is d, j-th of this rank's
 *   pairs to d: recv_rows_d[rank*S + j] = x[t], recv_leid_d[rank*S + j] = local expert
 *   (others of the block -1), slot_of_pair[t*topk + k] = d*S + j; then dflags_d[rank] =
 *   epoch at every d (release, system scope). T*topk <= min(S, 1024).
 * fus_ep_p2p_wait: until flags[w] >= epoch for every w; after timeout_ns (0 = 1 s,
 *   the maximum) sets FUS_ERR_TIMEOUT in *status and returns.
 * fus_ep_p2p_combine: for every live slot i = w*S + j of recv_leid:
 *   ret_rows_w[rank*S + j] = y[i]; then cflags_w[rank] = epoch at every w.
 * The merge then reads row (t, k) at ret_rows[slot_of_pair[t*topk + k]]
 * (fus_merge_pos). fus_ipc_handle / fus_ipc_open / fus_ipc_close wrap CUDA IPC for an
 * address inside any device allocation (handle = 64 bytes + the offset from the
 * allocation's base). */
int fus_ipc_handle(const void* ptr, void* handle_out, size_t* offset_out);
int fus_ipc_open(const void* handle, size_t offset, void** ptr_out);
int fus_ipc_close(void* ptr, size_t offset);
int fus_ep_p2p_dispatch(const void* x, long ldx, int H, const int* topi, int T, int topk,
                        int E_loc, int W, int S, int rank, const unsigned long long* peer_rows,
                        const unsigned long long* peer_leid,
                        const unsigned long long* peer_flags, int* epoch, int* slot_of_pair,
                        void* stream, int* status);
int fus_ep_p2p_wait(const int* flags, const int* epoch, int W, unsigned long long timeout_ns,
                    void* stream, int* status);
int fus_ep_p2p_combine(const void* y, long ldy, int H, const int* recv_leid, int W, int S,
                       int rank, const unsigned long long* peer_ret,
                       const unsigned long long* peer_cflags, const int* epoch, void* stream,
                       int* status);

/* The whole expert-parallel decode step of one rank over the NVLink exchange, as seven
 * launches chained with programmatic dependent launch: fused norm + router + top-k,
 * dispatch, [wait for every source + layout of the received slots], w13 + SwiGLU
 * (received rows gathered, shared expert as a second group), w2, combine, [wait for
 * every owner + merge]. blk->E counts all experts and blk->w13 / w2 hold this rank's
 * E_loc = E / W experts; S >= T*topk; the exchange buffers as described above.
 * Requires the fused front end (E <= 256, E even, T*topk <= 256). The workspace must be
 * zeroed before its first use (a front-end ticket that each call leaves at zero). */
typedef struct fus_ep_p2p_desc {
  const fus_moe_block_desc* blk;
  int E_loc, W, rank, S;
  const unsigned long long* peer_rows;    /* [W] every rank's recv_rows   */
  const unsigned long long* peer_leid;    /* [W] every rank's recv_leid   */
  const unsigned long long* peer_dflags;  /* [W] every rank's dflags      */
  const unsigned long long* peer_ret;     /* [W] every rank's ret_rows    */
  const unsigned long long* peer_cflags;  /* [W] every rank's cflags      */
  void* recv_rows;                        /* this rank's buffers          */
  int* recv_leid;
  void* ret_rows;
  int* dflags;
  int* cflags;
  int* epoch;
} fus_ep_p2p_desc;
size_t fus_ep_p2p_decode_workspace(const fus_ep_p2p_desc* d, int T);
int fus_ep_p2p_decode_forward(const fus_ep_p2p_desc* d, const void* h, const void* r, int T,
                              void* out, void* h1, float* topw, int* topi, void* workspace,
                              size_t ws_bytes, void* stream, int* status);

/* ---------------------------------------------------------------------------------
 * Seeded synthetic inputs, bit-identical on the GPU and the host (no reference
 * counterpart: the reference draws torch.randn on the device, which a CPU oracle
 * cannot reproduce). Element i of a stream is
 *   mean + std * z_i,  z_i = (sum of 12 uniform 16-bit draws - 393210) / 65536
 * (Irwin-Hall approximation of N(0,1)), rounded to the destination type; i runs
 * from `offset` so any slice (one expert) can be regenerated alone.
 * dtype 0 = bf16, 1 = fp32.
 * ------------------------------------------------------------------------------- */
int fus_synth_fill(void* dst, int dtype, long n, long offset, unsigned long long seed, float mean,
                   float std, void* stream);
void fus_synth_fill_host(void* dst, int dtype, long n, long offset, unsigned long long seed,
                         float mean, float std);

#ifdef __cplusplus
}
#endif
#endif /* FUSION_B200_H */
