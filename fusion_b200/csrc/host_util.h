// Host-side helpers shared by the C-ABI translation units: error reporting, launch
// checks and TMA tensor-map encoding (driver entry point fetched through the runtime,
// so the library links only against cudart).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fusion_b200.h"

namespace fus {

// Records a printf-style message retrievable by fus_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
// Turns a pending launch error into FUS_E_LAUNCH.
int check_launch(const char* what);
// Encodes a 2D bf16 tensor map with 128-byte swizzle: `inner` contiguous elements per
// row, `rows` rows, row pitch `ld` elements, box = box_inner x box_rows.
int make_tmap_bf16_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t ld,
                      uint32_t box_inner, uint32_t box_rows);
// row-major output tile map for TMA stores (no swizzle: the staging tile is row-major)
int make_tmap_store_2d(CUtensorMap* m, const void* base, bool f32, uint64_t inner, uint64_t rows,
                       uint64_t ld, uint32_t box_inner, uint32_t box_rows);
int num_sms();
// Raises `fn`'s dynamic shared-memory limit to `bytes` on the current device, once per
// (kernel, device): the attribute is per device, so a process that drives several GPUs
// sets it on each. Thread-safe. Returns FUS_OK or FUS_E_LAUNCH with the CUDA error text.
int ensure_smem_attr(const void* fn, int bytes, const char* what);

// Grouped GEMM entry used inside the library with programmatic dependent launch:
// pdl = 0 plain launch; 1 launched early, every thread waits for the predecessor before
// reading anything; 2 launched early, the dispatch layout is older than the predecessor
// so weight tiles are prefetched before waiting (token rows are loaded after the wait).
int grouped_gemm_launch(const fus_gemm_group* groups, int ngroups, int w_rows, int K,
                        int a_kplanes, int epilogue, int block_n, int ksplit, long split_stride,
                        int group_blocks, const fus_merge_spec* merge, int pdl, void* stream,
                        int* status);

// expert-parallel receive side: the single-CTA dispatch layout of `ids` after every
// flags[w] >= *epoch (w < W), and the merge over rows in dispatch order after the same
// kind of wait (pdl: launched as a programmatic dependent of the previous kernel)
int moe_align_small_after_flags(const int* flags, const int* epoch, int W, const int* ids,
                                int numel, int E, int block_m, int* sorted_ids, int sorted_cap,
                                int* expert_ids, int blocks_cap, int* ntp, int pdl, void* stream,
                                int* status);
int merge_pos_after_flags(const void* y, long ldy, const int* pos_of, int K, const float* w,
                          long ldw, const void* res, long ldr, const void* extra, long lde,
                          int extra_f32, void* out, long ldo, int T, int H, const int* flags,
                          const int* epoch, int W, int pdl, void* stream, int* status);

// o_proj split-K finish: out = bf16(sum of S fp32 planes (bf16-rounded if round_mid) + res)
// (out_f32: out is fp32, += when accumulate)
int oproj_finish(const float* part, long plane, int S, long ldp, const void* res, long ldr,
                 void* out, long ldo, int T, int N, int round_mid, void* stream,
                 int out_f32 = 0, int accumulate = 0, const float* row_scale = nullptr);

// the fused decode front end with noaux_tc group masking (fus_moe_route_small is n_group 1)
int route_small_launch(const void* h, const void* r, const void* gamma, float eps, const void* wa,
                       int nplanes, const float* bias, int T, int H, int E, int topk, float scale,
                       int renorm, int n_group, int topk_group, void* h1, void* x2, float* logits,
                       float* topw, int* topi, int block_m, int* sorted_ids, int sorted_cap,
                       int* expert_ids, int blocks_cap, int* ntp, int* done, int* zero,
                       int zero_n, void* stream, int* status);

// route_small_launch's shape checks, without pointers to device data
// (host only: fus_moe_block_check runs it on the CPU with the block's own arguments)
int route_small_check(int T, int H, int E, int topk, int n_group, int topk_group, int block_m,
                      int nplanes);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

}  // namespace fus
