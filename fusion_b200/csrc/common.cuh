// Shared device helpers for the fusion_b200 sm_100a kernels.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a): mbarrier
// phase waits with a time budget, TMA tiled loads (cp.async.bulk.tensor), and the
// tcgen05 family (TMEM alloc/dealloc, MMA issue, commit, TMEM->register loads).
// No wait in this library spins forever: every wait carries a globaltimer budget,
// on expiry it raises a bit in the caller's device status word and the kernel
// unwinds (frees TMEM, returns) instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fusion_b200.h"

#define FUS_DEVICE __device__ __forceinline__

namespace fus {

// ------------------------------------------------------------------------------------
// status word
// ------------------------------------------------------------------------------------
FUS_DEVICE void raise_status(int* status, int bits) {
  if (status) atomicOr(status, bits);
}

FUS_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// one second: generous against any legitimate stall, short enough that a broken
// pipeline returns control (with FUS_ERR_TIMEOUT set) instead of wedging the GPU.
constexpr uint64_t kWaitBudgetNs = 1000000000ull;

// ------------------------------------------------------------------------------------
// programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before its predecessor finishes; `pdl_wait` blocks until the
// predecessor grid completed and its writes are visible, `pdl_allow_dependents` lets
// the next kernel start launching. Both are no-ops without the launch attribute.
// ------------------------------------------------------------------------------------
// system-scope acquire / release on a flag another GPU writes / reads
FUS_DEVICE int ld_acquire_sys_i32(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FUS_DEVICE void st_release_sys_i32(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

FUS_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FUS_DEVICE void pdl_allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------------------------
// bf16 helpers
// ------------------------------------------------------------------------------------
FUS_DEVICE float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
FUS_DEVICE __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }
FUS_DEVICE float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// 8 bf16 packed in a uint4 <-> 8 floats
FUS_DEVICE void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
FUS_DEVICE uint4 pack8(const float* f) {
  uint4 u;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// streaming 128-bit global loads (read once: do not keep in L1)
FUS_DEVICE uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ------------------------------------------------------------------------------------
// warp / block reductions
// ------------------------------------------------------------------------------------
FUS_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------------------------
// shared-memory address helpers
// ------------------------------------------------------------------------------------
FUS_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------
FUS_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
FUS_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
FUS_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// named barrier `id` (1..15) over `n` threads (a multiple of 32)
FUS_DEVICE void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

FUS_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
FUS_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete. Gives up when `abort` is raised by
// another thread of the CTA or when the time budget is spent (then raises `abort`
// and FUS_ERR_TIMEOUT). Returns false when it gave up.
FUS_DEVICE bool mbar_wait_bounded(uint32_t bar, uint32_t parity, volatile int* abort,
                                  int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) {
      *abort = 1;
      raise_status(status, FUS_ERR_TIMEOUT);
      return false;
    }
  }
}

// ------------------------------------------------------------------------------------
// TMA (tiled tensor copies global -> shared, completion counted on an mbarrier)
// ------------------------------------------------------------------------------------
FUS_DEVICE void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
FUS_DEVICE uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
FUS_DEVICE uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
FUS_DEVICE uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2D tile load; c0 = inner (contiguous) coordinate in elements, c1 = row.
// SwiGLU of one fp32 gate/up pair in the GEMM epilogues: silu(g) * up with the fast
// exponential and division intrinsics (a few ulp from the IEEE expression, far inside the
// block's tolerance; the accumulators themselves are not exact to that level anyway)
FUS_DEVICE float silu_mul(float g, float up) { return __fdividef(g, 1.0f + __expf(-g)) * up; }

// ---- TMA tile store from shared memory (bulk-group completion) ----
// generic-proxy writes to the source tile must be fenced (fence_proxy_async_smem) and
// made CTA-visible (a barrier) before one thread issues the store
FUS_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
FUS_DEVICE void tma_store_2d(const CUtensorMap* m, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
FUS_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of all committed stores have been read (may be reused)
FUS_DEVICE void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// all committed stores are complete in global memory
FUS_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One warp copies a row of nv 16-byte vectors, eight loads in flight per lane (a plain
// strided loop keeps one load per lane outstanding and is latency-bound on 12 KB rows)
FUS_DEVICE void warp_copy_row(uint4* __restrict__ d, const uint4* __restrict__ s, int nv,
                              int lane) {
  int v = lane;
  for (; v + 7 * 32 < nv; v += 8 * 32) {
    uint4 t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) t[u] = __ldg(s + v + u * 32);
#pragma unroll
    for (int u = 0; u < 8; ++u) d[v + u * 32] = t[u];
  }
  for (; v < nv; v += 32) d[v] = __ldg(s + v);
}

// noaux_tc group masking for one token held by a warp, lane l owning choice values of
// experts 8l .. 8l+7 (reference.py:159-166): a group of E/n_group consecutive experts
// spans (E/n_group)/8 lanes; its score is the sum of its two largest choice values;
// experts outside the topk_group best groups (ties: lower group index) get choice * 0.
// n_group == 1 leaves ch untouched. Groups of 8 * 2^j experts, n_group <= 32.
FUS_DEVICE void group_mask_choice(float* ch, int lane, int E, int n_group, int topk_group) {
  if (n_group <= 1) return;
  float a1 = -INFINITY, a2 = -INFINITY;  // this lane's two largest
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float v = ch[j];
    if (v > a1) {
      a2 = a1;
      a1 = v;
    } else if (v > a2) {
      a2 = v;
    }
  }
  const int lpg = (E / n_group) >> 3;  // lanes per group
  for (int o = 1; o < lpg; o <<= 1) {  // merge the top-2 of lane pairs within a group
    const float b1 = __shfl_xor_sync(0xffffffffu, a1, o);
    const float b2 = __shfl_xor_sync(0xffffffffu, a2, o);
    const float hi = fmaxf(a1, b1);
    const float lo = fmaxf(fminf(a1, b1), fmaxf(a2, b2));
    a1 = hi;
    a2 = lo;
  }
  const float gscore = a1 + a2;  // the reference sums its descending top-2 values
  const int my_g = lane / lpg;
  int better = 0;  // groups ranked ahead of mine
  for (int g = 0; g < n_group; ++g) {
    const float og = __shfl_sync(0xffffffffu, gscore, g * lpg);
    better += (og > gscore) || (og == gscore && g < my_g);
  }
  if (lane * 8 < E && better >= topk_group) {
#pragma unroll
    for (int j = 0; j < 8; ++j) ch[j] = ch[j] * 0.0f;
  }
}

// 16-byte global store with an L2 eviction-policy hint
FUS_DEVICE void st_global_v4_hint(void* p, uint4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w), "l"(policy)
               : "memory");
}

// asynchronous prefetch of `bytes` (a multiple of 16, 16-byte aligned start) into L2
FUS_DEVICE void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

FUS_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1,
                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// 4 rows (one 128-byte box row each) gathered by row index into consecutive smem rows;
// the tensor map's box is one row high. Rows past the tensor's extent read zeros.
FUS_DEVICE void tma_gather4(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int r0,
                            int r1, int r2, int r3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(r0), "r"(r1), "r"(r2), "r"(r3),
      "l"(policy)
      : "memory");
}

// ------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)
// ------------------------------------------------------------------------------------
FUS_DEVICE void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
FUS_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
FUS_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
FUS_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
FUS_DEVICE void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)^T, bf16 inputs, fp32 accumulate.
FUS_DEVICE void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every previously issued tcgen05.mma of this thread completed
FUS_DEVICE void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread
// tcgen05.ld of 16 columns without the wait; tmem_ld_wait(r) completes it (its operands
// tie the registers to the wait so no use is scheduled before it)
FUS_DEVICE void tmem_ld16_issue(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
FUS_DEVICE void tmem_ld_wait(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

FUS_DEVICE void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand staged by TMA with 128-byte
// swizzle: rows of 64 bf16 (128 B), 8-row swizzle atoms of 1024 B stacked densely.
//   bits  0-13 start address >> 4
//   bits 16-29 leading byte offset >> 4 (unused for swizzled K-major; 1 by convention)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row atoms)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout: 2 = 128-byte swizzle
FUS_DEVICE uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: bf16 A and B (both K-major), fp32 D, shape M x N.
//   bits 4-5 D format (1 = f32); 7-9 A format (1 = bf16); 10-12 B format (1 = bf16)
//   bit 15/16 A/B major (0 = K); bits 17-22 N >> 3; bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

}  // namespace fus
