// Shared device helpers for the MOGT scan kernels (sm_100a).
//
// Everything here is small inline PTX for the data movement and tensor-core
// primitives the scan kernels use, plus the status codes of the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mogt_scan.h"

namespace mogt {

// Bounded spin: every wait on another CTA's flag or on an mbarrier gives up
// after this many polls, records MOGT_ERR_TIMEOUT in the workspace header and
// carries on, so a broken protocol can never hang the GPU.
constexpr uint32_t kSpinLimit = 1u << 22;

// ----------------------------------------------------------------------------
// Workspace header of the look-back kernels.  A zero-filled workspace is valid
// for the first call; each call leaves it valid for the next one (the last CTA
// to finish resets the ticket and done counters and advances the epoch that
// tags this call's flags).  err is sticky until the host clears it.
// ----------------------------------------------------------------------------
struct WsHeader {
  uint32_t ticket;
  uint32_t done;
  uint32_t epoch;
  uint32_t err;
  uint32_t err_unit;
  uint32_t pad[59];
};
static_assert(sizeof(WsHeader) == 256, "header is 256 bytes");

enum : uint32_t { kFlagNone = 0, kFlagAgg = 1, kFlagInc = 2 };

__device__ __forceinline__ uint32_t flag_tag(uint32_t epoch, uint32_t state) {
  return ((epoch & 0x3FFFFFFFu) << 2) | state;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Take a ticket (the scheduling order of look-back units) and read the epoch.
// Must be called by one thread.
__device__ __forceinline__ uint32_t take_ticket(WsHeader* h, uint32_t* epoch) {
  uint32_t t = atomicAdd(&h->ticket, 1u);
  *epoch = *reinterpret_cast<volatile uint32_t*>(&h->epoch);
  return t;
}

// Called by one thread of every CTA at exit: the last CTA re-arms the header.
__device__ __forceinline__ void finish_cta(WsHeader* h, uint32_t epoch, uint32_t nblocks) {
  __threadfence();
  uint32_t prev = atomicAdd(&h->done, 1u);
  if (prev == nblocks - 1) {
    h->ticket = 0;
    h->done = 0;
    __threadfence();
    atomicExch(&h->epoch, epoch + 1);
  }
}

__device__ __forceinline__ void record_error(WsHeader* h, uint32_t code, uint32_t unit) {
  if (atomicCAS(&h->err, 0u, code) == 0u) h->err_unit = unit;
}

// Wait until flags[m] carries this epoch's tag with a state >= AGG.  Returns the
// state, or kFlagNone after a timeout (which is recorded).
__device__ __forceinline__ uint32_t wait_flag(const uint32_t* flag, uint32_t epoch, WsHeader* h,
                                              uint32_t unit) {
  const uint32_t want = (epoch & 0x3FFFFFFFu);
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    uint32_t v = ld_acquire_u32(flag);
    if ((v >> 2) == want && (v & 3u) != 0u) return v & 3u;
    if (it > 64) __nanosleep(it > 4096 ? 256 : 32);
  }
  record_error(h, MOGT_ERR_TIMEOUT, unit);
  return kFlagNone;
}

// ----------------------------------------------------------------------------
// Shared-memory / TMA / mbarrier primitives
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a tile of 128-byte rows
// written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (tile base 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier over `count` threads (a multiple of 32); id 0 is __syncthreads.
__device__ __forceinline__ void group_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// One suspending parity probe: the thread sleeps until the phase completes or
// about `hint_ns` have passed.
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t phase, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(addr), "r"(phase), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Bounded parity wait: suspending probes, given up after kWaitLimitNs of
// wall time (the caller records MOGT_ERR_TIMEOUT).  Returns false on timeout.
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, phase, 1000000u)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(addr, phase, 1000000u)) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Bounded parity wait without a suspend hint: each probe returns after a
// short hardware-chosen interval, so a waiting warp resumes as soon as the
// phase completes.  Same time limit and return value as mbar_wait.
__device__ __forceinline__ bool mbar_try_wait_spin(uint32_t addr, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(addr), "r"(phase)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t phase) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait_spin(addr, phase)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_spin(addr, phase)) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
}

// 32-bit global store with an L2 eviction-priority hint (a createpolicy value).
__device__ __forceinline__ void st_global_hint(void* p, uint32_t v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.b32 [%0], %1, %2;" ::"l"(p), "r"(v), "l"(pol) : "memory");
}

// 3-D tiled TMA load (no multicast) into shared memory, completion counted on
// `bar` in bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 3-D tiled TMA store from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int32_t c0,
                                             int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------
// Warp-level tensor-core primitives (bf16 in, fp32 accumulate)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Ordered forms (volatile, memory clobber) for tiles that TMA or the tensor
// core also touch: they stay after the waits and before the fences around them.
__device__ __forceinline__ void ldsm_x4_v(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// D += A(16x16, row) * B(16x8, col)
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// Multiply both bf16 halves of `v` by (s0, s1) and repack.
__device__ __forceinline__ uint32_t scale_bf16x2(uint32_t v, float s0, float s1) {
  float2 f = unpack_bf16(v);
  return pack_bf16(f.x * s0, f.y * s1);
}

// PTX approximate base-2 exponent / logarithm (ex2.approx, lg2.approx).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

}  // namespace mogt

// Host-side helpers shared by the entry points.
namespace mogt_host {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MOGT_OK : MOGT_ERR_LAUNCH;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
                      CUtensorMapSwizzle swizzle);

}  // namespace mogt_host

// ----------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core) helpers: shared-memory matrix
// descriptors for 128B-swizzled bf16 tiles of 64-element (128-byte) rows,
// single-thread MMA issue into tensor memory, completion through an mbarrier,
// and warp-wide tensor-memory loads in the m16n8 fragment layout.
// ----------------------------------------------------------------------------
namespace mogt {

// K-major operand: rows are M (or N), 64 K-elements per 128-byte row, 8-row
// swizzle atoms of 1024 bytes.  A K=16 step advances the start by 32 bytes.
__device__ __forceinline__ uint64_t umma_desc_kmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major operand: rows are K, 64 M/N-elements per 128-byte row; groups of 8
// K-rows are 1024 bytes apart.  A K=16 step advances the start by 2048 bytes.
__device__ __forceinline__ uint64_t umma_desc_mnmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(8192 >> 4) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: kind::f16, bf16 x bf16 -> f32, M = 64, N = 64.
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((64u >> 4) << 24);
constexpr uint32_t kIdescAmn = 1u << 15;  // A is MN-major
constexpr uint32_t kIdescBmn = 1u << 16;  // B is MN-major

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate));
}

// D(64x64, f32, TMEM) (+)= A(64x64) * B(64x64): four K=16 steps; the first
// step accumulates onto D only when `accumulate` is set.  The descriptors are
// built once; a K step only adds to the 14-bit start-address field (shared
// memory addresses stay below 256 KB, so the field never carries).
__device__ __forceinline__ void umma_64x64x64(uint32_t d_tmem, uint32_t a_saddr, bool a_mn,
                                              uint32_t b_saddr, bool b_mn, bool accumulate) {
  const uint32_t idesc = kIdescBase | (a_mn ? kIdescAmn : 0u) | (b_mn ? kIdescBmn : 0u);
  const uint64_t ad0 = a_mn ? umma_desc_mnmajor(a_saddr) : umma_desc_kmajor(a_saddr);
  const uint64_t bd0 = b_mn ? umma_desc_mnmajor(b_saddr) : umma_desc_kmajor(b_saddr);
  const uint64_t astep = a_mn ? (2048 >> 4) : (32 >> 4);
  const uint64_t bstep = b_mn ? (2048 >> 4) : (32 >> 4);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    umma_bf16(d_tmem, ad0 + astep * kk, bd0 + bstep * kk, idesc, accumulate || kk > 0);
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Warp-wide: 16 rows x 32 f32 columns of an M=64 accumulator (lane field of
// taddr = 32 * (warp % 4)), in the m16n8 fragment layout acc[n][e]: rows g,
// g+8 and columns 8n + 2c, +1 of the 32-column slice.
__device__ __forceinline__ void tmem_ld_16x32(float (&acc)[4][4], uint32_t taddr) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = __uint_as_float(r[4 * n + e]);
}

// Same load without the wait: several loads can be in flight before one
// tmem_wait_ld(); the registers are valid only after it.
__device__ __forceinline__ void tmem_ld_16x32_async(uint32_t (&r)[16], uint32_t taddr) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Warp-wide: 32 TMEM lanes (lane field of taddr = 32 * (warp % 4)) x 32
// consecutive f32 columns; thread l gets lane 32 * (warp % 4) + l.  For an
// M = 64 accumulator only threads 0..15 hold rows (16 * (warp % 4) + l).
__device__ __forceinline__ void tmem_ld_32x32b_x32_async(uint32_t (&r)[32], uint32_t taddr) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void frag_from_u32(float (&acc)[4][4], const uint32_t (&r)[16]) {
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = __uint_as_float(r[4 * n + e]);
}

// Tensor-memory allocation by one full warp; the address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

}  // namespace mogt
