// Device helpers shared by the tensor-core gated-scan kernels (forward and
// backward): chunk geometry, warp-local gate arithmetic, scaled-tile builds
// and the 8-warp accumulator fragment layout.
#pragma once

#include "common.cuh"

namespace mogt {
namespace gated {

constexpr int D = 64;                     // dk = dv
constexpr int CH = 64;                    // tokens per chunk
constexpr int NTHREADS = 256;             // 8 warps
constexpr int TILE = CH * D * 2;          // one 64x64 bf16 tile, 8 KB
constexpr float kFactorMin = -100.f;      // log2 chunk decay above which D factorises

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int32_t c0, int32_t c1, int32_t c2, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(pol)
      : "memory");
}

__device__ __forceinline__ float clamped_log2(float f) { return fmaxf(fast_log2(f), -64.f); }

// Gates of chunk gc: lane l holds steps 2l, 2l+1 (t >= T reads as "no step":
// f = 1, so log2 f = 0 and 1 - f = 0).  Loaded one chunk ahead of use.
__device__ __forceinline__ float2 gate_load(const float* fh, int T, int gc, int lane) {
  const int t = gc * CH + 2 * lane;
  float2 r;
  r.x = t < T ? __ldg(fh + t) : 1.f;
  r.y = t + 1 < T ? __ldg(fh + t + 1) : 1.f;
  return r;
}

// Chunk-local gate values, held by every warp for itself: lane l owns steps
// 2l and 2l+1 (inclusive log2 cumulative gate l, 1 - f as w); tot is the log2
// decay of the whole chunk (all lanes).
struct WGates {
  float l0, l1, w0, w1, x0, x1, tot;
};
__device__ __forceinline__ WGates warp_gates(float2 fv, int lane) {
  WGates gt;
  const float x0 = clamped_log2(fv.x), x1 = clamped_log2(fv.y);
  gt.w0 = 1.f - fv.x;
  gt.w1 = 1.f - fv.y;
  gt.x0 = x0;
  gt.x1 = x1;
  const float pair = x0 + x1;
  float inc = pair;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  gt.l0 = inc - pair + x0;
  gt.l1 = inc;
  gt.tot = __shfl_sync(0xffffffffu, inc, 31);
  return gt;
}
// Value of step r (0..63) of a per-step quantity held as (v0, v1) pairs.
__device__ __forceinline__ float step_val(float v0, float v1, int r) {
  const float a = __shfl_sync(0xffffffffu, v0, r >> 1);
  const float b = __shfl_sync(0xffffffffu, v1, r >> 1);
  return (r & 1) ? b : a;
}
__device__ __forceinline__ bool factorises(const WGates& gt) { return gt.tot >= kFactorMin; }

// Rows this thread scales when building a 64x64 tile: 4w + lane/8 and 32 + that.
__device__ __forceinline__ int build_row(int tid, int j) { return (tid + NTHREADS * j) >> 3; }

// dst rows (r, swizzled 128-byte rows) = scale_r * src rows, for this thread's
// two rows (see build_row), 16 bytes each.  Packed bf16x2 arithmetic: the
// fp32 scale is split into bf16 hi + lo parts and y = x*hi + (x*lo), so the
// product is rounded to bf16 once, as an fp32 multiply followed by a cast.
__device__ __forceinline__ uint32_t bf2_scale(uint32_t x, __nv_bfloat162 hi, __nv_bfloat162 lo) {
  const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(&x);
  const __nv_bfloat162 y = __hfma2(xv, hi, __hmul2(xv, lo));
  return *reinterpret_cast<const uint32_t*>(&y);
}
__device__ __forceinline__ void build_rows(uint8_t* dst, const uint8_t* src, float s0, float s1,
                                           int tid) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int q = tid + NTHREADS * j, row = q >> 3, chunk = q & 7;
    const uint32_t off = sw128(row, chunk);
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    const float c = j ? s1 : s0;
    const __nv_bfloat16 h = __float2bfloat16_rn(c);
    const __nv_bfloat16 l = __float2bfloat16_rn(c - __bfloat162float(h));
    const __nv_bfloat162 hi = __halves2bfloat162(h, h), lo = __halves2bfloat162(l, l);
    uint4 w;
    w.x = bf2_scale(v.x, hi, lo);
    w.y = bf2_scale(v.y, hi, lo);
    w.z = bf2_scale(v.z, hi, lo);
    w.w = bf2_scale(v.w, hi, lo);
    *reinterpret_cast<uint4*>(dst + off) = w;
  }
}

// Fragment geometry of a thread in the 8-warp layout: rows r0 and r0 + 8,
// columns 8 * (4 hf + n) + 2 c4 (+1) for n = 0..3.
struct Frag {
  int r0, hf, c4;
};

__device__ __forceinline__ void store_frag_bf16(uint8_t* tile, const float (&s)[4][4], Frag fr) {
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const uint32_t chunk = 4 * fr.hf + n, col = 4u * fr.c4;
    *reinterpret_cast<uint32_t*>(tile + sw128(fr.r0, chunk) + col) = pack_bf16(s[n][0], s[n][1]);
    *reinterpret_cast<uint32_t*>(tile + sw128(fr.r0 + 8, chunk) + col) = pack_bf16(s[n][2], s[n][3]);
  }
}

__device__ __forceinline__ void store_frag_rowmajor(float* dst, const float (&s)[4][4], Frag fr) {
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int j = 8 * (4 * fr.hf + n) + 2 * fr.c4;
    *reinterpret_cast<float2*>(dst + fr.r0 * D + j) = make_float2(s[n][0], s[n][1]);
    *reinterpret_cast<float2*>(dst + (fr.r0 + 8) * D + j) = make_float2(s[n][2], s[n][3]);
  }
}

__device__ __forceinline__ void store_frag_rowmajor_bf16(__nv_bfloat16* dst, const float (&s)[4][4],
                                                         Frag fr) {
  uint32_t* d32 = reinterpret_cast<uint32_t*>(dst);
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int j = 8 * (4 * fr.hf + n) + 2 * fr.c4;
    d32[(fr.r0 * D + j) >> 1] = pack_bf16(s[n][0], s[n][1]);
    d32[((fr.r0 + 8) * D + j) >> 1] = pack_bf16(s[n][2], s[n][3]);
  }
}

// Inverse of store_frag_bf16: this thread's fragment of a swizzled bf16 tile.
__device__ __forceinline__ void load_frag_bf16(float (&s)[4][4], const uint8_t* tile, Frag fr) {
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const uint32_t chunk = 4 * fr.hf + n, col = 4u * fr.c4;
    const uint32_t a = *reinterpret_cast<const uint32_t*>(tile + sw128(fr.r0, chunk) + col);
    const uint32_t b = *reinterpret_cast<const uint32_t*>(tile + sw128(fr.r0 + 8, chunk) + col);
    s[n][0] = __uint_as_float(a << 16);
    s[n][1] = __uint_as_float(a & 0xFFFF0000u);
    s[n][2] = __uint_as_float(b << 16);
    s[n][3] = __uint_as_float(b & 0xFFFF0000u);
  }
}

__device__ __forceinline__ void load_frag_rowmajor(float (&s)[4][4], const float* src, Frag fr) {
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int j = 8 * (4 * fr.hf + n) + 2 * fr.c4;
    const float2 lo = __ldg(reinterpret_cast<const float2*>(src + fr.r0 * D + j));
    const float2 hi = __ldg(reinterpret_cast<const float2*>(src + (fr.r0 + 8) * D + j));
    s[n][0] = lo.x; s[n][1] = lo.y; s[n][2] = hi.x; s[n][3] = hi.y;
  }
}

// ---- host-side stripe planning and workspace layout (forward and backward) ----
constexpr int MAX_CPS = 256;              // chunks per stripe (per-stripe decay tables)

// Look-back workspace after the 256-byte header: per unit a flag, aggregate
// and inclusive decays, and aggregate and inclusive 64x64 fp32 states.
struct WsLayout {
  size_t flags, a_agg, a_inc, st_agg, st_inc, total;
};
inline WsLayout ws_layout(size_t NU) {
  WsLayout l;
  l.flags = sizeof(WsHeader);
  l.a_agg = l.flags + mogt_host::align_up(NU * 4, 256);
  l.a_inc = l.a_agg + mogt_host::align_up(NU * 4, 256);
  l.st_agg = l.a_inc + mogt_host::align_up(NU * 4, 256);
  l.st_inc = l.st_agg + NU * D * D * 4;
  l.total = l.st_inc + NU * D * D * 4;
  return l;
}

// Chunks of a head cut into stripes so that BH x stripes is about one wave of
// `resident` CTAs; a stripe holds at most MAX_CPS chunks.
struct Plan {
  int nchunks, cps, nstripes;
};
inline Plan make_plan(int64_t BH, int64_t T, int resident) {
  Plan p;
  p.nchunks = (int)((T + CH - 1) / CH);
  int64_t sph = BH >= resident ? 1 : resident / BH;
  if (sph > p.nchunks) sph = p.nchunks;
  if (sph < 1) sph = 1;
  const int64_t min_sph = (p.nchunks + MAX_CPS - 1) / MAX_CPS;
  if (sph < min_sph) sph = min_sph;
  p.cps = (int)((p.nchunks + sph - 1) / sph);
  p.nstripes = (p.nchunks + p.cps - 1) / p.cps;
  return p;
}

inline int sm_count() {
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  return nsm;
}

}  // namespace gated
}  // namespace mogt
