// Headed gated scan, forward, chunk-parallel form (bf16 q/k/v, dk = dv = 64,
// fp32 state):   S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,   o_t = S_t^T q_t.
// Reference semantics: affine_scan.py:14-62 run on U_t = f_t I,
// V_t = (1 - f_t) k_t v_t^T, followed by the readout einsum.
//
// The outputs of a 64-token chunk depend on the earlier tokens only through
// the state entering the chunk, S_in(c).  Three launches:
//   gated_chunk_local  one CTA per segment of consecutive chunks of a head:
//                      the segment-local state entering every chunk,
//                      L_c = sum over earlier chunks of the segment of their
//                      decayed k v^T (bf16, one 8 KB tile per chunk), the log2
//                      decay from the segment start to the chunk start, and
//                      the segment aggregate (fp32).  Per chunk one tcgen05
//                      product dS = K~^T V (K~ rows scaled by the decay to the
//                      chunk end, so every factor is <= 1); the products run
//                      LAG chunks ahead of the fp32 register recurrence
//                      L <- d_C L + dS that reads them back.
//   gated_seg_carry    the state entering every segment, a short sequential
//                      pass per head over the segment aggregates (plus the
//                      final state and decay).
//   gated_chunk_out    every chunk independently: S_in = a_c S_seg + L_c
//                      (a_c the decay from the segment start), then
//                      o = diag(e^l) [Q S_in + (mask(Q K^T) diag(w e^-l)) V]
//                      with two 64x64x64 tcgen05 products after P = Q K^T.
//                      Small CTAs (4 warps, 64 KB ring, 128 tensor-memory
//                      columns), three per SM, so that several chunks are in
//                      flight per SM and no chain of chunks is serial.
// Decays: chunk-local inclusive log2 cumulative gates l_t (per-step log2 f
// clamped at -64, so f = 0 is a full reset).  When the chunk's total decay is
// below 2^-100 the factorised form above could overflow; such a chunk uses
// the exact per-element decays exp2(l_t - l_s) instead, with Q rows scaled by
// exp2(l_t) in place.
#include "common.cuh"
#include "gated_common.cuh"
#include "gated_internal.h"

namespace mogt {
namespace gated {
namespace chunked {

// Programmatic dependent launch: a dependent kernel may start early and waits
// here for the complete results of the kernel before it.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Fragment tiles moved with ldmatrix / stmatrix.  A thread's accumulator
// fragment (tcgen05.ld 16x256b, warp w = rows 16w..16w+15) is, per 32-column
// half h, the m16n8 layout of four 8x8 blocks per row half; x4 number x of
// half h covers column blocks 4h + 2x and 4h + 2x + 1.  Lane l addresses row
// 8 (j & 1) + (l & 7) of block j = l / 8 in a 128B-swizzled 64x64 tile.
__device__ __forceinline__ uint32_t frag_row_addr(uint32_t tile, int rq, int lane, int h, int x) {
  const int j = lane >> 3, rr = lane & 7;
  const int row = 16 * rq + 8 * (j & 1) + rr;
  const int chunk = 4 * h + 2 * x + (j >> 1);
  return tile + (uint32_t)(row * 128 + ((chunk ^ rr) << 4));
}
// registers of x4 number x of half h <-> fragment values v[h][n][e]
__device__ __forceinline__ void frag_unpack(float (&v)[2][4][4], int h, int x, const uint32_t (&r)[4]) {
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const int n = 2 * x + jj;
    v[h][n][0] = __uint_as_float(r[2 * jj] << 16);
    v[h][n][1] = __uint_as_float(r[2 * jj] & 0xFFFF0000u);
    v[h][n][2] = __uint_as_float(r[2 * jj + 1] << 16);
    v[h][n][3] = __uint_as_float(r[2 * jj + 1] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void frag_pack(uint32_t (&r)[4], const float (&v)[2][4][4], int h, int x) {
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const int n = 2 * x + jj;
    r[2 * jj] = pack_bf16(v[h][n][0], v[h][n][1]);
    r[2 * jj + 1] = pack_bf16(v[h][n][2], v[h][n][3]);
  }
}

// ---------------------------------------------------------------------------
// gated_chunk_local
// ---------------------------------------------------------------------------
constexpr int A_RS = 4;                   // k/v ring slots
constexpr int A_NB = 2;                   // dS accumulators (64 columns each)
constexpr int A_LAG = 1;                  // chunks between a dS product and its read-back
constexpr int A_CTAS_PER_SM = 3;
constexpr int A_SLOT = 2 * TILE;
constexpr int A_SM_STAGE = A_RS * A_SLOT; // bf16 local state of one chunk, to its TMA store
constexpr int A_SM_TOT = A_SM_STAGE + TILE;   // per-chunk log2 decays of the segment
constexpr int A_SM_BAR = A_SM_TOT + MAX_CPS * 4;
constexpr int A_NBARS = A_RS + A_NB;
constexpr int A_SM_TSLOT = A_SM_BAR + 8 * A_NBARS;
constexpr int A_SM_TOTAL = A_SM_TSLOT + 16;
constexpr int A_SM_ALLOC = A_SM_TOTAL + 1024;
static_assert(A_CTAS_PER_SM * (A_SM_ALLOC + 1024) <= 228 * 1024, "three CTAs per SM");
static_assert(A_CTAS_PER_SM * A_NB * 64 <= 512, "tensor memory of three CTAs");

struct AParams {
  const float* f;
  __nv_bfloat16* Lst;   // [BH, nchunks, 64, 64] segment-local state entering each chunk
  float* lam;           // [BH, nchunks] log2 decay from the segment start to the chunk start
  float4* gtab;         // [BH, nchunks, 32] per step pair: (l, 1 - f, l, 1 - f), l the chunk-local
                        // inclusive log2 cumulative gate
  float* seg_agg;       // [BH, nseg, 64, 64] segment aggregate (row-major fp32)
  float* seg_lam;       // [BH, nseg] log2 decay over the segment
  WsHeader* hdr;
  int T, BH, nchunks, cps, nseg;
};

__global__ void __launch_bounds__(NTHREADS, A_CTAS_PER_SM)
    gated_chunk_local(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                      const __grid_constant__ CUtensorMap tl, const AParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2;
  const Frag fr{qd * 16 + (lane >> 2), hf, lane & 3};
  const int br0 = build_row(tid, 0), br1 = build_row(tid, 1);
  float* tot_s = reinterpret_cast<float*>(smem + A_SM_TOT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + A_SM_BAR);
  uint64_t* dsb = full + A_RS;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + A_SM_TSLOT);

  griddep_launch();
  if (warp == 0) tmem_alloc(tslot, A_NB * 64);
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < A_NBARS; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tw = tbase + ((uint32_t)(32 * qd) << 16) + 32u * hf;
  const int seg = blockIdx.x / p.BH, bh = blockIdx.x % p.BH;
  const int c0 = seg * p.cps;
  const int n = min(p.cps, p.nchunks - c0);
  const int T = p.T;
  const float* fh = p.f + (size_t)bh * T;
  const size_t ubase = (size_t)bh * p.nchunks + c0;
  bool ok = true;

  // k, v and the local states are read again by gated_chunk_out right after
  // this pass: keep them in L2
  uint64_t pol_keep;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_keep));
  auto issue = [&](int j) {
    if (j >= n) return;
    const int slot = j % A_RS;
    uint8_t* base = smem + slot * A_SLOT;
    mbar_arrive_expect_tx(&full[slot], 2 * TILE);
    tma_load_3d_hint(base, &tk, &full[slot], 0, (c0 + j) * CH, bh, pol_keep);
    tma_load_3d_hint(base + TILE, &tv, &full[slot], 0, (c0 + j) * CH, bh, pol_keep);
  };
  if (tid == 0)
    for (int j = 0; j < A_RS; ++j) issue(j);

  float Ls[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int e = 0; e < 4; ++e) Ls[a][e] = 0.f;
  float lam_run = 0.f;

  // read back dS_j, publish L_j (the state entering chunk j) through the
  // staging tile and a TMA store, advance L.  The staging tile is free: the
  // previous store's read was waited for before the barrier that precedes
  // this call (`drain`: before the barrier taken here).
  uint8_t* stage = smem + A_SM_STAGE;
  auto process = [&](int j, bool drain) {
    if (!mbar_wait_spin(&dsb[j % A_NB], (j / A_NB) & 1)) ok = false;
    __syncwarp();
    tc_fence_after();
    float ds[4][4];
    tmem_ld_16x32(ds, tw + 64u * (j % A_NB));
    tc_fence_before();
    if (drain) {
      if (tid == 0) bulk_wait_read<0>();
      __syncthreads();
    }
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      uint32_t r[4];
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        r[2 * jj] = pack_bf16(Ls[2 * x + jj][0], Ls[2 * x + jj][1]);
        r[2 * jj + 1] = pack_bf16(Ls[2 * x + jj][2], Ls[2 * x + jj][3]);
      }
      stsm_x4(frag_row_addr(smem_u32(stage), qd, lane, hf, x), r);
    }
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tma_store_3d(&tl, stage, 0, (c0 + j) * CH, bh);
      bulk_commit();
      p.lam[ubase + j] = lam_run;
    }
    const float tot = tot_s[j];
    const float dC = fast_exp2(tot);
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int e = 0; e < 4; ++e) Ls[a][e] = fmaf(Ls[a][e], dC, ds[a][e]);
    lam_run += tot;
    // the product that read slot j has completed: refill it
    if (tid == 0) issue(j + A_RS);
    __syncwarp();
  };

  float2 fnext = gate_load(fh, T, c0, lane);
  for (int j = 0; j < n; ++j) {
    const WGates gt = warp_gates(fnext, lane);
    if (j + 1 < n) fnext = gate_load(fh, T, c0 + j + 1, lane);
    if (tid == 0) tot_s[j] = gt.tot;
    if (warp == 0) p.gtab[(ubase + j) * 32 + lane] = make_float4(gt.l0, gt.w0, gt.l1, gt.w1);
    if (!mbar_wait_spin(&full[j % A_RS], (j / A_RS) & 1)) ok = false;
    uint8_t* base = smem + (j % A_RS) * A_SLOT;
    // K~ rows, in place: w_s exp2(tot - l_s) k_s (every factor <= 1)
    const float k0 = gt.w0 * fast_exp2(gt.tot - gt.l0), k1 = gt.w1 * fast_exp2(gt.tot - gt.l1);
    build_rows(base, base, step_val(k0, k1, br0), step_val(k0, k1, br1), tid);
    fence_proxy_async();
    tc_fence_before();
    if (tid == 0) bulk_wait_read<0>();   // the staging tile is free after this barrier
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      umma_64x64x64(tbase + 64u * (j % A_NB), smem_u32(base), true, smem_u32(base + TILE), true,
                    false);
      umma_commit(&dsb[j % A_NB]);
    }
    __syncwarp();
    if (j >= A_LAG) process(j - A_LAG, false);
  }
  for (int j = max(0, n - A_LAG); j < n; ++j) process(j, true);
  if (tid == 0) bulk_wait<0>();

  const size_t sidx = (size_t)bh * p.nseg + seg;
  store_frag_rowmajor(p.seg_agg + sidx * (D * D), Ls, fr);
  if (tid == 0) p.seg_lam[sidx] = lam_run;

  if (!ok) record_error(p.hdr, MOGT_ERR_TIMEOUT, blockIdx.x);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, A_NB * 64);
  }
}

// ---------------------------------------------------------------------------
// gated_seg_carry: the state entering every segment.  A CTA owns 32 state
// elements of one head (lane = element, coalesced) and its 8 warps split the
// segments into 8 consecutive groups: each group's affine composite (decay,
// sum) is formed in parallel, the groups are chained through shared memory,
// then every group re-runs its segments from its incoming state (the second
// reads hit L2).
// ---------------------------------------------------------------------------
constexpr int C_WARPS = 8;

__global__ void __launch_bounds__(32 * C_WARPS) gated_seg_carry(const float* __restrict__ seg_agg,
                                                             const float* __restrict__ seg_lam,
                                                             float* __restrict__ seg_state,
                                                             const float* __restrict__ S0,
                                                             float* __restrict__ S_final,
                                                             float* __restrict__ decay_final,
                                                             int nseg) {
  __shared__ float grp_l[C_WARPS];
  __shared__ float grp_b[C_WARPS][32];
  griddep_launch();
  griddep_wait();   // the segment aggregates of gated_chunk_local
  const int bh = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 32 + lane;
  const int G = (nseg + C_WARPS - 1) / C_WARPS;
  const int g0 = min(nseg, warp * G), g1 = min(nseg, g0 + G);
  const size_t b0 = (size_t)bh * nseg;
  // pass 1: this group's composite
  float lsum = 0.f, bsum = 0.f;
  for (int g = g0; g < g1; g += 8) {
    float ag[8], lg[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const bool in = g + q < g1;
      ag[q] = in ? __ldg(seg_agg + (b0 + g + q) * (D * D) + e) : 0.f;
      lg[q] = in ? __ldg(seg_lam + b0 + g + q) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      lsum += lg[q];
      bsum = fmaf(fast_exp2(lg[q]), bsum, ag[q]);
    }
  }
  grp_l[warp] = lsum;   // identical in every lane
  grp_b[warp][lane] = bsum;
  __syncthreads();
  // state entering this group
  float s = S0 ? S0[(size_t)bh * (D * D) + e] : 0.f;
  float ltot = 0.f;
  for (int w = 0; w < warp; ++w) {
    s = fmaf(fast_exp2(grp_l[w]), s, grp_b[w][lane]);
    ltot += grp_l[w];
  }
  // pass 2: the state entering every segment of the group
  for (int g = g0; g < g1; g += 8) {
    float ag[8], lg[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const bool in = g + q < g1;
      ag[q] = in ? __ldg(seg_agg + (b0 + g + q) * (D * D) + e) : 0.f;
      lg[q] = in ? __ldg(seg_lam + b0 + g + q) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (g + q < g1) {
        seg_state[(b0 + g + q) * (D * D) + e] = s;
        s = fmaf(fast_exp2(lg[q]), s, ag[q]);
      }
  }
  if (warp == C_WARPS - 1) {
    // the last group ends the sequence (empty trailing groups pass s through)
    if (S_final) S_final[(size_t)bh * (D * D) + e] = s;
    if (decay_final && e == 0) decay_final[bh] = fast_exp2(ltot + lsum);
  }
}

// ---------------------------------------------------------------------------
// gated_chunk_out
// ---------------------------------------------------------------------------
constexpr int B_THREADS = 128;            // 4 warps: warp w owns accumulator rows 16w..16w+15
constexpr int B_RS = 2;                   // ring slots of (q, k, v, L)
constexpr int B_SLOT = 4 * TILE;
constexpr int B_SM_STAGE = B_RS * B_SLOT;   // bf16 output staging, 16 rows per warp
constexpr int B_SM_BAR = B_SM_STAGE + TILE;
constexpr int B_NBARS = B_RS + 2;
constexpr int B_SM_TSLOT = B_SM_BAR + 8 * B_NBARS;
constexpr int B_SM_TOTAL = B_SM_TSLOT + 16;
constexpr int B_SM_ALLOC = B_SM_TOTAL + 1024;
constexpr int B_CTAS_PER_SM = 3;
static_assert(B_CTAS_PER_SM * (B_SM_ALLOC + 1024) <= 228 * 1024, "three CTAs per SM");
constexpr uint32_t TM_P = 0, TM_O = 64;

struct BParams {
  const float4* gtab;
  void* o;
  __nv_bfloat16* chunk_states;   // [BH, nchunks, 64, 64] full entering state, or null
  const float* lam;
  const float* seg_state;
  WsHeader* hdr;
  int T, BH, nchunks, cps, nseg, nunits, per_cta;
};

// 128-thread in-place row scaling of a swizzled 64x64 bf16 tile: thread tid
// scales 16-byte pieces tid + 128 j (rows (tid + 128 j) / 8), j = 0..3.
__device__ __forceinline__ void scale_rows128(uint8_t* tile, const float (&sc)[4], int tid) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = tid + B_THREADS * j, row = q >> 3, chunk = q & 7;
    const uint32_t off = sw128(row, chunk);
    const uint4 v = *reinterpret_cast<const uint4*>(tile + off);
    const float c = sc[j];
    const __nv_bfloat16 h = __float2bfloat16_rn(c);
    const __nv_bfloat16 l = __float2bfloat16_rn(c - __bfloat162float(h));
    const __nv_bfloat162 hi = __halves2bfloat162(h, h), lo = __halves2bfloat162(l, l);
    uint4 w;
    w.x = bf2_scale(v.x, hi, lo);
    w.y = bf2_scale(v.y, hi, lo);
    w.z = bf2_scale(v.z, hi, lo);
    w.w = bf2_scale(v.w, hi, lo);
    *reinterpret_cast<uint4*>(tile + off) = w;
  }
}

template <bool OUT_F32>
__global__ void __launch_bounds__(B_THREADS, B_CTAS_PER_SM)
    gated_chunk_out(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tl,
                    const __grid_constant__ CUtensorMap to, const BParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const Frag fa{16 * warp + g, 0, c4}, fb{16 * warp + g, 1, c4};
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + B_SM_BAR);
  uint64_t* bar_p = full + B_RS;
  uint64_t* bar_o = full + B_RS + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + B_SM_TSLOT);
  uint8_t* stage = smem + B_SM_STAGE;

  if (warp == 0) tmem_alloc(tslot, 128);
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < B_NBARS; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tw = tbase + ((uint32_t)(32 * warp) << 16);
  const int T = p.T, nchunks = p.nchunks;
  const int u_begin = blockIdx.x * p.per_cta;
  const int u_end = min(u_begin + p.per_cta, p.nunits);
  const int n = max(0, u_end - u_begin);
  const bool want_out = p.o != nullptr;
  bool ok = true;

  // roles of single threads: lane 0 of warp 0 issues the output products,
  // of warp 1 the P products, of warp 3 the TMA loads
  const bool tma_thr = tid == 96, p_thr = tid == 32, o_thr = tid == 0;
  uint64_t pol_last = 0;
  if (tma_thr) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_last));
  // items are taken from the end of the range backwards: the chunks the
  // local pass touched last are the most likely to still be in L2
  auto unit_of = [&](int i) { return u_end - 1 - i; };
  // every tile is read for the last time here; `part` 1: q, k, v only,
  // 2: the local state only (issued after the wait on the earlier kernels)
  auto issue = [&](int i, int part = 0) {
    if (i >= n) return;
    const int u = unit_of(i), bh = u / nchunks, c = u % nchunks;
    uint8_t* base = smem + (i & 1) * B_SLOT;
    if (part != 2) mbar_arrive_expect_tx(&full[i & 1], (want_out ? 4 : 1) * TILE);
    if (want_out && part != 2) {
      tma_load_3d_hint(base, &tq, &full[i & 1], 0, c * CH, bh, pol_last);
      tma_load_3d_hint(base + TILE, &tk, &full[i & 1], 0, c * CH, bh, pol_last);
      tma_load_3d_hint(base + 2 * TILE, &tv, &full[i & 1], 0, c * CH, bh, pol_last);
    }
    if (part != 1) tma_load_3d_hint(base + 3 * TILE, &tl, &full[i & 1], 0, c * CH, bh, pol_last);
  };
  auto issue_p = [&](int i) {   // P_i = Q K^T (raw tiles), one thread
    const uint8_t* base = smem + (i & 1) * B_SLOT;
    umma_64x64x64(tbase + TM_P, smem_u32(base), false, smem_u32(base + TILE), false, false);
    umma_commit(bar_p);
  };

  // q, k, v of the first two items do not depend on the earlier kernels of
  // the forward: their loads overlap the segment-carry kernel
  if (tma_thr && n > 0) {
    issue(0, 1);
    issue(1, 1);
  }
  griddep_wait();   // local states, gate tables and segment states are complete
  if (tma_thr && n > 0) {
    issue(0, 2);
    issue(1, 2);
  }
  if (p_thr && n > 0 && want_out) {
    if (!mbar_wait_spin(&full[0], 0)) ok = false;
    tc_fence_after();
    issue_p(0);
  }
  __syncwarp();

  float sseg[2][4][4];
  int cur_key = -1;
  float4 gcur = make_float4(0.f, 0.f, 0.f, 0.f);
  float lam_cur = 0.f;
  if (n > 0) {
    const int u = unit_of(0);
    gcur = __ldg(p.gtab + (size_t)u * 32 + lane);
    lam_cur = __ldg(p.lam + u);
  }
  const int t0 = 16 * warp + g, t1 = t0 + 8;   // this thread's rows of a chunk
  // this thread's stmatrix / ldmatrix row offsets in a 64x64 tile, per (half, x4)
  uint32_t fro[2][2];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int x = 0; x < 2; ++x) fro[h][x] = frag_row_addr(0u, warp, lane, h, x);
  // (head, chunk, segment) of the current item, stepped backwards without divisions
  int bh = 0, c = 0, seg = 0;
  if (n > 0) {
    bh = (u_end - 1) / nchunks;
    c = (u_end - 1) % nchunks;
    seg = c / p.cps;
  }

  for (int i = 0; i < n; ++i) {
    const int u = unit_of(i);
    const int s = i & 1;
    uint8_t* base = smem + s * B_SLOT;
    WGates gt;
    gt.l0 = gcur.x;
    gt.w0 = gcur.y;
    gt.l1 = gcur.z;
    gt.w1 = gcur.w;
    gt.tot = __shfl_sync(0xffffffffu, gcur.z, 31);
    const float a_c = fast_exp2(lam_cur);
    if (i + 1 < n) {
      const int un = unit_of(i + 1);
      gcur = __ldg(p.gtab + (size_t)un * 32 + lane);
      lam_cur = __ldg(p.lam + un);
    }
    const bool fast = factorises(gt);
    // state of the chunk's segment (changes every cps chunks)
    const int key = bh * p.nseg + seg;
    if (key != cur_key) {
      const float* src = p.seg_state + (size_t)key * (D * D);
      load_frag_rowmajor(sseg[0], src, fa);
      load_frag_rowmajor(sseg[1], src, fb);
      cur_key = key;
    }

    float pr[2][4][4];
    if (want_out) {
      if (!mbar_wait_spin(bar_p, i & 1)) ok = false;
      __syncwarp();
      tc_fence_after();
      uint32_t r0[16], r1[16];
      tmem_ld_16x32_async(r0, tw + TM_P);
      tmem_ld_16x32_async(r1, tw + TM_P + 32);
      tmem_wait_ld();
      frag_from_u32(pr[0], r0);
      frag_from_u32(pr[1], r1);
    }
    if (!mbar_wait_spin(&full[s], (i >> 1) & 1)) ok = false;
    __syncwarp();

    // S_in = a_c S_seg + L_c, in place of the L tile (and to chunk_states)
    {
      const uint32_t lt = smem_u32(base + 3 * TILE);
      float sv[2][4][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const uint32_t addr = lt + fro[h][x];
          uint32_t r[4];
          ldsm_x4_v(r, addr);
          frag_unpack(sv, h, x, r);
#pragma unroll
          for (int jj = 0; jj < 2; ++jj)
#pragma unroll
            for (int e = 0; e < 4; ++e)
              sv[h][2 * x + jj][e] = fmaf(a_c, sseg[h][2 * x + jj][e], sv[h][2 * x + jj][e]);
          frag_pack(r, sv, h, x);
          stsm_x4(addr, r);
        }
      if (p.chunk_states) {
        store_frag_rowmajor_bf16(p.chunk_states + (size_t)u * (D * D), sv[0], fa);
        store_frag_rowmajor_bf16(p.chunk_states + (size_t)u * (D * D), sv[1], fb);
      }
    }

    float e_t0 = 1.f, e_t1 = 1.f;
    if (want_out) {
      const float lt0 = step_val(gt.l0, gt.l1, t0), lt1 = step_val(gt.l0, gt.l1, t1);
      if (fast) {
        // P''[t,s] = [s <= t] P[t,s] w_s exp2(-l_s); the rows get exp2(l_t) at the output.
        // Column blocks wholly below this warp's rows need no mask, blocks wholly
        // above are zero (warp-uniform tests).
        e_t0 = fast_exp2(lt0);
        e_t1 = fast_exp2(lt1);
        const float cs0 = gt.w0 * fast_exp2(-gt.l0), cs1 = gt.w1 * fast_exp2(-gt.l1);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const int b = 4 * h + a;
            const int m = 4 * b + c4;                 // lane holding steps 2m, 2m+1
            const float x0 = __shfl_sync(0xffffffffu, cs0, m);
            const float x1 = __shfl_sync(0xffffffffu, cs1, m);
            if (8 * b + 7 <= 16 * warp) {
              pr[h][a][0] *= x0;
              pr[h][a][1] *= x1;
              pr[h][a][2] *= x0;
              pr[h][a][3] *= x1;
            } else if (8 * b > 16 * warp + 15) {
              pr[h][a][0] = pr[h][a][1] = pr[h][a][2] = pr[h][a][3] = 0.f;
            } else {
              const int s0 = 2 * m;
              pr[h][a][0] = (s0 <= t0) ? pr[h][a][0] * x0 : 0.f;
              pr[h][a][1] = (s0 + 1 <= t0) ? pr[h][a][1] * x1 : 0.f;
              pr[h][a][2] = (s0 <= t1) ? pr[h][a][2] * x0 : 0.f;
              pr[h][a][3] = (s0 + 1 <= t1) ? pr[h][a][3] * x1 : 0.f;
            }
          }
      } else {
        // exact per-element decays; Q rows get exp2(l_t) in place
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const int m = 4 * (4 * h + a) + c4;
            const float l0 = __shfl_sync(0xffffffffu, gt.l0, m);
            const float l1 = __shfl_sync(0xffffffffu, gt.l1, m);
            const float w0 = __shfl_sync(0xffffffffu, gt.w0, m);
            const float w1 = __shfl_sync(0xffffffffu, gt.w1, m);
            const int s0 = 2 * m;
            pr[h][a][0] = (s0 <= t0) ? pr[h][a][0] * fast_exp2(lt0 - l0) * w0 : 0.f;
            pr[h][a][1] = (s0 + 1 <= t0) ? pr[h][a][1] * fast_exp2(lt0 - l1) * w1 : 0.f;
            pr[h][a][2] = (s0 <= t1) ? pr[h][a][2] * fast_exp2(lt1 - l0) * w0 : 0.f;
            pr[h][a][3] = (s0 + 1 <= t1) ? pr[h][a][3] * fast_exp2(lt1 - l1) * w1 : 0.f;
          }
        const float e0 = fast_exp2(gt.l0), e1 = fast_exp2(gt.l1);
        float sc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[j] = step_val(e0, e1, (tid + B_THREADS * j) >> 3);
        scale_rows128(base, sc, tid);
      }
      // P'' in place of the K tile (the product that read K has completed)
      const uint32_t kt = smem_u32(base + TILE);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          uint32_t r[4];
          frag_pack(r, pr, h, x);
          stsm_x4(kt + fro[h][x], r);
        }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (want_out && lane == 0) {
      if (o_thr) {
        tc_fence_after();
        // O = Q S_in + P'' V
        umma_64x64x64(tbase + TM_O, smem_u32(base), false, smem_u32(base + 3 * TILE), true, false);
        umma_64x64x64(tbase + TM_O, smem_u32(base + TILE), false, smem_u32(base + 2 * TILE), true, true);
        umma_commit(bar_o);
      } else if (p_thr && i + 1 < n) {
        if (!mbar_wait_spin(&full[s ^ 1], ((i + 1) >> 1) & 1)) ok = false;
        tc_fence_after();
        issue_p(i + 1);
      }
    }
    __syncwarp();
    if (want_out) {
      if (!mbar_wait_spin(bar_o, i & 1)) ok = false;
      __syncwarp();
      tc_fence_after();
      uint32_t r0[16], r1[16];
      tmem_ld_16x32_async(r0, tw + TM_O);
      tmem_ld_16x32_async(r1, tw + TM_O + 32);
      tmem_wait_ld();
      tc_fence_before();
      float ov[2][4][4];
      frag_from_u32(ov[0], r0);
      frag_from_u32(ov[1], r1);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          ov[h][a][0] *= e_t0;
          ov[h][a][1] *= e_t0;
          ov[h][a][2] *= e_t1;
          ov[h][a][3] *= e_t1;
        }
      if (OUT_F32) {
        const int ta = c * CH + t0, tb = ta + 8;
        const size_t rowa = ((size_t)bh * T + ta) * D, rowb = ((size_t)bh * T + tb) * D;
        float* o = static_cast<float*>(p.o);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const int j = 8 * (4 * h + a) + 2 * c4;
            if (ta < T) __stcs(reinterpret_cast<float2*>(o + rowa + j), make_float2(ov[h][a][0], ov[h][a][1]));
            if (tb < T) __stcs(reinterpret_cast<float2*>(o + rowb + j), make_float2(ov[h][a][2], ov[h][a][3]));
          }
      } else {
        // this warp's 16 rows through its own staging block and TMA store
        // (rows past T are clipped by the tensor map)
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        const uint32_t st = smem_u32(stage);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            uint32_t r[4];
            frag_pack(r, ov, h, x);
            stsm_x4(st + fro[h][x], r);
          }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && c * CH + 16 * warp < T) {
          tma_store_3d(&to, stage + warp * (16 * 128), 0, c * CH + 16 * warp, bh);
          bulk_commit();
        }
      }
    }
    // every read of slot s (threads and products) is done: refill it
    if (tma_thr) issue(i + 2);
    __syncwarp();
    if (--c < 0) {
      c = nchunks - 1;
      --bh;
      seg = c / p.cps;
    } else if (c < seg * p.cps) {
      --seg;
    }
  }
  if (lane == 0) bulk_wait<0>();

  if (!ok) record_error(p.hdr, MOGT_ERR_TIMEOUT, blockIdx.x);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 128);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Layout {
  size_t Lst, lam, gtab, seg_agg, seg_lam, seg_state, total;
};
inline Layout layout(size_t BH, const Plan& pl) {
  using mogt_host::align_up;
  Layout l;
  const size_t U = BH * pl.nchunks, S = BH * pl.nstripes;
  l.Lst = sizeof(WsHeader);
  l.lam = l.Lst + U * D * D * 2;
  l.gtab = l.lam + align_up(U * 4, 256);
  l.seg_agg = l.gtab + U * CH * 8;
  l.seg_lam = l.seg_agg + S * D * D * 4;
  l.seg_state = l.seg_lam + align_up(S * 4, 256);
  l.total = l.seg_state + S * D * D * 4;
  return l;
}

int prepare() {
  constexpr int kMaxDev = 64;
  static bool done[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return MOGT_ERR_LAUNCH;
  if (dev < kMaxDev && done[dev]) return MOGT_OK;
  if (cudaFuncSetAttribute(gated_chunk_local, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           A_SM_ALLOC) != cudaSuccess ||
      cudaFuncSetAttribute(gated_chunk_out<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           B_SM_ALLOC) != cudaSuccess ||
      cudaFuncSetAttribute(gated_chunk_out<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           B_SM_ALLOC) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  if (dev < kMaxDev) done[dev] = true;
  return MOGT_OK;
}

}  // namespace chunked

size_t chunked_fwd_workspace_bytes(int64_t BH, int64_t T) {
  using chunked::A_CTAS_PER_SM;
  const Plan pl = make_plan(BH, T, A_CTAS_PER_SM * sm_count());
  return chunked::layout((size_t)BH, pl).total;
}

int launch_seg_carry(const float* agg, const float* lam, float* state, int64_t BH, int nseg,
                     cudaStream_t s) {
  chunked::gated_seg_carry<<<dim3(D * D / 32, (unsigned)BH), 32 * chunked::C_WARPS, 0, s>>>(
      agg, lam, state, nullptr, nullptr, nullptr, nseg);
  return mogt_host::launch_status();
}

int launch_chunked_fwd(const void* q, const void* k, const void* v, const float* f, void* o,
                       const float* S0, float* S_final, float* decay_final, void* chunk_states,
                       int64_t BH, int64_t T, int out_dtype, void* workspace,
                       size_t workspace_bytes, cudaStream_t s, bool resume) {
  using namespace chunked;
  const Plan pl = make_plan(BH, T, A_CTAS_PER_SM * sm_count());
  const Layout L = layout((size_t)BH, pl);
  if (!workspace || workspace_bytes < L.total) return MOGT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOGT_ERR_ALIGN;
  if ((size_t)BH * pl.nstripes >= ((size_t)1 << 31) || (size_t)BH * pl.nchunks >= ((size_t)1 << 31))
    return MOGT_ERR_UNSUPPORTED;
  if (prepare() != MOGT_OK) return MOGT_ERR_LAUNCH;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const bool need_out = o != nullptr || chunk_states != nullptr;

  CUtensorMap maps[5];
  const void* srcs[3] = {q ? q : k, k, v};
  for (int i = 0; i < 3; ++i) {
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)T * D * 2};
    cuuint32_t box[3] = {(cuuint32_t)D, (cuuint32_t)CH, 1};
    if (mogt_host::encode_tiled(&maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                                const_cast<void*>(srcs[i]), dims, strides, box,
                                CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return MOGT_ERR_LAUNCH;
  }
  // segment-local states: into chunk_states when the caller keeps them (the
  // output pass overwrites each with the full entering state), else workspace.
  // A resumed call finds them in the workspace, where the earlier call
  // (made without chunk_states) left them.
  __nv_bfloat16* Lst = (chunk_states && !resume) ? static_cast<__nv_bfloat16*>(chunk_states)
                                                 : reinterpret_cast<__nv_bfloat16*>(ws + L.Lst);
  {
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)pl.nchunks * CH, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)pl.nchunks * CH * D * 2};
    cuuint32_t box[3] = {(cuuint32_t)D, (cuuint32_t)CH, 1};
    if (mogt_host::encode_tiled(&maps[3], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, Lst, dims, strides,
                                box, CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return MOGT_ERR_LAUNCH;
  }

  // bf16 output: 16-row boxes, one TMA store per warp and chunk
  maps[4] = maps[0];
  if (o && out_dtype == MOGT_DTYPE_BF16) {
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)T * D * 2};
    cuuint32_t box[3] = {(cuuint32_t)D, 16, 1};
    if (mogt_host::encode_tiled(&maps[4], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, o, dims, strides,
                                box, CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return MOGT_ERR_LAUNCH;
  }

  AParams A;
  A.f = f;
  A.Lst = Lst;
  A.lam = reinterpret_cast<float*>(ws + L.lam);
  A.gtab = reinterpret_cast<float4*>(ws + L.gtab);
  A.seg_agg = reinterpret_cast<float*>(ws + L.seg_agg);
  A.seg_lam = reinterpret_cast<float*>(ws + L.seg_lam);
  A.hdr = reinterpret_cast<WsHeader*>(ws);
  A.T = (int)T;
  A.BH = (int)BH;
  A.nchunks = pl.nchunks;
  A.cps = pl.cps;
  A.nseg = pl.nstripes;
  if (!resume)
    gated_chunk_local<<<(unsigned)(BH * pl.nstripes), NTHREADS, A_SM_ALLOC, s>>>(maps[1], maps[2], maps[3], A);
  float* seg_state = reinterpret_cast<float*>(ws + L.seg_state);
  // the carry and output kernels are launched as programmatic dependents: they
  // may start while the previous kernel drains and wait for its results with
  // griddepcontrol.wait
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(D * D / 32, (unsigned)BH);
  cfg.blockDim = dim3(32 * C_WARPS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, gated_seg_carry, (const float*)A.seg_agg, (const float*)A.seg_lam,
                         seg_state, S0, S_final, decay_final, pl.nstripes) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  if (!need_out) return mogt_host::launch_status();

  BParams Bp;
  Bp.gtab = A.gtab;
  Bp.o = o;
  Bp.chunk_states = static_cast<__nv_bfloat16*>(chunk_states);
  Bp.lam = A.lam;
  Bp.seg_state = seg_state;
  Bp.hdr = A.hdr;
  Bp.T = (int)T;
  Bp.BH = (int)BH;
  Bp.nchunks = pl.nchunks;
  Bp.cps = pl.cps;
  Bp.nseg = pl.nstripes;
  Bp.nunits = (int)(BH * pl.nchunks);
  const int max_ctas = B_CTAS_PER_SM * sm_count();
  Bp.per_cta = (Bp.nunits + max_ctas - 1) / max_ctas;
  const unsigned grid = (unsigned)((Bp.nunits + Bp.per_cta - 1) / Bp.per_cta);
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(B_THREADS);
  cfg.dynamicSmemBytes = B_SM_ALLOC;
  const cudaError_t e =
      out_dtype == MOGT_DTYPE_F32
          ? cudaLaunchKernelEx(&cfg, gated_chunk_out<true>, maps[0], maps[1], maps[2], maps[3], maps[4], Bp)
          : cudaLaunchKernelEx(&cfg, gated_chunk_out<false>, maps[0], maps[1], maps[2], maps[3], maps[4], Bp);
  if (e != cudaSuccess) return MOGT_ERR_LAUNCH;
  return mogt_host::launch_status();
}

}  // namespace gated
}  // namespace mogt
