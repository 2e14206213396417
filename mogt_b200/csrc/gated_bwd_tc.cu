// Headed gated scan, backward on tensor cores (bf16 q/k/v/do, dk = dv = 64).
//
// Forward:  S_t = f_t S_{t-1} + w_t k_t v_t^T  (w = 1 - f),  o_t = S_t^T q_t.
// Adjoint:  G_t = q_t do_t^T + f_{t+1} G_{t+1};
//   dq_t = S_t do_t,  dk_t = w_t G_t v_t,  dv_t = w_t G_t^T k_t,
//   df_t = <G_t, S_{t-1}> - k_t^T G_t v_t,  dS_0 = f_0 G_0
// (the chain rule through affine_scan.py:65-124 with U_t = f_t I and
// V_t = w_t k_t v_t^T; same quantities as the sequential kernel).
//
// Reverse-time chunked scan.  Chunk = 64 steps with chunk-local inclusive
// log2 cumulative gates l_t (L = l_63), X = the adjoint carry entering the
// chunk from the later ones (G_63 = q_63 do_63^T + X), S_in = the state
// entering the chunk, read from the bf16 per-chunk states the forward saved.
// With decays d[u,s] = exp2(l_u - l_s) (u >= s):
//   M1 = dO V^T, PQ = Q K^T, M1d = d o M1, PQd = d o PQ (lower incl. diag),
//   dq = diag(exp2 l) dO S_in^T + M1d (diag(w) K)
//   dk = diag(w) [M1d^T Q + diag(exp2(L - l)) V X^T]
//   dv = diag(w) [PQd^T dO + diag(exp2(L - l)) K X]
//   X_prev = exp2(L) X + (diag(exp2 l) Q)^T dO        (carry into the chunk before)
// and df_t from four product terms, none of which cancels:
//   <G_t, S_{t-1}> = exp2(L - x_t) <X, S_in>                  x_t = l_t - l_{t-1}
//                  + exp2(l_{t-1}) R_t,  R_t = z_t + f_{t+1} R_{t+1},  z_u = q_u^T S_in do_u
//                  + exp2(L - l_t) P_{t-1},  P_t = f_t P_{t-1} + w_t y_t,  y_s = k_s^T X v_s
//                  + exp2(-x_t) sum_{u >= t > s} d[u,s] w_s (q_u.k_s)(do_u.v_s)
//   k_t^T G_t v_t  = k_t.(M1d^T Q)_t + exp2(L - l_t) y_t.
// Every decay is formed per element from differences of l, so the form is
// exact for any gates (no factorisation condition, no fallback path).
//
// Work decomposition: the chunks of a head are cut into stripes, each stripe
// into kSub segments.
//   gated_bwd_seg_agg  (three light CTAs per SM) every segment's carry
//           aggregate  sum_c exp2(lpre_c) Q^_c^T dO_c  (lpre = log2 decay of
//           the segment's chunks before c) and log2 decay, in reverse order;
//   the forward's segment carry kernel composes them into the carry entering
//           every segment's end from the later ones;
//   gated_bwd_stripe  (8 warps, one CTA per SM) per stripe, from the carry
//           entering its end, the chunks in reverse order: 9 tcgen05 MMAs
//           per chunk (6 of the carry and the raw tiles, 3 of the masked
//           products), epilogues in registers, and one warp forms df from
//           per-step partial sums.
#include "common.cuh"
#include "gated_common.cuh"
#include "gated_internal.h"

namespace mogt {
namespace gated {
namespace bwd {

constexpr int STAGES = 3;                  // pass-2 ring: q, k, v, do, S_in per slot
constexpr int SLOT = 5 * TILE;
constexpr int T_Q = 0, T_K = 1, T_V = 2, T_DO = 3, T_S = 4;

constexpr int SM_RING = 0;
constexpr int SM_QH = SM_RING + STAGES * SLOT;     // diag(exp2 l) Q, [t][i]
constexpr int SM_KW = SM_QH + TILE;                // diag(w) K, [s][i]
constexpr int SM_X = SM_KW + TILE;                 // bf16 carry X, [i][j]
constexpr int SM_M1 = SM_X + TILE;                 // M1d, [u][s]
constexpr int SM_PQ = SM_M1 + TILE;                // PQd, [u][s]
constexpr int SM_OUT = SM_PQ + TILE;               // dq, dk, dv staging tiles [3] (TMA stores)
constexpr int SM_GL = SM_OUT + 3 * TILE;           // l_t of the chunk [64]
constexpr int SM_GW = SM_GL + 256;                 // w_t [64]
// per-chunk partial sums for df, double-buffered by chunk parity (df of chunk
// j is formed during chunk j+1)
constexpr int PART = 512 * 3 + 1024 + 256 + 64;    // one parity's partials
constexpr int SM_ROWZ = SM_GW + 256;               // [2][64] halves of z_u
constexpr int SM_ROWY = SM_ROWZ + 512;             // [2][64] halves of y_s
constexpr int SM_ROWK = SM_ROWY + 512;             // [2][64] halves of k.(M1d^T Q)
constexpr int SM_COLW = SM_ROWK + 512;             // [4][64] column sums of the E prefix
constexpr int SM_ROWT = SM_COLW + 1024;            // [64] row totals of E, columns 0..31
constexpr int SM_SIG = SM_ROWT + 256;              // [8] <X, S_in> per warp
constexpr int SM_MISC = SM_ROWZ + 2 * PART;        // ticket, epoch
constexpr int NBARS = STAGES + 5;
constexpr int SM_BAR = SM_MISC + 256;
constexpr int SM_TSLOT = SM_BAR + 8 * NBARS;
constexpr int SM_TOTAL = SM_TSLOT + 16;
constexpr int SM_ALLOC = SM_TOTAL + 1024;
static_assert(SM_ALLOC <= 227 * 1024, "shared memory per CTA");

// tensor memory (fp32 M = 64 accumulators): group-1 products, then the
// group-2 products reuse the M1 / PQ columns once those are read
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TM_M1 = 0, TM_PQ = 64, TM_DOS = 128, TM_DX = 192, TM_VX = 256, TM_KX = 320,
                   TM_DV2 = 384;
constexpr uint32_t TM_DQ2 = TM_M1, TM_DK2 = TM_PQ;

struct Params {
  const float* f;
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  float* df;
  float* dS0;
  WsHeader* hdr;
  // the carry entering every stripe's end, from the segment passes
  // (gated_bwd_seg_agg + the segment carry): [BH][nseg_b][4096] in the
  // fragment-register order of the 8-warp layout, segments in reverse time
  // order, nsub segments per stripe
  const float* x_in;
  int nseg_b, nsub;
  int T, BH, nchunks, cps, nstripes;
};

__device__ __forceinline__ void zero44(float (&a)[4][4]) {
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) a[n][e] = 0.f;
}

// Sum over the 4 lanes of a quad (same fragment row, the four c4 lanes).
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

__global__ void __launch_bounds__(NTHREADS, 1)
    gated_bwd_stripe(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                     const __grid_constant__ CUtensorMap ts, const __grid_constant__ CUtensorMap tdq,
                     const __grid_constant__ CUtensorMap tdk, const __grid_constant__ CUtensorMap tdv,
                     const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2, g = lane >> 2, c4 = lane & 3;
  const Frag fr{qd * 16 + g, hf, c4};
  const int br0 = build_row(tid, 0), br1 = build_row(tid, 1);
  float* sgl = reinterpret_cast<float*>(smem + SM_GL);
  float* sgw = reinterpret_cast<float*>(smem + SM_GW);
  auto part = [&](int off, int par) { return reinterpret_cast<float*>(smem + off + par * PART); };
  volatile uint32_t* bc = reinterpret_cast<volatile uint32_t*>(smem + SM_MISC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
  uint64_t* bar_a = bars + STAGES;          // M1, PQ
  uint64_t* bar_b = bar_a + 1;              // dO S_in^T, Q^^T dO
  uint64_t* bar_c = bar_a + 2;              // V X^T, K X
  uint64_t* bar_d = bar_a + 3;              // M1d (w K)
  uint64_t* bar_e = bar_a + 4;              // M1d^T Q, PQd^T dO
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM_TSLOT);
  uint8_t* qh_tile = smem + SM_QH;
  uint8_t* kw_tile = smem + SM_KW;
  uint8_t* x_tile = smem + SM_X;
  uint8_t* m1_tile = smem + SM_M1;
  uint8_t* pq_tile = smem + SM_PQ;

  if (warp == 0) tmem_alloc(tslot, TMEM_COLS);
  if (tid == 0) {
    uint32_t epoch;
    bc[0] = take_ticket(p.hdr, &epoch);
    bc[1] = epoch;
#pragma unroll
    for (int s = 0; s < NBARS; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tw = tbase + ((uint32_t)(32 * qd) << 16) + 32u * hf;
  const uint32_t unit = bc[0], epoch = bc[1];
  const int BH = p.BH, T = p.T;
  // tickets run over the chain of each head from its last stripe backwards
  const int ci = (int)unit / BH, bh = (int)unit % BH;
  const int stripe = p.nstripes - 1 - ci;
  const int c_begin = stripe * p.cps;
  const int nc = min(p.cps, p.nchunks - c_begin);
  const int nit = nc;
  const float* fh = p.f + (size_t)bh * T;
  uint32_t ph_a = 0, ph_b = 0, ph_c = 0, ph_d = 0, ph_e = 0;
  bool ok = true;

  uint64_t pol_stream = 0;
  if (tid == 0)
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_stream));
  // TMA loads of pipeline iteration `it`: the stripe's chunks in reverse
  // (q, k, v, do, S_in)
  auto issue = [&](int it) {
    if (it >= nit) return;
    const int slot = it % STAGES;
    const int gc = c_begin + nc - 1 - it, t0 = gc * CH;
    uint8_t* base = smem + SM_RING + slot * SLOT;
    mbar_arrive_expect_tx(&bars[slot], 5 * TILE);
    tma_load_3d_hint(base + T_Q * TILE, &tq, &bars[slot], 0, t0, bh, pol_stream);
    tma_load_3d_hint(base + T_K * TILE, &tk, &bars[slot], 0, t0, bh, pol_stream);
    tma_load_3d_hint(base + T_V * TILE, &tv, &bars[slot], 0, t0, bh, pol_stream);
    tma_load_3d_hint(base + T_DO * TILE, &tdo, &bars[slot], 0, t0, bh, pol_stream);
    tma_load_3d_hint(base + T_S * TILE, &ts, &bars[slot], 0, t0, bh, pol_stream);
  };
  auto wait_bar = [&](uint64_t* bar, uint32_t& ph) {
    if (!mbar_wait(bar, ph)) ok = false;
    ph ^= 1u;
  };

  if (tid == 0)
    for (int it = 0; it < STAGES - 1; ++it) issue(it);

  // ---------------- carry entering the stripe's end ----------------
  // from the segment passes: the state of the reversed segment that follows
  // this stripe's last one (zero for the last stripe)
  float X[4][4];
  if (ci == 0) {
    zero44(X);
  } else {
    const int g_last = (stripe + 1) * p.nsub - 1;
    const float4* src = reinterpret_cast<const float4*>(
        p.x_in + ((size_t)bh * p.nseg_b + (p.nseg_b - 1 - g_last)) * (D * D) + (size_t)tid * 16);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const float4 v = __ldcg(src + n);
      X[n][0] = v.x;
      X[n][1] = v.y;
      X[n][2] = v.z;
      X[n][3] = v.w;
    }
  }

  // ---------------- pass 2: chunks in reverse ----------------
  // df of chunk gc from the partials of parity par: one warp, lane l owns
  // steps 2l and 2l+1
  auto compute_df = [&](int gc, const WGates& gt, int par) {
    const float* rowZ = part(SM_ROWZ, par);
    const float* rowY = part(SM_ROWY, par);
    const float* rowK = part(SM_ROWK, par);
    const float* colW = part(SM_COLW, par);
    const float* rowT = part(SM_ROWT, par);
    const float* sig = part(SM_SIG, par);
      const int t0 = 2 * lane;
      float z0 = rowZ[t0] + rowZ[64 + t0], z1 = rowZ[t0 + 1] + rowZ[64 + t0 + 1];
      float y0 = rowY[t0] + rowY[64 + t0], y1 = rowY[t0 + 1] + rowY[64 + t0 + 1];
      const float k0 = rowK[t0] + rowK[64 + t0], k1 = rowK[t0 + 1] + rowK[64 + t0 + 1];
      float S0sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) S0sum += sig[w];
      const float f0 = fast_exp2(gt.x0), f1 = fast_exp2(gt.x1);
      // R_t = z_t + f_{t+1} R_{t+1} (suffix), as affine maps over lanes
      const float f2 = __shfl_down_sync(0xffffffffu, f0, 1);  // f of step 2l+2 (lane 31: unused)
      float A = lane < 31 ? f1 * f2 : 0.f;
      float B = fmaf(f1, z1, z0);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float A2 = __shfl_down_sync(0xffffffffu, A, o);
        const float B2 = __shfl_down_sync(0xffffffffu, B, o);
        if (lane + o < 32) {
          B = fmaf(A, B2, B);
          A *= A2;
        }
      }
      const float Rnext = __shfl_down_sync(0xffffffffu, B, 1);  // R_{2l+2} (lane 31: none)
      const float R0 = B;
      const float R1 = lane < 31 ? fmaf(f2, Rnext, z1) : z1;
      // P_t = f_t P_{t-1} + w_t y_t (prefix)
      float PA = f0 * f1;
      float PB = fmaf(f1 * gt.w0, y0, gt.w1 * y1);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float A2 = __shfl_up_sync(0xffffffffu, PA, o);
        const float B2 = __shfl_up_sync(0xffffffffu, PB, o);
        if (lane >= o) {
          PB = fmaf(PA, B2, PB);
          PA *= A2;
        }
      }
      float Pm1 = __shfl_up_sync(0xffffffffu, PB, 1);  // P_{2l-1}
      if (lane == 0) Pm1 = 0.f;
      const float P0 = fmaf(f0, Pm1, gt.w0 * y0);      // P_{2l}
      // W_t: column sums of the E prefix plus, for t >= 32, the suffix of the
      // left half's row totals
      float W0 = colW[t0] + colW[64 + t0] + colW[128 + t0] + colW[192 + t0];
      float W1 = colW[t0 + 1] + colW[64 + t0 + 1] + colW[128 + t0 + 1] + colW[192 + t0 + 1];
      {
        const float r0 = rowT[t0], r1 = rowT[t0 + 1];
        float sfx = r0 + r1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, sfx, o);
          if (lane + o < 32) sfx += y;
        }
        float below = __shfl_down_sync(0xffffffffu, sfx, 1);  // rows >= 2l + 2
        if (lane == 31) below = 0.f;
        if (t0 >= 32) {
          W0 += sfx;
          W1 += r1 + below;
        }
      }
      const float lup = __shfl_up_sync(0xffffffffu, gt.l1, 1);
      const float lprev0 = lane > 0 ? lup : 0.f;  // l_{2l-1}
      const float L = gt.tot;
      const float d0 = fast_exp2(L - gt.x0) * S0sum + fast_exp2(lprev0) * R0 +
                       fast_exp2(L - gt.l0) * Pm1 + fast_exp2(-gt.x0) * W0 -
                       (k0 + fast_exp2(L - gt.l0) * y0);
      const float d1 = fast_exp2(L - gt.x1) * S0sum + fast_exp2(gt.l0) * R1 +
                       fast_exp2(L - gt.l1) * P0 + fast_exp2(-gt.x1) * W1 -
                       (k1 + fast_exp2(L - gt.l1) * y1);
      const int ta = gc * CH + t0;
      const size_t off = (size_t)bh * T + ta;
      float* dfo = p.df + off;
      if (ta + 1 < T && (off & 1) == 0) {
        *reinterpret_cast<float2*>(dfo) = make_float2(d0, d1);
      } else {
        if (ta < T) dfo[0] = d0;
        if (ta + 1 < T) dfo[1] = d1;
      }
  };
  const int gl = c_begin + nc - 1;
  float2 fnext = gate_load(fh, T, gl, lane);
  WGates gprev{};
  for (int j = 0; j < nc; ++j) {
    const int gc = gl - j;
    const int slot = j % STAGES;
    const uint8_t* base = smem + SM_RING + slot * SLOT;
    const WGates gt = warp_gates(fnext, lane);
    if (j + 1 < nc) fnext = gate_load(fh, T, gc - 1, lane);
    if (warp == 0) {
      *reinterpret_cast<float2*>(sgl + 2 * lane) = make_float2(gt.l0, gt.l1);
      *reinterpret_cast<float2*>(sgw + 2 * lane) = make_float2(gt.w0, gt.w1);
    }
    if (!mbar_wait(&bars[slot], (j / STAGES) & 1)) ok = false;
    {
      const float e0 = fast_exp2(gt.l0), e1 = fast_exp2(gt.l1);
      build_rows(qh_tile, base + T_Q * TILE, step_val(e0, e1, br0), step_val(e0, e1, br1), tid);
      build_rows(kw_tile, base + T_K * TILE, step_val(gt.w0, gt.w1, br0), step_val(gt.w0, gt.w1, br1),
                 tid);
      store_frag_bf16(x_tile, X, fr);
    }
    fence_proxy_async();
    tc_fence_before();
    if (tid == 0) bulk_wait_read<0>();   // the previous chunk's dq, dk, dv stores have read their tiles
    __syncthreads();
    // group 1: products of the raw tiles and the carry
    {
      const uint32_t qb = smem_u32(base + T_Q * TILE), kb = smem_u32(base + T_K * TILE),
                     vb = smem_u32(base + T_V * TILE), db = smem_u32(base + T_DO * TILE),
                     sb = smem_u32(base + T_S * TILE);
      if (warp == 0 && lane == 0) {
        tc_fence_after();
        umma_64x64x64(tbase + TM_M1, db, false, vb, false, false);   // dO V^T
        umma_64x64x64(tbase + TM_PQ, qb, false, kb, false, false);   // Q K^T
        umma_commit(bar_a);
      } else if (warp == 1 && lane == 0) {
        tc_fence_after();
        umma_64x64x64(tbase + TM_DOS, db, false, sb, false, false);                // dO S_in^T
        umma_64x64x64(tbase + TM_DX, smem_u32(qh_tile), true, db, true, false);   // Q^^T dO
        umma_commit(bar_b);
      } else if (warp == 2 && lane == 0) {
        tc_fence_after();
        umma_64x64x64(tbase + TM_VX, vb, false, smem_u32(x_tile), false, false);  // V X^T
        umma_64x64x64(tbase + TM_KX, kb, false, smem_u32(x_tile), true, false);   // K X
        umma_commit(bar_c);
      } else if (warp == 3 && lane == 0) {
        issue(j + STAGES - 1);  // into the slot of chunk j-1, released at the barrier
      }
      __syncwarp();
    }
    // the last warp forms df of the previous chunk while the MMAs run
    if (warp == NTHREADS / 32 - 1 && j > 0) compute_df(gc + 1, gprev, (j - 1) & 1);
    // per-element decays of this thread's fragment: rows u, columns s
    const int ua = fr.r0, ub = ua + 8;
    const float lua = sgl[ua], lub = sgl[ub];
    float ls[4][2], ws[4][2];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int s0 = 8 * (4 * hf + n) + 2 * c4;
      const float2 l2 = *reinterpret_cast<const float2*>(sgl + s0);
      const float2 w2 = *reinterpret_cast<const float2*>(sgw + s0);
      ls[n][0] = l2.x; ls[n][1] = l2.y;
      ws[n][0] = w2.x; ws[n][1] = w2.y;
    }
    wait_bar(bar_a, ph_a);
    tc_fence_after();
    {
      uint32_t r_m[16], r_p[16];
      tmem_ld_16x32_async(r_m, tw + TM_M1);
      tmem_ld_16x32_async(r_p, tw + TM_PQ);
      tmem_wait_ld();
      float m1[4][4], pq[4][4], E[4][4];
      frag_from_u32(m1, r_m);
      frag_from_u32(pq, r_p);
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int s = 8 * (4 * hf + n) + 2 * c4 + e;
          const float da = s <= ua ? fast_exp2(lua - ls[n][e]) : 0.f;
          const float db = s <= ub ? fast_exp2(lub - ls[n][e]) : 0.f;
          m1[n][e] *= da;
          m1[n][2 + e] *= db;
          // E = M1d o PQ o w (one decay factor), strictly below the diagonal
          E[n][e] = s < ua ? m1[n][e] * pq[n][e] * ws[n][e] : 0.f;
          E[n][2 + e] = s < ub ? m1[n][2 + e] * pq[n][2 + e] * ws[n][e] : 0.f;
          pq[n][e] *= da;
          pq[n][2 + e] *= db;
        }
      store_frag_bf16(m1_tile, m1, fr);
      store_frag_bf16(pq_tile, pq, fr);
      // W_t = sum_{u >= t > s} E[u][s]: row-exclusive prefix F over this warp's
      // 32 columns, then column sums of F over the rows u >= t.  The warps of
      // the upper triangle (rows < 32 <= columns) hold no E.
      const bool live = !(hf == 1 && qd < 2);
      float colp[4][2];
      if (live) {
        float rowtot[2] = {0.f, 0.f};
        float F[4][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float base_n = 0.f;
#pragma unroll
          for (int n = 0; n < 4; ++n) {
            const float pr = E[n][2 * h] + E[n][2 * h + 1];
            float inc = pr;
            float y = __shfl_up_sync(0xffffffffu, inc, 1, 4);
            if (c4 >= 1) inc += y;
            y = __shfl_up_sync(0xffffffffu, inc, 2, 4);
            if (c4 >= 2) inc += y;
            const float tot = __shfl_sync(0xffffffffu, inc, 3, 4);
            // exclusive value from the neighbour (not inc - pr: E[u][t] itself
            // can exceed the terms before it by many orders of magnitude)
            float prev = __shfl_up_sync(0xffffffffu, inc, 1, 4);
            if (c4 == 0) prev = 0.f;
            const float ex = base_n + prev;
            F[n][2 * h] = ex;
            F[n][2 * h + 1] = ex + E[n][2 * h];
            base_n += tot;
          }
          rowtot[h] = base_n;
        }
        if (hf == 0 && c4 == 0) {
          part(SM_ROWT, j & 1)[ua] = rowtot[0];
          part(SM_ROWT, j & 1)[ub] = rowtot[1];
        }
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int s = 8 * (4 * hf + n) + 2 * c4 + e;
            float v = (ua >= s ? F[n][e] : 0.f) + (ub >= s ? F[n][2 + e] : 0.f);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            colp[n][e] = v;
          }
      } else {
#pragma unroll
        for (int n = 0; n < 4; ++n) colp[n][0] = colp[n][1] = 0.f;
      }
      if (g == 0) {
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int s0 = 8 * (4 * hf + n) + 2 * c4;
          *reinterpret_cast<float2*>(part(SM_COLW, j & 1) + qd * 64 + s0) = make_float2(colp[n][0], colp[n][1]);
        }
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    // group 2: the masked products
    {
      const uint32_t qb = smem_u32(base + T_Q * TILE), db = smem_u32(base + T_DO * TILE);
      if (warp == 0 && lane == 0) {
        tc_fence_after();
        umma_64x64x64(tbase + TM_DQ2, smem_u32(m1_tile), false, smem_u32(kw_tile), true, false);
        umma_commit(bar_d);
      } else if (warp == 1 && lane == 0) {
        tc_fence_after();
        umma_64x64x64(tbase + TM_DK2, smem_u32(m1_tile), true, qb, true, false);
        umma_64x64x64(tbase + TM_DV2, smem_u32(pq_tile), true, db, true, false);
        umma_commit(bar_e);
      }
      __syncwarp();
    }
    // carry, z and y from group 1
    float dos[4][4], vx[4][4], kx[4][4];
    float zp[2] = {0.f, 0.f}, yp[2] = {0.f, 0.f}, sg = 0.f;
    const float eL = fast_exp2(gt.tot);
    {
      wait_bar(bar_b, ph_b);
      wait_bar(bar_c, ph_c);
      tc_fence_after();
      uint32_t r_dos[16], r_dx[16], r_vx[16], r_kx[16];
      tmem_ld_16x32_async(r_dos, tw + TM_DOS);
      tmem_ld_16x32_async(r_dx, tw + TM_DX);
      tmem_ld_16x32_async(r_vx, tw + TM_VX);
      tmem_ld_16x32_async(r_kx, tw + TM_KX);
      float sin_[4][4], qf[4][4], kf[4][4];
      load_frag_bf16(sin_, base + T_S * TILE, fr);
      load_frag_bf16(qf, base + T_Q * TILE, fr);
      load_frag_bf16(kf, base + T_K * TILE, fr);
      tmem_wait_ld();
      float dx[4][4];
      frag_from_u32(dos, r_dos);
      frag_from_u32(dx, r_dx);
      frag_from_u32(vx, r_vx);
      frag_from_u32(kx, r_kx);
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sg = fmaf(X[n][e], sin_[n][e], sg);
          X[n][e] = fmaf(eL, X[n][e], dx[n][e]);
          zp[e >> 1] = fmaf(qf[n][e], dos[n][e], zp[e >> 1]);
          yp[e >> 1] = fmaf(kf[n][e], vx[n][e], yp[e >> 1]);
        }
      wait_bar(bar_d, ph_d);
      wait_bar(bar_e, ph_e);
      tc_fence_after();
      uint32_t r_q2[16], r_k2[16], r_v2[16];
      tmem_ld_16x32_async(r_q2, tw + TM_DQ2);
      tmem_ld_16x32_async(r_k2, tw + TM_DK2);
      tmem_ld_16x32_async(r_v2, tw + TM_DV2);
      tmem_wait_ld();
      float q2[4][4], k2[4][4], v2[4][4];
      frag_from_u32(q2, r_q2);
      frag_from_u32(k2, r_k2);
      frag_from_u32(v2, r_v2);
      // rows of this thread: steps ua, ub (dq rows t, dk/dv rows s)
      const float ea = fast_exp2(lua), eb = fast_exp2(lub);
      const float La = fast_exp2(gt.tot - lua), Lb = fast_exp2(gt.tot - lub);
      const float wa = sgw[ua], wb = sgw[ub];
      float kp[2] = {0.f, 0.f};
      float o_q[4][4], o_k[4][4], o_v[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool hi = e >= 2;
          const float ex = hi ? eb : ea, Lx = hi ? Lb : La, wx = hi ? wb : wa;
          o_q[n][e] = fmaf(ex, dos[n][e], q2[n][e]);
          o_k[n][e] = wx * fmaf(Lx, vx[n][e], k2[n][e]);
          o_v[n][e] = wx * fmaf(Lx, kx[n][e], v2[n][e]);
          kp[e >> 1] = fmaf(kf[n][e], k2[n][e], kp[e >> 1]);
        }
      // staged in shared memory; one TMA store per matrix after the barrier
      // (rows past T are clipped by the tensor map)
      store_frag_bf16(smem + SM_OUT, o_q, fr);
      store_frag_bf16(smem + SM_OUT + TILE, o_k, fr);
      store_frag_bf16(smem + SM_OUT + 2 * TILE, o_v, fr);
      fence_proxy_async();
      // per-row partials over this warp's 32 columns
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        zp[h] = quad_sum(zp[h]);
        yp[h] = quad_sum(yp[h]);
        kp[h] = quad_sum(kp[h]);
      }
      if (c4 == 0) {
        float* rowZ = part(SM_ROWZ, j & 1);
        float* rowY = part(SM_ROWY, j & 1);
        float* rowK = part(SM_ROWK, j & 1);
        rowZ[hf * 64 + ua] = zp[0];
        rowZ[hf * 64 + ub] = zp[1];
        rowY[hf * 64 + ua] = yp[0];
        rowY[hf * 64 + ub] = yp[1];
        rowK[hf * 64 + ua] = kp[0];
        rowK[hf * 64 + ub] = kp[1];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sg += __shfl_xor_sync(0xffffffffu, sg, o);
      if (lane == 0) part(SM_SIG, j & 1)[warp] = sg;
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tma_store_3d(&tdq, smem + SM_OUT, 0, gc * CH, bh);
      tma_store_3d(&tdk, smem + SM_OUT + TILE, 0, gc * CH, bh);
      tma_store_3d(&tdv, smem + SM_OUT + 2 * TILE, 0, gc * CH, bh);
      bulk_commit();
    }
    gprev = gt;
  }
  if (warp == NTHREADS / 32 - 1 && nc > 0) compute_df(c_begin, gprev, (nc - 1) & 1);
  if (stripe == 0 && p.dS0) store_frag_rowmajor(p.dS0 + (size_t)bh * D * D, X, fr);
  if (tid == 0) bulk_wait<0>();
  if (!ok) record_error(p.hdr, MOGT_ERR_TIMEOUT, unit);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
  if (tid == 0) finish_cta(p.hdr, epoch, gridDim.x);
}

// ---------------------------------------------------------------------------
// gated_bwd_seg_agg: the backward carry's aggregate over a segment of chunks
// (a third of a stripe), sum_c exp2(lpre_c) (diag(exp2 l) Q_c)^T dO_c with
// lpre_c the log2 decay of the segment's chunks before c, and the segment's
// total log2 decay, with three
// light CTAs per SM and one accumulator in tensor memory.  Written in reverse
// segment order, so that the forward's segment carry kernel run over them
// gives the carry entering each segment's end from the later ones.
// ---------------------------------------------------------------------------
constexpr int AB_RS = 4;                      // (q, do) ring slots
constexpr int AB_NBARS = 2 * AB_RS + 1;       // full and empty per slot, all-done
constexpr int AB_SM_BAR = AB_RS * 2 * TILE;
constexpr int AB_SM_TSLOT = AB_SM_BAR + 8 * AB_NBARS;
constexpr int AB_SM_ALLOC = AB_SM_TSLOT + 16 + 1024;
static_assert(3 * (AB_SM_ALLOC + 1024) <= 228 * 1024, "three CTAs per SM");

struct AggParams {
  const float* f;
  float* agg;    // [BH][nseg][4096] reversed segment order, stripe-aggregate layout
  float* lam;    // [BH][nseg]
  WsHeader* hdr;
  int T, BH, nchunks, cps, nsub, seg_len, nseg;
};

__global__ void __launch_bounds__(NTHREADS, 3)
    gated_bwd_seg_agg(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                      const AggParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2;
  const int br0 = build_row(tid, 0), br1 = build_row(tid, 1);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + AB_SM_BAR);
  uint64_t* empty = full + AB_RS;
  uint64_t* done = full + 2 * AB_RS;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + AB_SM_TSLOT);
  if (warp == 0) tmem_alloc(tslot, 64);
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < AB_NBARS; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tw = tbase + ((uint32_t)(32 * qd) << 16) + 32u * hf;
  const int gseg = blockIdx.x / p.BH, bh = blockIdx.x % p.BH;   // gseg in time order
  const int stripe = gseg / p.nsub, j = gseg % p.nsub;
  const int s0 = stripe * p.cps, s1 = min(s0 + p.cps, p.nchunks);
  const int c0 = min(s0 + j * p.seg_len, s1), c1 = min(c0 + p.seg_len, s1);
  const int n = c1 - c0, T = p.T;
  const float* fh = p.f + (size_t)bh * T;
  bool ok = true;

  auto issue = [&](int i) {
    if (i >= n) return;
    const int slot = i % AB_RS;
    uint8_t* base = smem + slot * 2 * TILE;
    mbar_arrive_expect_tx(&full[slot], 2 * TILE);
    tma_load_3d(base, &tq, &full[slot], 0, (c0 + i) * CH, bh);
    tma_load_3d(base + TILE, &tdo, &full[slot], 0, (c0 + i) * CH, bh);
  };
  if (tid == 0)
    for (int i = 0; i < AB_RS; ++i) issue(i);

  float lrun = 0.f;
  float2 fnext = n > 0 ? gate_load(fh, T, c0, lane) : make_float2(1.f, 1.f);
  for (int i = 0; i < n; ++i) {
    const WGates gt = warp_gates(fnext, lane);
    if (i + 1 < n) fnext = gate_load(fh, T, c0 + i + 1, lane);
    const int slot = i % AB_RS;
    if (!mbar_wait(&full[slot], (i / AB_RS) & 1)) ok = false;
    uint8_t* base = smem + slot * 2 * TILE;
    // Q rows scaled in place by exp2(lpre + l_t) (every factor <= 1)
    const float e0 = fast_exp2(lrun + gt.l0), e1 = fast_exp2(lrun + gt.l1);
    build_rows(base, base, step_val(e0, e1, br0), step_val(e0, e1, br1), tid);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      umma_64x64x64(tbase, smem_u32(base), true, smem_u32(base + TILE), true, i > 0);
      umma_commit(&empty[slot]);
      // the slot of chunk i-1 is free once its product completed
      if (i >= 1 && i - 1 + AB_RS < n) {
        const int ps = (i - 1) % AB_RS;
        if (!mbar_wait(&empty[ps], ((i - 1) / AB_RS) & 1)) ok = false;
        issue(i - 1 + AB_RS);
      }
    }
    __syncwarp();
    lrun += gt.tot;
  }
  float acc[4][4];
  zero44(acc);
  if (n > 0) {
    if (tid == 0) umma_commit(done);
    __syncwarp();
    if (!mbar_wait(done, 0)) ok = false;
    __syncwarp();
    tc_fence_after();
    tmem_ld_16x32(acc, tw);
    tc_fence_before();
  }
  const size_t gi = (size_t)bh * p.nseg + (p.nseg - 1 - gseg);
  float4* dst = reinterpret_cast<float4*>(p.agg + gi * (D * D) + (size_t)tid * 16);
#pragma unroll
  for (int k = 0; k < 4; ++k) __stcg(dst + k, make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]));
  if (tid == 0) p.lam[gi] = lrun;
  if (!ok) record_error(p.hdr, MOGT_ERR_TIMEOUT, blockIdx.x);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 64);
  }
}

}  // namespace bwd
}  // namespace gated
}  // namespace mogt

using namespace mogt;
using namespace mogt::gated;


namespace mogt {
namespace gated {

// The 256-byte header (ticket, epoch, sticky error), then the segment aggregates, log2
// decays and carries of the segment passes (bwd::kSub segments per stripe).
namespace bwd {
constexpr int kSub = 3;
struct SegLayout {
  size_t agg, lam, state, total;
};
inline SegLayout seg_layout(size_t base, size_t BH, size_t nseg) {
  SegLayout l;
  l.agg = mogt_host::align_up(base, 256);
  l.lam = l.agg + BH * nseg * D * D * 4;
  l.state = l.lam + mogt_host::align_up(BH * nseg * 4, 256);
  l.total = l.state + BH * nseg * D * D * 4;
  return l;
}
}  // namespace bwd

size_t bwd_tc_workspace_bytes(int64_t BH, int64_t T) {
  const Plan pl = make_plan(BH, T, sm_count());
  const size_t base = sizeof(WsHeader);
  return bwd::seg_layout(base, (size_t)BH, (size_t)pl.nstripes * bwd::kSub).total;
}

// Tensor-core backward; arguments are checked by the caller.
int launch_bwd_tc(const void* q, const void* k, const void* v, const float* f, const void* d_o,
                  const void* chunk_states, void* dq, void* dk, void* dv, float* df, float* dS0,
                  int BH, int T, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  const Plan pl = make_plan(BH, T, sm_count());
  const size_t NU = (size_t)BH * pl.nstripes;
  if (NU >= ((size_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  const int nseg = pl.nstripes * bwd::kSub;
  const bwd::SegLayout SL = bwd::seg_layout(sizeof(WsHeader), (size_t)BH, (size_t)nseg);
  if (!workspace || workspace_bytes < SL.total) return MOGT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOGT_ERR_ALIGN;
  CUtensorMap maps[8];
  const void* srcs[8] = {q, k, v, d_o, chunk_states, dq, dk, dv};
  for (int i = 0; i < 8; ++i) {
    const cuuint64_t rows = i == 4 ? (cuuint64_t)pl.nchunks * CH : (cuuint64_t)T;
    cuuint64_t dims[3] = {(cuuint64_t)D, rows, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, rows * D * 2};
    cuuint32_t box[3] = {(cuuint32_t)D, (cuuint32_t)CH, 1};
    if (mogt_host::encode_tiled(&maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                                const_cast<void*>(srcs[i]), dims, strides, box,
                                CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return MOGT_ERR_LAUNCH;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  bwd::Params P;
  P.f = f;
  P.dq = static_cast<__nv_bfloat16*>(dq);
  P.dk = static_cast<__nv_bfloat16*>(dk);
  P.dv = static_cast<__nv_bfloat16*>(dv);
  P.df = df;
  P.dS0 = dS0;
  P.hdr = reinterpret_cast<WsHeader*>(ws);
  P.T = T;
  P.BH = BH;
  P.nchunks = pl.nchunks;
  P.cps = pl.cps;
  P.nstripes = pl.nstripes;
  // the carry entering every stripe's end: segment aggregates (three light
  // CTAs per SM) and the segment carry
  bwd::AggParams A;
  A.f = f;
  A.agg = reinterpret_cast<float*>(ws + SL.agg);
  A.lam = reinterpret_cast<float*>(ws + SL.lam);
  A.hdr = P.hdr;
  A.T = T;
  A.BH = BH;
  A.nchunks = pl.nchunks;
  A.cps = pl.cps;
  A.nsub = bwd::kSub;
  A.seg_len = (pl.cps + bwd::kSub - 1) / bwd::kSub;
  A.nseg = nseg;
  cudaFuncSetAttribute(bwd::gated_bwd_seg_agg, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       bwd::AB_SM_ALLOC);
  bwd::gated_bwd_seg_agg<<<(unsigned)((size_t)BH * nseg), NTHREADS, bwd::AB_SM_ALLOC, s>>>(maps[0], maps[3], A);
  float* xstate = reinterpret_cast<float*>(ws + SL.state);
  const int cs = launch_seg_carry(A.agg, A.lam, xstate, BH, nseg, s);
  if (cs != MOGT_OK) return cs;
  P.x_in = xstate;
  P.nseg_b = nseg;
  P.nsub = bwd::kSub;
  cudaFuncSetAttribute(bwd::gated_bwd_stripe, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       bwd::SM_ALLOC);
  bwd::gated_bwd_stripe<<<(unsigned)NU, NTHREADS, bwd::SM_ALLOC, s>>>(
      maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], maps[6], maps[7], P);
  return mogt_host::launch_status();
}

}  // namespace gated
}  // namespace mogt
