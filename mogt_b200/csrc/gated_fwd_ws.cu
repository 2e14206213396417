// Headed gated scan, forward, warp-specialised (bf16 q/k/v, dk = dv = 64):
//     S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,     o_t = S_t^T q_t.
// Reference semantics: affine_scan.py:14-62 run on U_t = f_t I,
// V_t = (1 - f_t) k_t v_t^T, followed by the readout einsum.
//
// Work decomposition: the 64-token chunks of every (batch, head) are cut into
// stripes, BH x stripes ~ one CTA per SM.  A CTA owns one stripe:
//   pass 1     stripe aggregate  sum_s decay(s -> stripe end) (1-f_s) k_s v_s^T
//              accumulated in tensor memory (K rows pre-scaled by their decay);
//   look-back  windowed decoupled look-back over the earlier stripes of the
//              head for the fp32 state entering the stripe;
//   pass 2     per chunk c: P = Q^ K~^T, dS = K~^T V (state independent),
//              O = Q^ S_c + P' V, S_{c+1} = a_C (S_c + dS)
// with the decay algebra of the lock-step kernel (chunk-local log2 cumulative
// gates l, factorised form when the chunk decay is above 2^-100, exact
// per-element form otherwise).
//
// Roles (22 warps, one CTA per SM, no CTA-wide barrier inside a pass):
//   warps 0-7    state group: pass-1 K~ tiles; aggregate read-back, look-back
//                and publication; the pass-2 state recurrence in registers
//                and the bf16 state tile (operand of O_c, per-chunk store);
//   warps 8-15   mask + output group: P' tiles, then O rows to global;
//   warps 16-19  pass-2 builders: scaled Q^ and K~ tiles from the TMA ring;
//   warp 20      TMA producer;  warp 21  tcgen05.mma issuer.
// Hand-offs are mbarriers (full/empty ring, built, mma1, dS-free, s-ready,
// p-ready, o-done, o-free, tiles-free), every wait bounded; tensor memory
// holds double-buffered P, dS and O (and the pass-1 aggregate).
#include "common.cuh"
#include "gated_common.cuh"
#include "lookback.cuh"
#include "trace.cuh"

namespace mogt {
namespace gated {
namespace ws {

constexpr int NWARPS = 22, NTH = NWARPS * 32;
constexpr int WG_S = 0, NST = 256, WG_O = 8, WG_B = 16, NB_WARPS = 4, W_TMA = 20, W_MMA = 21;
constexpr int NBT = 32 * NB_WARPS;    // builder threads
constexpr int BAR_S = 1;   // named barrier of the state group

constexpr int STAGES = 4;             // pass-2 ring: q, k, v per slot
constexpr int P1_STAGES = 6;          // pass-1 ring: k, v per slot
constexpr int SM_RING = 0;
constexpr int SM_QH = SM_RING + STAGES * 3 * TILE;   // Q^ [2]
constexpr int SM_KT = SM_QH + 2 * TILE;              // K~ [2]
constexpr int SM_SB = SM_KT + 2 * TILE;              // bf16 state [2]
constexpr int SM_PB = SM_SB + 2 * TILE;              // P' [2]
constexpr int SM_LSUF = SM_PB + 2 * TILE;            // pass-1 suffix decays
constexpr int SM_MISC = SM_LSUF + MAX_CPS * 4;       // ticket, stripe total, look-back scratch
static_assert(P1_STAGES * 2 * TILE <= SM_QH - SM_RING, "pass-1 ring fits");

enum : int {
  B_FULL = 0,
  B_EMPTY = B_FULL + STAGES,
  B_FULL1 = B_EMPTY + STAGES,
  B_EMPTY1 = B_FULL1 + P1_STAGES,
  B_BUILT1 = B_EMPTY1 + P1_STAGES,
  B_TFREE1 = B_BUILT1 + 2,
  B_AGG = B_TFREE1 + 2,
  B_BUILT = B_AGG + 1,
  B_TFREE = B_BUILT + 2,
  B_MMA1 = B_TFREE + 2,
  B_DSFREE = B_MMA1 + 2,
  B_SREADY = B_DSFREE + 2,
  B_PREADY = B_SREADY + 2,
  B_ODONE = B_PREADY + 2,
  B_OFREE = B_ODONE + 2,
  NBARS = B_OFREE + 2
};
constexpr int SM_BAR = SM_MISC + 256;
constexpr int SM_TSLOT = SM_BAR + 8 * NBARS;
constexpr int SM_TOTAL = SM_TSLOT + 16;
constexpr int SM_ALLOC = SM_TOTAL + 1024;
static_assert(SM_ALLOC <= 227 * 1024, "shared memory per CTA");

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TM_P = 0, TM_DS = 128, TM_O = 256, TM_AGG = 384;   // P, dS, O: [2] x 64

struct Params {
  const float* f;
  void* o;
  const float* S0;
  float* S_final;
  float* decay_final;
  bool states;       // per-chunk bf16 states stored through tstate
  WsHeader* hdr;
  uint32_t* flags;
  float* a_agg;
  float* a_inc;
  float* st_agg;
  float* st_inc;
  int T, BH, nchunks, cps, nstripes;
};

// dst rows of a 64x64 bf16 tile (swizzled) = scale_r * src rows for the
// rows (bt >> 3) + (NBT / 8) j of builder thread bt.
constexpr int BROWS = 512 / NBT;   // rows per builder thread
__device__ __forceinline__ void build_rows_b(uint8_t* dst, const uint8_t* src,
                                             const float (&sc)[BROWS], int bt) {
#pragma unroll
  for (int j = 0; j < BROWS; ++j) {
    const int q = bt + NBT * j, row = q >> 3, chunk = q & 7;
    const uint32_t off = sw128(row, chunk);
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    const __nv_bfloat16 h = __float2bfloat16_rn(sc[j]);
    const __nv_bfloat16 l = __float2bfloat16_rn(sc[j] - __bfloat162float(h));
    const __nv_bfloat162 hi = __halves2bfloat162(h, h), lo = __halves2bfloat162(l, l);
    uint4 w;
    w.x = bf2_scale(v.x, hi, lo);
    w.y = bf2_scale(v.y, hi, lo);
    w.z = bf2_scale(v.z, hi, lo);
    w.w = bf2_scale(v.w, hi, lo);
    *reinterpret_cast<uint4*>(dst + off) = w;
  }
}

template <bool OUT_F32>
__global__ void __launch_bounds__(NTH)
    gated_fwd_ws(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tst,
                 const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* lsuf = reinterpret_cast<float*>(smem + SM_LSUF);
  volatile uint32_t* bc = reinterpret_cast<volatile uint32_t*>(smem + SM_MISC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM_TSLOT);
  auto qh_tile = [&](int b) { return smem + SM_QH + b * TILE; };
  auto kt_tile = [&](int b) { return smem + SM_KT + b * TILE; };
  auto s_tile = [&](int b) { return smem + SM_SB + b * TILE; };
  auto p_tile = [&](int b) { return smem + SM_PB + b * TILE; };

  if (warp == WG_S) tmem_alloc(tslot, TMEM_COLS);
  if (tid == 0) {
    uint32_t epoch;
    bc[0] = take_ticket(p.hdr, &epoch);
    bc[1] = epoch;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars[B_FULL + s], 1);
      mbar_init(&bars[B_EMPTY + s], NB_WARPS + 1);
    }
    for (int s = 0; s < P1_STAGES; ++s) {
      mbar_init(&bars[B_FULL1 + s], 1);
      mbar_init(&bars[B_EMPTY1 + s], NST / 32 + 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars[B_BUILT1 + b], NST / 32);
      mbar_init(&bars[B_TFREE1 + b], 1);
      mbar_init(&bars[B_BUILT + b], NB_WARPS);
      mbar_init(&bars[B_TFREE + b], 1);
      mbar_init(&bars[B_MMA1 + b], 1);
      mbar_init(&bars[B_DSFREE + b], NST / 32);
      mbar_init(&bars[B_SREADY + b], NST / 32);
      mbar_init(&bars[B_PREADY + b], 8);
      mbar_init(&bars[B_ODONE + b], 1);
      mbar_init(&bars[B_OFREE + b], 8);
    }
    mbar_init(&bars[B_AGG], 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t unit = bc[0], epoch = bc[1];
  const int BH = p.BH, T = p.T;
  const int stripe = (int)unit / BH, bh = (int)unit % BH;
  const int c_begin = stripe * p.cps;
  const int nc = min(p.cps, p.nchunks - c_begin);
  const bool has_succ = stripe + 1 < p.nstripes;
  const bool want_out = p.o != nullptr;
  const bool need_p2 = want_out || p.states;
  const bool need_p1 = has_succ || !need_p2;
  const int n1 = need_p1 ? nc : 0;
  const int nc2 = need_p2 ? nc : 0;
  const float* fh = p.f + (size_t)bh * T;
  bool ok = true;
  auto wait = [&](int b, uint32_t parity) {
    if (!mbar_wait(&bars[b], parity)) ok = false;
  };
  MOGT_MARK(unit, 0);

  // pass-1 suffix decays (all warps), lsuf[c] = sum of the chunk log2 decays after c
  if (n1 > 0) {
    for (int c = warp; c < n1; c += NWARPS) {
      const float2 fv = gate_load(fh, T, c_begin + c, lane);
      float x = clamped_log2(fv.x) + clamped_log2(fv.y);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) lsuf[c] = x;
    }
    __syncthreads();
    if (warp == 0) {
      const int per = (n1 + 31) / 32, c0 = lane * per, c1 = min(c0 + per, n1);
      float part = 0.f;
      for (int c = c0; c < c1; ++c) part += lsuf[c];
      float sfx = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, sfx, o);
        if (lane + o < 32) sfx += y;
      }
      if (lane == 0) bc[2] = __float_as_uint(sfx);
      float run = sfx - part;
      for (int c = c1 - 1; c >= c0; --c) {
        const float x = lsuf[c];
        lsuf[c] = run;
        run += x;
      }
    }
    __syncthreads();
  }

  if (warp == W_TMA) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      uint64_t pol_keep, pol_stream;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_keep));
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_stream));
      for (int c = 0; c < n1; ++c) {
        const int s = c % P1_STAGES;
        wait(B_EMPTY1 + s, ((c / P1_STAGES) & 1) ^ 1);
        uint8_t* base = smem + SM_RING + s * 2 * TILE;
        mbar_arrive_expect_tx(&bars[B_FULL1 + s], 2 * TILE);
        tma_load_3d_hint(base, &tk, &bars[B_FULL1 + s], 0, (c_begin + c) * CH, bh, pol_keep);
        tma_load_3d_hint(base + TILE, &tv, &bars[B_FULL1 + s], 0, (c_begin + c) * CH, bh, pol_keep);
      }
      if (n1 > 0) wait(B_AGG, 0);   // pass 1 has released the ring
      for (int c = 0; c < nc2; ++c) {
        const int s = c % STAGES;
        wait(B_EMPTY + s, ((c / STAGES) & 1) ^ 1);
        uint8_t* base = smem + SM_RING + s * 3 * TILE;
        const int t0 = (c_begin + c) * CH;
        mbar_arrive_expect_tx(&bars[B_FULL + s], (want_out ? 3 : 2) * TILE);
        if (want_out) tma_load_3d_hint(base, &tq, &bars[B_FULL + s], 0, t0, bh, pol_stream);
        tma_load_3d_hint(base + TILE, &tk, &bars[B_FULL + s], 0, t0, bh, pol_stream);
        tma_load_3d_hint(base + 2 * TILE, &tv, &bars[B_FULL + s], 0, t0, bh, pol_stream);
      }
    }
  } else if (warp == W_MMA) {
    // ------------------------------ MMA issuer ------------------------------
    for (int c = 0; c < n1; ++c) {
      wait(B_BUILT1 + (c & 1), (c >> 1) & 1);
      if (lane == 0) {
        tc_fence_after();
        const uint8_t* base = smem + SM_RING + (c % P1_STAGES) * 2 * TILE;
        umma_64x64x64(tbase + TM_AGG, smem_u32(kt_tile(c & 1)), true, smem_u32(base + TILE), true,
                      c > 0);
        umma_commit(&bars[B_TFREE1 + (c & 1)]);
        umma_commit(&bars[B_EMPTY1 + c % P1_STAGES]);
      }
      __syncwarp();
    }
    if (n1 > 0 && lane == 0) umma_commit(&bars[B_AGG]);
    __syncwarp();
    if (nc2 > 0) {
      // P_c and dS_c (state independent) into buffer c & 1
      float2 fn = gate_load(fh, T, c_begin, lane);
      auto issue1 = [&](int c) {
        const WGates gt = warp_gates(fn, lane);
        if (c + 1 < nc2) fn = gate_load(fh, T, c_begin + c + 1, lane);
        const bool fast = factorises(gt);
        const uint32_t b = (uint32_t)(c & 1), ph = (c >> 1) & 1;
        wait(B_BUILT + b, ph);
        wait(B_DSFREE + b, ph ^ 1);   // dS_{c-2} read back (P_{c-2}: p-ready, waited before)
        if (lane == 0) {
          tc_fence_after();
          const uint8_t* base = smem + SM_RING + (c % STAGES) * 3 * TILE;
          if (want_out) {
            // P (factorised: Q^ K~^T, exact: Q K^T) interleaved with dS = K~^T V
            const uint32_t pa = fast ? smem_u32(qh_tile(b)) : smem_u32(base);
            const uint32_t pb = fast ? smem_u32(kt_tile(b)) : smem_u32(base + TILE);
            umma_64x64x64_x2(tbase + TM_P + 64u * b, pa, false, pb, false, tbase + TM_DS + 64u * b,
                             smem_u32(kt_tile(b)), true, smem_u32(base + 2 * TILE), true);
          } else {
            umma_64x64x64(tbase + TM_DS + 64u * b, smem_u32(kt_tile(b)), true,
                          smem_u32(base + 2 * TILE), true, false);
          }
          umma_commit(&bars[B_MMA1 + b]);
        }
        __syncwarp();
      };
      issue1(0);
      for (int c = 0; c < nc2; ++c) {
        MOGT_CLK_T(unit, 5, c == 5, 32 * W_MMA);
        if (c + 1 < nc2) issue1(c + 1);
        MOGT_CLK_T(unit, 6, c == 5, 32 * W_MMA);
        const uint32_t b = (uint32_t)(c & 1), ph = (c >> 1) & 1;
        const uint8_t* base = smem + SM_RING + (c % STAGES) * 3 * TILE;
        if (want_out) {
          wait(B_SREADY + b, ph);
          MOGT_CLK_T(unit, 7, c == 5, 32 * W_MMA);
          wait(B_OFREE + b, ph ^ 1);
          MOGT_CLK_T(unit, 8, c == 5, 32 * W_MMA);
          if (lane == 0) {
            tc_fence_after();
            umma_64x64x64(tbase + TM_O + 64u * b, smem_u32(qh_tile(b)), false, smem_u32(s_tile(b)),
                          true, false);
            umma_commit(&bars[B_TFREE + b]);
          }
          __syncwarp();
          wait(B_PREADY + b, ph);
          MOGT_CLK_T(unit, 9, c == 5, 32 * W_MMA);
          if (lane == 0) {
            tc_fence_after();
            umma_64x64x64(tbase + TM_O + 64u * b, smem_u32(p_tile(b)), false,
                          smem_u32(base + 2 * TILE), true, true);
            umma_commit(&bars[B_ODONE + b]);
            umma_commit(&bars[B_EMPTY + c % STAGES]);
          }
          __syncwarp();
        } else {
          if (lane == 0) {
            umma_commit(&bars[B_TFREE + b]);
            umma_commit(&bars[B_EMPTY + c % STAGES]);
          }
          __syncwarp();
        }
      }
    }
  } else if (warp >= WG_B && warp < WG_B + NB_WARPS) {
    // ------------------------------ builders (pass 2) ------------------------------
    const int bt = tid - 32 * WG_B;
    int rows[BROWS];
#pragma unroll
    for (int j = 0; j < BROWS; ++j) rows[j] = (bt >> 3) + (NBT / 8) * j;
    if (n1 > 0) wait(B_AGG, 0);   // the pass-1 MMAs have read the K~ tiles
    if (nc2 > 0) {
      float2 fn = gate_load(fh, T, c_begin, lane);
      for (int c = 0; c < nc2; ++c) {
        const WGates gt = warp_gates(fn, lane);
        if (c + 1 < nc2) fn = gate_load(fh, T, c_begin + c + 1, lane);
        const int s = c % STAGES;
        const uint8_t* base = smem + SM_RING + s * 3 * TILE;
        wait(B_FULL + s, (c / STAGES) & 1);
        wait(B_TFREE + (c & 1), ((c >> 1) & 1) ^ 1);
        // Q^ = diag(exp2 l) Q, K~ = diag(w exp2(-l)) K (factorised) or diag(w exp2(lgC - l)) K
        const bool fast = factorises(gt);
        const float kx = fast ? 0.f : gt.tot;
        const float k0 = gt.w0 > 0.f ? gt.w0 * fast_exp2(kx - gt.l0) : 0.f;
        const float k1 = gt.w1 > 0.f ? gt.w1 * fast_exp2(kx - gt.l1) : 0.f;
        float kr[BROWS];
#pragma unroll
        for (int j = 0; j < BROWS; ++j) kr[j] = step_val(k0, k1, rows[j]);
        build_rows_b(kt_tile(c & 1), base + TILE, kr, bt);
        if (want_out) {
          const float e0 = fast_exp2(gt.l0), e1 = fast_exp2(gt.l1);
          float qr[BROWS];
#pragma unroll
          for (int j = 0; j < BROWS; ++j) qr[j] = step_val(e0, e1, rows[j]);
          build_rows_b(qh_tile(c & 1), base, qr, bt);
        }
        fence_proxy_async();
        __syncwarp();
        MOGT_CLK_T(unit, 15, c == 6, 32 * WG_B);
        if (lane == 0) {
          mbar_arrive(&bars[B_BUILT + (c & 1)]);
          mbar_arrive(&bars[B_EMPTY + s]);
        }
      }
    }
  } else if (warp >= WG_O && warp < WG_O + 8) {
    // ------------------------- mask + output group (pass 2) -------------------------
    // warp (qd, hf): rows 16 qd.., columns 32 hf.. of P' and of O
    const int ow = warp - WG_O, qd = ow & 3, hf = ow >> 2;
    const int g = lane >> 2, c4 = lane & 3;
    const Frag fr{16 * qd + g, hf, c4};
    const uint32_t tw = tbase + ((uint32_t)(32 * qd) << 16) + 32u * hf;
    auto output = [&](int c) {
      const uint32_t b = (uint32_t)(c & 1);
      wait(B_ODONE + b, (c >> 1) & 1);
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32_async(r, tbase + ((uint32_t)(32 * qd) << 16) + TM_O + 64u * b + 32u * hf);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_OFREE + b]);
      const int t = (c_begin + c) * CH + 16 * qd + lane;
      if (lane < 16 && t < T) {
        const size_t row = ((size_t)bh * T + t) * D + 32 * hf;
        if (OUT_F32) {
          float4* o = reinterpret_cast<float4*>(static_cast<float*>(p.o) + row);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            __stcs(o + i, make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                      __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])));
        } else {
          uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.o) + row);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            __stcs(o + i, make_uint4(pack_bf16(__uint_as_float(r[8 * i]), __uint_as_float(r[8 * i + 1])),
                                     pack_bf16(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3])),
                                     pack_bf16(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5])),
                                     pack_bf16(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7]))));
        }
      }
    };
    if (want_out && nc2 > 0) {
      float2 fn = gate_load(fh, T, c_begin, lane);
      for (int c = 0; c < nc2; ++c) {
        const WGates gt = warp_gates(fn, lane);
        if (c + 1 < nc2) fn = gate_load(fh, T, c_begin + c + 1, lane);
        const uint32_t b = (uint32_t)(c & 1), ph = (c >> 1) & 1;
        const bool fast = factorises(gt);
        wait(B_MMA1 + b, ph);
        MOGT_CLK_T(unit, 12, c == 5, 32 * WG_O);
        tc_fence_after();
        uint32_t r_p[16];
        tmem_ld_16x32_async(r_p, tw + TM_P + 64u * b);
        tmem_wait_ld();
        tc_fence_before();
        // P'_c: causal mask (and the exact decays when they do not factorise)
        const int tl0 = fr.r0, tl1 = tl0 + 8;
        float pacc[4][4];
        frag_from_u32(pacc, r_p);
        if (fast) {
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int s = 8 * (4 * hf + n) + 2 * c4 + e;
              if (s > tl0) pacc[n][e] = 0.f;
              if (s > tl1) pacc[n][2 + e] = 0.f;
            }
        } else {
          const float lt0 = step_val(gt.l0, gt.l1, tl0), lt1 = step_val(gt.l0, gt.l1, tl1);
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int s = 8 * (4 * hf + n) + 2 * c4 + e;
              const float ls = step_val(gt.l0, gt.l1, s), wsv = step_val(gt.w0, gt.w1, s);
              pacc[n][e] = (s <= tl0) ? pacc[n][e] * fast_exp2(lt0 - ls) * wsv : 0.f;
              pacc[n][2 + e] = (s <= tl1) ? pacc[n][2 + e] * fast_exp2(lt1 - ls) * wsv : 0.f;
            }
        }
        wait(B_ODONE + b, ph ^ 1);   // P'_{c-2} V has read the tile
        store_frag_bf16(p_tile(b), pacc, fr);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_PREADY + b]);
        MOGT_CLK_T(unit, 13, c == 5, 32 * WG_O);
        if (c > 0) output(c - 1);
        MOGT_CLK_T(unit, 14, c == 5, 32 * WG_O);
      }
      output(nc2 - 1);
    }
  } else if (warp >= WG_S && warp < WG_S + 8) {
    // ------------------------------ state group ------------------------------
    // pass-1 builders, then the aggregate, look-back and the state recurrence
    const int qd = warp & 3, hf = warp >> 2, g = lane >> 2, c4 = lane & 3;
    const Frag fr{16 * qd + g, hf, c4};
    const uint32_t tw = tbase + ((uint32_t)(32 * qd) << 16) + 32u * hf;
    const int br0 = build_row(tid, 0), br1 = build_row(tid, 1);
    if (n1 > 0) {
      float2 fn = gate_load(fh, T, c_begin, lane);
      for (int c = 0; c < n1; ++c) {
        const WGates gt = warp_gates(fn, lane);
        if (c + 1 < n1) fn = gate_load(fh, T, c_begin + c + 1, lane);
        const int s = c % P1_STAGES;
        wait(B_FULL1 + s, (c / P1_STAGES) & 1);
        wait(B_TFREE1 + (c & 1), ((c >> 1) & 1) ^ 1);
        // K~ rows: decay(s -> stripe end) (1 - f_s) = exp2(lsuf + tot - l_s) (1 - f_s)
        const float sc = lsuf[c] + gt.tot;
        const float k0 = fast_exp2(sc - gt.l0) * gt.w0, k1 = fast_exp2(sc - gt.l1) * gt.w1;
        build_rows(kt_tile(c & 1), smem + SM_RING + s * 2 * TILE, step_val(k0, k1, br0),
                   step_val(k0, k1, br1), tid);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars[B_BUILT1 + (c & 1)]);
          mbar_arrive(&bars[B_EMPTY1 + s]);
        }
      }
    }
    float sin[4][4], agg[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) agg[n][e] = 0.f;
    float ltot = 0.f;
    if (n1 > 0) {
      wait(B_AGG, 0);
      tc_fence_after();
      tmem_ld_16x32(agg, tw + TM_AGG);
      tc_fence_before();
      ltot = __uint_as_float(bc[2]);
    }
    MOGT_MARK(unit, 1);
    const float A_agg = fast_exp2(ltot);
    const size_t st_off = (size_t)unit * (D * D) + (size_t)tid * 16;
    if (n1 > 0 && stripe > 0 && has_succ) {
      float4* dst = reinterpret_cast<float4*>(p.st_agg + st_off);
#pragma unroll
      for (int n = 0; n < 4; ++n) __stcg(dst + n, make_float4(agg[n][0], agg[n][1], agg[n][2], agg[n][3]));
      if (tid == 0) __stcg(p.a_agg + unit, A_agg);
      __threadfence();
      group_sync(BAR_S, NST);
      if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagAgg));
    }
    float a_in = 1.f;
    if (stripe == 0) {
      if (p.S0) {
        load_frag_rowmajor(sin, p.S0 + (size_t)bh * D * D, fr);
      } else {
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) sin[n][e] = 0.f;
      }
    } else {
      LookbackBufs lb{p.flags, p.a_agg, p.a_inc, p.st_agg, p.st_inc, p.hdr};
      lookback_scalar_state<4, NST>(sin, a_in, lb, stripe, (uint32_t)bh, (uint32_t)BH, epoch, unit,
                                    reinterpret_cast<float*>(smem + SM_MISC + 64),
                                    reinterpret_cast<volatile uint32_t*>(smem + SM_MISC + 16), tid,
                                    BAR_S);
    }
    MOGT_MARK(unit, 2);
    if (n1 > 0) {
      float inc[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) inc[n][e] = fmaf(A_agg, sin[n][e], agg[n][e]);
      if (has_succ) {
        float4* dst = reinterpret_cast<float4*>(p.st_inc + st_off);
#pragma unroll
        for (int n = 0; n < 4; ++n) __stcg(dst + n, make_float4(inc[n][0], inc[n][1], inc[n][2], inc[n][3]));
        if (tid == 0) __stcg(p.a_inc + unit, A_agg * a_in);
        __threadfence();
        group_sync(BAR_S, NST);
        if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagInc));
      } else {
        if (p.S_final) store_frag_rowmajor(p.S_final + (size_t)bh * D * D, inc, fr);
        if (tid == 0 && p.decay_final) p.decay_final[bh] = A_agg * a_in;
      }
    }
    MOGT_MARK(unit, 3);

    if (nc2 > 0) {
      const bool final_here = !has_succ && n1 == 0;
      // the state tile of chunk c: bf16 operand of O_c = Q^ S_c, and the
      // per-chunk state store
      auto put_state = [&](int c) {
        const uint32_t b = (uint32_t)(c & 1);
        wait(B_TFREE + b, ((c >> 1) & 1) ^ 1);   // O_{c-2} = Q^ S_{c-2} has read the tile
        if (p.states) {
          if (tid == 0) bulk_wait_read<1>();      // the store of S_{c-2} has read it too
          group_sync(BAR_S, NST);
        }
        store_frag_bf16(s_tile(b), sin, fr);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && want_out) mbar_arrive(&bars[B_SREADY + b]);
        if (p.states) {
          group_sync(BAR_S, NST);
          if (tid == 0) {
            tma_store_3d(&tst, s_tile(b), 0, (c_begin + c) * CH, bh);
            bulk_commit();
          }
        }
      };
      put_state(0);
      float2 fn = gate_load(fh, T, c_begin, lane);
      float ltot2 = 0.f;
      for (int c = 0; c < nc2; ++c) {
        const WGates gt = warp_gates(fn, lane);
        if (c + 1 < nc2) fn = gate_load(fh, T, c_begin + c + 1, lane);
        const uint32_t b = (uint32_t)(c & 1), ph = (c >> 1) & 1;
        const bool fast = factorises(gt);
        wait(B_MMA1 + b, ph);
        MOGT_CLK(unit, 10, c == 5);
        tc_fence_after();
        const bool need_ds = c + 1 < nc2 || (final_here && p.S_final);
        uint32_t r_ds[16];
        if (need_ds) {
          tmem_ld_16x32_async(r_ds, tw + TM_DS + 64u * b);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_DSFREE + b]);
        const float dC = fast_exp2(gt.tot);
        ltot2 += gt.tot;
        if (need_ds) {
          float ds[4][4];
          frag_from_u32(ds, r_ds);
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e)
              sin[n][e] = fast ? dC * (sin[n][e] + ds[n][e]) : fmaf(sin[n][e], dC, ds[n][e]);
        }
        if (c + 1 < nc2) put_state(c + 1);
        MOGT_CLK(unit, 11, c == 5);
      }
      if (final_here) {
        if (p.S_final) store_frag_rowmajor(p.S_final + (size_t)bh * D * D, sin, fr);
        if (tid == 0 && p.decay_final) p.decay_final[bh] = a_in * fast_exp2(ltot2);
      }
      if (p.states && tid == 0) bulk_wait<0>();
    }
  }
  MOGT_MARK(unit, 4);
  if (!ok) record_error(p.hdr, MOGT_ERR_TIMEOUT, unit);
  tc_fence_before();
  __syncthreads();
  if (warp == WG_S) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
  if (tid == 0) finish_cta(p.hdr, epoch, gridDim.x);
}

}  // namespace ws

// Launch of the warp-specialised forward (bf16 inputs, dk = dv = 64);
// arguments checked by the caller.
int launch_fwd_ws(const void* q, const void* k, const void* v, const float* f, void* o,
                  const float* S0, float* S_final, float* decay_final, void* chunk_states, int BH,
                  int T, bool out_f32, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  const Plan pl = make_plan(BH, T, sm_count());
  const size_t NU = (size_t)BH * pl.nstripes;
  if (NU >= ((size_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  const WsLayout L = ws_layout(NU);
  if (!workspace || workspace_bytes < L.total) return MOGT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOGT_ERR_ALIGN;
  CUtensorMap maps[4];
  const void* srcs[4] = {q ? q : k, k, v, chunk_states ? chunk_states : k};
  for (int i = 0; i < 4; ++i) {
    const cuuint64_t rows = (i == 3 && chunk_states) ? (cuuint64_t)pl.nchunks * CH : (cuuint64_t)T;
    cuuint64_t dims[3] = {(cuuint64_t)D, rows, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, rows * D * 2};
    cuuint32_t box[3] = {(cuuint32_t)D, (cuuint32_t)CH, 1};
    if (mogt_host::encode_tiled(&maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                                const_cast<void*>(srcs[i]), dims, strides, box,
                                CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return MOGT_ERR_LAUNCH;
  }
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  ws::Params P;
  P.f = f;
  P.o = o;
  P.S0 = S0;
  P.S_final = S_final;
  P.decay_final = decay_final;
  P.states = chunk_states != nullptr;
  P.hdr = reinterpret_cast<WsHeader*>(wsb);
  P.flags = reinterpret_cast<uint32_t*>(wsb + L.flags);
  P.a_agg = reinterpret_cast<float*>(wsb + L.a_agg);
  P.a_inc = reinterpret_cast<float*>(wsb + L.a_inc);
  P.st_agg = reinterpret_cast<float*>(wsb + L.st_agg);
  P.st_inc = reinterpret_cast<float*>(wsb + L.st_inc);
  P.T = T;
  P.BH = BH;
  P.nchunks = pl.nchunks;
  P.cps = pl.cps;
  P.nstripes = pl.nstripes;
  if (out_f32) {
    cudaFuncSetAttribute(ws::gated_fwd_ws<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ws::SM_ALLOC);
    ws::gated_fwd_ws<true><<<(unsigned)NU, ws::NTH, ws::SM_ALLOC, s>>>(maps[0], maps[1], maps[2], maps[3], P);
  } else {
    cudaFuncSetAttribute(ws::gated_fwd_ws<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ws::SM_ALLOC);
    ws::gated_fwd_ws<false><<<(unsigned)NU, ws::NTH, ws::SM_ALLOC, s>>>(maps[0], maps[1], maps[2], maps[3], P);
  }
  return mogt_host::launch_status();
}

size_t fwd_ws_workspace_bytes(int64_t BH, int64_t T) {
  const Plan pl = make_plan(BH, T, sm_count());
  return ws_layout((size_t)BH * pl.nstripes).total;
}

}  // namespace gated
}  // namespace mogt

#ifdef MOGT_TRACE
extern "C" int mogt_debug_set_trace_ws(void* buf) { return mogt::set_trace(buf); }
#endif
