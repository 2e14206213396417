// Headed gated scan, forward (bf16 q/k/v, dk = dv = 64, fp32 state):
//     S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,     o_t = S_t^T q_t.
// Reference semantics: affine_scan.py:14-62 run on U_t = f_t I,
// V_t = (1 - f_t) k_t v_t^T, followed by the readout einsum.
//
// Work decomposition ("stripes"): the T tokens of every (batch, head) are cut
// into 64-token chunks and the chunks into a few contiguous stripes, so that
// BH x stripes ~ one wave of resident CTAs.  A CTA (8 warps) owns one stripe:
//   pass 1  streams K, V chunks (TMA, 5-slot ring, L2 evict-last) and
//           accumulates the stripe's aggregate state
//               sum_s decay(s -> stripe end) (1 - f_s) k_s v_s^T
//           directly in tensor memory: chunk c's K rows are pre-scaled by
//           their decay to the stripe end, so no per-chunk read-back is needed;
//   look-back  a windowed decoupled look-back over the earlier stripes of the
//           same head yields the fp32 state entering the stripe; the stripe's
//           inclusive state is published for its successors;
//   pass 2  streams Q, K, V chunks again (3-slot ring, K, V mostly from L2)
//           and per chunk computes o = diag(a) Q S + ((Q K^T) o D) V and the
//           state update S <- a_C S + K~^T V.
// Tensor cores: every 64x64x64 product is a tcgen05.mma (kind::f16, bf16 ->
// fp32) issued by one thread from 128B-swizzled shared-memory tiles into
// tensor memory; the warps read accumulators back with tcgen05.ld, apply
// the causal mask (and exact decays when needed), and write the bf16
// operands of the next products.  Pass 2 is software-pipelined: the
// state-independent products of chunk c+1 run while chunk c is finished.
// Warp w owns rows 16(w%4)..+15 and columns 32(w/4)..+31 of every 64x64
// accumulator, and every warp derives the gate values it needs itself.
// Decays: chunk-local inclusive log2 cumulative gates l_t, D[t,s] =
// exp2(l_t - l_s) for s <= t.  When the chunk's total decay is above 2^-100
// the decay factorises, D[t,s] (1-f_s) = exp2(l_t) * [(1-f_s) exp2(-l_s)]:
// with Q^ = diag(exp2 l) Q and K~ = diag((1-f) exp2(-l)) K, P' is the
// causally masked Q^ K~^T and o = Q^ S + P' V; otherwise the exact
// per-element form is used.  Per-step log2 gates are
// clamped at -64 so f = 0 is a (numerically) full reset.
#include "common.cuh"
#include "gated_common.cuh"
#include "gated_internal.h"
#include "lookback.cuh"


namespace mogt {
namespace gated {

constexpr int STAGES = 3;                 // pass-2 ring: q, k, v per slot
constexpr int P1_STAGES = 5;              // pass-1 ring: k, v per slot
constexpr int P1_AHEAD = 3;               // pass-1 chunks loading ahead
constexpr int SLOT = 3 * TILE;            // q, k, v of one chunk

constexpr int SM_RING = 0;
constexpr int SM_SBUF = SM_RING + STAGES * SLOT;   // bf16 state operand [i][j] (+ pass-1 ring)
constexpr int SM_KT = SM_SBUF + TILE;              // scaled K, [s][i]
constexpr int SM_QT = SM_KT + TILE;                // scaled Q, [t][i]
constexpr int SM_PT = SM_QT + TILE;                // masked, decayed P, [t][s]
constexpr int SM_LSUF = SM_PT + TILE;              // pass-1 suffix decays
constexpr int SM_MISC = SM_LSUF + MAX_CPS * 4;
constexpr int NBARS = STAGES + P1_STAGES + 5;      // TMA rings, 2 pass-1 + 3 pass-2 MMA barriers
constexpr int SM_BAR = SM_MISC + 256;
constexpr int SM_TSLOT = SM_BAR + 8 * NBARS;
constexpr int SM_TOTAL = SM_TSLOT + 16;
// pass 1 reuses the q/k/v ring and the state-operand tile as a deeper k/v
// ring, and the scaled-K and scaled-Q tiles as a double-buffered scaled K;
// 2 CTAs per SM must fit
static_assert(2 * (SM_TOTAL + 1024 + 1024) <= 228 * 1024, "two CTAs per SM");
static_assert(P1_STAGES * 2 * TILE <= SM_KT - SM_RING, "pass-1 ring fits");
constexpr int SM_ALLOC = SM_TOTAL + 1024;
// tensor-memory columns (fp32, M = 64 accumulators in lanes 32q..32q+15):
// P, K~^T V and a double-buffered O (pass 2); pass 1 accumulates in TM_DS
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TM_P = 0, TM_DS = 64, TM_O0 = 128;

struct Params {
  const float* f;
  void* o;
  const float* S0;
  float* S_final;
  float* decay_final;
  __nv_bfloat16* chunk_states;  // [BH, nchunks, 64, 64] state entering each chunk, or null
  WsHeader* hdr;
  uint32_t* flags;
  float* a_agg;
  float* a_inc;
  float* st_agg;
  float* st_inc;
  int T, BH, nchunks, cps, nstripes;
};

template <bool OUT_F32>
__global__ void __launch_bounds__(NTHREADS, 2)
    gated_fwd_stripe(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2, g = lane >> 2, c4 = lane & 3;
  const Frag fr{qd * 16 + g, hf, c4};
  const int br0 = build_row(tid, 0), br1 = build_row(tid, 1);
  float* lsuf = reinterpret_cast<float*>(smem + SM_LSUF);
  volatile uint32_t* bc = reinterpret_cast<volatile uint32_t*>(smem + SM_MISC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
  uint64_t* bars1 = bars + STAGES;
  uint64_t* bar_k = bars + STAGES + P1_STAGES;   // pass-1 MMA commits (2)
  uint64_t* bar_m1 = bar_k + 2;                  // pass-2: P, Q^ S of a chunk
  uint64_t* bar_m2 = bar_k + 3;                  // pass-2: P' V of a chunk
  uint64_t* bar_m3 = bar_k + 4;                  // pass-2: K~^T V of a chunk
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM_TSLOT);
  uint8_t* kt_tile = smem + SM_KT;
  uint8_t* qt_tile = smem + SM_QT;
  uint8_t* pt_tile = smem + SM_PT;
  uint8_t* s_tile = smem + SM_SBUF;

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
  // this warp's accumulator slice: lanes 32 qd.., columns 32 hf..
  const uint32_t tw = tbase + ((uint32_t)(32 * qd) << 16) + 32u * hf;
  const uint32_t unit = bc[0], epoch = bc[1];
  const int BH = p.BH, T = p.T;
  const int stripe = (int)unit / BH, bh = (int)unit % BH;
  const int c_begin = stripe * p.cps;
  const int nc = min(p.cps, p.nchunks - c_begin);
  const bool has_succ = stripe + 1 < p.nstripes;
  const bool want_out = p.o != nullptr;
  const bool need_p2 = want_out || p.chunk_states != nullptr;
  const bool need_p1 = has_succ || !need_p2;
  const int n1 = need_p1 ? nc : 0;
  const int nit = n1 + (need_p2 ? nc : 0);
  const float* fh = p.f + (size_t)bh * T;
  uint32_t ph_m1 = 0, ph_m2 = 0, ph_m3 = 0;
  bool ok = true;

  uint64_t pol_keep = 0, pol_stream = 0;
  if (tid == 0) {
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_keep));
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_stream));
  }
  // TMA loads of pipeline iteration `it` (thread 0 only).  Pass-1 iterations
  // use the 5-slot k/v ring, pass-2 iterations the 3-slot q/k/v ring.
  auto issue = [&](int it) {
    if (it >= nit) return;
    const int t0 = (c_begin + (it < n1 ? it : it - n1)) * CH;
    if (it < n1) {
      const int slot = it % P1_STAGES;
      uint8_t* base = smem + SM_RING + slot * 2 * TILE;
      mbar_arrive_expect_tx(&bars1[slot], 2 * TILE);
      tma_load_3d_hint(base, &tk, &bars1[slot], 0, t0, bh, pol_keep);
      tma_load_3d_hint(base + TILE, &tv, &bars1[slot], 0, t0, bh, pol_keep);
    } else {
      const int j = it - n1, slot = j % STAGES;
      uint8_t* base = smem + SM_RING + slot * SLOT;
      mbar_arrive_expect_tx(&bars[slot], (want_out ? 3 : 2) * TILE);
      if (want_out) tma_load_3d_hint(base, &tq, &bars[slot], 0, t0, bh, pol_stream);
      tma_load_3d_hint(base + TILE, &tk, &bars[slot], 0, t0, bh, pol_stream);
      tma_load_3d_hint(base + 2 * TILE, &tv, &bars[slot], 0, t0, bh, pol_stream);
    }
  };
  auto wait_bar = [&](uint64_t* bar, uint32_t ph) {
    if (!mbar_wait(bar, ph)) ok = false;
  };

  if (tid == 0) {
    if (n1 > 0)
      for (int it = 0; it < P1_AHEAD && it < n1; ++it) issue(it);
    else
      for (int it = 0; it < STAGES - 1; ++it) issue(it);
  }

  // ---------------- pass 1: stripe aggregate in tensor memory ----------------
  float agg[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) agg[n][e] = 0.f;
  float ltot = 0.f;
  if (n1 > 0) {
    // suffix log2 decays: lsuf[c] = sum of the chunk log2 decays after c
    for (int c = warp; c < n1; c += NTHREADS / 32) {
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
      float sfx = part;  // inclusive suffix over lanes >= lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, sfx, o);
        if (lane + o < 32) sfx += y;
      }
      if (lane == 0) bc[2] = __float_as_uint(sfx);
      float run = sfx - part;  // sum over the chunks after this lane's block
      for (int c = c1 - 1; c >= c0; --c) {
        const float x = lsuf[c];
        lsuf[c] = run;
        run += x;
      }
    }
    __syncthreads();
  }
  {
    float2 fnext = n1 > 0 ? gate_load(fh, T, c_begin, lane) : make_float2(1.f, 1.f);
    for (int c = 0; c < n1; ++c) {
      const WGates gt = warp_gates(fnext, lane);
      if (c + 1 < n1) fnext = gate_load(fh, T, c_begin + c + 1, lane);
      if (c >= 2) wait_bar(&bar_k[c & 1], ((c - 2) >> 1) & 1);  // MMA of chunk c-2 done
      if (tid == 0 && c + P1_AHEAD < n1) issue(c + P1_AHEAD);    // into chunk c-2's slot
      if (!mbar_wait(&bars1[c % P1_STAGES], (c / P1_STAGES) & 1)) ok = false;
      // K~ rows: decay(s -> stripe end) (1 - f_s) = exp2(lsuf + tot - l_s) (1 - f_s)
      const float sc = lsuf[c] + gt.tot;
      const float k0 = fast_exp2(sc - gt.l0) * gt.w0, k1 = fast_exp2(sc - gt.l1) * gt.w1;
      const float s0 = step_val(k0, k1, br0), s1 = step_val(k0, k1, br1);
      uint8_t* base = smem + SM_RING + (c % P1_STAGES) * 2 * TILE;
      uint8_t* kt = (c & 1) ? qt_tile : kt_tile;
      build_rows(kt, base, s0, s1, tid);
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        umma_64x64x64(tbase + TM_DS, smem_u32(kt), true, smem_u32(base + TILE), true, c > 0);
        umma_commit(&bar_k[c & 1]);
      }
      __syncwarp();
    }
  }
  if (n1 > 0) {
    wait_bar(&bar_k[(n1 - 1) & 1], ((n1 - 1) >> 1) & 1);  // all pass-1 MMAs done
    tc_fence_after();
    tmem_ld_16x32(agg, tw + TM_DS);
    tc_fence_before();
    ltot = __uint_as_float(bc[2]);
  }
  if (n1 > 0) {
    // pass 1 has released the shared ring: prefetch the first pass-2 chunks so
    // they load during the look-back
    __syncthreads();
    if (tid == 0)
      for (int it = n1; it < n1 + STAGES - 1; ++it) issue(it);
  }
  const float A_agg = fast_exp2(ltot);
  const size_t st_off = (size_t)unit * (D * D) + (size_t)tid * 16;

  if (n1 > 0 && stripe > 0 && has_succ) {
    float4* dst = reinterpret_cast<float4*>(p.st_agg + st_off);
#pragma unroll
    for (int n = 0; n < 4; ++n) __stcg(dst + n, make_float4(agg[n][0], agg[n][1], agg[n][2], agg[n][3]));
    if (tid == 0) __stcg(p.a_agg + unit, A_agg);
    __threadfence();
    __syncthreads();
    if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagAgg));
  }

  // ---------------- state entering the stripe ----------------
  float sin[4][4];
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
    lookback_scalar_state<4>(sin, a_in, lb, stripe, (uint32_t)bh, (uint32_t)BH, epoch, unit,
                             reinterpret_cast<float*>(smem + SM_MISC + 64),
                             reinterpret_cast<volatile uint32_t*>(smem + SM_MISC + 16));
  }

  if (n1 > 0) {
    float inc_st[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) inc_st[n][e] = fmaf(A_agg, sin[n][e], agg[n][e]);
    if (has_succ) {
      float4* dst = reinterpret_cast<float4*>(p.st_inc + st_off);
#pragma unroll
      for (int n = 0; n < 4; ++n)
        __stcg(dst + n, make_float4(inc_st[n][0], inc_st[n][1], inc_st[n][2], inc_st[n][3]));
      if (tid == 0) __stcg(p.a_inc + unit, A_agg * a_in);
      __threadfence();
      __syncthreads();
      if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagInc));
    } else {
      if (p.S_final) store_frag_rowmajor(p.S_final + (size_t)bh * D * D, inc_st, fr);
      if (tid == 0 && p.decay_final) p.decay_final[bh] = A_agg * a_in;
    }
  }

  // ---------------- pass 2: outputs ----------------
  // Software pipeline, one CTA barrier per chunk.  In iteration c:
  //   wait the MMAs of chunk c (P, K~^T V, O_c = Q^ S_c, issued an iteration
  //   earlier) -> state S_{c+1} -> write the output of chunk c-1 -> mask P_c ->
  //   build Q^, K~ of chunk c+1 -> barrier -> one thread issues O_c += P'_c V_c
  //   and the state-independent MMAs of chunk c+1 and the TMA of chunk c+2.
  // O is double-buffered in tensor memory; the other operands are single.
  if (need_p2) {
    const bool final_here = !has_succ && n1 == 0;
    const int gc0 = c_begin;
    float2 fnext = gate_load(fh, T, gc0, lane);
    WGates gcur = warp_gates(fnext, lane);
    if (nc > 1) fnext = gate_load(fh, T, gc0 + 1, lane);
    float ltot2 = 0.f;
    // build the chunk-0 operands and issue its MMAs
    auto build_chunk = [&](int c, const WGates& gt) {
      // Q^ = diag(exp2 l_t) Q, K~ = diag(w_s exp2(-l_s)) K (factorised) or
      // diag(w_s exp2(lgC - l_s)) K (exact)
      const uint8_t* base = smem + SM_RING + (c % STAGES) * SLOT;
      const bool fast = factorises(gt);
      const float e0 = fast_exp2(gt.l0), e1 = fast_exp2(gt.l1);
      const float k0 = gt.w0 > 0.f ? gt.w0 * fast_exp2((fast ? 0.f : gt.tot) - gt.l0) : 0.f;
      const float k1 = gt.w1 > 0.f ? gt.w1 * fast_exp2((fast ? 0.f : gt.tot) - gt.l1) : 0.f;
      build_rows(kt_tile, base + TILE, step_val(k0, k1, br0), step_val(k0, k1, br1), tid);
      if (want_out) build_rows(qt_tile, base, step_val(e0, e1, br0), step_val(e0, e1, br1), tid);
    };
    // The MMA groups of a chunk touch disjoint tensor memory and are issued
    // by lane 0 of different warps so their issue latencies overlap:
    //   warp 1: P = Q^ K~^T (factorised) or Q K^T, and O_c = Q^ S_c -> bar_m1
    //   warp 2: dS = K~^T V                                       -> bar_m3
    //   warp 0: O_c += P' V (after the mask)                      -> bar_m2
    //   warp 3: TMA of the chunk two ahead
    auto issue_mma1 = [&](int c, bool fast) {
      const uint8_t* base = smem + SM_RING + (c % STAGES) * SLOT;
      const uint32_t qb = smem_u32(base), kb = smem_u32(base + TILE), vb = smem_u32(base + 2 * TILE);
      if (warp == 1 && lane == 0) {
        tc_fence_after();
        if (want_out) {
          if (fast)
            umma_64x64x64(tbase + TM_P, smem_u32(qt_tile), false, smem_u32(kt_tile), false, false);
          else
            umma_64x64x64(tbase + TM_P, qb, false, kb, false, false);
          umma_64x64x64(tbase + TM_O0 + 64u * (c & 1), smem_u32(qt_tile), false, smem_u32(s_tile),
                        true, false);
        }
        umma_commit(bar_m1);
      } else if (warp == 2 && lane == 0) {
        tc_fence_after();
        umma_64x64x64(tbase + TM_DS, smem_u32(kt_tile), true, vb, true, false);
        umma_commit(bar_m3);
      }
    };
    auto write_out_regs = [&](int c, const uint32_t (&r)[16]) {
      // output rows of chunk c from its O accumulator (already loaded)
      float oacc[4][4];
      frag_from_u32(oacc, r);
      const int ta = (gc0 + c) * CH + fr.r0, tb = ta + 8;
      const size_t rowa = ((size_t)bh * T + ta) * D, rowb = ((size_t)bh * T + tb) * D;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int j = 8 * (4 * hf + n) + 2 * c4;
        if (OUT_F32) {
          float* o = static_cast<float*>(p.o);
          if (ta < T) __stcs(reinterpret_cast<float2*>(o + rowa + j), make_float2(oacc[n][0], oacc[n][1]));
          if (tb < T) __stcs(reinterpret_cast<float2*>(o + rowb + j), make_float2(oacc[n][2], oacc[n][3]));
        } else {
          uint32_t* o = static_cast<uint32_t*>(p.o);
          if (ta < T) __stcs(o + (rowa + j) / 2, pack_bf16(oacc[n][0], oacc[n][1]));
          if (tb < T) __stcs(o + (rowb + j) / 2, pack_bf16(oacc[n][2], oacc[n][3]));
        }
      }
    };

    if (p.chunk_states)
      store_frag_rowmajor_bf16(p.chunk_states + ((size_t)bh * p.nchunks + gc0) * D * D, sin, fr);
    store_frag_bf16(s_tile, sin, fr);
    if (!mbar_wait(&bars[0], 0)) ok = false;
    build_chunk(0, gcur);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    issue_mma1(0, factorises(gcur));
    __syncwarp();

    for (int c = 0; c < nc; ++c) {
      const int it = n1 + c;
      const bool fast = factorises(gcur);
      // gates of chunk c+1: independent of the MMAs in flight
      WGates gnext = gcur;
      if (c + 1 < nc) {
        gnext = warp_gates(fnext, lane);
        if (c + 2 < nc) fnext = gate_load(fh, T, gc0 + c + 2, lane);
      }
      wait_bar(bar_m1, ph_m1);
      ph_m1 ^= 1u;
      wait_bar(bar_m3, ph_m3);
      ph_m3 ^= 1u;
      if (c > 0) {
        wait_bar(bar_m2, ph_m2);
        ph_m2 ^= 1u;
      }
      tc_fence_after();
      // the P and dS accumulators are read together
      const bool need_ds = c + 1 < nc || (final_here && p.S_final);
      uint32_t r_ds[16], r_p[16], r_o[16];
      if (need_ds) tmem_ld_16x32_async(r_ds, tw + TM_DS);
      if (want_out) tmem_ld_16x32_async(r_p, tw + TM_P);
      tmem_wait_ld();
      // state for chunk c+1 (or the final state)
      const float dC = fast_exp2(gcur.tot);
      ltot2 += gcur.tot;
      if (need_ds) {
        float ds[4][4];
        frag_from_u32(ds, r_ds);
        if (fast) {
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) sin[n][e] = dC * (sin[n][e] + ds[n][e]);
        } else {
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) sin[n][e] = fmaf(sin[n][e], dC, ds[n][e]);
        }
        if (c + 1 < nc) {
          store_frag_bf16(s_tile, sin, fr);
          if (p.chunk_states)
            store_frag_rowmajor_bf16(p.chunk_states + ((size_t)bh * p.nchunks + gc0 + c + 1) * D * D, sin, fr);
        }
      }
      // output of the previous chunk, read back only now: with all three
      // accumulators in flight at once the kernel spills at its 128-register cap
      if (want_out && c > 0) {
        tmem_ld_16x32_async(r_o, tw + TM_O0 + 64u * ((c - 1) & 1));
        tmem_wait_ld();
        write_out_regs(c - 1, r_o);
      }
      // P'_c: causal mask (and the exact decays when they do not factorise)
      if (want_out) {
        float pacc[4][4];
        frag_from_u32(pacc, r_p);
        const int tl0 = fr.r0, tl1 = tl0 + 8;
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
          const float lt0 = step_val(gcur.l0, gcur.l1, tl0), lt1 = step_val(gcur.l0, gcur.l1, tl1);
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int s = 8 * (4 * hf + n) + 2 * c4 + e;
              const float ls = step_val(gcur.l0, gcur.l1, s), ws = step_val(gcur.w0, gcur.w1, s);
              pacc[n][e] = (s <= tl0) ? pacc[n][e] * fast_exp2(lt0 - ls) * ws : 0.f;
              pacc[n][2 + e] = (s <= tl1) ? pacc[n][2 + e] * fast_exp2(lt1 - ls) * ws : 0.f;
            }
        }
        store_frag_bf16(pt_tile, pacc, fr);
      }
      // operands of chunk c+1
      if (c + 1 < nc) {
        if (!mbar_wait(&bars[(c + 1) % STAGES], ((c + 1) / STAGES) & 1)) ok = false;
        build_chunk(c + 1, gnext);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        if (want_out) {
          const uint32_t vb = smem_u32(smem + SM_RING + (c % STAGES) * SLOT + 2 * TILE);
          umma_64x64x64(tbase + TM_O0 + 64u * (c & 1), smem_u32(pt_tile), false, vb, true, true);
        }
        umma_commit(bar_m2);
      }
      if (c + 1 < nc) issue_mma1(c + 1, factorises(gnext));
      if (warp == 3 && lane == 0) issue(it + STAGES - 1);  // chunk c+2 into chunk c-1's slot
      __syncwarp();
      gcur = gnext;
    }
    // output of the last chunk
    wait_bar(bar_m2, ph_m2);
    ph_m2 ^= 1u;
    tc_fence_after();
    if (want_out) {
      uint32_t r_o[16];
      tmem_ld_16x32_async(r_o, tw + TM_O0 + 64u * ((nc - 1) & 1));
      tmem_wait_ld();
      write_out_regs(nc - 1, r_o);
    }
    if (final_here) {
      if (p.S_final) store_frag_rowmajor(p.S_final + (size_t)bh * D * D, sin, fr);
      if (tid == 0 && p.decay_final) p.decay_final[bh] = a_in * fast_exp2(ltot2);
    }
  }
  if (!ok) record_error(p.hdr, MOGT_ERR_TIMEOUT, unit);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
  if (tid == 0) finish_cta(p.hdr, epoch, gridDim.x);
}

}  // namespace gated
}  // namespace mogt

using namespace mogt;
using namespace mogt::gated;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }



extern "C" {


int64_t mogt_gated_scan_num_chunks(int64_t T, int64_t dk, int64_t dv, int in_dtype) {
  if (in_dtype != MOGT_DTYPE_BF16 || dk != D || dv != D || T <= 0) return 0;
  return (T + CH - 1) / CH;
}

size_t mogt_gated_scan_fwd_workspace_bytes(int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                           int in_dtype) {
  if (in_dtype != MOGT_DTYPE_BF16 || dk != D || dv != D || T <= 0 || BH <= 0)
    return sizeof(WsHeader);
  return chunked_fwd_workspace_bytes(BH, T);
}

// Checks every argument of a bf16 forward call and, when it is valid, returns
// the stripe plan and the workspace layout it needs.  Touches no memory.
static int validate_bf16_fwd(const void* q, const void* k, const void* v, const float* f,
                             const void* o, int64_t BH, int64_t T, int64_t dk, int64_t dv,
                             int out_dtype, Plan* pl, WsLayout* L) {
  if (!k || !v || !f || (o && !q)) return MOGT_ERR_ARG;
  if (BH >= ((int64_t)1 << 31) || T >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  if (dk != D || dv != D) return MOGT_ERR_UNSUPPORTED;
  if (out_dtype != MOGT_DTYPE_BF16 && out_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  if (!aligned16(k) || !aligned16(v) || (q && !aligned16(q)) || (o && !aligned16(o)))
    return MOGT_ERR_ALIGN;
  *pl = make_plan(BH, T, 2 * sm_count());
  const size_t NU = (size_t)BH * pl->nstripes;
  if (NU >= ((size_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  *L = ws_layout(NU);
  return MOGT_OK;
}

// The kernel's dynamic shared-memory limit is raised once per device.
static int prepare_kernels() {
  constexpr int kMaxDev = 64;
  static bool done[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return MOGT_ERR_LAUNCH;
  if (dev < kMaxDev && done[dev]) return MOGT_OK;
  if (cudaFuncSetAttribute(gated_fwd_stripe<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           SM_ALLOC) != cudaSuccess ||
      cudaFuncSetAttribute(gated_fwd_stripe<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           SM_ALLOC) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  if (dev < kMaxDev) done[dev] = true;
  return MOGT_OK;
}

}  // extern "C"

// The stripe kernel (one CTA per stripe, decoupled look-back between the
// stripes of a head): its workspace is the small look-back layout, so the
// allocation-free entry point runs it on its fixed scratch.
static int stripe_fwd(const void* q, const void* k, const void* v, const float* f, void* o,
                      const float* S0, float* S_final, float* decay_final, void* chunk_states,
                      int64_t BH, int64_t T, int64_t dk, int64_t dv, int out_dtype,
                      void* workspace, size_t workspace_bytes, cudaStream_t s) {
  Plan pl;
  WsLayout L;
  const int vs = validate_bf16_fwd(q, k, v, f, o, BH, T, dk, dv, out_dtype, &pl, &L);
  if (vs != MOGT_OK) return vs;
  if (!workspace || workspace_bytes < L.total) return MOGT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOGT_ERR_ALIGN;
  const size_t NU = (size_t)BH * pl.nstripes;
  if (prepare_kernels() != MOGT_OK) return MOGT_ERR_LAUNCH;

  CUtensorMap maps[3];
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
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  Params P;
  P.f = f;
  P.o = o;
  P.S0 = S0;
  P.S_final = S_final;
  P.decay_final = decay_final;
  P.chunk_states = static_cast<__nv_bfloat16*>(chunk_states);
  P.hdr = reinterpret_cast<WsHeader*>(ws);
  P.flags = reinterpret_cast<uint32_t*>(ws + L.flags);
  P.a_agg = reinterpret_cast<float*>(ws + L.a_agg);
  P.a_inc = reinterpret_cast<float*>(ws + L.a_inc);
  P.st_agg = reinterpret_cast<float*>(ws + L.st_agg);
  P.st_inc = reinterpret_cast<float*>(ws + L.st_inc);
  P.T = (int)T;
  P.BH = (int)BH;
  P.nchunks = pl.nchunks;
  P.cps = pl.cps;
  P.nstripes = pl.nstripes;
  if (out_dtype == MOGT_DTYPE_F32)
    gated_fwd_stripe<true><<<(unsigned)NU, NTHREADS, SM_ALLOC, s>>>(maps[0], maps[1], maps[2], P);
  else
    gated_fwd_stripe<false><<<(unsigned)NU, NTHREADS, SM_ALLOC, s>>>(maps[0], maps[1], maps[2], P);
  return mogt_host::launch_status();
}

extern "C" {

int mogt_gated_scan_fwd(const void* q, const void* k, const void* v, const float* f, void* o,
                        const float* S0, float* S_final, float* decay_final, void* chunk_states,
                        int64_t BH, int64_t T, int64_t dk, int64_t dv, int in_dtype, int out_dtype,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (BH <= 0 || T < 0 || dk <= 0 || dv <= 0) return MOGT_ERR_SHAPE;
  if (T == 0) return MOGT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (in_dtype == MOGT_DTYPE_F32) {
    if (!k || !v || !f || (o && !q)) return MOGT_ERR_ARG;
    if (BH >= ((int64_t)1 << 31) || T >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
    if (out_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
    if (chunk_states) return MOGT_ERR_UNSUPPORTED;
    return launch_fwd_seq(static_cast<const float*>(q), static_cast<const float*>(k),
                          static_cast<const float*>(v), f, static_cast<float*>(o), S0, S_final,
                          decay_final, (int)BH, (int)T, (int)dk, (int)dv, s);
  }
  if (in_dtype != MOGT_DTYPE_BF16) return MOGT_ERR_DTYPE;
  Plan pl;
  WsLayout L;
  const int vs = validate_bf16_fwd(q, k, v, f, o, BH, T, dk, dv, out_dtype, &pl, &L);
  if (vs != MOGT_OK) return vs;
  return launch_chunked_fwd(q, k, v, f, o, S0, S_final, decay_final, chunk_states, BH, T,
                            out_dtype, workspace, workspace_bytes, s, false);
}

int mogt_gated_scan_fwd_resume(const void* q, const void* k, const void* v, const float* f,
                               void* o, const float* S0, float* S_final, float* decay_final,
                               void* chunk_states, int64_t BH, int64_t T, int64_t dk, int64_t dv,
                               int in_dtype, int out_dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (BH <= 0 || T < 0 || dk <= 0 || dv <= 0) return MOGT_ERR_SHAPE;
  if (T == 0) return MOGT_OK;
  if (in_dtype != MOGT_DTYPE_BF16) return MOGT_ERR_UNSUPPORTED;
  Plan pl;
  WsLayout L;
  const int vs = validate_bf16_fwd(q, k, v, f, o, BH, T, dk, dv, out_dtype, &pl, &L);
  if (vs != MOGT_OK) return vs;
  return launch_chunked_fwd(q, k, v, f, o, S0, S_final, decay_final, chunk_states, BH, T,
                            out_dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                            true);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.  Its scratch is a fixed array in the library's
// device image instead of a caller-provided workspace, for callers that
// cannot allocate device memory.  The kernel and its arguments are exactly
// those of mogt_gated_scan_fwd.
//
// The array starts as the zero-filled .bss of the module, which is a valid
// look-back workspace; each call leaves the header (ticket, done counter,
// epoch) ready for the next call and clears only the per-unit flag words,
// because a call with another unit count lays its flags over words that an
// earlier call filled with state data.  The sticky error word is never
// cleared by a call: mogt_gated_scan_fwd_noalloc_status reads and clears it.
// ---------------------------------------------------------------------------
#include <mutex>

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of this device's copy of g_static_scratch.  In host code the
// symbol is only a host-side stand-in, so the address is looked up once per
// device with that device current.  Returns nullptr on failure.
void* static_scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess) return nullptr;
    g_scratch_addr[dev] = p;
  }
  return g_scratch_addr[dev];
}

}  // namespace

extern "C" int mogt_gated_scan_fwd_noalloc(const void* q, const void* k, const void* v,
                                           const float* f, void* o, const float* S0,
                                           float* S_final, float* decay_final, void* chunk_states,
                                           int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                           int in_dtype, int out_dtype, void* stream) {
  if (BH <= 0 || T < 0 || dk <= 0 || dv <= 0) return MOGT_ERR_SHAPE;
  if (T == 0) return MOGT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (in_dtype == MOGT_DTYPE_BF16) {
    // every argument is checked before the shared array is touched
    Plan pl;
    WsLayout L;
    const int vs = validate_bf16_fwd(q, k, v, f, o, BH, T, dk, dv, out_dtype, &pl, &L);
    if (vs != MOGT_OK) return vs;
    if (L.total > kStaticScratchBytes) return MOGT_ERR_TOO_LARGE;
    uint8_t* scratch = static_cast<uint8_t*>(static_scratch_for_current_device());
    if (!scratch) return MOGT_ERR_LAUNCH;
    if (cudaMemsetAsync(scratch + L.flags, 0, L.a_agg - L.flags, s) != cudaSuccess)
      return MOGT_ERR_LAUNCH;
    return stripe_fwd(q, k, v, f, o, S0, S_final, decay_final, chunk_states, BH, T, dk, dv,
                      out_dtype, scratch, kStaticScratchBytes, s);
  }
  // the fp32 path uses no scratch
  return mogt_gated_scan_fwd(q, k, v, f, o, S0, S_final, decay_final, chunk_states, BH, T, dk, dv,
                             in_dtype, out_dtype, nullptr, 0, stream);
}

extern "C" int mogt_gated_scan_fwd_noalloc_status(void* stream, int* err_out, uint32_t* unit_out) {
  if (!err_out) return MOGT_ERR_ARG;
  uint8_t* scratch = static_cast<uint8_t*>(static_scratch_for_current_device());
  if (!scratch) return MOGT_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t h[5];
  if (cudaMemcpyAsync(h, scratch, sizeof(h), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  *err_out = static_cast<int>(h[3]);
  if (unit_out) *unit_out = h[4];
  if (h[3] != 0) {
    // read and clear: the next error is recorded afresh
    if (cudaMemsetAsync(scratch + offsetof(WsHeader, err), 0, 2 * sizeof(uint32_t), s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return MOGT_ERR_LAUNCH;
  }
  return MOGT_OK;
}
