// Warp-specialised gated-scan forward kernel (design notes in gated_fwd_ws.cuh).
#include "gated_fwd_ws.cuh"

namespace mogt {
namespace gated {
namespace ws {

template <bool OUT_F32>
__global__ void __launch_bounds__(NTH, 1)
    gated_fwd_ws(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  volatile uint32_t* mw = reinterpret_cast<volatile uint32_t*>(smem + SM_MISC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM_TSLOT);
  float* lsuf = reinterpret_cast<float*>(smem + SM_LSUF);

  if (warp == W_TMA) tmem_alloc(tslot, TMEM_COLS);
  if (tid == 32 * W_MMA) {
    uint32_t epoch;
    mw[MW_TICKET] = take_ticket(p.hdr, &epoch);
    mw[MW_EPOCH] = epoch;
    mw[MW_ABORT] = 0;
    const uint8_t counts[NBARS] = {1, 1, 1, 1, 1, 1, 4, 4, 1, 1, 1, 1, 4, 4, 4, 4, 1, 1, 1, 1, 4, 4,
                                   4, 4, 1, 1, 1, 1, 4, 4};
#pragma unroll
    for (int i = 0; i < NBARS; ++i) mbar_init(&bars[i], counts[i]);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t unit = mw[MW_TICKET], epoch = mw[MW_EPOCH];
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
  const int has_agg = n1 > 0 ? 1 : 0;
  const float* fh = p.f + (size_t)bh * T;
  bool ok = true;
  // bounded wait; after the first timeout in the CTA every later wait returns
  // at once, so a broken protocol costs one wait limit, not one per wait
  auto wait = [&](int b, uint32_t parity) {
    if (mw[MW_ABORT]) return;
    if (!mbar_wait(&bars[b], parity)) {
      mw[MW_ABORT] = 1;
      ok = false;
    }
  };
  const int q4 = warp & 3, g = lane >> 2, c4 = lane & 3;

  if (warp == W_TMA) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint64_t pol_keep, pol_stream;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_keep));
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_stream));
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      for (int it = 0; it < nit; ++it) {
        const int slot = it % NS, use = it / NS;
        wait(B_EMPTY_IN + slot, prod_parity(use));
        if (mw[MW_ABORT]) break;
        uint8_t* base = smem + SM_IN + slot * 3 * TILE;
        const bool p1 = it < n1;
        const int t0 = (c_begin + (p1 ? it : it - n1)) * CH;
        const bool with_q = !p1 && want_out;
        const uint64_t pol = p1 ? pol_keep : pol_stream;
        mbar_arrive_expect_tx(&bars[B_FULL_IN + slot], (with_q ? 3 : 2) * TILE);
        if (with_q) tma_load_3d_hint(base, &tq, &bars[B_FULL_IN + slot], 0, t0, bh, pol);
        tma_load_3d_hint(base + TILE, &tk, &bars[B_FULL_IN + slot], 0, t0, bh, pol);
        tma_load_3d_hint(base + 2 * TILE, &tv, &bars[B_FULL_IN + slot], 0, t0, bh, pol);
      }
    }
  } else if (warp == W_MMA) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      auto commit = [&](int b) { umma_commit(&bars[b]); };
      // pass 1: stripe aggregate sum_c K~_c^T V_c in dS[0]
      for (int c = 0; c < n1; ++c) {
        const int slot = c % NS, b = c % NB;
        wait(B_FULL_IN + slot, cons_parity(c / NS));
        wait(B_FULL_B + b, cons_parity(c / NB));
        if (c == 0) wait(B_EMPTY_DS + 0, prod_parity(0));
        if (mw[MW_ABORT]) break;
        tc_fence_after();
        const uint8_t* kt = smem + SM_BLD + b * 2 * TILE + TILE;
        const uint8_t* vb = smem + SM_IN + slot * 3 * TILE + 2 * TILE;
        umma_64x64x64(tbase + TM_DS, smem_u32(kt), true, smem_u32(vb), true, c > 0);
        commit(B_EMPTY_IN + slot);
        commit(B_EMPTY_B + b);
      }
      if (n1 > 0) commit(B_FULL_DS + 0);
      // pass 2
      auto indep = [&](int j) {
        const int it = n1 + j, slot = it % NS, b = it % NB;
        wait(B_FULL_IN + slot, cons_parity(it / NS));
        wait(B_FULL_B + b, cons_parity(it / NB));
        const bool fast = mw[MW_FAST + b] != 0;
        const uint8_t* in = smem + SM_IN + slot * 3 * TILE;
        const uint8_t* bl = smem + SM_BLD + b * 2 * TILE;
        if (want_out) {
          wait(B_EMPTY_P + (j & 1), prod_parity(j >> 1));
          tc_fence_after();
          if (fast)
            umma_64x64x64(tbase + TM_P + 64u * (j & 1), smem_u32(bl), false, smem_u32(bl + TILE), false,
                          false);
          else
            umma_64x64x64(tbase + TM_P + 64u * (j & 1), smem_u32(in), false, smem_u32(in + TILE), false,
                          false);
          commit(B_FULL_P + (j & 1));
        }
        const int d = j + has_agg;
        wait(B_EMPTY_DS + (d & 1), prod_parity(d >> 1));
        tc_fence_after();
        umma_64x64x64(tbase + TM_DS + 64u * (d & 1), smem_u32(bl + TILE), true, smem_u32(in + 2 * TILE),
                      true, false);
        commit(B_FULL_DS + (d & 1));
      };
      if (need_p2) indep(0);
      for (int j = 0; need_p2 && j < nc; ++j) {
        if (mw[MW_ABORT]) break;
        if (j + 1 < nc) indep(j + 1);
        const int it = n1 + j, slot = it % NS, b = it % NB;
        if (want_out) {
          wait(B_FULL_S + (j & 1), cons_parity(j >> 1));
          wait(B_FULL_PP + (j & 1), cons_parity(j >> 1));
          wait(B_EMPTY_O + (j & 1), prod_parity(j >> 1));
          if (mw[MW_ABORT]) break;
          tc_fence_after();
          const uint32_t od = tbase + TM_O + 64u * (j & 1);
          const uint8_t* bl = smem + SM_BLD + b * 2 * TILE;
          const uint8_t* vb = smem + SM_IN + slot * 3 * TILE + 2 * TILE;
          umma_64x64x64(od, smem_u32(bl), false, smem_u32(smem + SM_S + (j & 1) * TILE), true, false);
          umma_64x64x64(od, smem_u32(smem + SM_PP + (j & 1) * TILE), false, smem_u32(vb), true, true);
          commit(B_FULL_O + (j & 1));
          commit(B_EMPTY_S + (j & 1));
          commit(B_EMPTY_PP + (j & 1));
        }
        commit(B_EMPTY_IN + slot);
        commit(B_EMPTY_B + b);
      }
    }
  } else if (warp < W_ST) {
    // ---------------- builders ----------------
    const int bt = tid - 32 * W_BLD;
    int rows[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) rows[j] = (bt >> 3) + 16 * j;
    if (n1 > 0) {
      // suffix log2 decays of the stripe's chunks: lsuf[c] = sum over c' > c
      for (int c = warp - W_BLD; c < n1; c += 4) {
        const float2 fv = gate_load(fh, T, c_begin + c, lane);
        float x = clamped_log2(fv.x) + clamped_log2(fv.y);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if (lane == 0) lsuf[c] = x;
      }
      group_sync(BAR_BLD, 128);
      if (warp == W_BLD) {
        const int per = (n1 + 31) / 32, c0 = lane * per, c1 = min(c0 + per, n1);
        float part = 0.f;
        for (int c = c0; c < c1; ++c) part += lsuf[c];
        float sfx = part;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, sfx, o);
          if (lane + o < 32) sfx += y;
        }
        float run = sfx - part;
        for (int c = c1 - 1; c >= c0; --c) {
          const float x = lsuf[c];
          lsuf[c] = run;
          run += x;
        }
      }
      group_sync(BAR_BLD, 128);
    }
    float2 fnext = gate_load(fh, T, c_begin, lane);
    for (int it = 0; it < nit; ++it) {
      const bool p1 = it < n1;
      const int c = p1 ? it : it - n1;
      const WGates gt = warp_gates(fnext, lane);
      const int cn = (it + 1 < n1) ? it + 1 : (it + 1 - n1);
      if (it + 1 < nit) fnext = gate_load(fh, T, c_begin + cn, lane);
      const int slot = it % NS, b = it % NB;
      float ks[4], qs[4];
      const bool fast = factorises(gt);
      if (p1) {
        // K~ rows: decay(s -> stripe end) (1 - f_s) = exp2(lsuf + tot - l_s) (1 - f_s)
        const float sc = lsuf[c] + gt.tot;
        const float k0 = fast_exp2(sc - gt.l0) * gt.w0, k1 = fast_exp2(sc - gt.l1) * gt.w1;
#pragma unroll
        for (int j = 0; j < 4; ++j) ks[j] = step_val(k0, k1, rows[j]);
      } else {
        const float e0 = fast_exp2(gt.l0), e1 = fast_exp2(gt.l1);
        const float base = fast ? 0.f : gt.tot;
        const float k0 = gt.w0 > 0.f ? gt.w0 * fast_exp2(base - gt.l0) : 0.f;
        const float k1 = gt.w1 > 0.f ? gt.w1 * fast_exp2(base - gt.l1) : 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ks[j] = step_val(k0, k1, rows[j]);
          qs[j] = step_val(e0, e1, rows[j]);
        }
      }
      wait(B_FULL_IN + slot, cons_parity(it / NS));
      wait(B_EMPTY_B + b, prod_parity(it / NB));
      if (mw[MW_ABORT]) break;
      const uint8_t* in = smem + SM_IN + slot * 3 * TILE;
      uint8_t* bl = smem + SM_BLD + b * 2 * TILE;
      build4(bl + TILE, in + TILE, ks, bt);
      if (!p1 && want_out) build4(bl, in, qs, bt);
      if (bt == 0) mw[MW_FAST + b] = fast ? 1u : 0u;
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_FULL_B + b]);
    }
  } else if (warp < W_MO) {
    // ---------------- state ----------------
    const int st = tid - 32 * W_ST;  // 0..127
    const Frag fr0{q4 * 16 + g, 0, c4}, fr1{q4 * 16 + g, 1, c4};
    const uint32_t tw = tbase + ((uint32_t)(32 * q4) << 16);
    // log2 decay of the whole stripe (pass 1 chunks): warps take chunks in turn
    float ltot = 0.f;
    if (n1 > 0) {
      float part = 0.f;
      for (int c = warp - W_ST; c < n1; c += 4) {
        const float2 fv = gate_load(fh, T, c_begin + c, lane);
        float x = clamped_log2(fv.x) + clamped_log2(fv.y);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        part += x;
      }
      float* pp = reinterpret_cast<float*>(const_cast<uint32_t*>(mw + MW_PART));
      if (lane == 0) pp[warp - W_ST] = part;
      group_sync(BAR_ST, 128);
      ltot = (pp[0] + pp[1]) + (pp[2] + pp[3]);
      // the stripe aggregate accumulated by pass 1 (dS[0] is released only
      // after the inclusive state is formed: it is read again then)
      wait(B_FULL_DS + 0, cons_parity(0));
      tc_fence_after();
    }
    const float A_agg = fast_exp2(ltot);
    const size_t st_off = (size_t)unit * (D * D) + (size_t)st * 32;
    auto publish = [&](float* dst_base, const float (&s)[2][4][4]) {
      float4* dst = reinterpret_cast<float4*>(dst_base + st_off);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int n = 0; n < 4; ++n) __stcg(dst + 4 * h + n, make_float4(s[h][n][0], s[h][n][1], s[h][n][2], s[h][n][3]));
    };
    if (n1 > 0 && stripe > 0 && has_succ) {
      float agg[2][4][4];
      tmem_ld_rows64(agg, tw + TM_DS);
      publish(p.st_agg, agg);
      if (st == 0) __stcg(p.a_agg + unit, A_agg);
      __threadfence();
      group_sync(BAR_ST, 128);
      if (st == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagAgg));
    }
    // state entering the stripe
    float S[2][4][4];
    float a_in = 1.f;
    if (stripe == 0) {
      if (p.S0) {
        load_frag_rowmajor(S[0], p.S0 + (size_t)bh * D * D, fr0);
        load_frag_rowmajor(S[1], p.S0 + (size_t)bh * D * D, fr1);
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) S[h][n][e] = 0.f;
      }
    } else {
      LookbackBufs lb{p.flags, p.a_agg, p.a_inc, p.st_agg, p.st_inc, p.hdr};
      float (&acc)[8][4] = *reinterpret_cast<float(*)[8][4]>(&S[0][0][0]);
      lookback_scalar_state<8, 128>(acc, a_in, lb, stripe, (uint32_t)bh, (uint32_t)BH, epoch, unit,
                                    reinterpret_cast<float*>(const_cast<uint32_t*>(mw + MW_LBSCL)),
                                    mw + MW_LBCTL, st, BAR_ST);
    }
    if (n1 > 0) {
      float inc[2][4][4];
      tmem_ld_rows64(inc, tw + TM_DS);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_EMPTY_DS + 0]);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) inc[h][n][e] = fmaf(A_agg, S[h][n][e], inc[h][n][e]);
      if (has_succ) {
        publish(p.st_inc, inc);
        if (st == 0) __stcg(p.a_inc + unit, A_agg * a_in);
        __threadfence();
        group_sync(BAR_ST, 128);
        if (st == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagInc));
      } else {
        if (p.S_final) {
          store_frag_rowmajor(p.S_final + (size_t)bh * D * D, inc[0], fr0);
          store_frag_rowmajor(p.S_final + (size_t)bh * D * D, inc[1], fr1);
        }
        if (st == 0 && p.decay_final) p.decay_final[bh] = A_agg * a_in;
      }
    }
    if (need_p2) {
      const bool final_here = !has_succ && n1 == 0;
      float ltot2 = 0.f;
      float2 fnext = gate_load(fh, T, c_begin, lane);
      for (int j = 0; j < nc; ++j) {
        const WGates gt = warp_gates(fnext, lane);
        if (j + 1 < nc) fnext = gate_load(fh, T, c_begin + j + 1, lane);
        // the state entering chunk j: bf16 operand of O_j = Q^_j S_j, and the
        // per-chunk copy kept for the backward
        if (p.chunk_states) {
          __nv_bfloat16* cs = p.chunk_states + ((size_t)bh * p.nchunks + c_begin + j) * D * D;
          store_frag_rowmajor_bf16(cs, S[0], fr0);
          store_frag_rowmajor_bf16(cs, S[1], fr1);
        }
        if (want_out) {
          wait(B_EMPTY_S + (j & 1), prod_parity(j >> 1));
          uint8_t* stile = smem + SM_S + (j & 1) * TILE;
          store_frag_bf16(stile, S[0], fr0);
          store_frag_bf16(stile, S[1], fr1);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[B_FULL_S + (j & 1)]);
        }
        // S <- a (S + K~^T V) (factorised) or a S + K~^T V (exact)
        const int d = j + has_agg;
        wait(B_FULL_DS + (d & 1), cons_parity(d >> 1));
        if (mw[MW_ABORT]) break;
        tc_fence_after();
        float ds[2][4][4];
        tmem_ld_rows64(ds, tw + TM_DS + 64u * (d & 1));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_EMPTY_DS + (d & 1)]);
        const float dC = fast_exp2(gt.tot);
        ltot2 += gt.tot;
        if (factorises(gt)) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
              for (int e = 0; e < 4; ++e) S[h][n][e] = dC * (S[h][n][e] + ds[h][n][e]);
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
              for (int e = 0; e < 4; ++e) S[h][n][e] = fmaf(S[h][n][e], dC, ds[h][n][e]);
        }
      }
      if (final_here) {
        if (p.S_final) {
          store_frag_rowmajor(p.S_final + (size_t)bh * D * D, S[0], fr0);
          store_frag_rowmajor(p.S_final + (size_t)bh * D * D, S[1], fr1);
        }
        if (st == 0 && p.decay_final) p.decay_final[bh] = a_in * fast_exp2(ltot2);
      }
    }
  } else {
    // ---------------- mask + output ----------------
    // iteration j: P'_j from P_j, then the output rows of chunk j - 1 (its
    // O product needs P'_{j-1}, formed an iteration earlier)
    const uint32_t tw = tbase + ((uint32_t)(32 * q4) << 16);
    const int tl0 = q4 * 16 + g, tl1 = tl0 + 8;
    auto write_out = [&](int j) {
      wait(B_FULL_O + (j & 1), cons_parity(j >> 1));
      if (mw[MW_ABORT]) return;
      tc_fence_after();
      float oa[2][4][4];
      tmem_ld_rows64(oa, tw + TM_O + 64u * (j & 1));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_EMPTY_O + (j & 1)]);
      const int ta = (c_begin + j) * CH + tl0, tb = ta + 8;
      const size_t rowa = ((size_t)bh * T + ta) * D, rowb = ((size_t)bh * T + tb) * D;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int col = 8 * (4 * h + n) + 2 * c4;
          if (OUT_F32) {
            float* o = static_cast<float*>(p.o);
            if (ta < T) __stcs(reinterpret_cast<float2*>(o + rowa + col), make_float2(oa[h][n][0], oa[h][n][1]));
            if (tb < T) __stcs(reinterpret_cast<float2*>(o + rowb + col), make_float2(oa[h][n][2], oa[h][n][3]));
          } else {
            uint32_t* o = static_cast<uint32_t*>(p.o);
            if (ta < T) __stcs(o + (rowa + col) / 2, pack_bf16(oa[h][n][0], oa[h][n][1]));
            if (tb < T) __stcs(o + (rowb + col) / 2, pack_bf16(oa[h][n][2], oa[h][n][3]));
          }
        }
    };
    float2 fnext = gate_load(fh, T, c_begin, lane);
    for (int j = 0; want_out && j < nc; ++j) {
      const WGates gt = warp_gates(fnext, lane);
      if (j + 1 < nc) fnext = gate_load(fh, T, c_begin + j + 1, lane);
      const bool fast = factorises(gt);
      wait(B_FULL_P + (j & 1), cons_parity(j >> 1));
      if (mw[MW_ABORT]) break;
      tc_fence_after();
      float pa[2][4][4];
      tmem_ld_rows64(pa, tw + TM_P + 64u * (j & 1));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_EMPTY_P + (j & 1)]);
      const float lt0 = step_val(gt.l0, gt.l1, tl0), lt1 = step_val(gt.l0, gt.l1, tl1);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int s = 8 * (4 * h + n) + 2 * c4 + e;
            if (fast) {
              if (s > tl0) pa[h][n][e] = 0.f;
              if (s > tl1) pa[h][n][2 + e] = 0.f;
            } else {
              const float ls = step_val(gt.l0, gt.l1, s), wsv = step_val(gt.w0, gt.w1, s);
              pa[h][n][e] = (s <= tl0) ? pa[h][n][e] * fast_exp2(lt0 - ls) * wsv : 0.f;
              pa[h][n][2 + e] = (s <= tl1) ? pa[h][n][2 + e] * fast_exp2(lt1 - ls) * wsv : 0.f;
            }
          }
      wait(B_EMPTY_PP + (j & 1), prod_parity(j >> 1));
      uint8_t* pt = smem + SM_PP + (j & 1) * TILE;
      store_frag_bf16(pt, pa[0], Frag{tl0, 0, c4});
      store_frag_bf16(pt, pa[1], Frag{tl0, 1, c4});
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_FULL_PP + (j & 1)]);
      if (j > 0) write_out(j - 1);
    }
    if (want_out && nc > 0 && !mw[MW_ABORT]) write_out(nc - 1);
  }

  // ---------------- teardown ----------------
  if (!ok) record_error(p.hdr, MOGT_ERR_TIMEOUT, unit);
  if (warp == W_TMA && lane == 0 && mw[MW_ABORT]) {
    // let copies still in flight land before the CTA exits (bounded waits)
    for (int it = max(0, nit - NS); it < nit; ++it) mbar_wait(&bars[B_FULL_IN + it % NS], cons_parity(it / NS));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == W_TMA) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
  if (tid == 0) finish_cta(p.hdr, epoch, gridDim.x);
}

template __global__ void gated_fwd_ws<true>(const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap,
                                            const __grid_constant__ CUtensorMap, const Params);
template __global__ void gated_fwd_ws<false>(const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap,
                                             const __grid_constant__ CUtensorMap, const Params);

}  // namespace ws
}  // namespace gated
}  // namespace mogt

namespace mogt {
namespace gated {

int launch_fwd_ws(const CUtensorMap* maps, const void* params, bool out_f32, unsigned grid,
                  cudaStream_t s) {
  constexpr int kMaxDev = 64;
  static bool prepared[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return MOGT_ERR_LAUNCH;
  if (dev >= kMaxDev || !prepared[dev]) {
    if (cudaFuncSetAttribute(ws::gated_fwd_ws<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ws::SM_ALLOC) != cudaSuccess ||
        cudaFuncSetAttribute(ws::gated_fwd_ws<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ws::SM_ALLOC) != cudaSuccess)
      return MOGT_ERR_LAUNCH;
    if (dev < kMaxDev) prepared[dev] = true;
  }
  const ws::Params& P = *static_cast<const ws::Params*>(params);
  if (out_f32)
    ws::gated_fwd_ws<true><<<grid, ws::NTH, ws::SM_ALLOC, s>>>(maps[0], maps[1], maps[2], P);
  else
    ws::gated_fwd_ws<false><<<grid, ws::NTH, ws::SM_ALLOC, s>>>(maps[0], maps[1], maps[2], P);
  return mogt_host::launch_status();
}

}  // namespace gated
}  // namespace mogt
