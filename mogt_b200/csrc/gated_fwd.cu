// Headed gated scan, forward (bf16 q/k/v, dk = dv = 64, fp32 state):
//     S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,     o_t = S_t^T q_t.
// Reference semantics: affine_scan.py:14-62 run on U_t = f_t I,
// V_t = (1 - f_t) k_t v_t^T, followed by the readout einsum.
//
// Work decomposition ("stripes"): the T tokens of every (batch, head) are cut
// into 64-token chunks and the chunks into a few contiguous stripes, so that
// BH x stripes ~ one wave of resident CTAs.  A CTA owns one stripe:
//   pass 1  streams K, V chunks (TMA, 5-stage ring, L2 evict-last) and builds
//           the stripe's aggregate state  sum_s decay(s->end) (1-f_s) k_s v_s^T
//           with tensor-core GEMMs (K~^T V per chunk), then publishes it;
//   look-back  a windowed decoupled look-back over the earlier stripes of the
//           same head yields the fp32 state entering the stripe; the stripe's
//           inclusive state is published for its successors;
//   pass 2  streams Q, K, V chunks again (3-stage ring, K, V mostly from L2)
//           and per chunk computes o = diag(a) Q S + ((Q K^T) o D) V and the
//           state update S <- a_C S + K~^T V (mma.sync bf16 -> fp32).
// Decays come from chunk-local inclusive log2 cumulative gates: D[t,s] =
// exp2(l_t - l_s) for s <= t, a_t = exp2(l_t), and per-step log2 gates are
// clamped at -64 so f = 0 is a (numerically) full reset.
#include "common.cuh"
#include "gated_internal.h"
#include "lookback.cuh"

#ifdef MOGT_TRACE
// Debug-only phase timestamps (built into a separate trace library, never
// into the product): trace[unit * 8 + k] = %globaltimer at phase k.
__device__ unsigned long long* g_mogt_trace = nullptr;
__device__ __forceinline__ void trace_mark(uint32_t unit, int k) {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  if (g_mogt_trace) g_mogt_trace[unit * 8 + k] = t;
}
#define MOGT_MARK(u, k) \
  if (threadIdx.x == 0) trace_mark(u, k)
#else
#define MOGT_MARK(u, k)
#endif

namespace mogt {
namespace gated {

constexpr int D = 64;
constexpr int CH = 64;
constexpr int NTHREADS = 128;
constexpr int STAGES = 3;                 // pass-2 ring: q, k, v per slot
constexpr int P1_STAGES = 5;              // pass-1 ring: k, v per slot
constexpr int SEG_CHUNKS = 4;             // saved-state granularity: 256 tokens
constexpr int TILE = CH * D * 2;          // one 64x64 bf16 tile, 8 KB
constexpr int SLOT = 3 * TILE;            // q, k, v of one chunk

struct GateBuf {
  float lg[CH];  // chunk-local inclusive log2 cumulative gate
  float ck[CH];  // (1 - f_s) * decay(s -> chunk end)
  float ea[CH];  // decay(chunk start -> t)
  float wv[CH];  // 1 - f_s
  float lgC;     // log2 decay of the whole chunk
  float pad[3];
};

constexpr int SM_RING = 0;
constexpr int SM_SBUF = SM_RING + STAGES * SLOT;   // 2 x bf16 state operand
constexpr int SM_GATE = SM_SBUF + 2 * TILE;        // 2 x GateBuf
constexpr int SM_MISC = SM_GATE + 2 * (int)sizeof(GateBuf);
constexpr int SM_BAR = SM_MISC + 256;      // STAGES pass-2 + P1_STAGES pass-1 mbarriers
constexpr int SM_TOTAL = SM_BAR + 8 * (STAGES + P1_STAGES);
// pass 1 reuses the ring and the state-operand buffers as a deeper k/v ring
static_assert(P1_STAGES * 2 * TILE <= SM_GATE - SM_RING, "pass-1 ring fits");
constexpr int SM_ALLOC = SM_TOTAL + 1024;

struct Params {
  const float* f;
  void* o;
  const float* S0;
  float* S_final;
  float* decay_final;
  float* seg_states;
  WsHeader* hdr;
  uint32_t* flags;
  float* a_agg;
  float* a_inc;
  float* st_agg;
  float* st_inc;
  int T, BH, nchunks, cps, nstripes, nseg;
};

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

struct Plan {
  int nchunks, cps, nstripes;
};
inline Plan make_plan(int64_t BH, int64_t T, int resident) {
  Plan p;
  p.nchunks = (int)((T + CH - 1) / CH);
  int64_t sph = BH >= resident ? 1 : resident / BH;
  if (sph > p.nchunks) sph = p.nchunks;
  if (sph < 1) sph = 1;
  p.cps = (int)((p.nchunks + sph - 1) / sph);
  p.nstripes = (p.nchunks + p.cps - 1) / p.cps;
  return p;
}

inline int resident_ctas() {
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  return 2 * nsm;
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int32_t c0, int32_t c1, int32_t c2, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(pol)
      : "memory");
}

// Gates of chunk gc for one warp: lane l holds steps 2l, 2l+1 (t >= T reads
// as "no step": f = 1, so log2 f = 0 and 1 - f = 0).  Issued one chunk ahead
// of gate_prep so the global-load latency is off the critical path.
__device__ __forceinline__ float2 gate_load(const float* fh, int T, int gc, int lane) {
  const int t = gc * CH + 2 * lane;
  float2 r;
  r.x = t < T ? __ldg(fh + t) : 1.f;
  r.y = t + 1 < T ? __ldg(fh + t + 1) : 1.f;
  return r;
}

// One warp: gate arrays of one chunk from its gates (see gate_load).
__device__ __forceinline__ void gate_prep(GateBuf* gb, float2 fv, int lane) {
  const int tl = 2 * lane;
  const float x0 = fmaxf(fast_log2(fv.x), -64.f), x1 = fmaxf(fast_log2(fv.y), -64.f);
  const float w0 = 1.f - fv.x, w1 = 1.f - fv.y;
  const float pair = x0 + x1;
  float inc = pair;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  const float l0 = inc - pair + x0, l1 = inc;
  const float tot = __shfl_sync(0xffffffffu, inc, 31);
  gb->lg[tl] = l0;
  gb->lg[tl + 1] = l1;
  gb->wv[tl] = w0;
  gb->wv[tl + 1] = w1;
  gb->ck[tl] = fast_exp2(tot - l0) * w0;
  gb->ck[tl + 1] = fast_exp2(tot - l1) * w1;
  gb->ea[tl] = fast_exp2(l0);
  gb->ea[tl + 1] = fast_exp2(l1);
  if (lane == 0) gb->lgC = tot;
}

// acc (this warp's 16 state rows x 64 cols) += K~^T V for one chunk tile pair.
__device__ __forceinline__ void add_ktv(float (&acc)[8][4], uint32_t kbase, uint32_t vbase,
                                        const float* ck, int warp, int lane) {
  const int mi = lane >> 3, r = lane & 7, c4 = lane & 3;
  const int i0 = warp * 16;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int s0 = kk * 16;
    uint32_t a[4];
    ldsm_x4_t(a, kbase + sw128(s0 + (mi >> 1) * 8 + r, (i0 >> 3) + (mi & 1)));
    const int sa = s0 + 2 * c4, sb = sa + 8;
    const float ca0 = ck[sa], ca1 = ck[sa + 1], cb0 = ck[sb], cb1 = ck[sb + 1];
    a[0] = scale_bf16x2(a[0], ca0, ca1);
    a[1] = scale_bf16x2(a[1], ca0, ca1);
    a[2] = scale_bf16x2(a[2], cb0, cb1);
    a[3] = scale_bf16x2(a[3], cb0, cb1);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, vbase + sw128(s0 + (mi & 1) * 8 + r, np * 2 + (mi >> 1)));
      mma_bf16(acc[2 * np], a, b[0], b[1]);
      mma_bf16(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// Write this thread's fragment of a 64x64 fp32 state as bf16 into a swizzled tile.
__device__ __forceinline__ void store_state_bf16(uint8_t* tile, const float (&s)[8][4], int i_lo,
                                                 int c4) {
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const uint32_t col = 4u * c4;
    *reinterpret_cast<uint32_t*>(tile + sw128(i_lo, n) + col) = pack_bf16(s[n][0], s[n][1]);
    *reinterpret_cast<uint32_t*>(tile + sw128(i_lo + 8, n) + col) = pack_bf16(s[n][2], s[n][3]);
  }
}

// Write this thread's fragment of a 64x64 fp32 state row-major to global memory.
__device__ __forceinline__ void store_state_rowmajor(float* dst, const float (&s)[8][4], int i_lo,
                                                     int c4) {
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int j = n * 8 + 2 * c4;
    *reinterpret_cast<float2*>(dst + i_lo * D + j) = make_float2(s[n][0], s[n][1]);
    *reinterpret_cast<float2*>(dst + (i_lo + 8) * D + j) = make_float2(s[n][2], s[n][3]);
  }
}

template <bool OUT_F32>
__global__ void __launch_bounds__(NTHREADS, 2)
    gated_fwd_stripe(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c4 = lane & 3, mi = lane >> 3, r8 = lane & 7;
  const int i_lo = warp * 16 + g;
  GateBuf* gbuf = reinterpret_cast<GateBuf*>(smem + SM_GATE);
  volatile uint32_t* bc = reinterpret_cast<volatile uint32_t*>(smem + SM_MISC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);

  if (tid == 0) {
    uint32_t epoch;
    bc[0] = take_ticket(p.hdr, &epoch);
    bc[1] = epoch;
#pragma unroll
    for (int s = 0; s < STAGES + P1_STAGES; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const uint32_t unit = bc[0], epoch = bc[1];
  const int BH = p.BH, T = p.T;
  const int stripe = (int)unit / BH, bh = (int)unit % BH;
  const int c_begin = stripe * p.cps;
  const int nc = min(p.cps, p.nchunks - c_begin);
  const bool has_succ = stripe + 1 < p.nstripes;
  const bool want_out = p.o != nullptr;
  const bool need_p2 = want_out || p.seg_states != nullptr;
  const bool need_p1 = has_succ || !need_p2;
  const int n1 = need_p1 ? nc : 0;
  const int nit = n1 + (need_p2 ? nc : 0);
  const float* fh = p.f + (size_t)bh * T;
  MOGT_MARK(unit, 0);

  uint64_t pol_keep = 0, pol_stream = 0;
  if (tid == 0) {
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_keep));
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_stream));
  }
  uint64_t* bars1 = bars + STAGES;
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
  // pass-1 loads may run P1_STAGES - 1 ahead; pass-2 loads STAGES - 1 ahead
  // and only once pass 1 has released the shared ring
  auto issue_upto = [&](int it_done) {
    // called at the top of iteration it_done (after the CTA barrier)
    if (it_done < n1) {
      const int nxt = it_done + P1_STAGES - 1;
      if (nxt < n1) issue(nxt);
    } else {
      const int nxt = it_done + STAGES - 1;
      if (nxt >= n1 + STAGES - 1) issue(nxt);
    }
  };
  auto chunk_of = [&](int it) { return c_begin + (it < n1 ? it : it - n1); };

  if (tid == 0) {
    if (n1 > 0)
      for (int it = 0; it < P1_STAGES - 1 && it < n1; ++it) issue(it);
    else
      for (int it = 0; it < STAGES - 1; ++it) issue(it);
  }
  // warp 0 prepares the gate arrays one chunk ahead; fpre holds the gates of
  // the next iteration, loaded one iteration before they are needed
  float2 fpre = make_float2(1.f, 1.f);
  if (warp == 0 && nit > 0) {
    gate_prep(&gbuf[0], gate_load(fh, T, chunk_of(0), lane), lane);
    if (nit > 1) fpre = gate_load(fh, T, chunk_of(1), lane);
  }
  auto gates_next = [&](int it) {
    if (warp == 0 && it + 1 < nit) {
      gate_prep(&gbuf[(it + 1) & 1], fpre, lane);
      if (it + 2 < nit) fpre = gate_load(fh, T, chunk_of(it + 2), lane);
    }
  };

  // ---------------- pass 1: stripe aggregate ----------------
  float agg[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) agg[n][e] = 0.f;
  float ltot = 0.f;
  for (int it = 0; it < n1; ++it) {
    __syncthreads();
    if (tid == 0) issue_upto(it);
    gates_next(it);
    if (!mbar_wait(&bars1[it % P1_STAGES], (it / P1_STAGES) & 1)) record_error(p.hdr, MOGT_ERR_TIMEOUT, unit);
    const GateBuf* gb = &gbuf[it & 1];
    const uint8_t* base = smem + SM_RING + (it % P1_STAGES) * 2 * TILE - TILE;
    const float lgC = gb->lgC;
    const float dC = fast_exp2(lgC);
    ltot += lgC;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) agg[n][e] *= dC;
    add_ktv(agg, smem_u32(base + TILE), smem_u32(base + 2 * TILE), gb->ck, warp, lane);
  }
  MOGT_MARK(unit, 1);
  if (n1 > 0) {
    // pass 1 has released the shared ring: prefetch the first pass-2 chunks so
    // they load during the look-back
    __syncthreads();
    if (tid == 0)
      for (int it = n1; it < n1 + STAGES - 1; ++it) issue(it);
  }
  const float A_agg = fast_exp2(ltot);
  const size_t st_off = (size_t)unit * (D * D) + (size_t)tid * 32;

  if (n1 > 0 && stripe > 0 && has_succ) {
    float4* dst = reinterpret_cast<float4*>(p.st_agg + st_off);
#pragma unroll
    for (int n = 0; n < 8; ++n) __stcg(dst + n, make_float4(agg[n][0], agg[n][1], agg[n][2], agg[n][3]));
    if (tid == 0) __stcg(p.a_agg + unit, A_agg);
    __threadfence();
    __syncthreads();
    if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagAgg));
  }

  // ---------------- state entering the stripe ----------------
  float sin[8][4];
  float a_in = 1.f;
  if (stripe == 0) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int j = n * 8 + 2 * c4;
      if (p.S0) {
        const float* s0p = p.S0 + (size_t)bh * D * D;
        const float2 lo = __ldg(reinterpret_cast<const float2*>(s0p + i_lo * D + j));
        const float2 hi = __ldg(reinterpret_cast<const float2*>(s0p + (i_lo + 8) * D + j));
        sin[n][0] = lo.x; sin[n][1] = lo.y; sin[n][2] = hi.x; sin[n][3] = hi.y;
      } else {
        sin[n][0] = sin[n][1] = sin[n][2] = sin[n][3] = 0.f;
      }
    }
  } else {
    LookbackBufs lb{p.flags, p.a_agg, p.a_inc, p.st_agg, p.st_inc, p.hdr};
    lookback_scalar_state(sin, a_in, lb, stripe, (uint32_t)bh, (uint32_t)BH, epoch, unit,
                          reinterpret_cast<float*>(smem + SM_MISC + 64),
                          reinterpret_cast<volatile uint32_t*>(smem + SM_MISC + 16));
  }
  MOGT_MARK(unit, 2);

  if (n1 > 0) {
    float inc_st[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) inc_st[n][e] = A_agg * sin[n][e] + agg[n][e];
    if (has_succ) {
      float4* dst = reinterpret_cast<float4*>(p.st_inc + st_off);
#pragma unroll
      for (int n = 0; n < 8; ++n)
        __stcg(dst + n, make_float4(inc_st[n][0], inc_st[n][1], inc_st[n][2], inc_st[n][3]));
      if (tid == 0) __stcg(p.a_inc + unit, A_agg * a_in);
      __threadfence();
      __syncthreads();
      if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagInc));
    } else {
      if (p.S_final) store_state_rowmajor(p.S_final + (size_t)bh * D * D, inc_st, i_lo, c4);
      if (tid == 0 && p.decay_final) p.decay_final[bh] = A_agg * a_in;
    }
  }
  MOGT_MARK(unit, 3);

  // ---------------- pass 2: outputs ----------------
  if (need_p2) {
    store_state_bf16(smem + SM_SBUF + (n1 & 1) * TILE, sin, i_lo, c4);
    const bool final_here = !has_succ && n1 == 0;
    float ltot2 = 0.f;
    for (int it = n1; it < nit; ++it) {
      const int c = it - n1, gc = c_begin + c;
      __syncthreads();
      if (tid == 0) issue_upto(it);
      gates_next(it);
      if (p.seg_states && (gc % SEG_CHUNKS) == 0)
        store_state_rowmajor(p.seg_states + ((size_t)bh * p.nseg + gc / SEG_CHUNKS) * D * D, sin,
                             i_lo, c4);
      if (!mbar_wait(&bars[c % STAGES], (c / STAGES) & 1)) record_error(p.hdr, MOGT_ERR_TIMEOUT, unit);
      const GateBuf* gb = &gbuf[it & 1];
      uint8_t* base = smem + SM_RING + (c % STAGES) * SLOT;
      const uint32_t qb = smem_u32(base), kb = smem_u32(base + TILE), vb = smem_u32(base + 2 * TILE);
      const uint32_t sb = smem_u32(smem + SM_SBUF + (it & 1) * TILE);
      if (want_out) {
        const int rq = warp * 16;
        uint32_t qa[4][4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) ldsm_x4(qa[kk], qb + sw128(rq + (lane & 15), kk * 2 + (lane >> 4)));
        float oacc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) oacc[n][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t b[4];
            ldsm_x4_t(b, sb + sw128(kk * 16 + (mi & 1) * 8 + r8, np * 2 + (mi >> 1)));
            mma_bf16(oacc[2 * np], qa[kk], b[0], b[1]);
            mma_bf16(oacc[2 * np + 1], qa[kk], b[2], b[3]);
          }
        {
          const float e0 = gb->ea[rq + g], e1 = gb->ea[rq + g + 8];
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            oacc[n][0] *= e0; oacc[n][1] *= e0;
            oacc[n][2] *= e1; oacc[n][3] *= e1;
          }
        }
        float pacc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) pacc[n][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            if (np <= warp) {
              uint32_t b[4];
              ldsm_x4(b, kb + sw128(np * 16 + (mi >> 1) * 8 + r8, kk * 2 + (mi & 1)));
              mma_bf16(pacc[2 * np], qa[kk], b[0], b[1]);
              mma_bf16(pacc[2 * np + 1], qa[kk], b[2], b[3]);
            }
          }
        {
          const int tl0 = rq + g, tl1 = tl0 + 8;
          const float lt0 = gb->lg[tl0], lt1 = gb->lg[tl1];
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            if ((n >> 1) <= warp) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int s = n * 8 + 2 * c4 + e;
                const float ls = gb->lg[s], ws = gb->wv[s];
                pacc[n][e] = (s <= tl0) ? pacc[n][e] * fast_exp2(lt0 - ls) * ws : 0.f;
                pacc[n][2 + e] = (s <= tl1) ? pacc[n][2 + e] * fast_exp2(lt1 - ls) * ws : 0.f;
              }
            }
          }
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          if (kk <= warp) {
            uint32_t a[4];
            a[0] = pack_bf16(pacc[2 * kk][0], pacc[2 * kk][1]);
            a[1] = pack_bf16(pacc[2 * kk][2], pacc[2 * kk][3]);
            a[2] = pack_bf16(pacc[2 * kk + 1][0], pacc[2 * kk + 1][1]);
            a[3] = pack_bf16(pacc[2 * kk + 1][2], pacc[2 * kk + 1][3]);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
              uint32_t b[4];
              ldsm_x4_t(b, vb + sw128(kk * 16 + (mi & 1) * 8 + r8, np * 2 + (mi >> 1)));
              mma_bf16(oacc[2 * np], a, b[0], b[1]);
              mma_bf16(oacc[2 * np + 1], a, b[2], b[3]);
            }
          }
        }
        const int ta = gc * CH + rq + g, tb = ta + 8;
        const size_t rowa = ((size_t)bh * T + ta) * D, rowb = ((size_t)bh * T + tb) * D;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int j = n * 8 + 2 * c4;
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
      }
      // running state for the next chunk (or the final state)
      const float lgC = gb->lgC;
      ltot2 += lgC;
      if (c + 1 < nc || (final_here && p.S_final)) {
        const float dC = fast_exp2(lgC);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) sin[n][e] *= dC;
        add_ktv(sin, kb, vb, gb->ck, warp, lane);
        if (c + 1 < nc) store_state_bf16(smem + SM_SBUF + ((it + 1) & 1) * TILE, sin, i_lo, c4);
      }
    }
    if (final_here) {
      if (p.S_final) store_state_rowmajor(p.S_final + (size_t)bh * D * D, sin, i_lo, c4);
      if (tid == 0 && p.decay_final) p.decay_final[bh] = a_in * fast_exp2(ltot2);
    }
  }
  MOGT_MARK(unit, 4);
  __syncthreads();
  if (tid == 0) finish_cta(p.hdr, epoch, gridDim.x);
}

}  // namespace gated
}  // namespace mogt

using namespace mogt;
using namespace mogt::gated;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" {

#ifdef MOGT_TRACE
int mogt_debug_set_trace(void* buf) {
  unsigned long long* p = static_cast<unsigned long long*>(buf);
  return cudaMemcpyToSymbol(g_mogt_trace, &p, sizeof(p)) == cudaSuccess ? 0 : 4;
}
#endif

int64_t mogt_gated_scan_num_segments(int64_t T, int64_t dk, int64_t dv, int in_dtype) {
  if (in_dtype != MOGT_DTYPE_BF16 || dk != D || dv != D || T <= 0) return 0;
  return (T + SEG_CHUNKS * CH - 1) / (SEG_CHUNKS * CH);
}

size_t mogt_gated_scan_fwd_workspace_bytes(int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                           int in_dtype) {
  if (in_dtype != MOGT_DTYPE_BF16 || dk != D || dv != D || T <= 0 || BH <= 0)
    return sizeof(WsHeader);
  const Plan pl = make_plan(BH, T, resident_ctas());
  return ws_layout((size_t)BH * pl.nstripes).total;
}

int mogt_gated_scan_fwd(const void* q, const void* k, const void* v, const float* f, void* o,
                        const float* S0, float* S_final, float* decay_final, float* seg_states,
                        int64_t BH, int64_t T, int64_t dk, int64_t dv, int in_dtype, int out_dtype,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (BH <= 0 || T < 0 || dk <= 0 || dv <= 0) return MOGT_ERR_SHAPE;
  if (T == 0) return MOGT_OK;
  if (!k || !v || !f || (o && !q)) return MOGT_ERR_ARG;
  if (BH >= ((int64_t)1 << 31) || T >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (in_dtype == MOGT_DTYPE_F32) {
    if (out_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
    if (seg_states) return MOGT_ERR_UNSUPPORTED;
    return launch_fwd_seq(static_cast<const float*>(q), static_cast<const float*>(k),
                          static_cast<const float*>(v), f, static_cast<float*>(o), S0, S_final,
                          decay_final, (int)BH, (int)T, (int)dk, (int)dv, s);
  }
  if (in_dtype != MOGT_DTYPE_BF16) return MOGT_ERR_DTYPE;
  if (dk != D || dv != D) return MOGT_ERR_UNSUPPORTED;
  if (out_dtype != MOGT_DTYPE_BF16 && out_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  if (!aligned16(k) || !aligned16(v) || (q && !aligned16(q)) || (o && !aligned16(o)))
    return MOGT_ERR_ALIGN;
  const Plan pl = make_plan(BH, T, resident_ctas());
  const size_t NU = (size_t)BH * pl.nstripes;
  if (NU >= ((size_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  const WsLayout L = ws_layout(NU);
  if (!workspace || workspace_bytes < L.total) return MOGT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOGT_ERR_ALIGN;

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
  P.seg_states = seg_states;
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
  P.nseg = (int)mogt_gated_scan_num_segments(T, dk, dv, in_dtype);
  if (out_dtype == MOGT_DTYPE_F32) {
    cudaFuncSetAttribute(gated_fwd_stripe<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_ALLOC);
    gated_fwd_stripe<true><<<(unsigned)NU, NTHREADS, SM_ALLOC, s>>>(maps[0], maps[1], maps[2], P);
  } else {
    cudaFuncSetAttribute(gated_fwd_stripe<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_ALLOC);
    gated_fwd_stripe<false><<<(unsigned)NU, NTHREADS, SM_ALLOC, s>>>(maps[0], maps[1], maps[2], P);
  }
  return mogt_host::launch_status();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.  Its scratch is a fixed array in the library's
// device image instead of a caller-provided workspace, for callers that
// cannot allocate device memory.  The kernel and its arguments are exactly
// those of mogt_gated_scan_fwd.
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
                                           float* S_final, float* decay_final, float* seg_states,
                                           int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                           int in_dtype, int out_dtype, void* stream) {
  if (BH <= 0 || T < 0 || dk <= 0 || dv <= 0) return MOGT_ERR_SHAPE;
  if (T == 0) return MOGT_OK;
  size_t clear_bytes = 0;
  if (in_dtype == MOGT_DTYPE_BF16 && dk == D && dv == D) {
    if (BH >= ((int64_t)1 << 31) || T >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
    const Plan pl = make_plan(BH, T, resident_ctas());
    const WsLayout L = ws_layout((size_t)BH * pl.nstripes);
    if (L.total > kStaticScratchBytes) return MOGT_ERR_TOO_LARGE;
    clear_bytes = L.st_agg;  // header, flags and decays must start at zero
  }
  void* scratch = static_scratch_for_current_device();
  if (!scratch) return MOGT_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (clear_bytes && cudaMemsetAsync(scratch, 0, clear_bytes, s) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  return mogt_gated_scan_fwd(q, k, v, f, o, S0, S_final, decay_final, seg_states, BH, T, dk, dv,
                             in_dtype, out_dtype, scratch, kStaticScratchBytes, stream);
}
