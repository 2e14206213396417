// Headed gated scan, forward: warp-specialised stripe kernel (bf16 q/k/v,
// dk = dv = 64, fp32 state).
//     S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,     o_t = S_t^T q_t.
// Reference semantics: affine_scan.py:14-62 run on U_t = f_t I,
// V_t = (1 - f_t) k_t v_t^T, followed by the readout einsum.
//
// Work decomposition: the 64-token chunks of every (batch, head) are cut
// into contiguous stripes, BH x stripes ~ one CTA per SM.  A CTA owns one
// stripe: pass 1 accumulates the stripe's aggregate state in tensor memory,
// a decoupled look-back over the earlier stripes of the head gives the state
// entering the stripe, and pass 2 forms the outputs chunk by chunk.  The
// arithmetic per chunk is the chunked form used throughout this library:
// chunk-local inclusive log2 cumulative gates l_t, Q^ = diag(exp2 l) Q,
// K~ = diag(w exp2(-l)) K (factorised, chunk decay above 2^-100) or
// diag(w exp2(L - l)) K (exact), P' = causally masked Q^ K~^T (or the exact
// per-element decays of Q K^T), o = Q^ S + P' V, S <- a (S + K~^T V) or
// a S + K~^T V.
//
// The CTA's 14 warps each play one role, connected by mbarrier rings, so
// the only serial dependency from chunk to chunk is the state update:
//   warp 0      TMA producer: q, k, v chunk tiles into a 3-slot ring;
//   warp 1      MMA issuer (one thread): per chunk P and K~^T V (state
//               independent, issued one chunk ahead), then O = Q^ S and
//               O += P' V once the state and the masked P' are ready;
//   warps 2-5   builders: gate arithmetic and the scaled operand tiles
//               Q^, K~ (2-slot ring);
//   warps 6-9   state: the fp32 state in registers, S <- a (S + dS) per
//               chunk, its bf16 copy for the O product, the stripe's
//               aggregate, the look-back and the published carries;
//   warps 10-13 mask and output: P from tensor memory, causal mask / exact
//               decays, bf16 P' tile (2-slot ring); then the previous
//               chunk's O from tensor memory to global memory.
// Tensor memory (512 columns): P[2], dS[2], O[2], 64 columns each (M = 64
// accumulators; warp w reads lanes 32 (w % 4) .. +15, i.e. rows
// 16 (w % 4) .. +15, of every accumulator).
#pragma once

#include "common.cuh"
#include "gated_common.cuh"
#include "lookback.cuh"

namespace mogt {
namespace gated {
namespace ws {

constexpr int NWARPS = 14;
constexpr int NTH = NWARPS * 32;
constexpr int W_TMA = 0, W_MMA = 1, W_BLD = 2, W_ST = 6, W_MO = 10;
constexpr int NS = 3;                          // input ring (q, k, v of a chunk)
constexpr int NB = 2;                          // build ring (Q^, K~)
constexpr int BAR_BLD = 1, BAR_ST = 2;         // named barriers (builders, state warps)

constexpr int SM_IN = 0;                                  // [NS][q | k | v]
constexpr int SM_BLD = SM_IN + NS * 3 * TILE;             // [NB][Q^ | K~]
constexpr int SM_S = SM_BLD + NB * 2 * TILE;              // [2] bf16 state tiles [i][j]
constexpr int SM_PP = SM_S + 2 * TILE;                    // [2] bf16 P' tiles [t][s]
constexpr int SM_LSUF = SM_PP + 2 * TILE;                 // pass-1 suffix log2 decays
constexpr int SM_MISC = SM_LSUF + MAX_CPS * 4;            // ctl words, look-back scratch
constexpr int SM_BAR = SM_MISC + 512;
// mbarriers
enum {
  B_FULL_IN = 0, B_EMPTY_IN = B_FULL_IN + NS, B_FULL_B = B_EMPTY_IN + NS, B_EMPTY_B = B_FULL_B + NB,
  B_FULL_P = B_EMPTY_B + NB, B_EMPTY_P = B_FULL_P + 2, B_FULL_PP = B_EMPTY_P + 2,
  B_EMPTY_PP = B_FULL_PP + 2, B_FULL_DS = B_EMPTY_PP + 2, B_EMPTY_DS = B_FULL_DS + 2,
  B_FULL_S = B_EMPTY_DS + 2, B_EMPTY_S = B_FULL_S + 2, B_FULL_O = B_EMPTY_S + 2,
  B_EMPTY_O = B_FULL_O + 2, NBARS = B_EMPTY_O + 2
};
constexpr int SM_TSLOT = SM_BAR + 8 * NBARS;
constexpr int SM_TOTAL = SM_TSLOT + 16;
constexpr int SM_ALLOC = SM_TOTAL + 1024;
static_assert(SM_ALLOC <= 227 * 1024, "shared memory");
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TM_P = 0, TM_DS = 128, TM_O = 256;

// misc words (SM_MISC): [0] ticket, [1] epoch, [2] abort flag, [4..5] fast
// flag per build slot, [8..11] state-warp partial sums, [16..19] look-back
// control, [32..63] look-back scale factors
constexpr int MW_TICKET = 0, MW_EPOCH = 1, MW_ABORT = 2, MW_FAST = 4, MW_PART = 8, MW_LBCTL = 16,
              MW_LBSCL = 32;

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

// Producer side of a ring slot: wait until the consumer released use k-1
// of the slot (the first use passes at once).
__device__ __forceinline__ uint32_t prod_parity(int use) { return ((use & 1) ^ 1); }
__device__ __forceinline__ uint32_t cons_parity(int use) { return use & 1; }

// 16 bytes x 4 pieces of a 64x64 bf16 tile per builder thread (128 threads):
// piece q = bt + 128 j -> row q / 8 = bt / 8 + 16 j, 16-byte chunk q % 8;
// dst rows = scale[j] * src rows (one bf16 rounding, as fp32 multiply + cast).
__device__ __forceinline__ void build4(uint8_t* dst, const uint8_t* src, const float (&sc)[4], int bt) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = bt + 128 * j, row = q >> 3, chunk = q & 7;
    const uint32_t off = sw128(row, chunk);
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    const float c = sc[j];
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

// Warp-wide read of rows 16 (warp % 4) .. +15, all 64 columns, of an M = 64
// accumulator: two 16x32 halves (hf = 0, 1) in the m16n8 fragment layout.
__device__ __forceinline__ void tmem_ld_rows64(float (&a)[2][4][4], uint32_t taddr) {
  uint32_t r0[16], r1[16];
  tmem_ld_16x32_async(r0, taddr);
  tmem_ld_16x32_async(r1, taddr + 32);
  tmem_wait_ld();
  frag_from_u32(a[0], r0);
  frag_from_u32(a[1], r1);
}

}  // namespace ws
}  // namespace gated
}  // namespace mogt
