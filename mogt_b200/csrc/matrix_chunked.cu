// Chunked dense-transition headed scan (long sequences):
//     S_t = A_t S_{t-1} + (1 - f_t) k_t v_t^T,      o_t = S_t^T q_t,
// A_t: [BH, T, 64, 64] fp32, q, k, v: [BH, T, 64].  Same semantics as the
// sequential kernel in matrix_scan.cu (affine_scan.py:14-62 with U_t = A_t,
// V_t = (1-f_t) k_t v_t^T, then the readout einsum), reorganised so that the
// whole sequence is not one dependency chain per head.
//
// Split T into chunks of 64 steps.  Inside chunk c (steps t0..t0+L-1), with
// S_in the state entering it,
//     S_t = P_t S_in + S^loc_t,   P_t = A_t ... A_{t0},
//     S^loc_t = A_t S^loc_{t-1} + w_t k_t v_t^T  (S^loc_{t0-1} = 0),
// so  o_t = S^loc_t^T q_t + S_in^T (P_t^T q_t).
//
// Kernel 1 (one CTA per head and chunk, all chunks in parallel) evolves the
// 64 x 128 matrix X = [P | S^loc] through the chunk (X <- A_t X, plus the
// rank-1 write in the S^loc half) and emits, per step, both readouts
// u_t = P_t^T q_t and o^loc_t = S^loc_t^T q_t, and at the end P and S^loc.
// This is 2x the multiply-adds of the plain recurrence, all of it in
// independent CTAs.  With norm-preserving A_t nothing is forgotten, so
// round-off accumulates over the whole sequence and the state is kept at
// fp32 accuracy: bf16 q/k/v use chunk_local_tc (tensor cores, three tf32
// products per step, described at that kernel); fp32 q/k/v use
// chunk_local_kernel (fp32 FMAs).  chunk_local_kernel's register tile: thread (warp w, half h, lane group g) owns rows
// 4(2w+h)..+3 and columns 4g..+3 of both halves: per 4 contraction indices
// it reads 4 float4 of A_t (two distinct rows per warp) and 8 float4 of X
// (256 contiguous bytes per half-warp) for 128 FMAs, issued as 64 packed
// fma.rn.f32x2 on (even k, odd k) pairs -- the kernel is issue bound, and the
// packed form does the same FMA work in half the instructions.
// Kernel 2 (one CTA per head and 8 state columns) composes the chunk carries
// sequentially, S_in[c+1] = P_c S_in[c] + S^loc_c: 64^2 x 8 FMAs per chunk.
// Kernel 3 (one CTA per head and chunk) forms o = o^loc + U S_in, U the
// chunk's 64 x 64 matrix of u_t rows, and writes o in the output dtype.
#include "common.cuh"

namespace mogt {
namespace mchunk {

constexpr int D = 64;       // state rows (k index) and columns (v index)
constexpr int C = 64;       // steps per chunk
constexpr int NT = 256;     // threads of kernels 1 and 3
constexpr int XP = 2 * D;   // row pitch of X = [P | S^loc] in floats
constexpr int CC = 8;       // state columns per carry CTA

template <typename TI>
struct Slot {  // one step's inputs in shared memory: A_t, k_t, q_t, v_t
  static constexpr int kBytesA = D * D * 4;
  static constexpr int kRow = D * (int)sizeof(TI);
  static constexpr int kBytes = kBytesA + 3 * kRow;
  static_assert(kRow % 16 == 0 && kBytes % 16 == 0, "bulk copies need 16-byte sizes");
};

template <typename TI>
constexpr size_t local_smem_bytes() {
  return 2 * (size_t)Slot<TI>::kBytes + 2 * (size_t)D * XP * 4 + 2 * 8 * (size_t)XP * 4 + C * 4 + 16;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 r = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
__device__ __forceinline__ float comp(const float4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}
// d = a * b + c on fp32 pairs (one packed FMA instruction for two lanes of work)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)),
        "l"(*reinterpret_cast<const uint64_t*>(&c)));
  return *reinterpret_cast<const float2*>(&d);
}
__device__ __forceinline__ float2 lo2(const float4& v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(const float4& v) { return make_float2(v.z, v.w); }

// Shared-memory layout of X = [P | S^loc] (64 x 128), interleaved by pairs of
// rows (the contraction index k) so that one float4 holds
// (X[2kp][c], X[2kp+1][c], X[2kp][c+1], X[2kp+1][c+1]): the operand pair of
// two packed FMAs that accumulate even and odd k separately.  Row pair kp
// holds 256 floats in four 64-float blocks (P columns 4g, 4g+1 | P 4g+2, 4g+3
// | the same two for S^loc), lane group g's float4 at 4g inside each block,
// so a half-warp's loads of one block are 256 contiguous bytes.
__device__ __forceinline__ int xidx(int k, int c) {
  const int cc = c & 63, g = cc >> 2, w = cc & 3;
  const int blk = (c >> 6) * 2 + (w >> 1);
  return (k >> 1) * 256 + blk * 64 + g * 4 + (w & 1) * 2 + (k & 1);
}

// ---------------------------------------------------------------------------
// Kernel 1: per-chunk prefix products and local states with both readouts.
// o_loc, u: [NB, C, D]; P_out, S_loc: [NB, D, D]; NB = BH * nch.
// ---------------------------------------------------------------------------
template <typename TI>
__global__ void __launch_bounds__(NT, 2)
    chunk_local_kernel(const float* __restrict__ A, const TI* __restrict__ q, const TI* __restrict__ k,
                       const TI* __restrict__ v, const float* __restrict__ f, float* __restrict__ o_loc,
                       float* __restrict__ u, float* __restrict__ P_out, float* __restrict__ S_loc, int T,
                       int nch, WsHeader* hdr) {
  using SL = Slot<TI>;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* slots = smem_raw;                                             // [2][SL::kBytes]
  float* X = reinterpret_cast<float*>(smem_raw + 2 * SL::kBytes);       // [2][D][XP]
  float* red = X + 2 * D * XP;                                           // [2][8][XP]
  float* fs = red + 2 * 8 * XP;                                          // [C]
  uint64_t* bars = reinterpret_cast<uint64_t*>(fs + C);                  // [2]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = lane >> 4, g = lane & 15;
  const int r0 = (2 * warp + h) * 4;  // this thread's rows r0..r0+3
  const int c0 = g * 4;               // its columns c0..c0+3 of P and of S^loc
  const int item = blockIdx.x;
  const int bh = item / nch, c = item % nch;
  const int t0 = c * C, L = min(C, T - t0);
  const size_t row0 = (size_t)bh * T + t0;  // global step index of the chunk's first step

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  for (int e = tid; e < D * XP; e += NT) {  // P = I, S^loc = 0
    const int kr = e / XP, c = e % XP;
    X[xidx(kr, c)] = (c == kr) ? 1.f : 0.f;
  }
  if (tid < C) fs[tid] = tid < L ? f[row0 + tid] : 1.f;
  __syncthreads();

  auto issue = [&](int s) {
    if (s < L) {
      uint8_t* sl = slots + (s & 1) * SL::kBytes;
      const size_t r = row0 + s;
      mbar_arrive_expect_tx(&bars[s & 1], SL::kBytes);
      bulk_g2s(sl, A + r * D * D, SL::kBytesA, &bars[s & 1]);
      bulk_g2s(sl + SL::kBytesA, k + r * D, SL::kRow, &bars[s & 1]);
      bulk_g2s(sl + SL::kBytesA + SL::kRow, q + r * D, SL::kRow, &bars[s & 1]);
      bulk_g2s(sl + SL::kBytesA + 2 * SL::kRow, v + r * D, SL::kRow, &bars[s & 1]);
    }
  };
  if (tid == 0) issue(0);

  float acc[4][8];
  int cur = 0, s = 0;
  bool ok = true;
  for (; s < L; ++s) {
    if (tid == 0) issue(s + 1);  // slot (s+1)&1 was last read before the previous step's barrier
    if (!mbar_wait(&bars[s & 1], (s >> 1) & 1)) ok = false;
    const uint8_t* sl = slots + (s & 1) * SL::kBytes;
    const float* At = reinterpret_cast<const float*>(sl);
    const TI* kt = reinterpret_cast<const TI*>(sl + SL::kBytesA);
    const TI* qt = kt + D;
    const TI* vt = qt + D;
    const float* Xc = X + cur * D * XP + g * 4;
    float2 acc2[4][8];  // (even-k, odd-k) partial sums
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) acc2[i][jj] = make_float2(0.f, 0.f);
#pragma unroll 2
    for (int kk = 0; kk < D; kk += 4) {
      float4 a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = ld4(At + (r0 + i) * D + kk);
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const float* xr = Xc + (kk / 2 + m) * 256;
        const float4 x0 = ld4(xr), x1 = ld4(xr + 64), x2 = ld4(xr + 128), x3 = ld4(xr + 192);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 ap = m == 0 ? lo2(a[i]) : hi2(a[i]);  // (A[r][k], A[r][k+1])
          acc2[i][0] = ffma2(ap, lo2(x0), acc2[i][0]);
          acc2[i][1] = ffma2(ap, hi2(x0), acc2[i][1]);
          acc2[i][2] = ffma2(ap, lo2(x1), acc2[i][2]);
          acc2[i][3] = ffma2(ap, hi2(x1), acc2[i][3]);
          acc2[i][4] = ffma2(ap, lo2(x2), acc2[i][4]);
          acc2[i][5] = ffma2(ap, hi2(x2), acc2[i][5]);
          acc2[i][6] = ffma2(ap, lo2(x3), acc2[i][6]);
          acc2[i][7] = ffma2(ap, hi2(x3), acc2[i][7]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) acc[i][jj] = acc2[i][jj].x + acc2[i][jj].y;
    // rank-1 write into the S^loc half, formed as the reference forms V_t
    const float w = 1.f - fs[s];
    const float4 kr = ld4(kt + r0), vc = ld4(vt + c0), qr = ld4(qt + r0);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][4 + j] += w * (comp(kr, i) * comp(vc, j));
    float* Xn = X + (cur ^ 1) * D * XP + g * 4;
#pragma unroll
    for (int m = 0; m < 2; ++m) {  // rows r0 + 2m, r0 + 2m + 1 form row pair r0/2 + m
      float* xw = Xn + (r0 / 2 + m) * 256;
      const float* e0 = acc[2 * m];
      const float* e1 = acc[2 * m + 1];
      st4(xw, e0[0], e1[0], e0[1], e1[1]);
      st4(xw + 64, e0[2], e1[2], e0[3], e1[3]);
      st4(xw + 128, e0[4], e1[4], e0[5], e1[5]);
      st4(xw + 192, e0[6], e1[6], e0[7], e1[7]);
    }
    // readouts: partial sums over this thread's 4 rows, then the warp's 8 rows
    float part[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      float p = acc[0][jj] * qr.x;
      p = fmaf(acc[1][jj], qr.y, p);
      p = fmaf(acc[2][jj], qr.z, p);
      p = fmaf(acc[3][jj], qr.w, p);
      part[jj] = p + __shfl_xor_sync(0xffffffffu, p, 16);
    }
    float* rd = red + (s & 1) * 8 * XP + warp * XP;
    if (h == 0) {
      st4(rd + c0, part[0], part[1], part[2], part[3]);
      st4(rd + D + c0, part[4], part[5], part[6], part[7]);
    }
    ok = __syncthreads_and(ok);
    if (tid < XP) {
      const float* rs = red + (s & 1) * 8 * XP + tid;
      float sum = 0.f;
#pragma unroll
      for (int ww = 0; ww < 8; ++ww) sum += rs[ww * XP];
      float* dst = tid < D ? u : o_loc;
      dst[((size_t)item * C + s) * D + (tid & (D - 1))] = sum;
    }
    cur ^= 1;
    if (!ok) break;
  }
  if (ok) {
    float* Pd = P_out + (size_t)item * D * D;
    float* Sd = S_loc + (size_t)item * D * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      st4(Pd + (r0 + i) * D + c0, acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      st4(Sd + (r0 + i) * D + c0, acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
    }
  } else if (tid == 0) {
    record_error(hdr, MOGT_ERR_TIMEOUT, (uint32_t)item);
    // the copy for step s+1 may still be in flight: let it land (bounded) before exit
    if (s + 1 < L) mbar_wait(&bars[(s + 1) & 1], ((s + 1) >> 1) & 1);
  }
}

// ---------------------------------------------------------------------------
// Kernel 2: chunk carries S_in[c+1] = P_c S_in[c] + S^loc_c, per head and
// CC-column group.  S_in: [NB, D, D] (S_in[0] = S0 or 0); S_final: [BH, D, D]
// or NULL.  Thread layout: row r = tid/4 (j = r % 8 inside the warp), columns
// 2*(tid%4)..+1.  The state lives column-major in shared memory (pitch SP) so
// that a thread reads four k values of a column with one float4, and each
// lane group starts its k loop 4j further on: the 8 rows of P_c a warp reads
// at once then fall in 8 different bank groups.  P_c arrives through a CR-slot
// bulk-copy ring, S^loc_c through registers four chunks ahead.
// ---------------------------------------------------------------------------
constexpr int CR = 6;        // ring slots for P_c
constexpr int SP = D + 4;    // column pitch of the state in shared memory
constexpr int SLA = 4;       // S^loc chunks loaded ahead
__global__ void __launch_bounds__(256)
    chunk_carry_kernel(const float* __restrict__ P, const float* __restrict__ S_loc,
                       const float* __restrict__ S0, float* __restrict__ S_in, float* __restrict__ S_final,
                       int nch, WsHeader* hdr) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* ring = reinterpret_cast<float*>(smem_raw);   // [CR][D][D]
  float* St = ring + CR * D * D;                       // [2][CC][SP]
  uint64_t* bars = reinterpret_cast<uint64_t*>(St + 2 * CC * SP);
  const int tid = threadIdx.x;
  const int groups = D / CC;
  const int bh = blockIdx.x / groups, cgp = blockIdx.x % groups;
  const int r = tid >> 2, jr = r & 7, cl = (tid & 3) * 2, col = cgp * CC + cl;
  const size_t item0 = (size_t)bh * nch;

  if (tid == 0) {
    for (int i = 0; i < CR; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  float2 s;
  s.x = S0 ? S0[((size_t)bh * D + r) * D + col] : 0.f;
  s.y = S0 ? S0[((size_t)bh * D + r) * D + col + 1] : 0.f;
  St[cl * SP + r] = s.x;
  St[(cl + 1) * SP + r] = s.y;
  *reinterpret_cast<float2*>(S_in + (item0 * D + r) * D + col) = s;
  __syncthreads();
  auto issue = [&](int cc) {
    if (cc < nch) {
      mbar_arrive_expect_tx(&bars[cc % CR], D * D * 4);
      bulk_g2s(ring + (cc % CR) * D * D, P + (item0 + cc) * D * D, D * D * 4, &bars[cc % CR]);
    }
  };
  if (tid == 0)
    for (int cc = 0; cc < CR - 1; ++cc) issue(cc);
  auto load_sl = [&](int cc) {
    return cc < nch ? *reinterpret_cast<const float2*>(S_loc + ((item0 + cc) * D + r) * D + col)
                    : make_float2(0.f, 0.f);
  };
  float2 slq[SLA];
#pragma unroll
  for (int u = 0; u < SLA; ++u) slq[u] = load_sl(u);
  bool ok = true;
  int cur = 0, cc = 0;
  for (; cc < nch; ++cc) {
    if (tid == 0) issue(cc + CR - 1);
    const float2 sl = slq[0];
#pragma unroll
    for (int u = 0; u + 1 < SLA; ++u) slq[u] = slq[u + 1];
    slq[SLA - 1] = load_sl(cc + SLA);
    if (!mbar_wait(&bars[cc % CR], (cc / CR) & 1)) ok = false;
    const float* Pc = ring + (cc % CR) * D * D + r * D;
    const float* S0c = St + cur * CC * SP + cl * SP;
    const float* S1c = S0c + SP;
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;  // two partial sums per column
#pragma unroll
    for (int kk = 0; kk < D; kk += 4) {
      const int kq = (kk + 4 * jr) & (D - 1);
      const float4 p = ld4(Pc + kq);
      const float4 x = ld4(S0c + kq);
      const float4 y = ld4(S1c + kq);
      a0 = fmaf(p.x, x.x, a0); a1 = fmaf(p.x, y.x, a1);
      b0 = fmaf(p.y, x.y, b0); b1 = fmaf(p.y, y.y, b1);
      a0 = fmaf(p.z, x.z, a0); a1 = fmaf(p.z, y.z, a1);
      b0 = fmaf(p.w, x.w, b0); b1 = fmaf(p.w, y.w, b1);
    }
    const float2 ns = make_float2((a0 + b0) + sl.x, (a1 + b1) + sl.y);
    float* Sn = St + (cur ^ 1) * CC * SP;
    Sn[cl * SP + r] = ns.x;
    Sn[(cl + 1) * SP + r] = ns.y;
    if (cc + 1 < nch)
      *reinterpret_cast<float2*>(S_in + ((item0 + cc + 1) * D + r) * D + col) = ns;
    else if (S_final)
      *reinterpret_cast<float2*>(S_final + ((size_t)bh * D + r) * D + col) = ns;
    cur ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
  }
  if (!ok && tid == 0) {
    record_error(hdr, MOGT_ERR_TIMEOUT, (uint32_t)blockIdx.x);
    for (int c2 = cc + 1; c2 < min(nch, cc + CR); ++c2) mbar_wait(&bars[c2 % CR], (c2 / CR) & 1);
  }
}

// ---------------------------------------------------------------------------
// Kernel 3: o = o^loc + U S_in per chunk (U rows u_t), rows t < L written.
// Thread layout: rows 4*(tid/16)..+3, columns 4*(tid%16)..+3.
// ---------------------------------------------------------------------------
template <typename TO>
__global__ void __launch_bounds__(NT)
    chunk_out_kernel(const float* __restrict__ o_loc, const float* __restrict__ u,
                     const float* __restrict__ S_in, TO* __restrict__ o, int T, int nch) {
  __shared__ __align__(16) float Us[C * D];
  __shared__ __align__(16) float Ss[D * D];
  const int tid = threadIdx.x;
  const int item = blockIdx.x;
  const int bh = item / nch, c = item % nch;
  const int t0 = c * C, L = min(C, T - t0);
  const float4* ug = reinterpret_cast<const float4*>(u + (size_t)item * C * D);
  const float4* sg = reinterpret_cast<const float4*>(S_in + (size_t)item * D * D);
  for (int e = tid; e < C * D / 4; e += NT) {
    reinterpret_cast<float4*>(Us)[e] = ug[e];
    reinterpret_cast<float4*>(Ss)[e] = sg[e];
  }
  const int rr = (tid >> 4) * 4, c0 = (tid & 15) * 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 z = ld4(o_loc + ((size_t)item * C + rr + i) * D + c0);
    acc[i][0] = z.x; acc[i][1] = z.y; acc[i][2] = z.z; acc[i][3] = z.w;
  }
  __syncthreads();
#pragma unroll 4
  for (int kk = 0; kk < D; kk += 4) {
    float4 a[4], y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = ld4(Us + (rr + i) * D + kk);
#pragma unroll
    for (int j = 0; j < 4; ++j) y[j] = ld4(Ss + (kk + j) * D + c0);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float aij = comp(a[i], j);
        acc[i][0] = fmaf(aij, y[j].x, acc[i][0]);
        acc[i][1] = fmaf(aij, y[j].y, acc[i][1]);
        acc[i][2] = fmaf(aij, y[j].z, acc[i][2]);
        acc[i][3] = fmaf(aij, y[j].w, acc[i][3]);
      }
  }
  TO* ob = o + ((size_t)bh * T + t0) * D;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (rr + i >= L) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) ob[(size_t)(rr + i) * D + c0 + j] = from_f32<TO>(acc[i][j]);
  }
}

// ---------------------------------------------------------------------------
// Kernel 1, tensor-core form (bf16 q/k/v): the same per-chunk recurrence and
// outputs as chunk_local_kernel, with X <- A_t X computed on the tensor cores
// as Y <- Y A_t^T for Y = X^T (M = 128 columns of X, N = 64, K = 64).  fp32
// accuracy from three tf32 products (3xTF32): A ~ Ah + Al and Y ~ Yh + Yl
// with Ah = rna_tf32(A), Al = rna_tf32(A - Ah) (A - Ah is exact in fp32),
// likewise for Y; Y A^T ~ Yh Ah^T + Yh Al^T + Yl Ah^T.  The remainders'
// rounding and the dropped Yl Al^T are ~2^-22 relative and unbiased (the
// tensor core would truncate a non-tf32 remainder, and that bias accumulates
// linearly over a norm-preserving sequence).  The products accumulate in three
// tensor-memory accumulators -- Yh Ah^T over k < 32, over k >= 32, and the two
// cross terms -- added in fp32 in the epilogue: the large terms then see 4
// accumulation steps per step instead of 24, which keeps the accumulator's
// rounding from building up over the sequence.  Per step: TMA brings A_t (two 32-column halves, 128B swizzle,
// K-major: A's row-major rows are the B operand's N rows) and bulk copies
// k_t, q_t, v_t; all threads split A_t in place into Ah and an Al tile; one
// thread issues 24 kind::tf32 MMAs into a 128 x 64 fp32 accumulator in
// tensor memory; then warp w reads lanes 32 (w % 4) + l (column c of X) and
// accumulator columns 32 (w / 4) .. +31 (rows r of X), adds the rank-1 write
// on the S^loc half, forms the readout partial sums, and writes Y's new
// hi / lo rows (128-byte swizzled, the next step's A operand).
// ---------------------------------------------------------------------------
namespace tc {
// Two A tiles ([2 halves][64 rows][128 B] each) swap roles every step: A_s
// arrives in tile s & 1 and is split there into Ah, Al goes to the other
// tile; once the Yh Al^T products of step s are complete that tile is free
// and A_{s+1} is loaded into it while the rest of step s runs.
constexpr int OFF_A = 0;
constexpr int OFF_YH = OFF_A + 2 * 16384;  // Yh: [2 halves][128 rows][128 B]
constexpr int OFF_YL = OFF_YH + 32768;     // Yl
constexpr int OFF_KQV = OFF_YL + 32768;    // [2 slots][k, q, v rows] (<= 3 x 256 B each)
constexpr int OFF_RED = OFF_KQV + 2 * 768; // [2 halves][128] readout partial sums
constexpr int OFF_FS = OFF_RED + 1024;     // gates of the chunk [64]
constexpr int OFF_BAR = OFF_FS + 256;      // A slots [2], MMA [1], TMEM address slot
constexpr int SMEM = OFF_BAR + 64;
constexpr int SMEM_ALLOC = SMEM + 1024;    // 1024-byte alignment of the swizzled tiles
constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"((uint32_t)accumulate));
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                            int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// x rounded to the nearest tf32 value (an fp32 bit pattern with a zero low
// 13-bit field, which the tensor core takes as is)
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
}  // namespace tc

template <typename TI>
__global__ void __launch_bounds__(NT, 2)
    chunk_local_tc(const __grid_constant__ CUtensorMap tA, const TI* __restrict__ q, const TI* __restrict__ k,
                   const TI* __restrict__ v, const float* __restrict__ f, float* __restrict__ o_loc,
                   float* __restrict__ u, float* __restrict__ P_out, float* __restrict__ S_loc, int T, int nch,
                   WsHeader* hdr) {
  using namespace tc;
  constexpr int KROW = D * (int)sizeof(TI);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(sm + OFF_RED);
  float* fs = reinterpret_cast<float*>(sm + OFF_FS);
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* bar_m = bar_a + 2;   // all products of a step
  uint64_t* bar_lo = bar_a + 3;  // the Yh Al^T products of a step (the Al tile is free)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_a + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lq = warp & 3, hh = warp >> 2;
  const int cx = 32 * lq + lane;  // column of X (row of Y) this thread reads back
  const int item = blockIdx.x;
  const int bh = item / nch, c = item % nch;
  const int t0 = c * C, L = min(C, T - t0);
  const size_t row0 = (size_t)bh * T + t0;

  if (warp == 0) tmem_alloc(tslot, 256);  // three 64-column accumulators
  if (tid == 0) {
    mbar_init(&bar_a[0], 1);
    mbar_init(&bar_a[1], 1);
    mbar_init(bar_m, 1);
    mbar_init(bar_lo, 1);
    fence_barrier_init();
  }
  // Y = X^T at the chunk start: P = I (rows c < 64 of Y), S^loc = 0; Yl = 0
  for (int e = tid; e < 2 * 128 * 8; e += NT) {
    const int half = e >> 10, row = (e >> 3) & 127, ch = e & 7;
    float4 hv = make_float4(0.f, 0.f, 0.f, 0.f);
    const int kb = 32 * half + 4 * ch;  // first k of the 16-byte chunk
    if (row < 64 && row >= kb && row < kb + 4) reinterpret_cast<float*>(&hv)[row - kb] = 1.f;
    const uint32_t off = half * 16384 + sw128(row, ch);
    *reinterpret_cast<float4*>(sm + OFF_YH + off) = hv;
    *reinterpret_cast<float4*>(sm + OFF_YL + off) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (tid < C) fs[tid] = tid < L ? f[row0 + tid] : 1.f;
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  // A_st into A tile st & 1 (step st-1's Al tile, free once its Yh Al^T
  // products are complete), k_st, q_st, v_st into row slot st & 1 (the
  // epilogue of step st-1 still reads the other one)
  auto issue = [&](int st) {
    if (st < L) {
      const int sl = st & 1;
      uint8_t* a = sm + OFF_A + sl * 16384;
      uint8_t* kq = sm + OFF_KQV + sl * 768;
      const size_t r = row0 + st;
      mbar_arrive_expect_tx(&bar_a[sl], 16384 + 3 * KROW);
      tma_load_2d(a, &tA, &bar_a[sl], 0, (int32_t)(r * D));
      tma_load_2d(a + 8192, &tA, &bar_a[sl], 32, (int32_t)(r * D));
      bulk_g2s(kq, k + r * D, KROW, &bar_a[sl]);
      bulk_g2s(kq + KROW, q + r * D, KROW, &bar_a[sl]);
      bulk_g2s(kq + 2 * KROW, v + r * D, KROW, &bar_a[sl]);
    }
  };
  if (tid == 0) issue(0);

  float x[32];
  bool ok = true;
  int s = 0;
  for (; s < L; ++s) {
    const int sl = s & 1;
    if (!mbar_wait(&bar_a[sl], (s >> 1) & 1)) ok = false;
    // split A_t in place into Ah, and Al into its own tile (same layout)
    {
      float4* a4 = reinterpret_cast<float4*>(sm + OFF_A + sl * 16384);
      float4* l4 = reinterpret_cast<float4*>(sm + OFF_A + (sl ^ 1) * 16384);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = a4[tid + NT * i];
        const float4 h = make_float4(tf32_rna(a.x), tf32_rna(a.y), tf32_rna(a.z), tf32_rna(a.w));
        a4[tid + NT * i] = h;
        l4[tid + NT * i] = make_float4(tf32_rna(a.x - h.x), tf32_rna(a.y - h.y), tf32_rna(a.z - h.z),
                                       tf32_rna(a.w - h.w));
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ya = smem_u32(sm + OFF_YH), yl = smem_u32(sm + OFF_YL);
      const uint32_t ah = smem_u32(sm + OFF_A + sl * 16384), al = smem_u32(sm + OFF_A + (sl ^ 1) * 16384);
      // 32 bytes per K=8 step, in 16-byte units of the descriptor's address field
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // cross term Yh Al^T first: it frees the Al tile
        const int half = kk >> 2;
        const uint64_t sub = 2u * (kk & 3);
        umma_tf32(tbase + 128u, umma_desc_kmajor(ya + half * 16384) + sub,
                  umma_desc_kmajor(al + half * 8192) + sub, kk > 0);
      }
      umma_commit(bar_lo);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int half = kk >> 2;
        const uint64_t sub = 2u * (kk & 3);
        const uint64_t dah = umma_desc_kmajor(ah + half * 8192) + sub;
        umma_tf32(tbase + 64u * half, umma_desc_kmajor(ya + half * 16384) + sub, dah,
                  (kk & 3) != 0);                                                         // Yh Ah^T per k-half
        umma_tf32(tbase + 128u, umma_desc_kmajor(yl + half * 16384) + sub, dah, true);  // cross term Yl Ah^T
      }
      umma_commit(bar_m);
      // A_{s+1} goes into the Al tile as soon as the products reading it are done
      if (mbar_wait(bar_lo, s & 1)) issue(s + 1);
      else ok = false;
    }
    if (!mbar_wait(bar_m, s & 1)) ok = false;
    tc_fence_after();
    {
      const uint32_t ta = tbase + ((uint32_t)(32 * lq) << 16) + 32u * hh;
      uint32_t r0[32];
      tmem_ld_32x32b_x32_async(r0, ta);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r0[j]);
      tmem_ld_32x32b_x32_async(r0, ta + 64u);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] += __uint_as_float(r0[j]);
      tmem_ld_32x32b_x32_async(r0, ta + 128u);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] += __uint_as_float(r0[j]);
    }
    const TI* kt = reinterpret_cast<const TI*>(sm + OFF_KQV + sl * 768);
    const TI* qt = kt + D;
    const TI* vt = qt + D;
    if (cx >= D) {  // rank-1 write into the S^loc half, formed as the reference forms V_t
      const float w = 1.f - fs[s];
      const float vc = to_f32(vt[cx - D]);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 k4 = ld4(kt + 32 * hh + j);
        x[j] += w * (k4.x * vc);
        x[j + 1] += w * (k4.y * vc);
        x[j + 2] += w * (k4.z * vc);
        x[j + 3] += w * (k4.w * vc);
      }
    }
    float part = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 q4 = ld4(qt + 32 * hh + j);
      part = fmaf(x[j], q4.x, part);
      part = fmaf(x[j + 1], q4.y, part);
      part = fmaf(x[j + 2], q4.z, part);
      part = fmaf(x[j + 3], q4.w, part);
    }
    red[hh * 128 + cx] = part;
    // the new Y row cx, k-half hh: hi and lo parts, 128-byte swizzled
    {
      uint8_t* yh = sm + OFF_YH + hh * 16384;
      uint8_t* ylo = sm + OFF_YL + hh * 16384;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const float4 hv = make_float4(tf32_rna(x[4 * ch]), tf32_rna(x[4 * ch + 1]), tf32_rna(x[4 * ch + 2]),
                                      tf32_rna(x[4 * ch + 3]));
        *reinterpret_cast<float4*>(yh + sw128(cx, ch)) = hv;
        *reinterpret_cast<float4*>(ylo + sw128(cx, ch)) =
            make_float4(tf32_rna(x[4 * ch] - hv.x), tf32_rna(x[4 * ch + 1] - hv.y),
                        tf32_rna(x[4 * ch + 2] - hv.z), tf32_rna(x[4 * ch + 3] - hv.w));
      }
    }
    fence_proxy_async();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    if (tid < 128) {
      const float sum = red[tid] + red[128 + tid];
      float* dst = tid < D ? u : o_loc;
      dst[((size_t)item * C + s) * D + (tid & (D - 1))] = sum;
    }
    if (!ok) break;
  }
  if (ok) {  // the chunk's P and S^loc: column cx of X, rows 32 hh .. +31
    float* dst = (cx < D ? P_out : S_loc) + (size_t)item * D * D + (cx & (D - 1));
#pragma unroll
    for (int j = 0; j < 32; ++j) dst[(size_t)(32 * hh + j) * D] = x[j];
  } else if (tid == 0) {
    record_error(hdr, MOGT_ERR_TIMEOUT, (uint32_t)item);
    mbar_wait(bar_m, s & 1);  // let this step's MMAs and the next step's copies finish
    if (s + 1 < L) mbar_wait(&bar_a[(s + 1) & 1], ((s + 1) >> 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

int launch_local_tc(const float* A, const void* q, const void* k, const void* v, const float* f, float* o_loc,
                    float* u, float* P, float* S_loc, int BH, int NB, int T, int nch, WsHeader* hdr,
                    cudaStream_t st) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)BH * T * D};
  cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)D};
  if (mogt_host::encode_tiled(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(A), dims, strides,
                              box, CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
    return MOGT_ERR_LAUNCH;
  auto kfn = chunk_local_tc<__nv_bfloat16>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM_ALLOC) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  kfn<<<NB, NT, tc::SMEM_ALLOC, st>>>(map, static_cast<const __nv_bfloat16*>(q),
                                      static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
                                      f, o_loc, u, P, S_loc, T, nch, hdr);
  return mogt_host::launch_status();
}

template <typename TI>
int launch_local(const float* A, const void* q, const void* k, const void* v, const float* f, float* o_loc,
                 float* u, float* P, float* S_loc, int NB, int T, int nch, WsHeader* hdr, cudaStream_t st) {
  const size_t smem = local_smem_bytes<TI>();
  auto kfn = chunk_local_kernel<TI>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  kfn<<<NB, NT, smem, st>>>(A, static_cast<const TI*>(q), static_cast<const TI*>(k),
                            static_cast<const TI*>(v), f, o_loc, u, P, S_loc, T, nch, hdr);
  return mogt_host::launch_status();
}

}  // namespace mchunk
}  // namespace mogt

extern "C" size_t mogt_matrix_scan_chunked_scratch_bytes(int64_t BH, int64_t T, int64_t d) {
  using namespace mogt::mchunk;
  if (BH <= 0 || T <= 0 || d != D) return 0;
  const int64_t nch = (T + C - 1) / C;
  return (size_t)5 * BH * nch * D * D * 4;  // o_loc, u, P, S_loc, S_in
}

extern "C" int mogt_matrix_scan_fwd_chunked(const float* A, const void* q, const void* k, const void* v,
                                            const float* f, void* o, const float* S0, float* S_final,
                                            int64_t BH, int64_t T, int64_t d, int in_dtype, int out_dtype,
                                            int mode, void* status, void* scratch, size_t scratch_bytes,
                                            void* stream) {
  using namespace mogt::mchunk;
  if (BH <= 0 || T < 0) return MOGT_ERR_SHAPE;
  if (d != D) return MOGT_ERR_UNSUPPORTED;
  if (T == 0) return MOGT_OK;
  if (!A || !q || !k || !v || !f || !o || !status || !scratch) return MOGT_ERR_ARG;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(q) |
                        reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                        reinterpret_cast<uintptr_t>(scratch);
  if (mis & 15u) return MOGT_ERR_ALIGN;
  const int64_t nch = (T + C - 1) / C, NB = BH * nch;
  if (NB >= ((int64_t)1 << 31) || BH * (D / CC) >= ((int64_t)1 << 31) || T >= ((int64_t)1 << 31))
    return MOGT_ERR_UNSUPPORTED;
  if (scratch_bytes < mogt_matrix_scan_chunked_scratch_bytes(BH, T, d)) return MOGT_ERR_WORKSPACE;
  if (in_dtype != MOGT_DTYPE_BF16 && in_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  if (out_dtype != MOGT_DTYPE_BF16 && out_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  if (in_dtype == MOGT_DTYPE_F32 && out_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  if (mode != MOGT_MATRIX_FP32 && mode != MOGT_MATRIX_TF32X3) return MOGT_ERR_ARG;
  if (mode == MOGT_MATRIX_TF32X3 && in_dtype != MOGT_DTYPE_BF16) return MOGT_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* hdr = static_cast<mogt::WsHeader*>(status);
  const size_t blk = (size_t)NB * D * D;
  float* o_loc = static_cast<float*>(scratch);
  float* u = o_loc + blk;
  float* P = u + blk;
  float* S_loc = P + blk;
  float* S_in = S_loc + blk;
  const int nb = (int)NB, Ti = (int)T, nc = (int)nch;
  // MOGT_MATRIX_FP32: fp32 FMAs (round-to-nearest, unbiased); MOGT_MATRIX_TF32X3:
  // the tensor-core chunk kernel (bf16 q/k/v only), whose accumulation rounding
  // is biased and drifts over long norm-preserving sequences
  int rc = mode == MOGT_MATRIX_TF32X3
               ? launch_local_tc(A, q, k, v, f, o_loc, u, P, S_loc, (int)BH, nb, Ti, nc, hdr, st)
           : in_dtype == MOGT_DTYPE_BF16
               ? launch_local<__nv_bfloat16>(A, q, k, v, f, o_loc, u, P, S_loc, nb, Ti, nc, hdr, st)
               : launch_local<float>(A, q, k, v, f, o_loc, u, P, S_loc, nb, Ti, nc, hdr, st);
  if (rc != MOGT_OK) return rc;
  const size_t csmem = (size_t)CR * D * D * 4 + 2 * CC * SP * 4 + 8 * CR;
  if (cudaFuncSetAttribute(chunk_carry_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem) !=
      cudaSuccess)
    return MOGT_ERR_LAUNCH;
  chunk_carry_kernel<<<(unsigned)(BH * (D / CC)), 256, csmem, st>>>(P, S_loc, S0, S_in, S_final, nc, hdr);
  if ((rc = mogt_host::launch_status()) != MOGT_OK) return rc;
  if (out_dtype == MOGT_DTYPE_BF16)
    chunk_out_kernel<__nv_bfloat16><<<nb, NT, 0, st>>>(o_loc, u, S_in, static_cast<__nv_bfloat16*>(o), Ti, nc);
  else
    chunk_out_kernel<float><<<nb, NT, 0, st>>>(o_loc, u, S_in, static_cast<float*>(o), Ti, nc);
  return mogt_host::launch_status();
}

