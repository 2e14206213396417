// Dense-transition headed scan, backward:
//     S_t = A_t S_{t-1} + w_t k_t v_t^T  (w_t = 1 - f_t),   o_t = S_t^T q_t,
// gradients of L = sum_t <o_t, do_t>.  Reference semantics: the affine
// backward affine_scan.py:65-124 (Sigma_t = g_t + U_{t+1}^T Sigma_{t+1},
// dU_t = Sigma_t H_{t-1}^T, dV_t = Sigma_t) with U = A, V = w k v^T and the
// readout's g_t = q_t do_t^T, chained to
//     dA_t = Sigma_t S_{t-1}^T,   dq_t = S_t do_t,   dk_t = w_t Sigma_t v_t,
//     dv_t = w_t Sigma_t^T k_t,   df_t = -k_t^T Sigma_t v_t,   dS0 = A_0^T Sigma_0.
//
// Reverse-time chunked form on the forward's stored chunk states.  The
// chunked forward (matrix_chunked.cu) leaves, per 64-step chunk c, the state
// entering it S_in[c] and the chunk's transition product P_c = A_{t1-1}..A_{t0}.
// With X_c = A_{t1}^T Sigma_{t1} the adjoint carried into chunk c from the
// later chunks, Sigma inside the chunk is Sigma^loc_t + R_t^T X_c with
// Sigma^loc the adjoint of the chunk alone (zero carry) and R_t the product
// of the chunk's transitions after t, so the carry between chunks is
//     X_{c-1} = P_c^T X_c + G_c,     G_c = A_{t0}^T Sigma^loc_{t0}.
// Kernel 1 (all chunks in parallel) runs the chunk-local reverse recurrence
// for G_c; kernel 2 (per head and 8 state columns, sequential over chunks)
// composes the carries X_c and dS0; kernel 3 (persistent, one CTA per SM,
// chunks in parallel) recomputes the chunk's forward states from S_in[c] --
// streamed to a per-CTA history buffer in global memory through shared-memory
// staging and bulk copies -- then walks the chunk backwards from X_c, forming
// Sigma_t, dA_t (written once, streaming) and the per-step vector gradients.
// fp32 arithmetic on the CUDA cores throughout (packed fma.rn.f32x2): with
// norm-preserving A_t round-off never decays, and round-to-nearest keeps it
// unbiased (a tensor-core tf32 product's accumulation is not).
// Thread tile of every 64x64 product: rows 4 (tid / 16) .. +3, columns
// 4 (tid % 16) .. +3.
#include <algorithm>

#include "common.cuh"

namespace mogt {
namespace mbwd {

constexpr int D = 64;        // state size (dk = dv)
constexpr int C = 64;        // steps per chunk (the forward's chunk)
constexpr int NT = 256;
constexpr int TSZ = D * D;   // floats per 64x64 tile
constexpr uint32_t TBYTES = TSZ * 4;

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)),
        "l"(*reinterpret_cast<const uint64_t*>(&c)));
  return *reinterpret_cast<const float2*>(&d);
}
__device__ __forceinline__ float comp(const float4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// out[r][c] (+)= sum_k L[k][r] R[k][c]  (both operands row-major 64x64 in
// shared memory; the contraction runs over their first index).
__device__ __forceinline__ void mm_kk(float (&acc)[4][4], const float* L, const float* R, int r0,
                                      int c0, bool accumulate) {
  float2 a[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a[i][0] = accumulate ? make_float2(acc[i][0], acc[i][1]) : make_float2(0.f, 0.f);
    a[i][1] = accumulate ? make_float2(acc[i][2], acc[i][3]) : make_float2(0.f, 0.f);
  }
#pragma unroll 8
  for (int k = 0; k < D; ++k) {
    const float4 l = ld4(L + k * D + r0);
    const float4 r = ld4(R + k * D + c0);
    const float2 r01 = make_float2(r.x, r.y), r23 = make_float2(r.z, r.w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float li = comp(l, i);
      a[i][0] = ffma2(make_float2(li, li), r01, a[i][0]);
      a[i][1] = ffma2(make_float2(li, li), r23, a[i][1]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[i][0] = a[i][0].x; acc[i][1] = a[i][0].y;
    acc[i][2] = a[i][1].x; acc[i][3] = a[i][1].y;
  }
}

// out[r][c] = sum_k L[r][k] R[k][c]  (L's rows are read four k at a time).
__device__ __forceinline__ void mm_rk(float (&acc)[4][4], const float* L, const float* R, int r0,
                                      int c0) {
  float2 a[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i][0] = a[i][1] = make_float2(0.f, 0.f);
#pragma unroll 2
  for (int k = 0; k < D; k += 4) {
    float4 l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) l[i] = ld4(L + (r0 + i) * D + k);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float4 r = ld4(R + (k + kk) * D + c0);
      const float2 r01 = make_float2(r.x, r.y), r23 = make_float2(r.z, r.w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float li = comp(l[i], kk);
        a[i][0] = ffma2(make_float2(li, li), r01, a[i][0]);
        a[i][1] = ffma2(make_float2(li, li), r23, a[i][1]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[i][0] = a[i][0].x; acc[i][1] = a[i][0].y;
    acc[i][2] = a[i][1].x; acc[i][3] = a[i][1].y;
  }
}

__device__ __forceinline__ void store_tile(float* dst, const float (&a)[4][4], int r0, int c0) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4*>(dst + (r0 + i) * D + c0) = make_float4(a[i][0], a[i][1], a[i][2], a[i][3]);
}
__device__ __forceinline__ void store_tile_t(float* dst, const float (&a)[4][4], int r0, int c0) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<float4*>(dst + (c0 + j) * D + r0) = make_float4(a[0][j], a[1][j], a[2][j], a[3][j]);
}
__device__ __forceinline__ void load_tile_g(float (&a)[4][4], const float* src, int r0, int c0) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(src + (r0 + i) * D + c0));
    a[i][0] = v.x; a[i][1] = v.y; a[i][2] = v.z; a[i][3] = v.w;
  }
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return to_f32(*p); }

// Per-step vectors of one chunk step, staged in shared memory: q, do, k, v
// (64 each) and the gate.  Thread i < 256 loads element i % 64 of vector i / 64.
template <typename TI>
struct StepVecs {
  const TI* q;
  const TI* d_o;
  const TI* k;
  const TI* v;
  __device__ __forceinline__ float load(size_t row, int tid) const {
    const int which = tid >> 6, e = tid & 63;
    const TI* p = which == 0 ? q : which == 1 ? d_o : which == 2 ? k : v;
    return p ? ldf(p + row * D + e) : 0.f;
  }
};

// ---------------------------------------------------------------------------
// Kernel 1: G_c = A_{t0}^T Sigma^loc_{t0}, the chunk's own adjoint carried out
// of it with a zero carry in.  One CTA per (head, chunk).
// ---------------------------------------------------------------------------
constexpr size_t K1_SMEM = 2 * TBYTES + TBYTES + 2 * 2 * D * 4 + 32;

template <typename TI>
__global__ void __launch_bounds__(NT, 2)
    rev_local_kernel(const float* __restrict__ A, StepVecs<TI> sv, float* __restrict__ G, int T,
                     int nch, WsHeader* hdr) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* Ab = reinterpret_cast<float*>(smem_raw);   // [2][64][64]
  float* Sg = Ab + 2 * TSZ;                          // Sigma, row-major
  float* vq = Sg + TSZ;                              // [2][q | do]
  uint64_t* bars = reinterpret_cast<uint64_t*>(vq + 4 * D);
  const int tid = threadIdx.x;
  const int r0 = (tid >> 4) * 4, c0 = (tid & 15) * 4;
  const int item = blockIdx.x, bh = item / nch, c = item % nch;
  const int t0 = c * C, L = min(C, T - t0);
  const size_t row0 = (size_t)bh * T + t0;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  // A of step s goes to slot (L - 1 - s) & 1 (the reverse walk's order)
  auto issue = [&](int s) {
    if (s >= 0) {
      const int sl = (L - 1 - s) & 1;
      mbar_arrive_expect_tx(&bars[sl], TBYTES);
      bulk_g2s(Ab + sl * TSZ, A + (row0 + s) * TSZ, TBYTES, &bars[sl]);
    }
  };
  if (tid == 0) {
    issue(L - 1);
    issue(L - 2);
  }
  float vnext = tid < 2 * D ? sv.load(row0 + L - 1, tid) : 0.f;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  bool ok = true;
  int it = 0;
  for (int s = L - 1; s >= 0; --s, ++it) {
    float* vb = vq + (it & 1) * 2 * D;
    if (tid < 2 * D) vb[tid] = vnext;
    if (tid < 2 * D && s > 0) vnext = sv.load(row0 + s - 1, tid);
    __syncthreads();  // vectors visible; the previous step's reads of Sg are done
    // Sigma^loc_t = carry + q_t do_t^T
    const float4 qv = ld4(vb + r0), dv = ld4(vb + D + c0);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(comp(qv, i), comp(dv, j), acc[i][j]);
    store_tile(Sg, acc, r0, c0);
    if (!mbar_wait(&bars[it & 1], (it >> 1) & 1)) ok = false;
    __syncthreads();
    // carry out of step t: A_t^T Sigma_t
    mm_kk(acc, Ab + (it & 1) * TSZ, Sg, r0, c0, false);
    ok = __syncthreads_and(ok);  // slot it & 1 is free again
    if (!ok) break;
    if (tid == 0) issue(s - 2);
  }
  if (ok) {
    store_tile(G + (size_t)item * TSZ, acc, r0, c0);
  } else if (tid == 0) {
    record_error(hdr, MOGT_ERR_TIMEOUT, (uint32_t)item);
    for (int i = 0; i < 2; ++i) mbar_wait(&bars[(it + 1 + i) & 1], ((it + 1 + i) >> 1) & 1);
  }
}

// ---------------------------------------------------------------------------
// Kernel 2: carries X_{c-1} = P_c^T X_c + G_c from the last chunk (X = 0)
// down, and dS0 = P_0^T X_0 + G_0.  One CTA per head and 8 state columns;
// thread row r = tid / 4 and columns 2 (tid % 4), +1 of the group.  P_c
// streams through a ring of bulk copies; X lives column-major in shared
// memory so a thread reads four k of a column with one float4.
// ---------------------------------------------------------------------------
constexpr int CC = 8, CR = 4, XPITCH = D + 4;
constexpr size_t K2_SMEM = (size_t)CR * TBYTES + 2 * CC * XPITCH * 4 + 8 * CR;

__global__ void __launch_bounds__(256)
    carry_rev_kernel(const float* __restrict__ P, const float* __restrict__ G, float* __restrict__ X,
                     float* __restrict__ dS0, int nch, WsHeader* hdr) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* ring = reinterpret_cast<float*>(smem_raw);  // [CR][64][64]
  float* Xs = ring + CR * TSZ;                        // [2][CC][XPITCH]
  uint64_t* bars = reinterpret_cast<uint64_t*>(Xs + 2 * CC * XPITCH);
  const int tid = threadIdx.x;
  const int groups = D / CC;
  const int bh = blockIdx.x / groups, cg = blockIdx.x % groups;
  const int r = tid >> 2, cl = (tid & 3) * 2, col = cg * CC + cl;
  const size_t item0 = (size_t)bh * nch;
  if (tid == 0) {
    for (int i = 0; i < CR; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  Xs[cl * XPITCH + r] = 0.f;
  Xs[(cl + 1) * XPITCH + r] = 0.f;
  *reinterpret_cast<float2*>(X + ((item0 + nch - 1) * D + r) * D + col) = make_float2(0.f, 0.f);
  __syncthreads();
  // chunk nch-1-i in ring slot i % CR
  auto issue = [&](int i) {
    if (i < nch) {
      mbar_arrive_expect_tx(&bars[i % CR], TBYTES);
      bulk_g2s(ring + (i % CR) * TSZ, P + (item0 + nch - 1 - i) * TSZ, TBYTES, &bars[i % CR]);
    }
  };
  if (tid == 0)
    for (int i = 0; i < CR - 1; ++i) issue(i);
  bool ok = true;
  int cur = 0, i = 0;
  for (; i < nch; ++i) {
    const int cc = nch - 1 - i;
    if (tid == 0) issue(i + CR - 1);
    const float2 g = __ldg(reinterpret_cast<const float2*>(G + ((item0 + cc) * D + r) * D + col));
    if (!mbar_wait(&bars[i % CR], (i / CR) & 1)) ok = false;
    const float* Pc = ring + (i % CR) * TSZ;
    const float* x0 = Xs + cur * CC * XPITCH + cl * XPITCH;
    const float* x1 = x0 + XPITCH;
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll 4
    for (int k = 0; k < D; k += 4) {
      const float4 xa = ld4(x0 + k), xb = ld4(x1 + k);
      const float p0 = Pc[(k + 0) * D + r], p1 = Pc[(k + 1) * D + r];
      const float p2 = Pc[(k + 2) * D + r], p3 = Pc[(k + 3) * D + r];
      a0 = fmaf(p0, xa.x, a0); b0 = fmaf(p0, xb.x, b0);
      a1 = fmaf(p1, xa.y, a1); b1 = fmaf(p1, xb.y, b1);
      a0 = fmaf(p2, xa.z, a0); b0 = fmaf(p2, xb.z, b0);
      a1 = fmaf(p3, xa.w, a1); b1 = fmaf(p3, xb.w, b1);
    }
    const float2 nx = make_float2((a0 + a1) + g.x, (b0 + b1) + g.y);
    float* xn = Xs + (cur ^ 1) * CC * XPITCH;
    xn[cl * XPITCH + r] = nx.x;
    xn[(cl + 1) * XPITCH + r] = nx.y;
    if (cc > 0)
      *reinterpret_cast<float2*>(X + ((item0 + cc - 1) * D + r) * D + col) = nx;
    else if (dS0)
      *reinterpret_cast<float2*>(dS0 + ((size_t)bh * D + r) * D + col) = nx;
    cur ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
  }
  if (!ok && tid == 0) {
    record_error(hdr, MOGT_ERR_TIMEOUT, (uint32_t)blockIdx.x);
    for (int j = i + 1; j < min(nch, i + CR); ++j) mbar_wait(&bars[j % CR], (j / CR) & 1);
  }
}

// ---------------------------------------------------------------------------
// Kernel 3: per chunk, forward states from S_in then the reverse walk with
// all gradients.  Persistent: CTA b takes chunks b, b + grid, ... and keeps
// the states of its current chunk (transposed, S^T_{t0-1} .. S^T_{t1-1}) in
// its own history slab hist[b][0..64].
// Shared memory: A ring (2 tiles), the state / Sigma tile (row-major), Sigma^T,
// a 3-tile ring of transposed states (staging in the forward, history reads
// in the reverse), per-step vectors and the vector-gradient partial sums.
// ---------------------------------------------------------------------------
constexpr int TR = 3;  // transposed-state ring
constexpr size_t K3_FLOATS = 2 * TSZ + TSZ + TSZ + TR * TSZ + 2 * 4 * D + 3 * 4 * D + 4 + 4;
constexpr size_t K3_SMEM = K3_FLOATS * 4 + 8 * 8;

template <typename TI, typename TO>
__global__ void __launch_bounds__(NT, 1)
    grad_kernel(const float* __restrict__ A, StepVecs<TI> sv, const float* __restrict__ f,
                const float* __restrict__ S_in, const float* __restrict__ X,
                float* __restrict__ hist, float* __restrict__ dA, TO* __restrict__ dq,
                TO* __restrict__ dk, TO* __restrict__ dv, float* __restrict__ df, int T, int nch,
                int NB, WsHeader* hdr) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* Ab = reinterpret_cast<float*>(smem_raw);  // [2][64][64]
  float* Sb = Ab + 2 * TSZ;                         // S (forward) / Sigma (reverse), row-major
  float* SgT = Sb + TSZ;                            // Sigma^T
  float* Tr = SgT + TSZ;                            // [TR][64][64] transposed states
  float* vec = Tr + TR * TSZ;                       // [2][q | do | k | v]
  float* red = vec + 2 * 4 * D;                     // [3][4][64]
  float* dfp = red + 3 * 4 * D;                     // [2] df partial sums (+2 spare)
  float* fsm = dfp + 4;                             // [2] gates (+2 spare)
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(fsm + 4);  // [2]
  uint64_t* bar_t = bar_a + 2;                              // [TR]
  const int tid = threadIdx.x, lane = tid & 31;
  const int r0 = (tid >> 4) * 4, c0 = (tid & 15) * 4;
  float* my_hist = hist + (size_t)blockIdx.x * (C + 1) * TSZ;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) mbar_init(&bar_a[i], 1);
    for (int i = 0; i < TR; ++i) mbar_init(&bar_t[i], 1);
    fence_barrier_init();
  }
  __syncthreads();
  uint32_t pa[2] = {0, 0}, pt[TR] = {0, 0, 0};  // mbarrier phases
  bool ok = true;
  auto wait_a = [&](int sl) {
    if (!mbar_wait(&bar_a[sl], pa[sl])) ok = false;
    pa[sl] ^= 1u;
  };
  auto wait_t = [&](int sl) {
    if (!mbar_wait(&bar_t[sl], pt[sl])) ok = false;
    pt[sl] ^= 1u;
  };
  auto load_a = [&](int sl, size_t row) {
    mbar_arrive_expect_tx(&bar_a[sl], TBYTES);
    bulk_g2s(Ab + sl * TSZ, A + row * TSZ, TBYTES, &bar_a[sl]);
  };

  for (int item = blockIdx.x; item < NB && ok; item += gridDim.x) {
    const int bh = item / nch, c = item % nch;
    const int t0 = c * C, L = min(C, T - t0);
    const size_t row0 = (size_t)bh * T + t0;
    // ---------------- forward: S_t for the chunk's steps, into the history ----
    if (tid == 0) {
      load_a(0, row0);
      if (L > 1) load_a(1, row0 + 1);
    }
    float s_reg[4][4];
    load_tile_g(s_reg, S_in + (size_t)item * TSZ, r0, c0);
    store_tile(Sb, s_reg, r0, c0);
    store_tile_t(Tr, s_reg, r0, c0);  // S^T_{t0-1} -> history slot 0
    float vnext = sv.load(row0, tid);
    float fnext = f[row0];
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      bulk_s2g(my_hist, Tr, TBYTES);
      bulk_commit();
    }
    for (int s = 0; s < L; ++s) {
      float* vb = vec + (s & 1) * 4 * D;
      vb[tid] = vnext;
      if (tid == 0) fsm[s & 1] = fnext;
      if (s + 1 < L) {
        vnext = sv.load(row0 + s + 1, tid);
        fnext = f[row0 + s + 1];
      }
      wait_a(s & 1);
      __syncthreads();  // vectors visible
      float acc[4][4];
      mm_rk(acc, Ab + (s & 1) * TSZ, Sb, r0, c0);
      const float w = 1.f - fsm[s & 1];
      const float4 kv = ld4(vb + 2 * D + r0), vv = ld4(vb + 3 * D + c0);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += w * (comp(kv, i) * comp(vv, j));
      // the staging slot of step s+1 was last read by the bulk store of step s-2
      if (tid == 0) bulk_wait_read<1>();
      ok = __syncthreads_and(ok);  // all reads of Sb and of A slot s & 1 are done
      if (!ok) break;
      if (tid == 0 && s + 2 < L) load_a(s & 1, row0 + s + 2);
      store_tile(Sb, acc, r0, c0);
      float* stg = Tr + ((s + 1) % TR) * TSZ;
      store_tile_t(stg, acc, r0, c0);
      fence_proxy_async();
      __syncthreads();
      if (tid == 0) {
        bulk_s2g(my_hist + (size_t)(s + 1) * TSZ, stg, TBYTES);
        bulk_commit();
      }
    }
    // the history must be in global memory before it is read back
    if (tid == 0) bulk_wait<0>();
    __syncthreads();
    if (!ok) break;
    // ---------------- reverse walk ----------------
    // Transposed states needed at reverse step s: hist[s + 1] (S_t, for dq)
    // and hist[s] (S_{t-1}, for dA).  hist[L] and hist[L-1] are still in their
    // staging slots L % TR and (L-1) % TR; hist[s] for s <= L-2 is reloaded
    // into slot s % TR, which last held hist[s + 3].
    // A_t is needed for the carry out of step t (t > t0): A_{t1-1} is still in
    // slot (L-1) & 1; the others are reloaded in reverse order.
    auto load_t = [&](int s) {
      const int sl = s % TR;
      mbar_arrive_expect_tx(&bar_t[sl], TBYTES);
      bulk_g2s(Tr + sl * TSZ, my_hist + (size_t)s * TSZ, TBYTES, &bar_t[sl]);
    };
    if (tid == 0) {
      if (L - 2 >= 0) load_t(L - 2);
      if (L - 2 >= 1) load_a(L & 1, row0 + L - 2);  // slot of A_{t1-2}: (L - 2) & 1
    }
    float acc[4][4];
    load_tile_g(acc, X + (size_t)item * TSZ, r0, c0);  // X_c: carry into the last step
    vnext = sv.load(row0 + L - 1, tid);
    fnext = f[row0 + L - 1];
    for (int s = L - 1, it = 0; s >= 0; --s, ++it) {
      const size_t row = row0 + s;
      float* vb = vec + (it & 1) * 4 * D;
      vb[tid] = vnext;
      if (tid == 0) fsm[it & 1] = fnext;
      if (s > 0) {
        vnext = sv.load(row - 1, tid);
        fnext = f[row - 1];
      }
      __syncthreads();  // vectors visible; the previous step's reads of Sb / SgT / red done
      // Sigma_t = carry + q_t do_t^T
      const float4 qv = ld4(vb + r0), dov = ld4(vb + D + c0);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(comp(qv, i), comp(dov, j), acc[i][j]);
      store_tile(Sb, acc, r0, c0);
      store_tile_t(SgT, acc, r0, c0);
      if (s <= L - 2) wait_t(s % TR);  // S^T_{t-1} landed
      __syncthreads();
      // prefetch S^T_{t-2} into the slot that held hist[s + 2] (last read at step s + 1)
      if (tid == 0 && s >= 1 && s <= L - 2) load_t(s - 1);
      // dA_t = Sigma_t S_{t-1}^T = sum_j Sigma^T[j][r] S^T_{t-1}[j][c]
      {
        float g[4][4];
        mm_kk(g, SgT, Tr + (s % TR) * TSZ, r0, c0, false);
        float* dst = dA + row * TSZ;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          __stcs(reinterpret_cast<float4*>(dst + (r0 + i) * D + c0), make_float4(g[i][0], g[i][1], g[i][2], g[i][3]));
      }
      // vector gradients: dq_t = S_t do_t (S^T_t = hist[s + 1]),
      // (Sigma_t v_t) and (Sigma_t^T k_t); 4 partial sums of 16 terms each
      {
        const int e = tid & 63, part = tid >> 6;
        const float* st = Tr + ((s + 1) % TR) * TSZ;
        float pq = 0.f, ps = 0.f, pv = 0.f;
#pragma unroll 4
        for (int j = part * 16; j < part * 16 + 16; ++j) {
          pq = fmaf(st[j * D + e], vb[D + j], pq);        // S_t[e][j] do[j]
          ps = fmaf(SgT[j * D + e], vb[3 * D + j], ps);   // Sigma[e][j] v[j]
          pv = fmaf(Sb[j * D + e], vb[2 * D + j], pv);    // Sigma[j][e] k[j]
        }
        red[(0 * 4 + part) * D + e] = pq;
        red[(1 * 4 + part) * D + e] = ps;
        red[(2 * 4 + part) * D + e] = pv;
      }
      // carry out of step t: A_t^T Sigma_t
      if (s > 0) {
        if (s < L - 1) wait_a(s & 1);  // A_{t1-1} is still in place from the forward walk
        mm_kk(acc, Ab + (s & 1) * TSZ, Sb, r0, c0, false);
      }
      ok = __syncthreads_and(ok);  // partial sums visible; A slot s & 1 free
      if (tid == 0 && s - 2 >= 1) load_a(s & 1, row0 + s - 2);
      const float w = 1.f - fsm[it & 1];
      if (tid < 3 * D) {
        const int which = tid >> 6, e = tid & 63;
        const float* rr = red + which * 4 * D + e;
        const float sum = (rr[0] + rr[D]) + (rr[2 * D] + rr[3 * D]);
        if (which == 0) {
          dq[row * D + e] = from_f32<TO>(sum);
        } else if (which == 1) {
          dk[row * D + e] = from_f32<TO>(w * sum);
          // df_t = -k_t . (Sigma_t v_t): two warps reduce, the first lane of each adds
          float x = vb[2 * D + e] * sum;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
          if (lane == 0) dfp[e >> 5] = x;
        } else {
          dv[row * D + e] = from_f32<TO>(w * sum);
        }
      }
      __syncthreads();
      if (tid == 0) df[row] = -(dfp[0] + dfp[1]);
      if (!ok) break;
    }
    __syncthreads();
  }
  if (!ok && tid == 0) {
    record_error(hdr, MOGT_ERR_TIMEOUT, (uint32_t)blockIdx.x);
    // let copies still in flight land (bounded) before the CTA exits
    for (int i = 0; i < 2; ++i) mbar_wait(&bar_a[i], pa[i]);
    for (int i = 0; i < TR; ++i) mbar_wait(&bar_t[i], pt[i]);
  }
  if (tid == 0) bulk_wait<0>();
}

}  // namespace mbwd
}  // namespace mogt

using namespace mogt;
using namespace mogt::mbwd;

namespace {

struct BwdScratch {
  float* G;
  float* X;
  float* hist;
  size_t total;
};

int bwd_grid() {
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  return nsm;
}

BwdScratch bwd_layout(void* base, int64_t NB, int grid) {
  BwdScratch s;
  char* p = static_cast<char*>(base);
  const size_t blk = (size_t)NB * TBYTES;
  s.G = reinterpret_cast<float*>(p);
  s.X = reinterpret_cast<float*>(p + blk);
  s.hist = reinterpret_cast<float*>(p + 2 * blk);
  s.total = 2 * blk + (size_t)grid * (C + 1) * TBYTES;
  return s;
}

template <typename TI>
int launch_bwd(const float* A, const void* q, const void* k, const void* v, const float* f,
               const void* d_o, const float* P, const float* S_in, float* dA, void* dq, void* dk,
               void* dv, float* df, float* dS0, int BH, int T, int nch, int NB, int grid,
               const BwdScratch& sc, WsHeader* hdr, cudaStream_t st) {
  StepVecs<TI> sv{static_cast<const TI*>(q), static_cast<const TI*>(d_o), static_cast<const TI*>(k),
                  static_cast<const TI*>(v)};
  auto k1 = rev_local_kernel<TI>;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K1_SMEM) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  k1<<<NB, NT, K1_SMEM, st>>>(A, sv, sc.G, T, nch, hdr);
  int rc = mogt_host::launch_status();
  if (rc != MOGT_OK) return rc;
  if (cudaFuncSetAttribute(carry_rev_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K2_SMEM) !=
      cudaSuccess)
    return MOGT_ERR_LAUNCH;
  carry_rev_kernel<<<BH * (D / CC), 256, K2_SMEM, st>>>(P, sc.G, sc.X, dS0, nch, hdr);
  if ((rc = mogt_host::launch_status()) != MOGT_OK) return rc;
  auto k3 = grad_kernel<TI, TI>;
  if (cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K3_SMEM) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  k3<<<grid, NT, K3_SMEM, st>>>(A, sv, f, S_in, sc.X, sc.hist, dA, static_cast<TI*>(dq),
                                static_cast<TI*>(dk), static_cast<TI*>(dv), df, T, nch, NB, hdr);
  return mogt_host::launch_status();
}

}  // namespace

extern "C" size_t mogt_matrix_scan_bwd_scratch_bytes(int64_t BH, int64_t T, int64_t d) {
  if (BH <= 0 || T <= 0 || d != D) return 0;
  const int64_t NB = BH * ((T + C - 1) / C);
  const int grid = (int)std::min<int64_t>(NB, bwd_grid());
  return bwd_layout(nullptr, NB, grid).total;
}

extern "C" int mogt_matrix_scan_bwd(const float* A, const void* q, const void* k, const void* v,
                                    const float* f, const void* d_o, const void* saved, float* dA,
                                    void* dq, void* dk, void* dv, float* df, float* dS0, int64_t BH,
                                    int64_t T, int64_t d, int in_dtype, void* status, void* scratch,
                                    size_t scratch_bytes, void* stream) {
  if (BH <= 0 || T < 0) return MOGT_ERR_SHAPE;
  if (d != D) return MOGT_ERR_UNSUPPORTED;
  if (T == 0) return MOGT_OK;
  if (!A || !q || !k || !v || !f || !d_o || !saved || !dA || !dq || !dk || !dv || !df || !status ||
      !scratch)
    return MOGT_ERR_ARG;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(saved) |
                        reinterpret_cast<uintptr_t>(dA) | reinterpret_cast<uintptr_t>(scratch) |
                        reinterpret_cast<uintptr_t>(dS0);
  if (mis & 15u) return MOGT_ERR_ALIGN;
  if (in_dtype != MOGT_DTYPE_BF16 && in_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  const int64_t nch = (T + C - 1) / C, NB = BH * nch;
  if (NB >= ((int64_t)1 << 31) || T >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  const int grid = (int)std::min<int64_t>(NB, bwd_grid());
  const BwdScratch sc = bwd_layout(scratch, NB, grid);
  if (scratch_bytes < sc.total) return MOGT_ERR_WORKSPACE;
  // the forward's chunked scratch: [o_loc | u | P | S_loc | S_in], NB tiles each
  const float* sv = static_cast<const float*>(saved);
  const size_t blk = (size_t)NB * TSZ;
  const float* P = sv + 2 * blk;
  const float* S_in = sv + 4 * blk;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* hdr = static_cast<WsHeader*>(status);
  if (in_dtype == MOGT_DTYPE_BF16)
    return launch_bwd<__nv_bfloat16>(A, q, k, v, f, d_o, P, S_in, dA, dq, dk, dv, df, dS0, (int)BH,
                                     (int)T, (int)nch, (int)NB, grid, sc, hdr, st);
  return launch_bwd<float>(A, q, k, v, f, d_o, P, S_in, dA, dq, dk, dv, df, dS0, (int)BH, (int)T,
                           (int)nch, (int)NB, grid, sc, hdr, st);
}
