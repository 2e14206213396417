// Backward of the fused diagonal gated scan + RMSNorm (diag_scan.cu):
//     h_t = a_t h_{t-1} + b_t,  a_t = damping (1 - z_t[row]),
//     b_t = v_t rnd(z_t[row]),  y_t = (h_t rs_t) w,  rs_t = rsqrt(mean(h_t^2) + eps).
// Gradients of L = sum <y, dy> (the chain rule the reference's autograd
// takes through V * z.to(V.dtype), the dense affine scan with U = damping
// (1 - z) I (affine_scan.py:65-124) and norm_out, model_mogt.py:168-240):
//     ŷ = h rs,  dŷ = dy w,   dw = sum_t dy_t ŷ_t,
//     dh_t = rs_t (dŷ_t - ŷ_t mean(ŷ_t dŷ_t))                 (RMSNorm)
//     λ_t = dh_t + a_{t+1} λ_{t+1}                             (adjoint scan)
//     dv_t = λ_t rnd(z_t),  dz_t[row] = sum_row (λ_t v_t - damping λ_t h_{t-1}),
//     dH0 = a_0 λ_0.
// Reverse-time chunked form, 8-token chunks, two channels per thread, one
// CTA per (chunk, batch row); a chunk's states are recomputed from the
// forward's chunk carries (h entering each forward chunk of lc_f tokens).
// With Λ_c = a_{t1} λ_{t1} the adjoint carried into chunk c from the right
// (t1 the next chunk's first token), λ inside the chunk is the chunk's own
// adjoint from a zero carry plus (prod of a after t) Λ_c, so
//     Λ_{c-1} = G_c + P_c Λ_c,  G_c = a_{t0} λ^loc_{t0},  P_c = prod_chunk a.
//   kernel 1  (chunks in parallel)  G_c, P_c;
//   kernel 2  (per channel, reverse over the chunks)  Λ_c and dH0;
//   kernel 3  (chunks in parallel)  dV, dz, per-chunk partial sums of dw;
//   kernel 4  dw = sum of the partials.
#include "common.cuh"

namespace mogt {
namespace diagb {

constexpr int G = 8;        // tokens per backward chunk (its states stay in registers)
constexpr int NPART = 64;   // dw partial-sum rows

struct Geo {
  int L, D, C, zs, R, nch, lc_f, nch_f;
  float damping, eps;
  WsHeader* hdr;
};

template <typename T>
__device__ __forceinline__ float2 ld2(const T* p);
template <>
__device__ __forceinline__ float2 ld2<float>(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }
template <>
__device__ __forceinline__ float2 ld2<__nv_bfloat16>(const __nv_bfloat16* p) {
  const unsigned int r = __ldg(reinterpret_cast<const unsigned int*>(p));
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r));
}
template <typename T>
__device__ __forceinline__ float rnd(float x) { return to_f32(from_f32<T>(x)); }
template <typename T>
__device__ __forceinline__ void st2(T* p, float a, float b);
template <>
__device__ __forceinline__ void st2<float>(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
template <>
__device__ __forceinline__ void st2<__nv_bfloat16>(__nv_bfloat16* p, float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  *reinterpret_cast<__nv_bfloat162*>(p) = v;
}
__device__ __forceinline__ float decay_of(float z, float damping) {
  const float omz = 1.f - z;
  return damping == 1.f ? omz : damping * omz;
}

// CTA-wide sums of G per-thread values (one per token); out[u] = the sum for
// token u.  red: [G][32] shared scratch.  Ends with a CTA barrier.
__device__ __forceinline__ void cta_sum(const float (&x)[G], float* red, float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int u = 0; u < G; ++u) {
    float s = x[u];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[u * 32 + warp] = s;
  }
  __syncthreads();
  for (int u = warp; u < G; u += nw) {
    float s = lane < nw ? red[u * 32 + lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[u] = s;
  }
  __syncthreads();
}

// The chunk's recomputed states and the RMSNorm backward, shared by kernels
// 1 and 3.  On return: hp[u] = h_{t0+u-1} (hp[G] the last state), dh[u]
// (two channels each),
// the decays a[u] and gates zr[u] of this thread's row, for tokens u < n.
template <typename TI, typename TD>
struct Chunk {
  float hp0[G + 1], hp1[G + 1], dh0[G], dh1[G], a[G], zr[G], v0[G], v1[G];
};

template <typename TI, typename TD>
__device__ __forceinline__ void recompute(Chunk<TI, TD>& k, const TI* __restrict__ V, const float* __restrict__ z,
                                          const TD* __restrict__ dy, const float* __restrict__ carry_f,
                                          const float* __restrict__ w, const Geo& g, int b, int c, float* red,
                                          float* tok, float2* dwpart) {
  const int ch = 2 * threadIdx.x;
  const int zi = g.zs == 1 ? 0 : ch / g.C;
  const int t0 = c * G, n = min(G, g.L - t0);
  // state entering the chunk: from the forward chunk carry, re-scanned to t0
  const int cf = t0 / g.lc_f, tf = cf * g.lc_f;
  const float2 cin = *reinterpret_cast<const float2*>(carry_f + ((size_t)b * g.nch_f + cf) * g.D + ch);
  float h0 = cin.x, h1 = cin.y;
  const size_t rowV = (size_t)b * g.L;
#pragma unroll 4
  for (int t = tf; t < t0; ++t) {
    const float2 v = ld2(V + (rowV + t) * g.D + ch);
    const float zz = __ldg(z + (rowV + t) * g.zs + zi);
    const float a = decay_of(zz, g.damping), zq = rnd<TI>(zz);
    h0 = __fadd_rn(__fmul_rn(a, h0), rnd<TI>(v.x * zq));
    h1 = __fadd_rn(__fmul_rn(a, h1), rnd<TI>(v.y * zq));
  }
  const float2 wv = *reinterpret_cast<const float2*>(w + ch);
  float sq[G], dyx[G], dyy[G];
#pragma unroll
  for (int u = 0; u < G; ++u) {
    const int t = t0 + min(u, n - 1);
    const float2 v = ld2(V + (rowV + t) * g.D + ch);
    const float zz = __ldg(z + (rowV + t) * g.zs + zi);
    const float2 d = ld2(dy + (rowV + t) * g.D + ch);
    k.v0[u] = v.x;
    k.v1[u] = v.y;
    k.a[u] = u < n ? decay_of(zz, g.damping) : 1.f;
    k.zr[u] = rnd<TI>(zz);
    dyx[u] = u < n ? d.x : 0.f;
    dyy[u] = u < n ? d.y : 0.f;
  }
  // hp[u] = h_{t0+u-1}; hp[G] = the chunk's last state
#pragma unroll
  for (int u = 0; u < G; ++u) {
    k.hp0[u] = h0;
    k.hp1[u] = h1;
    if (u < n) {
      h0 = __fadd_rn(__fmul_rn(k.a[u], h0), rnd<TI>(k.v0[u] * k.zr[u]));
      h1 = __fadd_rn(__fmul_rn(k.a[u], h1), rnd<TI>(k.v1[u] * k.zr[u]));
    }
    sq[u] = fmaf(h0, h0, h1 * h1);
  }
  k.hp0[G] = h0;
  k.hp1[G] = h1;
  float* rs = tok;       // [G] sum of h^2 over the channels
  float* mdot = tok + G; // [G] sum of ŷ dŷ
  cta_sum(sq, red, rs);
  const float inv_d = 1.f / (float)g.D;
  float dw0 = 0.f, dw1 = 0.f;
#pragma unroll
  for (int u = 0; u < G; ++u) {
    const float r = rsqrtf(rs[u] * inv_d + g.eps);
    const float y0 = k.hp0[u + 1] * r, y1 = k.hp1[u + 1] * r;
    dw0 = fmaf(dyx[u], y0, dw0);
    dw1 = fmaf(dyy[u], y1, dw1);
    dyx[u] *= wv.x;  // dŷ
    dyy[u] *= wv.y;
    sq[u] = fmaf(y0, dyx[u], y1 * dyy[u]);
  }
  cta_sum(sq, red, mdot);
#pragma unroll
  for (int u = 0; u < G; ++u) {
    const float r = rsqrtf(rs[u] * inv_d + g.eps), m = mdot[u] * inv_d;
    k.dh0[u] = u < n ? r * (dyx[u] - k.hp0[u + 1] * r * m) : 0.f;
    k.dh1[u] = u < n ? r * (dyy[u] - k.hp1[u + 1] * r * m) : 0.f;
  }
  if (dwpart) *dwpart = make_float2(dw0, dw1);
}

// Kernel 1: G_c = a_{t0} λ^loc_{t0} and P_c per channel.  gp: [B][nch][2][D].
template <typename TI, typename TD>
__global__ void __launch_bounds__(512)
    diag_bwd_local(const TI* __restrict__ V, const float* __restrict__ z, const TD* __restrict__ dy,
                   const float* __restrict__ carry_f, const float* __restrict__ w, float* __restrict__ gp,
                   Geo g) {
  __shared__ float red[G * 32];
  __shared__ float tok[2 * G];
  const int c = blockIdx.x, b = blockIdx.y, ch = 2 * threadIdx.x;
  Chunk<TI, TD> k;
  recompute(k, V, z, dy, carry_f, w, g, b, c, red, tok, nullptr);
  float l0 = 0.f, l1 = 0.f, an = 1.f, P = 1.f;
#pragma unroll
  for (int u = G - 1; u >= 0; --u) {
    l0 = fmaf(an, l0, k.dh0[u]);
    l1 = fmaf(an, l1, k.dh1[u]);
    an = k.a[u];
    P *= k.a[u];
  }
  float* dst = gp + ((size_t)b * g.nch + c) * 2 * g.D;
  *reinterpret_cast<float2*>(dst + ch) = make_float2(an * l0, an * l1);
  *reinterpret_cast<float2*>(dst + g.D + ch) = make_float2(P, P);
}

// Kernel 2: Λ_c for every chunk (reverse), dH0.  lam: [B][nch][D].
__global__ void __launch_bounds__(256)
    diag_bwd_carry(const float* __restrict__ gp, float* __restrict__ lam, float* __restrict__ dH0, Geo g) {
  const int b = blockIdx.y, ch = blockIdx.x * 256 + threadIdx.x;
  if (ch >= g.D) return;
  const float* gb = gp + (size_t)b * g.nch * 2 * g.D + ch;
  float* lb = lam + (size_t)b * g.nch * g.D + ch;
  float L = 0.f;
  constexpr int PF = 16;
  int c = g.nch - 1;
  for (; c - PF + 1 >= 0; c -= PF) {
    float Gv[PF], Pv[PF];
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      Gv[u] = __ldcg(gb + (size_t)(c - u) * 2 * g.D);
      Pv[u] = __ldcg(gb + (size_t)(c - u) * 2 * g.D + g.D);
    }
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      lb[(size_t)(c - u) * g.D] = L;
      L = fmaf(Pv[u], L, Gv[u]);
    }
  }
  for (; c >= 0; --c) {
    lb[(size_t)c * g.D] = L;
    L = fmaf(__ldcg(gb + (size_t)c * 2 * g.D + g.D), L, __ldcg(gb + (size_t)c * 2 * g.D));
  }
  if (dH0) dH0[(size_t)b * g.D + ch] = L;
}

// Kernel 3: dV, dz and the chunk's dw partial sums.
template <typename TI, typename TD>
__global__ void __launch_bounds__(512)
    diag_bwd_apply(const TI* __restrict__ V, const float* __restrict__ z, const TD* __restrict__ dy,
                   const float* __restrict__ carry_f, const float* __restrict__ w, const float* __restrict__ lam,
                   TI* __restrict__ dV, float* __restrict__ dz, float* __restrict__ dwp, Geo g) {
  __shared__ float red[G * 32];
  __shared__ float tok[2 * G];
  extern __shared__ float dzs[];  // [G][zs]
  const int c = blockIdx.x, b = blockIdx.y, ch = 2 * threadIdx.x;
  const int zi = g.zs == 1 ? 0 : ch / g.C;
  const int t0 = c * G, n = min(G, g.L - t0);
  for (int e = threadIdx.x; e < G * g.zs; e += blockDim.x) dzs[e] = 0.f;
  Chunk<TI, TD> k;
  float2 dwv;
  recompute(k, V, z, dy, carry_f, w, g, b, c, red, tok, &dwv);
  const float2 Lc = *reinterpret_cast<const float2*>(lam + ((size_t)b * g.nch + c) * g.D + ch);
  // λ_t = dh_t + a_{t+1} λ_{t+1}, the chunk's last token taking Λ_c (which
  // already carries a_{t1}); padded tokens past L have a = 1 and dh = 0, and
  // only the sequence's last chunk, whose Λ is 0, has them
  float l0 = Lc.x, l1 = Lc.y, an = 1.f;
  const size_t rowV = (size_t)b * g.L;
#pragma unroll
  for (int u = G - 1; u >= 0; --u) {
    l0 = fmaf(an, l0, k.dh0[u]);
    l1 = fmaf(an, l1, k.dh1[u]);
    if (u < n) {
      st2<TI>(dV + (rowV + t0 + u) * g.D + ch, l0 * k.zr[u], l1 * k.zr[u]);
      const float gz = (l0 * k.v0[u] + l1 * k.v1[u]) - g.damping * (l0 * k.hp0[u] + l1 * k.hp1[u]);
      atomicAdd(&dzs[u * g.zs + zi], gz);
    }
    an = k.a[u];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n * g.zs; e += blockDim.x) dz[(rowV + t0) * g.zs + e] = dzs[e];
  float* dp = dwp + (size_t)((b * g.nch + c) % NPART) * g.D + ch;
  atomicAdd(dp, dwv.x);
  atomicAdd(dp + 1, dwv.y);
}

// Kernel 4: dw[d] = sum of the NPART partial rows.
__global__ void diag_bwd_dw(const float* __restrict__ dwp, float* __restrict__ dw, int D) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  for (int p = 0; p < NPART; ++p) s += dwp[(size_t)p * D + d];
  dw[d] = s;
}

template <typename TI, typename TD>
int run(const void* V, const float* z, const void* dy, const float* carry_f, const float* w, void* dV,
        float* dz, float* dw, float* dH0, const Geo& g, int B, float* gp, float* lam, float* dwp,
        cudaStream_t s) {
  const int nt = g.D / 2;
  const dim3 grid(g.nch, B);
  if (cudaMemsetAsync(dwp, 0, (size_t)NPART * g.D * 4, s) != cudaSuccess) return MOGT_ERR_LAUNCH;
  diag_bwd_local<TI, TD><<<grid, nt, 0, s>>>(static_cast<const TI*>(V), z, static_cast<const TD*>(dy),
                                             carry_f, w, gp, g);
  int rc = mogt_host::launch_status();
  if (rc != MOGT_OK) return rc;
  diag_bwd_carry<<<dim3((g.D + 255) / 256, B), 256, 0, s>>>(gp, lam, dH0, g);
  if ((rc = mogt_host::launch_status()) != MOGT_OK) return rc;
  diag_bwd_apply<TI, TD><<<grid, nt, (size_t)G * g.zs * 4, s>>>(
      static_cast<const TI*>(V), z, static_cast<const TD*>(dy), carry_f, w, lam, static_cast<TI*>(dV), dz,
      dwp, g);
  if ((rc = mogt_host::launch_status()) != MOGT_OK) return rc;
  diag_bwd_dw<<<(g.D + 255) / 256, 256, 0, s>>>(dwp, dw, g.D);
  return mogt_host::launch_status();
}

}  // namespace diagb
}  // namespace mogt

namespace mogt {
namespace diag {
int forward_chunk_len(int64_t D, int in_dtype);
}
}  // namespace mogt

extern "C" size_t mogt_diag_scan_norm_bwd_scratch_bytes(int64_t B, int64_t L, int64_t R, int64_t C) {
  using namespace mogt::diagb;
  if (B <= 0 || L <= 0 || R <= 0 || C <= 0) return 0;
  const int64_t D = R * C, nch = (L + G - 1) / G;
  return (size_t)(B * nch * 3 * D + (int64_t)NPART * D) * sizeof(float);
}

extern "C" int mogt_diag_scan_norm_bwd(const void* V, const float* z, int64_t z_per_token, float damping,
                                       const float* norm_weight, float eps, const void* dy,
                                       const void* fwd_scratch, void* dV, float* dz, float* d_norm_weight,
                                       float* dH0, int64_t B, int64_t L, int64_t R, int64_t C, int in_dtype,
                                       int dy_dtype, void* status, void* scratch, size_t scratch_bytes,
                                       void* stream) {
  using namespace mogt::diagb;
  if (B <= 0 || L < 0 || R <= 0 || C <= 0) return MOGT_ERR_SHAPE;
  if (z_per_token != 1 && z_per_token != R) return MOGT_ERR_SHAPE;
  if (L == 0) return MOGT_OK;
  if (!V || !z || !norm_weight || !dy || !fwd_scratch || !dV || !dz || !d_norm_weight || !scratch || !status)
    return MOGT_ERR_ARG;
  if (in_dtype != MOGT_DTYPE_BF16 && in_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  if (dy_dtype != MOGT_DTYPE_BF16 && dy_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  const int64_t D = R * C;
  if (C % 2 != 0 || D % 64 != 0 || D > 1024 || R > 64) return MOGT_ERR_UNSUPPORTED;
  if (B > 65535 || L >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(dy) |
                        reinterpret_cast<uintptr_t>(dV) | reinterpret_cast<uintptr_t>(scratch) |
                        reinterpret_cast<uintptr_t>(fwd_scratch) | reinterpret_cast<uintptr_t>(norm_weight) |
                        (dH0 ? reinterpret_cast<uintptr_t>(dH0) : 0);
  if (mis & 7u) return MOGT_ERR_ALIGN;
  if (scratch_bytes < mogt_diag_scan_norm_bwd_scratch_bytes(B, L, R, C)) return MOGT_ERR_WORKSPACE;
  Geo g;
  g.L = (int)L;
  g.D = (int)D;
  g.C = (int)C;
  g.R = (int)R;
  g.zs = (int)z_per_token;
  g.nch = (int)((L + G - 1) / G);
  g.lc_f = mogt::diag::forward_chunk_len(D, in_dtype);
  g.nch_f = (int)((L + g.lc_f - 1) / g.lc_f);
  g.damping = damping;
  g.eps = eps;
  g.hdr = static_cast<mogt::WsHeader*>(status);
  // the forward's scratch: [aggregates (B, nch_f, 2, D) | carries (B, nch_f, D)]
  const float* carry_f = static_cast<const float*>(fwd_scratch) + (size_t)B * g.nch_f * 2 * D;
  float* gp = static_cast<float*>(scratch);
  float* lam = gp + (size_t)B * g.nch * 2 * D;
  float* dwp = lam + (size_t)B * g.nch * D;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using bf = __nv_bfloat16;
  const int bi = (int)B;
  if (in_dtype == MOGT_DTYPE_BF16 && dy_dtype == MOGT_DTYPE_BF16)
    return run<bf, bf>(V, z, dy, carry_f, norm_weight, dV, dz, d_norm_weight, dH0, g, bi, gp, lam, dwp, s);
  if (in_dtype == MOGT_DTYPE_BF16 && dy_dtype == MOGT_DTYPE_F32)
    return run<bf, float>(V, z, dy, carry_f, norm_weight, dV, dz, d_norm_weight, dH0, g, bi, gp, lam, dwp, s);
  if (in_dtype == MOGT_DTYPE_F32 && dy_dtype == MOGT_DTYPE_BF16)
    return run<float, bf>(V, z, dy, carry_f, norm_weight, dV, dz, d_norm_weight, dH0, g, bi, gp, lam, dwp, s);
  return run<float, float>(V, z, dy, carry_f, norm_weight, dV, dz, d_norm_weight, dH0, g, bi, gp, lam, dwp, s);
}
