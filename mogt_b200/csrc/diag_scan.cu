// Diagonal gated scan with the RMSNorm readout fused (the MOGT block with the
// identity connection and the forget gate coupled to a value gate,
// model_mogt.py:168-182, 185-240, as configured by
// benchmark_backbone_throughput.py:33-59):
//     U_t = damping (1 - z_t) I  (row-wise gate z_t[i], i < R),
//     V_t = V_t o z_t,   H_t = U_t H_{t-1} + V_t,   y_t = RMSNorm(H_t) * w.
// U_t is diagonal, so H is D = R * C independent channels h with
//     a_t = damping * (1 - z_t[row]),   b_t = rnd(v_t * rnd(z_t[row])),
//     h_t = a_t h_{t-1} + b_t,
// rnd() the input dtype's rounding (the reference multiplies V by
// z.to(V.dtype) in V's dtype); U_t H_{t-1} of the dense form adds exact zeros
// only, so a_t * h_{t-1} + b_t is its exact arithmetic (two roundings).
// The readout is y_t = (h_t * rsqrt(mean_d(h_t^2) + eps)) * w, written in the
// output dtype (bf16 under autocast: what the readout GEMM consumes).
//
// Three kernels, chunks of 64 tokens, one CTA per (chunk, batch row), two
// channels per thread:
//   1. chunk aggregates: P = prod a_t and the local end state (from 0);
//   2. carries: per channel, sequentially over the chunks,
//      h_in[c+1] = P_c h_in[c] + h_loc_c;
//   3. re-scan each chunk from its carry; per token the sum of squares is
//      reduced over the CTA (warp shuffles, then 8-token groups through
//      shared memory) and the normalised outputs written.
// HBM traffic per token: V twice, z twice, y once (bf16: 3 x 1536 B at
// D = 768); the per-chunk aggregates and carries are 3 x 8 B per channel and
// chunk.
#include "common.cuh"

namespace mogt {
namespace diag {

constexpr int LC = 64;   // tokens per chunk
constexpr int G = 8;     // tokens per normalisation group in kernel 3

template <typename T>
__device__ __forceinline__ float2 ld2(const T* p);
template <>
__device__ __forceinline__ float2 ld2<float>(const float* p) {
  return __ldcs(reinterpret_cast<const float2*>(p));
}
template <>
__device__ __forceinline__ float2 ld2<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint32_t r = __ldcs(reinterpret_cast<const unsigned int*>(p));
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r));
}
// v * z in the input dtype (z rounded to it first), as an fp32 value
template <typename T>
__device__ __forceinline__ float gated_value(float v, float z);
template <>
__device__ __forceinline__ float gated_value<float>(float v, float z) { return v * z; }
template <>
__device__ __forceinline__ float gated_value<__nv_bfloat16>(float v, float z) {
  const float zr = __bfloat162float(__float2bfloat16_rn(z));
  return __bfloat162float(__float2bfloat16_rn(v * zr));
}
template <typename T>
__device__ __forceinline__ void st2(T* p, float a, float b);
template <>
__device__ __forceinline__ void st2<float>(float* p, float a, float b) {
  __stcs(reinterpret_cast<float2*>(p), make_float2(a, b));
}
template <>
__device__ __forceinline__ void st2<__nv_bfloat16>(__nv_bfloat16* p, float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  __stcs(reinterpret_cast<unsigned int*>(p), *reinterpret_cast<const unsigned int*>(&v));
}

struct Geo {
  int L, D, C, zs, nch;  // zs: gates per token (R, or 1 for one scalar gate)
  float damping;
};

__device__ __forceinline__ float decay_of(float z, float damping) {
  const float omz = 1.f - z;
  return damping == 1.f ? omz : damping * omz;
}

// Kernel 1: P_c and the local end state of every chunk.  agg: [B][nch][2][D].
template <typename TI>
__global__ void __launch_bounds__(1024)
    diag_chunk_agg(const TI* __restrict__ V, const float* __restrict__ z, float* __restrict__ agg, Geo g) {
  const int c = blockIdx.x, b = blockIdx.y;
  const int ch = 2 * threadIdx.x;
  const int zi = g.zs == 1 ? 0 : ch / g.C;
  const int t0 = c * LC, n = min(LC, g.L - t0);
  const TI* vp = V + ((size_t)b * g.L + t0) * g.D + ch;
  const float* zp = z + ((size_t)b * g.L + t0) * g.zs + zi;
  float h0 = 0.f, h1 = 0.f, P = 1.f;
  int t = 0;
  for (; t + 8 <= n; t += 8) {
    float2 v[8];
    float zz[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      v[u] = ld2(vp + (size_t)(t + u) * g.D);
      zz[u] = __ldg(zp + (size_t)(t + u) * g.zs);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float a = decay_of(zz[u], g.damping);
      h0 = __fadd_rn(__fmul_rn(a, h0), gated_value<TI>(v[u].x, zz[u]));
      h1 = __fadd_rn(__fmul_rn(a, h1), gated_value<TI>(v[u].y, zz[u]));
      P *= a;
    }
  }
  for (; t < n; ++t) {
    const float2 v = ld2(vp + (size_t)t * g.D);
    const float zz = __ldg(zp + (size_t)t * g.zs);
    const float a = decay_of(zz, g.damping);
    h0 = __fadd_rn(__fmul_rn(a, h0), gated_value<TI>(v.x, zz));
    h1 = __fadd_rn(__fmul_rn(a, h1), gated_value<TI>(v.y, zz));
    P *= a;
  }
  float* dst = agg + ((size_t)b * g.nch + c) * 2 * g.D;
  *reinterpret_cast<float2*>(dst + ch) = make_float2(P, P);
  *reinterpret_cast<float2*>(dst + g.D + ch) = make_float2(h0, h1);
}

// Kernel 2: carries entering every chunk, per channel.  carry: [B][nch][D];
// H0 / H_final: [B][D] or null.
__global__ void __launch_bounds__(256)
    diag_carry(const float* __restrict__ agg, const float* __restrict__ H0, float* __restrict__ carry,
               float* __restrict__ H_final, Geo g) {
  const int b = blockIdx.y;
  const int ch = blockIdx.x * 256 + threadIdx.x;
  if (ch >= g.D) return;
  float h = H0 ? H0[(size_t)b * g.D + ch] : 0.f;
  const float* ap = agg + (size_t)b * g.nch * 2 * g.D + ch;
  float* cp = carry + (size_t)b * g.nch * g.D + ch;
  int c = 0;
  for (; c + 4 <= g.nch; c += 4) {
    float P[4], Hl[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      P[u] = __ldcg(ap + (size_t)(c + u) * 2 * g.D);
      Hl[u] = __ldcg(ap + (size_t)(c + u) * 2 * g.D + g.D);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      cp[(size_t)(c + u) * g.D] = h;
      h = __fadd_rn(__fmul_rn(P[u], h), Hl[u]);
    }
  }
  for (; c < g.nch; ++c) {
    cp[(size_t)c * g.D] = h;
    h = __fadd_rn(__fmul_rn(__ldcg(ap + (size_t)c * 2 * g.D), h), __ldcg(ap + (size_t)c * 2 * g.D + g.D));
  }
  if (H_final) H_final[(size_t)b * g.D + ch] = h;
}

// Kernel 3: re-scan from the carry, RMSNorm per token, outputs.
// Shared memory: red[2][G][32] partial sums of squares (one per warp).
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024)
    diag_apply_norm(const TI* __restrict__ V, const float* __restrict__ z, const float* __restrict__ carry,
                    const float* __restrict__ w, TO* __restrict__ y, float eps, Geo g) {
  __shared__ float red[2][G][32];
  const int c = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nw = blockDim.x >> 5;
  const int ch = 2 * tid;
  const int zi = g.zs == 1 ? 0 : ch / g.C;
  const int t0 = c * LC, n = min(LC, g.L - t0);
  const TI* vp = V + ((size_t)b * g.L + t0) * g.D + ch;
  const float* zp = z + ((size_t)b * g.L + t0) * g.zs + zi;
  TO* yp = y + ((size_t)b * g.L + t0) * g.D + ch;
  const float2 cw = *reinterpret_cast<const float2*>(w + ch);
  const float2 cin = *reinterpret_cast<const float2*>(carry + ((size_t)b * g.nch + c) * g.D + ch);
  float h0 = cin.x, h1 = cin.y;
  const float inv_d = 1.f / (float)g.D;
  int buf = 0;
  for (int tg = 0; tg < n; tg += G) {
    float2 v[G];
    float zz[G];
#pragma unroll
    for (int u = 0; u < G; ++u) {
      if (tg + u < n) {
        v[u] = ld2(vp + (size_t)(tg + u) * g.D);
        zz[u] = __ldg(zp + (size_t)(tg + u) * g.zs);
      } else {
        v[u] = make_float2(0.f, 0.f);
        zz[u] = 1.f;
      }
    }
    float hx[G], hy[G];
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const float a = decay_of(zz[u], g.damping);
      h0 = __fadd_rn(__fmul_rn(a, h0), gated_value<TI>(v[u].x, zz[u]));
      h1 = __fadd_rn(__fmul_rn(a, h1), gated_value<TI>(v[u].y, zz[u]));
      hx[u] = h0;
      hy[u] = h1;
      float s = fmaf(h0, h0, h1 * h1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) red[buf][u][warp] = s;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < G; ++u) {
      if (tg + u >= n) break;
      float s = 0.f;
      for (int ww = 0; ww < nw; ++ww) s += red[buf][u][ww];
      const float rs = rsqrtf(s * inv_d + eps);
      st2<TO>(yp + (size_t)(tg + u) * g.D, __fmul_rn(__fmul_rn(hx[u], rs), cw.x),
              __fmul_rn(__fmul_rn(hy[u], rs), cw.y));
    }
    buf ^= 1;  // the other buffer is written next; this one is read again two groups later
  }
}

template <typename TI, typename TO>
int run(const void* V, const float* z, const float* H0, const float* w, float eps, void* y, float* H_final,
        const Geo& g, int B, float* agg, float* carry, cudaStream_t s) {
  const int nt = g.D / 2;
  const dim3 grid(g.nch, B);
  diag_chunk_agg<TI><<<grid, nt, 0, s>>>(static_cast<const TI*>(V), z, agg, g);
  int rc = mogt_host::launch_status();
  if (rc != MOGT_OK) return rc;
  diag_carry<<<dim3((g.D + 255) / 256, B), 256, 0, s>>>(agg, H0, carry, H_final, g);
  if ((rc = mogt_host::launch_status()) != MOGT_OK) return rc;
  diag_apply_norm<TI, TO><<<grid, nt, 0, s>>>(static_cast<const TI*>(V), z, carry, w,
                                              static_cast<TO*>(y), eps, g);
  return mogt_host::launch_status();
}

}  // namespace diag
}  // namespace mogt

extern "C" size_t mogt_diag_scan_norm_scratch_bytes(int64_t B, int64_t L, int64_t R, int64_t C) {
  if (B <= 0 || L <= 0 || R <= 0 || C <= 0) return 0;
  const int64_t nch = (L + mogt::diag::LC - 1) / mogt::diag::LC;
  return (size_t)B * nch * R * C * 3 * sizeof(float);  // aggregates (P, h) and carries
}

extern "C" int mogt_diag_scan_norm_fwd(const void* V, const float* z, int64_t z_per_token,
                                       float damping, const float* H0, const float* norm_weight,
                                       float eps, void* y, float* H_final, int64_t B, int64_t L,
                                       int64_t R, int64_t C, int in_dtype, int out_dtype,
                                       void* scratch, size_t scratch_bytes, void* stream) {
  using namespace mogt::diag;
  if (B <= 0 || L < 0 || R <= 0 || C <= 0) return MOGT_ERR_SHAPE;
  if (z_per_token != 1 && z_per_token != R) return MOGT_ERR_SHAPE;
  if (L == 0) return MOGT_OK;
  if (!V || !z || !norm_weight || !y || !scratch) return MOGT_ERR_ARG;
  const int64_t D = R * C;
  // two channels of one row per thread, whole warps, one CTA per chunk
  if (C % 2 != 0 || D % 64 != 0 || D > 2048) return MOGT_ERR_UNSUPPORTED;
  if (B > 65535 || L >= ((int64_t)1 << 31) || B * L * D >= ((int64_t)1 << 62)) return MOGT_ERR_UNSUPPORTED;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(y) |
                        reinterpret_cast<uintptr_t>(norm_weight) | reinterpret_cast<uintptr_t>(scratch) |
                        (H0 ? reinterpret_cast<uintptr_t>(H0) : 0);
  if (mis & 7u) return MOGT_ERR_ALIGN;
  if (scratch_bytes < mogt_diag_scan_norm_scratch_bytes(B, L, R, C)) return MOGT_ERR_WORKSPACE;
  Geo g;
  g.L = (int)L;
  g.D = (int)D;
  g.C = (int)C;
  g.zs = (int)z_per_token;
  g.nch = (int)((L + LC - 1) / LC);
  g.damping = damping;
  float* agg = static_cast<float*>(scratch);
  float* carry = agg + (size_t)B * g.nch * 2 * D;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using bf = __nv_bfloat16;
  const int bi = (int)B;
  if (in_dtype == MOGT_DTYPE_BF16 && out_dtype == MOGT_DTYPE_BF16)
    return run<bf, bf>(V, z, H0, norm_weight, eps, y, H_final, g, bi, agg, carry, s);
  if (in_dtype == MOGT_DTYPE_BF16 && out_dtype == MOGT_DTYPE_F32)
    return run<bf, float>(V, z, H0, norm_weight, eps, y, H_final, g, bi, agg, carry, s);
  if (in_dtype == MOGT_DTYPE_F32 && out_dtype == MOGT_DTYPE_BF16)
    return run<float, bf>(V, z, H0, norm_weight, eps, y, H_final, g, bi, agg, carry, s);
  if (in_dtype == MOGT_DTYPE_F32 && out_dtype == MOGT_DTYPE_F32)
    return run<float, float>(V, z, H0, norm_weight, eps, y, H_final, g, bi, agg, carry, s);
  return MOGT_ERR_DTYPE;
}
