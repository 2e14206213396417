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
// Three kernels, chunks of `lc` tokens (64 for bf16 V at D = 768), one CTA
// per (chunk, batch row), two channels per thread.  Kernels 1 and 3 bring the
// chunk's V rows (one contiguous block) into shared memory with four bulk
// copies, one mbarrier each, so that the whole chunk is in flight at once and
// the scan starts on the first quarter while the rest lands:
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

constexpr int NPIECE = 4;         // bulk copies (and mbarriers) per chunk
constexpr int G = 16;             // tokens per normalisation group in kernel 3
constexpr int kTileBudget = 100 * 1024;  // V tile bytes per CTA (two CTAs per SM)

// tokens per chunk for D channels of `elt` bytes: 64, halved while the V tile
// exceeds the budget (at least 8)
inline int chunk_len(int64_t D, int elt) {
  int lc = 64;
  while (lc > 8 && (int64_t)lc * D * elt > kTileBudget) lc /= 2;
  return lc;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <typename T>
__device__ __forceinline__ float2 ld2(const T* p);
template <>
__device__ __forceinline__ float2 ld2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 ld2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
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
  int L, D, C, zs, nch, lc;  // zs: gates per token (R, or 1 for one scalar gate)
  float damping;
  WsHeader* hdr;
};

// Shared-memory chunk of V ([lc][D], input dtype) and z ([lc][zs] fp32),
// followed by NPIECE mbarriers.
template <typename TI>
struct ChunkTile {
  TI* v;
  float* z;
  uint64_t* bars;
  __device__ ChunkTile(uint8_t* smem, const Geo& g) {
    v = reinterpret_cast<TI*>(smem);
    z = reinterpret_cast<float*>(smem + (size_t)g.lc * g.D * sizeof(TI));
    bars = reinterpret_cast<uint64_t*>(z + ((g.lc * g.zs + 1) & ~1));
  }
};
template <typename TI>
inline size_t tile_smem_bytes(int lc, int D, int zs) {
  return (size_t)lc * D * sizeof(TI) + (size_t)((lc * zs + 1) & ~1) * 4 + 8 * NPIECE;
}

// Issue the chunk's V copies (thread 0) and load its gates (all threads);
// ends with a CTA barrier.  Tokens [t0, t0 + n) of batch row b.
template <typename TI>
__device__ __forceinline__ void load_chunk(const ChunkTile<TI>& tile, const TI* V, const float* z,
                                           const Geo& g, int b, int t0, int n) {
  const int pc = g.lc / NPIECE;
  if (threadIdx.x == 0) {
    for (int p = 0; p < NPIECE; ++p) mbar_init(&tile.bars[p], 1);
    fence_barrier_init();
    for (int p = 0; p < NPIECE; ++p) {
      const int a = p * pc, e = min(n, a + pc);
      if (a >= e) break;
      const uint32_t bytes = (uint32_t)((e - a) * g.D * sizeof(TI));
      mbar_arrive_expect_tx(&tile.bars[p], bytes);
      bulk_g2s(tile.v + (size_t)a * g.D, V + ((size_t)b * g.L + t0 + a) * g.D, bytes, &tile.bars[p]);
    }
  }
  const float* zg = z + ((size_t)b * g.L + t0) * g.zs;
  for (int e = threadIdx.x; e < n * g.zs; e += blockDim.x) tile.z[e] = __ldg(zg + e);
  __syncthreads();
}

__device__ __forceinline__ float decay_of(float z, float damping) {
  const float omz = 1.f - z;
  return damping == 1.f ? omz : damping * omz;
}

// Wait for piece p of the chunk (bounded); false after a timeout.
template <typename TI>
__device__ __forceinline__ bool wait_piece(const ChunkTile<TI>& tile, int p) {
  return mbar_wait(&tile.bars[p], 0);
}

// Kernel 1: P_c and the local end state of every chunk.  agg: [B][nch][2][D].
template <typename TI>
__global__ void __launch_bounds__(1024)
    diag_chunk_agg(const TI* __restrict__ V, const float* __restrict__ z, float* __restrict__ agg, Geo g) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const ChunkTile<TI> tile(smem_raw, g);
  const int c = blockIdx.x, b = blockIdx.y;
  const int ch = 2 * threadIdx.x;
  const int zi = g.zs == 1 ? 0 : ch / g.C;
  const int t0 = c * g.lc, n = min(g.lc, g.L - t0);
  load_chunk(tile, V, z, g, b, t0, n);
  const int pc = g.lc / NPIECE;
  float h0 = 0.f, h1 = 0.f, P = 1.f;
  bool ok = true;
  for (int p = 0; p * pc < n; ++p) {
    if (!wait_piece(tile, p)) ok = false;
    const int e = min(n, (p + 1) * pc);
#pragma unroll 4
    for (int t = p * pc; t < e; ++t) {
      const float2 v = ld2(tile.v + (size_t)t * g.D + ch);
      const float zz = tile.z[t * g.zs + zi];
      const float a = decay_of(zz, g.damping);
      h0 = __fadd_rn(__fmul_rn(a, h0), gated_value<TI>(v.x, zz));
      h1 = __fadd_rn(__fmul_rn(a, h1), gated_value<TI>(v.y, zz));
      P *= a;
    }
  }
  float* dst = agg + ((size_t)b * g.nch + c) * 2 * g.D;
  *reinterpret_cast<float2*>(dst + ch) = make_float2(P, P);
  *reinterpret_cast<float2*>(dst + g.D + ch) = make_float2(h0, h1);
  if (!ok) record_error(g.hdr, MOGT_ERR_TIMEOUT, (uint32_t)(b * g.nch + c));
}

// Kernel 2: carries entering every chunk, per channel.  carry: [B][nch][D];
// H0 / H_final: [B][D] or null.  The loads run 16 chunks ahead of the
// dependent multiply-add chain.
constexpr int CPF = 16;
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
  for (; c + CPF <= g.nch; c += CPF) {
    float P[CPF], Hl[CPF];
#pragma unroll
    for (int u = 0; u < CPF; ++u) {
      P[u] = __ldcg(ap + (size_t)(c + u) * 2 * g.D);
      Hl[u] = __ldcg(ap + (size_t)(c + u) * 2 * g.D + g.D);
    }
#pragma unroll
    for (int u = 0; u < CPF; ++u) {
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

// Sum over the warp of G = 16 per-lane values at once: each halving step
// keeps half of the values (the half selected by one lane bit) and adds the
// partner lane's copy of them, so 8 + 4 + 2 + 1 shuffles leave lane l with the
// partial sum of value (l >> 1) & 15 over pairs of lanes; one more shuffle
// completes it.  Returns the warp sum of value (lane >> 1).
__device__ __forceinline__ float warp_sum16(float (&x)[G], int lane) {
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int half = 8 >> step, off = 16 >> step;
    const bool hi = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float send = hi ? x[j] : x[j + half];
      const float keep = hi ? x[j + half] : x[j];
      x[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return x[0] + __shfl_xor_sync(0xffffffffu, x[0], 1);
}

// Kernel 3: re-scan from the carry, RMSNorm per token, outputs.
// red[G][32]: per-warp partial sums of squares; rsc[G]: the tokens' scales.
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024)
    diag_apply_norm(const TI* __restrict__ V, const float* __restrict__ z, const float* __restrict__ carry,
                    const float* __restrict__ w, TO* __restrict__ y, float eps, Geo g) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const ChunkTile<TI> tile(smem_raw, g);
  __shared__ float red[G][32];
  __shared__ float rsc[G];
  const int c = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nw = blockDim.x >> 5;
  const int ch = 2 * tid;
  const int zi = g.zs == 1 ? 0 : ch / g.C;
  const int t0 = c * g.lc, n = min(g.lc, g.L - t0);
  load_chunk(tile, V, z, g, b, t0, n);
  TO* yp = y + ((size_t)b * g.L + t0) * g.D + ch;
  const float2 cw = *reinterpret_cast<const float2*>(w + ch);
  const float2 cin = *reinterpret_cast<const float2*>(carry + ((size_t)b * g.nch + c) * g.D + ch);
  float h0 = cin.x, h1 = cin.y;
  const float inv_d = 1.f / (float)g.D;
  const int pc = g.lc / NPIECE;
  int piece = 0;
  bool ok = true;
  for (int tg = 0; tg < n; tg += G) {
    for (; piece < NPIECE && piece * pc < min(n, tg + G); ++piece)  // the pieces this group reads
      if (!wait_piece(tile, piece)) ok = false;
    float hx[G], hy[G], sq[G];
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const int t = min(tg + u, n - 1);  // tokens past the end repeat the last one, not written
      const float2 v = ld2(tile.v + (size_t)t * g.D + ch);
      const float zz = tile.z[t * g.zs + zi];
      const float a = decay_of(zz, g.damping);
      h0 = __fadd_rn(__fmul_rn(a, h0), gated_value<TI>(v.x, zz));
      h1 = __fadd_rn(__fmul_rn(a, h1), gated_value<TI>(v.y, zz));
      hx[u] = h0;
      hy[u] = h1;
      sq[u] = fmaf(h0, h0, h1 * h1);
    }
    const float ws = warp_sum16(sq, lane);
    if ((lane & 1) == 0) red[lane >> 1][warp] = ws;
    __syncthreads();
    for (int u = warp; u < G; u += nw) {  // warp w: the scales of tokens w, w + nw, ...
      float s = lane < nw ? red[u][lane] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) rsc[u] = rsqrtf(s * inv_d + eps);
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < G; ++u) {
      if (tg + u >= n) break;
      const float rs = rsc[u];
      st2<TO>(yp + (size_t)(tg + u) * g.D, __fmul_rn(__fmul_rn(hx[u], rs), cw.x),
              __fmul_rn(__fmul_rn(hy[u], rs), cw.y));
    }
    // red and rsc are written again only after every thread has passed the
    // next group's first barrier, i.e. after these reads
  }
  if (!ok) record_error(g.hdr, MOGT_ERR_TIMEOUT, (uint32_t)(b * g.nch + c));
}

template <typename TI, typename TO>
int run(const void* V, const float* z, const float* H0, const float* w, float eps, void* y, float* H_final,
        const Geo& g, int B, float* agg, float* carry, cudaStream_t s) {
  const int nt = g.D / 2;
  const dim3 grid(g.nch, B);
  const size_t smem = tile_smem_bytes<TI>(g.lc, g.D, g.zs);
  auto k1 = diag_chunk_agg<TI>;
  auto k3 = diag_apply_norm<TI, TO>;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  k1<<<grid, nt, smem, s>>>(static_cast<const TI*>(V), z, agg, g);
  int rc = mogt_host::launch_status();
  if (rc != MOGT_OK) return rc;
  diag_carry<<<dim3((g.D + 255) / 256, B), 256, 0, s>>>(agg, H0, carry, H_final, g);
  if ((rc = mogt_host::launch_status()) != MOGT_OK) return rc;
  k3<<<grid, nt, smem, s>>>(static_cast<const TI*>(V), z, carry, w, static_cast<TO*>(y), eps, g);
  return mogt_host::launch_status();
}

inline int elt_size(int dt) { return dt == MOGT_DTYPE_F32 ? 4 : 2; }

// the forward's chunk length, for the backward (diag_bwd.cu), which reads the
// forward's per-chunk carries
int forward_chunk_len(int64_t D, int in_dtype) { return chunk_len(D, elt_size(in_dtype)); }

}  // namespace diag
}  // namespace mogt

extern "C" size_t mogt_diag_scan_norm_scratch_bytes(int64_t B, int64_t L, int64_t R, int64_t C, int in_dtype) {
  using namespace mogt::diag;
  if (B <= 0 || L <= 0 || R <= 0 || C <= 0) return 0;
  const int lc = chunk_len(R * C, elt_size(in_dtype));
  const int64_t nch = (L + lc - 1) / lc;
  return (size_t)B * nch * R * C * 3 * sizeof(float);  // aggregates (P, h) and carries
}

extern "C" int mogt_diag_scan_norm_fwd(const void* V, const float* z, int64_t z_per_token,
                                       float damping, const float* H0, const float* norm_weight,
                                       float eps, void* y, float* H_final, int64_t B, int64_t L,
                                       int64_t R, int64_t C, int in_dtype, int out_dtype,
                                       void* status, void* scratch, size_t scratch_bytes,
                                       void* stream) {
  using namespace mogt::diag;
  if (B <= 0 || L < 0 || R <= 0 || C <= 0) return MOGT_ERR_SHAPE;
  if (z_per_token != 1 && z_per_token != R) return MOGT_ERR_SHAPE;
  if (L == 0) return MOGT_OK;
  if (!V || !z || !norm_weight || !y || !scratch || !status) return MOGT_ERR_ARG;
  if (in_dtype != MOGT_DTYPE_BF16 && in_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  const int64_t D = R * C;
  // two channels of one row per thread, whole warps, one CTA per chunk
  if (C % 2 != 0 || D % 64 != 0 || D > 2048 || R > 64) return MOGT_ERR_UNSUPPORTED;
  if (B > 65535 || L >= ((int64_t)1 << 31) || B * L * D >= ((int64_t)1 << 62)) return MOGT_ERR_UNSUPPORTED;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(scratch);
  const uintptr_t mis8 = reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(norm_weight) |
                         (H0 ? reinterpret_cast<uintptr_t>(H0) : 0);
  if ((mis & 15u) || (mis8 & 7u)) return MOGT_ERR_ALIGN;
  if (scratch_bytes < mogt_diag_scan_norm_scratch_bytes(B, L, R, C, in_dtype)) return MOGT_ERR_WORKSPACE;
  Geo g;
  g.L = (int)L;
  g.D = (int)D;
  g.C = (int)C;
  g.zs = (int)z_per_token;
  g.lc = chunk_len(D, elt_size(in_dtype));
  g.nch = (int)((L + g.lc - 1) / g.lc);
  g.damping = damping;
  g.hdr = static_cast<mogt::WsHeader*>(status);
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
