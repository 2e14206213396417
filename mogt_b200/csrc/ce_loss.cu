// Row-wise softmax cross-entropy on a chunk of fp32 logits, the part of the
// reference's chunked linear cross-entropy (chunked_lm_loss.py:5-80) that is
// not a GEMM.  One CTA per row, the row read once per direction:
//   forward   online max / sum of exp in one pass  ->  lse_i, and
//             loss_i = lse_i - x_i[label_i]  (0 for label -100, which
//             F.cross_entropy ignores by default)
//   backward  in place: x_ij <- (exp(x_ij - lse_i) - [j == label_i']) * scale
//             with label' = label, or label + V for a negative label -- the
//             reference's probs[arange, labels] -= 1 indexes from the end
//             for the ignored label -100 (chunked_lm_loss.py:61).
#include "common.cuh"

namespace mogt {
namespace ce {

constexpr int NT = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
  m = mn;
}

__global__ void __launch_bounds__(NT) ce_fwd_kernel(const float* __restrict__ logits,
                                                    const int64_t* __restrict__ labels, int64_t V,
                                                    float* __restrict__ lse_out, float* __restrict__ loss) {
  __shared__ float sm_m[NT / 32], sm_s[NT / 32];
  const int64_t row = blockIdx.x;
  const float* x = logits + row * V;
  float m = -INFINITY, s = 0.f;
  const bool vec = (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int64_t i = threadIdx.x; i < V / 4; i += NT) {
      const float4 v = __ldcs(x4 + i);
      const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      const float mn = fmaxf(m, mx);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + __expf(v.x - mn) + __expf(v.y - mn) +
          __expf(v.z - mn) + __expf(v.w - mn);
      m = mn;
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += NT) {
      const float v = x[i];
      const float mn = fmaxf(m, v);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + __expf(v - mn);
      m = mn;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[w] = m;
    sm_s[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = lane < NT / 32 ? sm_m[lane] : -INFINITY;
    s = lane < NT / 32 ? sm_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float lse = m + logf(s);
      lse_out[row] = lse;
      const int64_t lab = labels[row];
      loss[row] = (lab == -100) ? 0.f : lse - x[lab];
    }
  }
}

__global__ void __launch_bounds__(NT) ce_bwd_kernel(float* __restrict__ logits,
                                                    const int64_t* __restrict__ labels,
                                                    const float* __restrict__ lse_in, int64_t V,
                                                    float scale) {
  const int64_t row = blockIdx.x;
  float* x = logits + row * V;
  const float lse = lse_in[row];
  int64_t lab = labels[row];
  if (lab < 0) lab += V;
  const bool vec = (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
  if (vec) {
    float4* x4 = reinterpret_cast<float4*>(x);
    for (int64_t i = threadIdx.x; i < V / 4; i += NT) {
      float4 v = __ldcs(x4 + i);
      const int64_t j = 4 * i;
      v.x = (__expf(v.x - lse) - (j == lab ? 1.f : 0.f)) * scale;
      v.y = (__expf(v.y - lse) - (j + 1 == lab ? 1.f : 0.f)) * scale;
      v.z = (__expf(v.z - lse) - (j + 2 == lab ? 1.f : 0.f)) * scale;
      v.w = (__expf(v.w - lse) - (j + 3 == lab ? 1.f : 0.f)) * scale;
      __stcs(x4 + i, v);
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += NT) x[i] = (__expf(x[i] - lse) - (i == lab ? 1.f : 0.f)) * scale;
  }
}

}  // namespace ce
}  // namespace mogt

extern "C" int mogt_ce_rows_fwd(const float* logits, const int64_t* labels, int64_t rows, int64_t V,
                                float* lse, float* loss, void* stream) {
  if (rows < 0 || V <= 0) return MOGT_ERR_SHAPE;
  if (rows == 0) return MOGT_OK;
  if (!logits || !labels || !lse || !loss) return MOGT_ERR_ARG;
  if (rows >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  mogt::ce::ce_fwd_kernel<<<(unsigned)rows, mogt::ce::NT, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, labels, V, lse, loss);
  return mogt_host::launch_status();
}

extern "C" int mogt_ce_rows_bwd(float* logits, const int64_t* labels, const float* lse, int64_t rows,
                                int64_t V, float scale, void* stream) {
  if (rows < 0 || V <= 0) return MOGT_ERR_SHAPE;
  if (rows == 0) return MOGT_OK;
  if (!logits || !labels || !lse) return MOGT_ERR_ARG;
  if (rows >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  mogt::ce::ce_bwd_kernel<<<(unsigned)rows, mogt::ce::NT, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, labels, lse, V, scale);
  return mogt_host::launch_status();
}
