// Connection map of the MOGT block (model_mogt.py:79-102, _build_transport):
// per token, a skew-symmetric A = (M - M^T) * scale (M = the phi_conn output
// reshaped N x N, scale = 1 / r) is mapped to the transport
//     U = damping * expm(A)                               (matrix_exp)
//     U = damping * (I - A/2)^{-1} (I + A/2)              (cayley)
// in fp32, written in the output dtype.  The reference evaluates these with
// torch.matrix_exp / torch.linalg.solve on [B, L, 16, 16] batches.
//
// One warp per matrix: lane l owns row l / (32 / N) ... see `Lay` below;
// operands live in the warp's shared-memory tiles and products are plain
// fp32 FMAs.  expm: A is scaled by 2^-s so that its 1-norm is at most 1/2,
// a degree-12 Taylor polynomial is evaluated by Horner's rule (truncation
// error below 2^-40 at that norm), and the result is squared s times (the
// scaling-and-squaring method).  cayley: Gauss-Jordan elimination on
// [I - A/2 | I + A/2] without pivoting, which is safe because I - A/2 with A
// skew-symmetric has every eigenvalue on the line Re = 1.
// `skew` = 0 takes A as given (no antisymmetrisation, no scale): the
// backward evaluates expm of a 2N x 2N block matrix this way.
#include "common.cuh"

namespace mogt {
namespace conn {

constexpr int WARPS = 8;

template <int N>
struct Lay {
  static constexpr int RPL = N >= 32 ? N / 32 : 1;   // rows per lane
  static constexpr int LPR = N >= 32 ? 1 : 32 / N;   // lanes per row
  static constexpr int CPL = N / LPR;                // columns per lane (per row)
};

// C = A B for the warp's N x N tiles (row-major, pitch N); lane-parallel.
template <int N>
__device__ __forceinline__ void matmul(float* C, const float* A, const float* B, int lane) {
  using Ly = Lay<N>;
  float acc[Ly::RPL][Ly::CPL];
#pragma unroll
  for (int i = 0; i < Ly::RPL; ++i) {
    const int r = (lane / Ly::LPR) * Ly::RPL + i;
    const int c0 = (lane % Ly::LPR) * Ly::CPL;
#pragma unroll
    for (int j = 0; j < Ly::CPL; ++j) acc[i][j] = 0.f;
#pragma unroll 4
    for (int k = 0; k < N; ++k) {
      const float a = A[r * N + k];
#pragma unroll
      for (int j = 0; j < Ly::CPL; ++j) acc[i][j] = fmaf(a, B[k * N + c0 + j], acc[i][j]);
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < Ly::RPL; ++i) {
    const int r = (lane / Ly::LPR) * Ly::RPL + i;
    const int c0 = (lane % Ly::LPR) * Ly::CPL;
#pragma unroll
    for (int j = 0; j < Ly::CPL; ++j) C[r * N + c0 + j] = acc[i][j];
  }
  __syncwarp();
}

template <int N, typename TI, typename TO>
__global__ void __launch_bounds__(WARPS * 32)
    connection_kernel(const TI* __restrict__ M, TO* __restrict__ U, int64_t count, int mode, int skew,
                      float scale, float damping) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* A = sm + warp * 3 * N * N;  // the (scaled) generator; elimination factors (cayley)
  float* X = A + N * N;              // running result
  float* Y = X + N * N;              // scratch
  const int64_t step = (int64_t)gridDim.x * WARPS;
  for (int64_t m = (int64_t)blockIdx.x * WARPS + warp; m < count; m += step) {
    const TI* src = M + m * N * N;
    // generator: A = (M - M^T) * scale, or M itself
    for (int e = lane; e < N * N; e += 32) {
      const int r = e / N, c = e % N;
      // the difference is rounded to the input dtype, as M - M^T is formed
      // in that dtype before the fp32 map (model_mogt.py:132-133, 80)
      A[e] = skew ? to_f32(from_f32<TI>(to_f32(src[e]) - to_f32(src[c * N + r]))) * scale : to_f32(src[e]);
    }
    __syncwarp();
    if (mode == 0) {
      // ||A||_1 (max column sum) -> s with ||A / 2^s||_1 <= 1/2
      float colsum = 0.f;
      for (int c = lane; c < N; c += 32) {
        float t = 0.f;
        for (int r = 0; r < N; ++r) t += fabsf(A[r * N + c]);
        colsum = fmaxf(colsum, t);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) colsum = fmaxf(colsum, __shfl_xor_sync(0xffffffffu, colsum, o));
      int s = 0;
      float nrm = colsum;
      while (nrm > 0.5f && s < 60) {
        nrm *= 0.5f;
        ++s;
      }
      const float sc = ldexpf(1.f, -s);
      for (int e = lane; e < N * N; e += 32) A[e] *= sc;
      // Horner: X = I + A/1 (I + A/2 (I + ... (I + A/12)))
      for (int e = lane; e < N * N; e += 32) X[e] = (e / N == e % N) ? 1.f : 0.f;
      __syncwarp();
      for (int k = 12; k >= 1; --k) {
        matmul<N>(Y, A, X, lane);  // Y = A X
        const float inv = 1.f / (float)k;
        for (int e = lane; e < N * N; e += 32) X[e] = ((e / N == e % N) ? 1.f : 0.f) + Y[e] * inv;
        __syncwarp();
      }
      for (int i = 0; i < s; ++i) {
        matmul<N>(Y, X, X, lane);
        for (int e = lane; e < N * N; e += 32) X[e] = Y[e];
        __syncwarp();
      }
    } else {
      // Gauss-Jordan on [Y | X] = [I - A/2 | I + A/2]: X <- Y^{-1} X
      for (int e = lane; e < N * N; e += 32) {
        const float d = (e / N == e % N) ? 1.f : 0.f, h = 0.5f * A[e];
        Y[e] = d - h;
        X[e] = d + h;
      }
      __syncwarp();
      for (int p = 0; p < N; ++p) {
        const float inv = 1.f / Y[p * N + p];
        __syncwarp();
        for (int c = lane; c < N; c += 32) {  // scale the pivot row
          Y[p * N + c] *= inv;
          X[p * N + c] *= inv;
        }
        __syncwarp();
        for (int r = lane; r < N; r += 32) A[r] = Y[r * N + p];  // elimination factors
        __syncwarp();
        for (int e = lane; e < N * N; e += 32) {  // eliminate column p from the other rows
          const int r = e / N, c = e % N;
          if (r != p) {
            Y[e] -= A[r] * Y[p * N + c];
            X[e] -= A[r] * X[p * N + c];
          }
        }
        __syncwarp();
      }
    }
    TO* dst = U + m * N * N;
    for (int e = lane; e < N * N; e += 32) dst[e] = from_f32<TO>(X[e] * damping);
    __syncwarp();
  }
}

template <int N, typename TI, typename TO>
int launch(const void* M, void* U, int64_t count, int mode, int skew, float scale, float damping,
           cudaStream_t s) {
  const size_t smem = (size_t)WARPS * 3 * N * N * 4;
  auto k = connection_kernel<N, TI, TO>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (count + WARPS - 1) / WARPS;
  const unsigned grid = (unsigned)(want < (int64_t)nsm * 8 ? want : (int64_t)nsm * 8);
  k<<<grid, WARPS * 32, smem, s>>>(static_cast<const TI*>(M), static_cast<TO*>(U), count, mode, skew,
                                   scale, damping);
  return mogt_host::launch_status();
}

template <int N>
int dispatch(const void* M, void* U, int64_t count, int mode, int skew, float scale, float damping,
             int in_dt, int out_dt, cudaStream_t s) {
  using bf = __nv_bfloat16;
  if (in_dt == MOGT_DTYPE_F32 && out_dt == MOGT_DTYPE_F32)
    return launch<N, float, float>(M, U, count, mode, skew, scale, damping, s);
  if (in_dt == MOGT_DTYPE_BF16 && out_dt == MOGT_DTYPE_F32)
    return launch<N, bf, float>(M, U, count, mode, skew, scale, damping, s);
  if (in_dt == MOGT_DTYPE_BF16 && out_dt == MOGT_DTYPE_BF16)
    return launch<N, bf, bf>(M, U, count, mode, skew, scale, damping, s);
  if (in_dt == MOGT_DTYPE_F32 && out_dt == MOGT_DTYPE_BF16)
    return launch<N, float, bf>(M, U, count, mode, skew, scale, damping, s);
  return MOGT_ERR_DTYPE;
}

}  // namespace conn
}  // namespace mogt

extern "C" int mogt_connection_map(const void* M, void* U, int64_t count, int64_t n, int mode, int skew,
                                   float scale, float damping, int in_dtype, int out_dtype, void* stream) {
  if (count < 0 || n <= 0) return MOGT_ERR_SHAPE;
  if (count == 0) return MOGT_OK;
  if (!M || !U) return MOGT_ERR_ARG;
  if (mode != MOGT_CONN_EXPM && mode != MOGT_CONN_CAYLEY) return MOGT_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (n) {
    case 8: return mogt::conn::dispatch<8>(M, U, count, mode, skew, scale, damping, in_dtype, out_dtype, s);
    case 16: return mogt::conn::dispatch<16>(M, U, count, mode, skew, scale, damping, in_dtype, out_dtype, s);
    case 32: return mogt::conn::dispatch<32>(M, U, count, mode, skew, scale, damping, in_dtype, out_dtype, s);
    default: return MOGT_ERR_UNSUPPORTED;
  }
}
