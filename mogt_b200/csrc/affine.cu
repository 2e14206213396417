// Dense affine scan  H_t = U_t H_{t-1} + V_t  (U: [B,L,R,R], V: [B,L,R,C]).
//
// Reference semantics: affine_scan.py:14-62 (forward, optional prefix
// products P_t = U_t ... U_1) and affine_scan.py:65-124 (backward: the reverse
// scan Sigma_t = g_t + U_{t+1}^T Sigma_{t+1} and dU_t = Sigma_t H_{t-1}^T).
// This replaces triton_scan.py's local Triton kernel, its Python carry loop
// and its carry-apply matmul (triton_scan.py:55-148, 232-311) with one launch.
//
// Design (fp32 throughout, like the reference's tl.dot(allow_tf32=False)):
//   * work unit = LC consecutive steps of one batch row; units are taken in
//     order from an atomic ticket (decoupled look-back);
//   * one thread per COLUMN: C columns of H plus R columns of the running
//     transition product P.  A column evolves independently given U_t, so the
//     per-step update x <- U_t x (+ v) needs no cross-thread traffic: U_t is
//     read from shared memory as a broadcast, V_t is read coalesced from HBM;
//   * pass 1 runs the unit from (H=0, P=I) and publishes its aggregate (P_u,
//     H_u); the look-back composes predecessors into the state entering the
//     unit; pass 2 re-runs the unit from that state and writes H (and P).
//   * REV=true runs the backward's reverse scan in place: step tau reads
//     g at t = L-1-tau and U_{t+1}^T (transposed while staging).
#include "common.cuh"

namespace mogt {
namespace affine {

template <int R>
struct Cfg {
  static constexpr int LC = R <= 8 ? 64 : (R == 16 ? 32 : 16);
  // one thread per column: the per-thread column state grows with R, so the
  // block size cap shrinks to keep it in registers
  static constexpr int MAXT = R >= 32 ? 256 : 512;
};

struct Params {
  const void* U;
  const void* V;
  void* H;
  void* P;
  WsHeader* hdr;
  uint32_t* flags;
  float* agg;
  float* inc;
  int L, C, nunits;
};

inline void ws_offsets(size_t NU, int R, int C, size_t* flags, size_t* agg, size_t* inc,
                       size_t* total) {
  const size_t per = (size_t)R * (C + R) * 4;
  *flags = sizeof(WsHeader);
  *agg = *flags + mogt_host::align_up(NU * 4, 256);
  *inc = *agg + mogt_host::align_up(NU * per, 256);
  *total = *inc + mogt_host::align_up(NU * per, 256);
}

template <int R, bool REV, typename TU, typename TV, typename TO>
__global__ void __launch_bounds__(Cfg<R>::MAXT) affine_scan_kernel(const Params p) {
  constexpr int LC = Cfg<R>::LC;
  extern __shared__ float sm[];
  float* Us = sm;                 // [LC][R][R]
  float* Qs = Us + LC * R * R;    // [R][R] composite transition of the look-back
  float* Ps = Qs + R * R;         // [R][R] this unit's transition product
  volatile uint32_t* bc = reinterpret_cast<volatile uint32_t*>(Ps + R * R);

  const int tid = threadIdx.x, nthr = blockDim.x;
  const int C = p.C, NC = C + R, L = p.L;
  if (tid == 0) {
    uint32_t epoch;
    bc[0] = take_ticket(p.hdr, &epoch);
    bc[1] = epoch;
  }
  __syncthreads();
  const uint32_t unit = bc[0], epoch = bc[1];
  const int b = unit / p.nunits, u = unit % p.nunits;
  const int tau0 = u * LC;
  const int nsteps = min(LC, L - tau0);
  const TU* Ub = static_cast<const TU*>(p.U) + (size_t)b * L * R * R;
  const TV* Vb = static_cast<const TV*>(p.V) + (size_t)b * L * R * C;

  // ---- stage U (converted to fp32; transposed and shifted for REV) ----
  for (int e = tid; e < LC * R * R; e += nthr) {
    const int tl = e / (R * R), rk = e % (R * R), a = rk / R, c = rk % R;
    const int tau = tau0 + tl;
    float val;
    int r = a, k = c;
    if (!REV) {
      val = (tau < L) ? to_f32(Ub[(size_t)tau * R * R + rk]) : (a == c ? 1.f : 0.f);
    } else {
      const int tsrc = L - tau;  // U_{t+1} with t = L-1-tau
      val = (tau < L && tsrc < L) ? to_f32(Ub[(size_t)tsrc * R * R + rk]) : (a == c ? 1.f : 0.f);
      r = c;
      k = a;
    }
    Us[tl * R * R + r * R + k] = val;
  }
  __syncthreads();

  const int col = tid;
  const bool active = col < NC;
  const bool hcol = col < C;
  const int pj = col - C;  // P column index when !hcol
  TO* Hb = static_cast<TO*>(p.H) + (size_t)b * L * R * C;
  TO* Pb = p.P ? static_cast<TO*>(p.P) + (size_t)b * L * R * R : nullptr;
  const bool first = (u == 0);

  auto time_of = [&](int tau) { return REV ? (L - 1 - tau) : tau; };
  auto load_v = [&](int tau, float (&v)[R]) {
    const int t = time_of(tau);
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = to_f32(Vb[((size_t)t * R + r) * C + col]);
  };
  auto step = [&](int tl, float (&x)[R], const float (&v)[R]) {
    const float* Ut = Us + tl * R * R;
    float y[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float acc = 0.f;
      if constexpr (R % 4 == 0) {
#pragma unroll
        for (int k = 0; k < R; k += 4) {
          const float4 u4 = *reinterpret_cast<const float4*>(Ut + r * R + k);
          acc = fmaf(u4.x, x[k], acc);
          acc = fmaf(u4.y, x[k + 1], acc);
          acc = fmaf(u4.z, x[k + 2], acc);
          acc = fmaf(u4.w, x[k + 3], acc);
        }
      } else {
#pragma unroll
        for (int k = 0; k < R; ++k) acc = fmaf(Ut[r * R + k], x[k], acc);
      }
      y[r] = acc + v[r];
    }
#pragma unroll
    for (int r = 0; r < R; ++r) x[r] = y[r];
  };
  auto store = [&](int tau, const float (&x)[R]) {
    const int t = time_of(tau);
    if (hcol) {
#pragma unroll
      for (int r = 0; r < R; ++r) Hb[((size_t)t * R + r) * C + col] = from_f32<TO>(x[r]);
    } else if (Pb) {
#pragma unroll
      for (int r = 0; r < R; ++r) Pb[((size_t)t * R + r) * R + pj] = from_f32<TO>(x[r]);
    }
  };

  // ---- pass 1: unit from (H = 0, P = I) ----
  float x[R];
#pragma unroll
  for (int r = 0; r < R; ++r) x[r] = (!hcol && r == pj) ? 1.f : 0.f;
  if (active) {
    float v[R], vn[R];
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = 0.f;
    if (hcol && nsteps > 0) load_v(tau0, v);
    for (int tl = 0; tl < nsteps; ++tl) {
      if (hcol && tl + 1 < nsteps) load_v(tau0 + tl + 1, vn);
      step(tl, x, v);
      if (first) store(tau0 + tl, x);
      if (hcol) {
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = vn[r];
      }
    }
  }
  const bool has_succ = u + 1 < p.nunits;
  const size_t per = (size_t)R * NC;
  if (!first && has_succ && active) {
    float* dst = p.agg + unit * per;
#pragma unroll
    for (int r = 0; r < R; ++r) __stcg(dst + r * NC + col, x[r]);
  }
  if (!first && active && !hcol) {
#pragma unroll
    for (int r = 0; r < R; ++r) Ps[r * R + pj] = x[r];
  }
  if (!first && has_succ) {
    __threadfence();
    __syncthreads();
    if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagAgg));
  }

  if (first) {
    if (has_succ) {
      if (active) {
        float* dst = p.inc + unit * per;
#pragma unroll
        for (int r = 0; r < R; ++r) __stcg(dst + r * NC + col, x[r]);
      }
      __threadfence();
      __syncthreads();
      if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagInc));
    }
  } else {
    // ---- look-back: E = (Q, y) composed over predecessors ----
    for (int e = tid; e < R * R; e += nthr) Qs[e] = (e / R == e % R) ? 1.f : 0.f;
    float yv[R], E[R];
#pragma unroll
    for (int r = 0; r < R; ++r) yv[r] = 0.f;
    int m = (int)unit - 1;
    for (int it = 0;; ++it) {
      if (tid == 0) bc[2 + (it & 1)] = wait_flag(p.flags + m, epoch, p.hdr, unit);
      __syncthreads();
      const uint32_t st = bc[2 + (it & 1)];
      const bool inc = (st != kFlagAgg);
      const float* src = (inc ? p.inc : p.agg) + (size_t)m * per;
      float z[R];
      if (active) {
        float s[R];
#pragma unroll
        for (int r = 0; r < R; ++r) s[r] = __ldcg(src + r * NC + col);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < R; ++k) acc = fmaf(Qs[r * R + k], s[k], acc);
          z[r] = acc;
        }
      }
      if (inc) {
#pragma unroll
        for (int r = 0; r < R; ++r) E[r] = z[r] + yv[r];
        break;
      }
      if (hcol) {
#pragma unroll
        for (int r = 0; r < R; ++r) yv[r] += z[r];
      }
      __syncthreads();
      if (active && !hcol) {
#pragma unroll
        for (int r = 0; r < R; ++r) Qs[r * R + pj] = z[r];
      }
      __syncthreads();
      --m;
    }
    // inclusive = P_u E + (H columns: pass-1 result)
    if (has_succ) {
      if (active) {
        float* dst = p.inc + unit * per;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float acc = hcol ? x[r] : 0.f;
#pragma unroll
          for (int k = 0; k < R; ++k) acc = fmaf(Ps[r * R + k], E[k], acc);
          __stcg(dst + r * NC + col, acc);
        }
      }
      __threadfence();
      __syncthreads();
      if (tid == 0) st_release_u32(p.flags + unit, flag_tag(epoch, kFlagInc));
    }
    // ---- pass 2: re-run the unit from E and write outputs ----
    if (active && (hcol || Pb)) {
#pragma unroll
      for (int r = 0; r < R; ++r) x[r] = E[r];
      float v[R], vn[R];
#pragma unroll
      for (int r = 0; r < R; ++r) v[r] = 0.f;
      if (hcol && nsteps > 0) load_v(tau0, v);
      for (int tl = 0; tl < nsteps; ++tl) {
        if (hcol && tl + 1 < nsteps) load_v(tau0 + tl + 1, vn);
        step(tl, x, v);
        store(tau0 + tl, x);
        if (hcol) {
#pragma unroll
          for (int r = 0; r < R; ++r) v[r] = vn[r];
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) finish_cta(p.hdr, epoch, gridDim.x);
}

// dU_t = Sigma_t H_{t-1}^T   (affine_scan.py:117), fp32 inputs, one step per
// CTA iteration; thread (i, j) reduces over the C columns.
template <typename TO>
__global__ void __launch_bounds__(256) affine_grad_u_kernel(const float* __restrict__ sig,
                                                            const float* __restrict__ H,
                                                            TO* __restrict__ gU, int B, int L,
                                                            int R, int C) {
  extern __shared__ float sm[];
  float* ss = sm;          // [R][C]
  float* hs = sm + R * C;  // [R][C]
  const size_t nsteps = (size_t)B * L;
  for (size_t bt = blockIdx.x; bt < nsteps; bt += gridDim.x) {
    const int t = (int)(bt % L);
    const float* sp = sig + bt * R * C;
    const float* hp = H + (bt - 1) * R * C;
    __syncthreads();
    for (int e = threadIdx.x; e < R * C; e += blockDim.x) {
      ss[e] = sp[e];
      hs[e] = t > 0 ? hp[e] : 0.f;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < R * R; e += blockDim.x) {
      const int i = e / R, j = e % R;
      float acc = 0.f;
      for (int c = 0; c < C; ++c) acc = fmaf(ss[i * C + c], hs[j * C + c], acc);
      gU[bt * R * R + e] = from_f32<TO>(acc);
    }
  }
}

template <int R, bool REV, typename TU, typename TV, typename TO>
int launch(const Params& P, int B, cudaStream_t s) {
  constexpr int LC = Cfg<R>::LC;
  const int threads = ((P.C + R + 31) / 32) * 32;
  if (threads > Cfg<R>::MAXT) return MOGT_ERR_UNSUPPORTED;
  const size_t smem = (size_t)(LC * R * R + 2 * R * R) * 4 + 64;
  auto k = affine_scan_kernel<R, REV, TU, TV, TO>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  k<<<(unsigned)((size_t)B * P.nunits), threads, smem, s>>>(P);
  return mogt_host::launch_status();
}

template <int R, bool REV>
int dispatch_types(const Params& P, int B, int u_dt, int v_dt, int o_dt, cudaStream_t s) {
  using bf = __nv_bfloat16;
#define MOGT_AFF_CASE(UT, VT, OT, ut, vt, ot) \
  if (u_dt == ut && v_dt == vt && o_dt == ot) return launch<R, REV, UT, VT, OT>(P, B, s);
  MOGT_AFF_CASE(float, float, float, MOGT_DTYPE_F32, MOGT_DTYPE_F32, MOGT_DTYPE_F32)
  MOGT_AFF_CASE(float, bf, float, MOGT_DTYPE_F32, MOGT_DTYPE_BF16, MOGT_DTYPE_F32)
  MOGT_AFF_CASE(float, bf, bf, MOGT_DTYPE_F32, MOGT_DTYPE_BF16, MOGT_DTYPE_BF16)
  MOGT_AFF_CASE(float, float, bf, MOGT_DTYPE_F32, MOGT_DTYPE_F32, MOGT_DTYPE_BF16)
  MOGT_AFF_CASE(bf, bf, bf, MOGT_DTYPE_BF16, MOGT_DTYPE_BF16, MOGT_DTYPE_BF16)
  MOGT_AFF_CASE(bf, bf, float, MOGT_DTYPE_BF16, MOGT_DTYPE_BF16, MOGT_DTYPE_F32)
  MOGT_AFF_CASE(bf, float, float, MOGT_DTYPE_BF16, MOGT_DTYPE_F32, MOGT_DTYPE_F32)
#undef MOGT_AFF_CASE
  return MOGT_ERR_DTYPE;
}

template <bool REV>
int dispatch_r(int R, const Params& P, int B, int u_dt, int v_dt, int o_dt, cudaStream_t s) {
  switch (R) {
    case 2: return dispatch_types<2, REV>(P, B, u_dt, v_dt, o_dt, s);
    case 4: return dispatch_types<4, REV>(P, B, u_dt, v_dt, o_dt, s);
    case 8: return dispatch_types<8, REV>(P, B, u_dt, v_dt, o_dt, s);
    case 16: return dispatch_types<16, REV>(P, B, u_dt, v_dt, o_dt, s);
    case 32: return dispatch_types<32, REV>(P, B, u_dt, v_dt, o_dt, s);
    default: return MOGT_ERR_UNSUPPORTED;
  }
}

inline int lc_of(int R) {
  switch (R) {
    case 2: return Cfg<2>::LC;
    case 4: return Cfg<4>::LC;
    case 8: return Cfg<8>::LC;
    case 16: return Cfg<16>::LC;
    case 32: return Cfg<32>::LC;
    default: return 0;
  }
}

}  // namespace affine
}  // namespace mogt

using namespace mogt;

extern "C" {

size_t mogt_affine_scan_workspace_bytes(int64_t B, int64_t L, int64_t R, int64_t C) {
  const int lc = affine::lc_of((int)R);
  if (lc == 0 || B <= 0 || L <= 0 || C < 0) return sizeof(WsHeader);
  const size_t NU = (size_t)B * ((L + lc - 1) / lc);
  size_t f, a, i, tot;
  affine::ws_offsets(NU, (int)R, (int)C, &f, &a, &i, &tot);
  return tot;
}

int mogt_affine_scan_fwd(const void* U, const void* V, void* H, void* U_prefix, int64_t B,
                         int64_t L, int64_t R, int64_t C, int u_dtype, int v_dtype, int out_dtype,
                         int reverse, void* workspace, size_t workspace_bytes, void* stream) {
  if (B <= 0 || L < 0 || R <= 0 || C < 0) return MOGT_ERR_SHAPE;
  if (L == 0) return MOGT_OK;
  if (!U || (C > 0 && (!V || !H))) return MOGT_ERR_ARG;
  if (C == 0 && !U_prefix) return MOGT_ERR_ARG;
  if (reverse && U_prefix) return MOGT_ERR_UNSUPPORTED;
  const int lc = affine::lc_of((int)R);
  if (lc == 0) return MOGT_ERR_UNSUPPORTED;
  if (L >= ((int64_t)1 << 31) || C > 1024) return MOGT_ERR_UNSUPPORTED;
  affine::Params P;
  P.L = (int)L;
  P.C = (int)C;
  P.nunits = (int)((L + lc - 1) / lc);
  const size_t NU = (size_t)B * P.nunits;
  if (NU >= ((size_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  size_t fo, ao, io, tot;
  affine::ws_offsets(NU, (int)R, (int)C, &fo, &ao, &io, &tot);
  if (!workspace || workspace_bytes < tot) return MOGT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOGT_ERR_ALIGN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  P.U = U;
  P.V = V ? V : U;
  P.H = H ? H : U_prefix;
  P.P = U_prefix;
  P.hdr = reinterpret_cast<WsHeader*>(ws);
  P.flags = reinterpret_cast<uint32_t*>(ws + fo);
  P.agg = reinterpret_cast<float*>(ws + ao);
  P.inc = reinterpret_cast<float*>(ws + io);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int vdt = C > 0 ? v_dtype : u_dtype;
  return reverse ? affine::dispatch_r<true>((int)R, P, (int)B, u_dtype, vdt, out_dtype, s)
                 : affine::dispatch_r<false>((int)R, P, (int)B, u_dtype, vdt, out_dtype, s);
}

int mogt_affine_grad_u(const float* sigma, const float* H, void* grad_U, int64_t B, int64_t L,
                       int64_t R, int64_t C, int out_dtype, void* stream) {
  if (B <= 0 || L < 0 || R <= 0 || C <= 0) return MOGT_ERR_SHAPE;
  if (L == 0) return MOGT_OK;
  if (!sigma || !H || !grad_U) return MOGT_ERR_ARG;
  const size_t smem = (size_t)2 * R * C * 4;
  if (smem > 200 * 1024) return MOGT_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t steps = (size_t)B * L;
  const unsigned grid = (unsigned)(steps < 148 * 16 ? steps : 148 * 16);
  if (out_dtype == MOGT_DTYPE_F32) {
    cudaFuncSetAttribute(affine::affine_grad_u_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    affine::affine_grad_u_kernel<float><<<grid, 256, smem, s>>>(sigma, H, static_cast<float*>(grad_U),
                                                                (int)B, (int)L, (int)R, (int)C);
  } else if (out_dtype == MOGT_DTYPE_BF16) {
    cudaFuncSetAttribute(affine::affine_grad_u_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    affine::affine_grad_u_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>(
        sigma, H, static_cast<__nv_bfloat16*>(grad_U), (int)B, (int)L, (int)R, (int)C);
  } else {
    return MOGT_ERR_DTYPE;
  }
  return mogt_host::launch_status();
}

}  // extern "C"
