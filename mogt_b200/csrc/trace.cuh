// Debug-only phase timestamps for the stripe kernels, compiled in only with
// -DMOGT_TRACE (a separate debug build, never the product library):
// trace[unit * 16 + k] = %globaltimer (MOGT_MARK) or clock64 (MOGT_CLK) at
// phase k.  Each translation unit has its own trace pointer.
#pragma once

#ifdef MOGT_TRACE
namespace mogt {
static __device__ unsigned long long* g_mogt_trace = nullptr;
__device__ __forceinline__ void trace_mark(uint32_t unit, int k) {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  if (g_mogt_trace) g_mogt_trace[unit * 16 + k] = t;
}
__device__ __forceinline__ void trace_clk(uint32_t unit, int k) {
  if (g_mogt_trace) g_mogt_trace[unit * 16 + k] = clock64();
}
static inline int set_trace(void* buf) {
  unsigned long long* p = static_cast<unsigned long long*>(buf);
  return cudaMemcpyToSymbol(g_mogt_trace, &p, sizeof(p)) == cudaSuccess ? 0 : 4;
}
}  // namespace mogt
#define MOGT_MARK(u, k) \
  if (threadIdx.x == 0) ::mogt::trace_mark(u, k)
#define MOGT_CLK(u, k, cond) \
  if (threadIdx.x == 0 && (cond)) ::mogt::trace_clk(u, k)
#define MOGT_CLK_T(u, k, cond, tid) \
  if (threadIdx.x == (tid) && (cond)) ::mogt::trace_clk(u, k)
#else
#define MOGT_MARK(u, k)
#define MOGT_CLK(u, k, cond)
#define MOGT_CLK_T(u, k, cond, tid)
#endif
