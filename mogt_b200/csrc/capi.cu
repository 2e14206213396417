// Library-wide C ABI helpers: version, status strings, workspace status, and
// the TMA descriptor encoder shared by the kernels.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace mogt_host {

CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) return CUDA_ERROR_NOT_FOUND;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(map, dtype, rank, base, dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace mogt_host

extern "C" {

int mogt_abi_version(void) { return MOGT_ABI_VERSION; }

const char* mogt_status_string(int status) {
  switch (status) {
    case MOGT_OK: return "ok";
    case MOGT_ERR_SHAPE: return "bad shape";
    case MOGT_ERR_DTYPE: return "unsupported dtype";
    case MOGT_ERR_ALIGN: return "pointer not 16-byte aligned";
    case MOGT_ERR_LAUNCH: return "CUDA launch or TMA descriptor failure";
    case MOGT_ERR_TIMEOUT: return "device-side wait timed out";
    case MOGT_ERR_WORKSPACE: return "workspace missing or too small";
    case MOGT_ERR_UNSUPPORTED: return "unsupported configuration";
    case MOGT_ERR_ARG: return "null pointer argument";
    case MOGT_ERR_TOO_LARGE: return "problem exceeds the fixed 16 MiB scratch of the allocation-free entry point";
    default: return "unknown status";
  }
}

int mogt_workspace_status(const void* workspace, void* stream, int* err_out, uint32_t* unit_out) {
  if (!workspace || !err_out) return MOGT_ERR_ARG;
  uint32_t h[5];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(h, workspace, sizeof(h), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return MOGT_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return MOGT_ERR_LAUNCH;
  *err_out = static_cast<int>(h[3]);
  if (unit_out) *unit_out = h[4];
  return MOGT_OK;
}

int mogt_workspace_clear(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace) return MOGT_ERR_ARG;
  return cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? MOGT_OK
             : MOGT_ERR_LAUNCH;
}

}  // extern "C"
