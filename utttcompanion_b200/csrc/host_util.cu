// Library-level host entry points and shared host utilities.
#include <stdio.h>
#include <string.h>

#include "host_util.cuh"

namespace uttt {

int& last_cuda_error_ref() {
  static thread_local int e = 0;
  return e;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return UTTT_ERR_CUDA;
  if (((uintptr_t)base & 15u) != 0) return UTTT_ERR_INVALID;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t gbox[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    gbox[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) {
      if (strides_bytes[i] % 16 != 0) return UTTT_ERR_INVALID;
      gstride[i] = strides_bytes[i];
    }
  }
  if (box[0] * 2 != 128) return UTTT_ERR_INVALID;  // 128 B inner box for SWIZZLE_128B
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride,
                  gbox, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? UTTT_OK : UTTT_ERR_INVALID;
}

}  // namespace uttt

extern "C" {

int uttt_version(void) { return 1; }

const char* uttt_status_string(int status) {
  switch (status) {
    case UTTT_OK: return "ok";
    case UTTT_ERR_INVALID: return "invalid argument";
    case UTTT_ERR_UNSUPPORTED: return "unsupported size or option";
    case UTTT_ERR_CUDA: return "CUDA runtime error";
    case UTTT_ERR_TIMEOUT: return "bounded device wait expired";
    case UTTT_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

int uttt_last_cuda_error(void) { return uttt::last_cuda_error_ref(); }

int uttt_read_status(void* workspace, int reset, void* stream) {
  if (!workspace) return UTTT_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  int value = 0;
  UTTT_TRY(uttt::cuda_status(cudaMemcpyAsync(&value, workspace, sizeof(int), cudaMemcpyDeviceToHost, s)));
  UTTT_TRY(uttt::cuda_status(cudaStreamSynchronize(s)));
  if (reset && value != 0) {
    UTTT_TRY(uttt::cuda_status(cudaMemsetAsync(workspace, 0, sizeof(int), s)));
    UTTT_TRY(uttt::cuda_status(cudaStreamSynchronize(s)));
  }
  return value;
}

}  // extern "C"
