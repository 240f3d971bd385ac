// Library-level host entry points and shared host utilities.
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <utility>
#include <vector>

#include "host_util.cuh"

namespace uttt {

int& last_cuda_error_ref() {
  static thread_local int e = 0;
  return e;
}

namespace {
struct ProfState {
  bool on = false;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> events;
  std::mutex mu;
};
ProfState& prof() {
  static ProfState s;
  return s;
}
}  // namespace

bool prof_on() { return prof().on; }

void prof_record(int kind, cudaEvent_t start, cudaEvent_t stop) {
  std::lock_guard<std::mutex> g(prof().mu);
  prof().events.push_back({kind, {start, stop}});
}

unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
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

int make_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
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
  if ((box[0] * 4) % 16 != 0 || (swizzle128 && box[0] * 4 != 128)) return UTTT_ERR_INVALID;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride,
                  gbox, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
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

int uttt_profile_enable(int on) {
  uttt::prof().on = on != 0;
  return UTTT_OK;
}

int uttt_profile_read(float* total_ms, int* launches) {
  if (!total_ms || !launches) return UTTT_ERR_INVALID;
  for (int i = 0; i < UTTT_PROF_KINDS; ++i) {
    total_ms[i] = 0.f;
    launches[i] = 0;
  }
  std::lock_guard<std::mutex> g(uttt::prof().mu);
  int status = UTTT_OK;
  for (auto& e : uttt::prof().events) {
    float ms = 0.f;
    if (cudaEventSynchronize(e.second.second) != cudaSuccess ||
        cudaEventElapsedTime(&ms, e.second.first, e.second.second) != cudaSuccess)
      status = UTTT_ERR_CUDA;
    if (e.first >= 0 && e.first < UTTT_PROF_KINDS) {
      total_ms[e.first] += ms;
      launches[e.first] += 1;
    }
    cudaEventDestroy(e.second.first);
    cudaEventDestroy(e.second.second);
  }
  uttt::prof().events.clear();
  return status;
}

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
