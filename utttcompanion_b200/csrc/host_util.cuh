// Host-side helpers shared by the launchers: CUDA error capture, tensor-map
// encoding (through the runtime's driver entry point, so the library does not
// link libcuda), and workspace layout.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/uttt_b200.h"

namespace uttt {

int& last_cuda_error_ref();

inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return UTTT_OK;
  last_cuda_error_ref() = (int)e;
  return UTTT_ERR_CUDA;
}

// Unique id of the calling thread's current CUDA context (cuCtxGetId through the
// runtime's driver entry point), or 0 if there is none or it cannot be read.  A
// context re-created after cudaDeviceReset gets a new id.
unsigned long long current_context_id();

// A launcher's set-up step (a kernel's dynamic shared-memory limit, which belongs to
// the context it is set in) run once per device and context by whichever thread
// launches there first.  Only a successful run is remembered: a failed step is
// retried by the next caller, and a new context (after cudaDeviceReset) runs it again.
struct DeviceOnce {
  std::mutex mu;
  std::atomic<unsigned long long> ctx[64];   // context id of the last successful run, 0: none
};
template <class F>
inline int run_once_per_device(DeviceOnce& once, F&& step) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return UTTT_ERR_CUDA;
  const unsigned long long id = current_context_id();
  if (id != 0 && once.ctx[dev].load(std::memory_order_acquire) == id) return UTTT_OK;
  std::lock_guard<std::mutex> g(once.mu);
  if (id != 0 && once.ctx[dev].load(std::memory_order_relaxed) == id) return UTTT_OK;
  const int s = step();
  if (s == UTTT_OK) once.ctx[dev].store(current_context_id(), std::memory_order_release);
  return s;
}

// Check the launch that was just issued.
inline int launch_status() { return cuda_status(cudaGetLastError()); }

// Launch attribute: the kernel may start while the previous kernel of the stream
// runs; it calls pdl_wait() before touching anything an earlier launch wrote.
inline cudaLaunchAttribute pdl_attribute() {
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
  return a;
}

// SMs of the current device (cached per device ordinal).
inline int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

#define UTTT_TRY(expr)              \
  do {                              \
    int _s = (expr);                \
    if (_s != UTTT_OK) return _s;   \
  } while (0)

#define UTTT_REQUIRE(cond, code) \
  do {                           \
    if (!(cond)) return (code);  \
  } while (0)

// 2-D / 3-D BF16 tensor maps with 128-byte swizzle; out-of-bounds boxes are
// zero-filled.  `dims` / `strides_bytes` are innermost first.
int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box);
// FP32 tensor map; swizzle128 selects SWIZZLE_128B (inner box must then be 128 B), else none.
int make_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);

// Workspace: [status int (256 B slot)] [region 0] [region 1] ... each 256-B aligned.
struct WsCursor {
  uint8_t* base;
  size_t used;
  size_t cap;
  explicit WsCursor(void* b, size_t c) : base((uint8_t*)b), used(256), cap(c) {}
  template <class T>
  T* take(size_t count) {
    size_t bytes = (count * sizeof(T) + 255) & ~(size_t)255;
    T* p = (T*)(base + used);
    used += bytes;
    return p;
  }
  bool ok() const { return used <= cap; }
};

inline size_t ws_round(size_t bytes) { return (bytes + 255) & ~(size_t)255; }

inline int* ws_status(void* ws) { return (int*)ws; }

// Live per-kind kernel timing (see uttt_profile_enable).  Usage in a launcher:
//   ProfScope ps(UTTT_PROF_CHUNK_FWD, stream);  kernel<<<...>>>(...);
// The scope records a start event at construction and a stop event at
// destruction, both on `stream`.
bool prof_on();
void prof_record(int kind, cudaEvent_t start, cudaEvent_t stop);
struct ProfScope {
  int kind;
  cudaStream_t s;
  cudaEvent_t a = nullptr, b = nullptr;
  ProfScope(int k, cudaStream_t st) : kind(k), s(st) {
    if (prof_on()) {
      cudaEventCreate(&a);
      cudaEventCreate(&b);
      cudaEventRecord(a, s);
    }
  }
  ~ProfScope() {
    if (a) {
      cudaEventRecord(b, s);
      prof_record(kind, a, b);
    }
  }
};

}  // namespace uttt
