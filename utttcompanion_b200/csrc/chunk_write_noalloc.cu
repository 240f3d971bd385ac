// Allocation-free variant of the chunk-TTT write.
//
// Some callers of this library cannot call cudaMalloc: a serving loop whose
// HBM is reserved up front (persona arena, KV rings) has nothing left for an
// extra allocation, and cudaMalloc / cudaFree may synchronise the whole device,
// stalling the decode streams that run beside the write; and host code in a
// foreign-language binding (ctypes, cgo, JNI) often has no device allocator at
// all.  For them uttt_chunk_write_noalloc runs the same kernels as
// uttt_chunk_write with its scratch in the fixed array below instead of a
// caller-provided workspace.  The caller still passes all inputs and outputs.
//
// Every device that loads this library holds the array until the process
// exits.  All calls share it and it keeps the last call's contents, so calls
// that overlap on the GPU (two streams, or two host threads) race on it; the
// caller must order them.
#include <mutex>

#include "host_util.cuh"

namespace uttt {
namespace {

__device__ __align__(256) static unsigned char g_noalloc_scratch[UTTT_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};
unsigned long long g_ctx[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code the
// symbol itself is only a host-side stand-in, so the address is looked up with
// the device current and cached per device, together with the id of the CUDA
// context it belongs to: a context re-created after cudaDeviceReset reloads the
// module, and the next call then looks the address up again.
int scratch_address(void** out) {
  int dev = 0;
  UTTT_TRY(cuda_status(cudaGetDevice(&dev)));
  if (dev < 0 || dev >= kMaxDevices) return UTTT_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> g(g_mu);
  const unsigned long long ctx = current_context_id();
  if (!g_addr[dev] || ctx == 0 || ctx != g_ctx[dev]) {
    void* p = nullptr;
    UTTT_TRY(cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch)));
    g_addr[dev] = p;
    g_ctx[dev] = current_context_id();
  }
  *out = g_addr[dev];
  return UTTT_OK;
}

}  // namespace
}  // namespace uttt

extern "C" int uttt_chunk_write_noalloc(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks,
                                        const void* q, const void* k, const void* v, const float* eta,
                                        const float* alpha, const float* mask, float* w_up, float* w_gate,
                                        float* w_down, float* s_up, float* s_gate, float* s_down,
                                        const float* ln_weight, const float* ln_bias, float momentum_beta,
                                        float max_grad_norm, int normalize_by_dim, float eps, void* out,
                                        int out_dtype, float* token_loss, float* clip_scale, void* stream) {
  using namespace uttt;
  const size_t need = uttt_chunk_write_workspace(B, C, d, h);
  if (need == 0) return UTTT_ERR_INVALID;
  if (need > (size_t)UTTT_NOALLOC_SCRATCH_BYTES) return UTTT_ERR_WORKSPACE;  // larger than the fixed scratch
  void* scratch = nullptr;
  UTTT_TRY(scratch_address(&scratch));
  // The status word must start at zero: a previous call's expired wait would
  // otherwise make every wait of this call return at once.
  UTTT_TRY(cuda_status(cudaMemsetAsync(scratch, 0, sizeof(int), (cudaStream_t)stream)));
  return uttt_chunk_write(B, T, C, d, h, chunk_begin, n_chunks, q, k, v, eta, alpha, mask, w_up, w_gate, w_down,
                          s_up, s_gate, s_down, ln_weight, ln_bias, momentum_beta, max_grad_norm, normalize_by_dim,
                          eps, out, out_dtype, token_loss, clip_scale, B, nullptr, nullptr, nullptr, scratch, (size_t)UTTT_NOALLOC_SCRATCH_BYTES,
                          stream);
}

// Reads the scratch's status word on the current device (see the header).
extern "C" int uttt_chunk_write_noalloc_status(int reset, void* stream) {
  using namespace uttt;
  void* scratch = nullptr;
  UTTT_TRY(scratch_address(&scratch));
  cudaStream_t st = (cudaStream_t)stream;
  int word = 0;
  UTTT_TRY(cuda_status(cudaMemcpyAsync(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost, st)));
  if (reset) UTTT_TRY(cuda_status(cudaMemsetAsync(scratch, 0, sizeof(int), st)));
  UTTT_TRY(cuda_status(cudaStreamSynchronize(st)));
  return word;
}
