// Hidden-split readout: the exchange of partial z over NVLink peer memory, fused with the
// LayerNorm finish.
//
// With every persona's hidden units split over P GPUs, each rank's readout produces a partial
// z (rows, d) FP32 that must be summed over the ranks before the LayerNorm (hsplit.py).  Instead
// of an NCCL all-reduce followed by a finish launch, one kernel per exchange does both: each CTA
// owns one row, stores its partial row straight into every peer's receive buffer (plain P2P
// stores through CUDA IPC mappings; no multicast), raises a per-(sender, row) flag on each peer
// with a system-scope release, waits (bounded) for every peer's flag on its own GPU, sums the
// partials in rank order (so every rank holds the same bits) and applies the LayerNorm and the
// residual.  An epoch counter in each rank's own memory, bumped after every exchange, keys the
// flags and selects one of two receive buffers, so a rank one exchange ahead never overwrites
// data a peer is still reading.  Captured CUDA graphs replay it unchanged.
//
// Layout of one rank's exchange area (allocated by uttt_ipc_alloc, zero on allocation):
//   flags  [world][max_rows] u32        written by the peers, polled here
//   epoch  u32                          this rank's exchange count
//   recv   [2][world][max_rows][d] FP32 the peers' partial rows, by epoch parity and sender
#include <string.h>

#include "common.cuh"
#include "host_util.cuh"

namespace uttt {
namespace {

constexpr int XT = 256;           // threads per CTA (one row)
constexpr int XMAXD = 4096;
constexpr int XMAX_WORLD = 8;

struct ExchangePeers {
  uint8_t* base[XMAX_WORLD];      // every rank's exchange area (this rank's own included)
};

__host__ __device__ inline size_t xch_flags_bytes(int world, int max_rows) {
  return ((size_t)world * max_rows * sizeof(unsigned) + 255) & ~(size_t)255;
}
__host__ __device__ inline size_t xch_recv_offset(int world, int max_rows) {
  return xch_flags_bytes(world, max_rows) + 256;   // flags, then the epoch word in its own 256 bytes
}
__host__ __device__ inline size_t xch_area_bytes(int world, int max_rows, int d) {
  return xch_recv_offset(world, max_rows) + (size_t)2 * world * max_rows * d * sizeof(float);
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float cta_sum256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < XT / 32; ++i) s += red[i];
  return s;
}

template <int MD>
__global__ void __launch_bounds__(XT) exchange_finish_kernel(const float* __restrict__ zpart,
                                                             const __nv_bfloat16* __restrict__ x, int d,
                                                             const float* __restrict__ ln_w,
                                                             const float* __restrict__ ln_b, float eps, void* out,
                                                             int out_bf16, int z_bf16, const ExchangePeers peers,
                                                             int rank, int world, int max_rows, int* status,
                                                             unsigned max_polls) {
  __shared__ float red[XT / 32];
  constexpr int NZ = MD / XT;
  const int b = blockIdx.x, tid = threadIdx.x;
  const size_t recv_off = xch_recv_offset(world, max_rows);
  const unsigned* epoch = reinterpret_cast<const unsigned*>(peers.base[rank] + xch_flags_bytes(world, max_rows));
  const unsigned e = __ldcg(epoch);
  const int par = (int)(e & 1u);

  // 1. this rank's partial row into slot [par][rank][b] of every peer
  float mine[NZ];
#pragma unroll
  for (int i = 0; i < NZ; ++i) {
    const int c = tid + i * XT;
    mine[i] = c < d ? zpart[(size_t)b * d + c] : 0.f;
  }
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    float* dst = reinterpret_cast<float*>(peers.base[r] + recv_off) + (((size_t)par * world + rank) * max_rows + b) * d;
#pragma unroll
    for (int i = 0; i < NZ; ++i) {
      const int c = tid + i * XT;
      if (c < d) dst[c] = mine[i];
    }
  }
  __threadfence_system();
  __syncthreads();
  // 2. flag (sender = rank, row b) on every peer; then wait for every peer's flag here
  if (tid < world && tid != rank)
    st_release_sys(reinterpret_cast<unsigned*>(peers.base[tid]) + (size_t)rank * max_rows + b, e + 1u);
  if (tid < world && tid != rank) {
    const unsigned* f = reinterpret_cast<const unsigned*>(peers.base[rank]) + (size_t)tid * max_rows + b;
    uint32_t polls = 0;
    while (ld_acquire_sys(f) < e + 1u) {
      if (++polls > max_polls || status_set(status)) {
        set_status(status, UTTT_ERR_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  // 3. z over all ranks in rank order, then out = x + LN(z) * gamma + beta
  const float* recv = reinterpret_cast<const float*>(peers.base[rank] + recv_off);
  float zv[NZ];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NZ; ++i) {
    const int c = tid + i * XT;
    float z = 0.f;
    if (c < d) {
      for (int r = 0; r < world; ++r)
        z += (r == rank) ? mine[i] : __ldcg(recv + (((size_t)par * world + r) * max_rows + b) * d + c);
      if (z_bf16) z = __bfloat162float(__float2bfloat16(z));
    }
    zv[i] = z;
    sum += z;
  }
  const float dinv = 1.f / (float)d;
  const float mean = cta_sum256(sum, red) * dinv;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NZ; ++i)
    if (tid + i * XT < d) sq += (zv[i] - mean) * (zv[i] - mean);
  const float rstd = rsqrtf(cta_sum256(sq, red) * dinv + eps);
#pragma unroll
  for (int i = 0; i < NZ; ++i) {
    const int c = tid + i * XT;
    if (c < d) {
      const float y = __bfloat162float(x[(size_t)b * d + c]) + ((zv[i] - mean) * rstd * ln_w[c] + ln_b[c]);
      if (out_bf16)
        reinterpret_cast<__nv_bfloat16*>(out)[(size_t)b * d + c] = __float2bfloat16(y);
      else
        reinterpret_cast<float*>(out)[(size_t)b * d + c] = y;
    }
  }
}

// the exchange's epoch, after every CTA of the exchange has read it (stream order)
__global__ void epoch_bump_kernel(unsigned* epoch) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *epoch += 1u;
}

}  // namespace
}  // namespace uttt

using namespace uttt;

extern "C" size_t uttt_split_exchange_bytes(int world, int max_rows, int d) {
  if (world < 2 || world > XMAX_WORLD || max_rows <= 0 || d <= 0) return 0;
  return xch_area_bytes(world, max_rows, d);
}

extern "C" int uttt_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  UTTT_REQUIRE(bytes > 0 && ptr && handle, UTTT_ERR_INVALID);
  void* p = nullptr;
  UTTT_TRY(cuda_status(cudaMalloc(&p, bytes)));
  int s = cuda_status(cudaMemset(p, 0, bytes));
  if (s == UTTT_OK) s = cuda_status(cudaDeviceSynchronize());   // zero before any peer can map it
  if (s == UTTT_OK) s = cuda_status(cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), p));
  if (s != UTTT_OK) {
    cudaFree(p);
    return s;
  }
  *ptr = p;
  return UTTT_OK;
}

extern "C" int uttt_ipc_open(const void* handle, void** ptr) {
  UTTT_REQUIRE(handle && ptr, UTTT_ERR_INVALID);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int uttt_ipc_close(void* ptr) {
  UTTT_REQUIRE(ptr, UTTT_ERR_INVALID);
  return cuda_status(cudaIpcCloseMemHandle(ptr));
}

extern "C" int uttt_ipc_free(void* ptr) {
  UTTT_REQUIRE(ptr, UTTT_ERR_INVALID);
  return cuda_status(cudaFree(ptr));
}

extern "C" int uttt_split_exchange_finish(int rows, int d, const float* z_partial, const void* x,
                                          const float* ln_weight, const float* ln_bias, float eps, void* out,
                                          int out_dtype, int z_bf16, int rank, int world, int max_rows,
                                          void* const* areas, unsigned max_polls, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  UTTT_REQUIRE(rows > 0 && d > 0 && z_partial && x && ln_weight && ln_bias && out && areas && workspace,
               UTTT_ERR_INVALID);
  UTTT_REQUIRE(world >= 2 && world <= XMAX_WORLD && rank >= 0 && rank < world, UTTT_ERR_INVALID);
  UTTT_REQUIRE(rows <= max_rows, UTTT_ERR_INVALID);
  UTTT_REQUIRE(out_dtype == UTTT_DTYPE_F32 || out_dtype == UTTT_DTYPE_BF16, UTTT_ERR_INVALID);
  UTTT_REQUIRE(d % 128 == 0 && d <= XMAXD && eps > 0.f, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(max_polls >= 1 && workspace_bytes >= 256, UTTT_ERR_WORKSPACE);
  ExchangePeers peers;
  memset(&peers, 0, sizeof(peers));
  for (int r = 0; r < world; ++r) {
    UTTT_REQUIRE(areas[r] != nullptr, UTTT_ERR_INVALID);
    peers.base[r] = reinterpret_cast<uint8_t*>(areas[r]);
  }
  cudaStream_t st = (cudaStream_t)stream;
  int* status = ws_status(workspace);
  ProfScope ps(UTTT_PROF_READOUT_LN, st);
  const int ob = out_dtype == UTTT_DTYPE_BF16;
  if (d <= 1024)
    exchange_finish_kernel<1024><<<rows, XT, 0, st>>>(z_partial, (const __nv_bfloat16*)x, d, ln_weight, ln_bias, eps,
                                                      out, ob, z_bf16 != 0, peers, rank, world, max_rows, status,
                                                      max_polls);
  else
    exchange_finish_kernel<XMAXD><<<rows, XT, 0, st>>>(z_partial, (const __nv_bfloat16*)x, d, ln_weight, ln_bias,
                                                       eps, out, ob, z_bf16 != 0, peers, rank, world, max_rows,
                                                       status, max_polls);
  UTTT_TRY(launch_status());
  epoch_bump_kernel<<<1, 32, 0, st>>>(
      reinterpret_cast<unsigned*>(peers.base[rank] + xch_flags_bytes(world, max_rows)));
  return launch_status();
}
