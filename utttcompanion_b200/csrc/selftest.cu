// Tensor-core self-test GEMM: D = A * B^T with every operand orientation the
// hot-path kernels use (K-major / MN-major, TMA-loaded or converted from FP32
// by software producers).  It pins the UMMA descriptor, swizzle and TMEM
// conventions against a plain matmul before the fused kernels rely on them.
#include <string.h>

#include "common.cuh"
#include "host_util.cuh"

namespace uttt {
namespace {

constexpr int kThreads = 128;

__global__ void __launch_bounds__(kThreads) selftest_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                 const __grid_constant__ CUtensorMap tmB,
                                                                 const float* __restrict__ a_f32, int mode, int M,
                                                                 int N, int K, float* __restrict__ D,
                                                                 int* status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full, bar_mma;
  __shared__ uint32_t tmem_slot;
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* sA = smem_raw + pad;        // 16 KB: 128 x 64 bf16
  uint8_t* sB = sA + 16384;            // N x 64 bf16
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool a_mn = mode & 1, b_mn = (mode >> 1) & 1, a_sw = (mode >> 2) & 1;
  const int m0 = blockIdx.x * 128;
  const uint32_t ncols = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));

  if (tid == 0) {
    mbar_init(&bar_full, 1);
    mbar_init(&bar_mma, 1);
    fence_mbarrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t idesc = idesc_bf16(128, N, a_mn, b_mn);

  const int nkb = K / 64;
  for (int kb = 0; kb < nkb; ++kb) {
    if (a_sw) {
      // FP32 A given K x M (MN-major): convert to BF16 into the MN-major SW128 image.
      for (int i = tid; i < 64 * 32; i += kThreads) {
        const int kr = i / 32, m4 = (i % 32) * 4;
        const float4 f = *reinterpret_cast<const float4*>(a_f32 + (size_t)(kb * 64 + kr) * M + m0 + m4);
        uint2 p;
        p.x = pack_bf16x2(f.x, f.y);
        p.y = pack_bf16x2(f.z, f.w);
        const int mblk = m4 / 64, mm = m4 % 64;
        *reinterpret_cast<uint2*>(sA + mblk * 8192 + sw128_offset(kr, mm * 2)) = p;
      }
      fence_proxy_async_smem();
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t bytes = (uint32_t)N * 128u + (a_sw ? 0u : 16384u);
      mbar_arrive_expect_tx(&bar_full, bytes);
      if (!a_sw) {
        if (a_mn) {
          tma_load_2d(sA, &tmA, &bar_full, m0, kb * 64);
          tma_load_2d(sA + 8192, &tmA, &bar_full, m0 + 64, kb * 64);
        } else {
          tma_load_2d(sA, &tmA, &bar_full, kb * 64, m0);
        }
      }
      if (b_mn) {
        for (int j = 0; j < N / 64; ++j) tma_load_2d(sB + j * 8192, &tmB, &bar_full, j * 64, kb * 64);
      } else {
        tma_load_2d(sB, &tmB, &bar_full, kb * 64, 0);
      }
    }
    mbar_wait(&bar_full, kb & 1, status);
    if (tid == 0) {
      tc_fence_after();
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t ad = a_mn ? sdesc_sw128(smem_u32(sA) + ks * 2048, 8192, 1024)
                                 : sdesc_sw128(smem_u32(sA) + ks * 32, 16, 1024);
        const uint64_t bd = b_mn ? sdesc_sw128(smem_u32(sB) + ks * 2048, 8192, 1024)
                                 : sdesc_sw128(smem_u32(sB) + ks * 32, 16, 1024);
        mma_bf16(tmem, ad, bd, idesc, (kb > 0 || ks > 0) ? 1u : 0u);
      }
      mma_commit(&bar_mma);
    }
    mbar_wait(&bar_mma, kb & 1, status);
  }
  tc_fence_after();
  // 4 warps cover the 128 accumulator lanes.
  const int row = m0 + warp * 32 + lane;
  for (int n0 = 0; n0 < N; n0 += 16) {
    float v[16];
    tmem_ld16(tmem_addr(tmem, warp * 32, n0), v);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 16; ++i) D[(size_t)row * N + n0 + i] = v[i];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

}  // namespace
}  // namespace uttt

extern "C" int uttt_selftest_gemm(int mode, int M, int N, int K, const void* a, const void* b, float* d,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  using namespace uttt;
  UTTT_REQUIRE(a && b && d && workspace, UTTT_ERR_INVALID);
  UTTT_REQUIRE(workspace_bytes >= 256, UTTT_ERR_WORKSPACE);
  UTTT_REQUIRE(M > 0 && M % 128 == 0 && K > 0 && K % 64 == 0, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(N == 64 || N == 128 || N == 256, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE((mode & ~7) == 0, UTTT_ERR_INVALID);
  const bool a_mn = mode & 1, b_mn = (mode >> 1) & 1, a_sw = (mode >> 2) & 1;
  UTTT_REQUIRE(!a_sw || a_mn, UTTT_ERR_UNSUPPORTED);
  CUtensorMap tmA, tmB;
  memset(&tmA, 0, sizeof(tmA));
  if (!a_sw) {
    if (a_mn) {
      uint64_t dims[2] = {(uint64_t)M, (uint64_t)K}, str[1] = {(uint64_t)M * 2};
      uint32_t box[2] = {64, 64};
      UTTT_TRY(make_tmap_bf16(&tmA, a, 2, dims, str, box));
    } else {
      uint64_t dims[2] = {(uint64_t)K, (uint64_t)M}, str[1] = {(uint64_t)K * 2};
      uint32_t box[2] = {64, 128};
      UTTT_TRY(make_tmap_bf16(&tmA, a, 2, dims, str, box));
    }
  }
  if (b_mn) {
    uint64_t dims[2] = {(uint64_t)N, (uint64_t)K}, str[1] = {(uint64_t)N * 2};
    uint32_t box[2] = {64, 64};
    UTTT_TRY(make_tmap_bf16(&tmB, b, 2, dims, str, box));
  } else {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)N}, str[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {64, (uint32_t)N};
    UTTT_TRY(make_tmap_bf16(&tmB, b, 2, dims, str, box));
  }
  const size_t smem = 1024 + 16384 + (size_t)N * 128;
  UTTT_TRY(cuda_status(cudaFuncSetAttribute(selftest_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem)));
  selftest_gemm_kernel<<<M / 128, kThreads, smem, (cudaStream_t)stream>>>(
      tmA, tmB, (const float*)a, mode, M, N, K, d, ws_status(workspace));
  return launch_status();
}

// ----------------------------------------------------------------------------
// Bounded-wait self-test: one CTA runs the kernels' own bounded waits on an
// event that never happens (an mbarrier phase nothing arrives on, or a d-split
// exchange counter nothing increments), with a short caller-given poll limit.
// The wait expires, records UTTT_ERR_TIMEOUT in the workspace status word and
// the kernel returns; no copy or MMA is in flight, so the context stays usable.
// ----------------------------------------------------------------------------
namespace uttt {
namespace {
__global__ void __launch_bounds__(32) selftest_wait_kernel(int kind, uint32_t max_polls, unsigned* counter,
                                                           int* returned, int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    if (kind == 0)
      mbar_wait_limit(&bar, 0, status, max_polls);      // phase 0 never completes: no arrival
    else
      counter_wait(counter, 1u, status, max_polls);    // the counter stays 0
    *returned = 1;
  }
}
}  // namespace
}  // namespace uttt

extern "C" int uttt_selftest_wait(int kind, unsigned max_polls, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  using namespace uttt;
  UTTT_REQUIRE(workspace && workspace_bytes >= 512, UTTT_ERR_WORKSPACE);
  UTTT_REQUIRE(kind == 0 || kind == 1, UTTT_ERR_INVALID);
  UTTT_REQUIRE(max_polls >= 1 && max_polls <= (1u << 20), UTTT_ERR_INVALID);
  uint8_t* ws = (uint8_t*)workspace;
  unsigned* counter = (unsigned*)(ws + 256);
  int* returned = (int*)(ws + 260);
  cudaStream_t st = (cudaStream_t)stream;
  UTTT_TRY(cuda_status(cudaMemsetAsync(ws + 256, 0, 8, st)));
  selftest_wait_kernel<<<1, 32, 0, st>>>(kind, max_polls, counter, returned, ws_status(workspace));
  return launch_status();
}
