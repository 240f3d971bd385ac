// Stability guard of a persona write (step 3 of interact_and_evolve,
// engine/personalizer.py:524-552): the slow-anchor elastic pull with its
// optional drift clamp (SharedFastWeightPool.apply_elastic_pull,
// model/uttt_layer.py:773-832) and the Frobenius drift report
// (compute_drift, :834-874), over B FP32 states sharing one W_0.
//
// Pull:   w = (1 - lambda) W + lambda W0  = W0 + (1 - lambda)(W - W0)
// Clamp:  scale_b = min(1, ratio * ||W0||_F / sqrt(||w_b - W0||_F^2 + 1e-8)),
//         w_b = W0 + (w_b - W0) * scale_b        (norms over all three matrices)
// Two streaming passes: per-state sums of squares (block partials + one
// atomic per block), then the in-place update.  Both are HBM-bound.
#include "common.cuh"
#include "host_util.cuh"

namespace uttt {
namespace {

constexpr int G_THREADS = 256;

__device__ __forceinline__ float gblock_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < G_THREADS / 32; ++i) s += red[i];
  return s;
}

// sums[b*4 + m] += sum((lam_keep * (W_m - W0_m))^2) for matrix m of state b; sums[b*4+3] unused.
// Also base[m] += sum(W0_m^2) from state 0's blocks (one state's worth).
__global__ void __launch_bounds__(G_THREADS) guard_stats_kernel(const float* __restrict__ w0, const float* __restrict__ w1,
                                                               const float* __restrict__ w2, const float* __restrict__ a0,
                                                               const float* __restrict__ a1, const float* __restrict__ a2,
                                                               long long n4, float keep, float* __restrict__ sums,
                                                               float* __restrict__ base) {
  __shared__ float red[G_THREADS / 32];
  const int m = blockIdx.y, b = blockIdx.z;
  const float4* W = reinterpret_cast<const float4*>(m == 0 ? w0 : (m == 1 ? w1 : w2)) + (size_t)b * n4;
  const float4* A = reinterpret_cast<const float4*>(m == 0 ? a0 : (m == 1 ? a1 : a2));
  float s = 0.f, sb = 0.f;
  for (long long i = blockIdx.x * (long long)G_THREADS + threadIdx.x; i < n4; i += (long long)gridDim.x * G_THREADS) {
    const float4 w = W[i], a = A[i];
    const float dx = keep * (w.x - a.x), dy = keep * (w.y - a.y), dz = keep * (w.z - a.z), dw = keep * (w.w - a.w);
    s += dx * dx + dy * dy + dz * dz + dw * dw;
    if (b == 0 && base) sb += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  s = gblock_sum(s, red);
  if (threadIdx.x == 0) atomicAdd(sums + b * 4 + m, s);
  if (b == 0 && base) {
    sb = gblock_sum(sb, red);
    if (threadIdx.x == 0) atomicAdd(base + m, sb);
  }
}

__global__ void __launch_bounds__(G_THREADS) guard_apply_kernel(float* __restrict__ w0, float* __restrict__ w1,
                                                               float* __restrict__ w2, const float* __restrict__ a0,
                                                               const float* __restrict__ a1, const float* __restrict__ a2,
                                                               long long n4, float keep, float ratio,
                                                               const float* __restrict__ sums,
                                                               const float* __restrict__ base) {
  const int m = blockIdx.y, b = blockIdx.z;
  float scale = 1.f;
  if (ratio > 0.f) {
    const float bn = sqrtf(base[0] + base[1] + base[2] + 1e-8f);
    const float dn = sqrtf(sums[b * 4 + 0] + sums[b * 4 + 1] + sums[b * 4 + 2] + 1e-8f);
    scale = fminf(ratio * bn / dn, 1.f);
  }
  const float f = keep * scale;
  float4* W = reinterpret_cast<float4*>(m == 0 ? w0 : (m == 1 ? w1 : w2)) + (size_t)b * n4;
  const float4* A = reinterpret_cast<const float4*>(m == 0 ? a0 : (m == 1 ? a1 : a2));
  for (long long i = blockIdx.x * (long long)G_THREADS + threadIdx.x; i < n4; i += (long long)gridDim.x * G_THREADS) {
    float4 w = W[i];
    const float4 a = A[i];
    w.x = a.x + (w.x - a.x) * f;
    w.y = a.y + (w.y - a.y) * f;
    w.z = a.z + (w.z - a.z) * f;
    w.w = a.w + (w.w - a.w) * f;
    W[i] = w;
  }
}

}  // namespace
}  // namespace uttt

using namespace uttt;

extern "C" size_t uttt_guard_workspace(int B) { return B > 0 ? 256 + ws_round((size_t)(B * 4 + 4) * sizeof(float)) : 0; }

extern "C" int uttt_elastic_pull(int B, int d, int h, float* w_up, float* w_gate, float* w_down, const float* w_up0,
                                 const float* w_gate0, const float* w_down0, float anchor_lambda,
                                 float max_drift_ratio, void* workspace, size_t workspace_bytes, void* stream) {
  UTTT_REQUIRE(B > 0 && d > 0 && h > 0 && w_up && w_gate && w_down && w_up0 && w_gate0 && w_down0 && workspace,
               UTTT_ERR_INVALID);
  UTTT_REQUIRE(((long long)d * h) % 4 == 0, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(workspace_bytes >= uttt_guard_workspace(B), UTTT_ERR_WORKSPACE);
  if (anchor_lambda <= 0.f && !(max_drift_ratio > 0.f)) return UTTT_OK;   // nothing to do (:793-794)
  cudaStream_t st = (cudaStream_t)stream;
  WsCursor ws(workspace, workspace_bytes);
  float* sums = ws.take<float>((size_t)B * 4 + 4);
  float* base = sums + (size_t)B * 4;
  const long long n4 = (long long)d * h / 4;
  const float keep = 1.f - anchor_lambda;
  const dim3 grid(64, 3, B);
  ProfScope ps(UTTT_PROF_ROWWISE, st);
  if (max_drift_ratio > 0.f) {
    UTTT_TRY(cuda_status(cudaMemsetAsync(sums, 0, ((size_t)B * 4 + 4) * sizeof(float), st)));
    guard_stats_kernel<<<grid, G_THREADS, 0, st>>>(w_up, w_gate, w_down, w_up0, w_gate0, w_down0, n4, keep, sums,
                                                   base);
    UTTT_TRY(launch_status());
  }
  guard_apply_kernel<<<grid, G_THREADS, 0, st>>>(w_up, w_gate, w_down, w_up0, w_gate0, w_down0, n4, keep,
                                                 max_drift_ratio > 0.f ? max_drift_ratio : 0.f, sums, base);
  return launch_status();
}

extern "C" int uttt_drift_sums(int B, int d, int h, const float* w_up, const float* w_gate, const float* w_down,
                               const float* w_up0, const float* w_gate0, const float* w_down0, float* out,
                               void* stream) {
  UTTT_REQUIRE(B > 0 && d > 0 && h > 0 && w_up && w_gate && w_down && w_up0 && w_gate0 && w_down0 && out,
               UTTT_ERR_INVALID);
  UTTT_REQUIRE(((long long)d * h) % 4 == 0, UTTT_ERR_UNSUPPORTED);
  cudaStream_t st = (cudaStream_t)stream;
  UTTT_TRY(cuda_status(cudaMemsetAsync(out, 0, ((size_t)B * 4 + 4) * sizeof(float), st)));
  ProfScope ps(UTTT_PROF_ROWWISE, st);
  guard_stats_kernel<<<dim3(64, 3, B), G_THREADS, 0, st>>>(w_up, w_gate, w_down, w_up0, w_gate0, w_down0,
                                                            (long long)d * h / 4, 1.f, out, out + (size_t)B * 4);
  return launch_status();
}
