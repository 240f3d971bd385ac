// Row-wise kernels of the uTTT forward: RMSNorm (model/uttt_layer.py:881-896),
// the token-embedding gather (model/uttt_model.py:778-780) and the greedy
// pick of _sample_next_token at temperature 0 (model/uttt_model.py:1204-1221).
#include "common.cuh"
#include "host_util.cuh"

namespace uttt {
namespace {

constexpr int R_THREADS = 256;

__device__ __forceinline__ float rblock_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < R_THREADS / 32; ++i) s += red[i];
  return s;
}

// out = rms_norm(x) * bf16(weight): FP32 statistics, one rounding at the end
__global__ void __launch_bounds__(R_THREADS) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long long x_ld,
                                                            const float* __restrict__ w, int d, float eps,
                                                            __nv_bfloat16* __restrict__ out, long long out_ld) {
  __shared__ float red[R_THREADS / 32];
  const int r = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)r * x_ld;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += R_THREADS) {
    const float v = __bfloat162float(xr[i]);
    ss += v * v;
  }
  const float rinv = rsqrtf(rblock_sum(ss, red) / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += R_THREADS) {
    float v = __bfloat162float(xr[i]) * rinv;
    if (w) v *= __bfloat162float(__float2bfloat16(w[i]));
    out[(size_t)r * out_ld + i] = __float2bfloat16(v);
  }
}

// ids outside [0, V) are clamped, so no id can address memory outside the table
__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int d, int V,
                             __nv_bfloat16* __restrict__ out) {
  const int r = blockIdx.x;
  const int id = min(max(ids[r], 0), V - 1);
  const __nv_bfloat16* src = table + (size_t)id * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) out[(size_t)r * d + i] = src[i];
}

// Greedy pick over BF16-rounded logits with ids 0,1,3 (PAD/BOS/UNK) masked, or
// 0..5 in stop-free mode, and ids >= active_limit masked.  Ties go to the
// lowest id.  Writes the id and the top-1 / top-2 values.  A NaN logit counts
// as -inf, and a row with no finite candidate still returns an allowed id.
__global__ void __launch_bounds__(R_THREADS) argmax_kernel(const void* __restrict__ logits, int logits_f32,
                                                           long long ld, int V, int active_limit, int stop_free,
                                                           int* __restrict__ ids, float* __restrict__ top2) {
  __shared__ float sv1[R_THREADS], sv2[R_THREADS];
  __shared__ int si1[R_THREADS];
  const int r = blockIdx.x, tid = threadIdx.x;
  float v1 = -INFINITY, v2 = -INFINITY;
  int i1 = 0x7fffffff;
  const int lim = active_limit < V ? active_limit : V;
  for (int i = tid; i < lim; i += R_THREADS) {
    if (i == 0 || i == 1 || i == 3 || (stop_free && i < 6)) continue;
    float v = logits_f32 ? reinterpret_cast<const float*>(logits)[(size_t)r * ld + i]
                         : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits)[(size_t)r * ld + i]);
    v = __bfloat162float(__float2bfloat16(v));
    if (v != v) v = -INFINITY;
    if (v > v1 || (v == v1 && i < i1)) {
      v2 = v1;
      v1 = v;
      i1 = i;
    } else if (v > v2) {
      v2 = v;
    }
  }
  sv1[tid] = v1;
  sv2[tid] = v2;
  si1[tid] = i1;
  __syncthreads();
  for (int s = R_THREADS / 2; s > 0; s >>= 1) {
    if (tid < s) {
      const float a1 = sv1[tid], a2 = sv2[tid], b1 = sv1[tid + s], b2 = sv2[tid + s];
      const int ai = si1[tid], bi = si1[tid + s];
      const bool bwins = b1 > a1 || (b1 == a1 && bi < ai);
      const float n1 = bwins ? b1 : a1;
      const int ni = bwins ? bi : ai;
      const float n2 = bwins ? fmaxf(a1, b2) : fmaxf(a2, b1);
      sv1[tid] = n1;
      sv2[tid] = n2;
      si1[tid] = ni;
    }
    __syncthreads();
  }
  if (tid == 0) {
    ids[r] = si1[0] < lim ? si1[0] : (stop_free ? 6 : 2) % lim;   // only when no candidate was finite
    if (top2) {
      top2[2 * r] = sv1[0];
      top2[2 * r + 1] = sv2[0];
    }
  }
}

// BF16 read copies of S FP32 states: packed[s][k] = [w_up[s][k] | w_gate[s][k]] (2h), down = w_down.
__global__ void pack_read_kernel(const float4* __restrict__ w_up, const float4* __restrict__ w_gate,
                                 const float4* __restrict__ w_down, long long n_ug4, int h4,
                                 uint2* __restrict__ packed, uint2* __restrict__ down, long long n_d4) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_ug4; i += stride) {
    const long long row = i / h4, c = i % h4;  // row = s*d + k
    const float4 u = w_up[i], g = w_gate[i];
    packed[row * 2 * h4 + c] = make_uint2(pack_bf16x2(u.x, u.y), pack_bf16x2(u.z, u.w));
    packed[row * 2 * h4 + h4 + c] = make_uint2(pack_bf16x2(g.x, g.y), pack_bf16x2(g.z, g.w));
  }
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_d4; i += stride) {
    const float4 v = w_down[i];
    down[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

// apply_rope on (B, H, T, D) q and k with (T, D) cos / sin rows, every op rounded
// to BF16 as the reference's eager BF16 path does (model/uttt_layer.py:946-958).
__global__ void rope_apply_kernel(__nv_bfloat16* __restrict__ x, long long rows, int T, int D,
                                  const __nv_bfloat16* __restrict__ cs, const __nv_bfloat16* __restrict__ sn,
                                  __nv_bfloat16* __restrict__ out) {
  const long long r = blockIdx.x;          // row = (b, h, t)
  if (r >= rows) return;
  const int t = (int)(r % T);
  const int half = D / 2;
  const __nv_bfloat16* xr = x + r * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float xi = __bfloat162float(xr[i]);
    const float rot = i < half ? -__bfloat162float(xr[i + half]) : __bfloat162float(xr[i - half]);
    const float c = __bfloat162float(cs[(size_t)t * D + i]), s = __bfloat162float(sn[(size_t)t * D + i]);
    const float a = __bfloat162float(__float2bfloat16(xi * c));
    const float b = __bfloat162float(__float2bfloat16(rot * s));
    out[r * D + i] = __float2bfloat16(a + b);
  }
}

}  // namespace
}  // namespace uttt

using namespace uttt;

extern "C" int uttt_apply_rope(long long rows, int T, int D, const void* x, const void* cos_t, const void* sin_t,
                               void* out, void* stream) {
  UTTT_REQUIRE(rows > 0 && T > 0 && D > 0 && D % 2 == 0 && x && cos_t && sin_t && out, UTTT_ERR_INVALID);
  UTTT_REQUIRE(rows % T == 0, UTTT_ERR_INVALID);
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps(UTTT_PROF_ROWWISE, st);
  rope_apply_kernel<<<(unsigned)rows, 64, 0, st>>>((__nv_bfloat16*)x, rows, T, D, (const __nv_bfloat16*)cos_t,
                                                   (const __nv_bfloat16*)sin_t, (__nv_bfloat16*)out);
  return launch_status();
}

extern "C" int uttt_pack_read_copies(int S, int d, int h, const float* w_up, const float* w_gate,
                                     const float* w_down, void* packed_up_gate, void* down, void* stream) {
  UTTT_REQUIRE(S > 0 && d > 0 && h > 0 && w_up && w_gate && w_down && packed_up_gate && down, UTTT_ERR_INVALID);
  UTTT_REQUIRE(h % 4 == 0 && d % 4 == 0, UTTT_ERR_UNSUPPORTED);
  cudaStream_t st = (cudaStream_t)stream;
  const long long n_ug4 = (long long)S * d * h / 4, n_d4 = n_ug4;
  ProfScope ps(UTTT_PROF_ROWWISE, st);
  pack_read_kernel<<<148 * 8, 256, 0, st>>>((const float4*)w_up, (const float4*)w_gate, (const float4*)w_down, n_ug4,
                                            h / 4, (uint2*)packed_up_gate, (uint2*)down, n_d4);
  return launch_status();
}

extern "C" int uttt_rmsnorm(int rows, int d, const void* x, long long x_ld, const float* weight, float eps, void* out,
                            long long out_ld, void* stream) {
  UTTT_REQUIRE(rows > 0 && d > 0 && x && out, UTTT_ERR_INVALID);
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps(UTTT_PROF_ROWWISE, st);
  rmsnorm_kernel<<<rows, R_THREADS, 0, st>>>((const __nv_bfloat16*)x, x_ld, weight, d, eps, (__nv_bfloat16*)out,
                                             out_ld);
  return launch_status();
}

extern "C" int uttt_embed(int rows, int d, int V, const int* ids, const void* table, void* out, void* stream) {
  UTTT_REQUIRE(rows > 0 && d > 0 && ids && table && out, UTTT_ERR_INVALID);
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps(UTTT_PROF_ROWWISE, st);
  embed_kernel<<<rows, 256, 0, st>>>(ids, (const __nv_bfloat16*)table, d, V, (__nv_bfloat16*)out);
  return launch_status();
}

extern "C" int uttt_greedy_argmax(int rows, int V, const void* logits, int logits_f32, long long ld,
                                  int active_limit, int stop_free, int* ids, float* top2, void* stream) {
  UTTT_REQUIRE(rows > 0 && V > 6 && logits && ids && active_limit > 2, UTTT_ERR_INVALID);
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps(UTTT_PROF_ARGMAX, st);
  argmax_kernel<<<rows, R_THREADS, 0, st>>>(logits, logits_f32, ld, V, active_limit, stop_free, ids, top2);
  return launch_status();
}
