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
// One CTA of 512 threads per row; 8 logits per 16-byte load when the rows
// are aligned; top-1 / top-2 merged by warp shuffles, then across warps.
constexpr int A_THREADS = 512;

struct Top2 {
  float v1, v2;
  int i1;
};

__device__ __forceinline__ Top2 top2_merge(Top2 a, Top2 b) {
  const bool bwins = b.v1 > a.v1 || (b.v1 == a.v1 && b.i1 < a.i1);
  Top2 o;
  o.v1 = bwins ? b.v1 : a.v1;
  o.i1 = bwins ? b.i1 : a.i1;
  o.v2 = bwins ? fmaxf(a.v1, b.v2) : fmaxf(a.v2, b.v1);
  return o;
}

__global__ void __launch_bounds__(A_THREADS) argmax_kernel(const void* __restrict__ logits, int logits_f32,
                                                           long long ld, int V, int active_limit, int stop_free,
                                                           int* __restrict__ ids, float* __restrict__ top2) {
  __shared__ Top2 red[A_THREADS / 32];
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lim = active_limit < V ? active_limit : V;
  Top2 t = {-INFINITY, -INFINITY, 0x7fffffff};
  auto consider = [&](int i, float v) {
    if (i >= lim || i == 0 || i == 1 || i == 3 || (stop_free && i < 6)) return;
    v = __bfloat162float(__float2bfloat16(v));
    if (v != v) v = -INFINITY;
    if (v > t.v1 || (v == t.v1 && i < t.i1)) {
      t.v2 = t.v1;
      t.v1 = v;
      t.i1 = i;
    } else if (v > t.v2) {
      t.v2 = v;
    }
  };
  const float* lf = reinterpret_cast<const float*>(logits) + (size_t)r * ld;
  const __nv_bfloat16* lb = reinterpret_cast<const __nv_bfloat16*>(logits) + (size_t)r * ld;
  // vector loads only when every 8-logit group stays inside an aligned row
  const bool vec = (ld % 8 == 0) && (V % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15u) == 0);
  if (vec) {
    for (int j = tid; j * 8 < lim; j += A_THREADS) {
      float v[8];
      if (logits_f32) {
        const float4 a = reinterpret_cast<const float4*>(lf)[2 * j], b = reinterpret_cast<const float4*>(lf)[2 * j + 1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 a = reinterpret_cast<const uint4*>(lb)[j];
        v[0] = bf16_lo(a.x); v[1] = bf16_hi(a.x); v[2] = bf16_lo(a.y); v[3] = bf16_hi(a.y);
        v[4] = bf16_lo(a.z); v[5] = bf16_hi(a.z); v[6] = bf16_lo(a.w); v[7] = bf16_hi(a.w);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) consider(j * 8 + e, v[e]);
    }
  } else {
    for (int i = tid; i < lim; i += A_THREADS)
      consider(i, logits_f32 ? lf[i] : __bfloat162float(lb[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Top2 u;
    u.v1 = __shfl_down_sync(0xffffffffu, t.v1, o);
    u.v2 = __shfl_down_sync(0xffffffffu, t.v2, o);
    u.i1 = __shfl_down_sync(0xffffffffu, t.i1, o);
    t = top2_merge(t, u);
  }
  if (lane == 0) red[warp] = t;
  __syncthreads();
  if (tid == 0) {
    Top2 a = red[0];
    for (int w = 1; w < A_THREADS / 32; ++w) a = top2_merge(a, red[w]);
    ids[r] = a.i1 < lim ? a.i1 : (stop_free ? 6 : 2) % lim;   // only when no candidate was finite
    if (top2) {
      top2[2 * r] = a.v1;
      top2[2 * r + 1] = a.v2;
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
  argmax_kernel<<<rows, A_THREADS, 0, st>>>(logits, logits_f32, ld, V, active_limit, stop_free, ids, top2);
  return launch_status();
}
