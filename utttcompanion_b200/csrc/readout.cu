// Decode-time fast-weight readout: one token per state, each state reading its
// own BF16 read copies (packed [W_up | W_gate] (d, 2h) and W_down (h, d)),
// the layout of SharedFastWeightPool.inference_read_weights
// (model/uttt_layer.py:648-668).  The work is a pair of GEMVs per state, so
// the kernel is bound by HBM: every weight byte is read exactly once with
// 16-byte coalesced loads straight into registers, the K dimension is split
// across the 8 warps of a CTA and reduced through shared memory.
//
// grid = (ceil(h / 128) hidden tiles, B states).  A CTA computes u, g for its
// 128 hidden units, h = silu(g) * u, then the partial z = h W_down[tile, :]
// and adds it into z (FP32, L2-resident) with one red.add per element.
#include "common.cuh"
#include "host_util.cuh"

namespace uttt {
namespace {

constexpr int GT = 128;        // hidden units per CTA
constexpr int GTHREADS = 256;  // 8 warps
constexpr int MAXD = 4096;

__device__ __forceinline__ void bf16x4_to_f32(const uint2& v, float (&f)[4]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
  const float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

__global__ void __launch_bounds__(GTHREADS) readout_gemv_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const __nv_bfloat16* __restrict__ wp,
                                                                const __nv_bfloat16* __restrict__ wd,
                                                                const int* __restrict__ state_index, int d, int h,
                                                                float* __restrict__ zacc) {
  __shared__ float xs[MAXD];
  __shared__ float part[8][2][GT];
  __shared__ float hs[GT];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y, j0 = blockIdx.x * GT;
  const int state = state_index ? state_index[b] : b;
  for (int i = tid; i < d; i += GTHREADS) xs[i] = __bfloat162float(x[(size_t)b * d + i]);
  __syncthreads();

  // ---- u, g for 128 hidden units: lane -> 4 columns, warp -> 1/8 of K (= d)
  const __nv_bfloat16* wrow = wp + (size_t)state * d * 2 * h;
  const int col = j0 + lane * 4;
  const bool cval = col < h;
  float au[4] = {0.f, 0.f, 0.f, 0.f}, ag[4] = {0.f, 0.f, 0.f, 0.f};
  const int kper = d / 8;
  const int k0 = warp * kper;
  if (cval) {
#pragma unroll 8
    for (int k = k0; k < k0 + kper; ++k) {
      const uint2 vu = __ldg(reinterpret_cast<const uint2*>(wrow + (size_t)k * 2 * h + col));
      const uint2 vg = __ldg(reinterpret_cast<const uint2*>(wrow + (size_t)k * 2 * h + h + col));
      float fu[4], fg[4];
      bf16x4_to_f32(vu, fu);
      bf16x4_to_f32(vg, fg);
      const float xv = xs[k];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        au[i] = fmaf(xv, fu[i], au[i]);
        ag[i] = fmaf(xv, fg[i], ag[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    part[warp][0][lane * 4 + i] = au[i];
    part[warp][1][lane * 4 + i] = ag[i];
  }
  __syncthreads();
  if (tid < GT) {
    float u = 0.f, g = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      u += part[w][0][tid];
      g += part[w][1][tid];
    }
    hs[tid] = (j0 + tid < h) ? g * sigmoidf_(g) * u : 0.f;
  }
  __syncthreads();

  // ---- partial z over this tile's 128 rows of W_down: warp -> 16 rows, lane -> 4 d columns
  const __nv_bfloat16* drow = wd + (size_t)state * h * d;
  float* zb = zacc + (size_t)b * 64 * d;   // row 0 of this state's 64-row z block
  for (int dc = 0; dc < d; dc += 128) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int r = 0; r < 16; ++r) {
      const int j = warp * 16 + r;
      if (j0 + j < h) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(drow + (size_t)(j0 + j) * d + dc + lane * 4));
        float f[4];
        bf16x4_to_f32(v, f);
        const float hv = hs[j];
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = fmaf(hv, f[i], acc[i]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) part[warp][0][lane * 4 + i] = acc[i];
    __syncthreads();
    if (tid < 128) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) s += part[w][0][tid];
      red_add_f32(zb + dc + tid, s);
    }
  }
}

}  // namespace

int launch_readout_gemv(int B, int d, int h, const __nv_bfloat16* x, const __nv_bfloat16* wp,
                        const __nv_bfloat16* wd, const int* state_index, float* zacc, cudaStream_t st) {
  if (d % 128 != 0 || d > MAXD) return UTTT_ERR_UNSUPPORTED;
  readout_gemv_kernel<<<dim3((h + GT - 1) / GT, B), GTHREADS, 0, st>>>(x, wp, wd, state_index, d, h, zacc);
  return launch_status();
}

}  // namespace uttt
