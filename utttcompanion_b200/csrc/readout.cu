// Decode-time fast-weight readout: one token per state, each state reading its
// own BF16 read copies (packed [W_up | W_gate] (d, 2h) and W_down (h, d)),
// the layout of SharedFastWeightPool.inference_read_weights
// (model/uttt_layer.py:648-668), and returning x + LN(z) as
// swiglu_packed_forward does (:211-257).  The work is a pair of GEMVs per
// state, so the kernel is bound by HBM: every weight byte is read exactly
// once with 16-byte coalesced loads straight into registers.
//
// grid = (ceil(h / 128) hidden tiles, B states, KS splits), 8 warps.  A CTA
// computes u, g for its 128 hidden units over its K-slice of d rows (one warp
// instruction covers a row of both: lanes 0-15 read u, lanes 16-31 read g; the
// warps split the slice), h = silu(g) * u, then the partial z = h W_down[tile, :]
// over its slice of d columns (the warps split the tile's rows), reduced in
// shared memory and added into z (FP32) with one red.add per column.  With
// KS > 1 the KS CTAs of a tile form one thread-block cluster: their partial u, g
// meet in distributed shared memory, summed in rank order by every CTA, so all
// of them hold the same h.  KS grows when B * tiles would leave SMs idle (one
// persona of the 1.58B model has 54 tiles on 148 SMs): each CTA then streams
// 1/KS of the tile's bytes.  KS (2..8, not only powers of two) is the largest
// split whose clusters all fit on the GPU at once (the occupancy API counts
// them; 8-CTA clusters of this kernel fit 48 at a time, so one 1.58B persona's
// 54 tiles use smaller clusters in a single wave).  The last CTA of a state to finish (device-scope
// counter) applies the LayerNorm and the residual.  u, g, silu(g), h and z are
// rounded to BF16 where the reference's autocast rounds them.
#include <cooperative_groups.h>

#include "common.cuh"
#include "host_util.cuh"

namespace cg = cooperative_groups;

namespace uttt {
namespace {

constexpr int GT = 128;        // hidden units per CTA
constexpr int GTHREADS = 256;  // 8 warps
constexpr int MAXD = 4096;
constexpr int ZG = 512;        // z columns reduced per shared-memory pass

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x);
  f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
  f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z);
  f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
}

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16(v)); }

__device__ __forceinline__ float cta_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < GTHREADS / 32; ++i) s += red[i];
  return s;
}

// MD: the largest d of the instantiation (sizes the x stage and the LayerNorm
// registers); MINB: resident CTAs per SM the registers are budgeted for.
template <int MD, int MINB>
__global__ void __launch_bounds__(GTHREADS, MINB) readout_decode_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wp, const __nv_bfloat16* __restrict__ wd,
    const int* __restrict__ state_index, int d, int h, const float* __restrict__ ln_w,
    const float* __restrict__ ln_b, float eps, float* __restrict__ zacc, unsigned* __restrict__ done, void* out,
    int out_bf16) {
  // done == nullptr: partial mode (a slice of the hidden units): z only, no LayerNorm
  __shared__ __align__(16) float xs[MD];
  __shared__ __align__(16) float part[8][ZG];
  __shared__ float ug[2 * GT];
  __shared__ __align__(16) float ugp[2 * GT];   // this CTA's partial u, g (read by its cluster)
  __shared__ float hs[GT];
  __shared__ float red[GTHREADS / 32];
  __shared__ int last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y, j0 = blockIdx.x * GT;
  const int KS = gridDim.z, ks = blockIdx.z;
  const int kper = d / KS, kb = ks * kper, ke = kb + kper;   // this CTA's rows of W_up/W_gate, columns of W_down
  pdl_wait();      // launched after the accumulator memset: returns at once
  pdl_trigger();   // the projection after the readout may start its weight prefetch
  const int state = state_index ? state_index[b] : b;
  if (state < 0) {   // a padding row of a packed batch: no weights are read, out = x (whole clusters leave)
    if (blockIdx.x == 0 && ks == 0 && done != nullptr)
      for (int i = tid; i < d; i += GTHREADS) {
        const float xv = __bfloat162float(x[(size_t)b * d + i]);
        if (out_bf16)
          reinterpret_cast<__nv_bfloat16*>(out)[(size_t)b * d + i] = __float2bfloat16(xv);
        else
          reinterpret_cast<float*>(out)[(size_t)b * d + i] = xv;
      }
    return;
  }
  for (int i = tid; i < d / 8; i += GTHREADS) {
    float f[8];
    bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(x + (size_t)b * d) + i), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) xs[i * 8 + e] = f[e];
  }
  __syncthreads();

  // ---- u (lanes 0-15) and g (lanes 16-31), 8 columns per lane; warp w takes rows w, w+8, ...
  {
    const int c8 = (lane & 15) * 8;
    const size_t ld = (size_t)2 * h;
    const __nv_bfloat16* col = wp + (size_t)state * d * ld + (lane >> 4) * h + j0 + c8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (j0 + c8 < h) {
#pragma unroll 8
      for (int k = kb + warp; k < ke; k += 8) {
        float f[8];
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(col + (size_t)k * ld)), f);
        const float xv = xs[k];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(xv, f[e], acc[e]);
      }
    }
    float4* pw = reinterpret_cast<float4*>(&part[warp][lane * 8]);
    pw[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    pw[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
  {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += part[w][tid];
    if (KS == 1) {
      ug[tid] = round_bf16(s);
    } else {
      ugp[tid] = s;
    }
  }
  if (KS > 1) {
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();                                   // every partial of the cluster is in place
    float s = 0.f;
    for (int r = 0; r < KS; ++r) s += cl.map_shared_rank(ugp, r)[tid];
    ug[tid] = round_bf16(s);
    cl.sync();                                   // no CTA leaves while another still reads its partial
  }
  __syncthreads();
  if (tid < GT) {
    const float u = ug[tid], g = ug[GT + tid];
    const float sg = round_bf16(g * sigmoidf_(g));
    hs[tid] = (j0 + tid < h) ? round_bf16(sg * u) : 0.f;
  }
  __syncthreads();

  // ---- partial z: warp w takes the tile's rows 16w..16w+15, lane 8 columns of a 256-column chunk
  const __nv_bfloat16* drow = wd + (size_t)state * h * d + (size_t)j0 * d;
  float* zrow = zacc + (size_t)b * d;
  for (int c0 = kb; c0 < ke; c0 += ZG) {
    const int ncol = min(ZG, ke - c0);
    float acc[2][8];
#pragma unroll
    for (int cc = 0; cc < 2; ++cc)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[cc][e] = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const int j = warp * 16 + r;
      if (j0 + j < h) {
        const float hv = hs[j];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = cc * 256 + lane * 8;
          if (c < ncol) {
            float f[8];
            bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(drow + (size_t)j * d + c0 + c)), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[cc][e] = fmaf(hv, f[e], acc[cc][e]);
          }
        }
      }
    }
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = cc * 256 + lane * 8;
      if (c < ncol) {
        float4* pw = reinterpret_cast<float4*>(&part[warp][c]);
        pw[0] = make_float4(acc[cc][0], acc[cc][1], acc[cc][2], acc[cc][3]);
        pw[1] = make_float4(acc[cc][4], acc[cc][5], acc[cc][6], acc[cc][7]);
      }
    }
    __syncthreads();
    for (int t = tid; t < ncol; t += GTHREADS) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) s += part[w][t];
      red_add_f32(zrow + c0 + t, s);
    }
    __syncthreads();
  }

  // ---- the state's last CTA: out = x + LN(bf16(z)) * gamma + beta
  if (done == nullptr) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(done + b, 1u) == gridDim.x * gridDim.z - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  constexpr int NZ = MD / GTHREADS;
  float zv[NZ];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NZ; ++i) {
    const int c = tid + i * GTHREADS;
    zv[i] = 0.f;
    if (c < d) {
      zv[i] = round_bf16(__ldcg(zrow + c));
      sum += zv[i];
    }
  }
  const float dinv = 1.f / (float)d;
  const float mean = cta_sum(sum, red) * dinv;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NZ; ++i)
    if (tid + i * GTHREADS < d) sq += (zv[i] - mean) * (zv[i] - mean);
  const float rstd = rsqrtf(cta_sum(sq, red) * dinv + eps);
#pragma unroll
  for (int i = 0; i < NZ; ++i) {
    const int c = tid + i * GTHREADS;
    if (c < d) {
      const float y = xs[c] + ((zv[i] - mean) * rstd * ln_w[c] + ln_b[c]);
      if (out_bf16)
        reinterpret_cast<__nv_bfloat16*>(out)[(size_t)b * d + c] = __float2bfloat16(y);
      else
        reinterpret_cast<float*>(out)[(size_t)b * d + c] = y;
    }
  }
}

// out = x + LN(z) * gamma + beta for one row per CTA: the LayerNorm of a readout whose z was
// summed across ranks (hidden-dimension split); z_bf16: z rounded to BF16 first, as the decode
// readout does (the tensor-core readout of T > 1 tokens keeps z in FP32).
template <int MD>
__global__ void __launch_bounds__(GTHREADS) readout_finish_kernel(const float* __restrict__ z,
                                                                  const __nv_bfloat16* __restrict__ x, int d,
                                                                  const float* __restrict__ ln_w,
                                                                  const float* __restrict__ ln_b, float eps,
                                                                  void* out, int out_bf16, int z_bf16) {
  __shared__ float red[GTHREADS / 32];
  const int b = blockIdx.x, tid = threadIdx.x;
  constexpr int NZ = MD / GTHREADS;
  float zv[NZ];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NZ; ++i) {
    const int c = tid + i * GTHREADS;
    zv[i] = 0.f;
    if (c < d) {
      zv[i] = z[(size_t)b * d + c];
      if (z_bf16) zv[i] = round_bf16(zv[i]);
      sum += zv[i];
    }
  }
  const float dinv = 1.f / (float)d;
  const float mean = cta_sum(sum, red) * dinv;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NZ; ++i)
    if (tid + i * GTHREADS < d) sq += (zv[i] - mean) * (zv[i] - mean);
  const float rstd = rsqrtf(cta_sum(sq, red) * dinv + eps);
#pragma unroll
  for (int i = 0; i < NZ; ++i) {
    const int c = tid + i * GTHREADS;
    if (c < d) {
      const float y = __bfloat162float(x[(size_t)b * d + c]) + ((zv[i] - mean) * rstd * ln_w[c] + ln_b[c]);
      if (out_bf16)
        reinterpret_cast<__nv_bfloat16*>(out)[(size_t)b * d + c] = __float2bfloat16(y);
      else
        reinterpret_cast<float*>(out)[(size_t)b * d + c] = y;
    }
  }
}

}  // namespace

int launch_readout_finish(int B, int d, const float* z, const __nv_bfloat16* x, const float* ln_w, const float* ln_b,
                          float eps, void* out, int out_bf16, int z_bf16, cudaStream_t st) {
  if (d % 128 != 0 || d > MAXD) return UTTT_ERR_UNSUPPORTED;
  if (d <= 1024)
    readout_finish_kernel<1024><<<B, GTHREADS, 0, st>>>(z, x, d, ln_w, ln_b, eps, out, out_bf16, z_bf16);
  else
    readout_finish_kernel<MAXD><<<B, GTHREADS, 0, st>>>(z, x, d, ln_w, ln_b, eps, out, out_bf16, z_bf16);
  return launch_status();
}

// zacc: (B, d) FP32 zero on entry; done: (B) zero counters, or nullptr for a
// partial readout (z only).
int launch_readout_decode(int B, int d, int h, const __nv_bfloat16* x, const __nv_bfloat16* wp,
                          const __nv_bfloat16* wd, const int* state_index, const float* ln_w, const float* ln_b,
                          float eps, float* zacc, unsigned* done, void* out, int out_bf16, cudaStream_t st) {
  if (d % 128 != 0 || d > MAXD || h % 8 != 0) return UTTT_ERR_UNSUPPORTED;
  const int tiles = (h + GT - 1) / GT;
  const bool small = d <= 1024;
  const void* fn = small ? (const void*)readout_decode_kernel<1024, 4> : (const void*)readout_decode_kernel<MAXD, 3>;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(GTHREADS);
  cfg.stream = st;
  // The largest K split, 2..8 (a cluster of KS CTAs per tile, d / KS a multiple of 16 columns
  // so the 16-byte W_down loads stay aligned), whose B * tiles clusters are all resident at
  // once; a batch too large for any split to fit in one wave runs unsplit.
  static int ncl_cache[16][2][9];   // resident clusters of k CTAs per (device, variant); 0: unknown
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 15;
  int KS = 1;
  for (int k = 8; k >= 2; --k) {
    if (d % (16 * k) != 0) continue;
    int& ncl = ncl_cache[dev][small][k];
    if (ncl == 0) {
      cudaLaunchAttribute ca;
      ca.id = cudaLaunchAttributeClusterDimension;
      ca.val.clusterDim.x = 1;
      ca.val.clusterDim.y = 1;
      ca.val.clusterDim.z = k;
      cfg.gridDim = dim3(1, 1, k);
      cfg.attrs = &ca;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&ncl, fn, &cfg) != cudaSuccess || ncl <= 0) {
        cudaGetLastError();
        ncl = -1;
      }
    }
    if (ncl > 0 && (long long)tiles * B <= ncl) {
      KS = k;
      break;
    }
  }
  cfg.gridDim = dim3(tiles, B, KS);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = KS;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (d <= 1024)   // small states: 4 CTAs per SM keep a short launch in one wave
    e = cudaLaunchKernelEx(&cfg, readout_decode_kernel<1024, 4>, x, wp, wd, state_index, d, h, ln_w, ln_b, eps,
                           zacc, done, out, out_bf16);
  else
    e = cudaLaunchKernelEx(&cfg, readout_decode_kernel<MAXD, 3>, x, wp, wd, state_index, d, h, ln_w, ln_b, eps,
                           zacc, done, out, out_bf16);
  if (e != cudaSuccess) return UTTT_ERR_CUDA;
  return launch_status();
}

}  // namespace uttt
