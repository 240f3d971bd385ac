// Slow-weight projections of the uTTT model on the tensor cores.
//
//   Y32[M_tok, N] (+)= X[M_tok, K] . W[N, K]^T      X, W BF16, Y32 FP32
//
// W is an nn.Linear weight (out x in, K-major) and X the packed token rows
// (K-major), so both arrive by TMA with no transpose.  The MMA runs with the
// weights as the 128-row M side and the tokens as N (16..256): decode batches
// have few tokens, prefill many.  A CTA owns 128 output features x one token
// tile x one K range; with several K ranges (split-K, used when the output is
// too narrow to fill the GPU) the partials are red.add-ed into Y32.  The
// row-wise finishing kernel then applies the reference's epilogue of each
// projection (residual add, RMSNorm, sigmoid gates) and writes BF16.
#include <string.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "host_util.cuh"

namespace cg = cooperative_groups;

namespace uttt {
namespace {

constexpr int G_THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
constexpr int G_STAGES = 4;

struct GemmParams {
  int M, N, K, TN;
  int kb_per_split;
  int atomic;  // red.add (split-K) instead of stores
  float* y;    // (M, N) FP32
  int* status;
};

__global__ void __launch_bounds__(G_THREADS, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmW,
                                                            const __grid_constant__ CUtensorMap tmX,
                                                            const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[G_STAGES], empty[G_STAGES], done;
  __shared__ uint32_t tmem_slot;
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* base = smem_raw + pad;
  const int stage_bytes = 16384 + p.TN * 128;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * 128, m0 = blockIdx.y * p.TN;
  const int nkb_total = p.K / 64;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(nkb_total, kb0 + p.kb_per_split);
  const uint32_t ncols = p.TN <= 32 ? 32 : (p.TN <= 64 ? 64 : (p.TN <= 128 ? 128 : 256));

  if (tid == 0) {
    for (int i = 0; i < G_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&done, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      // the weights do not depend on earlier launches: the first stages' W tiles are
      // requested before waiting for the previous kernel (which wrote X)
      const int npre = min(G_STAGES, kb1 - kb0);
      for (int it = 0; it < npre; ++it) {
        mbar_arrive_expect_tx(&full[it], (uint32_t)stage_bytes);
        tma_load_2d(base + it * stage_bytes, &tmW, &full[it], (kb0 + it) * 64, n0);
      }
      pdl_wait();
      pdl_trigger();
      for (int it = 0; it < npre; ++it) tma_load_2d(base + it * stage_bytes + 16384, &tmX, &full[it], (kb0 + it) * 64, m0);
      for (int kb = kb0 + npre, it = npre; kb < kb1; ++kb, ++it) {
        const int s = it % G_STAGES;
        mbar_wait(&empty[s], ((it / G_STAGES) & 1) ^ 1, p.status);
        uint8_t* st = base + s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)stage_bytes);
        tma_load_2d(st, &tmW, &full[s], kb * 64, n0);
        tma_load_2d(st + 16384, &tmX, &full[s], kb * 64, m0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(128, p.TN, false, false);
      for (int kb = kb0, it = 0; kb < kb1; ++kb, ++it) {
        const int s = it % G_STAGES;
        mbar_wait(&full[s], (it / G_STAGES) & 1, p.status);
        tc_fence_after();
        const uint32_t a = smem_u32(base + s * stage_bytes), bb = a + 16384;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_bf16(tmem, sdesc_sw128(a + ks * 32, 16, 1024), sdesc_sw128(bb + ks * 32, 16, 1024), idesc,
                   (it > 0 || ks > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(&done);
    }
  } else {
    // epilogue: lane = output feature, TMEM columns = tokens (Y32 was last written by an earlier launch)
    pdl_wait();
    mbar_wait(&done, 0, p.status);
    tc_fence_after();
    const int q = warp & 3;
    const int n = n0 + q * 32 + lane;
    for (int c0 = 0; c0 < p.TN; c0 += 16) {
      float v[16];
      tmem_ld16(tmem_addr(tmem, q * 32, c0), v);
      tmem_wait_ld();
      if (n < p.N) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int m = m0 + c0 + i;
          if (m < p.M) {
            float* dst = p.y + (size_t)m * p.N + n;
            if (p.atomic)
              red_add_f32(dst, v[i]);
            else
              *dst = v[i];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, ncols);
}

// ---------------------------------------------------------------------------
// Row-wise finishing of a projection: up to 6 column segments per row.  A row
// is striped over a cluster of CF CTAs (grid (M, CF); CF grows while the rows
// alone would leave SMs idle, so a decode batch of one row still spreads over
// 8 SMs), 4 independent loads per thread in flight; a row statistic (the
// RMSNorm sums of squares) is summed over the cluster's CTAs in distributed
// shared memory, in rank order.  The FP32 accumulator row is zeroed after use,
// so the next projection can accumulate into it without a memset.
// ---------------------------------------------------------------------------
constexpr int F_THREADS = 256;
constexpr int F_UNROLL = 4;

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

__device__ __forceinline__ float fblock_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < F_THREADS / 32; ++i) s += red[i];
  return s;
}

struct SegPack {
  UtttSegment s[6];
};

__device__ __forceinline__ float seg_value(const UtttSegment& sg, float v, int r, int i, float rinv) {
  switch (sg.op) {
    case UTTT_SEG_RESID:
      return __bfloat162float((reinterpret_cast<const __nv_bfloat16*>(sg.aux) + (size_t)r * sg.aux_ld)[i]) + bf16r(v);
    case UTTT_SEG_RMSNORM: {
      // F.rms_norm of the BF16 projection: FP32 statistics, weight applied in FP32
      float o = bf16r(v) * rinv;
      if (sg.aux) o *= bf16r(reinterpret_cast<const float*>(sg.aux)[i]);
      return o;
    }
    case UTTT_SEG_SIGMOID: {
      // scale * sigmoid(linear + bias) with the BF16 roundings of F.linear, sigmoid and the product
      const float lin = bf16r(v + (sg.aux ? reinterpret_cast<const float*>(sg.aux)[i] : 0.f));
      return bf16r(sg.scale * bf16r(sigmoidf_(lin)));
    }
    default:
      return v;
  }
}

// A row statistic summed over the CTAs of the row's cluster (slot si of each CTA's cred).
__device__ __forceinline__ float cluster_row_sum(float v, float* cred, int si, int CF) {
  if (CF == 1) return v;
  cg::cluster_group cl = cg::this_cluster();
  if (threadIdx.x == 0) cred[si] = v;
  cl.sync();
  float s = 0.f;
  for (int k = 0; k < CF; ++k) s += cl.map_shared_rank(cred, k)[si];
  return s;
}

__device__ __forceinline__ void row_sync(int CF) {
  if (CF == 1)
    __syncthreads();
  else
    cg::this_cluster().sync();
}

__global__ void __launch_bounds__(F_THREADS) finish_kernel(float* __restrict__ y, int N, int nseg,
                                                           const __grid_constant__ SegPack sp, float eps) {
  __shared__ float red[F_THREADS / 32];
  __shared__ float cred[6];
  const int CF = gridDim.y, r = blockIdx.x, tid = threadIdx.x;
  const int first = blockIdx.y * F_THREADS + tid, stride = CF * F_THREADS;   // this CTA's stripe of the row
  pdl_wait();
  pdl_trigger();
  float* yrow = y + (size_t)r * N;
  for (int si = 0; si < nseg; ++si) {
    const UtttSegment& sg = sp.s[si];
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(sg.out) + (size_t)r * sg.out_ld;
    float* outf = reinterpret_cast<float*>(sg.out) + (size_t)r * sg.out_ld;
    if (sg.op == UTTT_SEG_NORM) {
      // rms_norm of a BF16 row an earlier segment of this row has just written (every CTA of the cluster)
      row_sync(CF);
      const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(sg.aux) + (size_t)r * sg.aux_ld;
      const float* gamma = reinterpret_cast<const float*>(sg.aux2);
      float ss = 0.f;
      for (int i = first; i < sg.len; i += stride) {
        const float v = __bfloat162float(src[i]);
        ss += v * v;
      }
      const float rinv = rsqrtf(cluster_row_sum(fblock_sum(ss, red), cred, si, CF) / (float)sg.len + eps);
      for (int i = first; i < sg.len; i += stride) {
        float v = __bfloat162float(src[i]) * rinv;
        if (gamma) v *= bf16r(gamma[i]);
        if (sg.out_f32)
          outf[i] = v;
        else
          out[i] = __float2bfloat16(v);
      }
      continue;
    }
    const float* ys = yrow + sg.start;
    float rinv = 1.f;
    if (sg.op == UTTT_SEG_RMSNORM) {
      float ss = 0.f;
      for (int i = first; i < sg.len; i += stride) {
        const float v = bf16r(ys[i]);
        ss += v * v;
      }
      rinv = rsqrtf(cluster_row_sum(fblock_sum(ss, red), cred, si, CF) / (float)sg.len + eps);
    }
    for (int i0 = first; i0 < sg.len; i0 += stride * F_UNROLL) {
      float v[F_UNROLL];
#pragma unroll
      for (int u = 0; u < F_UNROLL; ++u) {
        const int i = i0 + u * stride;
        v[u] = i < sg.len ? ys[i] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < F_UNROLL; ++u) {
        const int i = i0 + u * stride;
        if (i < sg.len) {
          const float o = seg_value(sg, v[u], r, i, rinv);
          if (sg.out_f32)
            outf[i] = o;
          else
            out[i] = __float2bfloat16(o);
        }
      }
    }
  }
  // every segment of every CTA has read this row (and its partial sums) before it is cleared
  row_sync(CF);
  for (int i = first; i < N; i += stride) yrow[i] = 0.f;   // leave the accumulator zero for the next call
}

}  // namespace
}  // namespace uttt

using namespace uttt;

extern "C" size_t uttt_linear_workspace(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  return 256 + ws_round((size_t)M * N * sizeof(float));
}

extern "C" int uttt_linear(int M, int N, int K, const void* x, const void* w, int nseg, const UtttSegment* segs,
                           float eps, void* workspace, size_t workspace_bytes, void* stream) {
  UTTT_REQUIRE(M > 0 && N > 0 && K > 0 && x && w && workspace && segs, UTTT_ERR_INVALID);
  UTTT_REQUIRE(nseg >= 1 && nseg <= 6, UTTT_ERR_INVALID);
  UTTT_REQUIRE(K % 64 == 0, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(workspace_bytes >= uttt_linear_workspace(M, N), UTTT_ERR_WORKSPACE);
  for (int i = 0; i < nseg; ++i) {
    UTTT_REQUIRE(segs[i].op >= UTTT_SEG_STORE && segs[i].op <= UTTT_SEG_NORM, UTTT_ERR_INVALID);
    UTTT_REQUIRE(segs[i].len > 0 && segs[i].out, UTTT_ERR_INVALID);
    UTTT_REQUIRE(segs[i].op == UTTT_SEG_NORM || (segs[i].start >= 0 && segs[i].start + segs[i].len <= N),
                 UTTT_ERR_INVALID);
    UTTT_REQUIRE((segs[i].op != UTTT_SEG_RESID && segs[i].op != UTTT_SEG_NORM) || segs[i].aux, UTTT_ERR_INVALID);
  }
  cudaStream_t st = (cudaStream_t)stream;
  WsCursor ws(workspace, workspace_bytes);
  float* y = ws.take<float>((size_t)M * N);
  if (!ws.ok()) return UTTT_ERR_WORKSPACE;

  // token tile: the whole batch when it fits one MMA (decode), else 128
  int TN = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  if (M > 128 && M <= 256) TN = ((M + 15) / 16) * 16;
  const int mtiles = (M + TN - 1) / TN;
  const int ntiles = (N + 127) / 128;
  const int nkb = K / 64;
  // split K until the grid covers the GPU (at least 1 k-block of 64 per split)
  int splits = 1;
  while (ntiles * mtiles * splits < 148 && splits * 2 <= nkb) splits *= 2;
  const int kbps = (nkb + splits - 1) / splits;
  splits = (nkb + kbps - 1) / kbps;

  GemmParams p;
  p.M = M; p.N = N; p.K = K; p.TN = TN; p.kb_per_split = kbps; p.atomic = splits > 1; p.y = y;
  p.status = ws_status(workspace);
  CUtensorMap tmW, tmX;
  {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)N}, str[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {64, 128};
    UTTT_TRY(make_tmap_bf16(&tmW, w, 2, dims, str, box));
  }
  {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)M}, str[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {64, (uint32_t)TN};
    UTTT_TRY(make_tmap_bf16(&tmX, x, 2, dims, str, box));
  }
  const size_t smem = 1024 + (size_t)G_STAGES * (16384 + TN * 128);
  static DeviceOnce attr;
  UTTT_TRY(run_once_per_device(attr, [] {
    return cuda_status(cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)(1024 + G_STAGES * (16384 + 256 * 128))));
  }));
  {
    ProfScope ps(UTTT_PROF_GEMM, st);
    cudaLaunchConfig_t gc = {};
    gc.gridDim = dim3(ntiles, mtiles, splits);
    gc.blockDim = dim3(G_THREADS);
    gc.dynamicSmemBytes = smem;
    gc.stream = st;
    cudaLaunchAttribute ga[1] = {pdl_attribute()};
    gc.attrs = ga;
    gc.numAttrs = 1;
    if (cudaLaunchKernelEx(&gc, gemm_kernel, tmW, tmX, p) != cudaSuccess) return launch_status();
  }
  UTTT_TRY(launch_status());
  SegPack sp;
  memset(&sp, 0, sizeof(sp));
  for (int i = 0; i < nseg; ++i) sp.s[i] = segs[i];
  int CF = 1;   // CTAs per row (a cluster): spread narrow batches over the SMs
  while (CF < 8 && (long long)M * CF < 2LL * num_sms() && N > CF * F_THREADS * F_UNROLL) CF *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, CF);
  cfg.blockDim = dim3(F_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute attr1[2];
  attr1[0].id = cudaLaunchAttributeClusterDimension;
  attr1[0].val.clusterDim.x = 1;
  attr1[0].val.clusterDim.y = CF;
  attr1[0].val.clusterDim.z = 1;
  attr1[1] = pdl_attribute();
  cfg.attrs = attr1;
  cfg.numAttrs = 2;
  {
    ProfScope ps(UTTT_PROF_FINISH, st);
    if (cudaLaunchKernelEx(&cfg, finish_kernel, y, N, nseg, sp, eps) != cudaSuccess) return launch_status();
  }
  return launch_status();
}
