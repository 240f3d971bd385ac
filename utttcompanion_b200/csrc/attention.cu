// Sliding-window GQA attention of the uTTT blocks (SlidingWindowAttention,
// model/uttt_layer.py:961-1168) for packed multi-persona batches.
//
// Decode (one new token per row): RoPE of q and k at the row's own position,
// k/v written in place into the persona's KV ring at slot pos % W, then
// attention over the min(pos+1, W) valid slots.  The ring holds exactly the
// keys the reference's trimmed cache holds (the last W positions), so the
// softmax runs over the same set.  One cluster per (row, kv head): its S CTAs
// split the ring's slots (S grows while the batch alone would leave SMs idle);
// the n_rep query heads of the group share every K/V load.  Each CTA's softmax
// partial (max, sum, unnormalised output) is merged with the others' in
// distributed shared memory, in rank order.
//
// Prefill / chunk (T new tokens per row): RoPE into a contiguous per-row KV
// window buffer that starts with up to W-1 history positions, then causal
// sliding-window attention (query at absolute position p sees keys in
// (p - W, p]) on the tensor cores for head dims 64 and 128 (attn_prefill_tc_kernel);
// other head dims use a CUDA-core kernel (64 queries per CTA, two threads per
// query, 64-key tiles staged in shared memory).
//
// RoPE tables are the reference's FP32 cos/sin (RotaryEmbedding._build_cache,
// :910-933); like apply_rope on BF16 activations (:946-958) every product and
// the sum are rounded to BF16.
#include <cooperative_groups.h>

#include "common.cuh"
#include "host_util.cuh"

namespace cg = cooperative_groups;

namespace uttt {
namespace {

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16(x)); }

// rotate-half RoPE of element i of a head vector x (length hd) at position pos
__device__ __forceinline__ float rope_elem(const __nv_bfloat16* x, int i, int hd, const float* cosr,
                                           const float* sinr) {
  const int half = hd >> 1;
  const float xi = __bfloat162float(x[i]);
  const float rot = i < half ? -__bfloat162float(x[i + half]) : __bfloat162float(x[i - half]);
  return bfr(bfr(xi * bfr(cosr[i])) + bfr(rot * bfr(sinr[i])));
}

constexpr int DEC_THREADS = 256;
constexpr int MAX_HD = 128;
constexpr int MAX_REP = 8;
constexpr int MAX_W = 1024;

// ring slots per CTA, padded to 4 floats so the partial outputs after them stay 16-byte aligned
__host__ __device__ constexpr int dec_span_pad(int span) { return (span + 3) & ~3; }

__host__ __device__ constexpr size_t dec_smem_floats(int hd, int rep, int span) {
  return (size_t)rep * (hd + dec_span_pad(span) + DEC_THREADS / 32 + (DEC_THREADS / 32) * hd) + (size_t)rep * (hd + 2);
}

// grid (B, kv groups, S), cluster (1, 1, S); CTA k of a cluster takes ring
// slots [k*W/S, (k+1)*W/S), REP query heads per group.  Scores: every thread
// owns one ring slot and reads its whole K row with 16-byte loads (all slots'
// loads in flight at once); softmax over the slots in shared memory; output:
// HD/8 threads cover one V row with 16-byte loads, so a pass reads 256*8/HD
// rows; every query head of the group accumulates from the same V load, the
// rows of a warp are combined by shuffles and the warps through shared memory.
// Shared memory (dynamic): q [REP][HD], p [REP][span padded to 4], reductions [REP][8],
// partial outputs [8][REP][HD], the CTA's merged partial [REP][HD] + max and
// sum [REP][2] (read by the cluster).
template <int HD, int REP>
__global__ void __launch_bounds__(DEC_THREADS) attn_decode_kernel(
    const __nv_bfloat16* __restrict__ qkv, int qkv_ld, const int* __restrict__ pos, const int* __restrict__ slot,
    __nv_bfloat16* __restrict__ kring, __nv_bfloat16* __restrict__ vring, int n_kv, int W,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, float scale, __nv_bfloat16* __restrict__ out,
    int out_ld) {
  const int S = gridDim.z, span = W / S, s_lo = blockIdx.z * span, sp = dec_span_pad(span);
  extern __shared__ float dsm[];
  float* qs = dsm;                                    // [REP][HD]
  float* ps = qs + REP * HD;                          // [REP][sp]
  float* red = ps + (size_t)REP * sp;                 // [REP][8]
  float* part = red + REP * (DEC_THREADS / 32);       // [8][REP][HD]
  float* cacc = part + (DEC_THREADS / 32) * REP * HD; // [REP][HD]
  float* cml = cacc + REP * HD;                       // [REP][2]: max, sum
  const int b = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_heads = n_kv * REP;
  pdl_wait();
  pdl_trigger();
  const int p = pos[b];
  const int sl = slot[b];
  const __nv_bfloat16* row = qkv + (size_t)b * qkv_ld;
  const float* cr = cos_t + (size_t)p * HD;
  const float* sr = sin_t + (size_t)p * HD;
  const size_t ring_base = (((size_t)sl * n_kv + g) * W) * HD;
  for (int i = tid; i < REP * HD; i += DEC_THREADS) {
    const int r = i / HD, e = i % HD;
    qs[i] = rope_elem(row + (size_t)(g * REP + r) * HD, e, HD, cr, sr);
  }
  const __nv_bfloat16* krow = row + (size_t)n_heads * HD + (size_t)g * HD;
  const __nv_bfloat16* vrow = row + (size_t)(n_heads + n_kv) * HD + (size_t)g * HD;
  const int ws = p % W;
  if (ws >= s_lo && ws < s_lo + span)   // the new slot is read by the CTA that owns it
    for (int e = tid; e < HD; e += DEC_THREADS) {
      kring[ring_base + (size_t)ws * HD + e] = __float2bfloat16(rope_elem(krow, e, HD, cr, sr));
      vring[ring_base + (size_t)ws * HD + e] = vrow[e];
    }
  __syncthreads();
  const int nvalid = p + 1 < W ? p + 1 : W;
  const int s_hi = min(s_lo + span, nvalid);   // may be empty (s_hi <= s_lo): the partial is then zero

  // ---- scores: one slot per thread
  float mloc[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) mloc[r] = -INFINITY;
  for (int s0 = s_lo; s0 < s_hi; s0 += DEC_THREADS) {
    const int s = s0 + tid;
    if (s < s_hi) {
      const uint4* kp = reinterpret_cast<const uint4*>(kring + ring_base + (size_t)s * HD);
      uint4 kv[HD / 8];
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) kv[c] = kp[c];
      float dot[REP];
#pragma unroll
      for (int r = 0; r < REP; ++r) dot[r] = 0.f;
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) {
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&kv[c]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h2[j]);
#pragma unroll
          for (int r = 0; r < REP; ++r) dot[r] += qs[r * HD + c * 8 + 2 * j] * f.x + qs[r * HD + c * 8 + 2 * j + 1] * f.y;
        }
      }
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        const float sc = dot[r] * scale;
        ps[(size_t)r * sp + (s - s_lo)] = sc;
        mloc[r] = fmaxf(mloc[r], sc);
      }
    }
  }
  // ---- softmax over the slots of every head
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float m = mloc[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[r * 8 + warp] = m;
  }
  __syncthreads();
  float mx[REP], lsum[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    mx[r] = -INFINITY;
    for (int w = 0; w < DEC_THREADS / 32; ++w) mx[r] = fmaxf(mx[r], red[r * 8 + w]);
    lsum[r] = 0.f;
  }
  __syncthreads();
  for (int s = s_lo + tid; s < s_hi; s += DEC_THREADS) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float e = __expf(ps[(size_t)r * sp + (s - s_lo)] - mx[r]);
      ps[(size_t)r * sp + (s - s_lo)] = e;
      lsum[r] += e;
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    const float l = warp_sum(lsum[r]);
    if (lane == 0) red[r * 8 + warp] = l;
  }
  __syncthreads();
  // ---- output: TPR threads per V row, 8 head-dim elements (16 bytes) each
  constexpr int TPR = HD / 8, RPI = DEC_THREADS / TPR;
  const int e8 = (tid % TPR) * 8, rsub = tid / TPR;
  float acc[REP][8];
#pragma unroll
  for (int r = 0; r < REP; ++r)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[r][i] = 0.f;
#pragma unroll 2
  for (int s = s_lo + rsub; s < s_hi; s += RPI) {
    const uint4 v4 = *reinterpret_cast<const uint4*>(vring + ring_base + (size_t)s * HD + e8);
    const float f[8] = {bf16_lo(v4.x), bf16_hi(v4.x), bf16_lo(v4.y), bf16_hi(v4.y),
                        bf16_lo(v4.z), bf16_hi(v4.z), bf16_lo(v4.w), bf16_hi(v4.w)};
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float pr = ps[(size_t)r * sp + (s - s_lo)];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[r][i] = fmaf(pr, f[i], acc[r][i]);
    }
  }
#pragma unroll
  for (int o = TPR; o < 32; o <<= 1)
#pragma unroll
    for (int r = 0; r < REP; ++r)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[r][i] += __shfl_xor_sync(0xffffffffu, acc[r][i], o);
  if (lane < TPR) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float4* pw = reinterpret_cast<float4*>(part + ((size_t)warp * REP + r) * HD + e8);
      pw[0] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
      pw[1] = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
    }
  }
  __syncthreads();
  for (int i = tid; i < REP * HD; i += DEC_THREADS) {
    const int r = i / HD, ee = i % HD;
    float a = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < DEC_THREADS / 32; ++w) {
      a += part[((size_t)w * REP + r) * HD + ee];
      l += red[r * 8 + w];
    }
    if (S == 1)
      out[(size_t)b * out_ld + (size_t)(g * REP + r) * HD + ee] = __float2bfloat16(a / l);
    else
      cacc[i] = a;
  }
  if (S == 1) return;
  if (tid == 0) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float l = 0.f;
      for (int w = 0; w < DEC_THREADS / 32; ++w) l += red[r * 8 + w];
      cml[2 * r] = mx[r];
      cml[2 * r + 1] = l;
    }
  }
  // ---- merge the cluster's partials: CTA k writes output elements k, k + S*256, ...
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  for (int i = blockIdx.z * DEC_THREADS + tid; i < REP * HD; i += S * DEC_THREADS) {
    const int r = i / HD;
    float M = -INFINITY;
    for (int k = 0; k < S; ++k) M = fmaxf(M, cl.map_shared_rank(cml, k)[2 * r]);
    float num = 0.f, den = 0.f;
    for (int k = 0; k < S; ++k) {
      const float* ml = cl.map_shared_rank(cml, k);
      const float m = ml[2 * r];
      if (m == -INFINITY) continue;   // a CTA whose slots are all beyond the valid ones
      const float sc = __expf(m - M);
      num += sc * cl.map_shared_rank(cacc, k)[i];
      den += sc * ml[2 * r + 1];
    }
    out[(size_t)b * out_ld + (size_t)(g * REP) * HD + i] = __float2bfloat16(num / den);
  }
  cl.sync();   // no CTA leaves while another still reads its partial
}

template <int HD, int REP>
int launch_attn_decode(int B, int n_kv, int W, const __nv_bfloat16* qkv, int qkv_ld, const int* pos, const int* slot,
                       __nv_bfloat16* kring, __nv_bfloat16* vring, const float* cos_t, const float* sin_t, float scale,
                       __nv_bfloat16* out, int out_ld, cudaStream_t st) {
  static DeviceOnce attr;
  UTTT_TRY(run_once_per_device(attr, [] {
    return cuda_status(cudaFuncSetAttribute(attn_decode_kernel<HD, REP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)(dec_smem_floats(HD, REP, MAX_W) * sizeof(float))));
  }));
  // split the ring over a cluster while the batch leaves SMs idle (at least 16 slots per CTA)
  int S = 1;
  while (S < 8 && (long long)B * n_kv * S < 2LL * num_sms() && W % (2 * S) == 0 && W / (2 * S) >= 16) S *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B, n_kv, S);
  cfg.blockDim = dim3(DEC_THREADS);
  cfg.dynamicSmemBytes = dec_smem_floats(HD, REP, W / S) * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = S;
  at[1] = pdl_attribute();
  cfg.attrs = at;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, attn_decode_kernel<HD, REP>, qkv, qkv_ld, pos, slot, kring, vring, n_kv, W, cos_t,
                         sin_t, scale, out, out_ld) != cudaSuccess)
    return launch_status();
  return launch_status();
}

template <int HD>
int attn_decode_rep(int rep, int B, int n_kv, int W, const __nv_bfloat16* qkv, int qkv_ld, const int* pos,
                    const int* slot, __nv_bfloat16* kring, __nv_bfloat16* vring, const float* cos_t, const float* sin_t,
                    float scale, __nv_bfloat16* out, int out_ld, cudaStream_t st) {
  switch (rep) {
#define UTTT_REP(R) \
  case R:           \
    return launch_attn_decode<HD, R>(B, n_kv, W, qkv, qkv_ld, pos, slot, kring, vring, cos_t, sin_t, scale, out, out_ld, st);
    UTTT_REP(1) UTTT_REP(2) UTTT_REP(3) UTTT_REP(4) UTTT_REP(5) UTTT_REP(6) UTTT_REP(7) UTTT_REP(8)
#undef UTTT_REP
    default:
      return UTTT_ERR_UNSUPPORTED;
  }
}

// RoPE of the new tokens' k into the KV window buffer (after `hist` history
// positions) and of q into qout; v copied.  One CTA per token row.
__global__ void rope_prefill_kernel(const __nv_bfloat16* __restrict__ qkv, int qkv_ld, int T, int start_pos,
                                    int n_heads, int n_kv, int hd, int hist, int L, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ qout,
                                    __nv_bfloat16* __restrict__ kbuf, __nv_bfloat16* __restrict__ vbuf) {
  const int bt = blockIdx.x;
  const int b = bt / T, t = bt % T;
  const int p = start_pos + t;
  const __nv_bfloat16* row = qkv + (size_t)bt * qkv_ld;
  const float* cr = cos_t + (size_t)p * hd;
  const float* sr = sin_t + (size_t)p * hd;
  for (int i = threadIdx.x; i < n_heads * hd; i += blockDim.x) {
    const int hh = i / hd, e = i % hd;
    qout[(size_t)bt * n_heads * hd + i] = __float2bfloat16(rope_elem(row + (size_t)hh * hd, e, hd, cr, sr));
  }
  for (int i = threadIdx.x; i < n_kv * hd; i += blockDim.x) {
    const int g = i / hd, e = i % hd;
    const size_t o = (((size_t)b * n_kv + g) * L + hist + t) * hd + e;
    kbuf[o] = __float2bfloat16(rope_elem(row + (size_t)n_heads * hd + (size_t)g * hd, e, hd, cr, sr));
    vbuf[o] = row[(size_t)(n_heads + n_kv) * hd + (size_t)g * hd + e];
  }
}

constexpr int PF_Q = 64;        // queries per CTA
constexpr int PF_KT = 64;       // keys per smem tile
constexpr int PF_THREADS = 128;  // two threads per query

template <int HD>
__global__ void __launch_bounds__(PF_THREADS) attn_prefill_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kbuf,
    const __nv_bfloat16* __restrict__ vbuf, int T, int hist, int L, int n_heads, int n_kv, int hd, int W, float scale,
    __nv_bfloat16* __restrict__ out) {
  __shared__ __nv_bfloat16 ks[PF_KT][MAX_HD];
  __shared__ __nv_bfloat16 vs[PF_KT][MAX_HD];
  const int qb = blockIdx.x, hh = blockIdx.y, b = blockIdx.z;
  const int g = hh / (n_heads / n_kv);
  const int tid = threadIdx.x, qi = tid >> 1, half = tid & 1;
  const int t = qb * PF_Q + qi;      // new-token index of this thread's query
  const bool qvalid = t < T;
  constexpr int hh2 = HD / 2;
  const int e0 = half * hh2;
  float qr[hh2], acc[hh2];
#pragma unroll
  for (int e = 0; e < hh2; ++e) {
    qr[e] = 0.f;
    acc[e] = 0.f;
  }
  if (qvalid) {
    const __nv_bfloat16* qp = q + (((size_t)b * T + t) * n_heads + hh) * HD + e0;
#pragma unroll
    for (int e = 0; e < hh2; ++e) qr[e] = __bfloat162float(qp[e]);
  }
  float m = -INFINITY, l = 0.f;
  const int kpos_q = hist + t;                           // this query's index in the KV buffer
  const int lo_blk = hist + qb * PF_Q - (W - 1);         // first key any query of the block needs
  const int hi_blk = hist + min(T, (qb + 1) * PF_Q) - 1;  // last key
  const int k0 = max(0, lo_blk);
  const __nv_bfloat16* kb = kbuf + (((size_t)b * n_kv + g) * L) * hd;
  const __nv_bfloat16* vb = vbuf + (((size_t)b * n_kv + g) * L) * hd;
  for (int kt = k0; kt <= hi_blk; kt += PF_KT) {
    __syncthreads();
    for (int i = tid; i < PF_KT * hd; i += PF_THREADS) {
      const int r = i / hd, e = i % hd;
      const int kk = kt + r;
      ks[r][e] = kk <= hi_blk ? kb[(size_t)kk * hd + e] : __float2bfloat16(0.f);
      vs[r][e] = kk <= hi_blk ? vb[(size_t)kk * hd + e] : __float2bfloat16(0.f);
    }
    __syncthreads();
    const int nk = min(PF_KT, hi_blk - kt + 1);
    for (int r = 0; r < nk; ++r) {
      const int kk = kt + r;
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < hh2; ++e) d += qr[e] * __bfloat162float(ks[r][e0 + e]);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      const bool ok = qvalid && kk <= kpos_q && kpos_q - kk < W;
      if (!ok) continue;
      d *= scale;
      const float mn = fmaxf(m, d);
      const float c = __expf(m - mn);
      const float pe = __expf(d - mn);
      l = l * c + pe;
#pragma unroll
      for (int e = 0; e < hh2; ++e) acc[e] = acc[e] * c + pe * __bfloat162float(vs[r][e0 + e]);
      m = mn;
    }
  }
  if (qvalid) {
    __nv_bfloat16* op = out + (((size_t)b * T + t) * n_heads + hh) * HD + e0;
#pragma unroll
    for (int e = 0; e < hh2; ++e) op[e] = __float2bfloat16(acc[e] / l);
  }
}

// ---------------------------------------------------------------------------
// Prefill / chunk attention on the tensor cores (head dim 64 or 128).
//
// One CTA per (query block, kv group, row): the REP query heads of the group
// and QB = 128 / REP queries stack into the 128 rows of the MMA (row i: query
// i / REP, head i % REP), so every K/V tile is read once for the whole group.
// The keys the block needs ([first query - W + 1, last query]) stream through
// shared memory by TMA in 64-key tiles.  Two passes over the tiles:
//   pass 1: S = Q K^T (TMEM) -> exact row max m and sum l of exp(s - m);
//   pass 2: S again -> P = exp(s - m) / l -> O += P V (TMEM);
// so O never needs the rescaling of an online softmax.  P enters the MMA as two
// BF16 tiles, P_hi = bf16(P) and P_lo = bf16(P - P_hi), accumulated into the
// same O: about 16 significant bits, as the reference's FP32 softmax feeds its
// P.V product (an FP32 P would need the lower-rate TF32 kind and FP32 V tiles).  Warp 0 issues the TMA
// loads, warp 1 the MMAs, warps 2-5 own one row each (TMEM lane = row).
// ---------------------------------------------------------------------------
constexpr int TP_THREADS = 192;
constexpr int TP_NS = 3;   // K/V tiles in flight

template <int HD>
struct TpLayout {
  static constexpr int QB = HD / 64;            // 64-column blocks of a head vector
  static constexpr int Q_BYTES = 128 * HD * 2;  // Q: [128 rows][HD], K-major SW128, per 64-column block 16 KB
  static constexpr int KT_BYTES = 64 * HD * 2;  // one K (or V) tile: [64 keys][HD], per block 8 KB
  static constexpr int SLOT = 2 * KT_BYTES;     // K then V
  static constexpr int P_BYTES = 128 * 64 * 2;  // P_hi or P_lo: [128 rows][64 keys], K-major SW128
  static constexpr int SMEM = 1024 + Q_BYTES + TP_NS * SLOT + 4 * P_BYTES;   // 2 buffers x (P_hi, P_lo)
};

template <int HD>
__global__ void __launch_bounds__(TP_THREADS, 1) attn_prefill_tc_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
    const __nv_bfloat16* __restrict__ q, int T, int hist, int L, int n_heads, int n_kv, int rep, int W, float scale,
    __nv_bfloat16* __restrict__ out) {
  using LY = TpLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t kv_full[TP_NS], kv_empty[TP_NS], s_full[2], s_empty[2], p_full[2], p_empty[2], q_ready,
      o_done;
  __shared__ uint32_t tmem_slot;
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sQ = base;
  uint8_t* sKV = sQ + LY::Q_BYTES;
  uint8_t* sP = sKV + TP_NS * LY::SLOT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int QBK = 128 / rep;                       // queries per block
  const int lo = max(0, hist + qb * QBK - (W - 1));
  const int hi = hist + min(T, (qb + 1) * QBK) - 1;
  const int ntiles = (hi - lo) / 64 + 1;
  const int row0 = (b * n_kv + g) * L;             // first KV-buffer row of this (row, group)

  if (tid == 0) {
    for (int i = 0; i < TP_NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(&q_ready, 128);
    mbar_init(&o_done, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;       // S: 2 x 64 columns, O: HD columns

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      // pass 1: K of tiles 0..n-1; pass 2: K and V of tiles 0..n-1 (slot = sequence % TP_NS)
      for (int it = 0; it < 2 * ntiles; ++it) {
        const int s = it % TP_NS, j = it < ntiles ? it : it - ntiles;
        const bool with_v = it >= ntiles;
        mbar_wait(&kv_empty[s], ((it / TP_NS) & 1) ^ 1, nullptr);
        uint8_t* dst = sKV + s * LY::SLOT;
        mbar_arrive_expect_tx(&kv_full[s], (uint32_t)(with_v ? 2 : 1) * LY::KT_BYTES);
#pragma unroll
        for (int h = 0; h < LY::QB; ++h) tma_load_2d(dst + h * 8192, &tmK, &kv_full[s], h * 64, row0 + lo + j * 64);
        if (with_v)
#pragma unroll
          for (int h = 0; h < LY::QB; ++h)
            tma_load_2d(dst + LY::KT_BYTES + h * 8192, &tmV, &kv_full[s], h * 64, row0 + lo + j * 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, 64, false, false);   // A = Q K-major, B = K K-major
      const uint32_t id_o = idesc_bf16(128, HD, false, true);    // A = P K-major, B = V MN-major
      const uint32_t qa = smem_u32(sQ);
      mbar_wait(&q_ready, 0, nullptr);
      tc_fence_after();
      auto issue_s = [&](int it) {                 // S tile of sequence it into TMEM buffer it & 1
        const int s = it % TP_NS, sb = it & 1;
        mbar_wait(&kv_full[s], (it / TP_NS) & 1, nullptr);
        mbar_wait(&s_empty[sb], ((it >> 1) & 1) ^ 1, nullptr);
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + s * LY::SLOT);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          mma_bf16(tS + sb * 64, sdesc_sw128(qa + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024),
                   sdesc_sw128(ka + (k >> 2) * 8192 + (k & 3) * 32, 16, 1024), id_s, k > 0 ? 1u : 0u);
        mma_commit(&s_full[sb]);
      };
      for (int it = 0; it < ntiles; ++it) {        // pass 1
        issue_s(it);
        mma_commit(&kv_empty[it % TP_NS]);
      }
      issue_s(ntiles);                             // pass 2: S of tile j + 1 goes out before P V of tile j
      for (int j = 0; j < ntiles; ++j) {
        if (j + 1 < ntiles) issue_s(ntiles + j + 1);
        const int it = ntiles + j, s = it % TP_NS, pb = j & 1;
        mbar_wait(&p_full[pb], (j >> 1) & 1, nullptr);
        tc_fence_after();
        const uint32_t va = smem_u32(sKV + s * LY::SLOT + LY::KT_BYTES), pa = smem_u32(sP + pb * 2 * LY::P_BYTES);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // P_hi V
          mma_bf16(tO, sdesc_sw128(pa + k * 32, 16, 1024), sdesc_sw128(va + k * 2048, 8192, 1024), id_o,
                   (j > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // + P_lo V
          mma_bf16(tO, sdesc_sw128(pa + LY::P_BYTES + k * 32, 16, 1024), sdesc_sw128(va + k * 2048, 8192, 1024),
                   id_o, 1u);
        mma_commit(&p_empty[pb]);
        mma_commit(&kv_empty[s]);
      }
      mma_commit(&o_done);
    }
  } else {
    // ---- one row per thread: row i = query i / rep, head i % rep of the group
    const int i = (warp & 3) * 32 + lane;
    const int tq = i / rep, r = i - tq * rep, t = qb * QBK + tq;
    const bool valid = i < rep * QBK && t < T;
    const int kpos = hist + t;                     // this query's index in the KV buffer
    const size_t qrow = ((size_t)b * T + t) * n_heads + (size_t)g * rep + r;
    {
      const uint4* src = reinterpret_cast<const uint4*>(q + qrow * HD);
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) {
        const uint4 v = valid ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(sQ + (c >> 3) * 16384 + sw128_offset(i, (c & 7) * 16)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&q_ready);
    }
    const uint32_t trow = (uint32_t)((warp & 3) * 32);
    float m = -INFINITY, l = 0.f;
    for (int it = 0; it < 2 * ntiles; ++it) {
      const int j = it < ntiles ? it : it - ntiles, sb = it & 1;
      const int kt = lo + j * 64;
      mbar_wait(&s_full[sb], (it >> 1) & 1, nullptr);
      tc_fence_after();
      float sv[64];
#pragma unroll
      for (int c = 0; c < 64; c += 16) tmem_ld16(tmem_addr(tS + sb * 64, trow, c), *reinterpret_cast<float(*)[16]>(&sv[c]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      // key kt + c is visible to this query when it is in (kpos - W, kpos]
      const int cmax = valid ? min(63, kpos - kt) : -1;        // keys past kpos are masked
      const int cmin = valid ? max(0, kpos - W + 1 - kt) : 64;  // keys at or before kpos - W are masked
      if (it < ntiles) {
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c >= cmin && c <= cmax) mt = fmaxf(mt, sv[c] * scale);
        if (mt > -INFINITY) {
          const float mn = fmaxf(m, mt);
          float sum = 0.f;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= cmin && c <= cmax) sum += __expf(sv[c] * scale - mn);
          l = (m > -INFINITY ? l * __expf(m - mn) : 0.f) + sum;
          m = mn;
        }
      } else {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int pb = j & 1;
        mbar_wait(&p_empty[pb], ((j >> 1) & 1) ^ 1, nullptr);
        uint8_t* phi = sP + pb * 2 * LY::P_BYTES;
        uint8_t* plo = phi + LY::P_BYTES;
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          float pv[8], lo8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int cc = c + e;
            pv[e] = (cc >= cmin && cc <= cmax) ? __expf(sv[cc] * scale - m) * inv : 0.f;
            lo8[e] = pv[e] - __bfloat162float(__float2bfloat16(pv[e]));
          }
          uint4 pk, pl;
          pk.x = pack_bf16x2(pv[0], pv[1]);
          pk.y = pack_bf16x2(pv[2], pv[3]);
          pk.z = pack_bf16x2(pv[4], pv[5]);
          pk.w = pack_bf16x2(pv[6], pv[7]);
          pl.x = pack_bf16x2(lo8[0], lo8[1]);
          pl.y = pack_bf16x2(lo8[2], lo8[3]);
          pl.z = pack_bf16x2(lo8[4], lo8[5]);
          pl.w = pack_bf16x2(lo8[6], lo8[7]);
          *reinterpret_cast<uint4*>(phi + sw128_offset(i, c * 2)) = pk;
          *reinterpret_cast<uint4*>(plo + sw128_offset(i, c * 2)) = pl;
        }
        fence_proxy_async_smem();
        mbar_arrive(&p_full[pb]);
      }
    }
    // ---- O (TMEM) -> BF16 rows of out
    mbar_wait(&o_done, 0, nullptr);
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < HD; c += 16) {
      float ov[16];
      tmem_ld16(tmem_addr(tO, trow, c), ov);
      tmem_wait_ld();
      if (valid) {
        uint4 a, bq;
        a.x = pack_bf16x2(ov[0], ov[1]);   a.y = pack_bf16x2(ov[2], ov[3]);
        a.z = pack_bf16x2(ov[4], ov[5]);   a.w = pack_bf16x2(ov[6], ov[7]);
        bq.x = pack_bf16x2(ov[8], ov[9]);  bq.y = pack_bf16x2(ov[10], ov[11]);
        bq.z = pack_bf16x2(ov[12], ov[13]); bq.w = pack_bf16x2(ov[14], ov[15]);
        uint4* dst = reinterpret_cast<uint4*>(out + qrow * HD + c);
        dst[0] = a;
        dst[1] = bq;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 256);
}

// Copy the last min(W, L) positions of a KV window buffer into the ring slots
// of the persona: position p -> slot p % W.
__global__ void ring_fill_kernel(const __nv_bfloat16* __restrict__ kbuf, const __nv_bfloat16* __restrict__ vbuf,
                                 int L, int end_pos, const int* __restrict__ slot, int n_kv, int hd, int W,
                                 __nv_bfloat16* __restrict__ kring, __nv_bfloat16* __restrict__ vring) {
  const int b = blockIdx.y, g = blockIdx.z;
  const int n = L < W ? L : W;
  const int sl = slot[b];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * hd; i += gridDim.x * blockDim.x) {
    const int j = i / hd, e = i % hd;
    const int li = L - n + j;              // index in the buffer
    const int p = end_pos - n + j;         // absolute position
    const size_t src = (((size_t)b * n_kv + g) * L + li) * hd + e;
    const size_t dst = ((((size_t)sl * n_kv + g) * W) + (p % W)) * hd + e;
    kring[dst] = kbuf[src];
    vring[dst] = vbuf[src];
  }
}

}  // namespace
}  // namespace uttt

using namespace uttt;

extern "C" int uttt_attn_decode(int B, int n_heads, int n_kv, int hd, int W, const void* qkv, int qkv_ld,
                                const int* pos, const int* slot, void* k_ring, void* v_ring, const float* rope_cos,
                                const float* rope_sin, void* out, int out_ld, void* stream) {
  UTTT_REQUIRE(B > 0 && n_heads > 0 && n_kv > 0 && hd > 0 && W > 0, UTTT_ERR_INVALID);
  UTTT_REQUIRE(qkv && pos && slot && k_ring && v_ring && rope_cos && rope_sin && out, UTTT_ERR_INVALID);
  UTTT_REQUIRE(n_heads % n_kv == 0 && n_heads / n_kv <= MAX_REP, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(hd == 32 || hd == 64 || hd == 128, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(W <= MAX_W, UTTT_ERR_UNSUPPORTED);
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps(UTTT_PROF_ATTN, st);
  const float scale = 1.f / sqrtf((float)hd);
  const int rep = n_heads / n_kv;
  auto q = (const __nv_bfloat16*)qkv;
  auto kr = (__nv_bfloat16*)k_ring;
  auto vr = (__nv_bfloat16*)v_ring;
  auto o = (__nv_bfloat16*)out;
  if (hd == 32) return attn_decode_rep<32>(rep, B, n_kv, W, q, qkv_ld, pos, slot, kr, vr, rope_cos, rope_sin, scale, o, out_ld, st);
  if (hd == 64) return attn_decode_rep<64>(rep, B, n_kv, W, q, qkv_ld, pos, slot, kr, vr, rope_cos, rope_sin, scale, o, out_ld, st);
  return attn_decode_rep<128>(rep, B, n_kv, W, q, qkv_ld, pos, slot, kr, vr, rope_cos, rope_sin, scale, o, out_ld, st);
}

extern "C" int uttt_attn_prefill(int B, int T, int start_pos, int hist, int n_heads, int n_kv, int hd, int W,
                                 const void* qkv, int qkv_ld, const float* rope_cos, const float* rope_sin,
                                 void* q_scratch, void* k_buf, void* v_buf, void* out, void* stream) {
  UTTT_REQUIRE(B > 0 && T > 0 && start_pos >= 0 && hist >= 0 && n_heads > 0 && n_kv > 0 && hd > 0 && W > 0,
               UTTT_ERR_INVALID);
  UTTT_REQUIRE(qkv && rope_cos && rope_sin && q_scratch && k_buf && v_buf && out, UTTT_ERR_INVALID);
  UTTT_REQUIRE(hist <= start_pos && hist <= W - 1, UTTT_ERR_INVALID);
  UTTT_REQUIRE(n_heads % n_kv == 0 && (hd == 32 || hd == 64 || hd == 128), UTTT_ERR_UNSUPPORTED);
  cudaStream_t st = (cudaStream_t)stream;
  const int L = hist + T;
  ProfScope ps(UTTT_PROF_ATTN, st);
  rope_prefill_kernel<<<B * T, 128, 0, st>>>((const __nv_bfloat16*)qkv, qkv_ld, T, start_pos, n_heads, n_kv, hd,
                                             hist, L, rope_cos, rope_sin, (__nv_bfloat16*)q_scratch,
                                             (__nv_bfloat16*)k_buf, (__nv_bfloat16*)v_buf);
  UTTT_TRY(launch_status());
  const float scale = 1.f / sqrtf((float)hd);
  const int rep = n_heads / n_kv;
  if ((hd == 64 || hd == 128) && rep <= 8) {
    // tensor-core path: K / V window buffers as 2-D [B * n_kv * L rows][hd] maps, 64 x 64 boxes
    CUtensorMap tmK, tmV;
    const uint64_t dims[2] = {(uint64_t)hd, (uint64_t)B * n_kv * L}, str[1] = {(uint64_t)hd * 2};
    const uint32_t box[2] = {64, 64};
    UTTT_TRY(make_tmap_bf16(&tmK, k_buf, 2, dims, str, box));
    UTTT_TRY(make_tmap_bf16(&tmV, v_buf, 2, dims, str, box));
    const int qbk = 128 / rep;
    const dim3 tgrid((T + qbk - 1) / qbk, n_kv, B);
#define UTTT_TP(HDV)                                                                                            \
  do {                                                                                                          \
    static DeviceOnce attr_set;                                                                                 \
    UTTT_TRY(run_once_per_device(attr_set, [] {                                                                 \
      return cuda_status(cudaFuncSetAttribute(attn_prefill_tc_kernel<HDV>,                                      \
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, TpLayout<HDV>::SMEM)); \
    }));                                                                                                        \
    attn_prefill_tc_kernel<HDV><<<tgrid, TP_THREADS, TpLayout<HDV>::SMEM, st>>>(                                \
        tmK, tmV, (const __nv_bfloat16*)q_scratch, T, hist, L, n_heads, n_kv, rep, W, scale, (__nv_bfloat16*)out); \
  } while (0)
    if (hd == 64)
      UTTT_TP(64);
    else
      UTTT_TP(128);
#undef UTTT_TP
    return launch_status();
  }
  const dim3 grid((T + PF_Q - 1) / PF_Q, n_heads, B);
#define UTTT_PF(HDV)                                                                                          \
  attn_prefill_kernel<HDV><<<grid, PF_THREADS, 0, st>>>((const __nv_bfloat16*)q_scratch,                       \
                                                       (const __nv_bfloat16*)k_buf, (const __nv_bfloat16*)v_buf, \
                                                       T, hist, L, n_heads, n_kv, hd, W, scale, (__nv_bfloat16*)out)
  if (hd == 32)
    UTTT_PF(32);
  else if (hd == 64)
    UTTT_PF(64);
  else
    UTTT_PF(128);
#undef UTTT_PF
  return launch_status();
}

extern "C" int uttt_kv_ring_fill(int B, int L, int end_pos, int n_kv, int hd, int W, const void* k_buf,
                                 const void* v_buf, const int* slot, void* k_ring, void* v_ring, void* stream) {
  UTTT_REQUIRE(B > 0 && L > 0 && end_pos >= L && n_kv > 0 && hd > 0 && W > 0, UTTT_ERR_INVALID);
  UTTT_REQUIRE(k_buf && v_buf && slot && k_ring && v_ring, UTTT_ERR_INVALID);
  cudaStream_t st = (cudaStream_t)stream;
  ring_fill_kernel<<<dim3(8, B, n_kv), 256, 0, st>>>((const __nv_bfloat16*)k_buf, (const __nv_bfloat16*)v_buf, L,
                                                    end_pos, slot, n_kv, hd, W, (__nv_bfloat16*)k_ring,
                                                    (__nv_bfloat16*)v_ring);
  return launch_status();
}
