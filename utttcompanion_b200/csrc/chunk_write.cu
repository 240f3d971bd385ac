// Chunk-wise TTT write for B independent FP32 fast-weight states on the
// tcgen05 tensor cores.  Replaces fused_chunk_ttt_step and
// analytical_swiglu_chunk_grad (model/uttt_layer.py:279-534).
//
// One chunk is three (four with gradient clipping) launches over a grid of
// (h / 128 hidden tiles) x (B states):
//
//   fwd   U,G = K W_up, K W_gate        (tile: 128 hidden x 64 tokens, K = d)
//         H   = silu(G) * U              (FP32 in registers -> BF16 operand)
//         Z  += H W_down                 (partial over this hidden tile; FP32
//                                         red.add into an L2-resident buffer)
//   ln    per token: LayerNorm stats of Z, v_hat = k + LN(Z), err = v_hat - v,
//         token loss, dZ (analytical LayerNorm backward, BF16)
//   bwd   dH  = dZ W_down^T              (K = d)
//         dU  = dH * silu(G),  dG = dH * U * silu'(G)
//         gradW_up^T = dU^T K,  gradW_gate^T = dG^T K,  gradW_down^T = dZ^T H
//         (K = 64 tokens, per 128-wide slice of d)  then, in the epilogue,
//         S' = beta S - clip * grad,  W' = (1 - alpha_bar) W + S'  in FP32,
//         in place.  With clipping, a first bwd pass only accumulates the
//         squared gradient norm of each state.
//
// W masters are FP32 in HBM; software producer warps convert them to BF16
// straight into 128B-swizzled UMMA operand tiles.  Activation tiles (K, dZ)
// arrive by TMA.  All accumulators live in tensor memory.
#include <string.h>

#include "common.cuh"
#include "host_util.cuh"

namespace uttt {
namespace {

constexpr int HT = 128;            // hidden rows per CTA
constexpr int CT = 64;             // token columns (chunk padded to 64)
constexpr int NPROD = 256;         // producer / epilogue threads (8 warps)
constexpr int NTHREADS = NPROD + 64;  // + TMA warp + MMA warp
constexpr int NSLOT = 4;
constexpr int SLOT_BYTES = 40 * 1024;
constexpr int TMA_WARP = 8, MMA_WARP = 9;
constexpr int STORE_WARP = 10;            // bwd only: W' stores and staging refills
constexpr int BWD_THREADS = NPROD + 96;
constexpr int BWD_SLOT = 24 * 1024;

struct ChunkParams {
  int B, T, C, Cc, d, h, tok0;
  const float* w_up;   // (B, d, h)
  const float* w_gate;
  const float* w_down;  // (B, h, d)
  float* w_up_out;
  float* w_gate_out;
  float* w_down_out;
  const float* s_up;
  const float* s_gate;
  const float* s_down;
  float* s_up_out;
  float* s_gate_out;
  float* s_down_out;
  const float* eta;    // (B, T)
  const float* alpha;  // (B, T)
  const float* mask;   // (B, T) or null
  const float* ln_w;
  const float* ln_b;
  const __nv_bfloat16* k;  // (B, T, d)
  const __nv_bfloat16* v;
  float* zacc;     // (B, 64, d)
  float* u_save;   // (B, 64, hp)
  float* g_save;   // (B, 64, hp)
  __nv_bfloat16* dz;  // (B, 64, d)
  float* norm2;    // (B)
  float* token_loss;  // (B, T) or null
  void* out;          // (B, T, d) or null
  int out_bf16;
  float* clip_out;    // (B, n_chunks) or null
  int chunk_index;
  int n_chunks;
  int call_end;       // token index one past the last chunk of this call
  int tok0_next, Cc_next;  // the fused forward's chunk (bwd kernel with kFuse)
  int hp;             // hidden padded to 128
  int z_rows;         // rows of zacc per state (0: 64, the chunk tile)
  int tiles;          // fwd readout over all token tiles in one launch: grid (T/64, h/128, B)
  float beta, clip, eps, inv_scale;
  int* status;
  // weight source of the fwd kernel: element (state, k, j) of up/gate at
  // src_up + state*ss_ug + k*ld_ug + j, of down (state, j, dd) at
  // src_down + state*ss_d + j*d + dd.  state = state_index ? state_index[b] : b.
  const void* src_up;
  const void* src_gate;
  const void* src_down;
  long long ss_ug, ss_d;
  int ld_ug;
  const int* state_index;
  int n_states;        // > 0: state_index entries must be below it (checked on the device)
  // bwd d-split (gridDim.z CTAs of a cluster share one hidden tile of one state): the
  // partial dH / next-chunk U', G' of every CTA, [b][tile][rank][3][128 rows][64 tokens]
  // FP32, and per (b, tile) two arrival counters (zero before the launch)
  float* xch;
  unsigned* xflag;
  int dsplit;          // fwd kernel d-split (its kSplit variant): CTAs per (tile, row), folded into blockIdx.x
  // stability guard in the last update of a row (uttt_chunk_write_guarded): on the call's last chunk,
  // rows with g_final[b] != 0 get W <- W0 + g_keep (W - W0) (the elastic pull) right after their
  // update, and sum ||W - W0||^2 of the pulled tiles per matrix into g_sums[4 b + m]
  const float* g_w0_up;   // (d, h)
  const float* g_w0_gate;
  const float* g_w0_down; // (h, d)
  const int* g_final;     // (B) or null: no guard
  float* g_sums;          // (B, 4)
  float g_keep;
  // clip-norm runs: the norm pass (update = 0) stores its epilogue-1 operands, the swizzled
  // shared-memory images of dU, dG and H of every (row, tile), [b][tile][3][16 KB]; the update
  // pass (update = 1) copies them back instead of reading W_down again for dH
  uint8_t* ops;
  // clip-norm runs: per row the chunk's Gram matrices K K^T and dZ dZ^T, [b][2][64][64] FP32 (zero
  // before chunk_gram_kernel); with them the norm pass needs no weight-gradient tiles:
  // ||K^T dU||^2 = <K K^T, dU^T dU> over the 64 x 64 token pairs, and likewise for dG and H^T dZ
  float* gram;
};
constexpr int OPS_BYTES = 3 * 16384;   // one (row, tile) entry of ChunkParams::ops

template <typename WT>
struct Quad;
template <>
struct Quad<float> {  // 4 FP32 masters -> 4 BF16 (8 bytes)
  using V = float4;
  static __device__ __forceinline__ V load(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
  static __device__ __forceinline__ V zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ __forceinline__ uint2 pack(V v) {
    uint2 r;
    r.x = pack_bf16x2(v.x, v.y);
    r.y = pack_bf16x2(v.z, v.w);
    return r;
  }
};
template <>
struct Quad<__nv_bfloat16> {  // 4 BF16 read-copy values, stored as they are
  using V = uint2;
  static __device__ __forceinline__ V load(const __nv_bfloat16* p) {
    return __ldg(reinterpret_cast<const uint2*>(p));
  }
  static __device__ __forceinline__ V zero() { return make_uint2(0u, 0u); }
  static __device__ __forceinline__ uint2 pack(V v) { return v; }
};

// Per-state chunk statistics: number of valid tokens, masked mean of alpha,
// whether any token is valid (model/uttt_layer.py:371-378,501-520).
struct ChunkStats {
  float count;   // valid tokens (Cc without a mask)
  float alpha_bar;
  bool active;
  bool later_active;  // a later chunk of this call changes this state
};

__device__ ChunkStats chunk_stats(const ChunkParams& p, int b) {
  // executed by one warp
  const int lane = threadIdx.x & 31;
  float cnt = 0.f, asum = 0.f;
  for (int c = lane; c < p.Cc; c += 32) {
    const size_t idx = (size_t)b * p.T + p.tok0 + c;
    const float m = p.mask ? p.mask[idx] : 1.f;
    cnt += m;
    asum += p.alpha[idx] * m;
  }
  cnt = warp_sum(cnt);
  asum = warp_sum(asum);
  ChunkStats s;
  s.count = cnt;
  s.alpha_bar = p.mask ? asum / fmaxf(cnt, 1.f) : asum / (float)p.Cc;
  s.active = p.mask ? (cnt != 0.f) : true;
  bool later = false;
  const int lo = p.tok0 + p.Cc;
  if (!p.mask) {
    later = lo < p.call_end;
  } else {
    for (int c = lo + lane; c < p.call_end && !later; c += 32) later = p.mask[(size_t)b * p.T + c] != 0.f;
    later = __any_sync(0xffffffffu, later);
  }
  s.later_active = later;
  return s;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* raw) {
  const uint32_t pad = (1024u - (smem_u32(raw) & 1023u)) & 1023u;
  return raw + pad;
}

// ============================================================================
// fwd: U, G, H and the partial Z of one 128-row hidden tile
// ============================================================================
// d-split exchange: the producers of every CTA of a (tile, state) cluster store
// their partial values (NP parts of one hidden row x 32 token columns) into parts
// part0.. of their rank's slot, count themselves in on counter `flag_i`, wait
// (bounded) until every rank has, and replace the values with the sum over ranks
// in rank order, so all ranks hold the same bits.  A wait that runs out records
// UTTT_ERR_TIMEOUT and uses what it has.
// `pair` indexes the (tile, row) whose KS ranks exchange; their slots are [pair][rank][3][128][64].
template <int NP>
__device__ __forceinline__ void dsplit_exchange(float (&v)[NP][32], const ChunkParams& p, size_t pair, int KS,
                                                int rank, int part0, int flag_i, int row, int c0) {
  const size_t cell = pair * KS;
  auto at = [&](int r, int part) { return p.xch + (((cell + r) * 3 + part) * HT + row) * CT + c0; };
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    float* mine = at(rank, part0 + k);
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      *reinterpret_cast<float4*>(mine + i) = make_float4(v[k][i], v[k][i + 1], v[k][i + 2], v[k][i + 3]);
  }
  __threadfence();
  named_bar(1, NPROD);
  unsigned* flag = p.xflag + pair * 2 + flag_i;
  if (threadIdx.x == 0) {
    atomicAdd(flag, 1u);
    counter_wait(flag, (unsigned)KS, p.status, kMaxCounterPolls);
  }
  named_bar(1, NPROD);
  __threadfence();
#pragma unroll
  for (int k = 0; k < NP; ++k) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[k][i] = 0.f;
    for (int r = 0; r < KS; ++r) {
      const float* src = at(r, part0 + k);
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(src + i));
        v[k][i] += x.x;
        v[k][i + 1] += x.y;
        v[k][i + 2] += x.z;
        v[k][i + 3] += x.w;
      }
    }
  }
}

template <typename WT, bool kSplit>
__global__ void __launch_bounds__(NTHREADS, 1) chunk_fwd_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                const ChunkParams p) {
  using Q = Quad<WT>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[NSLOT], empty[NSLOT], ug_done, h_ready, zfull[2], zfree[2];
  __shared__ uint32_t tmem_slot;
  uint8_t* slots = align1024(smem_raw);
  uint8_t* sH = slots + NSLOT * SLOT_BYTES;  // 16 KB: MN-major [hh 128 rows][64 tokens]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // one chunk (t = hidden tile, b = state) or, in tiles mode, every 64-token tile of a readout
  // (x = token tile, fastest, so the CTAs that share a hidden tile's weights run together)
  // kSplit: the p.dsplit CTAs of a cluster (consecutive blockIdx.x) share one (tile, row) and each
  // reduces U, G over its share of d (exchanged before H) and forms Z for its share of d's columns
  const int KS = kSplit ? p.dsplit : 1;
  const int xb = kSplit ? (int)blockIdx.x / KS : (int)blockIdx.x, ksr = kSplit ? (int)blockIdx.x % KS : 0;
  const int t = p.tiles ? blockIdx.y : xb, b = p.tiles ? blockIdx.z : blockIdx.y;
  const int tok0 = p.tiles ? xb * CT : p.tok0;
  const int Cc = p.tiles ? min(CT, p.T - tok0) : p.Cc;
  const int zr = p.z_rows ? p.z_rows : CT;
  const size_t zrow0 = (size_t)b * zr + (p.tiles ? tok0 : 0);   // this tile's first zacc row
  const int h0 = t * HT;
  const int nkb = kSplit ? p.d / 64 / KS : p.d / 64, kb0 = ksr * nkb;     // local k-blocks of U, G
  const int nmt = kSplit ? p.d / 128 / KS : p.d / 128, mt0 = ksr * nmt;   // local d tiles of Z
  if (p.state_index && p.n_states > 0 && (unsigned)p.state_index[b] >= (unsigned)p.n_states) {
    if (tid == 0) set_status(p.status, UTTT_ERR_INVALID);   // a bad row -> state map entry: touch nothing
    return;
  }
  if (p.state_index && p.state_index[b] < 0) return;       // a padding row of a readout: no weights read

  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&full[i], NPROD + 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&ug_done, 1);
    mbar_init(&h_ready, NPROD);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&zfull[i], 1);
      mbar_init(&zfree[i], NPROD);
    }
    fence_mbarrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tU = tmem, tG = tmem + 64, tZ = tmem + 128;

  const int state = p.state_index ? p.state_index[b] : b;
  if (warp < 8) {
    // ------------------------------------------------------------ producers
    // BF16 read copies need no conversion: every 16-byte chunk of a k-block / W_down tile goes
    // straight into its swizzled operand slot by cp.async, kAhead ring items ahead of the one being
    // handed to the tensor cores, so ~3 x 32 KB per CTA are in flight without registers (register
    // loads kept ~32 KB in flight and left the BF16 readout at a third of HBM).  FP32 masters are
    // converted by the producers as they arrive.
    constexpr bool kAsync = sizeof(WT) == 2;
    constexpr int kAhead = NSLOT - 1;
    const int n_items = nkb + nmt;
    int it = 0;
    // ring item i: k-block i of U/G (i < nkb) or W_down tile i - nkb
    auto issue = [&](int i) {
      const int s = i % NSLOT;
      mbar_wait(&empty[s], ((i / NSLOT) & 1) ^ 1, p.status);
      uint8_t* base = slots + s * SLOT_BYTES;
      if (i < nkb) {
        // 64 rows (k) x 128 cols (hidden) of W_up and of W_gate: [64-col half][64 rows][128 B]
        const __nv_bfloat16* wu = reinterpret_cast<const __nv_bfloat16*>(p.src_up) + (size_t)state * p.ss_ug;
        const __nv_bfloat16* wg = reinterpret_cast<const __nv_bfloat16*>(p.src_gate) + (size_t)state * p.ss_ug;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int idx = tid + j * NPROD;  // 0..1023: 64 rows x 16 chunks of 8 columns
          const int kr = idx >> 4, c8 = (idx & 15) * 8;
          const int col = h0 + c8;
          const bool ok = col < p.h;
          const size_t off = (size_t)((kb0 + i) * 64 + kr) * p.ld_ug + (ok ? col : 0);
          const uint32_t o = (c8 >> 6) * 8192 + sw128_offset(kr, (c8 & 63) * 2);
          cp_async_16(base + o, wu + off, ok);
          cp_async_16(base + 16384 + o, wg + off, ok);
        }
      } else {
        // W_down rows of this hidden tile, d columns of tile mt: [dblk 2][hh 128][64 d]
        const int mt = i - nkb;
        const __nv_bfloat16* wd = reinterpret_cast<const __nv_bfloat16*>(p.src_down) + (size_t)state * p.ss_d;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int idx = tid + j * NPROD;  // 0..2047: 128 rows x 16 chunks of 8 columns
          const int hh = idx >> 4, c8 = (idx & 15) * 8;
          const bool ok = h0 + hh < p.h;
          const size_t off = (size_t)(ok ? h0 + hh : h0) * p.d + (mt0 + mt) * 128 + c8;
          cp_async_16(base + (c8 >> 6) * 16384 + sw128_offset(hh, (c8 & 63) * 2), wd + off, ok);
        }
      }
    };
    if constexpr (kAsync) {
      for (int i = 0; i < kAhead; ++i) {
        if (i < n_items) issue(i);
        cp_async_commit();
      }
      for (int kb = 0; kb < nkb; ++kb) {
        if (kb + kAhead < n_items) issue(kb + kAhead);
        cp_async_commit();
        cp_async_wait<kAhead>();                        // this thread's copies of k-block kb have landed
        fence_proxy_async_smem();
        mbar_arrive(&full[kb % NSLOT]);
      }
      it = nkb;
    } else {
    const WT* wu = reinterpret_cast<const WT*>(p.src_up) + (size_t)state * p.ss_ug;
    const WT* wg = reinterpret_cast<const WT*>(p.src_gate) + (size_t)state * p.ss_ug;
    for (int kb = 0; kb < nkb; ++kb, ++it) {
      const int s = it % NSLOT;
      mbar_wait(&empty[s], ((it / NSLOT) & 1) ^ 1, p.status);
      uint8_t* sUp = slots + s * SLOT_BYTES;
      uint8_t* sGa = sUp + 16384;
      // 64 rows (k) x 128 cols (hidden) per matrix; thread -> 8 quads per matrix
      typename Q::V fu[8], fg[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int idx = tid + j * NPROD;  // 0..2047
        const int kr = idx >> 5, c4 = (idx & 31) * 4;
        const int col = h0 + c4;
        const size_t off = (size_t)((kb0 + kb) * 64 + kr) * p.ld_ug + col;
        if (col < p.h) {
          fu[j] = Q::load(wu + off);
          fg[j] = Q::load(wg + off);
        } else {
          fu[j] = Q::zero();
          fg[j] = fu[j];
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int idx = tid + j * NPROD;
        const int kr = idx >> 5, c4 = (idx & 31) * 4;
        const uint32_t o = (c4 >> 6) * 8192 + sw128_offset(kr, (c4 & 63) * 2);
        *reinterpret_cast<uint2*>(sUp + o) = Q::pack(fu[j]);
        *reinterpret_cast<uint2*>(sGa + o) = Q::pack(fg[j]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&full[s]);
    }

    }
    // ------------------------------------------------------------ epilogue 1: H
    mbar_wait(&ug_done, 0, p.status);
    tc_fence_after();
    {
      const int q = warp & 3, half = warp >> 2;
      const int row = q * 32 + lane;           // hidden row within tile
      const int c0 = half * 32;                // token columns
      float u[32], g[32];
      tmem_ld16(tmem_addr(tU, q * 32, c0), *reinterpret_cast<float(*)[16]>(&u[0]));
      tmem_ld16(tmem_addr(tU, q * 32, c0 + 16), *reinterpret_cast<float(*)[16]>(&u[16]));
      tmem_ld16(tmem_addr(tG, q * 32, c0), *reinterpret_cast<float(*)[16]>(&g[0]));
      tmem_ld16(tmem_addr(tG, q * 32, c0 + 16), *reinterpret_cast<float(*)[16]>(&g[16]));
      tmem_wait_ld();
      if constexpr (kSplit) {   // U, G over all of d (exchange counter 0, zeroed before the launch)
        float ug[2][32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          ug[0][i] = u[i];
          ug[1][i] = g[i];
        }
        const int ntile = p.tiles ? (int)gridDim.y : (int)gridDim.x / KS;
        dsplit_exchange(ug, p, (size_t)b * ntile + t, KS, ksr, 1, 0, row, c0);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          u[i] = ug[0][i];
          g[i] = ug[1][i];
        }
      }
      if (p.u_save && ksr == 0) {
        float* us = p.u_save + (size_t)b * CT * p.hp + h0 + row;
        float* gs = p.g_save + (size_t)b * CT * p.hp + h0 + row;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          us[(size_t)(c0 + i) * p.hp] = u[i];
          gs[(size_t)(c0 + i) * p.hp] = g[i];
        }
      }
      // H tile, MN-major: row = hidden, 64 token values per 128 B row
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 pk;
        float hv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float gg = g[i + e];
          hv[e] = (c0 + i + e < Cc) ? gg * sigmoidf_(gg) * u[i + e] : 0.f;
        }
        pk.x = pack_bf16x2(hv[0], hv[1]);
        pk.y = pack_bf16x2(hv[2], hv[3]);
        pk.z = pack_bf16x2(hv[4], hv[5]);
        pk.w = pack_bf16x2(hv[6], hv[7]);
        *reinterpret_cast<uint4*>(sH + sw128_offset(row, (c0 + i) * 2)) = pk;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&h_ready);
    }

    // ------------------------------------------------------------ W_down tiles + Z drain
    // drains Z tile pm (TMEM rows = d, columns = tokens) into zacc; `release`: give the TMEM
    // buffer back to the MMA warp (every tile but the last)
    auto drain = [&](int pm, bool release) {
      const int zb = pm & 1;
      mbar_wait(&zfull[zb], (pm >> 1) & 1, p.status);
      tc_fence_after();
      const int q = warp & 3, half = warp >> 2;
      const int row = q * 32 + lane, c0 = half * 32;
      float z[32];
      tmem_ld16(tmem_addr(tZ + zb * 64, q * 32, c0), *reinterpret_cast<float(*)[16]>(&z[0]));
      tmem_ld16(tmem_addr(tZ + zb * 64, q * 32, c0 + 16), *reinterpret_cast<float(*)[16]>(&z[16]));
      tmem_wait_ld();
      if (release) {
        tc_fence_before();
        mbar_arrive(&zfree[zb]);
      }
      float* za = p.zacc + zrow0 * p.d + (mt0 + pm) * 128 + row;
      for (int i = 0; i < 32; ++i)
        if (c0 + i < Cc) red_add_f32(za + (size_t)(c0 + i) * p.d, z[i]);
    };
    if constexpr (kAsync) {
      for (int mt = 0; mt < nmt; ++mt) {
        const int i = nkb + mt;
        if (i + kAhead < n_items) issue(i + kAhead);
        cp_async_commit();
        cp_async_wait<kAhead>();                        // this thread's copies of item i have landed
        fence_proxy_async_smem();
        mbar_arrive(&full[i % NSLOT]);
        if (mt > 0) drain(mt - 1, true);                // while the tensor cores work on tile mt
      }
    } else {
      const WT* wd = reinterpret_cast<const WT*>(p.src_down) + (size_t)state * p.ss_d;
      for (int mt = 0; mt < nmt; ++mt, ++it) {
        const int s = it % NSLOT;
        mbar_wait(&empty[s], ((it / NSLOT) & 1) ^ 1, p.status);
        uint8_t* sA = slots + s * SLOT_BYTES;
        // A (M = d slice of 128, K = 128 hidden rows), MN-major: [dblk 2][hh 128][64 d]
#pragma unroll 4
        for (int j = 0; j < 16; ++j) {
          const int idx = tid + j * NPROD;  // 0..4095
          const int hh = idx >> 5, c4 = (idx & 31) * 4;
          typename Q::V f = Q::zero();
          if (h0 + hh < p.h) f = Q::load(wd + (size_t)(h0 + hh) * p.d + (mt0 + mt) * 128 + c4);
          *reinterpret_cast<uint2*>(sA + (c4 >> 6) * 16384 + sw128_offset(hh, (c4 & 63) * 2)) = Q::pack(f);
        }
        fence_proxy_async_smem();
        mbar_arrive(&full[s]);
        if (mt > 0) drain(mt - 1, true);                // drain the previous Z tile meanwhile
      }
    }
    drain(nmt - 1, false);
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      int it = 0;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % NSLOT;
        mbar_wait(&empty[s], ((it / NSLOT) & 1) ^ 1, p.status);
        mbar_arrive_expect_tx(&full[s], 8192);
        tma_load_3d(slots + s * SLOT_BYTES + 32768, &tmK, &full[s], (kb0 + kb) * 64, tok0, b);
      }
      for (int mt = 0; mt < nmt; ++mt, ++it) {
        const int s = it % NSLOT;
        mbar_wait(&empty[s], ((it / NSLOT) & 1) ^ 1, p.status);
        mbar_arrive(&full[s]);
      }
    }
  } else {  // MMA warp
    if (lane == 0) {
      const uint32_t id_ug = idesc_bf16(128, 64, true, false);
      int it = 0;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % NSLOT;
        mbar_wait(&full[s], (it / NSLOT) & 1, p.status);
        tc_fence_after();
        const uint32_t a_up = smem_u32(slots + s * SLOT_BYTES);
        const uint32_t a_ga = a_up + 16384, bk = a_up + 32768;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t bd = sdesc_sw128(bk + ks * 32, 16, 1024);
          const uint32_t acc = (kb > 0 || ks > 0) ? 1u : 0u;
          mma_bf16(tU, sdesc_sw128(a_up + ks * 2048, 8192, 1024), bd, id_ug, acc);
          mma_bf16(tG, sdesc_sw128(a_ga + ks * 2048, 8192, 1024), bd, id_ug, acc);
        }
        mma_commit(&empty[s]);
      }
      mma_commit(&ug_done);
      mbar_wait(&h_ready, 0, p.status);
      tc_fence_after();
      const uint32_t id_z = idesc_bf16(128, 64, true, true);
      const uint32_t hb = smem_u32(sH);
      for (int mt = 0; mt < nmt; ++mt, ++it) {
        const int s = it % NSLOT, zb = mt & 1;
        mbar_wait(&full[s], (it / NSLOT) & 1, p.status);
        mbar_wait(&zfree[zb], ((mt >> 1) & 1) ^ 1, p.status);
        tc_fence_after();
        const uint32_t a = smem_u32(slots + s * SLOT_BYTES);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_bf16(tZ + zb * 64, sdesc_sw128(a + ks * 2048, 16384, 1024), sdesc_sw128(hb + ks * 2048, 8192, 1024),
                   id_z, ks > 0 ? 1u : 0u);
        mma_commit(&empty[s]);
        mma_commit(&zfull[zb]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ============================================================================
// ln: LayerNorm statistics, v_hat, token loss, analytical LayerNorm backward
// ============================================================================
constexpr int LN_THREADS = 256;
constexpr int LN_MAXV = 16;  // d <= 4096

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < LN_THREADS / 32; ++i) s += red[i];
  return s;
}

// One warp per token row (d = 128 * NV, NV float4 per lane), shuffle-only
// reductions: the chunk's 64 rows of a state are 8 blocks of 8 warps.
constexpr int LN_ROWS = 8;

template <int NV>
__global__ void __launch_bounds__(LN_ROWS * 32) chunk_ln_kernel(const ChunkParams p) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * LN_ROWS + (threadIdx.x >> 5), b = blockIdx.y;
  constexpr int d = NV * 128;
  uint2* dzrow = reinterpret_cast<uint2*>(p.dz + ((size_t)b * CT + c) * d);
  if (c >= p.Cc) {  // padded token row: zero gradient
#pragma unroll
    for (int i = 0; i < NV; ++i) dzrow[i * 32 + lane] = make_uint2(0u, 0u);
    return;
  }
  if (c == 0 && lane == 0) p.norm2[b] = 0.f;
  const size_t tok = (size_t)b * p.T + p.tok0 + c;
  float cnt = (float)p.Cc;  // valid tokens of this chunk (model/uttt_layer.py:371-378)
  if (p.mask) {
    float s = 0.f;
    for (int i = lane; i < p.Cc; i += 32) s += p.mask[(size_t)b * p.T + p.tok0 + i];
    cnt = warp_sum(s);
  }
  float4* zrow = reinterpret_cast<float4*>(p.zacc + ((size_t)b * CT + c) * d);
  const uint2* krow = reinterpret_cast<const uint2*>(p.k + tok * d);
  const uint2* vrow = reinterpret_cast<const uint2*>(p.v + tok * d);
  const float4* lw4 = reinterpret_cast<const float4*>(p.ln_w);
  const float4* lb4 = reinterpret_cast<const float4*>(p.ln_b);
  float z[4 * NV];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4 v = zrow[i * 32 + lane];
    zrow[i * 32 + lane] = make_float4(0.f, 0.f, 0.f, 0.f);   // ready for the next chunk's partial sums
    z[4 * i] = v.x; z[4 * i + 1] = v.y; z[4 * i + 2] = v.z; z[4 * i + 3] = v.w;
    sum += (v.x + v.y) + (v.z + v.w);
  }
  const float dinv = 1.f / (float)d;
  const float mean = warp_sum(sum) * dinv;
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < 4 * NV; ++j) {
    z[j] -= mean;
    sq += z[j] * z[j];
  }
  const float rstd = rsqrtf(warp_sum(sq) * dinv + p.eps);
  // above d = 2560 the residual is recomputed in the second pass instead of
  // being kept in registers
  constexpr bool kKeepE = NV <= 20;
  float e[kKeepE ? 4 * NV : 1];
  float err2 = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint2 kk = krow[i * 32 + lane], vv = vrow[i * 32 + lane];
    const float4 w = lw4[i * 32 + lane], bb = lb4[i * 32 + lane];
    const float kf[4] = {bf16_lo(kk.x), bf16_hi(kk.x), bf16_lo(kk.y), bf16_hi(kk.y)};
    const float vf[4] = {bf16_lo(vv.x), bf16_hi(vv.x), bf16_lo(vv.y), bf16_hi(vv.y)};
    const float wf4[4] = {w.x, w.y, w.z, w.w}, bf4[4] = {bb.x, bb.y, bb.z, bb.w};
    float vh[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = 4 * i + u;
      z[j] *= rstd;                                   // z now holds the normalised zh
      vh[u] = kf[u] + (z[j] * wf4[u] + bf4[u]);
      const float ej = vh[u] - vf[u];
      if constexpr (kKeepE) e[j] = ej;
      err2 += ej * ej;
    }
    if (p.out) {
      const size_t o = tok * d + (size_t)(i * 32 + lane) * 4;
      if (p.out_bf16) {
        uint2 pk;
        pk.x = pack_bf16x2(vh[0], vh[1]);
        pk.y = pack_bf16x2(vh[2], vh[3]);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + o) = pk;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + o) = make_float4(vh[0], vh[1], vh[2], vh[3]);
      }
    }
  }
  const float loss = 0.5f * warp_sum(err2) * p.inv_scale;
  if (lane == 0 && p.token_loss) p.token_loss[tok] = loss;
  const float m = p.mask ? p.mask[tok] : 1.f;
  const float wf = p.mask ? p.eta[tok] * m / fmaxf(cnt, 1.f) : p.eta[tok] / (float)p.Cc;
  const float coef = wf * p.inv_scale;
  // d(zh) = coef * e * gamma
  auto dzh = [&](int i, float (&out)[4]) {
    const float4 w = lw4[i * 32 + lane];
    const float wf4[4] = {w.x, w.y, w.z, w.w};
    if constexpr (kKeepE) {
#pragma unroll
      for (int u = 0; u < 4; ++u) out[u] = coef * e[4 * i + u] * wf4[u];
    } else {
      const uint2 kk = krow[i * 32 + lane], vv = vrow[i * 32 + lane];
      const float4 bb = lb4[i * 32 + lane];
      const float kf[4] = {bf16_lo(kk.x), bf16_hi(kk.x), bf16_lo(kk.y), bf16_hi(kk.y)};
      const float vf[4] = {bf16_lo(vv.x), bf16_hi(vv.x), bf16_lo(vv.y), bf16_hi(vv.y)};
      const float bf4[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float ej = (kf[u] + (z[4 * i + u] * wf4[u] + bf4[u])) - vf[u];
        out[u] = coef * ej * wf4[u];
      }
    }
  };
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float g[4];
    dzh(i, g);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if constexpr (kKeepE) e[4 * i + u] = g[u];
      s1 += g[u];
      s2 += g[u] * z[4 * i + u];
    }
  }
  const float mdz = warp_sum(s1) * dinv;
  const float mdzz = warp_sum(s2) * dinv;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float g[4];
    if constexpr (kKeepE) {
#pragma unroll
      for (int u = 0; u < 4; ++u) g[u] = e[4 * i + u];
    } else {
      dzh(i, g);
    }
    uint2 pk;
    pk.x = pack_bf16x2(rstd * (g[0] - mdz - z[4 * i] * mdzz), rstd * (g[1] - mdz - z[4 * i + 1] * mdzz));
    pk.y = pack_bf16x2(rstd * (g[2] - mdz - z[4 * i + 2] * mdzz), rstd * (g[3] - mdz - z[4 * i + 3] * mdzz));
    dzrow[i * 32 + lane] = pk;
  }
}

using LnKernel = void (*)(const ChunkParams);

LnKernel chunk_ln_for(int d) {
  switch (d / 128) {
#define UTTT_LN_CASE(n) case n: return chunk_ln_kernel<n>;
    UTTT_LN_CASE(1) UTTT_LN_CASE(2) UTTT_LN_CASE(3) UTTT_LN_CASE(4) UTTT_LN_CASE(5) UTTT_LN_CASE(6)
    UTTT_LN_CASE(7) UTTT_LN_CASE(8) UTTT_LN_CASE(9) UTTT_LN_CASE(10) UTTT_LN_CASE(11) UTTT_LN_CASE(12)
    UTTT_LN_CASE(13) UTTT_LN_CASE(14) UTTT_LN_CASE(15) UTTT_LN_CASE(16) UTTT_LN_CASE(17) UTTT_LN_CASE(18)
    UTTT_LN_CASE(19) UTTT_LN_CASE(20) UTTT_LN_CASE(21) UTTT_LN_CASE(22) UTTT_LN_CASE(23) UTTT_LN_CASE(24)
    UTTT_LN_CASE(25) UTTT_LN_CASE(26) UTTT_LN_CASE(27) UTTT_LN_CASE(28) UTTT_LN_CASE(29) UTTT_LN_CASE(30)
    UTTT_LN_CASE(31) UTTT_LN_CASE(32)
#undef UTTT_LN_CASE
    default: return nullptr;
  }
}

// ============================================================================
// readout epilogue: out = x + LN(z) * gamma + beta  (swiglu_fast_forward's
// last line, model/uttt_layer.py:243-247).  Consumes and re-zeroes z.
// ============================================================================
__global__ void __launch_bounds__(LN_THREADS) readout_ln_kernel(const float* __restrict__ zbase, int zrows,
                                                                const __nv_bfloat16* __restrict__ x, int T,
                                                                int tok0, int Cc, int d, const float* ln_w,
                                                                const float* ln_b, float eps, void* out,
                                                                int out_bf16) {
  __shared__ float red[LN_THREADS / 32];
  const int c = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  if (c >= Cc) return;
  float* zrow = const_cast<float*>(zbase) + ((size_t)b * zrows + c) * d;
  const size_t tok = (size_t)b * T + tok0 + c;
  float z[LN_MAXV];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < LN_MAXV; ++j) {
    const int i = tid + j * LN_THREADS;
    z[j] = 0.f;
    if (i < d) {
      z[j] = zrow[i];
      zrow[i] = 0.f;
      sum += z[j];
    }
  }
  const float dinv = 1.f / (float)d;
  const float mean = block_sum(sum, red) * dinv;
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < LN_MAXV; ++j) {
    const int i = tid + j * LN_THREADS;
    if (i < d) sq += (z[j] - mean) * (z[j] - mean);
  }
  const float rstd = rsqrtf(block_sum(sq, red) * dinv + eps);
#pragma unroll
  for (int j = 0; j < LN_MAXV; ++j) {
    const int i = tid + j * LN_THREADS;
    if (i < d) {
      const float y = __bfloat162float(x[tok * d + i]) + ((z[j] - mean) * rstd * ln_w[i] + ln_b[i]);
      if (out_bf16)
        reinterpret_cast<__nv_bfloat16*>(out)[tok * d + i] = __float2bfloat16(y);
      else
        reinterpret_cast<float*>(out)[tok * d + i] = y;
    }
  }
}

// ============================================================================
// bwd: dH, dU, dG and the three weight gradients; NORM pass accumulates
// ||grad||^2, UPDATE pass applies momentum / decay / clip in place.
// ============================================================================
// K K^T and dZ dZ^T of each row's chunk, summed over 128-wide slabs of d (grid (d / 128, B)).
// Token rows past the chunk are zero.  Thread (ti, tj) owns the entries (ti + 16 a, tj + 16 c),
// so a warp's 16-byte reads of the j rows fall in distinct banks of the padded rows.
constexpr int GRAM_D = 128;
__global__ void __launch_bounds__(256) chunk_gram_kernel(const ChunkParams p) {
  __shared__ __align__(16) __nv_bfloat16 sm[2][CT][GRAM_D + 8];
  const int tid = threadIdx.x, b = blockIdx.y, dd0 = blockIdx.x * GRAM_D;
  for (int i = tid; i < CT * (GRAM_D / 8); i += 256) {
    const int r = i / (GRAM_D / 8), c8 = (i % (GRAM_D / 8)) * 8;
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), zv = kv;
    if (r < p.Cc) {
      kv = __ldg(reinterpret_cast<const uint4*>(p.k + ((size_t)b * p.T + p.tok0 + r) * p.d + dd0 + c8));
      zv = __ldcg(reinterpret_cast<const uint4*>(p.dz + ((size_t)b * CT + r) * p.d + dd0 + c8));
    }
    *reinterpret_cast<uint4*>(&sm[0][r][c8]) = kv;
    *reinterpret_cast<uint4*>(&sm[1][r][c8]) = zv;
  }
  __syncthreads();
  const int ti = tid >> 4, tj = tid & 15;
#pragma unroll 1
  for (int m = 0; m < 2; ++m) {
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;
#pragma unroll 1
    for (int k8 = 0; k8 < GRAM_D; k8 += 8) {
      uint4 xi[4], xj[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        xi[a] = *reinterpret_cast<const uint4*>(&sm[m][ti + 16 * a][k8]);
        xj[a] = *reinterpret_cast<const uint4*>(&sm[m][tj + 16 * a][k8]);
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        float fi[4][2], fj[4][2];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const uint32_t vi = (&xi[a].x)[w], vj = (&xj[a].x)[w];
          fi[a][0] = bf16_lo(vi); fi[a][1] = bf16_hi(vi);
          fj[a][0] = bf16_lo(vj); fj[a][1] = bf16_hi(vj);
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[a][c] += fi[a][0] * fj[c][0] + fi[a][1] * fj[c][1];
      }
    }
    float* g = p.gram + ((size_t)b * 2 + m) * CT * CT;
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) red_add_f32(g + (ti + 16 * a) * CT + tj + 16 * c, acc[a][c]);
  }
}

// FP32 tensor maps of the W masters for the TMA-staged update epilogue:
// up/gate over (h, d, states) with 128 x 32 boxes, down over (d, h, states)
// with 32 x 128 boxes (128-byte swizzle).
struct WMaps {
  CUtensorMap up, gate, down;
  CUtensorMap zacc;   // FP32 (d, B * 64) partial-Z accumulator, 128 x 32 boxes
};
constexpr int QW = 32;                    // d columns per staged quarter chunk
constexpr int WTILE = HT * QW * 4;        // 16 KB: one staged FP32 tile
constexpr int NF = 5;                     // FP32 W_down quarter tiles in flight (phase-1 ring)
constexpr int ZSLOT = 32 * 1024;          // one BF16 [128 d][128 hidden] A tile of the next chunk's Z'

// kFuse: also run the NEXT chunk's forward (U', G', H', partial Z') from the
// weight tiles this kernel just updated, so the separate forward pass over
// the FP32 masters disappears for every chunk but the first of a call.
// kClip: a clip run (ChunkParams::ops and ::gram set): the norm pass (update = 0) takes the Gram
// route and keeps its epilogue-1 operands, the update pass (update = 1) starts from them.  A
// compile-time choice, so the unclipped kernels carry none of that code.
template <bool kMomentum, bool kFuse, bool kSplit, bool kClip>
__global__ void __launch_bounds__(BWD_THREADS, 1) chunk_bwd_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                const __grid_constant__ CUtensorMap tmDZ,
                                                                const __grid_constant__ WMaps wm,
                                                                const ChunkParams p, int update) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[NSLOT], empty[NSLOT], full3, empty3, dh_done, ops_ready, gfull, gfree, wfullA[3], wfullB[6];
  __shared__ uint64_t a_ready, kfull, ug_free, h_ready, fullz[2], emptyz[2], zfull[2], zfree[2];
  __shared__ uint64_t ffull[NF], fempty[NF], qdoneA[3], qdoneB[6];
  __shared__ uint32_t tmem_slot;
  __shared__ ChunkStats st_sh;
  uint8_t* slots = align1024(smem_raw);             // 96 KB: phase-1 ring | W staging | Z' ring
  uint8_t* slots3 = slots + NSLOT * BWD_SLOT;       // 32 KB: K slice + dZ slice of one 128-wide d chunk
  uint8_t* sDU = slots3 + 32768;                    // K-major [hh 128][64 tokens]
  uint8_t* sDG = sDU + 16384;
  uint8_t* sHt = sDG + 16384;
  uint8_t* sAU = sHt + 16384;                       // next chunk: bf16 W'_up^T  K-major [hh 128][64 d]
  uint8_t* sAG = sAU + 16384;                       //             bf16 W'_gate^T
  uint8_t* sKN = sAG + 16384;                       //             K' tile [64 tokens][64 d]
  uint8_t* sH = sDU;                                // next chunk H' (MN-major [hh][64 tokens]) after the loop
  // FP32 W_down quarter tiles [128 hidden][32 d] (TMA, 128B swizzle) of
  // phase 1, NF deep, in sDU..sAG (free until dH is done)
  uint8_t* fring1 = sDU;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x, b = blockIdx.y;
  // row b's activations and workspace rows are compact; its fast-weight state is sb
  const int sb = p.state_index ? p.state_index[b] : b;
  if (p.state_index && (unsigned)sb >= (unsigned)p.n_states) {
    if (tid == 0) set_status(p.status, UTTT_ERR_INVALID);
    return;
  }
  const int h0 = t * HT;
  const int nch_all = p.d / 128;
  // d-split: the gridDim.z CTAs of a cluster share this (tile, state); rank ksr owns the 128-wide
  // d chunks [j0, j0 + nch).  Loop counters below are local to that range (barrier phases);
  // global d coordinates add j0 (chunks), kb0 (64-wide k-blocks) or q0 (32-wide quarters).
  const int KS = kSplit ? (int)gridDim.z : 1, ksr = kSplit ? (int)blockIdx.z : 0;   // kSplit: a compile-time choice
  const int nch = kSplit ? nch_all / KS : nch_all, j0 = kSplit ? ksr * nch : 0;
  const int nkb = kSplit ? 2 * nch : p.d / 64, kb0 = 2 * j0;
  const int q0 = 4 * j0;

  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&full[i], NPROD + 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&full3, 1);
    mbar_init(&empty3, 1);
    mbar_init(&a_ready, NPROD);
    mbar_init(&kfull, 1);
    mbar_init(&ug_free, 1);
    mbar_init(&h_ready, NPROD);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&fullz[i], NPROD);
      mbar_init(&emptyz[i], 1);
      mbar_init(&zfull[i], 1);
      mbar_init(&zfree[i], NPROD);
    }
    mbar_init(&dh_done, 1);
    mbar_init(&ops_ready, NPROD);
    mbar_init(&gfull, 1);
    mbar_init(&gfree, NPROD);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&wfullA[i], 1);
      mbar_init(&qdoneA[i], NPROD);
    }
    for (int i = 0; i < 6; ++i) {
      mbar_init(&wfullB[i], 1);
      mbar_init(&qdoneB[i], NPROD);
    }
    for (int i = 0; i < NF; ++i) {
      mbar_init(&ffull[i], 1);
      mbar_init(&fempty[i], NPROD);
    }
    fence_mbarrier_init();
  }
  if (warp == 0) {
    ChunkStats s = chunk_stats(p, b);
    if (lane == 0) st_sh = s;
  }
  if (warp == 1) tmem_alloc(&tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tDH = tmem, tGU = tmem + 128, tGG = tmem + 256, tGD = tmem + 384;
  const uint32_t tUN = tmem, tGN = tmem + 64;       // next chunk U', G' (after dH is drained)
  const uint32_t tZN = tmem + 128;                   // next chunk Z' tiles (after the gradients)
  const ChunkStats st = st_sh;
  // A state with no valid token keeps W and S exactly (model/uttt_layer.py:513-520).
  const bool skip = !st.active;

  // ------------------------------------------------------------ update set-up
  // The FP32 masters move through shared memory by TMA in quarter chunks of
  // 32 d columns: W_up / W_gate tiles [32 d][128 hidden], W_down tiles
  // [128 hidden][32 d] 128B-swizzled.  Loop A updates W_up / W_gate (and
  // feeds the next chunk's U', G'), loop B updates W_down and turns each
  // updated quarter straight into the next chunk's Z' operand, so W'_down is
  // never read back.  The threads only touch TMEM and shared memory; the copy
  // engine keeps HBM busy with up to 3 (A) / 6 (B) quarters in flight.
  float scale = 1.f;
  if (update && p.clip > 0.f) scale = fminf(1.f, p.clip * rsqrtf(p.norm2[b] + 1e-8f));
  if (update && p.clip_out && t == 0 && tid == 0) p.clip_out[(size_t)b * p.n_chunks + p.chunk_index] = scale;
  const float decay = 1.f - st.alpha_bar;
  const float beta = p.beta;
  // With beta == 0 the momentum of this chunk is never read again unless this
  // is the last chunk of the call that changes this state.
  const bool write_s = kMomentum || !st.later_active;
  // Staging holds W only (3 quarters of W_up + W_gate, 6 of W_down in flight: loop B's stream is
  // bounded by its depth, so the next chunk's Z' operand has one A tile, not two);
  // each producer moves its own momentum values between registers and HBM
  // (lanes are consecutive hidden rows, so S_up / S_gate accesses coalesce).
  constexpr int bytesA = 2 * WTILE, nbufA = 3;
  constexpr int bytesB = WTILE, nbufB = 6;
  const int nq = kSplit ? 4 * nch : p.d / QW;   // this rank's 32-wide quarters (local counter)
  const bool fuse = kFuse && update;
  // the next chunk's forward reads the (possibly unchanged) tiles as well
  const bool stage = (update && !skip) || fuse;
  auto load_a = [&](int qi) {            // qi: local quarter
    const int buf = qi % nbufA;
    uint8_t* B0 = slots + buf * bytesA;
    mbar_arrive_expect_tx(&wfullA[buf], 2 * WTILE);
    tma_load_3d(B0, &wm.up, &wfullA[buf], h0, (q0 + qi) * QW, sb);
    tma_load_3d(B0 + WTILE, &wm.gate, &wfullA[buf], h0, (q0 + qi) * QW, sb);
  };
  auto load_b = [&](int qi) {
    const int buf = qi % nbufB;
    uint8_t* B0 = slots + buf * bytesB;
    mbar_arrive_expect_tx(&wfullB[buf], WTILE);
    tma_load_3d(B0, &wm.down, &wfullB[buf], (q0 + qi) * QW, h0, sb);
  };
  // momentum of this state: s_* (d, h) for up / gate, (h, d) for down
  const size_t s_off = (size_t)sb * p.d * p.h;

  // an update after a norm pass takes dU, dG, H from the norm pass: no phase 1, no W_down read for dH
  const bool ops_in = kClip && update;
  // a norm pass with the chunk's Gram matrices: no gradient tiles, the d-split's rank 0 sums for the pair
  const bool gram = kClip && !update;
  uint8_t* ops_at = kClip ? p.ops + ((size_t)b * gridDim.x + t) * OPS_BYTES : nullptr;

  if (warp < 8) {
    // ------------------------------------------------------------ W_down rows -> A (K-major)
    // Two FP32 quarter tiles (TMA; rows past h arrive as zeros) make one BF16
    // k-block of 64 d columns.
    int it = 0;
    for (int kb = 0; kb < (ops_in ? 0 : nkb); ++kb, ++it) {
      const int s = it % NSLOT;
      mbar_wait(&empty[s], ((it / NSLOT) & 1) ^ 1, p.status);
      uint8_t* sA = slots + s * BWD_SLOT;
#pragma unroll 1
      for (int hq = 0; hq < 2; ++hq) {
        const int qi = 2 * kb + hq, fs = qi % NF;
        float4 f[4];
        if (!skip) {
          mbar_wait(&ffull[fs], (qi / NF) & 1, p.status);
          const uint8_t* src = fring1 + fs * WTILE;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int idx = tid + j * NPROD;  // 0..1023 : 128 rows x 8 float4
            f[j] = *reinterpret_cast<const float4*>(src + sw128_offset(idx >> 3, (idx & 7) * 16));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) f[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int idx = tid + j * NPROD;
          const int hh = idx >> 3, c4 = (idx & 7) * 4;
          uint2 pk;
          pk.x = pack_bf16x2(f[j].x, f[j].y);
          pk.y = pack_bf16x2(f[j].z, f[j].w);
          *reinterpret_cast<uint2*>(sA + sw128_offset(hh, (hq * QW + c4) * 2)) = pk;
        }
        // the ring tile is released only once its values are used: an arrive right after the
        // shared loads let the TMA refill overwrite a tile before a delayed load had read it
        if (!skip) mbar_arrive(&fempty[(2 * kb + hq) % NF]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&full[s]);
    }

    // ------------------------------------------------------------ epilogue 1: dU, dG, H
    const int q = warp & 3, half = warp >> 2;
    const int row = q * 32 + lane;                   // hidden row within the tile
    if (ops_in) {
      // the norm pass's dU, dG, H tiles: 3072 16-byte pieces, 12 per thread, coalesced
      const uint4* src = reinterpret_cast<const uint4*>(ops_at);
      uint4* dst = reinterpret_cast<uint4*>(sDU);     // sDU, sDG, sHt are consecutive 16 KB tiles
      uint4 v[12];
#pragma unroll
      for (int i = 0; i < 12; ++i) v[i] = __ldcg(src + tid + i * NPROD);
#pragma unroll
      for (int i = 0; i < 12; ++i) dst[tid + i * NPROD] = v[i];
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&ops_ready);
    } else {
      const int c0 = half * 32;
      // the saved U / G of this thread's row are loaded while the dH MMAs finish
      const float* us = p.u_save + (size_t)b * CT * p.hp + h0 + row;
      const float* gs = p.g_save + (size_t)b * CT * p.hp + h0 + row;
      float uv[32], gv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        uv[i] = us[(size_t)(c0 + i) * p.hp];
        gv[i] = gs[(size_t)(c0 + i) * p.hp];
      }
      mbar_wait(&dh_done, 0, p.status);
      tc_fence_after();
      float dh[32];
      tmem_ld16(tmem_addr(tDH, q * 32, c0), *reinterpret_cast<float(*)[16]>(&dh[0]));
      tmem_ld16(tmem_addr(tDH, q * 32, c0 + 16), *reinterpret_cast<float(*)[16]>(&dh[16]));
      tmem_wait_ld();
      if constexpr (kSplit)   // dH over all of d
        dsplit_exchange(*reinterpret_cast<float(*)[1][32]>(&dh), p, (size_t)b * gridDim.x + t, KS, ksr, 0, 0, row, c0);
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        float du[8], dg[8], hv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = c0 + i + e;
          const float u = uv[i + e];
          const float g = gv[i + e];
          const float sg = sigmoidf_(g);
          const float a = g * sg;
          const bool valid = c < p.Cc;
          hv[e] = valid ? a * u : 0.f;
          du[e] = valid ? dh[i + e] * a : 0.f;
          dg[e] = valid ? dh[i + e] * u * (sg * (1.f + g * (1.f - sg))) : 0.f;
        }
        uint4 a4, b4, c4;
        a4.x = pack_bf16x2(du[0], du[1]); a4.y = pack_bf16x2(du[2], du[3]);
        a4.z = pack_bf16x2(du[4], du[5]); a4.w = pack_bf16x2(du[6], du[7]);
        b4.x = pack_bf16x2(dg[0], dg[1]); b4.y = pack_bf16x2(dg[2], dg[3]);
        b4.z = pack_bf16x2(dg[4], dg[5]); b4.w = pack_bf16x2(dg[6], dg[7]);
        c4.x = pack_bf16x2(hv[0], hv[1]); c4.y = pack_bf16x2(hv[2], hv[3]);
        c4.z = pack_bf16x2(hv[4], hv[5]); c4.w = pack_bf16x2(hv[6], hv[7]);
        const uint32_t o = sw128_offset(row, (c0 + i) * 2);
        *reinterpret_cast<uint4*>(sDU + o) = a4;
        *reinterpret_cast<uint4*>(sDG + o) = b4;
        *reinterpret_cast<uint4*>(sHt + o) = c4;
        if (kClip && !update && ksr == 0) {           // the norm pass keeps them for the update
          *reinterpret_cast<uint4*>(ops_at + o) = a4;
          *reinterpret_cast<uint4*>(ops_at + 16384 + o) = b4;
          *reinterpret_cast<uint4*>(ops_at + 32768 + o) = c4;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&ops_ready);
    }

    // ------------------------------------------------------------ loop A: W_up, W_gate
    const int cq = half * 16;                        // this thread's 16 of the quarter's 32 columns
    const bool row_ok = h0 + row < p.h;
    float acc = 0.f;
    if (gram && ksr == 0 && !skip) {
      // TMEM lanes 0-63 of D1 hold dU^T dU, lanes 64-127 of D1 dG^T dG (columns 64-127) and of D2
      // H^T H; each thread dots its 32 columns of its token row with the matching Gram row
      mbar_wait(&gfull, 0, p.status);
      tc_fence_after();
      const int i = row & 63, cb = (row < 64 ? 0 : 64) + half * 32;
      const float* gk = p.gram + (size_t)b * 2 * CT * CT + i * CT + half * 32;
      const float* gz = gk + CT * CT;
      float m1[32];
      tmem_ld16(tmem_addr(tGU, q * 32, cb), *reinterpret_cast<float(*)[16]>(&m1[0]));
      tmem_ld16(tmem_addr(tGU, q * 32, cb + 16), *reinterpret_cast<float(*)[16]>(&m1[16]));
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) acc += __ldcg(gk + e) * m1[e];
      if (row >= 64) {
        tmem_ld16(tmem_addr(tGG, q * 32, cb), *reinterpret_cast<float(*)[16]>(&m1[0]));
        tmem_ld16(tmem_addr(tGG, q * 32, cb + 16), *reinterpret_cast<float(*)[16]>(&m1[16]));
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) acc += __ldcg(gz + e) * m1[e];
      }
    }
    // stability guard: this row's last update of the call (never a fused chunk: the call's last)
    const bool guard = update && !skip && p.g_final != nullptr && p.g_final[b] != 0 &&
                       p.chunk_index == p.n_chunks - 1 && !fuse;
    float g_up = 0.f, g_gate = 0.f, g_down = 0.f;
    for (int qi = 0; qi < (gram ? 0 : nq); ++qi) {
      const int j = qi >> 2, qq = qi & 3;
      // this quarter's momentum (issued before the waits so its latency overlaps them)
      const bool s_io = update && !skip && row_ok;
      float su[16], sg[16];
      const size_t so = s_off + (size_t)((q0 + qi) * QW + cq) * p.h + h0 + row;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        su[e] = (kMomentum && s_io) ? p.s_up[so + (size_t)e * p.h] : 0.f;
        sg[e] = (kMomentum && s_io) ? p.s_gate[so + (size_t)e * p.h] : 0.f;
      }
      if (qq == 0) {
        mbar_wait(&gfull, j & 1, p.status);
        tc_fence_after();
      }
      float gu[16], gg[16];
      tmem_ld16(tmem_addr(tGU, q * 32, qq * QW + cq), gu);
      tmem_ld16(tmem_addr(tGG, q * 32, qq * QW + cq), gg);
      tmem_wait_ld();
      if (qq == 3) {
        tc_fence_before();
        mbar_arrive(&gfree);
      }
      if (!update) {
        if (row_ok && !skip) {
#pragma unroll
          for (int e = 0; e < 16; ++e) acc += gu[e] * gu[e] + gg[e] * gg[e];
        }
        continue;
      }
      if (!stage) continue;
      const int buf = qi % nbufA;
      mbar_wait(&wfullA[buf], (qi / nbufA) & 1, p.status);
      uint8_t* B0 = slots + buf * bytesA;
      float* wu = reinterpret_cast<float*>(B0);
      float* wg = reinterpret_cast<float*>(B0 + WTILE);
      if (!skip) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int o = (cq + e) * HT + row;            // [32 d][128 hidden]
          const float nsu = (kMomentum ? beta * su[e] : 0.f) - gu[e] * scale;
          const float nsg = (kMomentum ? beta * sg[e] : 0.f) - gg[e] * scale;
          wu[o] = decay * wu[o] + nsu;
          wg[o] = decay * wg[o] + nsg;
          su[e] = nsu;
          sg[e] = nsg;
        }
        if (write_s && row_ok) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            p.s_up_out[so + (size_t)e * p.h] = su[e];
            p.s_gate_out[so + (size_t)e * p.h] = sg[e];
          }
        }
        if (guard && row_ok) {          // elastic pull of the updated quarter (lanes: consecutive hidden rows)
          const size_t go = (size_t)((q0 + qi) * QW + cq) * p.h + h0 + row;
#pragma unroll 4
          for (int e = 0; e < 16; ++e) {
            const int o = (cq + e) * HT + row;
            const float au = __ldg(p.g_w0_up + go + (size_t)e * p.h);
            const float ag = __ldg(p.g_w0_gate + go + (size_t)e * p.h);
            const float du = p.g_keep * (wu[o] - au), dg = p.g_keep * (wg[o] - ag);
            wu[o] = au + du;
            wg[o] = ag + dg;
            g_up += du * du;
            g_gate += dg * dg;
          }
        }
      }
      if (fuse) {
        // bf16 W'_up^T / W'_gate^T columns of this quarter into the next-chunk A tiles
        const int kbi = qi >> 1, half_kb = qi & 1;
        if (half_kb == 0 && kbi > 0) mbar_wait(&ug_free, (kbi - 1) & 1, p.status);
#pragma unroll 1
        for (int i = 0; i < 2; ++i) {
          const float* pu = wu + (cq + 8 * i) * HT + row;
          const float* pg = wg + (cq + 8 * i) * HT + row;
          uint4 a, g;
          a.x = pack_bf16x2(pu[0 * HT], pu[1 * HT]); a.y = pack_bf16x2(pu[2 * HT], pu[3 * HT]);
          a.z = pack_bf16x2(pu[4 * HT], pu[5 * HT]); a.w = pack_bf16x2(pu[6 * HT], pu[7 * HT]);
          g.x = pack_bf16x2(pg[0 * HT], pg[1 * HT]); g.y = pack_bf16x2(pg[2 * HT], pg[3 * HT]);
          g.z = pack_bf16x2(pg[4 * HT], pg[5 * HT]); g.w = pack_bf16x2(pg[6 * HT], pg[7 * HT]);
          const uint32_t o = sw128_offset(row, (half_kb * 32 + cq + 8 * i) * 2);
          *reinterpret_cast<uint4*>(sAU + o) = a;
          *reinterpret_cast<uint4*>(sAG + o) = g;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&qdoneA[buf]);                     // the store warp takes the quarter from here
      if (fuse && (qi & 1)) mbar_arrive(&a_ready);
    }

    // ------------------------------------------------------------ next chunk: H'
    if (fuse) {
      mbar_wait(&ug_free, (nkb - 1) & 1, p.status);          // last U'/G' k-block done
      tc_fence_after();
      const int c0 = half * 32;
      float* us = p.u_save + (size_t)b * CT * p.hp + h0 + row;
      float* gs = p.g_save + (size_t)b * CT * p.hp + h0 + row;
      if constexpr (!kSplit) {
#pragma unroll 1
        for (int c16 = 0; c16 < 32; c16 += 16) {
          float u[16], g[16];
          tmem_ld16(tmem_addr(tUN, q * 32, c0 + c16), u);
          tmem_ld16(tmem_addr(tGN, q * 32, c0 + c16), g);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            us[(size_t)(c0 + c16 + i) * p.hp] = u[i];
            gs[(size_t)(c0 + c16 + i) * p.hp] = g[i];
          }
#pragma unroll
          for (int i = 0; i < 16; i += 8) {
            uint4 pk;
            float hv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float gg2 = g[i + e];
              hv[e] = (c0 + c16 + i + e < p.Cc_next) ? gg2 * sigmoidf_(gg2) * u[i + e] : 0.f;
            }
            pk.x = pack_bf16x2(hv[0], hv[1]);
            pk.y = pack_bf16x2(hv[2], hv[3]);
            pk.z = pack_bf16x2(hv[4], hv[5]);
            pk.w = pack_bf16x2(hv[6], hv[7]);
            *reinterpret_cast<uint4*>(sH + sw128_offset(row, (c0 + c16 + i) * 2)) = pk;
          }
        }
      } else {
        float ug[2][32];                                 // U', G' of this thread's row, 32 token columns
        tmem_ld16(tmem_addr(tUN, q * 32, c0), *reinterpret_cast<float(*)[16]>(&ug[0][0]));
        tmem_ld16(tmem_addr(tUN, q * 32, c0 + 16), *reinterpret_cast<float(*)[16]>(&ug[0][16]));
        tmem_ld16(tmem_addr(tGN, q * 32, c0), *reinterpret_cast<float(*)[16]>(&ug[1][0]));
        tmem_ld16(tmem_addr(tGN, q * 32, c0 + 16), *reinterpret_cast<float(*)[16]>(&ug[1][16]));
        tmem_wait_ld();
        dsplit_exchange(ug, p, (size_t)b * gridDim.x + t, KS, ksr, 1, 1, row, c0);   // U', G' over all of d
        if (ksr == 0) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            us[(size_t)(c0 + i) * p.hp] = ug[0][i];
            gs[(size_t)(c0 + i) * p.hp] = ug[1][i];
          }
        }
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 pk;
          float hv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float gg2 = ug[1][i + e];
            hv[e] = (c0 + i + e < p.Cc_next) ? gg2 * sigmoidf_(gg2) * ug[0][i + e] : 0.f;
          }
          pk.x = pack_bf16x2(hv[0], hv[1]);
          pk.y = pack_bf16x2(hv[2], hv[3]);
          pk.z = pack_bf16x2(hv[4], hv[5]);
          pk.w = pack_bf16x2(hv[6], hv[7]);
          *reinterpret_cast<uint4*>(sH + sw128_offset(row, (c0 + i) * 2)) = pk;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&h_ready);
    }

    // Drains the next chunk's Z' tile mt (TMEM rows = d, columns = tokens)
    // into zacc: each half (warps 0-3: tokens 0-31, warps 4-7: tokens 32-63)
    // stages [32 tokens][128 d] FP32 (slots3's free K-slice half, or sDG, both
    // idle in loop B) and adds it with one bulk tensor reduction.
    uint8_t* zstage = half ? sDG : slots3;
    const bool zissuer = (tid & 127) == 0;
    auto drain_z = [&](int mt) {
      const int zb = mt & 1;
      mbar_wait(&zfull[zb], (mt >> 1) & 1, p.status);
      tc_fence_after();
      float z[32];
      tmem_ld16(tmem_addr(tZN + zb * 64, q * 32, half * 32), *reinterpret_cast<float(*)[16]>(&z[0]));
      tmem_ld16(tmem_addr(tZN + zb * 64, q * 32, half * 32 + 16), *reinterpret_cast<float(*)[16]>(&z[16]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&zfree[zb]);
      if (zissuer) bulk_wait_read<0>();               // the previous add has left the staging tile
      named_bar(2 + half, 128);
      float* zs = reinterpret_cast<float*>(zstage);
#pragma unroll
      for (int i = 0; i < 32; ++i) zs[i * 128 + row] = (half * 32 + i < p.Cc_next) ? z[i] : 0.f;
      fence_proxy_async_smem();
      named_bar(2 + half, 128);
      if (zissuer) {
        tma_reduce_add_2d(&wm.zacc, zstage, (j0 + mt) * 128, b * CT + half * 32);   // mt: local d tile
        bulk_commit();
      }
    };

    // ------------------------------------------------------------ loop B: W_down
    for (int qi = 0; qi < (gram ? 0 : nq); ++qi) {
      const int j = qi >> 2, qq = qi & 3, jj = nch + j;
      if (qq == 0) {
        mbar_wait(&gfull, jj & 1, p.status);
        tc_fence_after();
      }
      float gd[16];
      tmem_ld16(tmem_addr(tGD, q * 32, qq * QW + cq), gd);
      tmem_wait_ld();
      if (qq == 3) {
        tc_fence_before();
        mbar_arrive(&gfree);
      }
      if (!update) {
        if (row_ok && !skip) {
#pragma unroll
          for (int e = 0; e < 16; ++e) acc += gd[e] * gd[e];
        }
        continue;
      }
      if (!stage) continue;
      const int buf = qi % nbufB;
      // this thread's 16 momentum values of S_down row h0 + row (64 contiguous bytes)
      const bool sd_io = update && !skip && row_ok;
      const size_t sdo = s_off + (size_t)(h0 + row) * p.d + (q0 + qi) * QW + cq;
      float4 sdv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        sdv[i] = (kMomentum && sd_io) ? reinterpret_cast<const float4*>(p.s_down + sdo)[i]
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
      mbar_wait(&wfullB[buf], (qi / nbufB) & 1, p.status);
      uint8_t* wd = slots + buf * bytesB;
      float4 w4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {                     // [128 hidden][32 d], 128B swizzle
        const uint32_t o = sw128_offset(row, (cq + 4 * i) * 4);
        w4[i] = *reinterpret_cast<float4*>(wd + o);
        if (!skip) {
          const float4 s4 = sdv[i];
          float4 ns;
          ns.x = (kMomentum ? beta * s4.x : 0.f) - gd[4 * i + 0] * scale;
          ns.y = (kMomentum ? beta * s4.y : 0.f) - gd[4 * i + 1] * scale;
          ns.z = (kMomentum ? beta * s4.z : 0.f) - gd[4 * i + 2] * scale;
          ns.w = (kMomentum ? beta * s4.w : 0.f) - gd[4 * i + 3] * scale;
          w4[i].x = decay * w4[i].x + ns.x;
          w4[i].y = decay * w4[i].y + ns.y;
          w4[i].z = decay * w4[i].z + ns.z;
          w4[i].w = decay * w4[i].w + ns.w;
          *reinterpret_cast<float4*>(wd + o) = w4[i];
          sdv[i] = ns;
        }
      }
      if (write_s && sd_io) {
#pragma unroll
        for (int i = 0; i < 4; ++i) reinterpret_cast<float4*>(p.s_down_out + sdo)[i] = sdv[i];
      }
      if (guard && row_ok) {            // elastic pull of this row's 16 updated W_down values
        const float4* a4 = reinterpret_cast<const float4*>(p.g_w0_down + (size_t)(h0 + row) * p.d + (q0 + qi) * QW + cq);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 a = __ldg(a4 + i);
          const float dx = p.g_keep * (w4[i].x - a.x), dy = p.g_keep * (w4[i].y - a.y);
          const float dz = p.g_keep * (w4[i].z - a.z), dw = p.g_keep * (w4[i].w - a.w);
          w4[i] = make_float4(a.x + dx, a.y + dy, a.z + dz, a.w + dw);
          *reinterpret_cast<float4*>(wd + sw128_offset(row, (cq + 4 * i) * 4)) = w4[i];
          g_down += dx * dx + dy * dy + dz * dz + dw * dw;
        }
      }
      uint8_t* zA = sAU;                                // Z' A tile [128 d][128 hidden], MN-major
      if (fuse) {
        // this thread's 16 W'_down values of its hidden row -> BF16 A tile of d tile j
        if (qq == 0) mbar_wait(&emptyz[0], (j & 1) ^ 1, p.status);   // one A tile: Z' of tile j-1 done
        const int dd = qq * QW + cq;                    // d within the 128-wide tile
        uint4 p0, p1;
        p0.x = pack_bf16x2(w4[0].x, w4[0].y); p0.y = pack_bf16x2(w4[0].z, w4[0].w);
        p0.z = pack_bf16x2(w4[1].x, w4[1].y); p0.w = pack_bf16x2(w4[1].z, w4[1].w);
        p1.x = pack_bf16x2(w4[2].x, w4[2].y); p1.y = pack_bf16x2(w4[2].z, w4[2].w);
        p1.z = pack_bf16x2(w4[3].x, w4[3].y); p1.w = pack_bf16x2(w4[3].z, w4[3].w);
        uint8_t* blk = zA + (dd >> 6) * 16384;
        *reinterpret_cast<uint4*>(blk + sw128_offset(row, (dd & 63) * 2)) = p0;
        *reinterpret_cast<uint4*>(blk + sw128_offset(row, (dd & 63) * 2 + 16)) = p1;
      }
      fence_proxy_async_smem();
      if (fuse && qq == 3) mbar_arrive(&fullz[0]);
      mbar_arrive(&qdoneB[buf]);
      if (fuse && qq == 3 && j > 0) drain_z(j - 1);
    }
    if (fuse) {
      drain_z(nch - 1);
      if (zissuer) bulk_wait_all();
    }
    if (!update) {
      acc = warp_sum(acc);
      if (lane == 0 && !skip) atomicAdd(p.norm2 + b, acc);
    }
    if (guard) {
      g_up = warp_sum(g_up);
      g_gate = warp_sum(g_gate);
      g_down = warp_sum(g_down);
      if (lane == 0) {
        atomicAdd(p.g_sums + 4 * b + 0, g_up);
        atomicAdd(p.g_sums + 4 * b + 1, g_gate);
        atomicAdd(p.g_sums + 4 * b + 2, g_down);
      }
    }
  } else if (warp == STORE_WARP) {
    // W' stores of loops A and B and the staging refills behind them, so the
    // producers never wait for a store to leave shared memory
    if (lane == 0 && stage) {
      mbar_wait(&dh_done, 0, p.status);              // the phase-1 ring is free
      for (int qi = 0; qi < nbufA && qi < nq; ++qi) load_a(qi);
      for (int qi = 0; qi < nq; ++qi) {
        const int buf = qi % nbufA;
        mbar_wait(&qdoneA[buf], (qi / nbufA) & 1, p.status);
        uint8_t* B0 = slots + buf * bytesA;
        if (!skip) {
          tma_store_3d(&wm.up, B0, h0, (q0 + qi) * QW, sb);
          tma_store_3d(&wm.gate, B0 + WTILE, h0, (q0 + qi) * QW, sb);
          bulk_commit();
        }
        if (qi + nbufA < nq) {
          bulk_wait_read<0>();
          load_a(qi + nbufA);
        }
      }
      bulk_wait_read<0>();                           // loop B's staging overlaps loop A's
      for (int qi = 0; qi < nbufB && qi < nq; ++qi) load_b(qi);
      for (int qi = 0; qi < nq; ++qi) {
        const int buf = qi % nbufB;
        mbar_wait(&qdoneB[buf], (qi / nbufB) & 1, p.status);
        uint8_t* B0 = slots + buf * bytesB;
        if (!skip) {
          tma_store_3d(&wm.down, B0, (q0 + qi) * QW, h0, sb);
          bulk_commit();
        }
        if (qi + nbufB < nq) {
          bulk_wait_read<0>();
          load_b(qi + nbufB);
        }
      }
      bulk_wait_all();
    }
  } else if (warp == TMA_WARP) {
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmDZ);
      int it = 0;
      for (int kb = 0; kb < (ops_in ? 0 : nkb); ++kb, ++it) {
        if (!skip) {
          for (int hq = 0; hq < 2; ++hq) {
            const int qi = 2 * kb + hq, fs = qi % NF;
            mbar_wait(&fempty[fs], ((qi / NF) & 1) ^ 1, p.status);
            mbar_arrive_expect_tx(&ffull[fs], WTILE);
            tma_load_3d(fring1 + fs * WTILE, &wm.down, &ffull[fs], (q0 + qi) * QW, h0, sb);
          }
        }
        const int s = it % NSLOT;
        mbar_wait(&empty[s], ((it / NSLOT) & 1) ^ 1, p.status);
        mbar_arrive_expect_tx(&full[s], 8192);
        tma_load_2d(slots + s * BWD_SLOT + 16384, &tmDZ, &full[s], (kb0 + kb) * 64, b * CT);
      }
      // loop A, in the MMA warp's order of use: K slice 0, then per d chunk j
      // the next chunk's K tile 2j, K slice j+1, K tile 2j+1
      auto kslice = [&](int j) {   // MN-major B of gradW_up / gradW_gate, 128 d
        mbar_wait(&empty3, (j & 1) ^ 1, p.status);
        mbar_arrive_expect_tx(&full3, 16384);
        tma_load_3d(slots3, &tmK, &full3, (j0 + j) * 128, p.tok0, b);
        tma_load_3d(slots3 + 8192, &tmK, &full3, (j0 + j) * 128 + 64, p.tok0, b);
      };
      auto knext = [&](int kbi) {  // the next chunk's K tile of 64 d
        if (kbi > 0) mbar_wait(&ug_free, (kbi - 1) & 1, p.status);
        mbar_arrive_expect_tx(&kfull, 8192);
        tma_load_3d(sKN, &tmK, &kfull, (kb0 + kbi) * 64, p.tok0_next, b);
      };
      const bool fuse = kFuse && update;
      if (!gram) kslice(0);
      for (int j = 0; j < (gram ? 0 : nch); ++j) {
        if (fuse) knext(2 * j);
        if (j + 1 < nch) kslice(j + 1);
        if (fuse) knext(2 * j + 1);
      }
      // loop B: dZ slices (MN-major B of gradW_down)
      for (int j = 0; j < (gram ? 0 : nch); ++j) {
        const int jj = nch + j;
        mbar_wait(&empty3, (jj & 1) ^ 1, p.status);
        mbar_arrive_expect_tx(&full3, 16384);
        tma_load_2d(slots3 + 16384, &tmDZ, &full3, (j0 + j) * 128, b * CT);
        tma_load_2d(slots3 + 24576, &tmDZ, &full3, (j0 + j) * 128 + 64, b * CT);
      }
    }
  } else {  // MMA warp
    if (lane == 0) {
      const uint32_t id_dh = idesc_bf16(128, 64, false, false);
      int it = 0;
      for (int kb = 0; kb < (ops_in ? 0 : nkb); ++kb, ++it) {
        const int s = it % NSLOT;
        mbar_wait(&full[s], (it / NSLOT) & 1, p.status);
        tc_fence_after();
        const uint32_t a = smem_u32(slots + s * BWD_SLOT), bz = a + 16384;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_bf16(tDH, sdesc_sw128(a + ks * 32, 16, 1024), sdesc_sw128(bz + ks * 32, 16, 1024), id_dh,
                   (kb > 0 || ks > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      if (ops_in)
        mbar_arrive(&dh_done);                       // no dH MMAs: the phase-1 ring is free at once
      else
        mma_commit(&dh_done);
      mbar_wait(&ops_ready, 0, p.status);
      tc_fence_after();
      const uint32_t id_uw = idesc_bf16(128, 128, false, true);   // A = dU^T K-major, B = K MN-major
      const uint32_t id_dw = idesc_bf16(128, 128, false, true);   // A = H^T K-major, B = dZ slice MN-major
      const uint32_t du = smem_u32(sDU), dg = smem_u32(sDG), ht = smem_u32(sHt);
      const uint32_t id_ug = idesc_bf16(128, 64, false, false);   // next chunk: A = W'^T K-major, B = K' K-major
      const bool fuse = kFuse && update;
      if (gram && ksr == 0 && !skip) {
        // D1 = [dU^T; dG^T] [dU | dG], D2 = [dG^T; H^T] [dG | H]: M = N = 128 tokens in two 64-wide
        // MN-major atoms 16 KB apart (sDU, sDG, sHt are consecutive), K = 128 hidden rows
        const uint32_t id_g = idesc_bf16(128, 128, true, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t d1 = sdesc_sw128(du + ks * 2048, 16384, 1024);
          const uint64_t d2 = sdesc_sw128(dg + ks * 2048, 16384, 1024);
          mma_bf16(tGU, d1, d1, id_g, ks > 0 ? 1u : 0u);
          mma_bf16(tGG, d2, d2, id_g, ks > 0 ? 1u : 0u);
        }
        mma_commit(&gfull);
      }
      auto grad_ug = [&](int j) {                 // gradW_up^T, gradW_gate^T of d chunk j
        mbar_wait(&full3, j & 1, p.status);
        mbar_wait(&gfree, (j & 1) ^ 1, p.status);
        tc_fence_after();
        const uint32_t kk = smem_u32(slots3);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t acc = ks > 0 ? 1u : 0u;
          const uint64_t kd = sdesc_sw128(kk + ks * 2048, 8192, 1024);
          mma_bf16(tGU, sdesc_sw128(du + ks * 32, 16, 1024), kd, id_uw, acc);
          mma_bf16(tGG, sdesc_sw128(dg + ks * 32, 16, 1024), kd, id_uw, acc);
        }
        mma_commit(&empty3);
        mma_commit(&gfull);
      };
      auto next_ug = [&](int kbi) {               // U', G' += K'[kbi] W'[kbi]
        mbar_wait(&a_ready, kbi & 1, p.status);
        mbar_wait(&kfull, kbi & 1, p.status);
        tc_fence_after();
        const uint32_t au = smem_u32(sAU), ag = smem_u32(sAG), kn = smem_u32(sKN);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t bd = sdesc_sw128(kn + ks * 32, 16, 1024);
          const uint32_t acc = (kbi > 0 || ks > 0) ? 1u : 0u;
          mma_bf16(tUN, sdesc_sw128(au + ks * 32, 16, 1024), bd, id_ug, acc);
          mma_bf16(tGN, sdesc_sw128(ag + ks * 32, 16, 1024), bd, id_ug, acc);
        }
        mma_commit(&ug_free);
      };
      // loop A: the gradient tiles of d chunk j+1 are issued as soon as the
      // producers have drained chunk j, ahead of the second U'/G' k-block
      if (!gram) grad_ug(0);
      for (int j = 0; j < (gram ? 0 : nch); ++j) {
        if (fuse) next_ug(2 * j);
        if (j + 1 < nch) grad_ug(j + 1);
        if (fuse) next_ug(2 * j + 1);
      }
      // loop B: gradW_down^T of d chunk j, then Z' of d tile j - 1
      const uint32_t id_z = idesc_bf16(128, 64, true, true);
      const uint32_t hb = smem_u32(sH);
      auto next_z = [&](int mt) {
        const int zb = mt & 1;                     // TMEM accumulator (double); A tile single
        mbar_wait(&fullz[0], mt & 1, p.status);
        mbar_wait(&zfree[zb], ((mt >> 1) & 1) ^ 1, p.status);
        tc_fence_after();
        const uint32_t a = smem_u32(sAU);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_bf16(tZN + zb * 64, sdesc_sw128(a + ks * 2048, 16384, 1024), sdesc_sw128(hb + ks * 2048, 8192, 1024),
                   id_z, ks > 0 ? 1u : 0u);
        mma_commit(&emptyz[0]);
        mma_commit(&zfull[zb]);
      };
      if (fuse) {
        mbar_wait(&h_ready, 0, p.status);
        tc_fence_after();
      }
      for (int j = 0; j < (gram ? 0 : nch); ++j) {
        const int jj = nch + j;
        mbar_wait(&full3, jj & 1, p.status);
        mbar_wait(&gfree, (jj & 1) ^ 1, p.status);
        tc_fence_after();
        const uint32_t zz = smem_u32(slots3) + 16384;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_bf16(tGD, sdesc_sw128(ht + ks * 32, 16, 1024), sdesc_sw128(zz + ks * 2048, 8192, 1024), id_dw,
                   ks > 0 ? 1u : 0u);
        mma_commit(&empty3);
        mma_commit(&gfull);
        if (fuse && j > 0) next_z(j - 1);
      }
      if (fuse) next_z(nch - 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

size_t fwd_smem() { return 1024 + NSLOT * SLOT_BYTES + 16384; }
size_t bwd_smem() { return 1024 + NSLOT * BWD_SLOT + 32768 + 3 * 16384 + 2 * 16384 + 8192; }

using BwdKernel = void (*)(const CUtensorMap, const CUtensorMap, const WMaps, const ChunkParams, int);
// the backward variant for (momentum, fuse, d-split, clip run)
BwdKernel bwd_kernel_table(bool mom, bool fuse, bool split, bool clip) {
  static const BwdKernel k[16] = {
      chunk_bwd_kernel<false, false, false, false>, chunk_bwd_kernel<true, false, false, false>,
      chunk_bwd_kernel<false, true, false, false>,  chunk_bwd_kernel<true, true, false, false>,
      chunk_bwd_kernel<false, false, true, false>,  chunk_bwd_kernel<true, false, true, false>,
      chunk_bwd_kernel<false, true, true, false>,   chunk_bwd_kernel<true, true, true, false>,
      chunk_bwd_kernel<false, false, false, true>,  chunk_bwd_kernel<true, false, false, true>,
      chunk_bwd_kernel<false, true, false, true>,   chunk_bwd_kernel<true, true, false, true>,
      chunk_bwd_kernel<false, false, true, true>,   chunk_bwd_kernel<true, false, true, true>,
      chunk_bwd_kernel<false, true, true, true>,    chunk_bwd_kernel<true, true, true, true>};
  return k[(mom ? 1 : 0) | (fuse ? 2 : 0) | (split ? 4 : 0) | (clip ? 8 : 0)];
}

}  // namespace
}  // namespace uttt

using namespace uttt;

namespace uttt {
namespace {
// Batches of at most this many rows may split d over 2-CTA clusters (the bwd kernel and the
// one-tile forward); at the 1.58B shape (54 hidden tiles) that saves waves for 1, 3, 4, 6, 9, 11,
// 12, 14 and 15 rows.  The workspace sizes include the exchange area up to this batch.
constexpr int DSPLIT_MAX_B = 16;
// ... and, once the unsplit grid fills the SMs, only when each CTA of the pair still streams at
// least 8 of the 128-wide d chunks: at d = 1024 and 8 states (176 CTAs) the split fused launch took
// 0.245 ms against 0.197 ms unsplit, the two exchanges outweighing the halved stream (a memory-bound
// partial last wave is cheap), while at d = 2560 it gains (6 rows: 1.29 -> 1.20 ms, 9 rows: 1.77 ->
// 1.72 ms).  Below one wave it always gains (d = 1024, 2 rows: 0.086 -> 0.073 ms; d = 768, 4 rows:
// 0.120 -> 0.093 ms).
constexpr int DSPLIT_MIN_D = 2048;
// the same for the tensor-core readout of one token tile (uttt_fast_readout)
constexpr int READOUT_DSPLIT_MAX_B = 4;
size_t dsplit_xch_bytes(int B, int h) {
  const size_t tiles = ((size_t)h + HT - 1) / HT;
  return ws_round((size_t)B * tiles * 2 * 3 * HT * CT * sizeof(float));
}
size_t dsplit_flag_bytes(int B, int h) {
  const size_t tiles = ((size_t)h + HT - 1) / HT;
  return ws_round((size_t)B * tiles * 2 * sizeof(unsigned));
}
// 2 when splitting d over 2-CTA clusters saves waves for n one-CTA-per-SM work items
int dsplit_factor(long long n) {
  const long long sms = num_sms();
  const long long w1 = (n + sms - 1) / sms, w2 = (2 * n + sms - 1) / sms;
  return w2 < 2 * w1 ? 2 : 1;
}
// The fwd kernel on `grid` (one CTA per (tile, row)); with KS > 1 its KS-CTA split variant on
// (grid.x * KS, grid.y, grid.z), each cluster one (tile, row), exchange counters zeroed first.
template <typename WT>
int launch_fwd(const CUtensorMap& tm, ChunkParams p, dim3 grid, int KS, size_t flag_bytes, cudaStream_t st) {
  if (KS <= 1) {
    chunk_fwd_kernel<WT, false><<<grid, NTHREADS, fwd_smem(), st>>>(tm, p);
    return launch_status();
  }
  p.dsplit = KS;
  UTTT_TRY(cuda_status(cudaMemsetAsync(p.xflag, 0, flag_bytes, st)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid.x * KS, grid.y, grid.z);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = fwd_smem();
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = KS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, chunk_fwd_kernel<WT, true>, tm, p));
}
int set_fwd_attributes() {
  const void* fns[4] = {(const void*)chunk_fwd_kernel<float, false>, (const void*)chunk_fwd_kernel<float, true>,
                        (const void*)chunk_fwd_kernel<__nv_bfloat16, false>,
                        (const void*)chunk_fwd_kernel<__nv_bfloat16, true>};
  for (const void* fn : fns)
    UTTT_TRY(cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_smem())));
  return UTTT_OK;
}
}  // namespace
}  // namespace uttt

extern "C" size_t uttt_chunk_write_workspace(int B, int C, int d, int h) {
  if (B <= 0 || d <= 0 || h <= 0) return 0;
  (void)C;
  const size_t hp = ((size_t)h + 127) / 128 * 128;
  size_t bytes = 256;
  bytes += ws_round((size_t)B * CT * d * sizeof(float));      // zacc
  bytes += 2 * ws_round((size_t)B * CT * hp * sizeof(float));  // u_save, g_save
  bytes += ws_round((size_t)B * CT * d * 2);                   // dz
  bytes += ws_round((size_t)B * sizeof(float));                 // norm2
  bytes += ws_round((size_t)B * ((h + HT - 1) / HT) * OPS_BYTES);   // clip runs: the norm pass's operands
  bytes += ws_round((size_t)B * 2 * CT * CT * sizeof(float));       //            and the Gram matrices
  if (B <= DSPLIT_MAX_B) bytes += dsplit_xch_bytes(B, h) + dsplit_flag_bytes(B, h);   // d-split exchange
  return bytes;
}

namespace uttt {
namespace {
struct GuardArgs {
  const float* w0_up;
  const float* w0_gate;
  const float* w0_down;
  float keep;
  const int* final_rows;
  float* sums;
};
int chunk_write_impl(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks, const void* q, const void* k,
                     const void* v, const float* eta, const float* alpha, const float* mask, float* w_up,
                     float* w_gate, float* w_down, float* s_up, float* s_gate, float* s_down,
                     const float* ln_weight, const float* ln_bias, float momentum_beta, float max_grad_norm,
                     int normalize_by_dim, float eps, void* out, int out_dtype, float* token_loss, float* clip_scale,
                     int n_states, const int* state_rows, uttt_partial_sum_fn partial_sum, void* partial_sum_ctx,
                     void* workspace, size_t workspace_bytes, void* stream, const GuardArgs* guard);
}  // namespace
}  // namespace uttt

extern "C" int uttt_chunk_write(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks, const void* q,
                                const void* k, const void* v, const float* eta, const float* alpha,
                                const float* mask, float* w_up, float* w_gate, float* w_down, float* s_up,
                                float* s_gate, float* s_down, const float* ln_weight, const float* ln_bias,
                                float momentum_beta, float max_grad_norm, int normalize_by_dim, float eps,
                                void* out, int out_dtype, float* token_loss, float* clip_scale, int n_states,
                                const int* state_rows, uttt_partial_sum_fn partial_sum, void* partial_sum_ctx,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return chunk_write_impl(B, T, C, d, h, chunk_begin, n_chunks, q, k, v, eta, alpha, mask, w_up, w_gate, w_down,
                          s_up, s_gate, s_down, ln_weight, ln_bias, momentum_beta, max_grad_norm, normalize_by_dim,
                          eps, out, out_dtype, token_loss, clip_scale, n_states, state_rows, partial_sum,
                          partial_sum_ctx, workspace, workspace_bytes, stream, nullptr);
}

extern "C" int uttt_chunk_write_guarded(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks,
                                        const void* q, const void* k, const void* v, const float* eta,
                                        const float* alpha, const float* mask, float* w_up, float* w_gate,
                                        float* w_down, float* s_up, float* s_gate, float* s_down,
                                        const float* ln_weight, const float* ln_bias, float momentum_beta,
                                        float max_grad_norm, int normalize_by_dim, float eps, float* token_loss,
                                        int n_states, const int* state_rows, const float* w_up0,
                                        const float* w_gate0, const float* w_down0, float anchor_lambda,
                                        const int* final_rows, float* drift_sums, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  UTTT_REQUIRE(w_up0 && w_gate0 && w_down0 && final_rows && drift_sums, UTTT_ERR_INVALID);
  UTTT_REQUIRE(anchor_lambda >= 0.f && anchor_lambda <= 1.f, UTTT_ERR_INVALID);
  UTTT_REQUIRE(((uintptr_t)w_down0 & 15u) == 0 && d % 4 == 0, UTTT_ERR_UNSUPPORTED);
  const GuardArgs g{w_up0, w_gate0, w_down0, 1.f - anchor_lambda, final_rows, drift_sums};
  return chunk_write_impl(B, T, C, d, h, chunk_begin, n_chunks, k, k, v, eta, alpha, mask, w_up, w_gate, w_down,
                          s_up, s_gate, s_down, ln_weight, ln_bias, momentum_beta, max_grad_norm, normalize_by_dim,
                          eps, nullptr, UTTT_DTYPE_F32, token_loss, nullptr, n_states, state_rows, nullptr, nullptr,
                          workspace, workspace_bytes, stream, &g);
}

namespace uttt {
namespace {
int chunk_write_impl(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks, const void* q, const void* k,
                     const void* v, const float* eta, const float* alpha, const float* mask, float* w_up,
                     float* w_gate, float* w_down, float* s_up, float* s_gate, float* s_down,
                     const float* ln_weight, const float* ln_bias, float momentum_beta, float max_grad_norm,
                     int normalize_by_dim, float eps, void* out, int out_dtype, float* token_loss, float* clip_scale,
                     int n_states, const int* state_rows, uttt_partial_sum_fn partial_sum, void* partial_sum_ctx,
                     void* workspace, size_t workspace_bytes, void* stream, const GuardArgs* guard) {
  UTTT_REQUIRE(B > 0 && T > 0 && C > 0 && d > 0 && h > 0 && n_chunks >= 0 && chunk_begin >= 0, UTTT_ERR_INVALID);
  if (n_states <= 0) n_states = B;
  UTTT_REQUIRE(state_rows != nullptr || n_states == B, UTTT_ERR_INVALID);
  UTTT_REQUIRE(k && v && eta && alpha && w_up && w_gate && w_down && s_up && s_gate && s_down && ln_weight &&
                   ln_bias && workspace,
               UTTT_ERR_INVALID);
  UTTT_REQUIRE(C <= CT, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(d % 128 == 0 && d <= 4096, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(h % 8 == 0, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE((long long)(chunk_begin + n_chunks - 1) * C < T || n_chunks == 0, UTTT_ERR_INVALID);
  UTTT_REQUIRE(out == nullptr || q == k, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(out_dtype == UTTT_DTYPE_F32 || out_dtype == UTTT_DTYPE_BF16, UTTT_ERR_INVALID);
  UTTT_REQUIRE(eps > 0.f && momentum_beta == momentum_beta && max_grad_norm >= 0.f, UTTT_ERR_INVALID);
  UTTT_REQUIRE(workspace_bytes >= uttt_chunk_write_workspace(B, C, d, h), UTTT_ERR_WORKSPACE);
  if (n_chunks == 0) return UTTT_OK;
  cudaStream_t st = (cudaStream_t)stream;

  WsCursor ws(workspace, workspace_bytes);
  const int hp = (h + 127) / 128 * 128;
  ChunkParams p;
  memset(&p, 0, sizeof(p));
  p.B = B; p.T = T; p.C = C; p.d = d; p.h = h; p.hp = hp;
  p.w_up = w_up; p.w_gate = w_gate; p.w_down = w_down;
  p.w_up_out = w_up; p.w_gate_out = w_gate; p.w_down_out = w_down;
  p.s_up = s_up; p.s_gate = s_gate; p.s_down = s_down;
  p.s_up_out = s_up; p.s_gate_out = s_gate; p.s_down_out = s_down;
  p.eta = eta; p.alpha = alpha; p.mask = mask; p.ln_w = ln_weight; p.ln_b = ln_bias;
  p.k = (const __nv_bfloat16*)k; p.v = (const __nv_bfloat16*)v;
  p.zacc = ws.take<float>((size_t)B * CT * d);
  p.u_save = ws.take<float>((size_t)B * CT * hp);
  p.g_save = ws.take<float>((size_t)B * CT * hp);
  p.dz = ws.take<__nv_bfloat16>((size_t)B * CT * d);
  p.norm2 = ws.take<float>(B);
  p.token_loss = token_loss; p.out = out; p.out_bf16 = out_dtype == UTTT_DTYPE_BF16;
  p.clip_out = clip_scale;
  p.n_chunks = n_chunks;
  p.call_end = (chunk_begin + n_chunks) * C < T ? (chunk_begin + n_chunks) * C : T;
  p.beta = momentum_beta; p.clip = max_grad_norm; p.eps = eps;
  p.inv_scale = normalize_by_dim ? 1.f / (float)d : 1.f;
  p.status = ws_status(workspace);
  p.src_up = w_up; p.src_gate = w_gate; p.src_down = w_down;
  p.ss_ug = (long long)d * h; p.ss_d = (long long)h * d; p.ld_ug = h;
  p.state_index = state_rows;
  p.n_states = n_states;
  if (guard) {
    p.g_w0_up = guard->w0_up;
    p.g_w0_gate = guard->w0_gate;
    p.g_w0_down = guard->w0_down;
    p.g_keep = guard->keep;
    p.g_final = guard->final_rows;
    p.g_sums = guard->sums;
  }
  if (max_grad_norm > 0.f) {
    p.ops = ws.take<uint8_t>((size_t)B * ((h + HT - 1) / HT) * OPS_BYTES);
    p.gram = ws.take<float>((size_t)B * 2 * CT * CT);
  }
  if (!ws.ok()) return UTTT_ERR_WORKSPACE;
  // d-split of the bwd kernel: with few rows, 54 hidden tiles per 1.58B state leave SMs idle or
  // end on a thin last wave; two CTAs per (tile, state), each streaming half of d, finish in
  // fewer waves.  Used when it saves waves and the caller's workspace holds the exchange area.
  const int ntiles = (h + HT - 1) / HT;
  int KS = 1;
  if (B <= DSPLIT_MAX_B && (d >= DSPLIT_MIN_D || (long long)ntiles * B < num_sms()) && (d / 128) % 2 == 0) {
    const size_t xb = dsplit_xch_bytes(B, h), fb = dsplit_flag_bytes(B, h);
    if (dsplit_factor((long long)ntiles * B) == 2 && ws.used + xb + fb <= ws.cap) {
      p.xch = ws.take<float>(xb / sizeof(float));
      p.xflag = ws.take<unsigned>(fb / sizeof(unsigned));
      KS = 2;
    }
  }

  CUtensorMap tmK, tmDZ;
  {
    uint64_t dims[3] = {(uint64_t)d, (uint64_t)T, (uint64_t)B};
    uint64_t str[2] = {(uint64_t)d * 2, (uint64_t)T * d * 2};
    uint32_t box[3] = {64, 64, 1};
    UTTT_TRY(make_tmap_bf16(&tmK, k, 3, dims, str, box));
  }
  {
    uint64_t dims[2] = {(uint64_t)d, (uint64_t)B * CT};
    uint64_t str[1] = {(uint64_t)d * 2};
    uint32_t box[2] = {64, 64};
    UTTT_TRY(make_tmap_bf16(&tmDZ, p.dz, 2, dims, str, box));
  }
  WMaps wmaps;
  {
    uint64_t dims_ug[3] = {(uint64_t)h, (uint64_t)d, (uint64_t)n_states};
    uint64_t str_ug[2] = {(uint64_t)h * 4, (uint64_t)d * h * 4};
    uint32_t box_ug[3] = {HT, QW, 1};
    uint64_t dims_d[3] = {(uint64_t)d, (uint64_t)h, (uint64_t)n_states};
    uint64_t str_d[2] = {(uint64_t)d * 4, (uint64_t)h * d * 4};
    uint32_t box_d[3] = {QW, HT, 1};
    UTTT_TRY(make_tmap_f32(&wmaps.up, w_up, 3, dims_ug, str_ug, box_ug, false));
    UTTT_TRY(make_tmap_f32(&wmaps.gate, w_gate, 3, dims_ug, str_ug, box_ug, false));
    UTTT_TRY(make_tmap_f32(&wmaps.down, w_down, 3, dims_d, str_d, box_d, true));
    uint64_t dims_z[2] = {(uint64_t)d, (uint64_t)B * CT};
    uint64_t str_z[1] = {(uint64_t)d * 4};
    uint32_t box_z[2] = {128, 32};
    UTTT_TRY(make_tmap_f32(&wmaps.zacc, p.zacc, 2, dims_z, str_z, box_z, false));
  }
  static DeviceOnce attr_done;
  UTTT_TRY(run_once_per_device(attr_done, [] {
    UTTT_TRY(set_fwd_attributes());
    for (int i = 0; i < 16; ++i)
      UTTT_TRY(cuda_status(cudaFuncSetAttribute((const void*)bwd_kernel_table(i & 1, i & 2, i & 4, i & 8),
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bwd_smem())));
    return (int)UTTT_OK;
  }));
  UTTT_TRY(cuda_status(cudaMemsetAsync(p.zacc, 0, (size_t)B * CT * d * sizeof(float), st)));
  const dim3 grid((h + HT - 1) / HT, B);
  // bwd launch: grid (tiles, rows, KS); with KS > 1 the KS CTAs of a (tile, row) form one
  // cluster (co-scheduled, so their exchange waits always end) and the exchange counters
  // start from zero
  auto launch_bwd = [&](BwdKernel kernel, int update, int ks) -> int {
    if (ks > 1)
      UTTT_TRY(cuda_status(cudaMemsetAsync(p.xflag, 0, dsplit_flag_bytes(B, h), st)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntiles, B, ks);
    cfg.blockDim = dim3(BWD_THREADS);
    cfg.dynamicSmemBytes = bwd_smem();
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = ks;
    cfg.attrs = at;
    cfg.numAttrs = ks > 1 ? 1 : 0;
    return cuda_status(cudaLaunchKernelEx(&cfg, kernel, tmK, tmDZ, wmaps, p, update));
  };
  // The forward of every chunk but the first runs inside the previous chunk's
  // backward kernel (kFuse), from the weight tiles it has just updated.
  for (int ci = 0; ci < n_chunks; ++ci) {
    p.tok0 = (chunk_begin + ci) * C;
    p.Cc = (T - p.tok0) < C ? (T - p.tok0) : C;
    p.chunk_index = ci;
    const bool fuse = ci + 1 < n_chunks;
    p.tok0_next = p.tok0 + C;
    p.Cc_next = fuse ? ((T - p.tok0_next) < C ? (T - p.tok0_next) : C) : 0;
    if (ci == 0) {
      ProfScope ps(UTTT_PROF_CHUNK_FWD, st);
      UTTT_TRY(launch_fwd<float>(tmK, p, grid, KS, dsplit_flag_bytes(B, h), st));
    }
    UTTT_TRY(launch_status());
    // hidden split: this chunk's Z is the sum of every rank's partial Z
    if (ci == 0 && partial_sum && partial_sum(p.zacc, (size_t)B * CT * d, partial_sum_ctx, stream) != 0)
      return UTTT_ERR_CUDA;
    {
      ProfScope ps(UTTT_PROF_CHUNK_LN, st);
      chunk_ln_for(d)<<<dim3(CT / LN_ROWS, B), LN_ROWS * 32, 0, st>>>(p);
    }
    UTTT_TRY(launch_status());
    if (max_grad_norm > 0.f) {
      ProfScope ps(UTTT_PROF_CHUNK_NORM, st);
      UTTT_TRY(cuda_status(cudaMemsetAsync(p.gram, 0, (size_t)B * 2 * CT * CT * sizeof(float), st)));
      chunk_gram_kernel<<<dim3(d / GRAM_D, B), 256, 0, st>>>(p);
      UTTT_TRY(launch_status());
      // unsplit: the norm pass streams only W_down, and a pair's exchange of dH plus rank 0's Gram
      // tail cost more than the halved stream saves (measured at 6 and 9 rows of the 1.58B shape)
      UTTT_TRY(launch_bwd(bwd_kernel_table(momentum_beta != 0.f, false, false, true), 0, 1));
      UTTT_TRY(launch_status());
      // hidden split: the clip norm runs over every rank's gradient slices
      if (partial_sum && partial_sum(p.norm2, (size_t)B, partial_sum_ctx, stream) != 0) return UTTT_ERR_CUDA;
    }
    UTTT_TRY(launch_status());
    {
      ProfScope ps(UTTT_PROF_CHUNK_BWD, st);
      UTTT_TRY(launch_bwd(bwd_kernel_table(momentum_beta != 0.f, fuse, KS > 1, max_grad_norm > 0.f), 1, KS));
    }
    UTTT_TRY(launch_status());
    // hidden split: the next chunk's Z (computed by the fused kernel) from every rank's slices
    if (fuse && partial_sum && partial_sum(p.zacc, (size_t)B * CT * d, partial_sum_ctx, stream) != 0)
      return UTTT_ERR_CUDA;
  }
  return UTTT_OK;
}
}  // namespace
}  // namespace uttt

// ============================================================================
// fast-weight readout entry point
// ============================================================================
namespace uttt {
int launch_readout_decode(int B, int d, int h, const __nv_bfloat16* x, const __nv_bfloat16* wp,
                          const __nv_bfloat16* wd, const int* state_index, const float* ln_w, const float* ln_b,
                          float eps, float* zacc, unsigned* done, void* out, int out_bf16, cudaStream_t st);
int launch_readout_finish(int B, int d, const float* z, const __nv_bfloat16* x, const float* ln_w, const float* ln_b,
                          float eps, void* out, int out_bf16, int z_bf16, cudaStream_t st);
}

extern "C" int uttt_fast_readout_partial(int B, int T, int d, int h, const void* x, const void* w_packed,
                                         const void* w_down, const int* state_index, float* z, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  UTTT_REQUIRE(B > 0 && T > 0 && d > 0 && h > 0 && x && w_packed && w_down && z && workspace, UTTT_ERR_INVALID);
  UTTT_REQUIRE(d % 128 == 0 && d <= 4096 && h % 8 == 0, UTTT_ERR_UNSUPPORTED);
  // the tensor-core readout copies the BF16 read copies in 16-byte pieces
  UTTT_REQUIRE((((uintptr_t)w_packed | (uintptr_t)w_down) & 15u) == 0, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(workspace_bytes >= 256, UTTT_ERR_WORKSPACE);
  cudaStream_t st = (cudaStream_t)stream;
  UTTT_TRY(cuda_status(cudaMemsetAsync(z, 0, (size_t)B * T * d * sizeof(float), st)));
  ProfScope ps(UTTT_PROF_READOUT, st);
  if (T == 1)
    return launch_readout_decode(B, d, h, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w_packed,
                                 (const __nv_bfloat16*)w_down, state_index, nullptr, nullptr, 1.f, z, nullptr, nullptr,
                                 1, st);
  static DeviceOnce attr_done;
  UTTT_TRY(run_once_per_device(attr_done, [] { return set_fwd_attributes(); }));
  ChunkParams p;
  memset(&p, 0, sizeof(p));
  p.B = B; p.T = T; p.C = CT; p.d = d; p.h = h; p.hp = (h + 127) / 128 * 128;
  p.zacc = z;
  p.z_rows = T;
  p.status = ws_status(workspace);
  p.k = (const __nv_bfloat16*)x;
  p.src_up = w_packed;
  p.src_gate = (const __nv_bfloat16*)w_packed + h;
  p.ld_ug = 2 * h;
  p.ss_ug = (long long)d * 2 * h;
  p.src_down = w_down;
  p.ss_d = (long long)h * d;
  p.state_index = state_index;
  p.tiles = 1;
  CUtensorMap tmX;
  {
    uint64_t dims[3] = {(uint64_t)d, (uint64_t)T, (uint64_t)B};
    uint64_t str[2] = {(uint64_t)d * 2, (uint64_t)T * d * 2};
    uint32_t box[3] = {64, 64, 1};
    UTTT_TRY(make_tmap_bf16(&tmX, x, 3, dims, str, box));
  }
  return launch_fwd<__nv_bfloat16>(tmX, p, dim3((T + CT - 1) / CT, (h + HT - 1) / HT, B), 1, 0, st);
}

extern "C" int uttt_readout_finish(int B, int d, const float* z, const void* x, const float* ln_weight,
                                   const float* ln_bias, float eps, void* out, int out_dtype, int z_bf16,
                                   void* stream) {
  UTTT_REQUIRE(B > 0 && d > 0 && z && x && ln_weight && ln_bias && out, UTTT_ERR_INVALID);
  UTTT_REQUIRE(out_dtype == UTTT_DTYPE_F32 || out_dtype == UTTT_DTYPE_BF16, UTTT_ERR_INVALID);
  UTTT_REQUIRE(d % 128 == 0 && d <= 4096 && eps > 0.f, UTTT_ERR_UNSUPPORTED);
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps(UTTT_PROF_READOUT_LN, st);
  return launch_readout_finish(B, d, z, (const __nv_bfloat16*)x, ln_weight, ln_bias, eps, out,
                               out_dtype == UTTT_DTYPE_BF16, z_bf16 != 0, st);
}

extern "C" size_t uttt_fast_readout_workspace(int B, int T, int d, int h) {
  if (B <= 0 || T <= 0 || d <= 0 || h <= 0) return 0;
  size_t bytes = 256 + ws_round((size_t)B * (T > CT ? T : CT) * d * sizeof(float));
  // one token tile of a few rows: room for the d-split exchange of the tensor-core readout
  if (T > 1 && T <= CT && B <= READOUT_DSPLIT_MAX_B) bytes += dsplit_xch_bytes(B, h) + dsplit_flag_bytes(B, h);
  return bytes;
}

extern "C" int uttt_fast_readout(int B, int T, int d, int h, const void* x, int w_dtype, const void* w_up,
                                 const void* w_gate, const void* w_down, const int* state_index,
                                 const float* ln_weight, const float* ln_bias, float eps, void* out, int out_dtype,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  UTTT_REQUIRE(B > 0 && T > 0 && d > 0 && h > 0, UTTT_ERR_INVALID);
  UTTT_REQUIRE(x && w_up && w_down && ln_weight && ln_bias && out && workspace, UTTT_ERR_INVALID);
  UTTT_REQUIRE(w_dtype == UTTT_DTYPE_F32 || w_dtype == UTTT_DTYPE_BF16, UTTT_ERR_INVALID);
  UTTT_REQUIRE(w_dtype == UTTT_DTYPE_BF16 || w_gate, UTTT_ERR_INVALID);
  UTTT_REQUIRE(out_dtype == UTTT_DTYPE_F32 || out_dtype == UTTT_DTYPE_BF16, UTTT_ERR_INVALID);
  UTTT_REQUIRE(d % 128 == 0 && d <= 4096 && h % 8 == 0, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(eps > 0.f, UTTT_ERR_INVALID);
  UTTT_REQUIRE(w_dtype == UTTT_DTYPE_F32 || (((uintptr_t)w_up | (uintptr_t)w_down) & 15u) == 0, UTTT_ERR_UNSUPPORTED);
  UTTT_REQUIRE(workspace_bytes >= uttt_fast_readout_workspace(B, T, d, h), UTTT_ERR_WORKSPACE);
  cudaStream_t st = (cudaStream_t)stream;
  WsCursor ws(workspace, workspace_bytes);
  float* zacc = ws.take<float>((size_t)B * (T > CT ? T : CT) * d);
  if (!ws.ok()) return UTTT_ERR_WORKSPACE;
  const int ob = out_dtype == UTTT_DTYPE_BF16;
  if (T == 1 && w_dtype == UTTT_DTYPE_BF16) {
    // decode: one token per state, memory-bound GEMV over the BF16 read copies
    // with the LayerNorm + residual in its last CTA per state; z (B, d) and the
    // per-state completion counters (B) sit at the front of the z buffer
    unsigned* done = reinterpret_cast<unsigned*>(zacc + (size_t)B * d);
    UTTT_TRY(cuda_status(cudaMemsetAsync(zacc, 0, (size_t)B * d * sizeof(float) + (size_t)B * sizeof(unsigned), st)));
    ProfScope ps(UTTT_PROF_READOUT, st);
    return launch_readout_decode(B, d, h, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w_up,
                                 (const __nv_bfloat16*)w_down, state_index, ln_weight, ln_bias, eps, zacc, done, out,
                                 ob, st);
  }
  UTTT_TRY(cuda_status(cudaMemsetAsync(zacc, 0, (size_t)B * T * d * sizeof(float), st)));
  static DeviceOnce attr_done;
  UTTT_TRY(run_once_per_device(attr_done, [] { return set_fwd_attributes(); }));
  ChunkParams p;
  memset(&p, 0, sizeof(p));
  p.B = B; p.T = T; p.C = CT; p.d = d; p.h = h; p.hp = (h + 127) / 128 * 128;
  p.zacc = zacc;
  p.status = ws_status(workspace);
  p.k = (const __nv_bfloat16*)x;
  if (w_dtype == UTTT_DTYPE_BF16) {
    p.src_up = w_up;
    p.src_gate = (const __nv_bfloat16*)w_up + h;
    p.ld_ug = 2 * h;
    p.ss_ug = (long long)d * 2 * h;
  } else {
    p.src_up = w_up;
    p.src_gate = w_gate;
    p.ld_ug = h;
    p.ss_ug = (long long)d * h;
  }
  p.src_down = w_down;
  p.ss_d = (long long)h * d;
  p.state_index = state_index;
  // every 64-token tile in one launch (token tiles fastest: the CTAs of a hidden tile share
  // its weight slice through L2), z rows (B, T, d), then one LayerNorm launch over all rows
  p.tiles = 1;
  p.z_rows = T;
  CUtensorMap tmX;
  {
    uint64_t dims[3] = {(uint64_t)d, (uint64_t)T, (uint64_t)B};
    uint64_t str[2] = {(uint64_t)d * 2, (uint64_t)T * d * 2};
    uint32_t box[3] = {64, 64, 1};
    UTTT_TRY(make_tmap_bf16(&tmX, x, 3, dims, str, box));
  }
  const dim3 grid((T + CT - 1) / CT, (h + HT - 1) / HT, B);
  // one token tile of a few rows (the write path's per-layer readout of a chunk): split d over
  // 2-CTA clusters when that saves waves and the workspace holds the exchange area
  int KS = 1;
  const size_t fbytes = dsplit_flag_bytes(B, h);
  if (T > 1 && T <= CT && B <= READOUT_DSPLIT_MAX_B && (d / 128) % 2 == 0 &&
      dsplit_factor((long long)grid.y * B) == 2) {
    const size_t xb = dsplit_xch_bytes(B, h);
    if (ws.used + xb + fbytes <= ws.cap) {
      p.xch = ws.take<float>(xb / sizeof(float));
      p.xflag = ws.take<unsigned>(fbytes / sizeof(unsigned));
      KS = 2;
    }
  }
  {
    ProfScope ps(UTTT_PROF_READOUT, st);
    if (w_dtype == UTTT_DTYPE_BF16)
      UTTT_TRY(launch_fwd<__nv_bfloat16>(tmX, p, grid, KS, fbytes, st));
    else
      UTTT_TRY(launch_fwd<float>(tmX, p, grid, KS, fbytes, st));
  }
  UTTT_TRY(launch_status());
  {
    ProfScope ps(UTTT_PROF_READOUT_LN, st);
    readout_ln_kernel<<<dim3(T, B), LN_THREADS, 0, st>>>(zacc, T, (const __nv_bfloat16*)x, T, 0, T, d, ln_weight,
                                                         ln_bias, eps, out, ob);
  }
  return launch_status();
}
