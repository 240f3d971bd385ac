/*
 * uttt_b200.h -- C ABI of the B200-native uTTT serving hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*), launches asynchronously on that stream and returns an
 * int status (UTTT_OK or one of the error codes below).  Invalid arguments
 * are rejected on the host before any launch.  Bounded device-side waits
 * that expire record UTTT_ERR_TIMEOUT in the first int of the workspace;
 * read it with uttt_read_status() after the stream is synchronised.
 *
 * Tensor layouts are the reference's (Phova/uTTTCompanion,
 * model/uttt_layer.py): activations (B, T, d) row-major, fast weights
 * w_up / w_gate (B, d, h) and w_down (B, h, d) row-major FP32 masters,
 * LayerNorm weight / bias (d,).  BF16 buffers hold IEEE bfloat16 bits.
 */
#ifndef UTTT_B200_H
#define UTTT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define UTTT_OK 0
#define UTTT_ERR_INVALID 1     /* bad argument or shape   -> Python ValueError   */
#define UTTT_ERR_UNSUPPORTED 2 /* unsupported size/option  -> Python ValueError   */
#define UTTT_ERR_CUDA 3        /* CUDA launch/runtime error -> Python RuntimeError */
#define UTTT_ERR_TIMEOUT 4     /* bounded device wait expired -> RuntimeError    */
#define UTTT_ERR_WORKSPACE 5   /* workspace too small       -> ValueError        */

/* dtype tags for outputs */
#define UTTT_DTYPE_F32 0
#define UTTT_DTYPE_BF16 1

/* ---- library ----------------------------------------------------------- */
int uttt_version(void);
const char* uttt_status_string(int status);
/* Last CUDA runtime error code seen by the library on this thread (0 if none). */
int uttt_last_cuda_error(void);
/* Reads (and, if reset != 0, clears) the device status word at the start of a
 * workspace.  Synchronises `stream`. */
int uttt_read_status(void* workspace, int reset, void* stream);

/* ---- live kernel timing ------------------------------------------------- */
/* When enabled, every launcher brackets its kernels with CUDA events on the
 * launch stream, per kernel kind.  uttt_profile_read synchronises, writes the
 * total milliseconds and launch count of each kind (arrays of length
 * UTTT_PROF_KINDS) and resets the counters.  No counterpart in the reference
 * (which times with torch.cuda.synchronize + perf_counter,
 * deploy/benchmark_inference_speed.py:136-183). */
#define UTTT_PROF_KINDS 16
#define UTTT_PROF_CHUNK_FWD 0
#define UTTT_PROF_CHUNK_LN 1
#define UTTT_PROF_CHUNK_NORM 2
#define UTTT_PROF_CHUNK_BWD 3
#define UTTT_PROF_READOUT 4
#define UTTT_PROF_READOUT_LN 5
#define UTTT_PROF_GEMM 6
#define UTTT_PROF_FINISH 7
#define UTTT_PROF_ATTN 8
#define UTTT_PROF_ROWWISE 9
#define UTTT_PROF_ARGMAX 10
int uttt_profile_enable(int on);
int uttt_profile_read(float* total_ms, int* launches);

/* ---- diagnostics -------------------------------------------------------- */
/* D(MxN, fp32) = A * B^T on the tensor cores, used by the self-tests that pin
 * the descriptor / swizzle / TMEM conventions.  mode bit0: A is given
 * MN-major (K x M row-major) instead of K-major (M x K); bit1: same for B;
 * bit2: A is FP32 (converted to BF16 by software producers).  M % 128 == 0,
 * N in {64,128,256}, K % 64 == 0.  No counterpart in the reference. */
int uttt_selftest_gemm(int mode, int M, int N, int K, const void* a, const void* b, float* d, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Bounded-wait self-test: launches one CTA that waits, with the kernels' own
 * bounded-wait code, on an event that never happens (kind 0: an mbarrier phase
 * with no arrival; kind 1: a d-split exchange counter that nothing increments)
 * for at most max_polls polls (1 .. 2^20).  The wait expires, records
 * UTTT_ERR_TIMEOUT in the workspace status word (read it with
 * uttt_read_status) and sets the int at byte 260 of the workspace to 1 when the
 * kernel returns.  workspace_bytes >= 512.  No counterpart in the reference;
 * it shows that an expired device wait reaches the caller as an error while the
 * context stays usable. */
int uttt_selftest_wait(int kind, unsigned max_polls, void* workspace, size_t workspace_bytes, void* stream);

/* ---- chunk-wise TTT write ---------------------------------------------- */
/* Host hook of a hidden-dimension split: replaces `count` FP32 values at
 * device address `data` by their sum over every rank of the split (an
 * all-reduce), ordered on `stream`; returns 0 on success. */
typedef int (*uttt_partial_sum_fn)(float* data, size_t count, void* ctx, void* stream);

/*
 * Replaces fused_chunk_ttt_step (model/uttt_layer.py:414-534) and its
 * analytical gradient analytical_swiglu_chunk_grad (:279-411), for B
 * independent states, over n_chunks consecutive chunks of C tokens starting
 * at token chunk_begin*C of every state's T-token sequence.  Chunks are
 * applied sequentially (each reads the state the previous one wrote), as
 * SharedFastWeightPool.chunk_step (:697-771) chains them.
 *
 *   q, k, v        BF16 (B, T, d); q may equal k.
 *   eta, alpha     FP32 (B, T) per-token inner lr and decay gate.
 *   mask           FP32 (B, T) right-padding mask or NULL.
 *   w_*, s_*       FP32 masters, updated IN PLACE.
 *   ln_weight/bias FP32 (d,).
 *   out            readout (B, T, d) of f_W(q) with each chunk's pre-update
 *                  weights, written only when q == k (it is then v_hat);
 *                  otherwise pass NULL and call uttt_fast_readout first.
 *   token_loss     FP32 (B, T): 0.5*||f_W(k_t) - v_t||^2 (/d if normalize)
 *                  per token (the unweighted surprise terms), or NULL.
 *   clip_scale     FP32 (B, n_chunks): applied clip factor per chunk, or NULL.
 *   n_states,      ragged batches: row b of the activations (and of mask,
 *   state_rows     token_loss, clip_scale, out) updates fast-weight state
 *                  state_rows[b] (int32 device array, B entries, distinct)
 *                  of w_* / s_*, which hold n_states states.  NULL: row b
 *                  updates state b and n_states must be B (or <= 0).  A row
 *                  whose entry is not below n_states touches nothing and
 *                  records UTTT_ERR_INVALID in the workspace status word.
 *   partial_sum,   hidden split over P ranks: w_* / s_* hold this rank's
 *   partial_sum_ctx hidden units (h = its slice width) and the call sums the
 *                  partial Z of every chunk (B*64*d floats of the workspace)
 *                  and, with clipping, the squared gradient norms (B floats)
 *                  through the hook between its launches; NULL: unsplit.
 *                  A hook that fails ends the call with UTTT_ERR_CUDA.
 *
 * Requires d % 128 == 0, 1 <= C <= 64.
 *
 * uttt_chunk_write_workspace: bytes of device scratch the call needs (the
 * status word, partial Z, saved U / G, dZ and norms of a 64-token chunk; for
 * clipped calls the norm pass's dU / dG / H tiles, 48 KB per row and 128
 * hidden units, and two 64 x 64 Gram matrices per row; for B <= 16 the
 * exchange area of the 2-CTA d-split).
 */
size_t uttt_chunk_write_workspace(int B, int C, int d, int h);
int uttt_chunk_write(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks, const void* q, const void* k,
                     const void* v, const float* eta, const float* alpha, const float* mask, float* w_up,
                     float* w_gate, float* w_down, float* s_up, float* s_gate, float* s_down,
                     const float* ln_weight, const float* ln_bias, float momentum_beta, float max_grad_norm,
                     int normalize_by_dim, float eps, void* out, int out_dtype, float* token_loss,
                     float* clip_scale, int n_states, const int* state_rows, uttt_partial_sum_fn partial_sum,
                     void* partial_sum_ctx, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The same write with the stability guard of a persona turn folded into it
 * (apply_elastic_pull, model/uttt_layer.py:773-832, and the sums of
 * compute_drift, :834-874; engine/personalizer.py:524-552 applies them after
 * the write): on the call's last chunk, every row b with final_rows[b] != 0
 * (int32 device array, B entries) is pulled towards the shared W_0 right after
 * its update, W <- W0 + (1 - anchor_lambda)(W - W0), inside the update kernel,
 * and drift_sums[4b + m] (FP32 device, B x 4; zero it before the first call)
 * receives ||W_m - W0_m||^2 of the pulled matrices m = up, gate, down.  The
 * caller derives the drift clamp's scale from those sums (a second pass only
 * when the clamp bites).  W0 is w_up0, w_gate0 (d, h) and w_down0 (h, d) FP32.
 * q = k (the write's own readout is not produced), no clip-scale output, no
 * hidden split; otherwise as uttt_chunk_write, with the same workspace.
 */
int uttt_chunk_write_guarded(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks, const void* q,
                             const void* k, const void* v, const float* eta, const float* alpha, const float* mask,
                             float* w_up, float* w_gate, float* w_down, float* s_up, float* s_gate, float* s_down,
                             const float* ln_weight, const float* ln_bias, float momentum_beta, float max_grad_norm,
                             int normalize_by_dim, float eps, float* token_loss, int n_states, const int* state_rows,
                             const float* w_up0, const float* w_gate0, const float* w_down0, float anchor_lambda,
                             const int* final_rows, float* drift_sums, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * Allocation-free chunk write.  No counterpart in the reference.  (Rows map
 * to states one to one: n_states = B, state_rows = NULL.)
 *
 * For callers that cannot call cudaMalloc: serving loops whose HBM is fully
 * reserved up front (an extra allocation would fail, and cudaMalloc / cudaFree
 * may synchronise the device and stall the decode streams), and host code in
 * foreign-language bindings that has no device allocator.  Same arguments and
 * results as uttt_chunk_write, minus the workspace: the scratch is a fixed
 * UTTT_NOALLOC_SCRATCH_BYTES device array inside the library, held on every
 * device that loads it until the process exits.  Sizes whose
 * uttt_chunk_write_workspace(B, C, d, h) exceeds it are rejected with
 * UTTT_ERR_WORKSPACE before any work.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress), so make that first call
 * before any stream capture.  All calls share the array: calls that overlap
 * on the GPU race and must be ordered by the caller.  The array's status word
 * is cleared at the start of each call; read it after the call (and before the
 * next one) with uttt_chunk_write_noalloc_status.  The array's device address
 * is cached per device and per CUDA context: after cudaDeviceReset (or any
 * re-creation of the primary context) the next call looks it up again, so
 * that call too must come before any stream capture.
 */
#define UTTT_NOALLOC_SCRATCH_BYTES (8u << 20)
int uttt_chunk_write_noalloc(int B, int T, int C, int d, int h, int chunk_begin, int n_chunks, const void* q,
                             const void* k, const void* v, const float* eta, const float* alpha, const float* mask,
                             float* w_up, float* w_gate, float* w_down, float* s_up, float* s_gate, float* s_down,
                             const float* ln_weight, const float* ln_bias, float momentum_beta,
                             float max_grad_norm, int normalize_by_dim, float eps, void* out, int out_dtype,
                             float* token_loss, float* clip_scale, void* stream);
/* Status word of the allocation-free write's static scratch on the current
 * device: synchronises `stream`, returns UTTT_OK if every bounded device wait of
 * the last uttt_chunk_write_noalloc call ended, UTTT_ERR_TIMEOUT if one expired
 * (that call's state may then be wrong), or UTTT_ERR_CUDA if the word could not
 * be read; reset != 0 clears the word.  Allocates nothing.  No counterpart in
 * the reference. */
int uttt_chunk_write_noalloc_status(int reset, void* stream);

/* ---- fast-weight readout ------------------------------------------------ */
/*
 * f_W(x) = x + LayerNorm(silu(x W_gate) * (x W_up) W_down) for B states of T
 * tokens each.  Replaces swiglu_fast_forward / swiglu_packed_forward
 * (model/uttt_layer.py:211-257) as called by
 * SharedFastWeightPool.forward_readout (:670-695).
 *
 *   x            BF16 (B, T, d)
 *   w_dtype      UTTT_DTYPE_F32: w_up, w_gate (S, d, h), w_down (S, h, d) FP32
 *                masters;  UTTT_DTYPE_BF16: w_up = packed [W_up | W_gate]
 *                (S, d, 2h) BF16 read copy (inference_read_weights, :648-668),
 *                w_gate unused, w_down (S, h, d) BF16.
 *   state_index  int32 (B): row b reads state state_index[b] (NULL: state b);
 *                with T == 1 and BF16 copies a negative entry marks a padding
 *                row of a packed batch: no weights are read and its output is x.
 *   ln_*         FP32 (d,) LayerNorm affine, as the reference applies it.
 *   out          (B, T, d) in out_dtype.
 * T == 1 with BF16 copies runs the decode GEMV; otherwise 64-token tiles on
 * the tensor cores.  Requires d % 128 == 0, h % 8 == 0.
 */
size_t uttt_fast_readout_workspace(int B, int T, int d, int h);
int uttt_fast_readout(int B, int T, int d, int h, const void* x, int w_dtype, const void* w_up, const void* w_gate,
                      const void* w_down, const int* state_index, const float* ln_weight, const float* ln_bias,
                      float eps, void* out, int out_dtype, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Hidden-dimension split of the decode readout (the 1.58B configuration over
 * P GPUs): each rank holds hidden units [r*h, (r+1)*h) of every persona, as
 * packed BF16 [W_up | W_gate] (S, d, 2h) and W_down (S, h, d) slices.
 * uttt_fast_readout_partial writes that slice's z = h_slice W_down_slice,
 * FP32 (B, T, d) (z is zeroed first; T == 1 runs the decode GEMV, T > 1 the
 * tensor-core tiles; the workspace only holds the status word).  After the ranks' z are summed (an all-reduce),
 * uttt_readout_finish applies out = x + LayerNorm(z) * ln_weight + ln_bias to
 * `rows` rows of (rows, d), z rounded to BF16 first when z_bf16 != 0 (as the
 * decode readout, T == 1, does; the tensor-core tiles of T > 1 keep z in
 * FP32).  Together they equal uttt_fast_readout
 * (swiglu_packed_forward, model/uttt_layer.py:250-257): every hidden unit's
 * u, g and h are computed whole on one rank.
 */
int uttt_fast_readout_partial(int B, int T, int d, int h, const void* x, const void* w_packed, const void* w_down,
                              const int* state_index, float* z, void* workspace, size_t workspace_bytes,
                              void* stream);
int uttt_readout_finish(int rows, int d, const float* z, const void* x, const float* ln_weight, const float* ln_bias,
                        float eps, void* out, int out_dtype, int z_bf16, void* stream);

/*
 * The same sum-and-finish without NCCL, over NVLink peer memory: each rank
 * owns an exchange area of uttt_split_exchange_bytes(world, max_rows, d)
 * bytes, allocated by uttt_ipc_alloc (zeroed; `handle` receives its 64-byte
 * CUDA IPC handle) and mapped by every other rank with uttt_ipc_open.
 * uttt_split_exchange_finish is one kernel per call: every row's CTA stores
 * this rank's partial z row into each peer's area, raises a flag there,
 * waits for every peer's flag (at most max_polls polls each; an expired wait
 * records UTTT_ERR_TIMEOUT in the workspace status word), sums the partials
 * in rank order and writes out = x + LayerNorm(z) * ln_weight + ln_bias (z
 * rounded to BF16 first when z_bf16 != 0), as uttt_readout_finish does after
 * an all-reduce.  `areas` is a host array of the world ranks' area addresses
 * as mapped in this process (this rank's own at index rank); rows <=
 * max_rows, 2 <= world <= 8.  Every rank must make the same sequence of
 * calls: a per-area epoch, bumped after each call, keys the flags and
 * alternates two receive buffers.  Plain P2P stores only (no multicast).
 * uttt_ipc_close unmaps a peer's area, uttt_ipc_free releases this rank's.
 * No counterpart in the reference (which runs one GPU).
 */
size_t uttt_split_exchange_bytes(int world, int max_rows, int d);
int uttt_ipc_alloc(size_t bytes, void** ptr, void* handle);
int uttt_ipc_open(const void* handle, void** ptr);
int uttt_ipc_close(void* ptr);
int uttt_ipc_free(void* ptr);
int uttt_split_exchange_finish(int rows, int d, const float* z_partial, const void* x, const float* ln_weight,
                               const float* ln_bias, float eps, void* out, int out_dtype, int z_bf16, int rank,
                               int world, int max_rows, void* const* areas, unsigned max_polls, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- slow-weight projections -------------------------------------------- */
/*
 * y = x W^T for BF16 x (M, K) and an nn.Linear weight W (N, K), FP32
 * accumulation on the tensor cores, followed by a per-row finishing pass over
 * column segments of y.  Replaces the F.linear calls of the reference's
 * blocks and their epilogues: the packed QKV projection
 * (model/uttt_layer.py:1068-1074), wo / w_o with the residual add
 * (:1168, :1305, :1544-1554), fused_fast_q_proj (:1175-1190),
 * fused_slow_projections (:1193-1231) and the tied lm_head
 * (model/uttt_model.py:944-950).  Segment ops reproduce the reference's BF16
 * roundings: STORE  y;  RESID  aux + bf16(y);  RMSNORM  rms_norm(bf16(y)) *
 * gamma (aux = FP32 gamma or NULL);  SIGMOID  scale * sigmoid(bf16(y + aux));
 * NORM  rms_norm(aux row) * gamma for a BF16 row `aux` written by an earlier
 * segment of the same call (aux2 = FP32 gamma or NULL; y is not read): a
 * residual projection can emit the next block's normalised input
 * (uTTTBlock.forward, :1544-1554).  Segments of a row run in order.
 * Requires K % 64 == 0.  out may alias a RESID segment's aux (in place).
 * The workspace must be zero on entry (a fresh uttt_linear_workspace buffer
 * is); every call leaves it zero again.
 */
#define UTTT_SEG_STORE 0
#define UTTT_SEG_RESID 1
#define UTTT_SEG_RMSNORM 2
#define UTTT_SEG_SIGMOID 3
#define UTTT_SEG_NORM 4
typedef struct UtttSegment {
  int start, len; /* columns [start, start + len) of y */
  int op;         /* UTTT_SEG_* */
  int out_f32;    /* 1: FP32 output rows, 0: BF16 */
  void* out;      /* row r at out + r * out_ld elements */
  long long out_ld;
  const void* aux; /* RESID: BF16 rows (aux_ld); RMSNORM: FP32 gamma (len); SIGMOID: FP32 bias (len) */
  long long aux_ld;
  float scale;      /* SIGMOID multiplier */
  const void* aux2; /* NORM: FP32 gamma (len) or NULL */
} UtttSegment;
size_t uttt_linear_workspace(int M, int N);
int uttt_linear(int M, int N, int K, const void* x, const void* w, int nseg, const UtttSegment* segs, float eps,
                void* workspace, size_t workspace_bytes, void* stream);

/* ---- attention ---------------------------------------------------------- */
/*
 * Decode step of SlidingWindowAttention (model/uttt_layer.py:1058-1168, the
 * T == 1 SDPA branch :1119-1124; ring layout of CUDAGraphDecoder,
 * engine/inference.py:240-259) for B rows of a packed batch.  Row b is persona
 * slot slot[b] at absolute position pos[b]: q, k get RoPE at pos[b]
 * (apply_rope :946-958), k / v are written into the ring at slot pos[b] % W,
 * and the n_heads / n_kv query heads of each group attend over the
 * min(pos[b]+1, W) valid slots.
 *   qkv    BF16 rows (B, qkv_ld): [q (n_heads*hd) | k (n_kv*hd) | v (n_kv*hd)]
 *   k_ring, v_ring  BF16 (slots, n_kv, W, hd) of one layer
 *   rope_cos/sin    FP32 (positions, hd) tables (RotaryEmbedding, :899-943)
 *   out    BF16 rows (B, out_ld), heads concatenated.
 * hd in {32, 64, 128}, n_heads / n_kv <= 8, W <= 1024.
 */
int uttt_attn_decode(int B, int n_heads, int n_kv, int hd, int W, const void* qkv, int qkv_ld, const int* pos,
                     const int* slot, void* k_ring, void* v_ring, const float* rope_cos, const float* rope_sin,
                     void* out, int out_ld, void* stream);
/*
 * Multi-token causal sliding-window attention (the prefill / chunk branches
 * :1125-1148) for B rows of T new tokens at positions start_pos.. with `hist`
 * history positions already at the start of the KV window buffers:
 *   k_buf, v_buf  BF16 (B, n_kv, hist + T, hd); this call writes positions
 *                 hist.. (RoPE'd k, v) and reads all of them.
 *   q_scratch     BF16 (B, T, n_heads, hd) scratch for the RoPE'd queries.
 *   out           BF16 (B, T, n_heads*hd).
 * Query at absolute position p attends keys in (p - W, p].  Head dims 64 and
 * 128 with n_heads / n_kv <= 8 run on the tensor cores (softmax statistics and
 * the P.V product keep FP32-level precision); head dim 32 on the CUDA cores.
 * Requires hist <= start_pos and hist <= W - 1.
 */
int uttt_attn_prefill(int B, int T, int start_pos, int hist, int n_heads, int n_kv, int hd, int W, const void* qkv,
                      int qkv_ld, const float* rope_cos, const float* rope_sin, void* q_scratch, void* k_buf,
                      void* v_buf, void* out, void* stream);
/* Copy the last min(W, L) positions (ending at absolute position end_pos) of
 * KV window buffers (B, n_kv, L, hd) into persona rings at slot[b]. */
int uttt_kv_ring_fill(int B, int L, int end_pos, int n_kv, int hd, int W, const void* k_buf, const void* v_buf,
                      const int* slot, void* k_ring, void* v_ring, void* stream);

/* ---- row-wise ops -------------------------------------------------------- */
/* RMSNorm (model/uttt_layer.py:881-896): out = x * rsqrt(mean(x^2) + eps) * weight
 * (weight FP32, rounded to BF16 as weight.to(x.dtype) does; NULL for none). */
int uttt_rmsnorm(int rows, int d, const void* x, long long x_ld, const float* weight, float eps, void* out,
                 long long out_ld, void* stream);
/* Token embedding gather (model/uttt_model.py:778-780): out[r] = table[ids[r]]
 * for a (V, d) table; ids outside [0, V) are clamped into it on the device
 * (callers validate ids on the host, as nn.Embedding raises for them). */
int uttt_embed(int rows, int d, int V, const int* ids, const void* table, void* out, void* stream);
/* Greedy pick of _sample_next_token at temperature <= 1e-5
 * (model/uttt_model.py:1204-1221): BF16-rounded logits, PAD/BOS/UNK (ids 0,1,3)
 * and ids >= active_limit masked (stop_free also masks 2,4,5 as the
 * reference's graph-vs-eager test does), lowest id on ties.  top2 (optional)
 * receives the best and second-best values per row. */
int uttt_greedy_argmax(int rows, int V, const void* logits, int logits_f32, long long ld, int active_limit,
                       int stop_free, int* ids, float* top2, void* stream);

/* ---- device-side scheduling of a packed decode batch ------------------------ */
/*
 * The continuous-batching engine keeps every row of its captured decode step in
 * device arrays of B int32 entries: tokens (next input token), pos (its absolute
 * position), slot (KV ring slot), state (fast-weight state index, -1: padding
 * row), produced (reply tokens yielded), max_new (reply length limit), eos (id
 * that ends the reply after being yielded, -1: none), status (UTTT_ROW_*), and
 * ring (B, UTTT_ENGINE_RING): reply token n of row b at ring[b][n % RING].
 *
 * uttt_engine_step runs after a step's greedy pick `ids` (B entries) and applies
 * stream_generate's stop rules (model/uttt_model.py:1036-1050) to every running
 * row: USER / ASSISTANT ids (4, 5) end the reply unyielded; otherwise the id is
 * yielded, and the reply ends at max_new tokens or after eos; stop_free != 0
 * turns the stop ids off (forced-length replies).  A running row advances
 * (tokens = id, pos += 1); a finished one becomes a padding row (slot =
 * pad_slot, state = -1).  It replaces the host loop of stream_generate
 * (:1020-1050) and of server/app.py's serialized worker: no host round trip
 * between steps.
 *
 * uttt_engine_admit starts row `row` for a turn whose prefill's greedy pick is
 * at device address first_id, at position pos0 with KV slot slot0 and state
 * state0, and applies the same rule to that first token.
 */
#define UTTT_ENGINE_RING 8
#define UTTT_ROW_IDLE 0
#define UTTT_ROW_RUNNING 1
#define UTTT_ROW_FINISHED 2
int uttt_engine_step(int B, const int* ids, int* tokens, int* pos, int* slot, int* state, int* produced,
                     const int* max_new, const int* eos, int* status, int* ring, int stop_free, int pad_slot,
                     void* stream);
int uttt_engine_admit(int row, const int* first_id, int pos0, int slot0, int state0, int max_new0, int eos0,
                      int* tokens, int* pos, int* slot, int* state, int* produced, int* max_new, int* eos,
                      int* status, int* ring, int stop_free, int pad_slot, void* stream);

/* BF16 read copies of S FP32 states (SharedFastWeightPool.inference_read_weights,
 * model/uttt_layer.py:648-668): packed_up_gate (S, d, 2h) = [w_up | w_gate],
 * down (S, h, d) = w_down, round-to-nearest-even. */
int uttt_pack_read_copies(int S, int d, int h, const float* w_up, const float* w_gate, const float* w_down,
                          void* packed_up_gate, void* down, void* stream);

/* apply_rope (model/uttt_layer.py:946-958) on `rows` = B*H*T head vectors of
 * length D (row r is token r % T), BF16 in / out, BF16 cos / sin rows (T, D)
 * (the reference casts its FP32 tables to the activation dtype, :935-943). */
int uttt_apply_rope(long long rows, int T, int D, const void* x, const void* cos_t, const void* sin_t, void* out,
                    void* stream);

/* ---- stability guard ------------------------------------------------------ */
/* Slow-anchor elastic pull of B FP32 states towards the shared W_0, in place,
 * with the optional drift clamp (SharedFastWeightPool.apply_elastic_pull,
 * model/uttt_layer.py:773-832): w = W0 + (1-lambda)(W - W0), then if
 * max_drift_ratio > 0 each state's deviation is scaled by
 * min(1, ratio * ||W0|| / sqrt(||w - W0||^2 + 1e-8)) (norms over all three
 * matrices).  lambda <= 0 and ratio <= 0 is a no-op, as in the reference. */
size_t uttt_guard_workspace(int B);
int uttt_elastic_pull(int B, int d, int h, float* w_up, float* w_gate, float* w_down, const float* w_up0,
                      const float* w_gate0, const float* w_down0, float anchor_lambda, float max_drift_ratio,
                      void* workspace, size_t workspace_bytes, void* stream);
/* Drift statistics for compute_drift (:834-874): out (device FP32, 4*B + 4):
 * out[4b+m] = ||W_m[b] - W0_m||^2 for m = up, gate, down; out[4B+m] = ||W0_m||^2. */
int uttt_drift_sums(int B, int d, int h, const float* w_up, const float* w_gate, const float* w_down,
                    const float* w_up0, const float* w_gate0, const float* w_down0, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* UTTT_B200_H */
