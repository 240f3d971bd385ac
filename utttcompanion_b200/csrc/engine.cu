// Device-side scheduling of a packed decode batch.
//
// The continuous-batching engine keeps the state of every row of its captured
// decode step in device memory (next token, position, KV slot, fast-weight
// state, reply length, limits, status and the last few reply tokens).  After
// each step's greedy pick, uttt_engine_step applies stream_generate's stop
// rules (model/uttt_model.py:1036-1050) to every running row and advances it,
// inside the same CUDA graph, so the next step needs nothing from the host:
// the host only admits turns into free rows (uttt_engine_admit, after their
// prefill) and reads the rows back one step behind to stream tokens and
// retire finished turns.  A row that finishes becomes a padding row (padding
// KV slot, no fast-weight state), which reads no weights in later steps.
#include "common.cuh"
#include "host_util.cuh"

namespace uttt {
namespace {

constexpr int kUserId = 4, kAssistantId = 5;

// Accept one picked token for row b (the rule of stream_generate): a role id ends the reply
// without being yielded; otherwise the token is yielded (recorded in the row's ring) and the
// reply ends at the length limit or after EOS.  Returns true while the row keeps running.
__device__ __forceinline__ bool accept(int b, int tok, int stop_free, int* produced, const int* max_new,
                                       const int* eos, int* ring) {
  if (!stop_free && (tok == kUserId || tok == kAssistantId)) return false;
  const int n = produced[b];
  ring[(size_t)b * UTTT_ENGINE_RING + (n % UTTT_ENGINE_RING)] = tok;
  produced[b] = n + 1;
  if (n + 1 >= max_new[b]) return false;
  if (!stop_free && eos[b] >= 0 && tok == eos[b]) return false;
  return true;
}

__device__ __forceinline__ void retire(int b, int* slot, int* state, int* status, int pad_slot) {
  status[b] = UTTT_ROW_FINISHED;
  slot[b] = pad_slot;
  state[b] = -1;
}

__global__ void engine_step_kernel(int B, const int* __restrict__ ids, int* tokens, int* pos, int* slot, int* state,
                                   int* produced, const int* max_new, const int* eos, int* status, int* ring,
                                   int stop_free, int pad_slot) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || status[b] != UTTT_ROW_RUNNING) return;
  const int tok = ids[b];
  if (accept(b, tok, stop_free, produced, max_new, eos, ring)) {
    tokens[b] = tok;
    pos[b] += 1;
  } else {
    retire(b, slot, state, status, pad_slot);
  }
}

__global__ void engine_admit_kernel(int row, const int* __restrict__ first_id, int pos0, int slot0, int state0,
                                    int max_new0, int eos0, int* tokens, int* pos, int* slot, int* state,
                                    int* produced, int* max_new, int* eos, int* status, int* ring, int stop_free,
                                    int pad_slot) {
  if (threadIdx.x != 0) return;
  const int tok = *first_id;
  produced[row] = 0;
  max_new[row] = max_new0;
  eos[row] = eos0;
  status[row] = UTTT_ROW_RUNNING;
  if (accept(row, tok, stop_free, produced, max_new, eos, ring)) {
    tokens[row] = tok;
    pos[row] = pos0;
    slot[row] = slot0;
    state[row] = state0;
  } else {
    tokens[row] = 0;
    pos[row] = 0;
    retire(row, slot, state, status, pad_slot);
  }
}

}  // namespace
}  // namespace uttt

using namespace uttt;

extern "C" int uttt_engine_step(int B, const int* ids, int* tokens, int* pos, int* slot, int* state, int* produced,
                                const int* max_new, const int* eos, int* status, int* ring, int stop_free,
                                int pad_slot, void* stream) {
  UTTT_REQUIRE(B > 0, UTTT_ERR_INVALID);
  UTTT_REQUIRE(ids && tokens && pos && slot && state && produced && max_new && eos && status && ring,
               UTTT_ERR_INVALID);
  engine_step_kernel<<<(B + 127) / 128, 128, 0, (cudaStream_t)stream>>>(
      B, ids, tokens, pos, slot, state, produced, max_new, eos, status, ring, stop_free, pad_slot);
  return launch_status();
}

extern "C" int uttt_engine_admit(int row, const int* first_id, int pos0, int slot0, int state0, int max_new0,
                                 int eos0, int* tokens, int* pos, int* slot, int* state, int* produced, int* max_new,
                                 int* eos, int* status, int* ring, int stop_free, int pad_slot, void* stream) {
  UTTT_REQUIRE(row >= 0 && max_new0 >= 1 && pos0 >= 0 && state0 >= 0, UTTT_ERR_INVALID);
  UTTT_REQUIRE(first_id && tokens && pos && slot && state && produced && max_new && eos && status && ring,
               UTTT_ERR_INVALID);
  engine_admit_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(row, first_id, pos0, slot0, state0, max_new0, eos0,
                                                          tokens, pos, slot, state, produced, max_new, eos, status,
                                                          ring, stop_free, pad_slot);
  return launch_status();
}
