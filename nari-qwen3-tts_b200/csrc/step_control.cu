// Device-side request control of a talker decode step: the per-request sampling parameters and
// generation state live in a slot table on the GPU, so a captured step needs no host staging before it
// and no per-row host read after it.
//
//   nqt_step_stage          gathers each row's sampling parameters from its request slot into the
//                           sampler's row buffers and computes the row's EOS-suppression flag
//                           (replaces the pinned host staging of executor/talker.py:527-563 and the
//                           suppress_eos rows of engine/input_builder.py:60-70);
//   nqt_talker_logits_mask  the codec head's suppress mask (executor/talker.py:170-183, 241-243):
//                           logits past the code-predictor vocabulary are -inf except the EOS token,
//                           which is -inf on rows whose EOS is suppressed;
//   nqt_step_finish         the decode completion rule of engine/pipeline.py:583-609 on the device:
//                           reached_limit = step + 1 >= max_tokens; eos = token == eos_id on rows whose
//                           EOS is not suppressed and that have not reached the limit; terminal = eos or
//                           reached_limit; then every live row's step advances by one and its RNG offset
//                           by the frame stride (executor/talker.py:606).
//
// A slot's `eos_from` is the first generation step at which EOS may end the request: INT32_MAX while
// EOS is suppressed indefinitely (ignore_eos, or a continuation whose input has not finished), else
// max(2, token_count - 1) for a terminal continuation and 2 otherwise (input_builder.py:60-70).
// Rows with slot < 0 are padding: they get the reference's padding defaults (temperature 0, top_k 1,
// top_p 1, penalty 1, seed 0, offset 0, EOS suppressed) and are never terminal.
#include "common.cuh"

namespace nqt {
namespace {

constexpr int kThreads = 256;

__global__ void stage_kernel(const int32_t* row_slot, int rows, int slots, const float* s_temp, const int32_t* s_top_k,
                             const float* s_top_p, const float* s_pen, const int64_t* s_seed, const int64_t* s_offset,
                             const int32_t* s_step, const int32_t* s_eos_from, float* temp, int32_t* top_k,
                             float* top_p, float* pen, int64_t* seed, int64_t* offset, uint8_t* suppress,
                             int32_t* status) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int s = row_slot[r];
  if (s < 0 || s >= slots) {
    if (s >= slots) report(status, NQT_DEV_BAD_SLOT);
    temp[r] = 0.f;
    top_k[r] = 1;
    top_p[r] = 1.f;
    if (pen != nullptr) pen[r] = 1.f;
    seed[r] = 0;
    offset[r] = 0;
    if (suppress != nullptr) suppress[r] = 1;
    return;
  }
  temp[r] = s_temp[s];
  top_k[r] = s_top_k[s];
  top_p[r] = s_top_p[s];
  if (pen != nullptr) pen[r] = s_pen[s];
  seed[r] = s_seed[s];
  offset[r] = s_offset[s];
  if (suppress != nullptr) suppress[r] = s_step[s] < s_eos_from[s] ? 1 : 0;
}

template <typename T>
__global__ void logits_mask_kernel(T* logits, int64_t stride, int vocab, int codec_vocab, int eos_id,
                                   const uint8_t* suppress) {
  const int r = blockIdx.y;
  T* row = logits + r * stride;
  const T neg_inf = from_f32<T>(-__builtin_huge_valf());
  for (int e = codec_vocab + blockIdx.x * blockDim.x + threadIdx.x; e < vocab; e += gridDim.x * blockDim.x) {
    if (e != eos_id || (suppress != nullptr && suppress[r] != 0)) row[e] = neg_inf;
  }
  // an EOS id inside the codec range is masked only by the row's suppression flag
  if (blockIdx.x == 0 && threadIdx.x == 0 && eos_id >= 0 && eos_id < codec_vocab && suppress != nullptr &&
      suppress[r] != 0)
    row[eos_id] = neg_inf;
}

__global__ void finish_kernel(const int32_t* row_slot, int rows, int slots, const int64_t* tokens, int eos_id,
                              int32_t* s_step, const int32_t* s_max_tokens, const int32_t* s_eos_from,
                              int64_t* s_offset, int64_t offset_stride, uint8_t* terminal, int32_t* n_terminal,
                              int32_t* status) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int s = row_slot[r];
  if (s < 0 || s >= slots) {
    if (s >= slots) report(status, NQT_DEV_BAD_SLOT);
    terminal[r] = 0;
    return;
  }
  const int step = s_step[s];
  const bool reached_limit = static_cast<int64_t>(step) + 1 >= s_max_tokens[s];
  const bool suppress = step < s_eos_from[s];
  const bool eos = !suppress && !reached_limit && tokens[r] == eos_id;
  const bool done = eos || reached_limit;
  terminal[r] = done ? 1 : 0;
  if (done && n_terminal != nullptr) atomicAdd(n_terminal, 1);
  s_step[s] = step + 1;
  s_offset[s] += offset_stride;
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" int nqt_step_stage(const int32_t* row_slot, int rows, int slots, const float* slot_temperature,
                              const int32_t* slot_top_k, const float* slot_top_p, const float* slot_penalty,
                              const int64_t* slot_seed, const int64_t* slot_offset, const int32_t* slot_step,
                              const int32_t* slot_eos_from, float* temperature, int32_t* top_k, float* top_p,
                              float* penalty, int64_t* seed, int64_t* offset, uint8_t* suppress_eos, int32_t* status,
                              void* stream) {
  if (!row_slot || !slot_temperature || !slot_top_k || !slot_top_p || !slot_seed || !slot_offset || !temperature ||
      !top_k || !top_p || !seed || !offset || rows < 0 || slots < 1)
    return NQT_ERR_ARG;
  if ((penalty != nullptr) != (slot_penalty != nullptr)) return NQT_ERR_ARG;
  if (suppress_eos != nullptr && (!slot_step || !slot_eos_from)) return NQT_ERR_ARG;
  if (rows == 0) return NQT_OK;
  stage_kernel<<<(rows + kThreads - 1) / kThreads, kThreads, 0, as_stream(stream)>>>(
      row_slot, rows, slots, slot_temperature, slot_top_k, slot_top_p, slot_penalty, slot_seed, slot_offset, slot_step,
      slot_eos_from, temperature, top_k, top_p, penalty, seed, offset, suppress_eos, status);
  return check_launch("step_stage");
}

extern "C" int nqt_talker_logits_mask(void* logits, int dtype, int64_t logits_stride, int rows, int vocab,
                                      int codec_vocab, int eos_id, const uint8_t* suppress_eos, void* stream) {
  if (!logits || rows < 0 || vocab < 1 || codec_vocab < 0 || codec_vocab > vocab || logits_stride < vocab)
    return NQT_ERR_ARG;
  if (eos_id >= vocab) return NQT_ERR_ARG;
  if (rows == 0) return NQT_OK;
  if (rows > 65535) return NQT_ERR_UNSUPPORTED;
  const int tail = vocab - codec_vocab;
  dim3 grid(tail > 0 ? (tail + kThreads - 1) / kThreads : 1, rows);
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case NQT_BF16:
      logits_mask_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(static_cast<__nv_bfloat16*>(logits), logits_stride,
                                                                  vocab, codec_vocab, eos_id, suppress_eos);
      break;
    case NQT_F16:
      logits_mask_kernel<__half><<<grid, kThreads, 0, s>>>(static_cast<__half*>(logits), logits_stride, vocab,
                                                           codec_vocab, eos_id, suppress_eos);
      break;
    case NQT_F32:
      logits_mask_kernel<float><<<grid, kThreads, 0, s>>>(static_cast<float*>(logits), logits_stride, vocab,
                                                          codec_vocab, eos_id, suppress_eos);
      break;
    default:
      return NQT_ERR_ARG;
  }
  return check_launch("talker_logits_mask");
}

extern "C" int nqt_step_finish(const int32_t* row_slot, int rows, int slots, const int64_t* tokens, int eos_id,
                               int32_t* slot_step, const int32_t* slot_max_tokens, const int32_t* slot_eos_from,
                               int64_t* slot_offset, int64_t offset_stride, uint8_t* terminal, int32_t* n_terminal,
                               int32_t* status, void* stream) {
  if (!row_slot || !tokens || !slot_step || !slot_max_tokens || !slot_eos_from || !slot_offset || !terminal ||
      rows < 0 || slots < 1)
    return NQT_ERR_ARG;
  if (rows == 0) return NQT_OK;
  finish_kernel<<<(rows + kThreads - 1) / kThreads, kThreads, 0, as_stream(stream)>>>(
      row_slot, rows, slots, tokens, eos_id, slot_step, slot_max_tokens, slot_eos_from, slot_offset, offset_stride,
      terminal, n_terminal, status);
  return check_launch("step_finish");
}
