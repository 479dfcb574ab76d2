// D2 batch planes from a token stream (host): the i64 input / target planes
// and the bool loss-mask plane of a fixed [N, T] batch that the fused
// training step takes (et_b200_lm_step_v1 plus et_b200_lm_set_loss_mask_v1).
//
// The row rule of the reference's D2 shard loader (docs/D2_SHARD_LOADER.md,
// "Rows, shift, mask, and ordering"), packed mode over one flat stream of L
// tokens: the stream holds 0 rows when L < 2, else 1 + floor((L - 2) / T);
// row r starts at s = r T and position t of it is a true position when
// s + t + 1 < L, with input token[s + t] and target token[s + t + 1]; every
// other position of the batch (the tail of the last row, and rows past the
// stream's end) holds token 0, target 0 and a false mask bit.  Window
// shuffling and shard handling stay with the host's loader.
#include <stdint.h>
#include <string.h>

#include "common.cuh"

using etb::set_error;

extern "C" {

int64_t et_b200_d2_row_count_v1(uint64_t tokens, int64_t seq_len) {
  if (seq_len < 1 || tokens < 2) return 0;
  return 1 + (int64_t)((tokens - 2) / (uint64_t)seq_len);
}

int32_t et_b200_d2_rows_v1(const int64_t* tokens, uint64_t length, int64_t seq_len,
                           int64_t first_row, int64_t rows, int64_t* ids, int64_t* targets,
                           uint8_t* mask, et_kernel_error* e) {
  const char* op = "d2-rows";
  if (ids == nullptr || targets == nullptr || mask == nullptr || (tokens == nullptr && length))
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_NULL_ARGUMENT, op,
                     "token stream and the three planes are required");
  if (seq_len < 1 || rows < 1 || first_row < 0)
    return set_error(e, ET_KERNEL_ERROR_SHAPE_MISMATCH, ET_KERNEL_CODE_INVALID_SHAPE, op,
                     "seq_len and rows must be positive, first_row non-negative");
  const int64_t available = et_b200_d2_row_count_v1(length, seq_len);
  if (first_row >= available)
    return set_error(e, ET_KERNEL_ERROR_INVALID_ARGUMENT, ET_KERNEL_CODE_PROVIDER_REJECTED, op,
                     "no row of the stream starts at first_row (a batch needs at least one true "
                     "mask bit)");
  const size_t plane = (size_t)rows * (size_t)seq_len;
  memset(ids, 0, plane * sizeof(int64_t));
  memset(targets, 0, plane * sizeof(int64_t));
  memset(mask, 0, plane);
  for (int64_t r = 0; r < rows && first_row + r < available; r++) {
    const uint64_t s = (uint64_t)(first_row + r) * (uint64_t)seq_len;
    for (int64_t t = 0; t < seq_len && s + (uint64_t)t + 1 < length; t++) {
      const size_t o = (size_t)r * (size_t)seq_len + (size_t)t;
      ids[o] = tokens[s + t];
      targets[o] = tokens[s + t + 1];
      mask[o] = 1;
    }
  }
  if (e) memset(e, 0, sizeof(*e));
  return 0;
}

}  // extern "C"
