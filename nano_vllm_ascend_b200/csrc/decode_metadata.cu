// Decode-step metadata built on the device: padded block tables, context
// lengths and the slot mapping of the tokens being appended.
//
// Replaces the host loops of BlockManager.prepare_decode_metadata
// (src/nanovllm_ascend/npu/block_manager.py:304-328) -> get_block_tables_tensor
// (:207-224), get_context_lens_tensor (:226-231) and get_slot_mapping
// (:233-250): slot = table[pos / block_size] * block_size + pos % block_size.
//
// The per-sequence tables live in a persistent device mirror [rows, stride]
// (row = the BlockManager's sequence slot). Each step the host passes only the
// entries added since the last step (block ids appended by ensure_blocks, or a
// whole table for a new sequence) as per-sequence update lists; the warp of a
// sequence applies its updates to the mirror, then writes that sequence's
// outputs. The host may also pass each row's context length and table size
// (the host path's seq_lens[slot] and whole table, which differ from
// start + q_len when a slot is named twice or decoded behind its length).
// Integer work, one warp per sequence.
#include "host_common.h"
#include "nvk_common.cuh"

namespace nvk {
namespace {

constexpr int kRowsPerBlock = 8;  // one warp per sequence

__global__ void __launch_bounds__(kRowsPerBlock * 32) decode_metadata_kernel(
    int32_t* __restrict__ mirror, int mirror_stride, int mirror_rows, const int32_t* __restrict__ seq_slots,
    const int64_t* __restrict__ start_positions, const int32_t* __restrict__ row_context_lens,
    const int32_t* __restrict__ row_blocks, int batch, int q_len, int block_size,
    const int32_t* __restrict__ update_offsets, const int32_t* __restrict__ update_idx,
    const int32_t* __restrict__ update_block, int32_t* __restrict__ tables_out, int out_stride, int out_width,
    int32_t* __restrict__ context_lens_out, int64_t* __restrict__ slot_mapping_out, int* __restrict__ error_word) {
  // No early trigger: the decode kernel reads the tables and lengths written
  // here before its griddepcontrol.wait, so a dependent grid may only start
  // once this one has finished (the implicit trigger at grid completion).
  pdl_wait();
  const int b = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= batch) return;
  const int row = seq_slots[b];
  const int64_t start = start_positions[b];
  const int64_t end = start + q_len;
  // the host path's length and table size for this slot (they exceed end when the slot is named
  // twice in the batch or decoded behind its length), else what this step's tokens need
  const int64_t ctx = row_context_lens ? row_context_lens[b] : end;
  const int64_t nblk = row_blocks ? row_blocks[b] : (end + block_size - 1) / block_size;
  if (row < 0 || row >= mirror_rows || start < 0 || ctx < end || nblk * block_size < end || nblk > mirror_stride ||
      nblk > out_width) {
    if (lane == 0 && error_word) atomicOr(error_word, kErrContextTooLong);
    for (int j = lane; j < out_width; j += 32) tables_out[static_cast<int64_t>(b) * out_stride + j] = 0;
    if (lane == 0) context_lens_out[b] = 0;
    for (int t = lane; t < q_len; t += 32) slot_mapping_out[static_cast<int64_t>(b) * q_len + t] = -1;
    return;
  }
  int32_t* mrow = mirror + static_cast<int64_t>(row) * mirror_stride;
  // 1. this sequence's new table entries
  for (int u = update_offsets[b] + lane; u < update_offsets[b + 1]; u += 32) {
    const int idx = update_idx[u];
    if (idx >= 0 && idx < mirror_stride) mrow[idx] = update_block[u];
  }
  __syncwarp();  // the reads below see every lane's updates
  // 2. padded table row: entries below ceil(context / block_size), zeros after
  int32_t* trow = tables_out + static_cast<int64_t>(b) * out_stride;
  for (int j = lane; j < out_width; j += 32) trow[j] = j < nblk ? mrow[j] : 0;
  // 3. context length (includes the appended tokens) and their slots
  if (lane == 0) context_lens_out[b] = static_cast<int32_t>(ctx);
  for (int t = lane; t < q_len; t += 32) {
    const int64_t pos = start + t;
    slot_mapping_out[static_cast<int64_t>(b) * q_len + t] =
        static_cast<int64_t>(mrow[pos / block_size]) * block_size + pos % block_size;
  }
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_decode_metadata(int32_t* table_mirror, int mirror_stride, int mirror_rows,
                                   const int32_t* seq_slots, const int64_t* start_positions,
                                   const int32_t* row_context_lens, const int32_t* row_blocks, int batch, int q_len,
                                   int block_size, const int32_t* update_offsets, const int32_t* update_idx,
                                   const int32_t* update_block, int32_t* block_tables, int block_table_stride,
                                   int block_table_width, int32_t* context_lens, int64_t* slot_mapping,
                                   int* error_word, nvk_stream_t stream) {
  using namespace nvk;
  if (batch < 0 || q_len <= 0 || block_size <= 0 || mirror_stride <= 0 || mirror_rows <= 0 ||
      block_table_width <= 0 || block_table_stride < block_table_width)
    return fail(NVK_ERR_INVALID_ARGUMENT,
                "decode_metadata: bad sizes (batch=%d q_len=%d block_size=%d mirror %dx%d width=%d stride=%d)", batch,
                q_len, block_size, mirror_rows, mirror_stride, block_table_width, block_table_stride);
  if (batch == 0) return NVK_OK;
  if (!table_mirror || !seq_slots || !start_positions || !update_offsets || !block_tables || !context_lens ||
      !slot_mapping)
    return fail(NVK_ERR_INVALID_ARGUMENT, "decode_metadata: null pointer");
  const int grid = (batch + kRowsPerBlock - 1) / kRowsPerBlock;
  const cudaError_t e =
      launch_pdl(decode_metadata_kernel, dim3(grid), dim3(kRowsPerBlock * 32), 0, reinterpret_cast<cudaStream_t>(stream),
                 table_mirror, mirror_stride, mirror_rows, seq_slots, start_positions, row_context_lens, row_blocks,
                 batch, q_len, block_size,
                 update_offsets, update_idx, update_block, block_tables, block_table_stride, block_table_width,
                 context_lens, slot_mapping, error_word);
  return check_cuda(e, "decode_metadata launch");
}
