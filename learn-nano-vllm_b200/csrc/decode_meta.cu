// Decode-step metadata on the device.  Replaces the per-sequence host loops of
// nanovllm/engine/model_runner.py:167-193 (prepare_decode, prepare_block_tables,
// prepare_sample) after one host-to-device copy of a packed int32 buffer:
//   [B] lengths, [B] last tokens, [B] temperatures (fp32 bits), [B + 1] offsets
//   of each sequence's block list in `flat`, then `flat` (every block id of the
//   batch, sequence after sequence).
// Outputs, as the reference builds them:
//   input_ids[b]   = last token                       (int64)
//   positions[b]   = len - 1                          (int64)
//   context_lens[b]= len                              (int32)
//   slot_mapping[b]= block_table[-1] * block_size + last_block_num_tokens - 1
//                    with last_block_num_tokens = len - (num_blocks - 1) * block_size
//   block_tables[b, j] = block_table[j] for j < num_blocks, else -1 ([B, W])
//   temperatures[b] (fp32)
#include "common.cuh"

namespace b200 {
namespace dm {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) decode_meta_kernel(const int32_t* __restrict__ packed, int32_t B, int32_t W,
                                                               int32_t block_size, int64_t* input_ids,
                                                               int64_t* positions, int32_t* slot_mapping,
                                                               int32_t* context_lens, int32_t* block_tables,
                                                               float* temperatures) {
    const int32_t* lens = packed;
    const int32_t* toks = packed + B;
    const int32_t* temps = packed + 2 * B;
    const int32_t* offs = packed + 3 * B;
    const int32_t* flat = packed + 4 * B + 1;
    const int64_t total = int64_t(B) * W;
    for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < total; i += int64_t(gridDim.x) * kThreads) {
        const int b = int(i / W), j = int(i - int64_t(b) * W);
        const int o = offs[b], n = offs[b + 1] - o;
        block_tables[i] = j < n ? flat[o + j] : -1;
        if (j == 0) {
            const int len = lens[b];
            input_ids[b] = toks[b];
            positions[b] = len - 1;
            context_lens[b] = len;
            slot_mapping[b] = n > 0 ? flat[o + n - 1] * block_size + (len - (n - 1) * block_size) - 1 : -1;
            temperatures[b] = __int_as_float(temps[b]);
        }
    }
}

}  // namespace dm
}  // namespace b200

extern "C" int32_t b200_decode_metadata(const int32_t* packed, int32_t batch, int32_t max_blocks,
                                        int32_t block_size, int64_t* input_ids, int64_t* positions,
                                        int32_t* slot_mapping, int32_t* context_lens, int32_t* block_tables,
                                        float* temperatures, void* stream) {
    using namespace b200;
    clear_error();
    B200_REQUIRE(batch >= 0 && max_blocks >= 1 && block_size > 0, "decode_metadata: batch %d, width %d, block %d",
                 batch, max_blocks, block_size);
    if (batch == 0) return B200_OK;
    B200_REQUIRE(packed && input_ids && positions && slot_mapping && context_lens && block_tables && temperatures,
                 "decode_metadata: null pointer");
    const int64_t total = int64_t(batch) * max_blocks;
    int64_t blocks = (total + dm::kThreads - 1) / dm::kThreads;
    const int64_t cap = int64_t(device_sm_count()) * 8;
    if (blocks > cap) blocks = cap;
    dm::decode_meta_kernel<<<unsigned(blocks), dm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        packed, batch, max_blocks, block_size, input_ids, positions, slot_mapping, context_lens, block_tables,
        temperatures);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
}
