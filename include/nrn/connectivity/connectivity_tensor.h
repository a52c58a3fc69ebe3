// nrn/connectivity/connectivity_tensor.h -- block-CSR connectivity
// (reference: include/nrn/connectivity/connectivity_tensor.h:25-91).
//
// This is the API's storage format: dense B x B blocks of weights, masks and
// delays, indexed by a CSR over target block rows.  The simulation engine
// compiles it once into a per-synapse, source-major CSR on the GPU (only
// structurally present synapses) and writes plastic weights back after a run.
#pragma once

#include <cstdint>
#include <optional>
#include <string>
#include <unordered_map>

#include <torch/torch.h>

namespace nrn {

struct BlockIndex {
    torch::Tensor row_ptr;   // [n_target_blocks + 1], int32
    torch::Tensor col_idx;   // [n_blocks], int32

    int64_t n_blocks() const { return col_idx.size(0); }
    int64_t n_rows() const { return row_ptr.size(0) > 0 ? row_ptr.size(0) - 1 : 0; }

    // Index of block (target block row, source block column), or -1.
    int64_t find_block(int64_t target_row, int64_t source_col) const;
};

struct ConnectivityTensor {
    BlockIndex block_index;
    int64_t block_size = 0;
    int64_t n_source = 0;
    int64_t n_target = 0;

    torch::Tensor weights;           // [n_blocks, B, B] float
    torch::Tensor structural_mask;   // [n_blocks, B, B] 0/1
    torch::Tensor modulatory_mask;   // [n_blocks, B, B] gain
    torch::Tensor delays;            // [n_blocks, B, B] int32, steps

    std::unordered_map<std::string, torch::Tensor> synapse_state;

    std::optional<torch::Tensor> trace_pre;
    std::optional<torch::Tensor> trace_post;

    // weights * structural_mask * modulatory_mask
    torch::Tensor effective_weights() const;
    void to(torch::Device device);
    int64_t total_capacity() const;
    int64_t active_count() const;
    double density() const;
};

}  // namespace nrn
