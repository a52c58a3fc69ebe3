// Writes the connectivity that connect() builds with the Erdos-Renyi
// generator after torch::manual_seed(seed), for comparison with the
// reference's (tests/golden/er_connect.npz).  Host only.
//   er_dump <out.bin> <n> <block> <p> <weight_scale> <seed>
// Output: int64 n_rows+1, n_blocks, then row_ptr (int32), col_idx (int32),
// weights and structural mask (float [n_blocks][B][B]).
#include <cstdio>
#include <cstdlib>
#include <memory>

#include <nrn/nrn.h>

using namespace nrn;

int main(int argc, char** argv) {
    if (argc < 7) return 2;
    const int64_t n = std::atoll(argv[2]), B = std::atoll(argv[3]);
    const double p = std::atof(argv[4]), scale = std::atof(argv[5]);
    torch::manual_seed(std::atoll(argv[6]));
    auto* topo = random_topology_create(RandomTopologyOptions().probability(p).allow_autapses(false));
    auto gen = random_topology_as_generator(topo);
    auto* syn = synapse::static_synapse_create(1);
    NrnModule dummy{nullptr, nullptr};
    auto pop = std::shared_ptr<Population>(population_create("s", dummy, n, torch::kCPU), population_destroy);
    auto c = connect(pop, pop, &gen, synapse::static_synapse_as_module(syn), ConnectOptions().block_size(B).weight_scale(scale));
    auto& ct = c->connectivity;
    FILE* f = std::fopen(argv[1], "wb");
    int64_t hdr[2] = {ct.block_index.row_ptr.size(0), ct.block_index.n_blocks()};
    std::fwrite(hdr, 8, 2, f);
    std::fwrite(ct.block_index.row_ptr.data_ptr<int32_t>(), 4, hdr[0], f);
    std::fwrite(ct.block_index.col_idx.data_ptr<int32_t>(), 4, hdr[1], f);
    auto w = ct.weights.contiguous(), m = ct.structural_mask.contiguous();
    std::fwrite(w.data_ptr<float>(), 4, w.numel(), f);
    std::fwrite(m.data_ptr<float>(), 4, m.numel(), f);
    std::fclose(f);
    random_topology_destroy(topo);
    synapse::static_synapse_destroy(syn);
    return 0;
}
