// memory_graph.h -- host-side multimodal memory graph, the input of
// upload_to_device().  Same declarations as the reference header
// (include/memory_graph.h of antonellof/cuda-multimodal-memory) so that its
// callers compile unchanged against this library: a node is a memory with an
// embedding row, a modality tag and a timestamp; edges are CSR.
//
// The member functions synthetic(), build_nsn_edges*(), print_summary() and
// device_bytes() are corpus-synthesis utilities that live outside the
// retrieval path; callers link their own implementation of them (the
// reference's src/memory_graph.cpp), this library does not provide them.
#ifndef MEMORY_GRAPH_H
#define MEMORY_GRAPH_H

#include <cstdint>
#include <string>
#include <vector>

enum Modality : int32_t {
    MOD_TEXT  = 0,
    MOD_AUDIO = 1,
    MOD_IMAGE = 2,
    MOD_COUNT = 3
};

struct MemoryGraph {
    int32_t num_nodes     = 0;
    int32_t num_edges     = 0;     // directed entries in col_indices
    int32_t embedding_dim = 0;

    std::vector<int32_t> row_offsets;   // num_nodes + 1
    std::vector<int32_t> col_indices;   // num_edges

    std::vector<float>   embeddings;    // num_nodes x embedding_dim, row-major
    std::vector<int32_t> modalities;    // num_nodes
    std::vector<float>   timestamps;    // num_nodes, seconds

    static MemoryGraph synthetic(int32_t n_text, int32_t n_audio, int32_t n_image,
                                 int32_t dim, uint32_t seed = 42);

    void build_nsn_edges(int32_t k = 6, double p = 0.15);

    struct NSNConfig {
        int32_t k              = 6;
        double  p              = 0.15;
        bool    enable_ring    = true;
        bool    enable_skips   = true;
        bool    enable_hubs    = true;
        bool    enable_rewire  = true;
        bool    enable_bridges = true;
    };

    void build_nsn_edges_configurable(const NSNConfig& cfg);

    void   print_summary() const;
    size_t device_bytes() const;
};

#endif  // MEMORY_GRAPH_H
