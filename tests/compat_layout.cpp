// A reference-style caller of the drop-in C++ API (include/memory_cuda.cuh):
// it names QueryContext members the reference declares, uploads a graph whose
// dimension is not a multiple of 4, and checks that DeviceMemoryGraph::
// d_embeddings holds the rows densely (N x D, as the reference lays them out)
// and that a query runs.  Built and run by tests/test_gpu_compat_layout.py.
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <vector>

#include "memory_cuda.cuh"
#include "memory_graph.h"

int main() {
    const int N = 500, D = 66;
    MemoryGraph g;
    g.num_nodes = N;
    g.embedding_dim = D;
    g.embeddings.resize((size_t)N * D);
    g.modalities.resize(N);
    g.timestamps.resize(N);
    unsigned x = 12345u;
    for (int i = 0; i < N; ++i) {
        float ss = 0.f;
        for (int d = 0; d < D; ++d) {
            x = x * 1664525u + 1013904223u;
            const float v = (float)((x >> 8) & 0xffff) / 65536.0f - 0.5f;
            g.embeddings[(size_t)i * D + d] = v;
            ss += v * v;
        }
        for (int d = 0; d < D; ++d) g.embeddings[(size_t)i * D + d] /= std::sqrt(ss);
        g.modalities[i] = i % 3;
        g.timestamps[i] = (float)i;
    }
    DeviceMemoryGraph dg = upload_to_device(g);
    std::vector<float> back((size_t)N * D);
    if (cudaMemcpy(back.data(), dg.d_embeddings, back.size() * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess) {
        std::printf("copy failed\n");
        return 2;
    }
    for (size_t i = 0; i < back.size(); ++i)
        if (back[i] != g.embeddings[i]) { std::printf("row layout differs at %zu\n", i); return 3; }

    QueryContext ctx = create_query_context(N, D, 10);
    // members of the reference's QueryContext that callers may name
    if (ctx.d_sim != nullptr || ctx.d_final != nullptr || ctx.graph_captured || ctx.cublas_handle != nullptr) {
        std::printf("reference scratch members should be left empty\n");
        return 4;
    }
    RetrievalConfig cfg;
    cfg.top_k = 5;
    cfg.bfs_max_hops = 0;
    RetrievalStats st;
    auto res = query_memory_fast(dg, ctx, &g.embeddings[(size_t)7 * D], 500.0f, cfg, st);
    if (res.empty() || res[0].node_id != 7) { std::printf("self query did not rank its row first\n"); return 5; }
    destroy_query_context(ctx);
    free_device(dg);
    std::printf("ok\n");
    return 0;
}
