// The three-layer forward on `world` GPUs of one node through the C++ mirror
// (gat_b200::Communicator / gat_b200::PartitionedModel), one process per rank:
//
//   part_test GRAPH WEIGHTS RANK WORLD ID_PATH EXCHANGE CHUNKS [LAYER2_INPUTS]
//
// LAYER2_INPUTS (P2P exchange only, default 1): 1 sends layer 2's input rows
// from the layer-1 aggregation, 0 sends its projected rows.
//
// Each rank checks its rows of the partitioned logits against the one-GPU
// model (gat_b200_model_*) of the whole graph run on its own GPU: relative L2
// <= 1e-5 (the same kernels, the same sources in the same order; only the
// row schedule differs), and three pipelined host-to-host requests
// (gat_b200_part_model_forward_async) equal the synchronous forward bit for
// bit. Prints one PART_TEST line; exit status 0 when both hold.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "gat_b200.hpp"

namespace gat = gat_b200;

int main(int argc, char** argv) {
    if (argc != 8 && argc != 9) {
        std::fprintf(stderr, "usage: %s GRAPH WEIGHTS RANK WORLD ID_PATH EXCHANGE CHUNKS [LAYER2_INPUTS]\n", argv[0]);
        return 2;
    }
    try {
        const int rank = std::atoi(argv[3]), world = std::atoi(argv[4]);
        const int exchange = std::atoi(argv[6]), chunks = std::atoi(argv[7]);
        const bool layer2_inputs = argc == 9 ? std::atoi(argv[8]) != 0 : true;
        const gat::Graph g = gat::load_graph(argv[1]);
        const gat::Model model = gat::load_model(argv[2], g.din, g.classes);
        gat::Communicator comm(argv[5], world, rank, rank);
        std::vector<float> got;
        uint64_t lo = 0, hi = 0;
        bool async_equal = true;
        {
            gat::PartitionedModel pm(comm, g, model, exchange, chunks);
            if (exchange == GAT_B200_EXCHANGE_P2P) pm.set_layer2_exchange(layer2_inputs);
            lo = pm.first_row();
            hi = pm.end_row();
            for (int i = 0; i < 3; ++i) got = pm.forward();
            std::vector<std::vector<float>> outs(3, std::vector<float>(got.size()));
            for (auto& o : outs) gat::check(gat_b200_part_model_forward_async(pm.handle(), pm.input().data(), o.data(), nullptr));
            gat::check(gat_b200_part_model_join(pm.handle(), nullptr));
            gat::check(gat_b200_check_device());
            for (const auto& o : outs) async_equal = async_equal && o == got;
        }
        // the one-GPU model of the whole graph on this rank's GPU
        gat_b200_graph* gg = nullptr;
        gat_b200_layer* ls[3] = {};
        gat_b200_model* m = nullptr;
        gat::check(gat_b200_graph_create(g.n, g.e, g.row.data(), g.col.data(), nullptr, &gg));
        for (int l = 0; l < 3; ++l)
            gat::check(gat_b200_layer_create(model[l].in, model[l].heads, model[l].dim, model[l].w.data(),
                                             model[l].al.data(), model[l].ar.data(), &ls[l]));
        gat::check(gat_b200_model_create(gg, ls, GAT_B200_PATH_STANDARD_BF16, &m));
        const int C = g.classes;
        std::vector<float> full(size_t(g.n) * C);
        gat::check(gat_b200_model_forward(m, g.x.data(), 1, full.data(), 1, nullptr));
        double d2 = 0, r2 = 0, mx = 0;
        for (uint64_t i = lo; i < hi; ++i)
            for (int c = 0; c < C; ++c) {
                const double a = full[i * C + c], b = got[(i - lo) * C + c], d = b - a;
                d2 += d * d;
                r2 += a * a;
                mx = std::fmax(mx, std::fabs(d));
            }
        gat_b200_model_destroy(m);
        for (auto* l : ls) gat_b200_layer_destroy(l);
        gat_b200_graph_destroy(gg);
        const double rel = r2 > 0 ? std::sqrt(d2 / r2) : std::sqrt(d2);
        const bool ok = std::isfinite(rel) && rel <= 1e-5 && async_equal;
        std::printf("PART_TEST rank=%d world=%d exchange=%d chunks=%d layer2_inputs=%d rows=%llu..%llu rel_l2=%.3e "
                    "max_abs=%.3e async_equal=%d %s\n",
                    rank, world, exchange, chunks, int(layer2_inputs), (unsigned long long)lo, (unsigned long long)hi, rel, mx,
                    int(async_equal), ok ? "PASS" : "FAIL");
        return ok ? 0 : 1;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FAIL %s\n", e.what());
        return 1;
    }
}
