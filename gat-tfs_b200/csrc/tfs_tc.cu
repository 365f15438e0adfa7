// Tensor-core TFS aggregation (placeholder until the tcgen05 kernel lands).
#include "device.cuh"
#include "graph.cuh"

namespace gatb {

bool tfs_tc_supported(const gat_b200_layer*) { return false; }

int tfs_tc_check_error() { return 0; }

int tfs_tc_dispatch(const gat_b200_graph*, const gat_b200_layer*, const uint16_t*, int, const float*, const float*,
                    const float*, int, int, void*, int, int, float*, cudaStream_t, int*) {
    return fail_code(GAT_B200_EUNSUPPORTED, "tfs: tensor-core kernel not built");
}

}  // namespace gatb
