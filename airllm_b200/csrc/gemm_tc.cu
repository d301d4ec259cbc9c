// gemm_tc.cu -- K4/K5: tcgen05 grouped expert GEMMs for prefill.
#include "amoe_internal.cuh"

namespace amoe {

size_t tc_scratch_bytes(int, int, int) { return 0; }
bool tc_supported() { return false; }
cudaError_t launch_tc_forward(const Dims &, const LayerDev &, const RouteOut &, int, __half *,
                              __half *, float *, void *, cudaStream_t, StageHook, void *, int *) {
    return cudaErrorNotSupported;
}

}  // namespace amoe
