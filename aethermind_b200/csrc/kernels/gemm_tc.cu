// Prefill dequant GEMM on the tcgen05 tensor cores.
#include "../amcu_internal.h"
#include "gemm_tc.cuh"

namespace amcu {

bool gemm_tc_supported(const GemmTcParams&, int) { return false; }
size_t gemm_tc_workspace_bytes(const GemmTcParams&, int) { return 0; }
am_status_code launch_gemm_tc(const GemmTcParams&, int, int, cudaStream_t) {
    return set_error(AM_STATUS_UNIMPLEMENTED, "tcgen05 GEMM not built");
}

}  // namespace amcu
