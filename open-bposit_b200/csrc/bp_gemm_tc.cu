// bp_gemm_tc.cu -- tensor-core (tcgen05) quire GEMM.  Placeholder until the
// sm_100a kernel lands: reports itself unsupported so the front end keeps the
// CUDA-core path.
#include <cuda_runtime.h>
#include <stdint.h>

#include "bp_internal.cuh"

namespace bp {

bool gemm_tc_supported(int, int, int, int) { return false; }
size_t gemm_tc_workspace(int, int, int, int) { return 0; }
int launch_gemm_tc(const GemmArgs &, const int4 *, const int4 *, void *, size_t, cudaStream_t) {
  return set_error(kEInval, "tensor-core quire GEMM not available");
}

}  // namespace bp
