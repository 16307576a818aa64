// Direct GEMV kernel variants for 4-bit codes (see gemv_direct.cuh).
#include "gemv_direct.cuh"

namespace dqg {

cudaError_t launch_direct_b4(int wpl, int gs, bool sym, bool inter, const DirectParams& p,
                             int grid, int smem, cudaStream_t stream) {
  return direct::launch_bits<4>(wpl, gs, sym, inter, p, grid, smem, stream);
}

}  // namespace dqg

DQG_STATUS_READER(read_status_direct_b4)
