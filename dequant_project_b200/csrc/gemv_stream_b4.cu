// Streaming GEMV kernel variants for 4-bit codes (see gemv_stream.cuh).
#include "gemv_stream.cuh"

namespace dqg {

cudaError_t launch_stream_b4(int wpl, int gs, bool sym, bool inter, const StreamParams& p,
                             int grid, int smem, cudaStream_t stream) {
  return stream::launch_bits<4>(wpl, gs, sym, inter, p, grid, smem, stream);
}

}  // namespace dqg

DQG_STATUS_READER(read_status_stream_b4)
