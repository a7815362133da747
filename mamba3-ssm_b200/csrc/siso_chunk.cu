// Chunked tensor-core (tcgen05) SISO forward for bf16 I/O on sm_100a.
#include "m3_common.cuh"
#include "siso_chunk.cuh"

namespace m3 {

bool siso_chunk_supported(const SisoParams&, int, int) { return false; }

int launch_siso_fwd_chunked(const SisoParams&, int, int, cudaStream_t) {
  return fail(M3_ERR_UNSUPPORTED, "chunked siso forward: not available");
}

}  // namespace m3
