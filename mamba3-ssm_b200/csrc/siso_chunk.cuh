// Chunked tensor-core (tcgen05) SISO forward for bf16 I/O on sm_100a.
#pragma once
#include "siso_scan.cuh"

namespace m3 {

// True when the chunked kernel covers this request (dtypes, d_state, headdim, alignment).
bool siso_chunk_supported(const SisoParams& p, int xdt, int bcdt);
int launch_siso_fwd_chunked(const SisoParams& p, int xdt, int bcdt, cudaStream_t s);
// Reads (and with `reset` clears) the chunked kernel's timeout word on the current device:
// nonzero once any of its bounded waits gave up. Synchronises the device.
int chunk_error_word(bool reset, int* out);

}  // namespace m3
