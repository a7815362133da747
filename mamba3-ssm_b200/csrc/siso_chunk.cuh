// Chunked tensor-core (tcgen05) SISO forward for bf16 I/O on sm_100a.
#pragma once
#include <cudaTypedefs.h>

#include "siso_scan.cuh"

namespace m3 {

// True when the chunked kernel covers this request (dtypes, d_state, headdim, alignment).
bool siso_chunk_supported(const SisoParams& p, int xdt, int bcdt);
int launch_siso_fwd_chunked(const SisoParams& p, int xdt, int bcdt, cudaStream_t s);
// Reads (and with `reset` clears) the chunked kernel's timeout word on the current device:
// nonzero once any of its bounded waits gave up. Synchronises the device.
int chunk_error_word(bool reset, int* out);

// Shared with the chunked backward: the driver's tensor-map encoder (null when the driver
// lacks it), a 4-d bf16 map over (inner, H, L, B) with a (64, 1, 128, 1) box and 128-byte
// swizzle, and the device's SM count.
PFN_cuTensorMapEncodeTiled_v12000 chunk_encode_fn();
int chunk_tmap_4d(CUtensorMap* m, const void* base, int64_t inner, int64_t H, int64_t L, int64_t Bn, const Str3& st);
int chunk_sm_count();

// Chunked tensor-core backward (siso_chunk_bwd.cu): bf16, P = 64, d_state 128 or 64.
bool siso_chunk_bwd_supported(const SisoParams& p, int xdt, int bcdt);
// bytes of the chunk-state array the forward writes for the backward
size_t siso_chunk_kstate_bytes(int64_t Bn, int64_t L, int64_t H);
// per-position fp32 scratch of the backward (three arrays of B*H*L floats)
size_t siso_chunk_bwd_scratch_bytes(int64_t Bn, int64_t L, int64_t H);
// p.kstates must hold the forward's chunk states; scratch >= siso_chunk_bwd_scratch_bytes
int launch_siso_bwd_chunked(const SisoParams& p, float* scratch, cudaStream_t s);
// the backward kernel's timeout word (as chunk_error_word)
int chunk_bwd_error_word(bool reset, int* out);

}  // namespace m3
