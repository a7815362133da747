// Row-wise argmax (greedy token choice of the decode step).
#pragma once
#include <stdint.h>

namespace m3 {

int launch_argmax_rows(const void* x, int dtype, int64_t rows, int64_t n, int64_t sx, int64_t* out,
                       cudaStream_t s);

}  // namespace m3
