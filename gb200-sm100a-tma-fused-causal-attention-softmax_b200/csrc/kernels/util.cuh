// Small utility kernels used by the host API: the reference's probe
// (gpu/src/main.rs:59-66), the output sentinel fill (gpu/src/driver.rs:78-79)
// and the padding-is-zero check (gpu/src/driver.rs:222-229).
#pragma once

#include <stdint.h>

namespace cs {

__global__ void probe_kernel(uint32_t* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (uint32_t)i ^ 0x5a5a5a5au;
}

__global__ void fill_u16_kernel(uint16_t* dst, int64_t n, uint16_t value) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = value;
}

// Counts nonzero entries in columns [cols, pitch) of every row.
__global__ void padding_check_kernel(const uint16_t* out, int64_t rows, int32_t cols,
                                     int32_t pitch, unsigned long long* bad) {
  const int32_t pad = pitch - cols;
  const int64_t n = rows * (int64_t)pad;
  unsigned long long local = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / pad;
    const int32_t c = cols + (int32_t)(i - r * pad);
    if (out[r * pitch + c] != 0) ++local;
  }
  if (local) atomicAdd(bad, local);
}

}  // namespace cs
