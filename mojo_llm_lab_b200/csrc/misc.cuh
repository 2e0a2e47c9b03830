// HBM read-roofline probe: stream a buffer once with 16-byte loads.
// Replaces kernels/stream_read_roofline.mojo:12-27 (8-byte loads on sm_86).
#pragma once

#include "common.cuh"

namespace mllb {

__global__ void __launch_bounds__(256) stream_read_kernel(const uint4* __restrict__ data, int64_t n16,
                                                          uint4* __restrict__ out) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  uint4 acc = make_uint4(0, 0, 0, 0);
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = ldg_stream128(data + i), b = ldg_stream128(data + i + stride);
    const uint4 c = ldg_stream128(data + i + 2 * stride), d = ldg_stream128(data + i + 3 * stride);
    acc.x ^= a.x ^ b.x ^ c.x ^ d.x;
    acc.y ^= a.y ^ b.y ^ c.y ^ d.y;
    acc.z ^= a.z ^ b.z ^ c.z ^ d.z;
    acc.w ^= a.w ^ b.w ^ c.w ^ d.w;
  }
  for (; i < n16; i += stride) {
    const uint4 a = ldg_stream128(data + i);
    acc.x ^= a.x;
    acc.y ^= a.y;
    acc.z ^= a.z;
    acc.w ^= a.w;
  }
  out[static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x] = acc;
}

}  // namespace mllb
