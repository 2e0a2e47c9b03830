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

// Bring `bytes` (a multiple of 16, 16-byte aligned) into L2 ahead of their
// use, marked evict-last: one thread per CTA issues bulk prefetches of up to
// 64 KB, grid-stride.  Nothing waits for them; the kernel ends once issued.
__global__ void __launch_bounds__(32) l2_prefetch_kernel(const uint8_t* __restrict__ data, int64_t bytes) {
  if (threadIdx.x != 0) return;
  constexpr int64_t kChunk = 64 * 1024;
  const uint64_t policy = l2_evict_last_policy();
  for (int64_t off = static_cast<int64_t>(blockIdx.x) * kChunk; off < bytes;
       off += static_cast<int64_t>(gridDim.x) * kChunk) {
    const int64_t n = bytes - off < kChunk ? bytes - off : kChunk;
    bulk_prefetch_l2(data + off, static_cast<uint32_t>(n), policy);
  }
}

}  // namespace mllb
