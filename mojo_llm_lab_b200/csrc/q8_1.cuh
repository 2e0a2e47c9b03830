// Q8_1 activation quantiser: fp32 x[k] -> k/32 blocks of 36 bytes
// (fp16 d, fp16 s, 32 x int8 q).
//
// Replaces GGML's quantize_q8_1 graph node that the reference clones in front
// of every matvec (benchmark/q4_compare.c:328-330, bytes checked at :351-357),
// with the fixture rule of tools/generate_q4_matvec_fixtures.py:56-59.
// Arithmetic (bit-exact with the CPU oracle):
//   amax = max |x|          d = amax / 127           (IEEE division)
//   q    = amax == 0 ? 0 : roundf(x / d)             (IEEE division, ties away)
//   d16  = fp16(d) RNE
//   s    = fp16(fp16(d) * sum(q))   [MLLB_Q8_1_S_D_SUMQ, default]
//        = fp16(sum(x))             [MLLB_Q8_1_S_SUM_X, butterfly order]
// One warp per block of 32 values; the quantiser is HBM/latency bound
// (4 B in, 1.125 B out per value).
#pragma once

#include "common.cuh"

namespace mllb {

enum : int { kQ8SumDTimesSumQ = 0, kQ8SumX = 1 };

// Quantise the 32 values held one per lane; returns this lane's int8 q and
// fills d16 / s16 (identical in every lane).
__device__ __forceinline__ int q8_1_quantize_lane(float x, int s_mode, uint32_t* d16, uint32_t* s16) {
  // max |x| over the warp as the fmaxf butterfly defines it (NaN lanes lose
  // unless every lane is NaN), in one warp reduction: non-negative floats
  // order as their bit patterns.
  const float ax = fabsf(x);
  const bool nan = ax != ax;
  const uint32_t mbits = __reduce_max_sync(0xffffffffu, nan ? 0u : __float_as_uint(ax));
  const float amax = __all_sync(0xffffffffu, nan) ? ax : __uint_as_float(mbits);
  const float d = __fdiv_rn(amax, 127.0f);
  const int q = amax == 0.0f ? 0 : static_cast<int>(roundf(__fdiv_rn(x, d)));
  const __half dh = __float2half_rn(d);
  float s;
  if (s_mode == kQ8SumX) {
    s = warp_sum_float_butterfly(x);
  } else {
    s = __half2float(dh) * static_cast<float>(__reduce_add_sync(0xffffffffu, q));  // exact product
  }
  *d16 = __half_as_ushort(dh);
  *s16 = __half_as_ushort(__float2half_rn(s));
  return q;
}

// Store one Q8_1 block (36 bytes) whose 32 values were quantised one per lane.
__device__ __forceinline__ void q8_1_store_block(uint8_t* blk, int q, uint32_t d16, uint32_t s16, int lane) {
  const uint32_t b = static_cast<uint32_t>(q) & 0xffu;
  const uint32_t b1 = __shfl_down_sync(0xffffffffu, b, 1);
  const uint32_t b2 = __shfl_down_sync(0xffffffffu, b, 2);
  const uint32_t b3 = __shfl_down_sync(0xffffffffu, b, 3);
  if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(blk + 4 + lane) = b | (b1 << 8) | (b2 << 16) | (b3 << 24);
  if (lane == 0) *reinterpret_cast<uint32_t*>(blk) = d16 | (s16 << 16);
}

// grid-stride over Q8_1 blocks, one warp each.
__global__ void __launch_bounds__(256) q8_1_quantize_kernel(const float* __restrict__ x, uint8_t* __restrict__ out,
                                                            int64_t blocks, int s_mode) {
  const int lane = threadIdx.x & 31;
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < blocks;
       g += warps) {
    const float v = x[g * 32 + lane];
    uint32_t d16, s16;
    const int q = q8_1_quantize_lane(v, s_mode, &d16, &s16);
    // Pack 4 consecutive int8 per lane group and store 8 words per block.
    const uint32_t b = static_cast<uint32_t>(q) & 0xffu;
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, b, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, b, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, b, 3);
    uint8_t* blk = out + g * 36;
    if ((lane & 3) == 0) {
      *reinterpret_cast<uint32_t*>(blk + 4 + lane) = b | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
    if (lane == 0) *reinterpret_cast<uint32_t*>(blk) = d16 | (s16 << 16);
  }
}

// Four values per lane: eight lanes per 32-value block, four blocks per warp
// (one 16-byte load per lane; x must be 16-byte aligned).  The same
// arithmetic as q8_1_quantize_lane -- max |x| with its NaN rule, IEEE
// d = amax / 127 and x / d, roundf, fp16 RNE, s by either convention with
// sum(x) in the same xor-butterfly association -- so the bytes are identical,
// with the per-block work (the d division, the reductions, the packing)
// shared by four values instead of repeated in every lane.
__global__ void __launch_bounds__(256) q8_1_quantize_x4_kernel(const float* __restrict__ x, uint8_t* __restrict__ out,
                                                               int64_t blocks, int s_mode) {
  const int lane = threadIdx.x & 31, sub = lane & 7;
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int64_t step = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5) * 4;
  for (int64_t g0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4; g0 < blocks;
       g0 += step) {
    const int64_t g = g0 + (lane >> 3);
    const bool live = g < blocks;
    const float4 v4 = live ? reinterpret_cast<const float4*>(x)[g * 8 + sub] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
    uint32_t mbits = 0u;
    bool all_nan = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = fabsf(v[i]);
      const bool nan = a != a;
      mbits = max(mbits, nan ? 0u : __float_as_uint(a));
      all_nan = all_nan && nan;
    }
    uint32_t every_nan = all_nan ? 1u : 0u;
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
      mbits = max(mbits, __shfl_xor_sync(0xffffffffu, mbits, off));
      every_nan &= __shfl_xor_sync(0xffffffffu, every_nan, off);
    }
    const float amax = every_nan ? fabsf(v[0]) : __uint_as_float(mbits);
    const float d = __fdiv_rn(amax, 127.0f);
    int q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = amax == 0.0f ? 0 : static_cast<int>(roundf(__fdiv_rn(v[i], d)));
    const __half dh = __float2half_rn(d);
    float s;
    if (s_mode == kQ8SumX) {
      // xor-butterfly over the block's 32 values (offsets 16, 8, 4 across
      // lanes, then 2, 1 inside the lane), as warp_sum_float_butterfly.
      float t[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
      for (int off = 4; off >= 1; off >>= 1)
#pragma unroll
        for (int i = 0; i < 4; ++i) t[i] += __shfl_xor_sync(0xffffffffu, t[i], off);
      const float u0 = t[0] + t[2], u1 = t[1] + t[3];
      s = u0 + u1;
    } else {
      int sum = q[0] + q[1] + q[2] + q[3];
#pragma unroll
      for (int off = 4; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      s = __half2float(dh) * static_cast<float>(sum);  // exact product
    }
    if (live) {
      uint8_t* blk = out + g * 36;
      *reinterpret_cast<uint32_t*>(blk + 4 + 4 * sub) =
          (static_cast<uint32_t>(q[0]) & 0xffu) | ((static_cast<uint32_t>(q[1]) & 0xffu) << 8) |
          ((static_cast<uint32_t>(q[2]) & 0xffu) << 16) | ((static_cast<uint32_t>(q[3]) & 0xffu) << 24);
      if (sub == 0)
        *reinterpret_cast<uint32_t*>(blk) =
            static_cast<uint32_t>(__half_as_ushort(dh)) | (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(s))) << 16);
    }
  }
}

// Peer all-gather of a Q8_1 activation: every rank quantises its slice and
// stores the blocks into every rank's buffer (NVLink stores), then (after one
// system-scope fence per CTA) counts one arrival per CTA into every rank's
// counter for its source slot.  CTA 0 of each rank polls its counters with
// volatile loads, then fences (acquire) once; it waits until every source has
// delivered this gather's CTAs (counters are cumulative: the target is
// (gathers so far + 1) x CTAs), so the kernel completes only when the whole
// activation is in local memory.  The wait is bounded (~1 s, then
// kErrPeerWaitTimeout).  Ranks run on separate GPUs and launch the same
// sequence with the same k, hence the same grid.
constexpr int kMaxPeers = 8;

struct PeerGather {
  int rank, world;
  uint8_t* buffers[kMaxPeers];  // every rank's destination, as seen from this GPU
  uint32_t* flags[kMaxPeers];   // every rank's counters [world], as seen from this GPU
  uint32_t* count;              // this rank's gathers so far (local)
};

__global__ void __launch_bounds__(256) q8_1_allgather_kernel(const float* __restrict__ x, int64_t blocks,
                                                             const PeerGather pg) {
  const int lane = threadIdx.x & 31;
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int64_t slice = static_cast<int64_t>(pg.rank) * blocks * 36;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < blocks;
       g += warps) {
    uint32_t d16, s16;
    const int q = q8_1_quantize_lane(x[g * 32 + lane], kQ8SumDTimesSumQ, &d16, &s16);
    for (int r = 0; r < pg.world; ++r) q8_1_store_block(pg.buffers[r] + slice + g * 36, q, d16, s16, lane);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_sys();  // the CTA's blocks (ordered by the barrier) before its arrivals
    for (int r = 0; r < pg.world; ++r) red_relaxed_sys_add(pg.flags[r] + pg.rank, 1u);
  }
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  const uint32_t target = (*pg.count + 1u) * gridDim.x;
  const uint32_t* mine = pg.flags[pg.rank];
  const uint64_t start = global_timer_ns();
  bool ok = true;
  for (int s = 0; s < pg.world && ok; ++s) {
    for (uint32_t i = 0;; ++i) {
      if (static_cast<int32_t>(ld_volatile_u32(mine + s) - target) >= 0) break;
      if ((i & 255u) == 255u && global_timer_ns() - start > kWaitLimitNs) {
        ok = false;
        break;
      }
      if (i >= kWaitMaxIters) {
        ok = false;
        break;
      }
    }
  }
  fence_sys();  // the peers' blocks are visible before this kernel completes
  if (!ok) record_error(kErrPeerWaitTimeout);
  *pg.count += 1u;
}

}  // namespace mllb
