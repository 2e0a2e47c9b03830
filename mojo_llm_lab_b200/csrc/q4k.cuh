// Q4_K x Q8_1 matrix-vector kernels (single-token decode).
//
// Replaces the reference's plain matvec entries
// (kernels/q4_k_q8_1_matvec*.mojo, e.g. q4_k_q8_1_matvec_dp4a_128.mojo:8-53)
// and the fused gate/up entry (kernels/q4_k_q8_1_gate_order.mojo:55-79):
//   out[r] = sum_b [ d_b * sum_g delta_g * sc_bg * dot_bg  -  dmin_b * sum_g delta_g * m_bg * asum_g ]
// with dot_bg = sum of 32 nibble * int8 products (exact int32, dp4a) and
// asum_g the sum of the 32 int8 activation quants of group g.
//
// B200 design (one weight stream = one HBM pass, nothing else touches DRAM):
// * persistent CTAs: 8 consumer warps + 1 producer warp; the producer's
//   elected lane streams TILE-row weight tiles HBM -> shared memory with
//   cp.async.bulk (TMA bulk engine, L2 evict-first) through a ring of
//   mbarrier-guarded stages, so every SM keeps tens of KB in flight;
// * the Q8_1 activation (2880 B at K=2560) is copied once per CTA into shared
//   memory and each lane keeps the int8 quants it needs in registers for the
//   whole kernel: the 16-byte nibble chunks a lane reads sit at the same column
//   positions in every row group, so after the prologue the only shared-memory
//   traffic is the weight tile itself;
// * a row is split into P = 8*NB chunks of 16 nibble bytes (32 weights of two
//   sub-block groups); a warp owns RG rows = 32/gcd(P,32) so each lane holds a
//   whole number of chunk slots (NB=10: 2 rows, 5 slots);
// * lanes 2c and 2c+1 hold the two 16-byte halves of the same two groups; one
//   shuffle completes each group's integer dot, after which lane parity h
//   takes group 2j+h's fp64 terms;
// * per group: d*(sc*dot) - dmin*(m*asum) is formed in fp64 from exact
//   integers and fp16 scales (every product exact), times delta, added into a
//   per-slot fp64 accumulator.  The row sum is therefore the exactly rounded
//   value up to ~1e-16 relative, independent of reduction order, before the
//   single final rounding to fp32.
// The streaming (TMA) kernels are in stream.cuh; this file holds the block
// decode helpers and the row-per-CTA kernels.
#pragma once

#include "common.cuh"

namespace mllb {

constexpr int kQ4kBlockBytes = 144;
constexpr int kQ8BlockBytes = 36;

// Scale and min of groups 2j and 2j+1 (bytes 0 and 1 of *sc2 / *mn2) from
// the packed 12-byte field (header words y, z, w = bytes 4..15).  Groups 0-3
// keep 6 bits in bytes 0-3 / 4-7; groups 4-7 combine a nibble of bytes 8-11
// with the top two bits of bytes 0-7 (tests/q4_reference.py:57-62).
__device__ __forceinline__ void q4k_scale_min_pair(const uint4& hd, int j, uint32_t* sc2, uint32_t* mn2) {
  const int shift = (j & 1) * 16;
  const uint32_t a = (hd.y >> shift) & 0xffffu;
  const uint32_t b = (hd.z >> shift) & 0xffffu;
  const uint32_t c = (hd.w >> shift) & 0xffffu;
  if (j >= 2) {
    *sc2 = (c & 0x0f0fu) | ((a & 0xc0c0u) >> 2);
    *mn2 = ((c >> 4) & 0x0f0fu) | ((b & 0xc0c0u) >> 2);
  } else {
    *sc2 = a & 0x3f3fu;
    *mn2 = b & 0x3f3fu;
  }
}

// Re-lay K/32 Q8_1 blocks at `q8` (global) into shared memory for the
// streaming kernels: int8 quants of group G at [32G, 32G+32) (16-byte
// aligned), then GROUPS fp64 deltas, then GROUPS int32 quant sums.  One
// thread per group.
template <int GROUPS>
__device__ __forceinline__ void stage_q8_1(const uint8_t* __restrict__ q8, uint8_t* act, int tid, int nthreads) {
  for (int g = tid; g < GROUPS; g += nthreads) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(q8 + g * kQ8BlockBytes);
    uint32_t w[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) w[t] = __ldg(src + t);
    int sum = 0;
#pragma unroll
    for (int t = 1; t < 9; ++t) sum = byte_sum_s8(w[t], sum);
    uint4* qdst = reinterpret_cast<uint4*>(act + g * 32);
    qdst[0] = make_uint4(w[1], w[2], w[3], w[4]);
    qdst[1] = make_uint4(w[5], w[6], w[7], w[8]);
    reinterpret_cast<double*>(act + GROUPS * 32)[g] = half_bits_to_double(w[0] & 0xffffu);
    reinterpret_cast<int*>(act + GROUPS * 40)[g] = sum;
  }
}

// Decode one 144-byte super-block header (raw, in shared memory) into
//   [0,8) fp64 d   [8,16) fp64 dmin   [16,32) (scale, min) byte pairs of groups 0..7
// Groups 0-3 keep their 6 bits in packed bytes 0-3 / 4-7; groups 4-7 take a
// nibble of bytes 8-11 and the top two bits of bytes 0-3 / 4-7
// (tests/q4_reference.py:57-62).
__device__ __forceinline__ void q4k_decode_header(const uint8_t* raw, uint8_t* dst) {
  const uint4 hd = lds128(raw);
  const uint32_t lo_sc = hd.y & 0x3f3f3f3fu;
  const uint32_t lo_mn = hd.z & 0x3f3f3f3fu;
  const uint32_t hi_sc = (hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u);
  const uint32_t hi_mn = ((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u);
  double2* f = reinterpret_cast<double2*>(dst);
  *f = make_double2(half_bits_to_double(hd.x), half_bits_to_double(hd.x >> 16));
  *reinterpret_cast<uint4*>(dst + 16) =
      make_uint4(__byte_perm(lo_sc, lo_mn, 0x5140), __byte_perm(lo_sc, lo_mn, 0x7362),
                 __byte_perm(hi_sc, hi_mn, 0x5140), __byte_perm(hi_sc, hi_mn, 0x7362));
}

// ----------------------------------------------------------------------------
// One chunk (16 nibble bytes of groups 2j and 2j+1, half h) computed whole by
// one thread, for the row-per-CTA kernels below.  `blk` is the Q4_K block,
// `acts` the 8 Q8_1 groups of that block; loads go through the read-only path.
__device__ __forceinline__ double q4k_chunk_full(const uint8_t* __restrict__ blk, const uint8_t* __restrict__ acts,
                                                int s) {
  const int j = s >> 1, h = s & 1;
  const uint4 hd = *reinterpret_cast<const uint4*>(blk);
  const uint4 wq = *reinterpret_cast<const uint4*>(blk + 16 + 16 * s);
  const uint8_t* glo = acts + (2 * j) * kQ8BlockBytes;
  const uint8_t* ghi = glo + kQ8BlockBytes;
  const uint32_t* alo = reinterpret_cast<const uint32_t*>(glo + 4 + 16 * h);
  const uint32_t* ahi = reinterpret_cast<const uint32_t*>(ghi + 4 + 16 * h);
  const uint32_t w[4] = {wq.x, wq.y, wq.z, wq.w};
  int dlo = 0, dhi = 0, slo = 0, shi = 0;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t al = __ldg(alo + t), ah = __ldg(ahi + t);
    dlo = dp4a_ss(w[t] & 0x0f0f0f0fu, al, dlo);
    dhi = dp4a_ss((w[t] >> 4) & 0x0f0f0f0fu, ah, dhi);
    slo = byte_sum_s8(al, slo);
    shi = byte_sum_s8(ah, shi);
  }
  uint32_t sc2, mn2;
  q4k_scale_min_pair(hd, j, &sc2, &mn2);
  const double d = half_bits_to_double(hd.x), dmin = half_bits_to_double(hd.x >> 16);
  const double delta_lo = half_bits_to_double(__ldg(reinterpret_cast<const unsigned short*>(glo)));
  const double delta_hi = half_bits_to_double(__ldg(reinterpret_cast<const unsigned short*>(ghi)));
  const double t_lo = fma(d, static_cast<double>(static_cast<int>(sc2 & 0xffu) * dlo),
                          -dmin * static_cast<double>(static_cast<int>(mn2 & 0xffu) * slo));
  const double t_hi = fma(d, static_cast<double>(static_cast<int>(sc2 >> 8) * dhi),
                          -dmin * static_cast<double>(static_cast<int>(mn2 >> 8) * shi));
  return fma(delta_lo, t_lo, delta_hi * t_hi);
}

// Block-wide fp64 sum in fixed order (warp sums, then warp 0 over warps).
__device__ __forceinline__ double block_sum_double(double v, double* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_double(v);
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  double total = 0.0;
  if (threadIdx.x == 0)
    for (int i = 0; i < nw; ++i) total += scratch[i];
  return total;  // valid in thread 0
}

// Row-per-CTA kernel for any K (nb = K/256 blocks per row), any blockDim that
// is a multiple of 32.  This is the launch geometry of the reference's
// harnesses (grid = rows, block = 32 or 128) and the fallback for K values
// without a streaming specialisation.  w1 == nullptr means single stream.
__device__ __forceinline__ void q4k_rowblock_body(const uint8_t* __restrict__ w0, const uint8_t* __restrict__ w1,
                                                  const uint8_t* __restrict__ q8, float* __restrict__ out0,
                                                  float* __restrict__ out1, float* __restrict__ out2, int nb) {
  __shared__ double scratch[32];
  const int row = blockIdx.x;
  const size_t rowoff = static_cast<size_t>(row) * nb * kQ4kBlockBytes;
  double up = 0.0, gate = 0.0;
  for (int c = threadIdx.x; c < nb * 8; c += blockDim.x) {
    const int b = c >> 3, s = c & 7;
    const uint8_t* acts = q8 + static_cast<size_t>(b) * 8 * kQ8BlockBytes;
    up += q4k_chunk_full(w0 + rowoff + b * kQ4kBlockBytes, acts, s);
    if (w1) gate += q4k_chunk_full(w1 + rowoff + b * kQ4kBlockBytes, acts, s);
  }
  up = block_sum_double(up, scratch);
  if (w1) {
    __syncthreads();
    gate = block_sum_double(gate, scratch);
  }
  if (threadIdx.x == 0) {
    if (!w1) {
      if (out0) out0[row] = static_cast<float>(up);
    } else {
      if (out0) out0[row] = static_cast<float>(up);
      if (out1) out1[row] = static_cast<float>(gate);
      if (out2) out2[row] = static_cast<float>(up * (gate / (1.0 + exp(-gate))));
    }
  }
}

__global__ void q4k_rowblock_kernel(const uint8_t* __restrict__ w0, const uint8_t* __restrict__ w1,
                                    const uint8_t* __restrict__ q8, float* __restrict__ out0,
                                    float* __restrict__ out1, float* __restrict__ out2, int nb) {
  q4k_rowblock_body(w0, w1, q8, out0, out1, out2, nb);
}

// ----------------------------------------------------------------------------
// Exact integer parts (the bit-exact parity target): dots[r][G] for every row
// and Q8_1 group G, and asums[G] = sum of the group's int8 quants.
__global__ void q4k_subdots_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ q8,
                                   int32_t* __restrict__ dots, int32_t* __restrict__ asums, int64_t n_rows,
                                   int nb) {
  const int64_t groups = static_cast<int64_t>(nb) * 8;
  const int64_t total = n_rows * groups;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total + groups;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (idx < total) {
      const int64_t row = idx / groups;
      const int G = static_cast<int>(idx % groups);
      const int b = G >> 3, g = G & 7;
      const uint8_t* qs = w + (row * nb + b) * kQ4kBlockBytes + 16 + (g >> 1) * 32;
      const uint32_t* a = reinterpret_cast<const uint32_t*>(q8 + static_cast<int64_t>(G) * kQ8BlockBytes + 4);
      int dot = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t word = *reinterpret_cast<const uint32_t*>(qs + 4 * t);
        dot = dp4a_ss((word >> (4 * (g & 1))) & 0x0f0f0f0fu, __ldg(a + t), dot);
      }
      dots[idx] = dot;
    } else {
      const int64_t G = idx - total;
      const uint32_t* a = reinterpret_cast<const uint32_t*>(q8 + G * kQ8BlockBytes + 4);
      int sum = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) sum = byte_sum_s8(__ldg(a + t), sum);
      asums[G] = sum;
    }
  }
}

}  // namespace mllb
