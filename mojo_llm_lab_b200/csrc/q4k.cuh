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
#pragma once

#include "common.cuh"

namespace mllb {

constexpr int kQ4kBlockBytes = 144;
constexpr int kQ8BlockBytes = 36;
constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = (kConsumerWarps + 1) * 32;

template <int NB>
struct Q4kGeom {
  static constexpr int kRowBytes = NB * kQ4kBlockBytes;
  static constexpr int kChunks = NB * 8;                                 // P
  static constexpr int kRowsPerWarp = 32 / gcd_constexpr(kChunks, 32);   // RG
  static constexpr int kSlots = kChunks * kRowsPerWarp / 32;
  static constexpr int kTileRows = kConsumerWarps * kRowsPerWarp;
  static constexpr int kActBytes = NB * 8 * kQ8BlockBytes;
  static constexpr int kActBytesPadded = (kActBytes + 15) / 16 * 16;
};

template <int NB, bool DUAL>
struct Q4kStreamConfig {
  using G = Q4kGeom<NB>;
  static constexpr int kStages = DUAL ? 2 : 4;
  static constexpr int kStageBytes = G::kTileRows * G::kRowBytes * (DUAL ? 2 : 1);
  static constexpr int kActOffset = kStages * kStageBytes;
  static constexpr int kBarOffset = kActOffset + G::kActBytesPadded;
  static constexpr int kSmemBytes = kBarOffset + 2 * kStages * 8;
};

// Scale and min of group (2j + h) of a block from the packed 12-byte field
// (header words y, z, w = bytes 4..15).  Groups 0-3 keep 6 bits in bytes
// 0-3 / 4-7; groups 4-7 combine a nibble of bytes 8-11 with the top two bits
// of bytes 0-7 (tests/q4_reference.py:57-62).
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

// ----------------------------------------------------------------------------
// Persistent TMA-pipelined kernel.  DUAL: two weight streams (up, gate) over
// the same activation, SwiGLU epilogue.
// Outputs (any may be null): out0 = first stream (up), out1 = second (gate),
// out2 = up * silu(gate).
template <int NB, bool DUAL>
__global__ void __launch_bounds__(kStreamThreads, 2)
    q4k_stream_kernel(const uint8_t* __restrict__ w0, const uint8_t* __restrict__ w1,
                      const uint8_t* __restrict__ q8, float* __restrict__ out0, float* __restrict__ out1,
                      float* __restrict__ out2, int n_rows) {
  using G = Q4kGeom<NB>;
  using Cfg = Q4kStreamConfig<NB, DUAL>;
  constexpr int S = Cfg::kStages;
  constexpr int SLOTS = G::kSlots;
  constexpr int RG = G::kRowsPerWarp;
  constexpr int TILE = G::kTileRows;
  constexpr int ROWB = G::kRowBytes;
  constexpr int P = G::kChunks;

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* act = smem + Cfg::kActOffset;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* empty = full + S;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntiles = (n_rows + TILE - 1) / TILE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      int k = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++k) {
        const int s = k % S;
        if (k >= S && !mbar_wait_bounded(&empty[s], ((k / S) - 1) & 1)) {
          record_error(kErrEmptyWaitTimeout);
          ok = false;
          break;
        }
        const int rows = min(TILE, n_rows - tile * TILE);
        const uint32_t bytes = static_cast<uint32_t>(rows * ROWB);
        uint8_t* stage = smem + s * Cfg::kStageBytes;
        const size_t goff = static_cast<size_t>(tile) * TILE * ROWB;
        mbar_arrive_expect_tx(&full[s], DUAL ? 2 * bytes : bytes);
        bulk_copy_g2s(stage, w0 + goff, bytes, &full[s], policy);
        if (DUAL) bulk_copy_g2s(stage + TILE * ROWB, w1 + goff, bytes, &full[s], policy);
      }
      // Never leave the CTA with copies in flight: wait for the last fill of
      // every stage (already complete in the normal path).
      const int issued = k;
      for (int u = issued - 1; u >= 0 && u >= issued - S; --u) {
        if (!mbar_wait_bounded(&full[u % S], (u / S) & 1)) {
          record_error(kErrDrainTimeout);
          break;
        }
      }
      (void)ok;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // The activation is the only input a preceding kernel may have produced
  // (weights are constant): wait for it here, not in the producer.
  pdl_wait_prerequisite();
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(q8);
    uint32_t* dst = reinterpret_cast<uint32_t*>(act);
    for (int i = threadIdx.x; i < G::kActBytes / 4; i += kConsumerWarps * 32) dst[i] = __ldg(src + i);
  }
  named_barrier(1, kConsumerWarps * 32);

  const int h = lane & 1;  // which 16-byte half of the 32-weight groups
  uint32_t a_lo[SLOTS][4], a_hi[SLOTS][4];
  double delta[SLOTS];
  int asum[SLOTS];
  int slot_row[SLOTS], slot_j[SLOTS], slot_block[SLOTS], slot_chunk[SLOTS];
#pragma unroll
  for (int i = 0; i < SLOTS; ++i) {
    const int vp = lane + 32 * i;
    const int p = vp % P;
    const int b = p >> 3, s = p & 7, j = s >> 1;
    slot_row[i] = vp / P;
    slot_j[i] = j;
    slot_block[i] = b;
    slot_chunk[i] = s;
    const uint8_t* glo = act + (b * 8 + 2 * j) * kQ8BlockBytes;
    const uint8_t* ghi = glo + kQ8BlockBytes;
    const uint8_t* gme = act + (b * 8 + s) * kQ8BlockBytes;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      a_lo[i][t] = lds32(glo + 4 + 16 * h + 4 * t);
      a_hi[i][t] = lds32(ghi + 4 + 16 * h + 4 * t);
    }
    int sum = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) sum = byte_sum_s8(lds32(gme + 4 + 4 * t), sum);
    asum[i] = sum;
    delta[i] = half_bits_to_double(lds32(gme) & 0xffffu);
  }

  int k = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++k) {
    const int s = k % S;
    if (!mbar_wait_bounded(&full[s], (k / S) & 1)) {
      record_error(kErrFullWaitTimeout);
      break;
    }
    const uint8_t* stage = smem + s * Cfg::kStageBytes;
    double acc0[SLOTS], acc1[SLOTS];
#pragma unroll
    for (int i = 0; i < SLOTS; ++i) {
      const uint8_t* rowp = stage + (warp * RG + slot_row[i]) * ROWB + slot_block[i] * kQ4kBlockBytes;
#pragma unroll
      for (int m = 0; m < (DUAL ? 2 : 1); ++m) {
        const uint8_t* bp = rowp + m * TILE * ROWB;
        const uint4 hd = lds128(bp);
        const uint4 wq = lds128(bp + 16 + 16 * slot_chunk[i]);
        int dlo = 0, dhi = 0;
        dlo = dp4a_ss(wq.x & 0x0f0f0f0fu, a_lo[i][0], dlo);
        dhi = dp4a_ss((wq.x >> 4) & 0x0f0f0f0fu, a_hi[i][0], dhi);
        dlo = dp4a_ss(wq.y & 0x0f0f0f0fu, a_lo[i][1], dlo);
        dhi = dp4a_ss((wq.y >> 4) & 0x0f0f0f0fu, a_hi[i][1], dhi);
        dlo = dp4a_ss(wq.z & 0x0f0f0f0fu, a_lo[i][2], dlo);
        dhi = dp4a_ss((wq.z >> 4) & 0x0f0f0f0fu, a_hi[i][2], dhi);
        dlo = dp4a_ss(wq.w & 0x0f0f0f0fu, a_lo[i][3], dlo);
        dhi = dp4a_ss((wq.w >> 4) & 0x0f0f0f0fu, a_hi[i][3], dhi);
        // Lane h keeps group 2j+h; its partner holds the other 16 weights.
        const int mine = h ? dhi : dlo;
        const int send = h ? dlo : dhi;
        const int dot = mine + __shfl_xor_sync(0xffffffffu, send, 1);
        uint32_t sc2, mn2;
        q4k_scale_min_pair(hd, slot_j[i], &sc2, &mn2);
        const int sc = static_cast<int>((sc2 >> (8 * h)) & 0xffu);
        const int mn = static_cast<int>((mn2 >> (8 * h)) & 0xffu);
        const double d = half_bits_to_double(hd.x);
        const double dmin = half_bits_to_double(hd.x >> 16);
        const double term = fma(d, static_cast<double>(sc * dot), -dmin * static_cast<double>(mn * asum[i]));
        if (m == 0)
          acc0[i] = delta[i] * term;
        else
          acc1[i] = delta[i] * term;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

#pragma unroll
    for (int r = 0; r < RG; ++r) {
      double v0 = 0.0, v1 = 0.0;
#pragma unroll
      for (int i = 0; i < SLOTS; ++i) {
        if (slot_row[i] == r) {
          v0 += acc0[i];
          if (DUAL) v1 += acc1[i];
        }
      }
      v0 = warp_sum_double(v0);
      if (DUAL) v1 = warp_sum_double(v1);
      const int row = tile * TILE + warp * RG + r;
      if (lane == 0 && row < n_rows) {
        if (out0) out0[row] = static_cast<float>(v0);
        if (DUAL) {
          if (out1) out1[row] = static_cast<float>(v1);
          if (out2) out2[row] = static_cast<float>(v0 * (v1 / (1.0 + exp(-v1))));
        }
      }
    }
  }
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
