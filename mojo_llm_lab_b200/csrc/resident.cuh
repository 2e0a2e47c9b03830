// Resident-weights Q4_K (and Q5_K) x Q8_1 matvec for matrices that fit in the
// SMs' shared memory (a decode step's Q / K / V / O projections: N <= 32 rows
// per SM).  One body for both formats: Q5_K's 176-byte blocks carry the same
// header and nibbles plus qh[32], whose fifth bits are merged into the
// nibbles after the wait (resident_q5k_kernel).
//
// A matvec launched right after the kernel that produces its activation is
// latency-bound, not bandwidth-bound: one 5.9 MB matrix streams in ~0.9 us,
// while a launch's dependent chain (wait for the producer, read the
// activation, compute, reduce, store) takes longer.  So this kernel moves
// everything that depends only on the weights ahead of the dependency wait:
//
// * One CTA per SM takes a contiguous run of R <= 32 rows (R = ceil(N / SMs)).
//   Before griddepcontrol.wait, one thread brings the run into shared memory
//   with a single cp.async.bulk (R x NB x 144 bytes, L2 evict-first), and
//   every lane decodes the 6-bit (scale, min) pair of the groups it
//   finalises into exact products d*sc and dmin*m (11 + 6 significant bits),
//   held in fp64 with the 1/16 of its unshifted high nibbles folded into
//   d*sc, and (NB = 10) loads its weight nibbles into registers.  The CTA
//   triggers launch_dependents at once, so the next launch of a chain starts
//   its own prefetch on the SM's second CTA slot while this one waits and
//   computes.
// * After the wait only activation-dependent work remains: one thread per
//   Q8_1 group re-lays the activation into shared memory (its 32 quants at a
//   bank-spread 16-byte-aligned slot, then its fp64 delta and the exact int
//   sum of its quants), one CTA barrier, and each lane reads per unit two
//   16-byte quant vectors, a delta and a sum, forms 8 dp4a, swaps one partial
//   dot with its partner lane, adds its terms in fp64 (no conversion after
//   the wait but the exact int -> fp64 adds), and the half-warp reduces by
//   xor-shuffles; lane 0 stores the row.
//
// Layout: a half-warp per row (warp w: rows 2w, 2w+1), 16 lanes x NB/2 units
// of 16 nibble bytes.  Lane l16 (h = l16 & 1, m = l16 >> 1) takes the units
// of group pairs q = m + 8i (i < NB/2): block b = q >> 2, pair j = q & 3,
// bytes [16 + 32j + 16h, +16) -- groups 2j (low nibbles) and 2j+1 (high
// nibbles), elements [16h, 16h + 16) of each.  Lanes 2m and 2m+1 hold the two
// halves of both groups; after one exchange lane h finalises group s = 2j+h.
//
// Numerics as the streaming kernels (csrc/stream.cuh): integer sub-block dots
// exact; d*sc*dot and dmin*m*sum(q) exact in fp64; one rounding for their
// difference, one for the Q8_1 scale, then a fixed-order fp64 sum per row and
// one rounding to fp32.
//
// Trace points (-DMLLB_TRACE builds): 0 start, 1 weights landed, 2 dependency
// wait returned, 3 activation staged, 7 row stored.
#pragma once

#include "common.cuh"
#include "q4k.cuh"

namespace mllb {

// Units per lane up to which a lane keeps its weight nibbles in registers.
#ifndef MLLB_RESIDENT_WQ_REGS_MAX
#define MLLB_RESIDENT_WQ_REGS_MAX 5
#endif

constexpr int kResidentMaxRowsPerCta = 32;
constexpr int kResidentThreads = 32 * (kResidentMaxRowsPerCta / 2);

// Shared-memory slot of Q8_1 group G's 32 quants: 32 bytes per group plus 32
// bytes of padding after every 4 groups, so that the 8 lanes of a quarter-warp
// (groups 2m and 2m + 1, halves h) read 8 disjoint 4-bank runs.
__host__ __device__ constexpr int resident_act_slot(int g) { return 32 * (g + (g >> 2)); }

template <int NB>
struct ResidentAct {
  static constexpr int kGroups = NB * 8;
  static constexpr int kQuantBytes = resident_act_slot(kGroups);
  static constexpr int kBytes = kQuantBytes + kGroups * 12;  // + fp64 delta, then int32 sum q, per group
};

// Super-block layout of the two formats: Q4_K (144 B: d, dmin, 12 scale
// bytes, 128 nibble bytes) and Q5_K (176 B: the same header, qh[32] -- bit g
// of qh[l] is the fifth bit of element l of group g -- then the 128 nibble
// bytes).
template <bool kQ5>
struct ResidentBlock {
  static constexpr int kBytes = kQ5 ? 176 : kQ4kBlockBytes;
  static constexpr int kQsOffset = kQ5 ? 48 : 16;
  static constexpr int kQhOffset = 16;
};

template <int NB, bool kQ5>
__device__ __forceinline__ void resident_body(const uint8_t* __restrict__ w, const uint8_t* __restrict__ q8,
                                              float* __restrict__ out, int n_rows, int rows_per_cta) {
  static_assert(NB % 2 == 0, "two units per group pair: NB must be even");
  using B = ResidentBlock<kQ5>;
  constexpr int UPL = NB / 2;  // units per lane
  constexpr int ROWB = NB * B::kBytes;
  constexpr int G = NB * 8;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  __shared__ __align__(16) uint8_t act[ResidentAct<NB>::kBytes];
  double* act_delta = reinterpret_cast<double*>(act + ResidentAct<NB>::kQuantBytes);
  int* act_sum = reinterpret_cast<int*>(act + ResidentAct<NB>::kQuantBytes + G * 8);

  MLLB_TRACE_POINT(0);
  const int row0 = blockIdx.x * rows_per_cta;
  const int rows = min(rows_per_cta, n_rows - row0);  // >= 1 by the host's grid
  const uint32_t bytes = static_cast<uint32_t>(rows * ROWB);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar, bytes);
    bulk_copy_g2s(smem, w + static_cast<size_t>(row0) * ROWB, bytes, &bar, l2_evict_first_policy());
  }
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = 2 * warp + (lane >> 4);
  const int l16 = lane & 15, h = l16 & 1, m = l16 >> 1;
  __syncthreads();  // the barrier's initialisation before anyone waits on it
  const bool landed = __syncthreads_and(mbar_wait_bounded(&bar, 0));
  if (!landed) {
    if (threadIdx.x == 0) {
      record_error(kErrFullWaitTimeout);
      if (!mbar_wait_bounded(&bar, 0)) record_error(kErrDrainTimeout);  // never leave with the copy in flight
    }
    return;
  }
  MLLB_TRACE_POINT(1);

  // ---- weights only: before the dependency wait
  const uint8_t* row = smem + (r < rows ? r : rows - 1) * ROWB;
  // Nibbles in registers before the wait when they fit the 64-register
  // budget (NB = 10); wider rows re-read them from shared memory after it.
  // (Q5_K reads its nibbles and fifth bits from shared memory after the
  // wait: the two would not fit beside the fp64 scales.)
  constexpr bool kWeightsInRegs = !kQ5 && UPL <= MLLB_RESIDENT_WQ_REGS_MAX;
  uint4 wq[kWeightsInRegs ? UPL : 1];
  double dsc[UPL], dmn[UPL];
#pragma unroll
  for (int i = 0; i < UPL; ++i) {
    const int q = m + 8 * i, b = q >> 2, j = q & 3, s = 2 * j + h;
    const uint8_t* blk = row + b * B::kBytes;
    if constexpr (kWeightsInRegs) wq[i] = lds128(blk + B::kQsOffset + 32 * j + 16 * h);
    const uint32_t dd = lds32(blk);
    const uint8_t* sm = blk + 4;
    int sc, mn;
    if (s < 4) {
      sc = sm[s] & 63;
      mn = sm[s + 4] & 63;
    } else {
      sc = (sm[s + 4] & 15) | ((sm[s - 4] >> 6) << 4);
      mn = (sm[s + 4] >> 4) | ((sm[s] >> 6) << 4);
    }
    // fp16 d (11 significant bits) x 6-bit scale: exact in fp32.
    // Q4_K: the lane's high-nibble dots are 16x (unshifted nibbles): 1/16
    // enters its d * sc here, exactly, so no conversion or scaling remains
    // after the wait.  Q5_K shifts its high nibbles down to merge the fifth
    // bits, so its dots are 1x.
    dsc[i] = static_cast<double>(__half2float(__ushort_as_half(static_cast<unsigned short>(dd & 0xffffu))) *
                                 static_cast<float>(sc)) * ((h && !kQ5) ? 0.0625 : 1.0);
    dmn[i] = static_cast<double>(__half2float(__ushort_as_half(static_cast<unsigned short>(dd >> 16))) *
                                 static_cast<float>(mn));
  }

  pdl_wait_prerequisite();  // the activation may come from the preceding kernel
  MLLB_TRACE_POINT(2);

  // ---- activation-dependent work: stage, then compute
  for (int g = threadIdx.x; g < G; g += blockDim.x) {  // blockDim can be below G for small row counts
    const uint32_t* src = reinterpret_cast<const uint32_t*>(q8 + g * kQ8BlockBytes);
    uint32_t v[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) v[t] = __ldg(src + t);
    int sum = 0;
#pragma unroll
    for (int t = 1; t < 9; ++t) sum = byte_sum_s8(v[t], sum);
    uint4* dst = reinterpret_cast<uint4*>(act + resident_act_slot(g));
    dst[0] = make_uint4(v[1], v[2], v[3], v[4]);
    dst[1] = make_uint4(v[5], v[6], v[7], v[8]);
    act_delta[g] = half_bits_to_double(v[0]);
    act_sum[g] = sum;
  }
  __syncthreads();
  MLLB_TRACE_POINT(3);
  double acc = 0.0;
#pragma unroll
  for (int i = 0; i < UPL; ++i) {
    const int q = m + 8 * i;  // group pair: groups 2q (low nibbles) and 2q + 1 (high nibbles)
    const uint4 al = lds128(act + resident_act_slot(2 * q) + 16 * h);
    const uint4 ah = lds128(act + resident_act_slot(2 * q + 1) + 16 * h);
    const double delta = act_delta[2 * q + h];
    const int sum = act_sum[2 * q + h];
    uint4 wv;
    const uint8_t* blk = row + (q >> 2) * B::kBytes;
    if constexpr (kWeightsInRegs) wv = wq[i];
    else wv = lds128(blk + B::kQsOffset + 32 * (q & 3) + 16 * h);
    int dlo, dhi;
    if constexpr (kQ5) {
      // 5-bit values: low nibbles | fifth bit 2j, high nibbles >> 4 | fifth bit 2j + 1.
      const uint4 hv = lds128(blk + B::kQhOffset + 16 * h);
      const int lb = 2 * (q & 3);
      const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w}, ha[4] = {hv.x, hv.y, hv.z, hv.w};
      const uint32_t xl[4] = {al.x, al.y, al.z, al.w}, xh[4] = {ah.x, ah.y, ah.z, ah.w};
      dlo = 0;
      dhi = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        dlo = dp4a_us((wa[t] & 0x0f0f0f0fu) | (((ha[t] >> lb) & 0x01010101u) << 4), xl[t], dlo);
        dhi = dp4a_us(((wa[t] >> 4) & 0x0f0f0f0fu) | (((ha[t] >> (lb + 1)) & 0x01010101u) << 4), xh[t], dhi);
      }
    } else {
      // Low nibbles x group 2q; high nibbles (unshifted, 16x) x group 2q + 1.
      dlo = dp4a_us(wv.x & 0x0f0f0f0fu, al.x, 0);
      dhi = dp4a_us(wv.x & 0xf0f0f0f0u, ah.x, 0);
      dlo = dp4a_us(wv.y & 0x0f0f0f0fu, al.y, dlo);
      dhi = dp4a_us(wv.y & 0xf0f0f0f0u, ah.y, dhi);
      dlo = dp4a_us(wv.z & 0x0f0f0f0fu, al.z, dlo);
      dhi = dp4a_us(wv.z & 0xf0f0f0f0u, ah.z, dhi);
      dlo = dp4a_us(wv.w & 0x0f0f0f0fu, al.w, dlo);
      dhi = dp4a_us(wv.w & 0xf0f0f0f0u, ah.w, dhi);
    }
    // Lane h keeps group 2q+h and takes the partner's half of it.
    const int dot = (h ? dhi : dlo) + __shfl_xor_sync(0xffffffffu, h ? dlo : dhi, 1);
    const double t = fma(dsc[i], i2d_exact(dot), -dmn[i] * i2d_exact(sum));
    acc = fma(delta, t, acc);
  }
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (l16 == 0 && r < rows) out[row0 + r] = static_cast<float>(acc);
  MLLB_TRACE_POINT(7);
}

template <int NB>
__global__ void __launch_bounds__(kResidentThreads, 2)
    resident_q4k_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ q8, float* __restrict__ out,
                        int n_rows, int rows_per_cta) {
  resident_body<NB, false>(w, q8, out, n_rows, rows_per_cta);
}

template <int NB>
__global__ void __launch_bounds__(kResidentThreads, 2)
    resident_q5k_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ q8, float* __restrict__ out,
                        int n_rows, int rows_per_cta) {
  resident_body<NB, true>(w, q8, out, n_rows, rows_per_cta);
}

}  // namespace mllb
