// Q6_K x Q8_1 matrix-vector kernel: the vocabulary projection
// (151,936 rows x K 2560, 319 MB of weights per token).
//
// The reference ships no kernel for it: its decode runs GGML's
// mul_mat_vec_q<Q6_K> (docs/q6k-vocab-roofline.md:7-12), which this replaces.
// Layout per 256 weights (210 bytes, public GGML block_q6_K): ql[128] low
// nibbles, qh[64] high 2-bit pairs, 16 int8 scales, fp16 d;
//   weight(128h + 32k + l) = d * sc[8h + 2k + l/16] * (q6 - 32),
//   q6 = nibble(ql[64h + 32*(k&1) + l], k>>1) | bits(qh[32h + l], 2k) << 4.
//
// Same streaming structure as the Q4_K kernel (persistent CTAs, TMA bulk
// copies of 16-row tiles into a 3-stage shared-memory ring, activation quants
// resident in registers).  Work unit = 8 consecutive l of one (half h,
// 16-column run): 8 bytes each of ql-low, ql-high and qh feed 32 weights in
// four Q8_1 groups.  Blocks start every 210 bytes, so odd blocks sit 2 bytes
// off a word boundary in shared memory; each 8-byte field is read as three
// aligned words and funnel-shifted.  q6 stays unsigned in dp4a.u32.s32 and
// the -32 offset enters as the accumulator start -32 * sum(a).  Lane pairs
// hold the two 8-column halves of a 16-column run (same scale); one shuffle
// per group pair completes each group's integer sum, then each lane forms two
// groups' fp64 terms (exact products) -- so, as for Q4_K, the row sum is the
// exactly rounded value before the final fp32 rounding.
#pragma once

#include "common.cuh"
#include "q4k.cuh"

namespace mllb {

constexpr int kQ6kBlockBytes = 210;

// Two words from an 8-byte field that starts 0 or 2 bytes past a word
// boundary (sh = 0 or 16 bits).
__device__ __forceinline__ void load_field8(const uint8_t* p, uint32_t sh, uint32_t* x0, uint32_t* x1) {
  const uint32_t* a = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
  const uint32_t w0 = a[0], w1 = a[1], w2 = a[2];
  *x0 = __funnelshift_r(w0, w1, sh);
  *x1 = __funnelshift_r(w1, w2, sh);
}

// Integer partial sums t[k] = sc_k * sum(q6 * a) - 32 * sc_k * sum(a) over
// the unit's 8 columns of groups 4h+k (c[k] = -32 * sum(a) is precomputed).
__device__ __forceinline__ void q6k_unit_ints(const uint8_t* blk, int h, int l0, const uint32_t (&a)[4][2],
                                              const int (&c)[4], int (&t)[4]) {
  const uint32_t sh = (reinterpret_cast<uintptr_t>(blk) & 2u) ? 16u : 0u;
  uint32_t lo0, lo1, hi0, hi1, qh0, qh1;
  load_field8(blk + 64 * h + l0, sh, &lo0, &lo1);
  load_field8(blk + 64 * h + 32 + l0, sh, &hi0, &hi1);
  load_field8(blk + 128 + 32 * h + l0, sh, &qh0, &qh1);
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h + (l0 >> 4));
  const uint32_t m4 = 0x0f0f0f0fu, m2 = 0x30303030u;
  const uint32_t q00 = (lo0 & m4) | ((qh0 << 4) & m2), q01 = (lo1 & m4) | ((qh1 << 4) & m2);
  const uint32_t q10 = (hi0 & m4) | ((qh0 << 2) & m2), q11 = (hi1 & m4) | ((qh1 << 2) & m2);
  const uint32_t q20 = ((lo0 >> 4) & m4) | (qh0 & m2), q21 = ((lo1 >> 4) & m4) | (qh1 & m2);
  const uint32_t q30 = ((hi0 >> 4) & m4) | ((qh0 >> 2) & m2), q31 = ((hi1 >> 4) & m4) | ((qh1 >> 2) & m2);
  t[0] = static_cast<int>(sc[0]) * dp4a_us(q01, a[0][1], dp4a_us(q00, a[0][0], c[0]));
  t[1] = static_cast<int>(sc[2]) * dp4a_us(q11, a[1][1], dp4a_us(q10, a[1][0], c[1]));
  t[2] = static_cast<int>(sc[4]) * dp4a_us(q21, a[2][1], dp4a_us(q20, a[2][0], c[2]));
  t[3] = static_cast<int>(sc[6]) * dp4a_us(q31, a[3][1], dp4a_us(q30, a[3][0], c[3]));
}

// Row-per-CTA fallback for any K and any row count (plain global loads; the
// 2-byte-aligned fields are read as halfwords).
__device__ __forceinline__ void q6k_rowblock_body(const uint8_t* __restrict__ w, const uint8_t* __restrict__ q8,
                                                  float* __restrict__ out, int nb) {
  __shared__ double scratch[32];
  const int row = blockIdx.x;
  double acc = 0.0;
  for (int u = threadIdx.x; u < nb * 8; u += blockDim.x) {
    const int b = u >> 3, u8 = u & 7;
    const int h = u8 >> 2, l0 = ((u8 >> 1) & 1) * 16 + (u8 & 1) * 8;
    const uint8_t* blk = w + (static_cast<size_t>(row) * nb + b) * kQ6kBlockBytes;
    uint32_t av[4][2];
    int cv[4];
    for (int kk = 0; kk < 4; ++kk) {
      const uint8_t* g = q8 + static_cast<size_t>(b * 8 + 4 * h + kk) * kQ8BlockBytes + 4 + l0;
      av[kk][0] = __ldg(reinterpret_cast<const uint32_t*>(g));
      av[kk][1] = __ldg(reinterpret_cast<const uint32_t*>(g + 4));
      cv[kk] = -32 * byte_sum_s8(av[kk][1], byte_sum_s8(av[kk][0], 0));
    }
    // Assemble the three 8-byte fields from halfwords (2-byte alignment).
    const unsigned short* hw = reinterpret_cast<const unsigned short*>(blk);
    auto field = [&](int off, uint32_t* x0, uint32_t* x1) {
      const unsigned short* f = hw + off / 2;
      *x0 = static_cast<uint32_t>(__ldg(f)) | (static_cast<uint32_t>(__ldg(f + 1)) << 16);
      *x1 = static_cast<uint32_t>(__ldg(f + 2)) | (static_cast<uint32_t>(__ldg(f + 3)) << 16);
    };
    uint32_t lo0, lo1, hi0, hi1, qh0, qh1;
    field(64 * h + l0, &lo0, &lo1);
    field(64 * h + 32 + l0, &hi0, &hi1);
    field(128 + 32 * h + l0, &qh0, &qh1);
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h + (l0 >> 4));
    const uint32_t m4 = 0x0f0f0f0fu, m2 = 0x30303030u;
    const uint32_t q[4][2] = {{(lo0 & m4) | ((qh0 << 4) & m2), (lo1 & m4) | ((qh1 << 4) & m2)},
                              {(hi0 & m4) | ((qh0 << 2) & m2), (hi1 & m4) | ((qh1 << 2) & m2)},
                              {((lo0 >> 4) & m4) | (qh0 & m2), ((lo1 >> 4) & m4) | (qh1 & m2)},
                              {((hi0 >> 4) & m4) | ((qh0 >> 2) & m2), ((hi1 >> 4) & m4) | ((qh1 >> 2) & m2)}};
    const double d = half_bits_to_double(__ldg(hw + 104));
    double part = 0.0;
    for (int kk = 0; kk < 4; ++kk) {
      const int tk = static_cast<int>(__ldg(sc + 2 * kk)) * dp4a_us(q[kk][1], av[kk][1], dp4a_us(q[kk][0], av[kk][0], cv[kk]));
      const double delta = half_bits_to_double(
          __ldg(reinterpret_cast<const unsigned short*>(q8 + static_cast<size_t>(b * 8 + 4 * h + kk) * kQ8BlockBytes)));
      part = fma(static_cast<double>(tk), delta, part);
    }
    acc = fma(d, part, acc);
  }
  acc = block_sum_double(acc, scratch);
  if (threadIdx.x == 0) out[row] = static_cast<float>(acc);
}

__global__ void q6k_rowblock_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ q8,
                                    float* __restrict__ out, int nb) {
  q6k_rowblock_body(w, q8, out, nb);
}

}  // namespace mllb
