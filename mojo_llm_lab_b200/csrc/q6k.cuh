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
// copies of row tiles into a shared-memory ring, activation quants resident
// in registers).  Work unit = one 16-column run of one half h: 16 bytes each
// of ql-low, ql-high and qh feed 64 weights in four Q8_1 groups, one scale
// each, so a lane finishes its four groups alone.  Blocks start every 210
// bytes, so odd blocks sit 2 bytes off a word boundary in shared memory; each
// 16-byte field is read as five aligned words and funnel-shifted (rows are
// whole words apart, so a lane's word offsets and shift are the same in every
// row).  The q6 bytes of a group are one bit-select of a nibble word and a
// shifted high-pair word under the nibble mask:
//   k0: ql-low  & 0x0f | qh bits 0-1 << 4    k1: ql-high & 0x0f | qh bits 2-3 << 2
//   k2: ql-low >> 4    | qh bits 4-5         k3: ql-high >> 4   | qh bits 6-7 >> 2
// with qh pre-masked to its (0-1, 4-5) and (2-3, 6-7) pairs so no shifted
// neighbour bit survives the select.  q6 stays unsigned in dp4a.u32.s32 and
// the -32 offset enters as the accumulator start -32 * sum(a).  Each group's
// integer sum times its scale is exact; the fp64 terms are exact products, so
// the row sum is the exactly rounded value to ~1e-16 before the final fp32
// rounding.
#pragma once

#include "common.cuh"
#include "q4k.cuh"

namespace mllb {

constexpr int kQ6kBlockBytes = 210;

// The four groups' raw integer dots of a 16-column run (the streaming
// kernel's unit): u[k] = sum(q6 * a) - 32 * sum(a) over columns
// [l0, l0 + 16) of group 4h + k (c[k] = -32 * sum(a) precomputed).  `lo_w`
// is the word holding the run's first ql-low byte (its ql-high bytes lie 32
// bytes on, at the same alignment), `qh_w` the word of its first qh byte;
// each field starts sh = 0 or 16 bits past its word.
__device__ __forceinline__ void q6k_run_dots(const uint8_t* lo_w, const uint8_t* qh_w, uint32_t sh,
                                             const uint32_t (&a)[4][4], const int (&c)[4], int (&u)[4]) {
  const uint32_t* pl = reinterpret_cast<const uint32_t*>(lo_w);
  const uint32_t* ph = reinterpret_cast<const uint32_t*>(qh_w);
  const uint32_t m4 = 0x0f0f0f0fu;
  int acc[4] = {c[0], c[1], c[2], c[3]};
  uint32_t lw = pl[0], hw = pl[8], qw = ph[0];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t ln = pl[j + 1], hn = pl[j + 9], qn = ph[j + 1];
    const uint32_t lo = __funnelshift_r(lw, ln, sh), hi = __funnelshift_r(hw, hn, sh);
    const uint32_t qh = __funnelshift_r(qw, qn, sh);
    lw = ln;
    hw = hn;
    qw = qn;
    const uint32_t qa = qh & 0x33333333u, qb = qh & 0xccccccccu;
    acc[0] = dp4a_us((lo & m4) | ((qa << 4) & ~m4), a[0][j], acc[0]);
    acc[1] = dp4a_us((hi & m4) | ((qb << 2) & ~m4), a[1][j], acc[1]);
    acc[2] = dp4a_us(((lo >> 4) & m4) | (qa & ~m4), a[2][j], acc[2]);
    acc[3] = dp4a_us(((hi >> 4) & m4) | ((qb >> 2) & ~m4), a[3][j], acc[3]);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) u[k] = acc[k];
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
