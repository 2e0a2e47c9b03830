// Batched-token (prefill) Q4_K x Q8_1 on the 5th-generation tensor cores.
//
// out[t][r] = sum over the Q4_K blocks b and groups s of row r of
//   d_b * sc_bs * delta_ts * dot(q4_rbs, q8_ts) - dmin_b * m_bs * delta_ts * asum_ts
// for T tokens t at once -- the operation llama.cpp runs as MMQ for prompt
// processing (the reference's prefill profile, docs/prefill-baseline.md, at
// 32-token ubatches), of which the single-token matvec is the T = 1 case.
//
// One 32-element group is exactly one K step of a tcgen05 kind::i8 MMA, so
// the integer dots of a whole 128-row x 32-token tile and one group are one
// instruction: A = the group's 4-bit quants as unsigned bytes (128 x 32,
// K-major), B = the tokens' int8 Q8_1 quants (32 x 32, K-major), D = int32 in
// tensor memory.  Each group's D is scaled on its own (the scales differ per
// group), so the MMA never accumulates: the 8 groups of a block land in 8
// TMEM column ranges, double-buffered by block (2 x 8 x 32 = 512 columns).
// The scaling runs in fp64 (each product exact; one rounding per fma), as
// in the single-token kernels, so the result is within 1e-5 + 1e-5 |ref| of
// the exact sums.
//
// CTA (672 threads, one per SM): warps 0-15 scale (warp w reads TMEM lanes
// 32 (w % 4).. for tokens 8 (w / 4)..), warps 16-19 unpack the weights (one
// row per thread), warp 20 owns the TMEM allocation and its lane 0 issues the
// MMAs.  The tokens' Q8_1 quants of the CTA's groups are staged once; the
// weight rows are read block by block with 16-byte loads, unpacked in
// registers into the canonical no-swizzle K-major layout (8-row x 16-byte
// core matrices), and their (d * sc, dmin * m) pairs stored as exact fp32.
// A grid of (row tiles, token tiles, K splits) covers the SMs; with more than
// one split each CTA writes fp64 partials and a second kernel adds them in
// split order.
#pragma once

#include "common.cuh"
#include "q4k.cuh"

namespace mllb {

constexpr int kPfRows = 128;                 // weight rows per CTA (MMA M)
constexpr int kPfTok = 32;                   // tokens per CTA (MMA N)
constexpr int kPfScaleWarps = 16;            // warps 0..15: fp64 scaling (TMEM readers)
constexpr int kPfUnpackWarps = 4;            // warps 16..19: weight unpack, one row per thread
constexpr int kPfMmaWarp = kPfScaleWarps + kPfUnpackWarps;  // warp 20: TMEM owner, lane 0 issues MMAs
constexpr int kPfThreads = (kPfMmaWarp + 1) * 32;          // 672
constexpr int kPfTokPerWarp = kPfTok / (kPfScaleWarps / 4); // tokens a scaling warp covers: 8
constexpr int kPfMaxGroups = 80;             // groups (32-element K steps) per CTA: 10 blocks
constexpr int kPfATile = kPfRows * 32;       // bytes of one group's A tile
constexpr int kPfBTile = kPfTok * 32;        // bytes of one group's B tile
constexpr int kPfTmemCols = 512;             // 2 blocks x 8 groups x 32 columns

// Shared memory (bytes; all offsets multiples of 128).
constexpr int kPfBOff = 0;                                             // B tiles [group]
constexpr int kPfTokScaleOff = kPfBOff + kPfMaxGroups * kPfBTile;      // double2 (delta, delta*asum) [group][token]
constexpr int kPfAOff = kPfTokScaleOff + kPfMaxGroups * kPfTok * 16;   // A tiles [buf][group of block]
constexpr int kPfRowScaleOff = kPfAOff + 2 * 8 * kPfATile;             // float2 (d*sc, dmin*m) [buf][s][row]
constexpr int kPfBarOff = kPfRowScaleOff + 2 * 8 * kPfRows * 8;        // mbarriers
constexpr int kPfSmemBytes = kPfBarOff + 128;

__device__ __forceinline__ uint64_t pf_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  // K-major, no swizzle: start >> 4 [0,14), LBO >> 4 [16,30), SBO >> 4 [32,46),
  // version 1 [46,48), base offset 0, LBO mode 0, layout type 0 [61,64).
  return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) | (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// kind::i8 instruction descriptor: D s32, A u8, B s8, both K-major, N = 32, M = 128.
constexpr uint32_t kPfIdesc = (2u << 4) | (0u << 7) | (1u << 10) | ((kPfTok >> 3) << 17) | ((kPfRows >> 4) << 24);

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// 8 consecutive 32-bit TMEM columns of this thread's lane (issue only;
// tc_wait_ld completes every load issued before it).
__device__ __forceinline__ void tc_ld8(uint32_t taddr, int32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of element (row m, k) of a K-major no-swizzle tile whose 8-row
// x 16-byte core matrices sit k-chunk-minor: LBO = 128 B, SBO = 256 B.
__device__ __forceinline__ int pf_tile_off(int m, int kchunk) { return (m >> 3) * 256 + kchunk * 128 + (m & 7) * 16; }

// Grid: (rows / 128, ceil(T / 32), splits).  Split z covers blocks
// [z * bps, min((z + 1) * bps, nb)).  partial == nullptr: one split, fp32 to
// out; otherwise fp64 to partial[z][t][row].
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_q4k_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ q8, int rows, int nb, int tokens,
                       int bps, float* __restrict__ out, double* __restrict__ partial) {
  extern __shared__ __align__(1024) uint8_t pf_smem[];
  uint8_t* smem = pf_smem;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + kPfBarOff);  // [2], count kPfUnpackWarps * 32
  uint64_t* d_full = a_full + 2;                                       // [2], tcgen05.commit
  uint64_t* d_free = a_full + 4;                                       // [2], count kPfScaleWarps * 32
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_full + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(a_full + 7);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kPfRows, tok0 = blockIdx.y * kPfTok;
  const int b0 = blockIdx.z * bps, b1 = min(b0 + bps, nb), nblk = b1 - b0;
  const int groups = nblk * 8;
  const int kq8 = nb * 8;  // Q8_1 blocks per token

  if (threadIdx.x == 0) {
    mbar_init(&a_full[0], kPfUnpackWarps * 32);
    mbar_init(&a_full[1], kPfUnpackWarps * 32);
    mbar_init(&d_full[0], 1);
    mbar_init(&d_full[1], 1);
    mbar_init(&d_free[0], kPfScaleWarps * 32);
    mbar_init(&d_free[1], kPfScaleWarps * 32);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kPfMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kPfTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Stage the tokens' quants of this CTA's groups (B tiles) and their scales.
  {
    double2* tok_scale = reinterpret_cast<double2*>(smem + kPfTokScaleOff);
    for (int i = threadIdx.x; i < groups * kPfTok; i += kPfThreads) {
      const int g = i / kPfTok, t = i % kPfTok;
      const int tg = tok0 + t;
      uint32_t qw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      double delta = 0.0;
      int asum = 0;
      if (tg < tokens) {
        const uint8_t* blk = q8 + (static_cast<size_t>(tg) * kq8 + b0 * 8 + g) * kQ8BlockBytes;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(blk);
        delta = half_bits_to_double(src[0] & 0xffffu);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          qw[u] = src[1 + u];
          asum = byte_sum_s8(qw[u], asum);
        }
      }
      uint8_t* tile = smem + kPfBOff + g * kPfBTile;
      *reinterpret_cast<uint4*>(tile + pf_tile_off(t, 0)) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
      *reinterpret_cast<uint4*>(tile + pf_tile_off(t, 1)) = make_uint4(qw[4], qw[5], qw[6], qw[7]);
      tok_scale[g * kPfTok + t] = make_double2(delta, delta * static_cast<double>(asum));  // both exact
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= kPfScaleWarps && warp < kPfMmaWarp) {
    // ------------------------------------------------ unpack: one row per thread
    const int r = threadIdx.x - kPfScaleWarps * 32;
    const uint8_t* wrow = w + static_cast<size_t>(row0 + r) * nb * kQ4kBlockBytes;
    float2* row_scale = reinterpret_cast<float2*>(smem + kPfRowScaleOff);
    for (int i = 0; i < nblk; ++i) {
      const int buf = i & 1;
      // Buffer `buf` (A tiles and row scales) was last read by block i - 2's
      // MMAs and scaling warps: wait until the scaling is done.
      if (i >= 2 && !mbar_wait_bounded(&d_free[buf], ((i - 2) >> 1) & 1)) {
        record_error(kErrEmptyWaitTimeout);
        *abort_flag = 1;
      }
      const uint4* src = reinterpret_cast<const uint4*>(wrow + static_cast<size_t>(b0 + i) * kQ4kBlockBytes);
      uint4 raw[9];
#pragma unroll
      for (int u = 0; u < 9; ++u) raw[u] = __ldg(src + u);
      const uint4 hd = raw[0];
      const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(hd.x & 0xffffu)));
      const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(hd.x >> 16)));
      const uint32_t lo_sc = hd.y & 0x3f3f3f3fu, lo_mn = hd.z & 0x3f3f3f3fu;
      const uint32_t hi_sc = (hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u);
      const uint32_t hi_mn = ((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u);
      uint8_t* atiles = smem + kPfAOff + buf * 8 * kPfATile;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t scw = s < 4 ? lo_sc : hi_sc, mnw = s < 4 ? lo_mn : hi_mn;
        const int sh = (s & 3) * 8;
        row_scale[(buf * 8 + s) * kPfRows + r] = make_float2(d * static_cast<float>((scw >> sh) & 0xffu),
                                                            dmin * static_cast<float>((mnw >> sh) & 0xffu));
        // Group s: the low (even s) or high (odd s) nibbles of qs bytes 32 (s / 2)...
        const uint4 c0 = raw[1 + 2 * (s >> 1)], c1 = raw[2 + 2 * (s >> 1)];
        const int shift = (s & 1) * 4;
        const uint4 n0 = make_uint4((c0.x >> shift) & 0x0f0f0f0fu, (c0.y >> shift) & 0x0f0f0f0fu,
                                    (c0.z >> shift) & 0x0f0f0f0fu, (c0.w >> shift) & 0x0f0f0f0fu);
        const uint4 n1 = make_uint4((c1.x >> shift) & 0x0f0f0f0fu, (c1.y >> shift) & 0x0f0f0f0fu,
                                    (c1.z >> shift) & 0x0f0f0f0fu, (c1.w >> shift) & 0x0f0f0f0fu);
        uint8_t* tile = atiles + s * kPfATile;
        *reinterpret_cast<uint4*>(tile + pf_tile_off(r, 0)) = n0;
        *reinterpret_cast<uint4*>(tile + pf_tile_off(r, 1)) = n1;
      }
      fence_proxy_async_smem();
      mbar_arrive(&a_full[buf]);
    }
  } else if (warp == kPfMmaWarp) {
    // ------------------------------------------------ MMA issue (one thread)
    if (lane == 0) {
      const uint32_t a_base = smem_addr(smem + kPfAOff), b_base = smem_addr(smem + kPfBOff);
      for (int i = 0; i < nblk; ++i) {
        const int buf = i & 1;
        bool ok = mbar_wait_bounded(&a_full[buf], (i >> 1) & 1);
        if (ok && i >= 2) ok = mbar_wait_bounded(&d_free[buf], ((i - 2) >> 1) & 1);
        if (!ok) {
          record_error(kErrFullWaitTimeout);
          *abort_flag = 1;
        }
        tc_fence_after();
        if (ok) {
#pragma unroll 1
          for (int s = 0; s < 8; ++s) {
            const uint64_t a_desc = pf_smem_desc(a_base + (buf * 8 + s) * kPfATile, 128, 256);
            const uint64_t b_desc = pf_smem_desc(b_base + (i * 8 + s) * kPfBTile, 128, 256);
            tc_mma_i8(tmem + buf * 256 + s * 32, a_desc, b_desc, kPfIdesc);
          }
        }
        tc_commit(&d_full[buf]);  // arrives once the MMAs above (if any) are done
      }
    }
  } else {
    // ------------------------------------------------ fp64 scaling
    // Warp w: TMEM lanes 32 (w % 4).. (its rows) and tokens 8 (w / 4)..; the
    // next group's TMEM columns load while this group's are scaled.
    const int lgrp = warp & 3;
    const int r = lgrp * 32 + lane;
    const int tq = warp >> 2;
    const double2* tok_scale = reinterpret_cast<const double2*>(smem + kPfTokScaleOff);
    const float2* row_scale = reinterpret_cast<const float2*>(smem + kPfRowScaleOff);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(lgrp * 32) << 16) + tq * kPfTokPerWarp;
    double acc[kPfTokPerWarp];
#pragma unroll
    for (int t = 0; t < kPfTokPerWarp; ++t) acc[t] = 0.0;
    auto scale_group = [&](const int32_t (&dv)[kPfTokPerWarp], int i, int buf, int s) {
      const float2 rs = row_scale[(buf * 8 + s) * kPfRows + r];
      const double as = rs.x, bs = rs.y;
      const double2* ts = tok_scale + (i * 8 + s) * kPfTok + tq * kPfTokPerWarp;
#pragma unroll
      for (int t = 0; t < kPfTokPerWarp; ++t) {
        const double2 sc = ts[t];
        const double x = as * static_cast<double>(dv[t]);  // exact
        acc[t] = fma(x, sc.x, acc[t]);
        acc[t] = fma(-bs, sc.y, acc[t]);
      }
    };
    for (int i = 0; i < nblk; ++i) {
      const int buf = i & 1;
      if (!mbar_wait_bounded(&d_full[buf], (i >> 1) & 1)) {
        record_error(kErrFullWaitTimeout);
        *abort_flag = 1;
      }
      tc_fence_after();
      if (!*abort_flag) {
        const uint32_t base = lane_base + buf * 256;
        int32_t d0[kPfTokPerWarp], d1[kPfTokPerWarp];
        tc_ld8(base, d0);
        tc_wait_ld();
#pragma unroll
        for (int s = 0; s < 8; s += 2) {
          tc_ld8(base + (s + 1) * 32, d1);
          scale_group(d0, i, buf, s);
          tc_wait_ld();
          if (s + 2 < 8) tc_ld8(base + (s + 2) * 32, d0);
          scale_group(d1, i, buf, s + 1);
          tc_wait_ld();
        }
      }
      tc_fence_before();
      mbar_arrive(&d_free[buf]);
    }
    // Write this thread's row for its tokens.
    for (int t = 0; t < kPfTokPerWarp; ++t) {
      const int tg = tok0 + tq * kPfTokPerWarp + t;
      if (tg >= tokens) break;
      if (partial)
        partial[(static_cast<size_t>(blockIdx.z) * tokens + tg) * rows + row0 + r] = acc[t];
      else
        out[static_cast<size_t>(tg) * rows + row0 + r] = static_cast<float>(acc[t]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPfMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols) : "memory");
  }
}

// out[t][r] = fp32(sum over splits z in order of partial[z][t][r]).
__global__ void __launch_bounds__(256) prefill_sum_kernel(const double* __restrict__ partial, int splits,
                                                          int64_t n, float* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    double s = 0.0;
    for (int z = 0; z < splits; ++z) s += partial[static_cast<size_t>(z) * n + i];
    out[i] = static_cast<float>(s);
  }
}

}  // namespace mllb
