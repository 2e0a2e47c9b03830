// Persistent streaming matvec kernels of the decode hot path (sm_100a).
//
// One HBM pass over the weights, everything else on chip:
//
// * A CTA = a loader warp, a forwarder warp and TEAMS consumer teams of W
//   warps.  The loader's lane 0 streams tiles of T weight rows HBM -> shared
//   memory with cp.async.bulk (the TMA bulk engine, L2 evict-first) through an
//   S-stage ring guarded by mbarriers (full: bytes landed; ready: re-signalled
//   in tile order by the forwarder; empty: consumed).  Tile k goes to team
//   k % TEAMS, which first decodes the tile's super-block headers once, one
//   per lane (Q4_K 6-bit scales/mins and fp16 d/dmin -> fp64; Q6_K fp16 d ->
//   fp64), so the lanes never repeat that work per unit.
// * Column-stationary lanes: a row is P = 8*NB units of 32 weights; the team
//   covers RG = 32/gcd(P,32) rows x P units with exactly W = P*RG/32 warps, so
//   every consumer lane owns ONE unit position (and row-in-group) for the
//   whole kernel and keeps that position's Q8_1 activation in registers.  Per
//   tile a lane computes V rows (its position in V row groups).
// * Lanes 2c and 2c+1 hold two halves of the same sub-block; one shuffle joins
//   their integer partial sums, after which each lane forms the fp64 terms of
//   its share (every product exact: int32 sums times fp16-derived scales).
// * Row totals: lane l visits its row groups in the order q ^ f(l), f(l) =
//   (l >> 1) & (V-1), which makes the cross-lane transpose-reduction
//   select-free (v[t] += shfl_xor(v[t + half], offset)); team partials meet in
//   shared memory and one lane per row adds them in a fixed order.  The fp64
//   row sum is therefore deterministic and exact up to ~1e-16 relative before
//   the single rounding to fp32.
// * Every mbarrier wait is bounded (~1 s, csrc/common.cuh).  A consumer warp
//   that gives up still reaches the team barrier with an abort flag set, so no
//   warp can be left waiting on a barrier.
// * PDL: the loader sends a first batch of (constant) weight tiles at once,
//   one per team; the consumers wait
//   for the preceding kernel only before reading the activation, and the CTA
//   signals launch_dependents once that activation is staged, so the next
//   kernel's prefetch cannot delay this kernel's activation read.
#pragma once

#include "common.cuh"
#include "q4k.cuh"
#include "q6k.cuh"
#include "q8_1.cuh"

namespace mllb {

// Where a streaming kernel's activation comes from: Q8_1 bytes (q8), or
// produced in the kernel from fp32 (x != nullptr): h = x + delta (fp32),
// y = gamma ? fp32(h / sqrt(mean(h^2) + eps) * gamma) : h (fp64 inside), then
// Q8_1 of y (s = d * sum q) -- what rmsnorm_q8_1 / q8_1_quantize would have
// written, built by every CTA in its own shared memory.  CTA 0 stores h to
// x_out (which must not overlap x) and, with `advance`, moves a decode state
// to its next position (the step's final norm).
struct ActSource {
  const uint8_t* q8;
  const float* x;
  const float* delta;
  const float* gamma;
  float* x_out;
  double eps;
  DecodeState* advance;
};

// Work a streaming kernel does after its rows are out, in place of a separate
// launch (each dependent launch of a decode step costs more than its own
// duration):
//  * kEpiQuantProduct (fused gate/up): the Q8_1 blocks of out2 (the SwiGLU
//    product).  counters[g] counts the stored tiles of the 32 rows of group
//    g; after its last tile each CTA arrives once per tile, and the CTA whose
//    arrival completes a group quantises it (as q8_1_quantize: s = d * sum q)
//    into q8_out and zeroes the counter.
//  * kEpiResidualNorm (a single matrix whose n_rows outputs are the delta
//    of a residual stream): h = x + out0 (fp32) -> x_out, then the Q8_1 of
//    y = fp32(h * r * gamma), r = 1 / sqrt(sum(h^2) / n_rows + eps) (fp64),
//    into q8_out -- the residual + RMSNorm + quantiser that otherwise runs
//    as a separate launch.  Each CTA sums the squares of its rows (per team,
//    in tile order), stores the sum to partials[blockIdx.x] and arrives on
//    counters[0]; once all gridDim.x CTAs have arrived (every CTA of these
//    grids is resident at once: one per SM at most), each sums the partials
//    in index order -- the same r in every CTA, run after run -- and
//    quantises the 32-row groups g = blockIdx.x, blockIdx.x + gridDim.x, ...
//    On leaving, the last CTA to depart (counters[1]) zeroes both counters.
//  * kEpiQuantProductPeer (row-sharded fused gate/up over `world` GPUs): as
//    kEpiQuantProduct, but each completed group's Q8_1 block is stored into
//    EVERY rank's buffer (peer.buffers[r], at this rank's slice: rank x
//    n_rows/32 blocks, then the group) over NVLink.  After its groups each
//    CTA arrives (release, GPU scope) on a local counter, counters[n_rows /
//    32]; the last CTA to arrive (acquiring every other CTA's release) resets
//    it, fences once at system scope and arrives on every rank's counter for
//    this rank (peer.flags[r][rank]).  CTA 0 then waits (bounded, ~1 s, then
//    kErrPeerWaitTimeout) until every rank has arrived for this gather
//    (gathers so far + 1; counters cumulative) and counts the gather -- so
//    the launch completes only when the whole product's Q8_1 is in this
//    GPU's buffer, and the next kernel's dependency wait covers it.  Every
//    rank launches the same sequence with the same shapes; plain peer stores
//    only.
// Counters must be zero before the first launch; every launch leaves them
// zero.  Launches that share counters must not overlap on the GPU.
struct Epilogue {
  uint32_t* counters;
  uint8_t* q8_out;
  const float* x;      // kEpiResidualNorm: residual stream in
  float* x_out;        //   h = x + out0 (may alias x)
  const float* gamma;  //   RMSNorm weights [n_rows]
  double* partials;    //   one per CTA of the grid
  double eps;
  PeerGather peer;     // kEpiQuantProductPeer
};
enum : int { kEpiNone = 0, kEpiQuantProduct = 1, kEpiResidualNorm = 2, kEpiQuantProductPeer = 3 };

// ============================================================== formats

// Q4_K: unit = 16 nibble bytes (halves h of groups 2j, 2j+1 of a super-block).
struct Q4kFormat {
  static constexpr int kBlockBytes = kQ4kBlockBytes;
  static constexpr int kUnitsPerBlock = 8;
  static constexpr int kDecBytes = 32;  // per super-block: fp64 d, dmin, (scale,min) x 8

  template <int NB>
  struct ActLayout {  // shared-memory activation: quants, fp64 deltas, int sums
    static constexpr int kGroups = NB * 8;
    static constexpr int kBytes = (kGroups * (32 + 8 + 4) + 15) / 16 * 16;
  };

  struct Slot {
    uint4 a_lo, a_hi;
    double delta;
    int asum;
    int raw_off, dec_off;
    int s;
  };

  template <int NB>
  __device__ static void stage_activation(const uint8_t* q8, uint8_t* act, int tid, int nthreads) {
    stage_q8_1<NB * 8>(q8, act, tid, nthreads);
  }

  // Write Q8_1 group g (quantised one value per lane) in this layout.
  template <int NB>
  __device__ static void store_group(uint8_t* act, int g, int lane, int q, uint32_t d16, uint32_t) {
    constexpr int G = NB * 8;
    const uint32_t b = static_cast<uint32_t>(q) & 0xffu;
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, b, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, b, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, b, 3);
    const int sum = warp_sum_int(q);
    if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(act + g * 32 + lane) = b | (b1 << 8) | (b2 << 16) | (b3 << 24);
    if (lane == 0) {
      reinterpret_cast<double*>(act + G * 32)[g] = half_bits_to_double(d16);
      reinterpret_cast<int*>(act + G * 40)[g] = sum;
    }
  }

  template <int NB>
  __device__ static Slot load_slot(const uint8_t* act, int p) {
    constexpr int G = NB * 8;
    Slot sl;
    const int b = p >> 3, s = p & 7, j = s >> 1, h = s & 1;
    sl.a_lo = *reinterpret_cast<const uint4*>(act + (b * 8 + 2 * j) * 32 + 16 * h);
    sl.a_hi = *reinterpret_cast<const uint4*>(act + (b * 8 + 2 * j + 1) * 32 + 16 * h);
    // High nibbles enter dp4a unshifted (16x): pre-scale delta and the sum.
    sl.delta = reinterpret_cast<const double*>(act + G * 32)[b * 8 + s] * (h ? 0.0625 : 1.0);
    sl.asum = reinterpret_cast<const int*>(act + G * 40)[b * 8 + s] << (4 * h);
    sl.raw_off = b * kBlockBytes + 16 + 16 * s;
    sl.dec_off = b * kDecBytes;
    sl.s = s;
    return sl;
  }

  __device__ static void decode(const uint8_t* raw_block, uint8_t* dec) { q4k_decode_header(raw_block, dec); }

  // fp64 contribution of this lane's unit in one row.  Must be called by all
  // 32 lanes (pair shuffle).
  __device__ static double term(const uint8_t* row_raw, const uint8_t* row_dec, const Slot& sl) {
    const uint4 wq = lds128(row_raw + sl.raw_off);
    const double2 dd = *reinterpret_cast<const double2*>(row_dec + sl.dec_off);
    const uint32_t scmn = *reinterpret_cast<const unsigned short*>(row_dec + sl.dec_off + 16 + 2 * sl.s);
    int dlo = dp4a_us(wq.x & 0x0f0f0f0fu, sl.a_lo.x, 0);
    int dhi = dp4a_us(wq.x & 0xf0f0f0f0u, sl.a_hi.x, 0);
    dlo = dp4a_us(wq.y & 0x0f0f0f0fu, sl.a_lo.y, dlo);
    dhi = dp4a_us(wq.y & 0xf0f0f0f0u, sl.a_hi.y, dhi);
    dlo = dp4a_us(wq.z & 0x0f0f0f0fu, sl.a_lo.z, dlo);
    dhi = dp4a_us(wq.z & 0xf0f0f0f0u, sl.a_hi.z, dhi);
    dlo = dp4a_us(wq.w & 0x0f0f0f0fu, sl.a_lo.w, dlo);
    dhi = dp4a_us(wq.w & 0xf0f0f0f0u, sl.a_hi.w, dhi);
    const bool h = sl.s & 1;  // keep group 2j+h; the partner holds its other 16 weights
    const int dot = (h ? dhi : dlo) + __shfl_xor_sync(0xffffffffu, h ? dlo : dhi, 1);
    const int sc = static_cast<int>(scmn & 0xffu), mn = static_cast<int>(scmn >> 8);
    return sl.delta * fma(dd.x, i2d_exact(sc * dot), -dd.y * i2d_exact(mn * sl.asum));
  }
};

// Q5_K (GGML block_q5_K, 176 B / 256 weights): fp16 d, fp16 dmin, the 12
// scale/min bytes of Q4_K, qh[32] (bit g of qh[l] is the fifth bit of element
// l of group g) and qs[128] (nibbles as Q4_K).  Unit, header decode and
// activation layout are Q4_K's; the fifth bits enter each nibble word before
// dp4a, so the dots are exact integers of the 5-bit quants.
struct Q5kFormat {
  static constexpr int kBlockBytes = 176;
  static constexpr int kUnitsPerBlock = 8;
  static constexpr int kDecBytes = 32;

  template <int NB>
  struct ActLayout : Q4kFormat::ActLayout<NB> {};

  struct Slot {
    uint4 a_lo, a_hi;
    double delta;
    int asum;
    int qs_off, qh_off, dec_off;
    int s;
  };

  template <int NB>
  __device__ static void stage_activation(const uint8_t* q8, uint8_t* act, int tid, int nthreads) {
    stage_q8_1<NB * 8>(q8, act, tid, nthreads);
  }

  template <int NB>
  __device__ static void store_group(uint8_t* act, int g, int lane, int q, uint32_t d16, uint32_t s16) {
    Q4kFormat::store_group<NB>(act, g, lane, q, d16, s16);
  }

  template <int NB>
  __device__ static Slot load_slot(const uint8_t* act, int p) {
    constexpr int G = NB * 8;
    Slot sl;
    const int b = p >> 3, s = p & 7, j = s >> 1, h = s & 1;
    sl.a_lo = *reinterpret_cast<const uint4*>(act + (b * 8 + 2 * j) * 32 + 16 * h);
    sl.a_hi = *reinterpret_cast<const uint4*>(act + (b * 8 + 2 * j + 1) * 32 + 16 * h);
    sl.delta = reinterpret_cast<const double*>(act + G * 32)[b * 8 + s];
    sl.asum = reinterpret_cast<const int*>(act + G * 40)[b * 8 + s];
    sl.qs_off = b * kBlockBytes + 48 + 16 * s;
    sl.qh_off = b * kBlockBytes + 16 + 16 * h;
    sl.dec_off = b * kDecBytes;
    sl.s = s;
    return sl;
  }

  __device__ static void decode(const uint8_t* raw_block, uint8_t* dec) { q4k_decode_header(raw_block, dec); }

  __device__ static double term(const uint8_t* row_raw, const uint8_t* row_dec, const Slot& sl) {
    const uint4 wq = lds128(row_raw + sl.qs_off);
    const uint4 wh = lds128(row_raw + sl.qh_off);
    const double2 dd = *reinterpret_cast<const double2*>(row_dec + sl.dec_off);
    const uint32_t scmn = *reinterpret_cast<const unsigned short*>(row_dec + sl.dec_off + 16 + 2 * sl.s);
    const int lo_bit = sl.s & 6, hi_bit = lo_bit + 1;  // groups 2j and 2j + 1
    const uint32_t q[4] = {wq.x, wq.y, wq.z, wq.w}, hb[4] = {wh.x, wh.y, wh.z, wh.w};
    const uint32_t al[4] = {sl.a_lo.x, sl.a_lo.y, sl.a_lo.z, sl.a_lo.w};
    const uint32_t ah[4] = {sl.a_hi.x, sl.a_hi.y, sl.a_hi.z, sl.a_hi.w};
    int dlo = 0, dhi = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t lo = (q[w] & 0x0f0f0f0fu) | (((hb[w] >> lo_bit) & 0x01010101u) << 4);
      const uint32_t hi = ((q[w] >> 4) & 0x0f0f0f0fu) | (((hb[w] >> hi_bit) & 0x01010101u) << 4);
      dlo = dp4a_us(lo, al[w], dlo);
      dhi = dp4a_us(hi, ah[w], dhi);
    }
    const bool h = sl.s & 1;  // keep group 2j+h; the partner holds its other 16 weights
    const int dot = (h ? dhi : dlo) + __shfl_xor_sync(0xffffffffu, h ? dlo : dhi, 1);
    const int sc = static_cast<int>(scmn & 0xffu), mn = static_cast<int>(scmn >> 8);
    return sl.delta * fma(dd.x, i2d_exact(sc * dot), -dd.y * i2d_exact(mn * sl.asum));
  }
};

// Q6_K: unit = one 16-column run of one half: columns [l0, l0 + 16) of the
// four Q8_1 groups 4h + k (64 weights, one scale per group); a lane finishes
// its groups alone, so no lane exchange.
struct Q6kFormat {
  static constexpr int kBlockBytes = kQ6kBlockBytes;
  static constexpr int kUnitsPerBlock = 4;
  // No header stage: a unit reads its block's fp16 d itself (one 2-byte load
  // per row), so a tile needs no decode pass and no team barrier before it.
  static constexpr int kDecBytes = 0;

  template <int NB>
  struct ActLayout {  // raw Q8_1 copy
    static constexpr int kBytes = (NB * 8 * kQ8BlockBytes + 15) / 16 * 16;
  };

  // A lane's unit in every row: its quants, group sums and deltas, and the
  // offsets of its fields from the row start (rows of an even number of
  // 210-byte blocks are whole words apart in the stage, so the offsets and
  // the shift hold for every row).
  struct Slot {
    uint32_t a[4][4];  // group 4h + k, columns l0 .. l0 + 15
    int c[4];          // -32 * sum of those quants
    double dl[4];      // the groups' Q8_1 deltas
    int lo_off;        // word holding the first ql-low byte
    int qh_off;        // word holding the first qh byte
    int sc_off;        // scale of group 4h (groups 4h + k: + 2k)
    int d_off;         // fp16 d of the block
    uint32_t sh;       // bit offset of the fields in their words: 0 or 16
  };

  template <int NB>
  __device__ static void stage_activation(const uint8_t* q8, uint8_t* act, int tid, int nthreads) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(q8);
    uint32_t* dst = reinterpret_cast<uint32_t*>(act);
    for (int i = tid; i < NB * 8 * kQ8BlockBytes / 4; i += nthreads) dst[i] = __ldg(src + i);
  }

  template <int NB>
  __device__ static void store_group(uint8_t* act, int g, int lane, int q, uint32_t d16, uint32_t s16) {
    q8_1_store_block(act + g * kQ8BlockBytes, q, d16, s16, lane);
  }

  template <int NB>
  __device__ static Slot load_slot(const uint8_t* act, int p) {
    static_assert(NB % 2 == 0, "rows must be whole words apart in the stage");
    Slot sl;
    const int b = p >> 2, u = p & 3;
    const int h = u >> 1, l0 = (u & 1) * 16;
    const int blk_off = b * kBlockBytes;
    sl.lo_off = (blk_off + 64 * h + l0) & ~3;
    sl.qh_off = (blk_off + 128 + 32 * h + l0) & ~3;
    sl.sc_off = blk_off + 192 + 8 * h + (l0 >> 4);
    sl.d_off = blk_off + 208;
    sl.sh = (blk_off & 2) ? 16u : 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint8_t* g = act + (b * 8 + 4 * h + k) * kQ8BlockBytes;
      int sum = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sl.a[k][i] = lds32(g + 4 + l0 + 4 * i);
        sum = byte_sum_s8(sl.a[k][i], sum);
      }
      sl.c[k] = -32 * sum;
      sl.dl[k] = half_bits_to_double(lds32(g) & 0xffffu);
    }
    return sl;
  }

  __device__ static void decode(const uint8_t*, uint8_t*) {}

  __device__ static double term(const uint8_t* row_raw, const uint8_t*, const Slot& sl) {
    int u[4];
    q6k_run_dots(row_raw + sl.lo_off, row_raw + sl.qh_off, sl.sh, sl.a, sl.c, u);
    const int8_t* sc = reinterpret_cast<const int8_t*>(row_raw + sl.sc_off);
    // Each group's integer sum times its scale is exact in int32 (|.| < 2^24)
    // and in fp64; the four products, then d, each take one fp64 rounding.
    double t = static_cast<double>(static_cast<int>(sc[0]) * u[0]) * sl.dl[0];
#pragma unroll
    for (int k = 1; k < 4; ++k) t = fma(static_cast<double>(static_cast<int>(sc[2 * k]) * u[k]), sl.dl[k], t);
    const double d = half_bits_to_double(*reinterpret_cast<const unsigned short*>(row_raw + sl.d_off));
    return d * t;
  }
};

// ============================================================== producer

// Build the activation of an ActSource with x != nullptr in shared memory,
// by the `nthreads` consumer threads (warp-aligned; named barrier 1).
// `red` holds one double per consumer warp.  Loads are issued in batches
// before their first use: each is an L2 round trip.
template <class Fmt, int NB, int NTHREADS>
__device__ __forceinline__ void produce_activation(const ActSource& src, uint8_t* act, double* red, int tid) {
  constexpr int K = NB * 256, G = NB * 8, NW = NTHREADS / 32;
  constexpr int kPer = (G + NW - 1) / NW;   // Q8_1 groups per warp
  constexpr int kBatch = 8;
  const int lane = tid & 31, warp = tid >> 5;
  double r = 1.0;
  if (src.gamma) {
    double ss = 0.0;
    for (int base = tid; base < K; base += kBatch * NTHREADS) {
      float xv[kBatch], dv[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = base + u * NTHREADS;
        xv[u] = i < K ? src.x[i] : 0.0f;
        dv[u] = (src.delta && i < K) ? src.delta[i] : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const float h = src.delta ? xv[u] + dv[u] : xv[u];
        ss = fma(static_cast<double>(h), static_cast<double>(h), ss);
      }
    }
    ss = warp_sum_double(ss);
    if (lane == 0) red[warp] = ss;
    named_barrier(1, NTHREADS);
    double total = 0.0;
#pragma unroll 4
    for (int w = 0; w < NW; ++w) total += red[w];
    r = 1.0 / sqrt(total / static_cast<double>(K) + src.eps);
  }
  float hv[kPer], gv[kPer];
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int g = warp + u * NW;
    const int i = g * 32 + lane;
    float h = 0.0f, gm = 1.0f;
    if (g < G) {
      h = src.x[i];
      if (src.delta) h += src.delta[i];
      if (src.gamma) gm = src.gamma[i];
    }
    hv[u] = h;
    gv[u] = gm;
  }
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int g = warp + u * NW;
    if (g < G) {
      if (src.x_out && blockIdx.x == 0) src.x_out[g * 32 + lane] = hv[u];
      const float y = src.gamma ? static_cast<float>(static_cast<double>(hv[u]) * r * static_cast<double>(gv[u]))
                                : hv[u];
      uint32_t d16, s16;
      const int q = q8_1_quantize_lane(y, kQ8SumDTimesSumQ, &d16, &s16);
      Fmt::template store_group<NB>(act, g, lane, q, d16, s16);
    }
  }
  if (src.advance && blockIdx.x == 0 && tid == 0) {
    src.advance->next_token_key = kNoToken;
    src.advance->pos += 1;
    src.advance->steps += 1;
  }
}

// ============================================================== geometry

template <class Fmt, int NB, int MATS, int V, int S, int TEAMS>
struct TeamConfig {
  static constexpr int kP = NB * Fmt::kUnitsPerBlock;        // units per row
  static constexpr int kRG = 32 / gcd_constexpr(kP, 32);     // rows per row group
  static constexpr int kW = kP * kRG / 32;                   // consumer warps per team
  static constexpr int kConsumers = TEAMS * kW * 32;
  static constexpr int kThreads = kConsumers + 64;  // + loader warp + decoder warp
  static constexpr int kT = V * kRG;                         // rows per tile
  static constexpr int kRowBytes = NB * Fmt::kBlockBytes;
  static constexpr int kTileBytes = kT * kRowBytes;          // per matrix
  static constexpr int kStageBytes = kTileBytes * MATS;
  static constexpr int kDecTile = MATS * kT * NB * Fmt::kDecBytes;  // decoded headers of one tile
  // Lanes per partial segment: a half-warp, or 8 lanes when rows do not
  // start on half-warps (the V = 4 reduction then stops after lane bit 2).
  static constexpr int kSegLanes = kP % 16 == 0 ? 16 : 8;
  static constexpr int kSegs = (32 / kSegLanes) * kW;        // partial segments per team
  static constexpr int kTeamPartials = 2 * MATS * kT * kSegs;  // doubles, double-buffered
  static constexpr int kDecOffset = S * kStageBytes;                 // one decode buffer per team
  static constexpr int kActOffset = kDecOffset + TEAMS * kDecTile;
  static constexpr int kPartOffset = kActOffset + Fmt::template ActLayout<NB>::kBytes;
  static constexpr int kBarOffset = kPartOffset + TEAMS * kTeamPartials * 8;
  static constexpr int kAbortOffset = kBarOffset + (3 * S + 1) * 8;
  static constexpr int kRedOffset = kAbortOffset + 16;               // producer: one double per consumer warp
  static constexpr int kSmemBytes = kRedOffset + (kConsumers / 32) * 8;
  // Two resident CTAs (this kernel + the next of a stream) when the ring is
  // small enough; deep rings take the whole SM.
  static constexpr int kMinBlocks = kSmemBytes <= 112 * 1024 ? 2 : 1;
  static_assert(kStageBytes % 16 == 0 && kTileBytes % 16 == 0, "TMA tiles must be whole 16-byte runs");
  static_assert(V == 4 || V == 8, "row groups per tile");
  static_assert(kP % 8 == 0 && (kSegLanes == 16 || V == 4), "rows start on 8-lane segments; V = 8 needs 16");
  static_assert(kT <= 32, "one lane per row in the final combine");
  static_assert(kThreads <= 1024 && TEAMS + 1 < 16, "CTA size / named barriers");
  // A team waits on the ready barrier of tile k only after its previous tile
  // k - TEAMS, so with TEAMS <= S the barrier is never more than one phase
  // behind and the parity wait is unambiguous.  With TEAMS > S a wait could
  // pass on a stale phase and corrupt the stage accounting.
  static_assert(TEAMS <= S, "more consumer teams than pipeline stages");
};

// ============================================================== kernel
// out0 = first matrix, out1 = second (DUAL), out2 = out0 * silu(out1) (DUAL).
// Tile k of a CTA (global tile blockIdx.x + k*gridDim.x) goes to team k % TEAMS;
// the teams of a CTA share one producer and stage ring, so an SM's teams take
// their work from one queue.  pdl: launched with programmatic serialisation --
// the producer sends one tile per team (at least two) at once; otherwise one
// tile.  It holds the rest until the activation is staged so that the
// activation read does not queue behind a flood of weight requests.
// PRODUCE: the activation is built in the kernel from fp32 (ActSource.x);
// otherwise it is staged from Q8_1 bytes.  A separate instantiation, so the
// plain kernels carry none of the producer's registers.
template <class Fmt, int NB, int MATS, int V, int S, int TEAMS, bool PRODUCE = false, int EPI = kEpiNone>
__global__ void __launch_bounds__(TeamConfig<Fmt, NB, MATS, V, S, TEAMS>::kThreads,
                                  TeamConfig<Fmt, NB, MATS, V, S, TEAMS>::kMinBlocks)
    team_stream_kernel(const uint8_t* __restrict__ w0, const uint8_t* __restrict__ w1, const ActSource src,
                       float* __restrict__ out0, float* __restrict__ out1, float* __restrict__ out2, int n_rows,
                       int pdl, const Epilogue epi) {
  using C = TeamConfig<Fmt, NB, MATS, V, S, TEAMS>;
  constexpr bool kQuantTail = EPI == kEpiQuantProduct || EPI == kEpiQuantProductPeer;
  static_assert(!kQuantTail || (MATS == 2 && 32 % C::kT == 0), "product groups of whole tiles");
  static_assert(EPI != kEpiResidualNorm || MATS == 1, "the residual norm follows a single matrix");
  constexpr int W = C::kW, RG = C::kRG, T = C::kT, P = C::kP, ROWB = C::kRowBytes;
  constexpr int kFirstBatch = TEAMS > 2 ? TEAMS : 2;
  constexpr int DECB = Fmt::kDecBytes;

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* act = smem + C::kActOffset;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* ready = full + S;
  uint64_t* empty = ready + S;
  uint64_t* act_ready = empty + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kAbortOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntiles = (n_rows + T - 1) / T;
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 1);
      mbar_init(&empty[s], W);
    }
    mbar_init(act_ready, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __shared__ double s_norm_ss[EPI == kEpiResidualNorm ? TEAMS : 1];  // kEpiResidualNorm: each team's sum of h^2
  {
    double* partials = reinterpret_cast<double*>(smem + C::kPartOffset);
    for (int i = threadIdx.x; i < TEAMS * C::kTeamPartials; i += blockDim.x) partials[i] = 0.0;
    if (EPI == kEpiResidualNorm && threadIdx.x < TEAMS) s_norm_ss[threadIdx.x] = 0.0;
  }
  __syncthreads();
  MLLB_TRACE_POINT(0);

  if (warp == TEAMS * W) {
    // ================================================= loader warp (lane 0)
    // Prefetch the first batch (under PDL; one tile otherwise), then hold further
    // requests until the teams have their activation: the activation read
    // must not queue behind weight traffic.  Only then may the next kernel of
    // the stream start and send its own prefetch.
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      auto issue = [&](int k) {
        const int s = k % S;
        const int tile = blockIdx.x + k * gridDim.x;
        const int rows = min(T, n_rows - tile * T);
        const uint32_t bytes = static_cast<uint32_t>(rows * ROWB);
        const size_t goff = static_cast<size_t>(tile) * T * ROWB;
        mbar_arrive_expect_tx(&full[s], MATS * bytes);
        bulk_copy_g2s(smem + s * C::kStageBytes, w0 + goff, bytes, &full[s], policy);
        if (MATS == 2) bulk_copy_g2s(smem + s * C::kStageBytes + C::kTileBytes, w1 + goff, bytes, &full[s], policy);
      };
      int k = 0;
      // Under PDL the first batch is one tile per team (at least two): the
      // rest of the ring fills once the activation is staged, so the
      // activation read does not queue behind the whole ring's weight
      // requests, and a deeper ring then keeps each team's next tile in
      // flight (gate/up 2 x 9728 x 2560, ring of 6 for 3 teams: 7.79 vs 8.26 us).
      const int first_batch = pdl ? (S < kFirstBatch ? S : kFirstBatch) : 1;
      for (; k < first_batch && k < my_tiles; ++k) issue(k);
      bool ok = mbar_wait_bounded(act_ready, 0);
      if (!ok) record_error(kErrEmptyWaitTimeout);
      pdl_launch_dependents();
      for (; ok && k < my_tiles; ++k) {
        if (k >= S && !mbar_wait_bounded(&empty[k % S], ((k / S) - 1) & 1)) {
          record_error(kErrEmptyWaitTimeout);
          break;
        }
        issue(k);
      }
      // Never leave with copies in flight (normally all consumed already).
      for (int u = k - 1; u >= 0 && u >= k - S; --u) {
        if (!mbar_wait_bounded(&full[u % S], (u / S) & 1)) {
          record_error(kErrDrainTimeout);
          break;
        }
      }
    }
    return;
  }
  if (warp == TEAMS * W + 1) {
    // ================================================= forwarder warp
    // Observes the tiles landing strictly in order and re-signals each on
    // `ready`.  Teams wait on `ready`, never on `full` directly: a team's
    // previous tile is k - TEAMS, which says nothing about whether tile k - S
    // (the previous user of the stage) has landed, while the forwarder only
    // waits for tile k after tile k - 1, so every parity wait here and in the
    // teams is at most one phase ahead.
    if (lane == 0) {
      for (int k = 0; k < my_tiles; ++k) {
        const int s = k % S;
        if (!mbar_wait_bounded(&full[s], (k / S) & 1)) {
          record_error(kErrFullWaitTimeout);
          break;
        }
        mbar_arrive(&ready[s]);
      }
    }
    return;
  }

  // =================================================== consumer teams
  const int team = warp / W;
  const int twarp = warp % W;  // warp index inside the team
  pdl_wait_prerequisite();     // the activation may come from the preceding kernel
  MLLB_TRACE_POINT(1);
  if constexpr (PRODUCE)
    produce_activation<Fmt, NB, C::kConsumers>(src, act, reinterpret_cast<double*>(smem + C::kRedOffset),
                                               threadIdx.x);
  else
    Fmt::template stage_activation<NB>(src.q8, act, threadIdx.x, C::kConsumers);
  named_barrier(1, C::kConsumers);
  if (threadIdx.x == 0) mbar_arrive(act_ready);
  pdl_launch_dependents();  // with the loader's: the CTA triggers once staged
  MLLB_TRACE_POINT(2);

  const int vp = twarp * 32 + lane;
  const int r_in_group = vp / P;
  const typename Fmt::Slot slot = Fmt::template load_slot<NB>(act, vp % P);
  const int f = (lane >> 1) & (V - 1);  // row-group visiting order
  // Half-warps with the same row-in-group are combined before the partials
  // (16-lane segments; with 8-lane segments each keeps its own partial).
  constexpr int SL = C::kSegLanes;
  const bool merge_halves = SL == 16 && (twarp * 32) / P == (twarp * 32 + 16) / P;
  const int seg = SL == 16 ? 2 * twarp + (merge_halves ? 0 : (lane >> 4)) : 4 * twarp + (lane >> 3);
  // One lane per (row, segment) writes: bit 0 and the lane bits outside f(l)
  // must be zero; bit 4 selects the half unless the halves were merged.
  const bool writer = SL == 16 ? (lane & 1) == 0 && (lane & (0x0e & ~((V - 1) << 1))) == 0 &&
                                     (!merge_halves || lane < 16)
                               : (lane & 1) == 0;
  double* partials = reinterpret_cast<double*>(smem + C::kPartOffset) + team * C::kTeamPartials;
  uint8_t* dec = smem + C::kDecOffset + team * C::kDecTile;
  const int team_barrier = 2 + team;

  for (int k = team; k < my_tiles; k += TEAMS) {
    const int s = k % S;
    const int tile = blockIdx.x + k * gridDim.x;
    const bool have = mbar_wait_bounded(&ready[s], (k / S) & 1);
    if (!have) {
      record_error(kErrFullWaitTimeout);
      *abort_flag = 1;
    }
    if (k < 2) MLLB_TRACE_POINT(3 + 2 * k);
    const int parity = (k / TEAMS) & 1;
    double* part = partials + parity * (MATS * T * C::kSegs);
    const uint8_t* stage = smem + s * C::kStageBytes;
    if constexpr (DECB > 0) {
      if (have) {
        // The team decodes this tile's super-block headers (about one per lane).
        const int rows = min(T, n_rows - tile * T);
        for (int e = vp; e < MATS * T * NB; e += W * 32) {
          const int m = e / (T * NB), rest = e % (T * NB), row = rest / NB, b = rest % NB;
          if (row < rows) Fmt::decode(stage + m * C::kTileBytes + row * ROWB + b * Fmt::kBlockBytes, dec + e * DECB);
        }
      }
      named_barrier(team_barrier, W * 32);
    }
    if (have) {
      double v[MATS][V];
#pragma unroll
      for (int q = 0; q < V; ++q) {
        const int row = (q ^ f) * RG + r_in_group;  // tile row visited at step q
#pragma unroll
        for (int m = 0; m < MATS; ++m)
          v[m][q] = Fmt::term(stage + m * C::kTileBytes + row * ROWB, dec + (m * T + row) * NB * DECB, slot);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (k < 2) MLLB_TRACE_POINT(4 + 2 * k);
#pragma unroll
      for (int m = 0; m < MATS; ++m) {
        // select-free transpose reduction over lane bits log2(V)..1
#pragma unroll
        for (int half = V / 2, off = V; half >= 1; half >>= 1, off >>= 1)
#pragma unroll
          for (int t = 0; t < half; ++t) v[m][t] += __shfl_xor_sync(0xffffffffu, v[m][t + half], off);
        double x = v[m][0];
        x += __shfl_xor_sync(0xffffffffu, x, 1);
        if (V == 4 && SL == 16) x += __shfl_xor_sync(0xffffffffu, x, 8);
        if (merge_halves) x += __shfl_xor_sync(0xffffffffu, x, 16);
        if (writer) part[(m * T + f * RG + r_in_group) * C::kSegs + seg] = x;
      }
    }
    named_barrier(team_barrier, W * 32);
    if (*abort_flag) break;
    // The warp that adds the tile's partials: warp 0 when a header pass
    // follows (it overlaps the others' decoding of the next tile); otherwise
    // each warp in turn, so no warp lags the team by every tile's sum.
    if (twarp == (DECB > 0 ? 0 : (k / TEAMS) % W)) {
      double sq = 0.0;  // kEpiResidualNorm: h^2 of this lane's row
      if (lane < T) {
        const int row = tile * T + lane;
        double tot[MATS];
#pragma unroll
        for (int m = 0; m < MATS; ++m) {
          double acc = 0.0;
#pragma unroll
          for (int g = 0; g < C::kSegs; ++g) acc += part[(m * T + lane) * C::kSegs + g];
          tot[m] = acc;
        }
        if (row < n_rows) {
          if (out0) out0[row] = static_cast<float>(tot[0]);
          if (MATS == 2) {
            if (out1) out1[row] = static_cast<float>(tot[MATS - 1]);
            if (out2) out2[row] = static_cast<float>(tot[0] * (tot[MATS - 1] / (1.0 + exp(-tot[MATS - 1]))));
          }
          if constexpr (EPI == kEpiResidualNorm) {
            const float h = epi.x[row] + static_cast<float>(tot[0]);
            epi.x_out[row] = h;
            sq = static_cast<double>(h) * static_cast<double>(h);
          }
        }
      }
      if constexpr (EPI == kEpiResidualNorm) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
        if (lane == 0) s_norm_ss[team] += sq;
      }
    }
  }
  MLLB_TRACE_POINT(7);
  if constexpr (EPI == kEpiResidualNorm) {
    __shared__ int s_all_arrived;
    const int tid = threadIdx.x;
    const int g0 = blockIdx.x;  // this CTA's first 32-row group
    const bool has_group = g0 < n_rows / 32;
    const float gamma0 = (tid < 32 && has_group) ? epi.gamma[g0 * 32 + lane] : 0.0f;
    __threadfence();  // this CTA's x_out rows before its arrival
    named_barrier(1, C::kConsumers);
    if (tid == 0) {
      double cta = 0.0;
#pragma unroll
      for (int t = 0; t < TEAMS; ++t) cta += s_norm_ss[t];
      epi.partials[blockIdx.x] = cta;
      __threadfence();
      atom_add_release_gpu(&epi.counters[0], 1u);
      const bool ok = wait_count_bounded(&epi.counters[0], gridDim.x);
      if (!ok) record_error(kErrGridWaitTimeout);
      s_all_arrived = ok;
    }
    named_barrier(1, C::kConsumers);
    if (s_all_arrived && tid < 32) {
      // The first group's h is loaded with the partials: one L2 round trip.
      const float h0 = has_group ? ld_cg_f32(epi.x_out + g0 * 32 + lane) : 0.0f;
      double ss = 0.0;
      for (int i = lane; i < static_cast<int>(gridDim.x); i += 32) ss += ld_cg_f64(epi.partials + i);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const double r = 1.0 / sqrt(ss / static_cast<double>(n_rows) + epi.eps);
      for (int g = g0; g < n_rows / 32; g += gridDim.x) {
        const int i = g * 32 + lane;
        const float h = g == g0 ? h0 : ld_cg_f32(epi.x_out + i);
        const float gm = g == g0 ? gamma0 : epi.gamma[i];
        const float y = static_cast<float>(static_cast<double>(h) * r * static_cast<double>(gm));
        uint32_t d16, s16;
        const int q = q8_1_quantize_lane(y, kQ8SumDTimesSumQ, &d16, &s16);
        q8_1_store_block(epi.q8_out + static_cast<size_t>(g) * kQ8BlockBytes, q, d16, s16, lane);
      }
    }
    // Every CTA has passed the wait once the last one departs: it resets both.
    if (tid == 0 && atomicAdd(&epi.counters[1], 1u) == gridDim.x - 1) {
      epi.counters[0] = 0u;
      epi.counters[1] = 0u;
    }
  }
  if constexpr (kQuantTail) {
    // One arrival per stored tile, then the groups this CTA completed.
    __shared__ uint32_t s_done[32];
    __shared__ int s_ndone;
    __threadfence();  // this CTA's out2 rows before its arrivals
    named_barrier(1, C::kConsumers);
    if (threadIdx.x == 0) s_ndone = 0;
    named_barrier(1, C::kConsumers);
    const int tid = threadIdx.x;
    for (int k0 = 0; k0 < my_tiles; k0 += 32) {
      if (tid < 32 && k0 + tid < my_tiles) {
        const int g = (blockIdx.x + (k0 + tid) * gridDim.x) * T / 32;
        if (atomicAdd(&epi.counters[g], 1u) == 32 / T - 1) s_done[atomicAdd(&s_ndone, 1)] = g;
      }
      named_barrier(1, C::kConsumers);
      const int nd = s_ndone;
      if (nd > 0) {
        __threadfence();
        for (int i = tid >> 5; i < nd; i += C::kConsumers / 32) {
          const int g = s_done[i];
          uint32_t d16, s16;
          const int q = q8_1_quantize_lane(ld_cg_f32(out2 + g * 32 + lane), kQ8SumDTimesSumQ, &d16, &s16);
          if constexpr (EPI == kEpiQuantProductPeer) {
            const size_t off = (static_cast<size_t>(epi.peer.rank) * (n_rows / 32) + g) * kQ8BlockBytes;
            for (int r = 0; r < epi.peer.world; ++r) q8_1_store_block(epi.peer.buffers[r] + off, q, d16, s16, lane);
          } else {
            q8_1_store_block(epi.q8_out + static_cast<size_t>(g) * kQ8BlockBytes, q, d16, s16, lane);
          }
          if (lane == 0) epi.counters[g] = 0;
        }
      }
      named_barrier(1, C::kConsumers);
      if (tid == 0) s_ndone = 0;
      named_barrier(1, C::kConsumers);
    }
    if constexpr (EPI == kEpiQuantProductPeer) {
      // The barrier above orders this CTA's peer stores before thread 0's
      // release; the last CTA's acquire + system-scope fence carries every
      // CTA's stores ahead of its arrivals on the ranks' counters.
      if (tid == 0) {
        const PeerGather& pg = epi.peer;
        uint32_t* arrived = epi.counters + n_rows / 32;
        if (atom_add_acq_rel_gpu(arrived, 1u) == gridDim.x - 1) {
          *arrived = 0u;
          fence_sys();
          for (int r = 0; r < pg.world; ++r) red_relaxed_sys_add(pg.flags[r] + pg.rank, 1u);
        }
        if (blockIdx.x == 0) {
          const uint32_t target = *pg.count + 1u;
          const uint32_t* mine = pg.flags[pg.rank];
          const uint64_t start = global_timer_ns();
          bool ok = true;
          for (int src = 0; src < pg.world && ok; ++src) {
            for (uint32_t i = 0;; ++i) {
              if (static_cast<int32_t>(ld_volatile_u32(mine + src) - target) >= 0) break;
              if (((i & 255u) == 255u && global_timer_ns() - start > kWaitLimitNs) || i >= kWaitMaxIters) {
                ok = false;
                break;
              }
            }
          }
          fence_sys();  // the peers' blocks are visible before this launch completes
          if (!ok) record_error(kErrPeerWaitTimeout);
          *pg.count += 1u;
        }
      }
    }
  }
}

}  // namespace mllb
