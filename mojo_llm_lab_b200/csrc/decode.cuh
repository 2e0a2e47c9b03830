// Kernels of one single-token decode step around the matvecs of a
// Qwen3-style stack (embedding -> 36 x [norm, QKV, q/k norm + IMROPE + KV
// append, attention, O, residual + norm, gate/up, down] -> norm -> Q6_K
// logits -> greedy argmax):
//
//   embed_q6k_kernel        token row of the tied Q6_K output matrix -> fp32
//   rmsnorm_q8_1_kernel     h = x + delta (fp32); y = h * r * gamma -> Q8_1
//   qk_rope_append_kernel   per-head RMSNorm + gamma + IMROPE of the Q and K
//                           heads; K and V appended to the fp16 cache
//   kv_q4_0_store_kernel    fp32 K/V rows -> the Q4_0 cache (GGML rule)
//   attn_split_kernel<G,KV> one (KV head, context chunk) per CTA: scores,
//                           chunk softmax, P.V partials; fp16 or Q4_0 cache
//   attn_combine_kernel     merge the chunk partials -> fp32 -> Q8_1
//   argmax_kernel           greedy next token as a packed (value, index) key
//
// The reference decodes through llama.cpp, with the same chain of GGML ops
// around its kernels (integration/resident_decode.cpp, the profile of
// docs/decode-profile.md:5-11); the matvecs and the RMSNorm + IMROPE op are
// its kernels, the rest are the GGML ops of that graph.
//
// Numerics.  Values crossing a kernel boundary are fp32 (fp16 in the KV
// cache, Q8_1 as matvec inputs).  Inside a kernel everything is fp64 and is
// rounded once at the boundary, so each boundary value is the correctly
// rounded result up to ~1e-16 relative, and a float64 restatement of the
// step reproduces it bit for bit except in (rare) rounding ties.  That is
// what keeps the Q8_1 re-quantisation inside every layer from amplifying
// last-bit differences over 36 layers.  In the attention the fp16 cache
// values enter fp64 through an exact bit move (value x 2^-1008, see
// half_bits_scaled) instead of two conversions per element, and the queries
// and softmax weights carry the compensating 2^1008.
#pragma once

#include "common.cuh"
#include "imrope.cuh"
#include "q8_1.cuh"

namespace mllb {

constexpr int kQ6kBytes = 210;

// Order-preserving key: larger value first, then the lower index.  The high
// word is the fp32 value mapped to a signed integer of the same order (NaN
// sorts above +inf); the low word is 0xffffffff - index.
__device__ __forceinline__ long long argmax_key(float v, uint32_t index) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t hi = (u & 0x80000000u) ? (u ^ 0x7fffffffu) : u;
  return static_cast<long long>((static_cast<unsigned long long>(hi) << 32) | (0xffffffffu - index));
}

__device__ __forceinline__ uint32_t argmax_key_index(long long key) {
  return 0xffffffffu - static_cast<uint32_t>(static_cast<unsigned long long>(key) & 0xffffffffull);
}

__device__ __forceinline__ long long warp_max_ll(long long v) {
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) {
    const long long o = __shfl_xor_sync(0xffffffffu, v, offset);
    v = o > v ? o : v;
  }
  return v;
}

__device__ __forceinline__ double warp_max_double(double v) {
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, offset));
  return v;
}

// ------------------------------------------------------------ embedding

// hidden[i] = fp32(d * scale * (q6 - 32)) of row `token` of the Q6_K matrix
// (the output projection, tied to the embedding).  The token comes from the
// state's next-token key; a key outside [0, vocab) raises kErrBadToken and
// embeds row 0.  Block 0 records the token (state->token and, if given,
// tokens[state->steps]).
__global__ void __launch_bounds__(256) embed_q6k_kernel(const uint8_t* __restrict__ w, int nb, int64_t vocab,
                                                        DecodeState* state, int32_t* tokens, int64_t capacity,
                                                        float* __restrict__ out) {
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const long long key = state->next_token_key;
  uint32_t token = argmax_key_index(key);
  const bool bad = key == kNoToken || token >= static_cast<uint64_t>(vocab);
  if (bad) token = 0;
  const uint8_t* row = w + static_cast<size_t>(token) * nb * kQ6kBytes;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nb * 256; i += gridDim.x * blockDim.x) {
    const uint8_t* blk = row + (i >> 8) * kQ6kBytes;
    const int e = i & 255, h = e >> 7, quad = (e >> 5) & 3, l = e & 31;
    const uint32_t lo = (blk[64 * h + l + 32 * (quad & 1)] >> (4 * (quad >> 1))) & 15u;
    const uint32_t hi = (blk[128 + 32 * h + l] >> (2 * quad)) & 3u;
    const int scale = static_cast<int8_t>(blk[192 + 8 * h + (l >> 4) + 2 * quad]);
    const double d = half_bits_to_double(blk[208] | (blk[209] << 8));
    out[i] = static_cast<float>(d * static_cast<double>(scale) * static_cast<double>(static_cast<int>(lo | (hi << 4)) - 32));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (bad) record_error(kErrBadToken);
    state->token = static_cast<int>(token);
    const int step = state->steps;
    if (tokens && step >= 0 && step < capacity) tokens[step] = static_cast<int32_t>(token);
  }
}

// ------------------------------------------------ residual + RMSNorm -> Q8_1

// h = x (+ delta) in fp32, written to x_out when given; r = 1 / sqrt(sum(h^2)
// / k + eps) in fp64; y = fp32(h * r * gamma); Q8_1 of y.  Every CTA sums
// the squares of all k values itself (the same order in each, so the same r)
// and quantises the Q8_1 blocks b = blockIdx.x + i * gridDim.x..., one per
// warp, storing their h to x_out.  x_out may alias x only with one CTA.
// With `advance` (the step's final norm) CTA 0 also resets the next-token
// key and moves the state to the next position.
__global__ void __launch_bounds__(256) rmsnorm_q8_1_kernel(const float* x, const float* __restrict__ delta,
                                                           float* x_out, const float* __restrict__ gamma,
                                                           double eps, uint8_t* __restrict__ q8, int k, int s_mode,
                                                           DecodeState* advance) {
  __shared__ double partial[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  // gamma is a weight: this warp's first block's value is read before the
  // dependency wait.
  const int b0 = blockIdx.x * warps + warp;
  const float gamma0 = b0 < k / 32 ? __ldg(gamma + b0 * 32 + lane) : 0.0f;
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  // Loads in batches of 16 per thread, all issued before their first use:
  // one round trip to L2 for k <= 4096 with 256 threads.  Thread t's batch
  // holds elements t + 256 u; block b = blockIdx.x * warps + warp, which its
  // warp quantises below, is element blockIdx.x * 256 + t, i.e. u =
  // blockIdx.x: with a single batch (k <= 16 * blockDim) and blockDim = 256
  // that h is kept rather than read again after the reduction.
  constexpr int kBatch = 16;
  double ss = 0.0;
  float h_mine = 0.0f;
  const bool single = k <= kBatch * static_cast<int>(blockDim.x) && blockDim.x == 256;
  for (int base = threadIdx.x; base < k; base += kBatch * blockDim.x) {
    float xv[kBatch], dv[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * blockDim.x;
      xv[u] = i < k ? x[i] : 0.0f;
      dv[u] = (delta && i < k) ? delta[i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const float h = delta ? xv[u] + dv[u] : xv[u];
      ss = fma(static_cast<double>(h), static_cast<double>(h), ss);
      if (u == static_cast<int>(blockIdx.x)) h_mine = h;
    }
  }
  ss = warp_sum_double(ss);
  if (lane == 0) partial[warp] = ss;
  __syncthreads();
  double total = lane < warps ? partial[lane] : 0.0;
  total = warp_sum_double(total);
  const double r = 1.0 / sqrt(total / static_cast<double>(k) + eps);
  // Every thread has read all of x above; only then may an aliasing x_out
  // (single CTA) be written.
  __syncthreads();
  for (int b = b0; b < k / 32; b += gridDim.x * warps) {
    const int i = b * 32 + lane;
    float h;
    if (single && b == b0) {
      h = h_mine;
    } else {
      h = x[i];
      if (delta) h += delta[i];
    }
    if (x_out) x_out[i] = h;
    const float g = b == b0 ? gamma0 : gamma[i];
    const float y = static_cast<float>(static_cast<double>(h) * r * static_cast<double>(g));
    uint32_t d16, s16;
    const int q = q8_1_quantize_lane(y, s_mode, &d16, &s16);
    q8_1_store_block(q8 + static_cast<size_t>(b) * 36, q, d16, s16, lane);
  }
  if (advance && blockIdx.x == 0 && threadIdx.x == 0) {
    advance->next_token_key = kNoToken;
    advance->pos += 1;
    advance->steps += 1;
  }
}

// ------------------------------------ q/k RMSNorm + IMROPE, KV cache append

// One warp per head of the fused QKV projection output (q heads, then k
// heads, then v heads, 128 values each).  Q heads: RMSNorm + q_gamma +
// IMROPE -> q_out (fp32).  K heads: RMSNorm + k_gamma + IMROPE, rounded to
// fp32 and then to fp16 at row `pos` of the cache.  V heads: fp16 of the
// projection at row `pos`.  The four IMROPE axis positions of a text token
// are (pos, pos, pos, 0), the same for every head, so each CTA first builds
// the 64 (cos, sin) pairs once (one fp64 pow + sincos per thread).  pos
// outside [0, ctx) raises kErrKvOverflow and appends nothing.  Cache layout:
// [kv_head][ctx][128] fp16.
__global__ void __launch_bounds__(128) qk_rope_append_kernel(const float* __restrict__ qkv,
                                                             const float* __restrict__ q_gamma,
                                                             const float* __restrict__ k_gamma,
                                                             const DecodeState* __restrict__ state, double theta,
                                                             float* __restrict__ q_out, __half* __restrict__ k_cache,
                                                             __half* __restrict__ v_cache, int hq, int hkv, int ctx) {
  __shared__ double2 rot[kHeadDim / 2];
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int pos = state->pos;
  if (threadIdx.x < kHeadDim / 2) rot[threadIdx.x] = imrope_rotation(threadIdx.x, pos, pos, pos, 0, theta);
  __syncthreads();
  if (w >= hq + 2 * hkv) return;
  double o[4];
  if (w < hq) {
    imrope_head_table(qkv + static_cast<size_t>(w) * kHeadDim, q_gamma, rot, lane, o);
    float* dst = q_out + static_cast<size_t>(w) * kHeadDim;
    dst[lane] = static_cast<float>(o[0]);
    dst[lane + 64] = static_cast<float>(o[1]);
    dst[lane + 32] = static_cast<float>(o[2]);
    dst[lane + 96] = static_cast<float>(o[3]);
    return;
  }
  if (pos < 0 || pos >= ctx) {
    if (lane == 0) record_error(kErrKvOverflow);
    return;
  }
  const int j = w < hq + hkv ? w - hq : w - hq - hkv;
  const size_t row = (static_cast<size_t>(j) * ctx + pos) * kHeadDim;
  if (w < hq + hkv) {
    imrope_head_table(qkv + static_cast<size_t>(w) * kHeadDim, k_gamma, rot, lane, o);
    k_cache[row + lane] = __float2half_rn(static_cast<float>(o[0]));
    k_cache[row + lane + 64] = __float2half_rn(static_cast<float>(o[1]));
    k_cache[row + lane + 32] = __float2half_rn(static_cast<float>(o[2]));
    k_cache[row + lane + 96] = __float2half_rn(static_cast<float>(o[3]));
  } else {
    const float* src = qkv + static_cast<size_t>(w) * kHeadDim;
#pragma unroll
    for (int i = 0; i < 4; ++i) v_cache[row + lane + 32 * i] = __float2half_rn(src[lane + 32 * i]);
  }
}

// --------------------------------------------------------- Q4_0 KV cache

// The Q4_0 cache (GGML's Q4_0 block: fp16 d and 32 4-bit q, value
// d * (q - 8); the KV type the reference's llama.cpp contexts use,
// integration/resident_decode.cpp:70) is kept as three planes per layer so
// that every cache row is a 16-byte multiple and whole row ranges move with
// one bulk copy:
//   k_qs [kv_head][ctx][64]  the 4 blocks' 16 nibble bytes of the K row
//   v_qs [kv_head][ctx][64]  the same for V
//   kv_d [kv_head][ctx][8]   fp16 d of the K blocks 0..3, then of V 0..3
// Within a block's 16 bytes, element e < 16 is the low nibble of byte e and
// element e + 16 its high nibble (GGML's order).
constexpr int kKvF16 = 0;
constexpr int kKvQ4_0 = 1;
constexpr int kQ4_0RowBytes = kHeadDim / 2;  // nibbles of one K or V row
constexpr int kQ4_0DRowBytes = 16;           // the 8 fp16 block scales of one row

// GGML's quantize_row_q4_0 (llama.cpp ggml-quants.c) for the block whose
// element `lane` this lane holds: the element of largest magnitude (the
// first on ties; NaN never wins) is vmax, d = vmax / -8, id = 1 / d (0 when
// d == 0), q = min(15, trunc(x * id + 8.5)) with the product and the sum
// each rounded to fp32 (no contraction).  Returns q | q(lane + 16) << 4 --
// byte `lane` of the block on lanes 0..15 -- and d as fp16 bits.
__device__ __forceinline__ uint32_t q4_0_quantize_lane(float x, uint16_t* d16) {
  const uint32_t key = isnan(x) ? 0u : __float_as_uint(fabsf(x));
  const uint32_t m = __reduce_max_sync(0xffffffffu, key);
  const int first = __ffs(__ballot_sync(0xffffffffu, key == m)) - 1;
  float vmax = __shfl_sync(0xffffffffu, x, first);
  if (m == 0u) vmax = 0.0f;  // no element above zero: GGML keeps its +0 start value
  const float d = __fdiv_rn(vmax, -8.0f);
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  const int q = min(15, __float2int_rz(__fadd_rn(__fmul_rn(x, id), 8.5f)));
  *d16 = __half_as_ushort(__float2half_rn(d));
  const int hi = __shfl_down_sync(0xffffffffu, q, 16);
  return static_cast<uint32_t>(q | (hi << 4));
}

// One warp quantises one 128-value row (4 blocks; x[i] is element lane of
// block i) into `qs` (64 bytes) and `d` (4 fp16).
__device__ __forceinline__ void q4_0_store_row(const float (&x)[4], int lane, uint8_t* qs, uint16_t* d) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint16_t d16;
    const uint32_t byte = q4_0_quantize_lane(x[i], &d16);
    if (lane < 16) qs[i * 16 + lane] = static_cast<uint8_t>(byte);
    if (lane == 0) d[i] = d16;
  }
}

// Rows [row0, row0 + rows) of every KV head from fp32 k and v, each
// [kv_head][rows][128]: one warp per (head, row, K or V).
__global__ void __launch_bounds__(128) kv_q4_0_store_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                                            uint8_t* __restrict__ k_qs, uint8_t* __restrict__ v_qs,
                                                            uint16_t* __restrict__ kv_d, int hkv, int ctx, int row0,
                                                            int rows) {
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const long long w = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long per_head = 2ll * rows;
  if (w >= per_head * hkv) return;
  const int j = static_cast<int>(w / per_head);
  const int r = static_cast<int>((w % per_head) >> 1);
  const bool is_v = (w & 1) != 0;
  const float* src = (is_v ? v : k) + (static_cast<size_t>(j) * rows + r) * kHeadDim;
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = src[lane + 32 * i];
  const size_t row = static_cast<size_t>(j) * ctx + row0 + r;
  q4_0_store_row(x, lane, (is_v ? v_qs : k_qs) + row * kQ4_0RowBytes, kv_d + row * 8 + (is_v ? 4 : 0));
}

// ------------------------------------------------------------- attention

// fp16 bit pattern -> its value x 2^-1008, exactly, for every finite half
// (normal and subnormal): moving the 15 magnitude bits up by 42 places
// re-biases the exponent by 1023 - 15 and turns a subnormal half into a
// subnormal double of the same scaled value.  Integer ops only.
__device__ __forceinline__ double half_bits_scaled(uint32_t h16) {
  const uint32_t hi = ((h16 & 0x7fffu) << 10) | ((h16 & 0x8000u) << 16);
  return __hiloint2double(static_cast<int>(hi), 0);
}

constexpr double kTwo1008 = 0x1p1008;

// Sum, over the 32 lanes of a warp, each of 32 values v[slot] at once:
// afterwards lane l holds the total of logical index l = key * G + head.
// Lane l keeps logical index i in slot i ^ (l & ~(G - 1)) (key bits XORed
// with its own), so on every key-bit step the value to send is the upper
// half of the live slots and the one to keep the lower half: no selects.
// The head bits (unpermuted) take the select form.  31 shuffles.
template <int G>
__device__ __forceinline__ double transpose_reduce32(double (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= G; off >>= 1) {
#pragma unroll
    for (int p = 0; p < off; ++p) v[p] += __shfl_xor_sync(0xffffffffu, v[p + off], off);
  }
#pragma unroll
  for (int off = G / 2; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const double send = upper ? v[i] : v[i + off];
      const double keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// One CTA per (context chunk, KV head); G query heads share the KV head.
// Default shape: 16 warps where 128 registers a thread suffice (G = 4, the
// decode shape, and G = 1), otherwise 8, one CTA per SM, chunks of up to 256
// keys.  Long contexts (more chunks than one wave of SMs) take a smaller
// shape with several CTAs per SM (WARPS warps, CHUNK keys), so that one CTA's
// K/V copies and barriers overlap another's arithmetic.  KV: kKvF16 (rows of
// 128 fp16) or kKvQ4_0 (the three planes above; the scale rows travel with
// the K rows).
template <int G, int KV = kKvF16, int WARPS = ((G == 4 || G == 1) ? 16 : 8), int CHUNK = 256, int CTAS = 1>
struct AttnConfig {
  static constexpr int kWarps = WARPS;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kCtasPerSm = CTAS;                 // resident CTAs per SM the launch bounds ask for
  static constexpr int kMaxChunk = CHUNK;                 // keys per CTA
  static constexpr int kSub = CHUNK < 64 ? CHUNK : 64;    // keys per staged sub-chunk
  static constexpr int kNumSub = kMaxChunk / kSub;
  static constexpr int kRowBytes = KV == kKvQ4_0 ? kQ4_0RowBytes : kHeadDim * 2;  // one K or V row
  static constexpr int kDRowBytes = KV == kKvQ4_0 ? kQ4_0DRowBytes : 0;
  static constexpr int kKeysPerPass = 32 / G;             // keys per warp per score pass
  static constexpr int kWarpsPerHead = kWarps / G;
  static constexpr int kKOffset = 0;
  static constexpr int kVOffset = kMaxChunk * kRowBytes;
  static constexpr int kDOffset = 2 * kMaxChunk * kRowBytes;                // Q4_0 scale rows
  static constexpr int kKvBytes = kDOffset + kMaxChunk * kDRowBytes;
  static constexpr int kRedBytes = kWarps * G * kHeadDim * 8;               // P.V cross-warp sums
  static constexpr int kScoreOffset = ((kKvBytes > kRedBytes ? kKvBytes : kRedBytes) + 127) & ~127;  // fp64 [G][kMaxChunk]
  static constexpr int kQOffset = kScoreOffset + G * kMaxChunk * 8;         // fp32 [G][128]
  static constexpr int kRotOffset = kQOffset + G * kHeadDim * 4;            // double2 [64]
  static constexpr int kRedOffset = kRotOffset + kHeadDim / 2 * 16;         // fp64 [2][kWarps]
  static constexpr int kBarOffset = kRedOffset + 2 * kWarps * 8;            // 2 x kNumSub mbarriers
  static constexpr int kSmemBytes = kBarOffset + 2 * kNumSub * 8;
  static_assert(32 % G == 0 && G <= kWarps && kWarps % G == 0, "query heads per KV head");
  static_assert(kSub % kKeysPerPass == 0 && kMaxChunk % kSub == 0, "score passes stay inside one sub-chunk");
  static_assert(kMaxChunk % 16 == 0, "chunks are multiples of 16 keys");
  static_assert(KV == kKvF16 || KV == kKvQ4_0, "KV cache type");
  static_assert(kSmemBytes * kCtasPerSm <= 227 * 1024, "resident CTAs fit in shared memory");
};

// 2^52 + n as a double (exact for 0 <= n < 2^32), minus 2^52 + 8: the
// Q4_0 value n - 8 without an integer-to-fp64 conversion.
__device__ __forceinline__ double q4_0_value(uint32_t n) {
  return __hiloint2double(0x43300000, static_cast<int>(n)) - 0x1.0000000000008p52;
}

// Chunk c of the n = pos + 1 keys: per = roundup16(ceil(n / splits)) keys
// from c * per.  Writes, per query head hh = kv_head * G + g and chunk c:
//   part_ml[(hh * splits + c) * 2 + {0, 1}] = m (max score), l = sum exp(s - m)
//   part_acc[(hh * splits + c) * 128 + d]   = sum exp(s - m) * v[d]
// with s = (q . k) * scale, all fp64.  An empty chunk writes m = -inf, l = 0.
//
// K/V rows below pos are final (written by earlier steps): they are copied
// in 64-row sub-chunks (one mbarrier each, so scoring starts on the first)
// before waiting on the preceding kernel.  Row pos, the token's own:
//  - qkv == nullptr: the preceding kernel appended it; it is read after the
//    wait, and q is the already normalised and rotated query;
//  - qkv != nullptr (fused): this kernel does the per-head RMSNorm + gamma +
//    IMROPE of the G query heads from the raw QKV projection, and the CTA
//    whose chunk holds pos also forms the K row (RMSNorm + k_gamma + IMROPE
//    -> fp32 -> fp16 or Q4_0) and the V row (fp32 -> fp16 or Q4_0), appends
//    both to the caches and uses them directly.  The 64 rotations are built
//    before the wait.
// Q4_0 (KV == kKvQ4_0): k_cache / v_cache are the nibble planes and kv_d the
// scale plane; cache values d * (q - 8) enter fp64 exactly (d through
// half_bits_scaled, q - 8 through q4_0_value).
template <int G, int KV, int WARPS, int CHUNK, int CTAS>
__global__ void __launch_bounds__(AttnConfig<G, KV, WARPS, CHUNK, CTAS>::kThreads,
                                  AttnConfig<G, KV, WARPS, CHUNK, CTAS>::kCtasPerSm)
    attn_split_kernel(const float* __restrict__ q, const float* __restrict__ qkv, const float* __restrict__ q_gamma,
                      const float* __restrict__ k_gamma, double theta, int hq, int hkv,
                      const DecodeState* __restrict__ state, uint8_t* __restrict__ k_cache,
                      uint8_t* __restrict__ v_cache, uint8_t* __restrict__ kv_d, double* __restrict__ part_acc,
                      double* __restrict__ part_ml, int ctx, int splits, double scale) {
  using C = AttnConfig<G, KV, WARPS, CHUNK, CTAS>;
  constexpr int W = C::kWarps, KB = C::kKeysPerPass, WG = C::kWarpsPerHead;
  constexpr bool kQ4 = KV == kKvQ4_0;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ks = smem + C::kKOffset;
  uint8_t* vs = smem + C::kVOffset;
  uint8_t* ds = smem + C::kDOffset;
  double* sc = reinterpret_cast<double*>(smem + C::kScoreOffset);
  float* qs = reinterpret_cast<float*>(smem + C::kQOffset);
  double2* rot = reinterpret_cast<double2*>(smem + C::kRotOffset);
  double* red_m = reinterpret_cast<double*>(smem + C::kRedOffset);
  double* red_l = red_m + W;
  uint64_t* bar_k = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* bar_v = bar_k + C::kNumSub;
  const int split = blockIdx.x, j = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool fused = qkv != nullptr;
  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 0);

  const int pos = state->pos;
  const int n = pos < 0 ? 0 : (pos < ctx ? pos + 1 : ctx);
  const int per = ((n + splits - 1) / splits + 15) & ~15;
  const int t0 = min(split * per, n), t1 = min(t0 + per, n);
  const int cnt = t1 - t0;
  const int old_cnt = max(min(t1, pos) - t0, 0);
  const bool has_new = cnt > old_cnt;  // this chunk holds row pos
  const int sub_new = old_cnt / C::kSub;
  const size_t first_row = static_cast<size_t>(j) * ctx + t0;
  const size_t row0 = first_row * C::kRowBytes;

  if (tid == 0) {
    for (int s = 0; s < C::kNumSub; ++s) {
      const uint32_t count = (has_new && s == sub_new) ? 2u : 1u;
      mbar_init(&bar_k[s], count);
      mbar_init(&bar_v[s], count);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint64_t policy = l2_evict_first_policy();
    for (int s = 0; s < C::kNumSub; ++s) {
      const int rows = min(max(old_cnt - s * C::kSub, 0), C::kSub);
      if (rows > 0) {
        const uint32_t bytes = static_cast<uint32_t>(rows) * C::kRowBytes;
        const size_t off = static_cast<size_t>(s) * C::kSub * C::kRowBytes;
        if constexpr (kQ4) {
          const uint32_t dbytes = static_cast<uint32_t>(rows) * C::kDRowBytes;
          const size_t doff = static_cast<size_t>(s) * C::kSub * C::kDRowBytes;
          mbar_arrive_expect_tx(&bar_k[s], bytes + dbytes);
          bulk_copy_g2s(ds + doff, kv_d + first_row * C::kDRowBytes + doff, dbytes, &bar_k[s], policy);
        } else {
          mbar_arrive_expect_tx(&bar_k[s], bytes);
        }
        bulk_copy_g2s(ks + off, k_cache + row0 + off, bytes, &bar_k[s], policy);
      } else {
        mbar_arrive(&bar_k[s]);
      }
    }
    for (int s = 0; s < C::kNumSub; ++s) {
      const int rows = min(max(old_cnt - s * C::kSub, 0), C::kSub);
      if (rows > 0) {
        const uint32_t bytes = static_cast<uint32_t>(rows) * C::kRowBytes;
        const size_t off = static_cast<size_t>(s) * C::kSub * C::kRowBytes;
        mbar_arrive_expect_tx(&bar_v[s], bytes);
        bulk_copy_g2s(vs + off, v_cache + row0 + off, bytes, &bar_v[s], policy);
      } else {
        mbar_arrive(&bar_v[s]);
      }
    }
  }
  if (fused && tid < kHeadDim / 2) rot[tid] = imrope_rotation(tid, pos, pos, pos, 0, theta);
  __syncthreads();
  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 1);
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 2);

  // The query heads (and, in the chunk holding pos, the new K/V row).
  if (fused) {
    const int tasks = G + (has_new ? 2 : 0);
    for (int task = warp; task < tasks; task += W) {
      double o[4];
      if (task < G) {
        imrope_head_table(qkv + static_cast<size_t>(j * G + task) * kHeadDim, q_gamma, rot, lane, o);
        float* dst = qs + task * kHeadDim;
        dst[lane] = static_cast<float>(o[0]);
        dst[lane + 64] = static_cast<float>(o[1]);
        dst[lane + 32] = static_cast<float>(o[2]);
        dst[lane + 96] = static_cast<float>(o[3]);
      } else {
        const bool is_k = task == G;
        float f[4];  // dims lane + 32 i, fp32
        if (is_k) {
          imrope_head_table(qkv + static_cast<size_t>(hq + j) * kHeadDim, k_gamma, rot, lane, o);
          f[0] = static_cast<float>(o[0]);
          f[1] = static_cast<float>(o[2]);
          f[2] = static_cast<float>(o[1]);
          f[3] = static_cast<float>(o[3]);
        } else {
          const float* src = qkv + static_cast<size_t>(hq + hkv + j) * kHeadDim;
#pragma unroll
          for (int i = 0; i < 4; ++i) f[i] = src[lane + 32 * i];
        }
        uint8_t* srow = (is_k ? ks : vs) + old_cnt * C::kRowBytes;
        uint8_t* grow = (is_k ? k_cache : v_cache) + row0 + old_cnt * C::kRowBytes;
        if constexpr (kQ4) {
          const int dslot = is_k ? 0 : 4;
          uint16_t* sd = reinterpret_cast<uint16_t*>(ds + old_cnt * C::kDRowBytes) + dslot;
          uint16_t* gd = reinterpret_cast<uint16_t*>(kv_d + (first_row + old_cnt) * C::kDRowBytes) + dslot;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint16_t d16;
            const uint32_t byte = q4_0_quantize_lane(f[i], &d16);
            if (lane < 16) {
              srow[i * 16 + lane] = static_cast<uint8_t>(byte);
              grow[i * 16 + lane] = static_cast<uint8_t>(byte);
            }
            if (lane == 0) {
              sd[i] = d16;
              gd[i] = d16;
            }
          }
        } else {
          __half* sh = reinterpret_cast<__half*>(srow);
          __half* gh = reinterpret_cast<__half*>(grow);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const __half hv = __float2half_rn(f[i]);
            sh[lane + 32 * i] = hv;
            gh[lane + 32 * i] = hv;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(is_k ? &bar_k[sub_new] : &bar_v[sub_new]);
      }
    }
    if (pos >= ctx && split == 0 && j == 0 && tid == 0) record_error(kErrKvOverflow);
    __syncthreads();
  } else if (has_new && (tid == 0 || tid == 32)) {
    // The appended row, read after the wait (K's thread also takes the Q4_0
    // scale row, which holds the V scales too).
    const bool is_k = tid == 0;
    constexpr int kChunks = C::kRowBytes / 16;
    const uint4* src = reinterpret_cast<const uint4*>((is_k ? k_cache : v_cache) + row0 + old_cnt * C::kRowBytes);
    uint4* dst = reinterpret_cast<uint4*>((is_k ? ks : vs) + old_cnt * C::kRowBytes);
    uint4 row[kChunks];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) row[i] = src[i];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) dst[i] = row[i];
    if constexpr (kQ4) {
      if (is_k)
        *reinterpret_cast<uint4*>(ds + old_cnt * C::kDRowBytes) =
            *reinterpret_cast<const uint4*>(kv_d + (first_row + old_cnt) * C::kDRowBytes);
    }
    mbar_arrive(is_k ? &bar_k[sub_new] : &bar_v[sub_new]);
  }
  // Lane l owns dims 4l..4l+3 of the G query heads, scaled by 2^1008.
  double qd[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float4 v = fused ? reinterpret_cast<const float4*>(qs + g * kHeadDim)[lane]
                           : reinterpret_cast<const float4*>(q + static_cast<size_t>(j * G + g) * kHeadDim)[lane];
    qd[g][0] = static_cast<double>(v.x) * kTwo1008;
    qd[g][1] = static_cast<double>(v.y) * kTwo1008;
    qd[g][2] = static_cast<double>(v.z) * kTwo1008;
    qd[g][3] = static_cast<double>(v.w) * kTwo1008;
  }
  // Q4_0: dims 4l..4l+3 are elements 4 (l % 8) .. + 3 of block l / 8, held
  // in the low (l % 8 < 4) or high nibbles of the block's bytes 4 (l % 4)..+3.
  const int q4_blk = lane >> 3;
  const int q4_word = q4_blk * 16 + (lane & 3) * 4;
  const int q4_shift = (lane & 4) ? 4 : 0;
  const uint16_t* dsh = reinterpret_cast<const uint16_t*>(ds);

  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 3);
  // Scores: a warp pass covers KB keys x G heads = 32 dot products; lane l
  // reads key (slot ^ l / G) of the pass, the layout transpose_reduce32 wants.
  bool ok = true;
  const int lane_key = lane / G;
  for (int pass = warp; pass * KB < cnt; pass += W) {
    const int base = pass * KB;
    ok = mbar_wait_bounded(&bar_k[base / C::kSub], 0) && ok;
    double v[32];
#pragma unroll
    for (int kp = 0; kp < KB; ++kp) {
      const int t = base + (kp ^ lane_key);
      if constexpr (kQ4) {
        uint32_t w = 0u, dh = 0u;
        if (t < cnt) {
          w = *reinterpret_cast<const uint32_t*>(ks + t * C::kRowBytes + q4_word) >> q4_shift;
          dh = dsh[t * 8 + q4_blk];
        }
        const double k0 = q4_0_value(w & 15u), k1 = q4_0_value((w >> 8) & 15u);
        const double k2 = q4_0_value((w >> 16) & 15u), k3 = q4_0_value((w >> 24) & 15u);
        const double dk = half_bits_scaled(dh);
#pragma unroll
        for (int g = 0; g < G; ++g)
          v[kp * G + g] = dk * fma(qd[g][3], k3, fma(qd[g][2], k2, fma(qd[g][1], k1, qd[g][0] * k0)));
      } else {
        uint2 w = make_uint2(0u, 0u);
        if (t < cnt) w = *reinterpret_cast<const uint2*>(ks + t * C::kRowBytes + lane * 8);
        const double k0 = half_bits_scaled(w.x & 0xffffu), k1 = half_bits_scaled(w.x >> 16);
        const double k2 = half_bits_scaled(w.y & 0xffffu), k3 = half_bits_scaled(w.y >> 16);
#pragma unroll
        for (int g = 0; g < G; ++g)
          v[kp * G + g] = fma(qd[g][3], k3, fma(qd[g][2], k2, fma(qd[g][1], k1, qd[g][0] * k0)));
      }
    }
    const double total = transpose_reduce32<G>(v, lane);
    const int t = base + lane_key;
    if (t < cnt) sc[(lane % G) * C::kMaxChunk + t] = total * scale;
  }
  __syncthreads();
  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 4);

  // Chunk softmax: WG warps per query head; weights stored x 2^1008.
  {
    const int g = warp / WG, r = warp % WG;
    double* s = sc + g * C::kMaxChunk;
    double m = -INFINITY;
    for (int t = r * 32 + lane; t < cnt; t += WG * 32) m = fmax(m, s[t]);
    m = warp_max_double(m);
    if (lane == 0) red_m[warp] = m;
    __syncthreads();
    m = -INFINITY;
#pragma unroll
    for (int i = 0; i < WG; ++i) m = fmax(m, red_m[g * WG + i]);
    double l = 0.0;
    for (int t = r * 32 + lane; t < cnt; t += WG * 32) {
      const double p = exp(s[t] - m);
      s[t] = p * kTwo1008;
      l += p;
    }
    l = warp_sum_double(l);
    if (lane == 0) red_l[warp] = l;
    __syncthreads();
    if (r == 0 && lane == 0) {
      double total = 0.0;
#pragma unroll
      for (int i = 0; i < WG; ++i) total += red_l[g * WG + i];
      double* ml = part_ml + (static_cast<size_t>(j * G + g) * splits + split) * 2;
      ml[0] = cnt > 0 ? m : -INFINITY;
      ml[1] = cnt > 0 ? total : 0.0;
    }
  }

  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 5);
  // P.V: warp w takes keys w, w + W, ...; lane l owns dims 4l..4l+3.  (The
  // Q4_0 V scales came with the K copies: those barriers are waited on too.)
  for (int s = 0; s < C::kNumSub; ++s) {
    ok = mbar_wait_bounded(&bar_v[s], 0) && ok;
    if constexpr (kQ4) ok = mbar_wait_bounded(&bar_k[s], 0) && ok;
  }
  double acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0;
  for (int t = warp; t < cnt; t += W) {
    if constexpr (kQ4) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(vs + t * C::kRowBytes + q4_word) >> q4_shift;
      const double v0 = q4_0_value(w & 15u), v1 = q4_0_value((w >> 8) & 15u);
      const double v2 = q4_0_value((w >> 16) & 15u), v3 = q4_0_value((w >> 24) & 15u);
      const double dv = half_bits_scaled(dsh[t * 8 + 4 + q4_blk]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const double p = sc[g * C::kMaxChunk + t] * dv;
        acc[g][0] = fma(p, v0, acc[g][0]);
        acc[g][1] = fma(p, v1, acc[g][1]);
        acc[g][2] = fma(p, v2, acc[g][2]);
        acc[g][3] = fma(p, v3, acc[g][3]);
      }
    } else {
      const uint2 w = *reinterpret_cast<const uint2*>(vs + t * C::kRowBytes + lane * 8);
      const double v0 = half_bits_scaled(w.x & 0xffffu), v1 = half_bits_scaled(w.x >> 16);
      const double v2 = half_bits_scaled(w.y & 0xffffu), v3 = half_bits_scaled(w.y >> 16);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const double p = sc[g * C::kMaxChunk + t];
        acc[g][0] = fma(p, v0, acc[g][0]);
        acc[g][1] = fma(p, v1, acc[g][1]);
        acc[g][2] = fma(p, v2, acc[g][2]);
        acc[g][3] = fma(p, v3, acc[g][3]);
      }
    }
  }
  if (!ok && tid == 0) record_error(kErrKvWaitTimeout);
  __syncthreads();
  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 6);
  // Cross-warp sum in warp order through the K / V / scale buffers (no
  // longer read; the region holds at least kRedBytes).
  double* red = reinterpret_cast<double*>(smem);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    double* dst = red + (warp * G + g) * kHeadDim + 4 * lane;
    dst[0] = acc[g][0];
    dst[1] = acc[g][1];
    dst[2] = acc[g][2];
    dst[3] = acc[g][3];
  }
  __syncthreads();
  for (int idx = tid; idx < G * kHeadDim; idx += C::kThreads) {
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < W; ++w) s += red[w * G * kHeadDim + idx];
    const int g = idx / kHeadDim, d = idx % kHeadDim;
    part_acc[(static_cast<size_t>(j * G + g) * splits + split) * kHeadDim + d] = s;
  }
  MLLB_TRACE_CTA(blockIdx.y * gridDim.x + blockIdx.x, 7);
  // After a timed-out wait, give the copies another bounded wait before the
  // shared memory is released.
  if (!ok && tid == 0) {
    for (int s = 0; s < C::kNumSub; ++s) {
      mbar_wait_bounded(&bar_k[s], 0);
      mbar_wait_bounded(&bar_v[s], 0);
    }
  }
}

// One CTA of 128 threads per query head: merge the chunk partials,
//   M = max m_c,  L = sum l_c e^(m_c - M),  out[d] = fp32(sum acc_c[d] e^(m_c - M) / L),
// then quantise the head's 128 values to 4 Q8_1 blocks (one per warp).
// Warp 0 turns the chunk maxima into weights e^(m_c - M) in shared memory
// (dynamic, `splits` doubles); every thread then sums its dimension over the
// chunks with independent loads.
__global__ void __launch_bounds__(128) attn_combine_kernel(const double* __restrict__ part_acc,
                                                           const double* __restrict__ part_ml, int splits,
                                                           float* __restrict__ out, uint8_t* __restrict__ q8,
                                                           int s_mode) {
  extern __shared__ double weight[];
  __shared__ double total_l;
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int h = blockIdx.x, d = threadIdx.x, lane = d & 31;
  const double* ml = part_ml + static_cast<size_t>(h) * splits * 2;
  const double* acc = part_acc + static_cast<size_t>(h) * splits * kHeadDim + d;
  // The first batch of this thread's partials is in flight while warp 0
  // turns the chunk maxima into weights.
  constexpr int kBatch = 32;
  double a[kBatch];
#pragma unroll
  for (int u = 0; u < kBatch; ++u) a[u] = u < splits ? acc[static_cast<size_t>(u) * kHeadDim] : 0.0;
  if (d < 32) {
    double m_max = -INFINITY;
    for (int c = lane; c < splits; c += 32) m_max = fmax(m_max, ml[2 * c]);
    m_max = warp_max_double(m_max);
    double l = 0.0;
    for (int c = lane; c < splits; c += 32) {
      const double m = ml[2 * c];
      const double w = m == -INFINITY ? 0.0 : exp(m - m_max);
      weight[c] = w;
      l += ml[2 * c + 1] * w;
    }
    l = warp_sum_double(l);
    if (lane == 0) total_l = l;
  }
  __syncthreads();
  // All loads of a batch of 32 chunks are issued before the sums use them.
  double o = 0.0;
  for (int c0 = 0; c0 < splits; c0 += kBatch) {
    if (c0 > 0) {
#pragma unroll
      for (int u = 0; u < kBatch; ++u) a[u] = c0 + u < splits ? acc[static_cast<size_t>(c0 + u) * kHeadDim] : 0.0;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (c0 + u < splits) o = fma(a[u], weight[c0 + u], o);
  }
  const double l = total_l;
  const float y = l > 0.0 ? static_cast<float>(o / l) : 0.0f;
  if (out) out[static_cast<size_t>(h) * kHeadDim + d] = y;
  if (q8) {
    uint32_t d16, s16;
    const int qv = q8_1_quantize_lane(y, s_mode, &d16, &s16);
    q8_1_store_block(q8 + (static_cast<size_t>(h) * 4 + (d >> 5)) * 36, qv, d16, s16, lane);
  }
}

// ---------------------------------------------------------------- argmax

// key = max(key, max_i argmax_key(x[i], offset + i)).  The key must hold
// kNoToken (or an earlier maximum) before the launch; the decode step's final
// norm resets it.
__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ x, int64_t n, int64_t offset,
                                                     long long* key) {
  __shared__ long long best_warp[8];
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  long long best = kNoToken;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const long long k = argmax_key(x[i], static_cast<uint32_t>(offset + i));
    best = k > best ? k : best;
  }
  best = warp_max_ll(best);
  if ((threadIdx.x & 31) == 0) best_warp[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = best_warp[w] > best ? best_warp[w] : best;
    if (best != kNoToken) atomicMax(key, best);
  }
}

}  // namespace mllb
