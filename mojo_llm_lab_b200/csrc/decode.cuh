// Kernels of one single-token decode step around the matvecs of a
// Qwen3-style stack (embedding -> 36 x [norm, QKV, q/k norm + IMROPE + KV
// append, attention, O, residual + norm, gate/up, down] -> norm -> Q6_K
// logits -> greedy argmax):
//
//   embed_q6k_kernel        token row of the tied Q6_K output matrix -> fp32
//   rmsnorm_q8_1_kernel     h = x + delta (fp32); y = h * r * gamma -> Q8_1
//   qk_rope_append_kernel   per-head RMSNorm + gamma + IMROPE of the Q and K
//                           heads; K and V appended to the fp16 cache
//   attn_split_kernel<G>    one (KV head, context chunk) per CTA: scores,
//                           chunk softmax, P.V partials
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

#include <climits>

#include "common.cuh"
#include "imrope.cuh"
#include "q8_1.cuh"

namespace mllb {

// Mirrors mllb_decode_state of the public header (32 bytes).
struct DecodeState {
  long long next_token_key;  // packed (value, index) of the greedy next token
  int pos;                   // position / KV row of the token being decoded
  int token;                 // token being decoded (written by the embedding)
  int steps;                 // completed decode steps
  int reserved[3];
};
static_assert(sizeof(DecodeState) == 32, "decode state layout");

constexpr long long kNoToken = LLONG_MIN;
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

// Store one Q8_1 block whose 32 values were quantised one per lane.
__device__ __forceinline__ void q8_1_store_block(uint8_t* blk, int q, uint32_t d16, uint32_t s16, int lane) {
  const uint32_t b = static_cast<uint32_t>(q) & 0xffu;
  const uint32_t b1 = __shfl_down_sync(0xffffffffu, b, 1);
  const uint32_t b2 = __shfl_down_sync(0xffffffffu, b, 2);
  const uint32_t b3 = __shfl_down_sync(0xffffffffu, b, 3);
  if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(blk + 4 + lane) = b | (b1 << 8) | (b2 << 16) | (b3 << 24);
  if (lane == 0) *reinterpret_cast<uint32_t*>(blk) = d16 | (s16 << 16);
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

// One CTA: h = x (+ delta) in fp32, written to x_out when given (x_out may
// alias x); r = 1 / sqrt(sum(h^2) / k + eps) in fp64; y = fp32(h * r * gamma);
// Q8_1 of y.  With `advance` (the step's final norm) thread 0 also resets the
// next-token key and moves the state to the next position.
__global__ void __launch_bounds__(1024) rmsnorm_q8_1_kernel(const float* x, const float* __restrict__ delta,
                                                            float* x_out, const float* __restrict__ gamma,
                                                            double eps, uint8_t* __restrict__ q8, int k, int s_mode,
                                                            DecodeState* advance) {
  extern __shared__ float hs[];
  __shared__ double partial[32];
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  double ss = 0.0;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    float h = x[i];
    if (delta) h += delta[i];
    hs[i] = h;
    if (x_out) x_out[i] = h;
    ss = fma(static_cast<double>(h), static_cast<double>(h), ss);
  }
  ss = warp_sum_double(ss);
  if (lane == 0) partial[warp] = ss;
  __syncthreads();
  double total = lane < warps ? partial[lane] : 0.0;
  total = warp_sum_double(total);
  const double r = 1.0 / sqrt(total / static_cast<double>(k) + eps);
  for (int b = warp; b < k / 32; b += warps) {
    const int i = b * 32 + lane;
    const float y = static_cast<float>(static_cast<double>(hs[i]) * r * static_cast<double>(gamma[i]));
    uint32_t d16, s16;
    const int q = q8_1_quantize_lane(y, s_mode, &d16, &s16);
    q8_1_store_block(q8 + static_cast<size_t>(b) * 36, q, d16, s16, lane);
  }
  if (advance && threadIdx.x == 0) {
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
// are (pos, pos, pos, 0).  pos outside [0, ctx) raises kErrKvOverflow and
// appends nothing.  Cache layout: [kv_head][ctx][128] fp16.
__global__ void __launch_bounds__(256) qk_rope_append_kernel(const float* __restrict__ qkv,
                                                             const float* __restrict__ q_gamma,
                                                             const float* __restrict__ k_gamma,
                                                             const DecodeState* __restrict__ state, double theta,
                                                             float* __restrict__ q_out, __half* __restrict__ k_cache,
                                                             __half* __restrict__ v_cache, int hq, int hkv, int ctx) {
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= hq + 2 * hkv) return;
  const int pos = state->pos;
  double o[4];
  if (w < hq) {
    imrope_head_values(qkv + static_cast<size_t>(w) * kHeadDim, q_gamma, pos, pos, pos, 0, theta, lane, o);
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
    imrope_head_values(qkv + static_cast<size_t>(w) * kHeadDim, k_gamma, pos, pos, pos, 0, theta, lane, o);
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

// Sum a value index i (0..31) over the 32 lanes of a warp for all 32
// indices at once: after five exchange steps lane l holds the total of
// index l.  31 shuffles for 32 sums.
__device__ __forceinline__ double transpose_reduce32(double (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
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
template <int G>
struct AttnConfig {
  static constexpr int kWarps = 8;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kMaxChunk = 256;                   // keys per CTA
  static constexpr int kRowBytes = kHeadDim * 2;          // one fp16 K or V row
  static constexpr int kKeysPerPass = 32 / G;             // keys per warp per score pass
  static constexpr int kKOffset = 0;
  static constexpr int kVOffset = kMaxChunk * kRowBytes;
  static constexpr int kScoreOffset = 2 * kMaxChunk * kRowBytes;  // fp64 [G][kMaxChunk]
  static constexpr int kBarOffset = kScoreOffset + G * kMaxChunk * 8;
  static constexpr int kSmemBytes = kBarOffset + 16;
  static_assert(32 % G == 0 && G <= kWarps, "query heads per KV head");
  static_assert(kWarps * G * kHeadDim * 8 <= kVOffset, "P.V reduction buffer fits in the K buffer");
};

// Chunk c of the n = pos + 1 keys: per = roundup16(ceil(n / splits)) keys
// from c * per.  Writes, per query head hh = kv_head * G + g and chunk c:
//   part_ml[(hh * splits + c) * 2 + {0, 1}] = m (max score), l = sum exp(s - m)
//   part_acc[(hh * splits + c) * 128 + d]   = sum exp(s - m) * v[d]
// with s = (q . k) * scale, all fp64.  An empty chunk writes m = -inf, l = 0.
// K/V rows below pos are final (written by earlier steps) and are copied in
// before waiting on the preceding kernel; row pos, appended by that kernel,
// is read after the wait.
template <int G>
__global__ void __launch_bounds__(AttnConfig<G>::kThreads, 1)
    attn_split_kernel(const float* __restrict__ q, const uint8_t* __restrict__ k_cache,
                      const uint8_t* __restrict__ v_cache, const DecodeState* __restrict__ state,
                      double* __restrict__ part_acc, double* __restrict__ part_ml, int ctx, int splits,
                      double scale) {
  using C = AttnConfig<G>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ks = smem + C::kKOffset;
  uint8_t* vs = smem + C::kVOffset;
  double* sc = reinterpret_cast<double*>(smem + C::kScoreOffset);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  const int split = blockIdx.x, j = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  const int pos = state->pos;
  const int n = pos < 0 ? 0 : (pos < ctx ? pos + 1 : ctx);
  const int per = ((n + splits - 1) / splits + 15) & ~15;
  const int t0 = min(split * per, n), t1 = min(t0 + per, n);
  const int cnt = t1 - t0;
  const int old_cnt = max(min(t1, pos) - t0, 0);
  const size_t row0 = (static_cast<size_t>(j) * ctx + t0) * C::kRowBytes;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    if (old_cnt > 0) {
      const uint64_t policy = l2_evict_first_policy();
      const uint32_t bytes = static_cast<uint32_t>(old_cnt) * C::kRowBytes;
      mbar_arrive_expect_tx(&bar[0], bytes);
      bulk_copy_g2s(ks, k_cache + row0, bytes, &bar[0], policy);
      mbar_arrive_expect_tx(&bar[1], bytes);
      bulk_copy_g2s(vs, v_cache + row0, bytes, &bar[1], policy);
    } else {
      mbar_arrive(&bar[0]);
      mbar_arrive(&bar[1]);
    }
  }
  pdl_wait_prerequisite();
  pdl_launch_dependents();

  // The row appended by the preceding kernel (at most one per chunk).
  if (cnt > old_cnt && tid < 32) {
    const size_t off = row0 + static_cast<size_t>(old_cnt) * C::kRowBytes;
    const uint8_t* src = (tid < 16 ? k_cache : v_cache) + off;
    uint8_t* dst = (tid < 16 ? ks : vs) + old_cnt * C::kRowBytes;
    reinterpret_cast<uint4*>(dst)[tid & 15] = reinterpret_cast<const uint4*>(src)[tid & 15];
  }
  // Lane l owns dims 4l..4l+3 of the G query heads, scaled by 2^1008.
  double qd[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float4 v = reinterpret_cast<const float4*>(q + static_cast<size_t>(j * G + g) * kHeadDim)[lane];
    qd[g][0] = static_cast<double>(v.x) * kTwo1008;
    qd[g][1] = static_cast<double>(v.y) * kTwo1008;
    qd[g][2] = static_cast<double>(v.z) * kTwo1008;
    qd[g][3] = static_cast<double>(v.w) * kTwo1008;
  }
  bool ok = mbar_wait_bounded(&bar[0], 0);
  __syncthreads();

  // Scores: each warp pass covers kKeysPerPass keys x G heads = 32 dot products.
  constexpr int KB = C::kKeysPerPass;
  if (ok) {
    for (int base = warp * KB; base < cnt; base += C::kWarps * KB) {
      double v[32];
#pragma unroll
      for (int kk = 0; kk < KB; ++kk) {
        const int t = base + kk;
        uint2 w = make_uint2(0u, 0u);
        if (t < cnt) w = *reinterpret_cast<const uint2*>(ks + t * C::kRowBytes + lane * 8);
        const double k0 = half_bits_scaled(w.x & 0xffffu), k1 = half_bits_scaled(w.x >> 16);
        const double k2 = half_bits_scaled(w.y & 0xffffu), k3 = half_bits_scaled(w.y >> 16);
#pragma unroll
        for (int g = 0; g < G; ++g)
          v[kk * G + g] = fma(qd[g][3], k3, fma(qd[g][2], k2, fma(qd[g][1], k1, qd[g][0] * k0)));
      }
      const double total = transpose_reduce32(v, lane);
      const int t = base + lane / G;
      if (t < cnt) sc[(lane % G) * C::kMaxChunk + t] = total * scale;
    }
  }
  __syncthreads();

  // Chunk softmax, one warp per query head; the weights are stored x 2^1008.
  if (warp < G) {
    double* s = sc + warp * C::kMaxChunk;
    double m = -INFINITY;
    for (int t = lane; t < cnt; t += 32) m = fmax(m, s[t]);
    m = warp_max_double(m);
    double l = 0.0;
    for (int t = lane; t < cnt; t += 32) {
      const double p = exp(s[t] - m);
      s[t] = p * kTwo1008;
      l += p;
    }
    l = warp_sum_double(l);
    if (lane == 0) {
      double* ml = part_ml + (static_cast<size_t>(j * G + warp) * splits + split) * 2;
      ml[0] = (ok && cnt > 0) ? m : -INFINITY;
      ml[1] = (ok && cnt > 0) ? l : 0.0;
    }
  }
  ok = mbar_wait_bounded(&bar[1], 0) && ok;
  if (!ok && tid == 0) record_error(kErrKvWaitTimeout);
  __syncthreads();

  // P.V: warp w takes keys w, w + 8, ...; lane l owns dims 4l..4l+3.
  double acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0;
  if (ok) {
    for (int t = warp; t < cnt; t += C::kWarps) {
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
  // Cross-warp sum in warp order through the K buffer (no longer read).
  double* red = reinterpret_cast<double*>(ks);
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
    for (int w = 0; w < C::kWarps; ++w) s += red[w * G * kHeadDim + idx];
    const int g = idx / kHeadDim, d = idx % kHeadDim;
    part_acc[(static_cast<size_t>(j * G + g) * splits + split) * kHeadDim + d] = s;
  }
  // After a timed-out wait, give the copy another bounded wait before the
  // shared memory is released.
  if (!ok && tid == 0) mbar_wait_bounded(&bar[0], 0);
}

// One CTA of 128 threads per query head: merge the chunk partials,
//   M = max m_c,  L = sum l_c e^(m_c - M),  out[d] = fp32(sum acc_c[d] e^(m_c - M) / L),
// then quantise the head's 128 values to 4 Q8_1 blocks (one per warp).
__global__ void __launch_bounds__(128) attn_combine_kernel(const double* __restrict__ part_acc,
                                                           const double* __restrict__ part_ml, int splits,
                                                           float* __restrict__ out, uint8_t* __restrict__ q8,
                                                           int s_mode) {
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  const int h = blockIdx.x, d = threadIdx.x, lane = d & 31;
  const double* ml = part_ml + static_cast<size_t>(h) * splits * 2;
  const double* acc = part_acc + static_cast<size_t>(h) * splits * kHeadDim + d;
  double m_max = -INFINITY;
  for (int c = 0; c < splits; ++c) m_max = fmax(m_max, ml[2 * c]);
  double l = 0.0, o = 0.0;
  for (int c = 0; c < splits; ++c) {
    const double m = ml[2 * c];
    if (m == -INFINITY) continue;
    const double w = exp(m - m_max);
    l += ml[2 * c + 1] * w;
    o += acc[static_cast<size_t>(c) * kHeadDim] * w;
  }
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
