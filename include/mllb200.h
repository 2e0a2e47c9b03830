/*
 * mllb200.h -- C ABI of the B200 (sm_100a) decode hot path.
 *
 * Drop-in for the kernel entry points of HundredBillion/mojo-llm-lab
 * (citations are path:line in that project).  Plain pointers, sizes and an
 * opaque stream; no C++ or framework types, so ctypes, cgo or a C harness
 * bind it directly.
 *
 * Conventions
 * - All data pointers are DEVICE pointers owned by the caller.  No function
 *   allocates, frees or synchronises; every launch is asynchronous on
 *   `stream` (a cudaStream_t / CUstream; NULL = the legacy default stream)
 *   and may be captured into a CUDA graph.
 * - Weights and activations are read only; outputs are written in place.
 * - Return value: MLLB_OK (0) or a negative MLLB_E* code; mllb_last_error()
 *   gives a message for the calling thread.  Nothing aborts the process.
 * - Block formats (byte-exact GGML layouts, as the reference's fixtures):
 *     Q4_K: 144 B / 256 weights  (tests/q4_reference.py:6-24)
 *     Q8_1:  36 B /  32 values   (tests/q4_reference.py:27-33)
 *     Q6_K: 210 B / 256 weights  (GGML block_q6_K)
 *   Rows are contiguous: row r of a K-wide matrix starts at r * (K/256) * block bytes.
 * - Alignment: weight pointers 16-byte aligned, Q8_1 / fp32 pointers 4-byte
 *   aligned (cuMemAlloc / cudaMalloc give 256).  Otherwise MLLB_EALIGN.
 */
#ifndef MLLB200_H
#define MLLB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLLB_ABI_VERSION 1

#define MLLB_OK 0
#define MLLB_EINVAL (-1)       /* null pointer, bad size or shape (reference harness exit 4) */
#define MLLB_EALIGN (-2)       /* pointer alignment below the contract */
#define MLLB_ECUDA (-3)        /* CUDA launch or runtime error (reference harness exit 20) */
#define MLLB_EUNSUPPORTED (-4) /* shape outside what the library implements */

/*
 * Launch flags of the *_ex entry points.
 * MLLB_LAUNCH_PDL: programmatic dependent launch.  The kernel may be scheduled
 * while the preceding kernel in `stream` is still running and starts
 * streaming its weight matrix at once; it waits for that kernel to complete
 * before reading the activation or writing any output.  Only valid when the
 * preceding kernels do not write the weight matrix (model weights are
 * constant during decode).  Chains of such launches overlap each matvec's
 * launch and DRAM latency with the previous one's tail.
 */
#define MLLB_LAUNCH_PDL 1u

/*
 * MLLB_LAUNCH_CONST_AUX (IMROPE entries, with MLLB_LAUNCH_PDL): gamma, the
 * positions and the theta scale are not written by the preceding kernel (they
 * are set by the host or by an earlier, finished kernel), so the kernel reads
 * them and builds its 64 fp64 rotations before the dependency wait; only q is
 * read after it.  The weights rule of MLLB_LAUNCH_PDL, for these operands.
 */
#define MLLB_LAUNCH_CONST_AUX 2u

/* Q8_1 `s` field convention (the dot products never read s). */
#define MLLB_Q8_1_S_D_SUMQ 0 /* s = fp16(fp16(d) * sum(q)): tools/generate_q4_matvec_fixtures.py:59 */
#define MLLB_Q8_1_S_SUM_X 1  /* s = fp16(sum(x)): GGML quantize_q8_1 */

int mllb_abi_version(void);

/* Message for the last failed call on this thread ("" if none). */
const char *mllb_last_error(void);

/*
 * Device error word (bit n = mask 1 << n): bit 0/1/2 = a kernel gave up a bounded (~1 s) wait on
 * its TMA pipeline (see csrc/common.cuh); bit 3 = decode next-token key out
 * of range; bit 4 = decode position outside the KV cache; bit 5 = decode
 * attention gave up waiting for its K/V copies; bit 6 = a peer all-gather
 * gave up waiting for another rank; bit 7 = a grid-wide epilogue
 * (mllb_q4k_matvec_norm) gave up waiting for the other CTAs of its grid.
 * Copies the word of the current device to *bits (synchronising),
 * optionally clearing it.  0 in normal runs.
 */
int mllb_device_error(uint32_t *bits, int clear);

/*
 * Q8_1 quantiser: x[k] fp32 -> k/32 blocks of 36 bytes.  k % 32 == 0.
 * d = amax/127 (IEEE), q = roundf(x/d), d and s stored as fp16 (RNE).
 * Replaces GGML's quantize_q8_1 node the reference clones in front of every
 * matvec (benchmark/q4_compare.c:328-330; bytes checked at :351-357).
 */
int mllb_q8_1_quantize(const float *x, void *q8, int64_t k, int s_mode, void *stream);
/* Same, with launch flags (MLLB_LAUNCH_PDL). */
int mllb_q8_1_quantize_ex(const float *x, void *q8, int64_t k, int s_mode, unsigned flags, void *stream);

/*
 * out[r] = sum_k W[r,k] * a[k] for Q4_K weights (n rows, k columns) and a
 * Q8_1 activation (k/32 blocks).  k % 256 == 0.
 * Replaces kernels/q4_k_q8_1_matvec_dp4a_128.mojo:8-13 (and its siblings
 * q4_k_q8_1_matvec*.mojo), launched by tools/q4_comparison_worker.py:30-31
 * and benchmark/q4_compare.c:382,389-399 as (weights, activations, output).
 */
int mllb_q4k_matvec(const void *weights, const void *q8, float *out, int64_t n, int64_t k, void *stream);
/* Same, with launch flags (MLLB_LAUNCH_PDL). */
int mllb_q4k_matvec_ex(const void *weights, const void *q8, float *out, int64_t n, int64_t k, unsigned flags,
                       void *stream);

/*
 * Fused gate/up: up[r], gate[r] and prod[r] = up[r] * silu(gate[r]) with
 * silu(g) = g / (1 + exp(-g)), two Q4_K matrices over one Q8_1 activation.
 * Any of up / gate / prod may be NULL (not all three).
 * Replaces kernels/q4_k_q8_1_gate_order.mojo:55-79 (up_weights, gate_weights,
 * activations, output) as launched at benchmark/q4_compare.c:379-380 and
 * integration/observe_launches.cpp:89-94; that entry emits prod only.
 */
int mllb_q4k_gate_up(const void *up_weights, const void *gate_weights, const void *q8, float *up, float *gate,
                     float *prod, int64_t n, int64_t k, void *stream);
/* Same, with launch flags (MLLB_LAUNCH_PDL). */
int mllb_q4k_gate_up_ex(const void *up_weights, const void *gate_weights, const void *q8, float *up, float *gate,
                        float *prod, int64_t n, int64_t k, unsigned flags, void *stream);

/*
 * Q6_K x Q8_1 matvec (vocabulary projection): out[r] for n rows, k columns.
 * Replaces GGML's mul_mat_vec_q<Q6_K> in the reference's decode
 * (docs/q6k-vocab-roofline.md:7-12); the reference has no kernel of its own.
 */
int mllb_q6k_matvec(const void *weights, const void *q8, float *out, int64_t n, int64_t k, void *stream);
/* Same, with launch flags (MLLB_LAUNCH_PDL). */
int mllb_q6k_matvec_ex(const void *weights, const void *q8, float *out, int64_t n, int64_t k, unsigned flags,
                       void *stream);

/*
 * Q5_K x Q8_1 matvec: out[r] for n rows of K = 2048, 2560 or 4096 (others:
 * MLLB_EUNSUPPORTED).  Q5_K: 176 B / 256 weights (GGML block_q5_K: fp16 d,
 * fp16 dmin, 12 B of 6-bit scales / mins packed as Q4_K, qh[32], qs[128]).
 * The next format of the family (the reference profiles GGML's Q5_K matvec
 * at 10-15 % of a 2B decode, docs/qwen35-2b-profile.md:7-14; no kernel of
 * its own).
 */
int mllb_q5k_matvec(const void *weights, const void *q8, float *out, int64_t n, int64_t k, void *stream);
/* Same, with launch flags (MLLB_LAUNCH_PDL). */
int mllb_q5k_matvec_ex(const void *weights, const void *q8, float *out, int64_t n, int64_t k, unsigned flags,
                       void *stream);

/*
 * Fused RMSNorm (eps 1e-6) * gamma[128] + IMROPE (sections 24/20/20/0,
 * split-half pairs (p, p+64)) on `heads` contiguous fp32 heads of 128.
 * positions: int32[4] (axis-major) shared by all heads; theta_scale: device
 * fp32[1] (the reference passes bits 0x3f492c27).
 * Replaces kernels/fused_q_imrope_runtime_fastpow.mojo:8-14 with the
 * (q, gamma, positions, output, theta_scale) pointer list of
 * benchmark/bench.c:252-258.
 */
int mllb_rmsnorm_imrope_q(const float *q, const float *gamma, const int32_t *positions, const float *theta_scale,
                          float *out, int64_t heads, void *stream);

/*
 * Throughput form: `tokens` independent Q tensors of heads_per_token heads
 * each, token t using positions[4t..4t+3].  theta_scale may be NULL, in which
 * case theta_value (host double) is used, e.g. pow(5e6, -2/128) exactly.
 * No reference counterpart (the reference fixes one token of 32 heads).
 */
int mllb_rmsnorm_imrope_q_batched(const float *q, const float *gamma, const int32_t *positions,
                                  const float *theta_scale, double theta_value, float *out, int64_t tokens,
                                  int64_t heads_per_token, void *stream);
/* Same, with launch flags (MLLB_LAUNCH_PDL: the kernel may start while the
 * preceding kernel runs; it waits for it before reading anything, or, with
 * MLLB_LAUNCH_CONST_AUX too, before reading q). */
int mllb_rmsnorm_imrope_q_batched_ex(const float *q, const float *gamma, const int32_t *positions,
                                     const float *theta_scale, double theta_value, float *out, int64_t tokens,
                                     int64_t heads_per_token, unsigned flags, void *stream);

/*
 * Exact integer parts of the Q4_K x Q8_1 dot: dots[r * (k/32) + G] =
 * sum of the 32 nibble * int8 products of group G in row r, asums[G] = sum
 * of group G's int8 quants.  The bit-exact parity hook for the integer half
 * of tests/q4_reference.py:36-47.
 */
int mllb_q4k_subdots(const void *weights, const void *q8, int32_t *dots, int32_t *asums, int64_t n, int64_t k,
                     void *stream);

/*
 * HBM read-roofline probe: XOR of `bytes` bytes (multiple of 16, 16-byte
 * aligned) read with 16-byte streaming loads by `blocks` x 256 threads; each
 * thread writes its 16-byte XOR to out[thread].  blocks <= 0 picks one wave.
 * Replaces kernels/stream_read_roofline.mojo:12-27
 * (tools/run_bandwidth_roofline.py:96-110), which used 8-byte loads.
 */
int mllb_stream_read(const void *data, int64_t bytes, void *out, int64_t blocks, void *stream);

/* ------------------------------------------------------------------------
 * Single-token decode step of a Qwen3-style stack (36 layers, hidden 2560,
 * 32 Q / 8 KV heads of 128, SwiGLU 9728, vocab 151936): the GGML ops that
 * the reference's decode runs around its kernels (llama.cpp graph driven by
 * integration/resident_decode.cpp; op shares in docs/decode-profile.md:5-11).
 * The matvecs above plus these entries make one step; all of them can be
 * captured into one CUDA graph and replayed per token, because everything
 * that changes between tokens lives in device memory (mllb_decode_state).
 *
 * Numerics: fp64 inside each kernel, rounded once to the fp32 (or fp16 / Q8_1)
 * value that leaves it.
 *
 * PDL: with MLLB_LAUNCH_PDL the attention copies the K/V rows below
 * state->pos before waiting on the preceding kernel, so neither those rows
 * nor state->pos may be written by the kernels launched just before it (in
 * the decode step only the final norm moves pos).
 * ---------------------------------------------------------------------- */

/* Device-resident state of a decode loop (32 bytes, 8-byte aligned). */
typedef struct mllb_decode_state {
    int64_t next_token_key; /* greedy next token, packed (see mllb_token_key) */
    int32_t pos;            /* position and KV row of the token being decoded */
    int32_t token;          /* token being decoded (written by mllb_decode_embed) */
    int32_t steps;          /* decode steps completed (advanced by the final norm) */
    int32_t reserved[3];
} mllb_decode_state;

/*
 * An activation produced inside a streaming matvec from fp32, instead of a
 * Q8_1 buffer written by a kernel before it:
 *   h = x + delta (fp32; delta may be NULL), stored to x_out when not NULL
 *   (x_out must not overlap x or delta);
 *   y = gamma ? fp32(h / sqrt(mean(h^2) + eps) * gamma) : h;
 *   activation = Q8_1(y) with s = d * sum(q) -- the bytes mllb_rmsnorm_q8_1
 *   (or mllb_q8_1_quantize) would write, built by every CTA for itself.
 * advance (may be NULL): the step's final norm -- reset next_token_key and
 * advance pos and steps as mllb_decode_final_norm does.
 */
typedef struct mllb_act_f32 {
    const float *x;
    const float *delta;
    const float *gamma;
    float *x_out;
    double eps;
    mllb_decode_state *advance;
} mllb_act_f32;

/* The streaming matvecs with that activation (K/256 in {8, 10, 16, 38} for
 * Q4_K, {8, 10, 16} for gate/up and Q6_K; Q6_K rows a multiple of 8;
 * MLLB_EUNSUPPORTED otherwise).  One kernel instead of two per matvec.  The
 * host struct is read during the call only. */
int mllb_q4k_matvec_act(const void *weights, const mllb_act_f32 *act, float *out, int64_t n, int64_t k,
                        unsigned flags, void *stream);
int mllb_q4k_gate_up_act(const void *up_weights, const void *gate_weights, const mllb_act_f32 *act, float *up,
                         float *gate, float *prod, int64_t n, int64_t k, unsigned flags, void *stream);
int mllb_q6k_matvec_act(const void *weights, const mllb_act_f32 *act, float *out, int64_t n, int64_t k,
                        unsigned flags, void *stream);

/*
 * Batched tokens (prompt processing): out[t][r] = (W @ x_t)[r] for T tokens,
 * W a Q4_K matrix of `rows` rows (a multiple of 128) and K columns, x_t the
 * t-th of T consecutive Q8_1 rows (K/32 blocks each); out is [T][rows] fp32,
 * each value within 1e-5 + 1e-5 |ref| of the exact sum.  The integer group
 * dots run on the tensor cores (tcgen05, int8); see csrc/prefill.cuh.  The
 * grid may split K; then `workspace` must hold
 * mllb_q4k_matmul_tokens_workspace(rows, k, tokens) bytes (0 when no split;
 * the plan depends on the current device's SM count).  The reference's
 * counterpart is llama.cpp's MMQ, which it profiles but does not replace
 * (docs/prefill-baseline.md).  flags: as mllb_q4k_matvec_ex (PDL is not
 * used).
 */
int64_t mllb_q4k_matmul_tokens_workspace(int64_t rows, int64_t k, int64_t tokens);
int mllb_q4k_matmul_tokens(const void *weights, const void *q8, float *out, int64_t rows, int64_t k, int64_t tokens,
                           void *workspace, int64_t workspace_bytes, unsigned flags, void *stream);

/*
 * Q4_K matvec whose output is the delta of a residual stream, with the next
 * RMSNorm + Q8_1 built in (no separate mllb_rmsnorm_q8_1 launch):
 *   out[r] = sum_k W[r,k] a[k]             (fp32; out may be NULL)
 *   h[r]   = x[r] + fp32(out[r])  -> x_out  (fp32; x_out may equal x)
 *   q8_out = Q8_1(fp32(h * r * gamma)), r = 1 / sqrt(sum(h^2) / n + eps)  (fp64)
 * i.e. mllb_q4k_matvec_ex followed by mllb_rmsnorm_q8_1(x, out, x_out, gamma,
 * eps, q8_out, n, MLLB_Q8_1_S_D_SUMQ).  n % 32 == 0; K/256 in {8, 10, 16, 38}
 * (others MLLB_EUNSUPPORTED).  workspace: at least
 * mllb_q4k_matvec_norm_workspace(n, k) bytes, 16-byte aligned, its first 16
 * bytes zero before the first call (every call leaves them zero); calls
 * sharing a workspace must not overlap on the GPU.  The CTAs of the launch
 * meet once (a bounded wait: device error bit 7 if the grid never gathers).
 * The O projection and the FFN's down projection of the reference's decode
 * graph, each followed by GGML's add + rms_norm + mul + quantize_q8_1 nodes
 * (docs/decode-profile.md:5-11).
 */
int64_t mllb_q4k_matvec_norm_workspace(int64_t n, int64_t k);
int mllb_q4k_matvec_norm(const void *weights, const void *q8, float *out, int64_t n, int64_t k, const float *x,
                         float *x_out, const float *gamma, double eps, void *q8_out, void *workspace,
                         int64_t workspace_bytes, unsigned flags, void *stream);

/*
 * mllb_q4k_gate_up_q8: mllb_q4k_gate_up_ex that also writes the Q8_1 of prod
 * (s = d * sum q, the bytes mllb_q8_1_quantize would write) into q8_out
 * (n / 32 blocks): the launch that would follow the gate/up in a decode step
 * is folded into it.  The CTA whose stored rows complete a 32-row group
 * quantises that group.  prod must not be NULL; n a multiple of 32;
 * counters: n / 32 uint32, zero before the first call and left zero by each
 * call; calls that share them must not overlap on the GPU.  K/256 in
 * {8, 10, 16}, otherwise MLLB_EUNSUPPORTED.  No counterpart in the reference:
 * there the quantiser is a GGML graph node of its own.
 */
int mllb_q4k_gate_up_q8(const void *up_weights, const void *gate_weights, const void *q8, float *up, float *gate,
                        float *prod, void *q8_out, uint32_t *counters, int64_t n, int64_t k, unsigned flags,
                        void *stream);

/*
 * Peer all-gather of a Q8_1 activation over NVLink (no NCCL): rank r
 * quantises its slice x[0..k) (k = the full length / world, a multiple of
 * 32) and stores the k/32 blocks into every rank's buffer at block offset
 * r * k/32, then signals every rank; the call's kernel finishes on each rank
 * only when all slices have arrived there.  buffers[i] / flags[i]: rank i's
 * destination (world * k/32 * 36 bytes) and counter array (world uint32,
 * zero before the first gather), as device addresses valid on this GPU
 * (peer mappings, e.g. symmetric memory); count: this rank's gather counter
 * (one uint32, zero before the first gather).  Every rank must issue the
 * same sequence of gathers with the same k, each on its own GPU.  A rank
 * that does not arrive within ~1 s sets device error bit 6 (mask 0x40).  Replaces the
 * NCCL all-gather of the sharded SwiGLU product.  world <= 8.
 */
typedef struct mllb_peer_gather {
    int32_t rank, world;
    void *buffers[8];
    uint32_t *flags[8];
    uint32_t *count;
} mllb_peer_gather;

int mllb_q8_1_quantize_allgather(const float *x, int64_t k, const mllb_peer_gather *peers, unsigned flags,
                                 void *stream);

/*
 * mllb_q4k_gate_up_q8 for one rank of a row-sharded gate/up (n = this rank's
 * rows, a multiple of 32) with the all-gather built in: each completed
 * 32-row group's Q8_1 block of the product goes straight into every rank's
 * buffer (peers->buffers[r] + (rank * n / 32 + group) * 36, NVLink stores),
 * the rank then arrives once on every rank's counter for it, and the launch
 * completes only when every rank's blocks are in this GPU's buffer (a rank
 * that does not arrive within ~1 s sets device error bit 6, mask 0x40).  So
 * the down projection, launched next, reads the whole product's Q8_1 from
 * peers->buffers[rank].  counters: n / 32 + 1 zeroed uint32 (the groups, then
 * the CTAs' arrivals), left zero.  Each gather adds 1 to every rank's
 * flags[rank].  peers as
 * for mllb_q8_1_quantize_allgather; every rank issues the same sequence of
 * these launches with the same n and k.  One launch in place of the gate/up
 * launch plus mllb_q8_1_quantize_allgather.  No reference counterpart (the
 * reference runs on one GPU).
 */
int mllb_q4k_gate_up_q8_gather(const void *up_weights, const void *gate_weights, const void *q8, float *up,
                               float *gate, float *prod, uint32_t *counters, int64_t n, int64_t k,
                               const mllb_peer_gather *peers, unsigned flags, void *stream);

/*
 * Bring bytes [data, data + bytes) into L2 ahead of their use, marked
 * evict-last (TMA bulk prefetch; returns as soon as the prefetches are
 * issued, nothing to wait for).  bytes a multiple of 16, data 16-byte aligned.
 * The decode step runs it on a side stream for the next layer's weights and
 * KV rows while the current layer computes.  No reference counterpart.
 */
int mllb_prefetch_l2(const void *data, int64_t bytes, void *stream);

/* Host helpers for the packed next-token key: high 32 bits order the fp32
 * value, low 32 bits are 0xffffffff - index (ties go to the lower index).
 * mllb_token_key(t) is a key that selects token t (to seed a decode loop);
 * mllb_key_token() returns -1 for the "no token" key INT64_MIN. */
int64_t mllb_token_key(int32_t token);
int64_t mllb_key_token(int64_t key);

/*
 * hidden[0..k) = the dequantised row (token) of a Q6_K matrix of `vocab`
 * rows x k (the output projection, tied to the token embedding), token taken
 * from state->next_token_key.  Records state->token and, when tokens is not
 * NULL, tokens[state->steps] (if steps < capacity).  An out-of-range key
 * sets device error bit 3 (mask 0x08) and embeds row 0.  GGML get_rows on the token
 * embedding (no reference kernel).
 */
int mllb_decode_embed(const void *q6k_weights, int64_t vocab, int64_t k, mllb_decode_state *state, int32_t *tokens,
                      int64_t capacity, float *hidden, unsigned flags, void *stream);

/*
 * Residual + RMSNorm + gamma + Q8_1 in one kernel:
 *   h = x + delta (fp32; delta may be NULL), stored to x_out when not NULL;
 *   y = fp32(h / sqrt(mean(h^2) + eps) * gamma);
 *   q8 = Q8_1(y) (s_mode as mllb_q8_1_quantize).  k: multiple of 32, <= 32768.
 * x_out may be x itself (in place; then one CTA does all the work) but must
 * not otherwise overlap x or delta.  A separate x_out spreads the blocks over
 * k/256 CTAs.  With MLLB_LAUNCH_PDL, gamma (a weight) is read before the
 * wait on the preceding kernel; x and delta after it.
 * GGML add -> rms_norm -> mul -> quantize_q8_1 (benchmark/q4_compare.c:328-330
 * is the quantise node this absorbs).
 */
int mllb_rmsnorm_q8_1(const float *x, const float *delta, float *x_out, const float *gamma, double eps, void *q8,
                      int64_t k, int s_mode, unsigned flags, void *stream);

/* The step's final norm: mllb_rmsnorm_q8_1 that also resets
 * state->next_token_key to INT64_MIN and advances state->pos and state->steps. */
int mllb_decode_final_norm(const float *x, const float *delta, float *x_out, const float *gamma, double eps,
                           void *q8, int64_t k, mllb_decode_state *state, unsigned flags, void *stream);

/*
 * qkv: fp32 output of the fused QKV projection, (q_heads + 2 kv_heads) x 128
 * (Q heads, then K heads, then V heads).  Q heads: RMSNorm (eps 1e-6) *
 * q_gamma + IMROPE -> q_out.  K heads: RMSNorm * k_gamma + IMROPE, then fp16
 * at row state->pos of k_cache.  V heads: fp16 at row state->pos of v_cache.
 * IMROPE axis positions (pos, pos, pos, 0), theta scale theta_scale (host
 * double; the reference's runtime value is the fp32 0x3f492c27).
 * Caches: fp16 [kv_heads][ctx][128].  pos outside [0, ctx) sets device error
 * bit 4 (mask 0x10) and appends nothing.  The q part is the reference's
 * kernels/fused_q_imrope_runtime_fastpow.mojo:8-36 per head.
 */
int mllb_decode_qk_rope_append(const float *qkv, const float *q_gamma, const float *k_gamma,
                               const mllb_decode_state *state, double theta_scale, float *q_out, void *k_cache,
                               void *v_cache, int64_t q_heads, int64_t kv_heads, int64_t ctx, unsigned flags,
                               void *stream);

/* Scratch (in doubles) that mllb_decode_attention needs for these shapes on
 * the current device, or a negative MLLB_E* code. */
int64_t mllb_decode_attention_scratch(int64_t q_heads, int64_t kv_heads, int64_t ctx);

/*
 * Attention of the token at state->pos over cache rows 0..pos (grouped
 * query heads: q head h reads kv head h / (q_heads / kv_heads); ratio 1, 2,
 * 4 or 8): softmax(q . k / sqrt(128)) . v per q head, fp64 throughout,
 * split over context chunks into `scratch` and merged.  Writes out (fp32
 * q_heads x 128, may be NULL) and q8 (its Q8_1, the O projection input, may
 * be NULL).  Two kernels.  GGML flash_attn_ext on the fp16 cache (the
 * reference enables flash attention: integration/resident_decode.cpp:71).
 */
int mllb_decode_attention(const float *q, const void *k_cache, const void *v_cache, const mllb_decode_state *state,
                          double *scratch, int64_t scratch_doubles, float *out, void *q8, int64_t q_heads,
                          int64_t kv_heads, int64_t ctx, unsigned flags, void *stream);

/*
 * Fused form for the decode step: qkv is the raw fused QKV projection (as
 * mllb_decode_qk_rope_append takes it).  The kernel does the q-head RMSNorm
 * + q_gamma + IMROPE itself, appends the K row (RMSNorm + k_gamma + IMROPE,
 * fp16) and the V row (fp16) at state->pos, and attends as
 * mllb_decode_attention -- one launch fewer, the same numbers.  pos outside
 * [0, ctx) sets device error bit 4 (mask 0x10) and appends nothing.
 */
int mllb_decode_attention_qkv(const float *qkv, const float *q_gamma, const float *k_gamma, double theta_scale,
                              const mllb_decode_state *state, void *k_cache, void *v_cache, double *scratch,
                              int64_t scratch_doubles, float *out, void *q8, int64_t q_heads, int64_t kv_heads,
                              int64_t ctx, unsigned flags, void *stream);

/*
 * mllb_decode_attention_qkv without a scratch argument: the chunk partials go
 * to a 1 MiB array inside the library (q_heads x splits x 130 doubles must
 * fit in 131072; the decode shape, 32 heads x 18 chunks, uses 74880).  For
 * callers that cannot allocate a buffer (an interposer that only sees the
 * host framework's tensors and stream).  No counterpart in the reference.
 * Allocates nothing: the array's device address is looked up once per device
 * (cudaGetSymbolAddress) on the first call with that device current, so make
 * one call per device before capturing a stream.  Nothing in the array needs
 * to start at zero.  Calls that overlap in time share the array and race;
 * larger shapes return MLLB_EUNSUPPORTED.
 */
int mllb_decode_attention_qkv_noalloc(const float *qkv, const float *q_gamma, const float *k_gamma,
                                      double theta_scale, const mllb_decode_state *state, void *k_cache,
                                      void *v_cache, float *out, void *q8, int64_t q_heads, int64_t kv_heads,
                                      int64_t ctx, unsigned flags, void *stream);

/*
 * Q4_0 KV cache: the KV type of the reference's llama.cpp contexts
 * (integration/resident_decode.cpp:70, cp.type_k = cp.type_v =
 * GGML_TYPE_Q4_0; "-ctk q4_0 -ctv q4_0" in tools/run_prefill_bench.py:26).
 * GGML's Q4_0 block (fp16 d, 32 x 4 bits, value d * (q - 8)), held as three
 * planes so that every cache row is a 16-byte multiple:
 *   k_qs [kv_heads][ctx][64]  nibbles of the 4 blocks of a K row (16 bytes
 *                             per block: element e < 16 in the low nibble of
 *                             byte e, element e + 16 in its high nibble)
 *   v_qs [kv_heads][ctx][64]  the same for V
 *   kv_d [kv_heads][ctx][8]   fp16 d of K blocks 0..3, then of V blocks 0..3
 * All three 16-byte aligned for the attention entries.
 */

/*
 * Quantise rows [row0, row0 + rows) of every KV head into the Q4_0 cache from
 * fp32 k and v ([kv_heads][rows][128] each) by GGML's quantize_row_q4_0 rule
 * (the element of largest magnitude, first on ties, gives d = max / -8;
 * q = min(15, trunc(x * (1 / d) + 8.5)), the product and the sum each
 * rounded to fp32; 1 / d taken as 0 when d is 0).  The prefill write of the cache; llama.cpp's
 * set_rows into a Q4_0 cache.
 */
int mllb_kv_q4_0_store(const float *k, const float *v, void *k_qs, void *v_qs, void *kv_d, int64_t kv_heads,
                       int64_t ctx, int64_t row0, int64_t rows, unsigned flags, void *stream);

/*
 * mllb_decode_attention over the Q4_0 cache (row state->pos already stored,
 * e.g. by mllb_kv_q4_0_store).  Cache values enter the fp64 arithmetic
 * exactly (d * (q - 8)); scratch as mllb_decode_attention_scratch.
 */
int mllb_decode_attention_q4_0(const float *q, const void *k_qs, const void *v_qs, const void *kv_d,
                               const mllb_decode_state *state, double *scratch, int64_t scratch_doubles, float *out,
                               void *q8, int64_t q_heads, int64_t kv_heads, int64_t ctx, unsigned flags,
                               void *stream);

/*
 * mllb_decode_attention_qkv over the Q4_0 cache: the K row (RMSNorm + k_gamma
 * + IMROPE, fp32) and the V row (fp32) of the token are quantised by the
 * mllb_kv_q4_0_store rule and appended at state->pos.  GGML flash_attn_ext
 * with Q4_0 K/V, as the reference runs it (integration/resident_decode.cpp:70-71).
 */
int mllb_decode_attention_qkv_q4_0(const float *qkv, const float *q_gamma, const float *k_gamma, double theta_scale,
                                   const mllb_decode_state *state, void *k_qs, void *v_qs, void *kv_d,
                                   double *scratch, int64_t scratch_doubles, float *out, void *q8, int64_t q_heads,
                                   int64_t kv_heads, int64_t ctx, unsigned flags, void *stream);

/*
 * *key = max(*key, max over i of key(x[i], index_offset + i)) with the packed
 * key of mllb_token_key (the greedy argmax; for a row shard pass the shard's
 * first row as index_offset).  *key must hold INT64_MIN or an earlier
 * maximum.  GGML argmax / the reference's LogitValidation top-1
 * (integration/logit_validation.h:76-80).
 */
int mllb_argmax_f32(const float *x, int64_t n, int64_t index_offset, int64_t *key, unsigned flags, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MLLB200_H */
