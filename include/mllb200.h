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
#define MLLB_EUNSUPPORTED (-4) /* shape outside what this build implements */

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

/* Q8_1 `s` field convention (the dot products never read s). */
#define MLLB_Q8_1_S_D_SUMQ 0 /* s = fp16(fp16(d) * sum(q)): tools/generate_q4_matvec_fixtures.py:59 */
#define MLLB_Q8_1_S_SUM_X 1  /* s = fp16(sum(x)): GGML quantize_q8_1 */

int mllb_abi_version(void);

/* Message for the last failed call on this thread ("" if none). */
const char *mllb_last_error(void);

/*
 * Device error word: bit 0/1/2 = a kernel gave up a bounded (~1 s) wait on
 * its TMA pipeline (see csrc/common.cuh).  Copies the word of the current
 * device to *bits (synchronising), optionally clearing it.  0 in normal runs.
 */
int mllb_device_error(uint32_t *bits, int clear);

/*
 * Q8_1 quantiser: x[k] fp32 -> k/32 blocks of 36 bytes.  k % 32 == 0.
 * d = amax/127 (IEEE), q = roundf(x/d), d and s stored as fp16 (RNE).
 * Replaces GGML's quantize_q8_1 node the reference clones in front of every
 * matvec (benchmark/q4_compare.c:328-330; bytes checked at :351-357).
 */
int mllb_q8_1_quantize(const float *x, void *q8, int64_t k, int s_mode, void *stream);

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

#ifdef __cplusplus
}
#endif

#endif /* MLLB200_H */
