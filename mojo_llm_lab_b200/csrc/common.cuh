// Device-side building blocks shared by the decode hot-path kernels (sm_100a).
//
// * mbarrier + cp.async.bulk (the TMA bulk-copy engine) for streaming weight
//   tiles from HBM into shared memory without tying up registers;
// * bounded waits: every wait on an mbarrier gives up after ~1 s of
//   %globaltimer time (and an iteration cap), records an error bit in the
//   library's device error word and lets the kernel finish, so a lost
//   transaction can never hang the GPU;
// * exact conversions and warp reductions used by the fp64 row accumulation.
#pragma once

#include <climits>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mllb {

// Bits of the device error word (read with mllb_device_error()).
enum : uint32_t {
  kErrFullWaitTimeout = 1u << 0,   // consumer gave up waiting for a weight tile
  kErrEmptyWaitTimeout = 1u << 1,  // producer gave up waiting for a free stage
  kErrDrainTimeout = 1u << 2,      // producer gave up waiting for its last copies
  kErrBadToken = 1u << 3,          // decode: next-token key outside the vocabulary (row 0 used)
  kErrKvOverflow = 1u << 4,        // decode: position at or past the KV capacity (nothing written)
  kErrKvWaitTimeout = 1u << 5,     // decode attention gave up waiting for its K/V copies
  kErrPeerWaitTimeout = 1u << 6,   // peer all-gather gave up waiting for another rank's slice
  kErrGridWaitTimeout = 1u << 7,   // a grid-wide epilogue gave up waiting for the grid's other CTAs
};

// Device-resident state of a decode loop; mirrors mllb_decode_state of the
// public header (32 bytes).
struct DecodeState {
  long long next_token_key;  // packed (value, index) of the greedy next token
  int pos;                   // position / KV row of the token being decoded
  int token;                 // token being decoded (written by the embedding)
  int steps;                 // completed decode steps
  int reserved[3];
};
static_assert(sizeof(DecodeState) == 32, "decode state layout");

constexpr long long kNoToken = LLONG_MIN;

// 1 s of wall time, and a hard iteration cap behind it.
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr uint32_t kWaitMaxIters = 1u << 28;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase of `bar` with the given parity to complete.  Returns
// false (after ~1 s) if it never does; the caller records the error.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 0; i < kWaitMaxIters; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && global_timer_ns() - start > kWaitLimitNs) break;
  }
  return false;
}

// ---- cross-GPU signalling (peer memory mapped over NVLink)

// *addr += v on (possibly another GPU's) memory, relaxed, system scope; the
// caller orders its data before it with fence_sys().
__device__ __forceinline__ void red_relaxed_sys_add(uint32_t* addr, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

// Polling load of a counter that other GPUs update (not cached in L1).
__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// L2 policy for data read exactly once (weights): evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// L2 policy for data fetched ahead of its use (next layer's weights): evict last.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// TMA bulk prefetch global -> L2 (no shared memory, no completion to wait
// for).  addr 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* addr, uint32_t bytes, uint64_t policy) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(addr), "r"(bytes), "l"(policy)
               : "memory");
}

// TMA bulk copy global -> shared, completion signalled on `bar` (tx bytes).
// dst and src must be 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch (PDL).  launch_dependents lets the next
// kernel in the stream start its prologue (e.g. streaming constant weights)
// while this one finishes; wait_prerequisite blocks until the preceding
// kernel has completed and its writes are visible.  Both are no-ops when the
// launches carry no programmatic-serialisation attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prerequisite() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over `threads` threads (id 0 is __syncthreads()).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// fp32 global load cached in L2 only: for values that other CTAs of the same
// grid wrote (ordered by a fence and an atomic arrival), which this SM's L1
// may hold stale.
__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ double ld_cg_f64(const double* p) {
  double v;
  asm volatile("ld.global.cg.f64 %0, [%1];" : "=d"(v) : "l"(p));
  return v;
}

// Arrival on a grid-wide counter: everything this thread wrote before (and,
// through a preceding CTA barrier and fence, what its CTA wrote) is visible
// to a thread that acquires the new value.
__device__ __forceinline__ uint32_t atom_add_release_gpu(uint32_t* addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// Arrival that both publishes this thread's earlier writes (release) and,
// for the thread that sees the final count, acquires everyone else's.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Wait until *count reaches target (the other CTAs of this grid arriving).
// Only for grids whose CTAs are all resident at once.  Returns false (after
// ~1 s) if it never does; the caller records the error.
__device__ __forceinline__ bool wait_count_bounded(const uint32_t* count, uint32_t target) {
  if (ld_acquire_gpu_u32(count) >= target) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 0; i < kWaitMaxIters; ++i) {
    if (ld_acquire_gpu_u32(count) >= target) return true;
    if (i >= 1024) __nanosleep(64);  // spin first: the grid usually gathers within microseconds
    if ((i & 63u) == 63u && global_timer_ns() - start > kWaitLimitNs) break;
  }
  return false;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream128(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// dot of 4 unsigned bytes with 4 signed bytes, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// Sum of the 4 signed bytes of w.
__device__ __forceinline__ int byte_sum_s8(uint32_t w, int c) { return dp4a_us(0x01010101u, w, c); }

// fp16 bit pattern -> double, exact (fp16 -> fp32 is exact, fp32 -> fp64 is exact).
__device__ __forceinline__ double half_bits_to_double(uint32_t bits16) {
  return static_cast<double>(__half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu))));
}

// int32 -> double, exact, on the fp64 pipe: the double with high word
// 0x43300000 and low word (x ^ 2^31) is 2^52 + 2^31 + x; subtracting
// 2^52 + 2^31 leaves x (every int32 is representable).  Avoids the
// conversion unit, which the inner loops would otherwise saturate.
__device__ __forceinline__ double i2d_exact(int x) {
  return __hiloint2double(0x43300000, static_cast<int>(static_cast<uint32_t>(x) ^ 0x80000000u)) -
         4503601774854144.0;
}

__device__ __forceinline__ double warp_sum_double(double v) {
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
  return v;
}

__device__ __forceinline__ float warp_max_float(float v) {
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
  return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
  return v;
}

// Sum of 32 floats in xor-butterfly order (offsets 16, 8, 4, 2, 1).
__device__ __forceinline__ float warp_sum_float_butterfly(float v) {
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
  return v;
}

constexpr int gcd_constexpr(int a, int b) { return b == 0 ? a : gcd_constexpr(b, a % b); }

}  // namespace mllb

// The device error word of this module (bounded-wait timeouts).  Each module
// is one translation unit (the library is built from capi.cu alone), so this
// definition exists once per module.
__device__ uint32_t g_mllb_device_error;

namespace mllb {
__device__ __forceinline__ void record_error(uint32_t bits) { atomicOr(&g_mllb_device_error, bits); }
}  // namespace mllb

// Timeline instrumentation, compiled in only with -DMLLB_TRACE (a debug
// build): thread 0 of CTA b records %globaltimer at point p in
// g_mllb_trace[b][p].  Points of the streaming kernels: 0 start, 1 after the
// PDL wait, 2 activation staged, 3/5 first/second tile ready, 4/6 first/second
// tile computed, 7 exit.
#ifdef MLLB_TRACE
__device__ unsigned long long g_mllb_trace[4096][8];
#define MLLB_TRACE_POINT(p)                                                                  \
  do {                                                                                       \
    if (threadIdx.x == 0 && blockIdx.x < 4096) g_mllb_trace[blockIdx.x][p] = mllb::global_timer_ns(); \
  } while (0)
#define MLLB_TRACE_CTA(cta, p)                                                                    \
  do {                                                                                            \
    if (threadIdx.x == 0 && (cta) < 4096) g_mllb_trace[(cta)][p] = mllb::global_timer_ns();       \
  } while (0)
#else
#define MLLB_TRACE_POINT(p) \
  do {                      \
  } while (0)
#define MLLB_TRACE_CTA(cta, p) \
  do {                         \
  } while (0)
#endif
