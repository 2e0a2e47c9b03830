// extern "C" launchers of the decode hot path (declared in include/mllb200.h).
//
// The whole library is this one translation unit: every kernel header is
// included here, so device code needs no relocatable linking and each module
// owns exactly one device error word.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "mllb200.h"
#include "common.cuh"
#include "imrope.cuh"
#include "misc.cuh"
#include "q4k.cuh"
#include "q6k.cuh"
#include "q8_1.cuh"
#include "stream.cuh"
#include "decode.cuh"
#include "prefill.cuh"
#include "resident.cuh"

// Streaming-kernel configurations: V (row groups per tile), S (stages),
// TEAMS (consumer teams per CTA) per format, matrices and K/256.  Each can
// be overridden at build time (-DMLLB_CFG_...) for tuning sweeps.
#ifndef MLLB_CFG_Q4K_8
#define MLLB_CFG_Q4K_8 8, 8, 6
#endif
#ifndef MLLB_CFG_Q4K_10
#define MLLB_CFG_Q4K_10 8, 4, 3
#endif
// K = 2560 when every SM gets at most two 16-row tiles (N <= 32 x SMs): a
// two-stage ring issued whole at start and a footprint that leaves room for a
// second resident CTA, so the next kernel of a PDL chain streams its tiles
// while this one computes (4096 rows: 2.70 vs 3.07 us per launch).
#ifndef MLLB_CFG_Q4K_10_SMALL
#define MLLB_CFG_Q4K_10_SMALL 8, 2, 2
#endif
// Row tiles per SM up to which K = 2560 takes the small configuration.
#ifndef MLLB_Q4K_10_SMALL_TILES_PER_SM
#define MLLB_Q4K_10_SMALL_TILES_PER_SM 2
#endif
#ifndef MLLB_CFG_Q4K_16
#define MLLB_CFG_Q4K_16 8, 4, 3
#endif
#ifndef MLLB_CFG_Q4K_38
#define MLLB_CFG_Q4K_38 8, 2, 1
#endif
#ifndef MLLB_CFG_Q4K_DUAL_8
#define MLLB_CFG_Q4K_DUAL_8 8, 4, 4
#endif
#ifndef MLLB_CFG_Q4K_DUAL_10
#define MLLB_CFG_Q4K_DUAL_10 4, 6, 3
#endif
#ifndef MLLB_CFG_Q4K_DUAL_16
#define MLLB_CFG_Q4K_DUAL_16 4, 4, 2
#endif
#ifndef MLLB_CFG_Q5K_8
#define MLLB_CFG_Q5K_8 8, 8, 6
#endif
#ifndef MLLB_CFG_Q5K_10
#define MLLB_CFG_Q5K_10 4, 6, 4
#endif
// Q5_K, K = 2560, up to two 16-row tiles per SM (as the Q4_K small shape):
// 3.29 vs 3.88 us per launch at 4096 rows.
#ifndef MLLB_CFG_Q5K_10_SMALL
#define MLLB_CFG_Q5K_10_SMALL 8, 2, 2
#endif
#ifndef MLLB_CFG_Q5K_16
#define MLLB_CFG_Q5K_16 8, 4, 3
#endif
#ifndef MLLB_CFG_Q6K_8
#define MLLB_CFG_Q6K_8 4, 8, 6
#endif
#ifndef MLLB_CFG_Q6K_10
#define MLLB_CFG_Q6K_10 4, 6, 5
#endif
#ifndef MLLB_CFG_Q6K_16
#define MLLB_CFG_Q6K_16 4, 6, 3
#endif

namespace {

thread_local char g_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MLLB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  g_error[0] = '\0';
  return MLLB_OK;
}

// Launch with an optional programmatic-stream-serialisation attribute (PDL).
template <typename... Params, typename... Args>
cudaError_t launch(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

int launched(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MLLB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return check_launch(what);
}

bool known_flags(unsigned flags) { return (flags & ~static_cast<unsigned>(MLLB_LAUNCH_PDL)) == 0; }
bool known_flags_aux(unsigned flags) {
  return (flags & ~static_cast<unsigned>(MLLB_LAUNCH_PDL | MLLB_LAUNCH_CONST_AUX)) == 0;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

constexpr int kMaxDevices = 64;

int current_device(int* dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(MLLB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(MLLB_EUNSUPPORTED, "device index %d out of range", *dev);
  return MLLB_OK;
}

int sm_count(int dev) {
  static int cache[kMaxDevices] = {0};
  if (cache[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 1;
  }
  return cache[dev];
}

// Per-kernel, per-device launch preparation for the streaming kernels:
// opt in to the dynamic shared memory once and cache the resident CTAs per SM.
struct OccupancyEntry {
  const void* fn;
  int dev;
  int blocks_per_sm;
};
constexpr int kOccupancySlots = 256;
OccupancyEntry g_occupancy[kOccupancySlots];
int g_occupancy_used = 0;
std::mutex g_occupancy_mutex;

template <typename Kernel>
int stream_grid(Kernel kernel, int smem_bytes, int threads, int dev, int tiles, int* grid, int* per_sm) {
  const void* fn = reinterpret_cast<const void*>(kernel);
  int blocks_per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(g_occupancy_mutex);
    for (int i = 0; i < g_occupancy_used; ++i)
      if (g_occupancy[i].fn == fn && g_occupancy[i].dev == dev) blocks_per_sm = g_occupancy[i].blocks_per_sm;
    if (blocks_per_sm == 0) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
      if (e != cudaSuccess) return fail(MLLB_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      int occ = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem_bytes);
      if (e != cudaSuccess) return fail(MLLB_ECUDA, "occupancy query: %s", cudaGetErrorString(e));
      blocks_per_sm = occ > 0 ? occ : 1;
      if (g_occupancy_used < kOccupancySlots) g_occupancy[g_occupancy_used++] = {fn, dev, blocks_per_sm};
    }
  }
  const int wave = sm_count(dev) * blocks_per_sm;
  *grid = tiles < wave ? tiles : wave;
  *per_sm = blocks_per_sm;
  return MLLB_OK;
}

// Resident CTAs per SM a PDL launch may take: leaving room on every SM lets
// the next kernel of a chain start streaming its weights before this one
// ends.  Default: all but one of the CTAs that fit; tuning knob
// MLLB_PDL_CTAS_PER_SM overrides it.
// One persistent CTA per SM: every SM takes an equal share of the tiles, and
// a second CTA slot stays free so that the next kernel of a stream can start
// (and stream its weights) while this one finishes.  Tuning knob
// MLLB_CTAS_PER_SM overrides the 1.
int grid_cap(int dev, int grid, int per_sm) {
  static const int env_cap = [] {
    const char* env = getenv("MLLB_CTAS_PER_SM");
    return env ? atoi(env) : 0;
  }();
  int ctas = env_cap > 0 ? env_cap : 1;
  if (ctas > per_sm) ctas = per_sm;
  const int cap = sm_count(dev) * ctas;
  return grid < cap ? grid : cap;
}

template <class Fmt, int NB, int MATS, int V, int S, int TEAMS, bool PRODUCE, int EPI = mllb::kEpiNone>
int launch_team_kernel(const uint8_t* w0, const uint8_t* w1, const mllb::ActSource& src, float* o0, float* o1,
                       float* o2, int n, cudaStream_t stream, bool pdl, const mllb::Epilogue& epi = {}) {
  using C = mllb::TeamConfig<Fmt, NB, MATS, V, S, TEAMS>;
  int dev, grid, per_sm, rc;
  if ((rc = current_device(&dev))) return rc;
  auto kernel = mllb::team_stream_kernel<Fmt, NB, MATS, V, S, TEAMS, PRODUCE, EPI>;
  const int tiles = (n + C::kT - 1) / C::kT;
  if ((rc = stream_grid(kernel, C::kSmemBytes, C::kThreads, dev, tiles, &grid, &per_sm))) return rc;
  grid = grid_cap(dev, grid, per_sm);
  return launched(launch(kernel, dim3(grid), dim3(C::kThreads), C::kSmemBytes, stream, pdl, w0, w1, src, o0, o1, o2,
                         n, pdl ? 1 : 0, epi),
                  "streaming matvec kernel");
}

// Activation staged from Q8_1 (src.q8) or built in the kernel (src.x).
template <class Fmt, int NB, int MATS, int V, int S, int TEAMS>
int launch_team(const uint8_t* w0, const uint8_t* w1, const mllb::ActSource& src, float* o0, float* o1, float* o2,
                int n, cudaStream_t stream, bool pdl) {
  if (src.x)
    return launch_team_kernel<Fmt, NB, MATS, V, S, TEAMS, true>(w0, w1, src, o0, o1, o2, n, stream, pdl);
  return launch_team_kernel<Fmt, NB, MATS, V, S, TEAMS, false>(w0, w1, src, o0, o1, o2, n, stream, pdl);
}

int check_rows(int64_t n, int64_t k, int64_t max_rows) {
  if (n <= 0 || n > max_rows) return fail(MLLB_EINVAL, "row count %lld out of range", static_cast<long long>(n));
  if (k <= 0 || k % 256) return fail(MLLB_EINVAL, "K=%lld is not a positive multiple of 256", static_cast<long long>(k));
  if (k / 256 > 4096) return fail(MLLB_EUNSUPPORTED, "K=%lld too large", static_cast<long long>(k));
  return MLLB_OK;
}

mllb::ActSource q8_source(const uint8_t* q8) {
  mllb::ActSource src = {};
  src.q8 = q8;
  return src;
}

// Streaming Q4_K launch for the shapes with a team configuration; returns
// MLLB_EUNSUPPORTED (and launches nothing) for the others.
int q4k_team(const uint8_t* w0, const uint8_t* w1, const mllb::ActSource& src, float* o0, float* o1, float* o2,
             int64_t n, int64_t k, cudaStream_t stream, bool pdl) {
  using F = mllb::Q4kFormat;
  const int nb = static_cast<int>(k / 256);
  const int rows = static_cast<int>(n);
  if (w1 == nullptr) {
    switch (nb) {
      case 8: return launch_team<F, 8, 1, MLLB_CFG_Q4K_8>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
      case 10: {
        using Small = mllb::TeamConfig<F, 10, 1, MLLB_CFG_Q4K_10_SMALL>;
        int dev, rc;
        if ((rc = current_device(&dev))) return rc;
        if ((rows + Small::kT - 1) / Small::kT <= MLLB_Q4K_10_SMALL_TILES_PER_SM * sm_count(dev))
          return launch_team<F, 10, 1, MLLB_CFG_Q4K_10_SMALL>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
        return launch_team<F, 10, 1, MLLB_CFG_Q4K_10>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
      }
      case 16: return launch_team<F, 16, 1, MLLB_CFG_Q4K_16>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
      case 38: return launch_team<F, 38, 1, MLLB_CFG_Q4K_38>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
      default: break;
    }
  } else {
    switch (nb) {
      case 8: return launch_team<F, 8, 2, MLLB_CFG_Q4K_DUAL_8>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
      case 10: return launch_team<F, 10, 2, MLLB_CFG_Q4K_DUAL_10>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
      case 16: return launch_team<F, 16, 2, MLLB_CFG_Q4K_DUAL_16>(w0, w1, src, o0, o1, o2, rows, stream, pdl);
      default: break;
    }
  }
  return fail(MLLB_EUNSUPPORTED, "no streaming configuration for K=%lld%s", static_cast<long long>(k),
              w1 ? " (gate/up)" : "");
}

// Q4_K gate/up streaming launch with the Q8_1 of the product fused in
// (Q8_1 activation).
template <int E = mllb::kEpiQuantProduct>
int q4k_gate_up_q8_team(const uint8_t* w0, const uint8_t* w1, const uint8_t* q8, float* o0, float* o1, float* o2,
                        int64_t n, int64_t k, cudaStream_t stream, bool pdl, const mllb::Epilogue& epi) {
  using F = mllb::Q4kFormat;
  const mllb::ActSource src = q8_source(q8);
  const int rows = static_cast<int>(n);
  switch (k / 256) {
    case 8: return launch_team_kernel<F, 8, 2, MLLB_CFG_Q4K_DUAL_8, false, E>(w0, w1, src, o0, o1, o2, rows, stream, pdl, epi);
    case 10: return launch_team_kernel<F, 10, 2, MLLB_CFG_Q4K_DUAL_10, false, E>(w0, w1, src, o0, o1, o2, rows, stream, pdl, epi);
    case 16: return launch_team_kernel<F, 16, 2, MLLB_CFG_Q4K_DUAL_16, false, E>(w0, w1, src, o0, o1, o2, rows, stream, pdl, epi);
    default: break;
  }
  return fail(MLLB_EUNSUPPORTED, "no gate/up configuration for K=%lld", static_cast<long long>(k));
}

// Q4_K streaming launch with the residual + RMSNorm + Q8_1 epilogue
// (kEpiResidualNorm; Q8_1 activation).
int q4k_norm_team(const uint8_t* w, const uint8_t* q8, float* out, int64_t n, int64_t k, cudaStream_t stream,
                  bool pdl, const mllb::Epilogue& epi) {
  using F = mllb::Q4kFormat;
  constexpr int E = mllb::kEpiResidualNorm;
  const mllb::ActSource src = q8_source(q8);
  const int rows = static_cast<int>(n);
  switch (k / 256) {
    case 8: return launch_team_kernel<F, 8, 1, MLLB_CFG_Q4K_8, false, E>(w, nullptr, src, out, nullptr, nullptr, rows, stream, pdl, epi);
    case 10: {
      using Small = mllb::TeamConfig<F, 10, 1, MLLB_CFG_Q4K_10_SMALL>;
      int dev, rc;
      if ((rc = current_device(&dev))) return rc;
      if ((rows + Small::kT - 1) / Small::kT <= MLLB_Q4K_10_SMALL_TILES_PER_SM * sm_count(dev))
        return launch_team_kernel<F, 10, 1, MLLB_CFG_Q4K_10_SMALL, false, E>(w, nullptr, src, out, nullptr, nullptr, rows, stream, pdl, epi);
      return launch_team_kernel<F, 10, 1, MLLB_CFG_Q4K_10, false, E>(w, nullptr, src, out, nullptr, nullptr, rows, stream, pdl, epi);
    }
    case 16: return launch_team_kernel<F, 16, 1, MLLB_CFG_Q4K_16, false, E>(w, nullptr, src, out, nullptr, nullptr, rows, stream, pdl, epi);
    case 38: return launch_team_kernel<F, 38, 1, MLLB_CFG_Q4K_38, false, E>(w, nullptr, src, out, nullptr, nullptr, rows, stream, pdl, epi);
    default: break;
  }
  return fail(MLLB_EUNSUPPORTED, "no streaming configuration for K=%lld", static_cast<long long>(k));
}

// Resident-weights path (csrc/resident.cuh): a plain Q4_K or Q5_K matvec of
// at most 32 rows per SM with K = 2560 or 4096 runs with all its weights in
// shared memory, brought in before the dependency wait.  MLLB_EUNSUPPORTED
// (nothing launched) for other shapes.  MLLB_Q4K_RESIDENT=0 turns it off (the
// streaming kernels then take every shape).
template <int NB, bool kQ5>
int launch_resident(int dev, const uint8_t* w, const uint8_t* q8, float* out, int rows, int per_cta,
                    cudaStream_t stream, bool pdl) {
  auto kernel = kQ5 ? mllb::resident_q5k_kernel<NB> : mllb::resident_q4k_kernel<NB>;
  constexpr int block_bytes = mllb::ResidentBlock<kQ5>::kBytes;
  static std::once_flag once[kMaxDevices];
  static cudaError_t attr_err[kMaxDevices];
  std::call_once(once[dev], [&] {
    attr_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         mllb::kResidentMaxRowsPerCta * NB * block_bytes);
  });
  if (attr_err[dev] != cudaSuccess)
    return fail(MLLB_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err[dev]));
  const int grid = (rows + per_cta - 1) / per_cta;
  const int threads = 32 * ((per_cta + 1) / 2);
  const size_t smem = static_cast<size_t>(per_cta) * NB * block_bytes;
  return launched(launch(kernel, dim3(grid), dim3(threads), smem, stream, pdl, w, q8, out, rows, per_cta),
                  kQ5 ? "resident Q5_K matvec kernel" : "resident Q4_K matvec kernel");
}

template <bool kQ5>
int k_resident(const uint8_t* w, const uint8_t* q8, float* out, int64_t n, int64_t k, cudaStream_t stream,
               bool pdl) {
  static const bool enabled = [] {
    const char* env = getenv("MLLB_Q4K_RESIDENT");
    return !(env && env[0] == '0');
  }();
  if (!enabled) return MLLB_EUNSUPPORTED;
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  const int sms = sm_count(dev);
  if (n > static_cast<int64_t>(sms) * mllb::kResidentMaxRowsPerCta) return MLLB_EUNSUPPORTED;
  const int rows = static_cast<int>(n);
  const int per_cta = (rows + sms - 1) / sms;
  switch (k / 256) {
    case 10: return launch_resident<10, kQ5>(dev, w, q8, out, rows, per_cta, stream, pdl);
    case 16: return launch_resident<16, kQ5>(dev, w, q8, out, rows, per_cta, stream, pdl);
    default: return MLLB_EUNSUPPORTED;
  }
}

int q4k_resident(const uint8_t* w, const uint8_t* q8, float* out, int64_t n, int64_t k, cudaStream_t stream,
                 bool pdl) {
  return k_resident<false>(w, q8, out, n, k, stream, pdl);
}

int q4k_dispatch(const uint8_t* w0, const uint8_t* w1, const uint8_t* q8, float* o0, float* o1, float* o2,
                 int64_t n, int64_t k, cudaStream_t stream, bool pdl) {
  if (w1 == nullptr) {
    const int rr = q4k_resident(w0, q8, o0, n, k, stream, pdl);
    if (rr != MLLB_EUNSUPPORTED) return rr;
  }
  const int rc = q4k_team(w0, w1, q8_source(q8), o0, o1, o2, n, k, stream, pdl);
  if (rc != MLLB_EUNSUPPORTED) return rc;
  // The row kernel reads its weights only after the preceding kernel is done,
  // so it never takes the PDL attribute.
  mllb::q4k_rowblock_kernel<<<static_cast<int>(n), 128, 0, stream>>>(w0, w1, q8, o0, o1, o2,
                                                                      static_cast<int>(k / 256));
  return check_launch("q4k row kernel");
}

// Q6_K streaming launch (rows a multiple of 8); MLLB_EUNSUPPORTED for other K.
int q6k_team(const uint8_t* w, const mllb::ActSource& src, float* out, int64_t rows, int64_t k, cudaStream_t s,
             bool pdl) {
  using F = mllb::Q6kFormat;
  const int mr = static_cast<int>(rows);
  switch (k / 256) {
    case 8: return launch_team<F, 8, 1, MLLB_CFG_Q6K_8>(w, nullptr, src, out, nullptr, nullptr, mr, s, pdl);
    case 10: return launch_team<F, 10, 1, MLLB_CFG_Q6K_10>(w, nullptr, src, out, nullptr, nullptr, mr, s, pdl);
    case 16: return launch_team<F, 16, 1, MLLB_CFG_Q6K_16>(w, nullptr, src, out, nullptr, nullptr, mr, s, pdl);
    default: return fail(MLLB_EUNSUPPORTED, "no Q6_K streaming configuration for K=%lld", static_cast<long long>(k));
  }
}

// Validate a host-side mllb_act_f32 and turn it into the kernel's ActSource.
int act_source(const mllb_act_f32* a, int64_t k, mllb::ActSource* src) {
  if (!a || !a->x) return fail(MLLB_EINVAL, "null pointer: activation source");
  if (k > 65536) return fail(MLLB_EUNSUPPORTED, "K=%lld too large for an in-kernel activation", static_cast<long long>(k));
  if (!aligned(a->x, 4) || !aligned(a->delta, 4) || !aligned(a->gamma, 4) || !aligned(a->x_out, 4) ||
      !aligned(a->advance, 8))
    return fail(MLLB_EALIGN, "activation pointers must be 4-byte (state 8-byte) aligned");
  const auto overlaps = [](const float* p, const float* q, int64_t n) { return p && q && p < q + n && q < p + n; };
  if (overlaps(a->x_out, a->x, k) || overlaps(a->x_out, a->delta, k))
    return fail(MLLB_EINVAL, "x_out must not overlap x or delta");
  if (a->gamma && !(a->eps >= 0.0)) return fail(MLLB_EINVAL, "eps must be >= 0");
  *src = {};
  src->x = a->x;
  src->delta = a->delta;
  src->gamma = a->gamma;
  src->x_out = a->x_out;
  src->eps = a->eps;
  src->advance = reinterpret_cast<mllb::DecodeState*>(a->advance);
  return MLLB_OK;
}

}  // namespace

#ifdef MLLB_TRACE
// Debug-build accessors of the timeline buffer (not part of the public ABI).
extern "C" int mllb_trace_read(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_mllb_trace, sizeof(g_mllb_trace)) == cudaSuccess ? MLLB_OK : MLLB_ECUDA;
}
extern "C" int mllb_trace_clear(void) {
  static unsigned long long zeros[4096 * 8];
  return cudaMemcpyToSymbol(g_mllb_trace, zeros, sizeof(zeros)) == cudaSuccess ? MLLB_OK : MLLB_ECUDA;
}
#endif

extern "C" {

int mllb_abi_version(void) { return MLLB_ABI_VERSION; }

const char* mllb_last_error(void) { return g_error; }

int mllb_device_error(uint32_t* bits, int clear) {
  if (!bits) return fail(MLLB_EINVAL, "null pointer: bits");
  cudaError_t e = cudaMemcpyFromSymbol(bits, g_mllb_device_error, sizeof(uint32_t));
  if (e != cudaSuccess) return fail(MLLB_ECUDA, "reading the device error word: %s", cudaGetErrorString(e));
  if (clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_mllb_device_error, &zero, sizeof(uint32_t));
    if (e != cudaSuccess) return fail(MLLB_ECUDA, "clearing the device error word: %s", cudaGetErrorString(e));
  }
  return MLLB_OK;
}

int mllb_q8_1_quantize(const float* x, void* q8, int64_t k, int s_mode, void* stream) {
  return mllb_q8_1_quantize_ex(x, q8, k, s_mode, 0u, stream);
}

int mllb_q8_1_quantize_ex(const float* x, void* q8, int64_t k, int s_mode, unsigned flags, void* stream) {
  if (!x || !q8) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (k <= 0 || k % 32) return fail(MLLB_EINVAL, "k=%lld is not a positive multiple of 32", static_cast<long long>(k));
  if (s_mode != MLLB_Q8_1_S_D_SUMQ && s_mode != MLLB_Q8_1_S_SUM_X) return fail(MLLB_EINVAL, "unknown s_mode %d", s_mode);
  if (!aligned(x, 4) || !aligned(q8, 4)) return fail(MLLB_EALIGN, "x and q8 must be 4-byte aligned");
  const int64_t blocks = k / 32;
  if (aligned(x, 16)) {  // four values per lane (one 16-byte load each)
    int64_t grid = (blocks + 31) / 32;
    if (grid > 65535) grid = 65535;
    return launched(launch(mllb::q8_1_quantize_x4_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL, x, static_cast<uint8_t*>(q8),
                           blocks, s_mode),
                    "q8_1 quantize kernel");
  }
  int64_t grid = (blocks + 7) / 8;
  if (grid > 65535) grid = 65535;
  return launched(launch(mllb::q8_1_quantize_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0,
                         static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL, x, static_cast<uint8_t*>(q8),
                         blocks, s_mode),
                  "q8_1 quantize kernel");
}

int mllb_q4k_matvec(const void* weights, const void* q8, float* out, int64_t n, int64_t k, void* stream) {
  return mllb_q4k_matvec_ex(weights, q8, out, n, k, 0u, stream);
}

int mllb_q4k_matvec_ex(const void* weights, const void* q8, float* out, int64_t n, int64_t k, unsigned flags,
                       void* stream) {
  if (!weights || !q8 || !out) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (!aligned(weights, 16) || !aligned(q8, 4) || !aligned(out, 4))
    return fail(MLLB_EALIGN, "weights need 16-byte, q8/out 4-byte alignment");
  return q4k_dispatch(static_cast<const uint8_t*>(weights), nullptr, static_cast<const uint8_t*>(q8), out, nullptr,
                      nullptr, n, k, static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL);
}

int mllb_q4k_gate_up(const void* up_weights, const void* gate_weights, const void* q8, float* up, float* gate,
                     float* prod, int64_t n, int64_t k, void* stream) {
  return mllb_q4k_gate_up_ex(up_weights, gate_weights, q8, up, gate, prod, n, k, 0u, stream);
}

int mllb_q4k_gate_up_ex(const void* up_weights, const void* gate_weights, const void* q8, float* up, float* gate,
                        float* prod, int64_t n, int64_t k, unsigned flags, void* stream) {
  if (!up_weights || !gate_weights || !q8) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (!up && !gate && !prod) return fail(MLLB_EINVAL, "no output requested");
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (!aligned(up_weights, 16) || !aligned(gate_weights, 16) || !aligned(q8, 4) || !aligned(up, 4) ||
      !aligned(gate, 4) || !aligned(prod, 4))
    return fail(MLLB_EALIGN, "weights need 16-byte, q8/outputs 4-byte alignment");
  return q4k_dispatch(static_cast<const uint8_t*>(up_weights), static_cast<const uint8_t*>(gate_weights),
                      static_cast<const uint8_t*>(q8), up, gate, prod, n, k, static_cast<cudaStream_t>(stream),
                      flags & MLLB_LAUNCH_PDL);
}

int mllb_q6k_matvec(const void* weights, const void* q8, float* out, int64_t n, int64_t k, void* stream) {
  return mllb_q6k_matvec_ex(weights, q8, out, n, k, 0u, stream);
}

int mllb_q6k_matvec_ex(const void* weights, const void* q8, float* out, int64_t n, int64_t k, unsigned flags,
                       void* stream) {
  if (!weights || !q8 || !out) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  const bool pdl = flags & MLLB_LAUNCH_PDL;
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (!aligned(weights, 16) || !aligned(q8, 4) || !aligned(out, 4))
    return fail(MLLB_EALIGN, "weights need 16-byte, q8/out 4-byte alignment");
  const uint8_t* w = static_cast<const uint8_t*>(weights);
  const uint8_t* a = static_cast<const uint8_t*>(q8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nb = static_cast<int>(k / 256);
  // Streaming tiles are whole 16-byte runs only when rows * nb % 8 == 0;
  // the last (n % 8) rows go through the row-per-CTA kernel.
  const int64_t main_rows = n - n % 8;
  const int64_t tail = n - main_rows;
  if (main_rows > 0) {
    rc = q6k_team(w, q8_source(a), out, main_rows, k, s, pdl);
    if (rc == MLLB_EUNSUPPORTED) {
      mllb::q6k_rowblock_kernel<<<static_cast<int>(main_rows), 128, 0, s>>>(w, a, out, nb);
      rc = check_launch("q6k row kernel");
    }
    if (rc) return rc;
  }
  if (tail > 0) {
    mllb::q6k_rowblock_kernel<<<static_cast<int>(tail), 128, 0, s>>>(w + main_rows * nb * mllb::kQ6kBlockBytes, a,
                                                                     out + main_rows, nb);
    rc = check_launch("q6k row kernel (tail)");
  }
  return rc;
}

int mllb_rmsnorm_imrope_q_batched(const float* q, const float* gamma, const int32_t* positions,
                                  const float* theta_scale, double theta_value, float* out, int64_t tokens,
                                  int64_t heads_per_token, void* stream) {
  return mllb_rmsnorm_imrope_q_batched_ex(q, gamma, positions, theta_scale, theta_value, out, tokens, heads_per_token,
                                          0u, stream);
}

int mllb_rmsnorm_imrope_q_batched_ex(const float* q, const float* gamma, const int32_t* positions,
                                     const float* theta_scale, double theta_value, float* out, int64_t tokens,
                                     int64_t heads_per_token, unsigned flags, void* stream) {
  if (!q || !gamma || !positions || !out) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags_aux(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (tokens <= 0 || heads_per_token <= 0) return fail(MLLB_EINVAL, "empty shape");
  if (!aligned(q, 4) || !aligned(gamma, 4) || !aligned(positions, 4) || !aligned(out, 4) ||
      (theta_scale && !aligned(theta_scale, 4)))
    return fail(MLLB_EALIGN, "fp32/int32 pointers must be 4-byte aligned");
  const int64_t per_cta = heads_per_token < mllb::kImropeMaxHeadsPerCta ? heads_per_token : mllb::kImropeMaxHeadsPerCta;
  const int64_t grid = tokens * ((heads_per_token + per_cta - 1) / per_cta);
  if (grid > 0x7fffffff) return fail(MLLB_EUNSUPPORTED, "too many heads");
  return launched(launch(tokens > 1 ? mllb::imrope_q_kernel<true> : mllb::imrope_q_kernel<false>,
                         dim3(static_cast<unsigned>(grid)), dim3(static_cast<unsigned>(per_cta * 32)),
                         0, static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL, q, gamma, positions,
                         theta_scale, theta_value, out, tokens, heads_per_token,
                         (flags & MLLB_LAUNCH_CONST_AUX) ? 1 : 0),
                  "imrope kernel");
}

int mllb_rmsnorm_imrope_q(const float* q, const float* gamma, const int32_t* positions, const float* theta_scale,
                          float* out, int64_t heads, void* stream) {
  if (!theta_scale) return fail(MLLB_EINVAL, "null pointer: theta_scale");
  return mllb_rmsnorm_imrope_q_batched(q, gamma, positions, theta_scale, 0.0, out, 1, heads, stream);
}

int mllb_q4k_subdots(const void* weights, const void* q8, int32_t* dots, int32_t* asums, int64_t n, int64_t k,
                     void* stream) {
  if (!weights || !q8 || !dots || !asums) return fail(MLLB_EINVAL, "null pointer");
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (!aligned(weights, 4) || !aligned(q8, 4) || !aligned(dots, 4) || !aligned(asums, 4))
    return fail(MLLB_EALIGN, "pointers must be 4-byte aligned");
  const int64_t total = n * (k / 32) + k / 32;
  int64_t grid = (total + 255) / 256;
  if (grid > 65535) grid = 65535;
  mllb::q4k_subdots_kernel<<<static_cast<int>(grid), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(weights), static_cast<const uint8_t*>(q8), dots, asums, n,
      static_cast<int>(k / 256));
  return check_launch("q4k subdots kernel");
}

int mllb_stream_read(const void* data, int64_t bytes, void* out, int64_t blocks, void* stream) {
  if (!data || !out) return fail(MLLB_EINVAL, "null pointer");
  if (bytes <= 0 || bytes % 16) return fail(MLLB_EINVAL, "bytes must be a positive multiple of 16");
  if (!aligned(data, 16) || !aligned(out, 16)) return fail(MLLB_EALIGN, "data and out must be 16-byte aligned");
  if (blocks <= 0) {
    int dev, rc;
    if ((rc = current_device(&dev))) return rc;
    blocks = static_cast<int64_t>(sm_count(dev)) * 8;
  }
  if (blocks > 1 << 20) return fail(MLLB_EINVAL, "too many blocks");
  mllb::stream_read_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(data), bytes / 16, static_cast<uint4*>(out));
  return check_launch("stream read kernel");
}

}  // extern "C"

// ------------------------------------------------------------------ decode

namespace {

constexpr int64_t kAttnMaxSplits = 6144;  // combine weights: 48 KB of shared memory

// The long-context shape of the split kernel: LongShape<G>::kWarps warps
// (at least G), chunks of MLLB_ATTN_LONG_CHUNK keys, as many resident CTAs
// per SM as 128 registers a thread allow.  Only for 1 and 4 query heads per
// KV head (2 and 8 need more than 128 registers a thread and keep the
// default shape).  Build-time overridable for sweeps.
#ifndef MLLB_ATTN_LONG_WARPS
#define MLLB_ATTN_LONG_WARPS 8
#endif
#ifndef MLLB_ATTN_LONG_CHUNK
#define MLLB_ATTN_LONG_CHUNK 128
#endif
#ifndef MLLB_ATTN_LONG_ALWAYS
#define MLLB_ATTN_LONG_ALWAYS 0
#endif

template <int G>
struct LongShape {
  static constexpr int kWarps = G > MLLB_ATTN_LONG_WARPS ? G : MLLB_ATTN_LONG_WARPS;
  static constexpr int kCtas = 512 / (kWarps * 32) > 0 ? 512 / (kWarps * 32) : 1;
  template <int KV>
  using Config = mllb::AttnConfig<G, KV, kWarps, MLLB_ATTN_LONG_CHUNK, kCtas>;
};

struct AttnPlan {
  bool long_shape;
  int64_t splits;
};

// Context chunks per KV head for one shape: enough CTAs to give every SM
// its resident share, and chunks of at most the shape's chunk size.
template <class C>
int64_t shape_splits(int dev, int64_t kv_heads, int64_t ctx) {
  int64_t base = static_cast<int64_t>(sm_count(dev)) * C::kCtasPerSm / kv_heads;
  if (base < 1) base = 1;
  const int64_t need = (ctx + C::kMaxChunk - 1) / C::kMaxChunk;
  return base > need ? base : need;
}

// The default shape (one CTA per SM, up to 256 keys) while its chunks fit in
// one wave of CTAs; past that the long shape.
template <int G>
AttnPlan plan_for(int dev, int64_t kv_heads, int64_t ctx) {
  using D = mllb::AttnConfig<G>;
  const int64_t d = shape_splits<D>(dev, kv_heads, ctx);
  if constexpr (G == 1 || G == 4) {
    using L = typename LongShape<G>::template Config<mllb::kKvF16>;
    const int64_t one_wave = static_cast<int64_t>(sm_count(dev)) * D::kCtasPerSm / kv_heads;
    const int64_t l = shape_splits<L>(dev, kv_heads, ctx);
    if ((MLLB_ATTN_LONG_ALWAYS || d > one_wave) && l <= kAttnMaxSplits) return {true, l};
  }
  return {false, d};
}

AttnPlan attention_plan(int dev, int64_t q_heads, int64_t kv_heads, int64_t ctx) {
  switch (q_heads / kv_heads) {
    case 1: return plan_for<1>(dev, kv_heads, ctx);
    case 2: return plan_for<2>(dev, kv_heads, ctx);
    case 4: return plan_for<4>(dev, kv_heads, ctx);
    default: return plan_for<8>(dev, kv_heads, ctx);
  }
}

int check_attention_shape(int64_t q_heads, int64_t kv_heads, int64_t ctx) {
  if (q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
    return fail(MLLB_EINVAL, "q_heads=%lld is not a positive multiple of kv_heads=%lld",
                static_cast<long long>(q_heads), static_cast<long long>(kv_heads));
  const int64_t g = q_heads / kv_heads;
  if (g != 1 && g != 2 && g != 4 && g != 8)
    return fail(MLLB_EUNSUPPORTED, "query heads per KV head must be 1, 2, 4 or 8 (got %lld)", static_cast<long long>(g));
  if (ctx <= 0 || ctx > (1 << 24)) return fail(MLLB_EINVAL, "ctx=%lld out of range", static_cast<long long>(ctx));
  if (kv_heads > 65535) return fail(MLLB_EUNSUPPORTED, "too many KV heads");
  return MLLB_OK;
}

struct AttentionArgs {
  const float* q;        // rotated queries (unfused), or nullptr
  const float* qkv;      // raw QKV projection (fused), or nullptr
  const float* q_gamma;
  const float* k_gamma;
  double theta;
  int64_t q_heads, kv_heads, ctx;
  const mllb::DecodeState* state;
  uint8_t* k_cache;      // fp16 rows, or the Q4_0 K nibble plane
  uint8_t* v_cache;      // fp16 rows, or the Q4_0 V nibble plane
  uint8_t* kv_d;         // Q4_0 scale plane (nullptr for fp16)
  int kv;                // mllb::kKvF16 or mllb::kKvQ4_0
  bool long_shape;       // AttnPlan::long_shape
  double* part_acc;
  double* part_ml;
  int64_t splits;
};

template <class C, int G, int KV, int W, int CH, int CTAS>
int launch_shape(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  int dev, rc, grid, per_sm;
  if ((rc = current_device(&dev))) return rc;
  auto kernel = mllb::attn_split_kernel<G, KV, W, CH, CTAS>;
  if ((rc = stream_grid(kernel, C::kSmemBytes, C::kThreads, dev, 1, &grid, &per_sm))) return rc;
  return launched(launch(kernel, dim3(static_cast<unsigned>(a.splits), static_cast<unsigned>(a.kv_heads)),
                         dim3(C::kThreads), C::kSmemBytes, stream, pdl, a.q, a.qkv, a.q_gamma, a.k_gamma, a.theta,
                         static_cast<int>(a.q_heads), static_cast<int>(a.kv_heads), a.state, a.k_cache, a.v_cache,
                         a.kv_d, a.part_acc, a.part_ml, static_cast<int>(a.ctx), static_cast<int>(a.splits),
                         1.0 / sqrt(128.0)),
                  "decode attention kernel");
}

template <int G, int KV>
int launch_attention(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  if constexpr (G == 1 || G == 4) {
    if (a.long_shape) {
      using S = LongShape<G>;
      using C = typename S::template Config<KV>;
      return launch_shape<C, G, KV, S::kWarps, MLLB_ATTN_LONG_CHUNK, S::kCtas>(a, stream, pdl);
    }
  }
  using C = mllb::AttnConfig<G, KV>;
  return launch_shape<C, G, KV, C::kWarps, C::kMaxChunk, C::kCtasPerSm>(a, stream, pdl);
}

// Split kernel + combine for both entry points.
int attention_impl(AttentionArgs a, double* scratch, int64_t scratch_doubles, float* out, void* q8, unsigned flags,
                   void* stream) {
  if (!a.k_cache || !a.v_cache || !a.state || !scratch) return fail(MLLB_EINVAL, "null pointer");
  if (a.kv == mllb::kKvQ4_0 && (!a.kv_d || !aligned(a.kv_d, 16)))
    return fail(!a.kv_d ? MLLB_EINVAL : MLLB_EALIGN, "the Q4_0 scale plane must be non-null and 16-byte aligned");
  if (!out && !q8) return fail(MLLB_EINVAL, "no output requested");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_attention_shape(a.q_heads, a.kv_heads, a.ctx);
  if (rc) return rc;
  if (!aligned(a.q, 16) || !aligned(a.qkv, 16) || !aligned(a.q_gamma, 4) || !aligned(a.k_gamma, 4) ||
      !aligned(a.k_cache, 16) || !aligned(a.v_cache, 16) || !aligned(a.state, 8) || !aligned(scratch, 8) ||
      !aligned(out, 4) || !aligned(q8, 4))
    return fail(MLLB_EALIGN, "q/qkv and caches need 16-byte, state/scratch 8-byte, others 4-byte alignment");
  int dev;
  if ((rc = current_device(&dev))) return rc;
  const AttnPlan plan = attention_plan(dev, a.q_heads, a.kv_heads, a.ctx);
  a.splits = plan.splits;
  a.long_shape = plan.long_shape;
  const int64_t need = a.q_heads * a.splits * (128 + 2);
  if (scratch_doubles < need)
    return fail(MLLB_EINVAL, "scratch holds %lld doubles, %lld needed", static_cast<long long>(scratch_doubles),
                static_cast<long long>(need));
  if (a.splits > kAttnMaxSplits) return fail(MLLB_EUNSUPPORTED, "context too long");
  a.part_acc = scratch;
  a.part_ml = scratch + a.q_heads * a.splits * 128;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = flags & MLLB_LAUNCH_PDL;
  const bool q4 = a.kv == mllb::kKvQ4_0;
  switch (a.q_heads / a.kv_heads) {
    case 1: rc = q4 ? launch_attention<1, mllb::kKvQ4_0>(a, s, pdl) : launch_attention<1, mllb::kKvF16>(a, s, pdl); break;
    case 2: rc = q4 ? launch_attention<2, mllb::kKvQ4_0>(a, s, pdl) : launch_attention<2, mllb::kKvF16>(a, s, pdl); break;
    case 4: rc = q4 ? launch_attention<4, mllb::kKvQ4_0>(a, s, pdl) : launch_attention<4, mllb::kKvF16>(a, s, pdl); break;
    default: rc = q4 ? launch_attention<8, mllb::kKvQ4_0>(a, s, pdl) : launch_attention<8, mllb::kKvF16>(a, s, pdl); break;
  }
  if (rc) return rc;
  return launched(launch(mllb::attn_combine_kernel, dim3(static_cast<unsigned>(a.q_heads)), dim3(128),
                         static_cast<size_t>(a.splits) * sizeof(double), s, pdl,
                         static_cast<const double*>(a.part_acc), static_cast<const double*>(a.part_ml),
                         static_cast<int>(a.splits), out, static_cast<uint8_t*>(q8), MLLB_Q8_1_S_D_SUMQ),
                  "attention combine kernel");
}

// Scratch of mllb_decode_attention_qkv_noalloc: chunk partials in a
// file-scope device array (1 MiB), so that entry allocates nothing.  Every
// partial is written before it is read within a call: nothing needs to start
// at zero.  Calls that overlap in time (other streams, other host threads)
// share it and would race.
constexpr int64_t kNoAllocScratchDoubles = 131072;
static __device__ __align__(256) double g_attn_noalloc_scratch[kNoAllocScratchDoubles];

// Device address of g_attn_noalloc_scratch for the current device, looked up
// with cudaGetSymbolAddress on the first call per device and cached.
int noalloc_scratch(double** out) {
  static double* cache[kMaxDevices] = {nullptr};
  static std::mutex m;
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  std::lock_guard<std::mutex> lock(m);
  if (!cache[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess) return fail(MLLB_ECUDA, "cudaGetSymbolAddress(attention scratch): %s", cudaGetErrorString(e));
    cache[dev] = static_cast<double*>(p);
  }
  *out = cache[dev];
  return MLLB_OK;
}

int rmsnorm_q8_1_launch(const float* x, const float* delta, float* x_out, const float* gamma, double eps, void* q8,
                        int64_t k, int s_mode, mllb::DecodeState* advance, unsigned flags, void* stream) {
  if (!x || !gamma || !q8) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (k <= 0 || k % 32 || k > 32768)
    return fail(MLLB_EINVAL, "k=%lld is not a positive multiple of 32 up to 32768", static_cast<long long>(k));
  if (s_mode != MLLB_Q8_1_S_D_SUMQ && s_mode != MLLB_Q8_1_S_SUM_X) return fail(MLLB_EINVAL, "unknown s_mode %d", s_mode);
  if (!(eps >= 0.0)) return fail(MLLB_EINVAL, "eps must be >= 0");
  if (!aligned(x, 4) || !aligned(delta, 4) || !aligned(x_out, 4) || !aligned(gamma, 4) || !aligned(q8, 4))
    return fail(MLLB_EALIGN, "fp32 and Q8_1 pointers must be 4-byte aligned");
  const auto overlaps = [](const float* a, const float* b, int64_t n) { return a && b && a < b + n && b < a + n; };
  if (overlaps(x_out, x, k) && x_out != x) return fail(MLLB_EINVAL, "x_out overlaps x without being x");
  if (overlaps(x_out, delta, k)) return fail(MLLB_EINVAL, "x_out overlaps delta");
  // In place (x_out == x) one CTA reads every x before any is written;
  // otherwise one CTA per 8 Q8_1 blocks, each summing all k squares itself.
  const int64_t blocks = k / 32;
  const int grid = x_out == x ? 1 : static_cast<int>((blocks + 7) / 8);
  return launched(launch(mllb::rmsnorm_q8_1_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream),
                         flags & MLLB_LAUNCH_PDL, x, delta, x_out, gamma, eps, static_cast<uint8_t*>(q8),
                         static_cast<int>(k), s_mode, advance),
                  "rmsnorm q8_1 kernel");
}

}  // namespace

extern "C" {

int64_t mllb_token_key(int32_t token) {
  return static_cast<int64_t>(0xffffffffull - static_cast<uint32_t>(token));
}

int64_t mllb_key_token(int64_t key) {
  if (key == INT64_MIN) return -1;
  return static_cast<int64_t>(0xffffffffull - (static_cast<uint64_t>(key) & 0xffffffffull));
}

int mllb_decode_embed(const void* q6k_weights, int64_t vocab, int64_t k, mllb_decode_state* state, int32_t* tokens,
                      int64_t capacity, float* hidden, unsigned flags, void* stream) {
  if (!q6k_weights || !state || !hidden) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (vocab <= 0 || vocab > 0xffffffffll) return fail(MLLB_EINVAL, "vocab=%lld out of range", static_cast<long long>(vocab));
  if (k <= 0 || k % 256 || k > (1 << 20))
    return fail(MLLB_EINVAL, "k=%lld is not a positive multiple of 256", static_cast<long long>(k));
  if (tokens && capacity < 0) return fail(MLLB_EINVAL, "negative capacity");
  if (!aligned(state, 8) || !aligned(hidden, 4) || (tokens && !aligned(tokens, 4)))
    return fail(MLLB_EALIGN, "state needs 8-byte, hidden/tokens 4-byte alignment");
  const int grid = static_cast<int>((k + 255) / 256);
  return launched(launch(mllb::embed_q6k_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream),
                         flags & MLLB_LAUNCH_PDL, static_cast<const uint8_t*>(q6k_weights),
                         static_cast<int>(k / 256), vocab, reinterpret_cast<mllb::DecodeState*>(state), tokens,
                         tokens ? capacity : 0, hidden),
                  "embedding kernel");
}

int mllb_rmsnorm_q8_1(const float* x, const float* delta, float* x_out, const float* gamma, double eps, void* q8,
                      int64_t k, int s_mode, unsigned flags, void* stream) {
  return rmsnorm_q8_1_launch(x, delta, x_out, gamma, eps, q8, k, s_mode, nullptr, flags, stream);
}

int mllb_decode_final_norm(const float* x, const float* delta, float* x_out, const float* gamma, double eps,
                           void* q8, int64_t k, mllb_decode_state* state, unsigned flags, void* stream) {
  if (!state) return fail(MLLB_EINVAL, "null pointer: state");
  if (!aligned(state, 8)) return fail(MLLB_EALIGN, "state needs 8-byte alignment");
  return rmsnorm_q8_1_launch(x, delta, x_out, gamma, eps, q8, k, MLLB_Q8_1_S_D_SUMQ,
                             reinterpret_cast<mllb::DecodeState*>(state), flags, stream);
}

int mllb_decode_qk_rope_append(const float* qkv, const float* q_gamma, const float* k_gamma,
                               const mllb_decode_state* state, double theta_scale, float* q_out, void* k_cache,
                               void* v_cache, int64_t q_heads, int64_t kv_heads, int64_t ctx, unsigned flags,
                               void* stream) {
  if (!qkv || !q_gamma || !k_gamma || !state || !q_out || !k_cache || !v_cache) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (q_heads <= 0 || kv_heads <= 0 || q_heads + 2 * kv_heads > (1 << 20))
    return fail(MLLB_EINVAL, "head counts out of range");
  if (ctx <= 0 || ctx > (1 << 24)) return fail(MLLB_EINVAL, "ctx=%lld out of range", static_cast<long long>(ctx));
  if (!(theta_scale > 0.0)) return fail(MLLB_EINVAL, "theta_scale must be positive");
  if (!aligned(qkv, 4) || !aligned(q_gamma, 4) || !aligned(k_gamma, 4) || !aligned(state, 8) || !aligned(q_out, 4) ||
      !aligned(k_cache, 2) || !aligned(v_cache, 2))
    return fail(MLLB_EALIGN, "fp32 pointers need 4-byte, caches 2-byte, state 8-byte alignment");
  const int64_t warps = q_heads + 2 * kv_heads;
  const int grid = static_cast<int>((warps + 3) / 4);
  return launched(launch(mllb::qk_rope_append_kernel, dim3(grid), dim3(128), 0, static_cast<cudaStream_t>(stream),
                         flags & MLLB_LAUNCH_PDL, qkv, q_gamma, k_gamma,
                         reinterpret_cast<const mllb::DecodeState*>(state), theta_scale, q_out,
                         static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), static_cast<int>(q_heads),
                         static_cast<int>(kv_heads), static_cast<int>(ctx)),
                  "q/k rope + KV append kernel");
}

int64_t mllb_decode_attention_scratch(int64_t q_heads, int64_t kv_heads, int64_t ctx) {
  int rc = check_attention_shape(q_heads, kv_heads, ctx);
  if (rc) return rc;
  int dev;
  if ((rc = current_device(&dev))) return rc;
  return q_heads * attention_plan(dev, q_heads, kv_heads, ctx).splits * (128 + 2);
}

int mllb_decode_attention(const float* q, const void* k_cache, const void* v_cache, const mllb_decode_state* state,
                          double* scratch, int64_t scratch_doubles, float* out, void* q8, int64_t q_heads,
                          int64_t kv_heads, int64_t ctx, unsigned flags, void* stream) {
  if (!q) return fail(MLLB_EINVAL, "null pointer: q");
  AttentionArgs a = {};
  a.q = q;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.ctx = ctx;
  a.state = reinterpret_cast<const mllb::DecodeState*>(state);
  // The unfused kernel only reads the caches.
  a.k_cache = static_cast<uint8_t*>(const_cast<void*>(k_cache));
  a.v_cache = static_cast<uint8_t*>(const_cast<void*>(v_cache));
  return attention_impl(a, scratch, scratch_doubles, out, q8, flags, stream);
}

int mllb_decode_attention_qkv(const float* qkv, const float* q_gamma, const float* k_gamma, double theta_scale,
                              const mllb_decode_state* state, void* k_cache, void* v_cache, double* scratch,
                              int64_t scratch_doubles, float* out, void* q8, int64_t q_heads, int64_t kv_heads,
                              int64_t ctx, unsigned flags, void* stream) {
  if (!qkv || !q_gamma || !k_gamma) return fail(MLLB_EINVAL, "null pointer");
  if (!(theta_scale > 0.0)) return fail(MLLB_EINVAL, "theta_scale must be positive");
  AttentionArgs a = {};
  a.qkv = qkv;
  a.q_gamma = q_gamma;
  a.k_gamma = k_gamma;
  a.theta = theta_scale;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.ctx = ctx;
  a.state = reinterpret_cast<const mllb::DecodeState*>(state);
  a.k_cache = static_cast<uint8_t*>(k_cache);
  a.v_cache = static_cast<uint8_t*>(v_cache);
  return attention_impl(a, scratch, scratch_doubles, out, q8, flags, stream);
}

int mllb_kv_q4_0_store(const float* k, const float* v, void* k_qs, void* v_qs, void* kv_d, int64_t kv_heads,
                       int64_t ctx, int64_t row0, int64_t rows, unsigned flags, void* stream) {
  if (!k || !v || !k_qs || !v_qs || !kv_d) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (kv_heads <= 0 || kv_heads > 65535) return fail(MLLB_EINVAL, "kv_heads=%lld out of range", static_cast<long long>(kv_heads));
  if (ctx <= 0 || ctx > (1 << 24)) return fail(MLLB_EINVAL, "ctx=%lld out of range", static_cast<long long>(ctx));
  if (rows <= 0 || row0 < 0 || row0 + rows > ctx)
    return fail(MLLB_EINVAL, "rows [%lld, %lld) outside the cache's %lld", static_cast<long long>(row0),
                static_cast<long long>(row0 + rows), static_cast<long long>(ctx));
  if (!aligned(k, 4) || !aligned(v, 4) || !aligned(kv_d, 2))
    return fail(MLLB_EALIGN, "k/v need 4-byte, kv_d 2-byte alignment");
  const int64_t warps = 2 * kv_heads * rows;
  if (warps / 4 >= (1ll << 31)) return fail(MLLB_EINVAL, "too many rows");
  return launched(launch(mllb::kv_q4_0_store_kernel, dim3(static_cast<unsigned>((warps + 3) / 4)), dim3(128), 0,
                         static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL, k, v,
                         static_cast<uint8_t*>(k_qs), static_cast<uint8_t*>(v_qs), static_cast<uint16_t*>(kv_d),
                         static_cast<int>(kv_heads), static_cast<int>(ctx), static_cast<int>(row0),
                         static_cast<int>(rows)),
                  "Q4_0 KV store kernel");
}

int mllb_decode_attention_q4_0(const float* q, const void* k_qs, const void* v_qs, const void* kv_d,
                               const mllb_decode_state* state, double* scratch, int64_t scratch_doubles, float* out,
                               void* q8, int64_t q_heads, int64_t kv_heads, int64_t ctx, unsigned flags,
                               void* stream) {
  if (!q) return fail(MLLB_EINVAL, "null pointer: q");
  AttentionArgs a = {};
  a.q = q;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.ctx = ctx;
  a.state = reinterpret_cast<const mllb::DecodeState*>(state);
  a.k_cache = static_cast<uint8_t*>(const_cast<void*>(k_qs));
  a.v_cache = static_cast<uint8_t*>(const_cast<void*>(v_qs));
  a.kv_d = static_cast<uint8_t*>(const_cast<void*>(kv_d));
  a.kv = mllb::kKvQ4_0;
  return attention_impl(a, scratch, scratch_doubles, out, q8, flags, stream);
}

int mllb_decode_attention_qkv_q4_0(const float* qkv, const float* q_gamma, const float* k_gamma, double theta_scale,
                                   const mllb_decode_state* state, void* k_qs, void* v_qs, void* kv_d,
                                   double* scratch, int64_t scratch_doubles, float* out, void* q8, int64_t q_heads,
                                   int64_t kv_heads, int64_t ctx, unsigned flags, void* stream) {
  if (!qkv || !q_gamma || !k_gamma) return fail(MLLB_EINVAL, "null pointer");
  if (!(theta_scale > 0.0)) return fail(MLLB_EINVAL, "theta_scale must be positive");
  AttentionArgs a = {};
  a.qkv = qkv;
  a.q_gamma = q_gamma;
  a.k_gamma = k_gamma;
  a.theta = theta_scale;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.ctx = ctx;
  a.state = reinterpret_cast<const mllb::DecodeState*>(state);
  a.k_cache = static_cast<uint8_t*>(k_qs);
  a.v_cache = static_cast<uint8_t*>(v_qs);
  a.kv_d = static_cast<uint8_t*>(kv_d);
  a.kv = mllb::kKvQ4_0;
  return attention_impl(a, scratch, scratch_doubles, out, q8, flags, stream);
}

int mllb_argmax_f32(const float* x, int64_t n, int64_t index_offset, int64_t* key, unsigned flags, void* stream) {
  if (!x || !key) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (n <= 0 || index_offset < 0 || index_offset + n > 0xffffffffll)
    return fail(MLLB_EINVAL, "indices must lie in [0, 2^32 - 1)");
  if (!aligned(x, 4) || !aligned(key, 8)) return fail(MLLB_EALIGN, "x needs 4-byte, key 8-byte alignment");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  int64_t grid = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * 2;
  if (grid > cap) grid = cap;
  return launched(launch(mllb::argmax_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0,
                         static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL, x, n, index_offset,
                         reinterpret_cast<long long*>(key)),
                  "argmax kernel");
}

}  // extern "C"

extern "C" {

int mllb_q4k_matvec_act(const void* weights, const mllb_act_f32* act, float* out, int64_t n, int64_t k,
                        unsigned flags, void* stream) {
  if (!weights || !out) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  mllb::ActSource src;
  if ((rc = act_source(act, k, &src))) return rc;
  if (!aligned(weights, 16) || !aligned(out, 4)) return fail(MLLB_EALIGN, "weights need 16-byte, out 4-byte alignment");
  return q4k_team(static_cast<const uint8_t*>(weights), nullptr, src, out, nullptr, nullptr, n, k,
                  static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL);
}

int mllb_q4k_gate_up_act(const void* up_weights, const void* gate_weights, const mllb_act_f32* act, float* up,
                         float* gate, float* prod, int64_t n, int64_t k, unsigned flags, void* stream) {
  if (!up_weights || !gate_weights) return fail(MLLB_EINVAL, "null pointer");
  if (!up && !gate && !prod) return fail(MLLB_EINVAL, "no output requested");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  mllb::ActSource src;
  if ((rc = act_source(act, k, &src))) return rc;
  if (!aligned(up_weights, 16) || !aligned(gate_weights, 16) || !aligned(up, 4) || !aligned(gate, 4) ||
      !aligned(prod, 4))
    return fail(MLLB_EALIGN, "weights need 16-byte, outputs 4-byte alignment");
  return q4k_team(static_cast<const uint8_t*>(up_weights), static_cast<const uint8_t*>(gate_weights), src, up,
                  gate, prod, n, k, static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL);
}

int mllb_q6k_matvec_act(const void* weights, const mllb_act_f32* act, float* out, int64_t n, int64_t k,
                        unsigned flags, void* stream) {
  if (!weights || !out) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (n % 8) return fail(MLLB_EUNSUPPORTED, "in-kernel activation needs a multiple of 8 rows");
  mllb::ActSource src;
  if ((rc = act_source(act, k, &src))) return rc;
  if (!aligned(weights, 16) || !aligned(out, 4)) return fail(MLLB_EALIGN, "weights need 16-byte, out 4-byte alignment");
  return q6k_team(static_cast<const uint8_t*>(weights), src, out, n, k, static_cast<cudaStream_t>(stream),
                  flags & MLLB_LAUNCH_PDL);
}

int mllb_q4k_gate_up_q8(const void* up_weights, const void* gate_weights, const void* q8, float* up, float* gate,
                        float* prod, void* q8_out, uint32_t* counters, int64_t n, int64_t k, unsigned flags,
                        void* stream) {
  if (!up_weights || !gate_weights || !q8 || !prod || !q8_out || !counters) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (n % 32) return fail(MLLB_EINVAL, "the product's Q8_1 needs a multiple of 32 rows");
  if (!aligned(up_weights, 16) || !aligned(gate_weights, 16) || !aligned(q8, 4) || !aligned(up, 4) ||
      !aligned(gate, 4) || !aligned(prod, 4) || !aligned(q8_out, 4) || !aligned(counters, 4))
    return fail(MLLB_EALIGN, "weights need 16-byte, the rest 4-byte alignment");
  mllb::Epilogue epi = {};
  epi.counters = counters;
  epi.q8_out = static_cast<uint8_t*>(q8_out);
  return q4k_gate_up_q8_team(static_cast<const uint8_t*>(up_weights), static_cast<const uint8_t*>(gate_weights),
                             static_cast<const uint8_t*>(q8), up, gate, prod, n, k, static_cast<cudaStream_t>(stream),
                             flags & MLLB_LAUNCH_PDL, epi);
}

int mllb_q4k_gate_up_q8_gather(const void* up_weights, const void* gate_weights, const void* q8, float* up,
                               float* gate, float* prod, uint32_t* counters, int64_t n, int64_t k,
                               const mllb_peer_gather* peers, unsigned flags, void* stream) {
  if (!up_weights || !gate_weights || !q8 || !prod || !counters || !peers || !peers->count)
    return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (n % 32) return fail(MLLB_EINVAL, "the product's Q8_1 needs a multiple of 32 rows");
  if (peers->world < 1 || peers->world > mllb::kMaxPeers || peers->rank < 0 || peers->rank >= peers->world)
    return fail(MLLB_EINVAL, "rank %d / world %d out of range", peers->rank, peers->world);
  if (!aligned(up_weights, 16) || !aligned(gate_weights, 16) || !aligned(q8, 4) || !aligned(up, 4) ||
      !aligned(gate, 4) || !aligned(prod, 4) || !aligned(counters, 4) || !aligned(peers->count, 4))
    return fail(MLLB_EALIGN, "weights need 16-byte, the rest 4-byte alignment");
  mllb::Epilogue epi = {};
  epi.counters = counters;
  epi.peer.rank = peers->rank;
  epi.peer.world = peers->world;
  for (int r = 0; r < peers->world; ++r) {
    if (!peers->buffers[r] || !peers->flags[r]) return fail(MLLB_EINVAL, "null peer pointer for rank %d", r);
    if (!aligned(peers->buffers[r], 4) || !aligned(peers->flags[r], 4))
      return fail(MLLB_EALIGN, "peer buffers and counters must be 4-byte aligned");
    epi.peer.buffers[r] = static_cast<uint8_t*>(peers->buffers[r]);
    epi.peer.flags[r] = peers->flags[r];
  }
  epi.peer.count = peers->count;
  return q4k_gate_up_q8_team<mllb::kEpiQuantProductPeer>(
      static_cast<const uint8_t*>(up_weights), static_cast<const uint8_t*>(gate_weights),
      static_cast<const uint8_t*>(q8), up, gate, prod, n, k, static_cast<cudaStream_t>(stream),
      flags & MLLB_LAUNCH_PDL, epi);
}

int64_t mllb_q4k_matvec_norm_workspace(int64_t n, int64_t k) {
  const int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  return 16 + 8 * ((n + 3) / 4);  // two counters (padded) + one double per CTA (at most one per 4-row tile)
}

int mllb_q4k_matvec_norm(const void* weights, const void* q8, float* out, int64_t n, int64_t k, const float* x,
                         float* x_out, const float* gamma, double eps, void* q8_out, void* workspace,
                         int64_t workspace_bytes, unsigned flags, void* stream) {
  if (!weights || !q8 || !x || !x_out || !gamma || !q8_out || !workspace) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (n % 32) return fail(MLLB_EINVAL, "the norm's Q8_1 needs a multiple of 32 rows");
  if (!(eps >= 0.0)) return fail(MLLB_EINVAL, "eps must be >= 0");
  if (!aligned(weights, 16) || !aligned(q8, 4) || !aligned(out, 4) || !aligned(x, 4) || !aligned(x_out, 4) ||
      !aligned(gamma, 4) || !aligned(q8_out, 4) || !aligned(workspace, 16))
    return fail(MLLB_EALIGN, "weights and workspace need 16-byte, the rest 4-byte alignment");
  const int64_t need = mllb_q4k_matvec_norm_workspace(n, k);
  if (workspace_bytes < need)
    return fail(MLLB_EINVAL, "workspace holds %lld bytes, %lld needed", static_cast<long long>(workspace_bytes),
                static_cast<long long>(need));
  const auto overlaps = [](const void* p, int64_t pb, const void* q, int64_t qb) {
    const char* a = static_cast<const char*>(p);
    const char* b = static_cast<const char*>(q);
    return a && b && a < b + qb && b < a + pb;
  };
  if ((x_out != x && overlaps(x_out, n * 4, x, n * 4)) || overlaps(x_out, n * 4, gamma, n * 4) ||
      overlaps(out, n * 4, x, n * 4) || overlaps(out, n * 4, x_out, n * 4))
    return fail(MLLB_EINVAL, "x_out may equal x but must not otherwise overlap x, gamma or out");
  const int64_t q8_bytes = n / 32 * 36;
  if (overlaps(q8_out, q8_bytes, x, n * 4) || overlaps(q8_out, q8_bytes, x_out, n * 4) ||
      overlaps(q8_out, q8_bytes, gamma, n * 4) || overlaps(q8_out, q8_bytes, out, n * 4) ||
      overlaps(q8_out, q8_bytes, workspace, need) || overlaps(workspace, need, x_out, n * 4) ||
      overlaps(workspace, need, out, n * 4) || overlaps(workspace, need, x, n * 4) ||
      overlaps(workspace, need, gamma, n * 4) || overlaps(workspace, need, q8, k / 32 * 36) ||
      overlaps(q8_out, q8_bytes, q8, k / 32 * 36))
    return fail(MLLB_EINVAL, "q8_out and workspace must not overlap each other, the Q8_1 input or the fp32 buffers");
  mllb::Epilogue epi = {};
  epi.counters = static_cast<uint32_t*>(workspace);
  epi.q8_out = static_cast<uint8_t*>(q8_out);
  epi.x = x;
  epi.x_out = x_out;
  epi.gamma = gamma;
  epi.partials = reinterpret_cast<double*>(static_cast<uint8_t*>(workspace) + 16);
  epi.eps = eps;
  return q4k_norm_team(static_cast<const uint8_t*>(weights), static_cast<const uint8_t*>(q8), out, n, k,
                       static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL, epi);
}

// ---------------------------------------------------------------- prefill

}  // extern "C"

namespace {

struct PrefillPlan {
  int row_tiles, tok_tiles, splits, bps;
  int64_t workspace;  // bytes of fp64 partials (0 with one split)
};

PrefillPlan prefill_plan(int dev, int64_t rows, int64_t k, int64_t tokens) {
  PrefillPlan p;
  const int nb = static_cast<int>(k / 256);
  p.row_tiles = static_cast<int>(rows / mllb::kPfRows);
  p.tok_tiles = static_cast<int>((tokens + mllb::kPfTok - 1) / mllb::kPfTok);
  const int ctas = p.row_tiles * p.tok_tiles;
  int splits = sm_count(dev) / (ctas > 0 ? ctas : 1);
  const int min_splits = (nb + mllb::kPfMaxGroups / 8 - 1) / (mllb::kPfMaxGroups / 8);
  if (splits < min_splits) splits = min_splits;
  if (splits > nb) splits = nb;
  if (splits < 1) splits = 1;
  p.bps = (nb + splits - 1) / splits;
  p.splits = (nb + p.bps - 1) / p.bps;
  p.workspace = p.splits > 1 ? static_cast<int64_t>(p.splits) * tokens * rows * 8 : 0;
  return p;
}

int check_prefill(int64_t rows, int64_t k, int64_t tokens) {
  if (rows <= 0 || rows % mllb::kPfRows || rows > (1 << 24))
    return fail(MLLB_EINVAL, "rows=%lld is not a positive multiple of %d", static_cast<long long>(rows), mllb::kPfRows);
  if (k <= 0 || k % 256 || k / 256 > 4096) return fail(MLLB_EINVAL, "K=%lld is not a positive multiple of 256", static_cast<long long>(k));
  if (tokens <= 0 || tokens > (1 << 20)) return fail(MLLB_EINVAL, "token count %lld out of range", static_cast<long long>(tokens));
  if (rows * tokens > (int64_t{1} << 31)) return fail(MLLB_EUNSUPPORTED, "output too large");
  return MLLB_OK;
}

}  // namespace

extern "C" {

int64_t mllb_q4k_matmul_tokens_workspace(int64_t rows, int64_t k, int64_t tokens) {
  int rc = check_prefill(rows, k, tokens);
  if (rc) return rc;
  int dev;
  if ((rc = current_device(&dev))) return rc;
  return prefill_plan(dev, rows, k, tokens).workspace;
}

int mllb_q4k_matmul_tokens(const void* weights, const void* q8, float* out, int64_t rows, int64_t k, int64_t tokens,
                           void* workspace, int64_t workspace_bytes, unsigned flags, void* stream) {
  if (!weights || !q8 || !out) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_prefill(rows, k, tokens);
  if (rc) return rc;
  if (!aligned(weights, 16) || !aligned(q8, 4) || !aligned(out, 4) || !aligned(workspace, 8))
    return fail(MLLB_EALIGN, "weights need 16-byte, q8/out 4-byte, workspace 8-byte alignment");
  int dev;
  if ((rc = current_device(&dev))) return rc;
  const PrefillPlan p = prefill_plan(dev, rows, k, tokens);
  if (p.workspace > 0 && (!workspace || workspace_bytes < p.workspace))
    return fail(MLLB_EINVAL, "workspace of %lld bytes needed (mllb_q4k_matmul_tokens_workspace)",
                static_cast<long long>(p.workspace));
  static bool attr_set[kMaxDevices] = {false};
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(mllb::prefill_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         mllb::kPfSmemBytes);
    if (e != cudaSuccess) return fail(MLLB_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  const auto s = static_cast<cudaStream_t>(stream);
  double* partial = p.splits > 1 ? static_cast<double*>(workspace) : nullptr;
  mllb::prefill_q4k_kernel<<<dim3(p.row_tiles, p.tok_tiles, p.splits), mllb::kPfThreads, mllb::kPfSmemBytes, s>>>(
      static_cast<const uint8_t*>(weights), static_cast<const uint8_t*>(q8), static_cast<int>(rows),
      static_cast<int>(k / 256), static_cast<int>(tokens), p.bps, out, partial);
  if ((rc = check_launch("prefill q4k kernel"))) return rc;
  if (partial) {
    const int64_t n = rows * tokens;
    const int grid = static_cast<int>((n + 255) / 256 < 4 * sm_count(dev) ? (n + 255) / 256 : 4 * sm_count(dev));
    mllb::prefill_sum_kernel<<<grid, 256, 0, s>>>(partial, p.splits, n, out);
    return check_launch("prefill sum kernel");
  }
  return MLLB_OK;
}

}  // extern "C"

extern "C" int mllb_decode_attention_qkv_noalloc(const float* qkv, const float* q_gamma, const float* k_gamma,
                                                 double theta_scale, const mllb_decode_state* state, void* k_cache,
                                                 void* v_cache, float* out, void* q8, int64_t q_heads,
                                                 int64_t kv_heads, int64_t ctx, unsigned flags, void* stream) {
  const int64_t need = mllb_decode_attention_scratch(q_heads, kv_heads, ctx);
  if (need < 0) return static_cast<int>(need);
  if (need > kNoAllocScratchDoubles)
    return fail(MLLB_EUNSUPPORTED,
                "attention needs %lld doubles of scratch for q_heads=%lld kv_heads=%lld ctx=%lld; the built-in "
                "scratch holds %lld (use mllb_decode_attention_qkv with a caller buffer)",
                static_cast<long long>(need), static_cast<long long>(q_heads), static_cast<long long>(kv_heads),
                static_cast<long long>(ctx), static_cast<long long>(kNoAllocScratchDoubles));
  double* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return mllb_decode_attention_qkv(qkv, q_gamma, k_gamma, theta_scale, state, k_cache, v_cache, scratch, need, out,
                                   q8, q_heads, kv_heads, ctx, flags, stream);
}

extern "C" int mllb_q8_1_quantize_allgather(const float* x, int64_t k, const mllb_peer_gather* peers, unsigned flags,
                                            void* stream) {
  if (!x || !peers || !peers->count) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  if (k <= 0 || k % 32) return fail(MLLB_EINVAL, "k=%lld is not a positive multiple of 32", static_cast<long long>(k));
  if (peers->world < 1 || peers->world > mllb::kMaxPeers || peers->rank < 0 || peers->rank >= peers->world)
    return fail(MLLB_EINVAL, "rank %d / world %d out of range", peers->rank, peers->world);
  mllb::PeerGather pg = {};
  pg.rank = peers->rank;
  pg.world = peers->world;
  for (int r = 0; r < pg.world; ++r) {
    if (!peers->buffers[r] || !peers->flags[r]) return fail(MLLB_EINVAL, "null peer pointer for rank %d", r);
    if (!aligned(peers->buffers[r], 4) || !aligned(peers->flags[r], 4))
      return fail(MLLB_EALIGN, "peer buffers and counters must be 4-byte aligned");
    pg.buffers[r] = static_cast<uint8_t*>(peers->buffers[r]);
    pg.flags[r] = peers->flags[r];
  }
  pg.count = peers->count;
  if (!aligned(x, 4) || !aligned(pg.count, 4)) return fail(MLLB_EALIGN, "x and count must be 4-byte aligned");
  const int64_t blocks = k / 32;
  int64_t grid = (blocks + 7) / 8;
  if (grid > 1024) grid = 1024;
  return launched(launch(mllb::q8_1_allgather_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0,
                         static_cast<cudaStream_t>(stream), flags & MLLB_LAUNCH_PDL, x, blocks, pg),
                  "q8_1 all-gather kernel");
}

extern "C" int mllb_prefetch_l2(const void* data, int64_t bytes, void* stream) {
  if (!data) return fail(MLLB_EINVAL, "null pointer");
  if (bytes <= 0 || bytes % 16) return fail(MLLB_EINVAL, "bytes must be a positive multiple of 16");
  if (!aligned(data, 16)) return fail(MLLB_EALIGN, "data must be 16-byte aligned");
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  int64_t grid = (bytes + 65535) / 65536;
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * 2;
  if (grid > cap) grid = cap;
  mllb::l2_prefetch_kernel<<<static_cast<unsigned>(grid), 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(data), bytes);
  return check_launch("l2 prefetch kernel");
}

extern "C" int mllb_q5k_matvec_ex(const void* weights, const void* q8, float* out, int64_t n, int64_t k,
                                  unsigned flags, void* stream) {
  if (!weights || !q8 || !out) return fail(MLLB_EINVAL, "null pointer");
  if (!known_flags(flags)) return fail(MLLB_EINVAL, "unknown flags %#x", flags);
  int rc = check_rows(n, k, 1 << 30);
  if (rc) return rc;
  if (!aligned(weights, 16) || !aligned(q8, 4) || !aligned(out, 4))
    return fail(MLLB_EALIGN, "weights need 16-byte, q8/out 4-byte alignment");
  using F = mllb::Q5kFormat;
  const auto* w = static_cast<const uint8_t*>(weights);
  const mllb::ActSource src = q8_source(static_cast<const uint8_t*>(q8));
  const int rows = static_cast<int>(n);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = flags & MLLB_LAUNCH_PDL;
  rc = k_resident<true>(w, static_cast<const uint8_t*>(q8), out, n, k, s, pdl);
  if (rc != MLLB_EUNSUPPORTED) return rc;
  switch (k / 256) {
    case 8: return launch_team<F, 8, 1, MLLB_CFG_Q5K_8>(w, nullptr, src, out, nullptr, nullptr, rows, s, pdl);
    case 10: {
      using Small = mllb::TeamConfig<F, 10, 1, MLLB_CFG_Q5K_10_SMALL>;
      int dev;
      if ((rc = current_device(&dev))) return rc;
      if ((rows + Small::kT - 1) / Small::kT <= MLLB_Q4K_10_SMALL_TILES_PER_SM * sm_count(dev))
        return launch_team<F, 10, 1, MLLB_CFG_Q5K_10_SMALL>(w, nullptr, src, out, nullptr, nullptr, rows, s, pdl);
      return launch_team<F, 10, 1, MLLB_CFG_Q5K_10>(w, nullptr, src, out, nullptr, nullptr, rows, s, pdl);
    }
    case 16: return launch_team<F, 16, 1, MLLB_CFG_Q5K_16>(w, nullptr, src, out, nullptr, nullptr, rows, s, pdl);
    default:
      return fail(MLLB_EUNSUPPORTED, "Q5_K matvec is built for K = 2048, 2560, 4096 (got %lld)",
                  static_cast<long long>(k));
  }
}

extern "C" int mllb_q5k_matvec(const void* weights, const void* q8, float* out, int64_t n, int64_t k, void* stream) {
  return mllb_q5k_matvec_ex(weights, q8, out, n, k, 0u, stream);
}
