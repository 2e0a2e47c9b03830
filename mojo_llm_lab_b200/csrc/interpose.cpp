// In-model drop-in for a GGML CUDA build: an LD_PRELOAD library that sends
// GGML's fused Q4_K gate/up matvec launch to this library's streaming kernel.
//
// Replaces the reference's interposer (integration/observe_launches.cpp:
// 76-98 relaunch, 165-205 launch hooks; integration/fusion_eligibility.h:
// 24-32 eligibility), which relaunches a Mojo PTX kernel through the driver
// API on sm_86.  Here the relaunch is mllb_q4k_gate_up_ex: no module to load,
// sm_100a, any K the library streams (K/256 in {8, 10, 16}).
//
// The hooked entries are the CUDA runtime's cudaLaunchKernel and
// cudaLaunchKernelExC (GGML's <<<>>> launches of a dynamically linked
// libcudart).  A launch is GGML's fused mul_mat_vec_q<Q4_K, 1 column> when
// the device function's name is kTarget, the grid is rows x 1 x 1 and the
// block 32 x 4 x 1.  It is replaced when the fusion arguments ask for exactly
// up * silu(gate) (SWIGLU, no biases, scales or shared operands, no ids) and
// the strides are those of one dense row-major matrix and one Q8_1 column:
// stride_row_x = K / 256 blocks, stride_col_y = K / 32 blocks, stride_col_dst
// = rows.  Everything else goes to the real launch untouched.
//
// Environment:
//   MLLB_REPLACE=1     replace eligible launches (otherwise only count them)
//   MLLB_VALIDATE=N    for the first N eligible launches outside stream
//                      capture, run GGML's kernel, then this library's into a
//                      scratch buffer, and compare (|d| <= 1e-5 + 1e-5 |ref|);
//                      a mismatch aborts.  The outputs stay GGML's.
// A launch inside stream capture is replaced only once this library has run
// the shape on the device outside capture (its first call on a device sets
// kernel attributes, which is not captured); until then the real launch runs.
// Counters (matched, eligible, replaced, captured, validated) print at exit
// and are readable through mllb_interpose_counts.
#include <cuda_runtime_api.h>
#include <dlfcn.h>

#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "mllb200.h"

namespace {

// GGML's device-side fusion arguments of the quantised matvec: the layout is
// GGML's ABI (80 bytes; gate at 8, glu_op at 40, shared_dst at 64).
struct GgmlFusion {
  const void* x_bias;
  const void* gate;
  const void* gate_bias;
  const void* x_scale;
  const void* gate_scale;
  int glu_op;
  float glu_limit;
  const void* shared_up;
  const void* shared_gate;
  float* shared_dst;
  uint32_t shared_stride_col_dst;
};
static_assert(sizeof(GgmlFusion) == 80, "GGML fusion arguments");
static_assert(offsetof(GgmlFusion, gate) == 8 && offsetof(GgmlFusion, glu_op) == 40 &&
                  offsetof(GgmlFusion, shared_dst) == 64,
              "GGML fusion argument offsets");
constexpr int kGgmlGluSwiglu = 2;

// mul_mat_vec_q<GGML_TYPE_Q4_K, 1, has_fusion = true, false, false>: params
// (vx, vy, ids, fusion, dst, ncols_x, nchannels_y, stride_row_x, stride_col_y,
// stride_col_dst, ...).
constexpr const char* kTarget =
    "_Z13mul_mat_vec_qIL9ggml_type12ELi1ELb1ELb0ELb0EEvPKvS2_PKi31ggml_cuda_mm_fusion_args_devicePfj5uint3jjjS7_jjjS7_"
    "jjjj";

template <class T>
T arg(void** args, int i) {
  T v;
  std::memcpy(&v, args[i], sizeof(v));
  return v;
}

template <class F>
F real(const char* name) {
  void* p = dlsym(RTLD_NEXT, name);
  if (!p) {
    static void* rt = dlopen("libcudart.so.12", RTLD_NOW | RTLD_NOLOAD);
    if (rt) p = dlsym(rt, name);
  }
  if (!p) {
    std::fprintf(stderr, "mllb_interpose: %s not found\n", name);
    std::abort();
  }
  return reinterpret_cast<F>(p);
}

std::atomic<unsigned long> g_matched{0}, g_eligible{0}, g_replaced{0}, g_captured{0}, g_validated{0};
std::mutex g_mutex;
constexpr int kMaxDevices = 64;
constexpr int kMaxShapes = 16;
struct Prepared {
  int64_t rows, width;
};
Prepared g_prepared[kMaxDevices][kMaxShapes];
int g_prepared_n[kMaxDevices];

bool flag(const char* name) {
  const char* v = std::getenv(name);
  return v && *v && std::strcmp(v, "0") != 0;
}

struct Call {
  const void* up;
  const void* gate;
  const void* q8;
  float* dst;
  int64_t rows, width;
};

// GGML's fused Q4_K launch that this library computes exactly.
bool eligible(const void* func, dim3 grid, dim3 block, void** args, Call* c) {
  if (grid.y != 1 || grid.z != 1 || block.x != 32 || block.y != 4 || block.z != 1) return false;
  static auto get_name = real<cudaError_t (*)(const char**, const void*)>("cudaFuncGetName");
  const char* name = nullptr;
  if (get_name(&name, func) != cudaSuccess || !name || std::strcmp(name, kTarget) != 0) return false;
  ++g_matched;
  const GgmlFusion f = arg<GgmlFusion>(args, 3);
  const uint32_t width = arg<uint32_t>(args, 5), stride_row = arg<uint32_t>(args, 7);
  const uint32_t stride_col_y = arg<uint32_t>(args, 8), stride_col_dst = arg<uint32_t>(args, 9);
  const uint32_t rows = grid.x;
  const uint32_t nb = width / 256;
  const bool ok = arg<const void*>(args, 0) && arg<const void*>(args, 1) && !arg<const void*>(args, 2) &&
                  arg<float*>(args, 4) && f.gate && !f.x_bias && !f.gate_bias && !f.x_scale && !f.gate_scale &&
                  !f.shared_up && !f.shared_gate && !f.shared_dst && f.glu_op == kGgmlGluSwiglu &&
                  f.glu_limit == 0.0f && width % 256 == 0 && (nb == 8 || nb == 10 || nb == 16) &&
                  stride_row == nb && stride_col_y == width / 32 && stride_col_dst == rows;
  if (!ok) return false;
  ++g_eligible;
  *c = {arg<const void*>(args, 0), f.gate, arg<const void*>(args, 1), arg<float*>(args, 4), rows, width};
  return true;
}

int current_device() {
  static auto get = real<cudaError_t (*)(int*)>("cudaGetDevice");
  int d = -1;
  return get(&d) == cudaSuccess && d >= 0 && d < kMaxDevices ? d : -1;
}

bool prepared(int dev, const Call& c) {
  for (int i = 0; i < g_prepared_n[dev]; ++i)
    if (g_prepared[dev][i].rows == c.rows && g_prepared[dev][i].width == c.width) return true;
  return false;
}

int run_ours(const Call& c, float* dst, cudaStream_t stream) {
  return mllb_q4k_gate_up_ex(c.up, c.gate, c.q8, nullptr, nullptr, dst, c.rows, c.width, 0, stream);
}

bool capturing(cudaStream_t stream) {
  static auto is_capturing = real<cudaError_t (*)(cudaStream_t, cudaStreamCaptureStatus*)>("cudaStreamIsCapturing");
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (is_capturing(stream, &st) != cudaSuccess) return true;  // unknown: treat as capturing
  return st != cudaStreamCaptureStatusNone;
}

// GGML's kernel has run (outputs in c.dst); run ours into scratch and compare.
void validate(const Call& c, cudaStream_t stream) {
  static auto sync = real<cudaError_t (*)(cudaStream_t)>("cudaStreamSynchronize");
  static auto alloc = real<cudaError_t (*)(void**, size_t)>("cudaMalloc");
  static auto release = real<cudaError_t (*)(void*)>("cudaFree");
  static auto copy = real<cudaError_t (*)(void*, const void*, size_t, cudaMemcpyKind)>("cudaMemcpy");
  void* scratch = nullptr;
  const size_t bytes = static_cast<size_t>(c.rows) * sizeof(float);
  if (sync(stream) != cudaSuccess || alloc(&scratch, bytes) != cudaSuccess) {
    std::fprintf(stderr, "mllb_interpose: validation set-up failed\n");
    std::abort();
  }
  const int rc = run_ours(c, static_cast<float*>(scratch), stream);
  std::vector<float> ref(c.rows), got(c.rows);
  if (rc != MLLB_OK || sync(stream) != cudaSuccess ||
      copy(ref.data(), c.dst, bytes, cudaMemcpyDeviceToHost) != cudaSuccess ||
      copy(got.data(), scratch, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
    std::fprintf(stderr, "mllb_interpose: validation run failed (%s)\n", mllb_last_error());
    std::abort();
  }
  release(scratch);
  double worst = 0.0;
  for (int64_t i = 0; i < c.rows; ++i) {
    const double r = ref[i], g = got[i], d = std::fabs(r - g);
    if (!std::isfinite(r) || !std::isfinite(g) || d > 1e-5 + 1e-5 * std::fabs(r)) {
      std::fprintf(stderr, "mllb_interpose: validation mismatch row %lld: ggml %.9g, ours %.9g\n",
                   static_cast<long long>(i), r, g);
      std::abort();
    }
    worst = d > worst ? d : worst;
  }
  std::fprintf(stderr, "mllb_interpose: validated call %lu (%lld x %lld), max |d| %.3g\n", ++g_validated,
               static_cast<long long>(c.rows), static_cast<long long>(c.width), worst);
}

// Returns true when the launch was done here (the real one must not run).
bool maybe_replace(const void* func, dim3 grid, dim3 block, void** args, size_t smem, cudaStream_t stream,
                   Call* call, bool* is_eligible) {
  *is_eligible = eligible(func, grid, block, args, call);
  if (!*is_eligible || smem != 0 || !flag("MLLB_REPLACE")) return false;
  const int dev = current_device();
  if (dev < 0) return false;
  const bool in_capture = capturing(stream);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (in_capture && !prepared(dev, *call)) return false;
  if (run_ours(*call, call->dst, stream) != MLLB_OK) return false;
  if (!in_capture && !prepared(dev, *call) && g_prepared_n[dev] < kMaxShapes)
    g_prepared[dev][g_prepared_n[dev]++] = {call->rows, call->width};
  ++g_replaced;
  if (in_capture) ++g_captured;
  return true;
}

unsigned long validate_limit() {
  const char* v = std::getenv("MLLB_VALIDATE");
  return v ? std::strtoul(v, nullptr, 10) : 0;
}

void after_real(bool is_eligible, const Call& call, cudaStream_t stream) {
  if (!is_eligible || flag("MLLB_REPLACE") || g_validated.load() >= validate_limit() || capturing(stream)) return;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_validated.load() < validate_limit()) validate(call, stream);
}

__attribute__((destructor)) void report() {
  std::fprintf(stderr, "mllb_interpose matched=%lu eligible=%lu replaced=%lu captured=%lu validated=%lu\n",
               g_matched.load(), g_eligible.load(), g_replaced.load(), g_captured.load(), g_validated.load());
}

}  // namespace

extern "C" {

// matched, eligible, replaced, captured, validated.
void mllb_interpose_counts(unsigned long* out) {
  out[0] = g_matched.load();
  out[1] = g_eligible.load();
  out[2] = g_replaced.load();
  out[3] = g_captured.load();
  out[4] = g_validated.load();
}

cudaError_t cudaLaunchKernel(const void* func, dim3 grid, dim3 block, void** args, size_t smem,
                             cudaStream_t stream) {
  static auto real_launch =
      real<cudaError_t (*)(const void*, dim3, dim3, void**, size_t, cudaStream_t)>("cudaLaunchKernel");
  Call call;
  bool is_eligible = false;
  if (maybe_replace(func, grid, block, args, smem, stream, &call, &is_eligible)) return cudaSuccess;
  const cudaError_t st = real_launch(func, grid, block, args, smem, stream);
  if (st == cudaSuccess) after_real(is_eligible, call, stream);
  return st;
}

cudaError_t cudaLaunchKernelExC(const cudaLaunchConfig_t* config, const void* func, void** args) {
  static auto real_launch = real<cudaError_t (*)(const cudaLaunchConfig_t*, const void*, void**)>("cudaLaunchKernelExC");
  Call call;
  bool is_eligible = false;
  if (config->numAttrs == 0 &&
      maybe_replace(func, config->gridDim, config->blockDim, args, config->dynamicSmemBytes, config->stream, &call,
                    &is_eligible))
    return cudaSuccess;
  const cudaError_t st = real_launch(config, func, args);
  if (st == cudaSuccess) after_real(is_eligible, call, config->stream);
  return st;
}

}  // extern "C"
