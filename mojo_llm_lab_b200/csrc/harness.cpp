// mllb200_harness -- native timing / correctness harness for the Q4_K matvecs.
//
// The pattern of the reference's C harnesses (benchmark/q4_compare.c,
// benchmark/bench.c), rebuilt around this library:
//   * inputs: a fixture directory as tools/generate_q4_matvec_fixtures.py
//     writes it (weights.bin [gate.bin] activations.bin; a 64-row weight
//     file is repeated up to --rows, q4_compare.c:148-163);
//   * two arms: "native" (the C ABI, mllb_q4k_matvec_ex / mllb_q4k_gate_up_ex,
//     PDL-chained) and "compat" (the reference-named kernel of
//     lib/mllb200_compat.cubin, driver API, grid rows x 128 / 32 -- the
//     reference's own calling convention);
//   * each arm is one CUDA graph of --reps serialised launches bracketed by
//     two event records (q4_compare.c:108-122); arms alternate A B B A for
//     --rounds rounds after warm-up pairs (q4_compare.c:426-458), with the
//     SM and memory clocks read through NVML before and after every sample;
//   * after timing: both arms' outputs against an fp64 host evaluation of
//     the same dot products, |got - ref| <= 1e-5 + 1e-5 |ref|
//     (q4_compare.c:129-147), and red zones on both sides of every output
//     (q4_compare.c:359-363, 463-467).
// One JSON object on stdout.  Exit codes as the reference's harnesses:
// 2 usage, 3 missing kernel, 4 bad input, 12 bad timing, 13 red zone,
// 14 NVML, 20 CUDA, 25 tolerance.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <string>
#include <vector>

#include "mllb200.h"

namespace {

constexpr int kBlockBytes = 144;
constexpr int kQ8Bytes = 36;
constexpr uint32_t kRedZone = 0x7fc0dead;  // a NaN pattern no kernel writes

[[noreturn]] void die(int code, const char* fmt, const char* a = "", const char* b = "") {
  std::fprintf(stderr, fmt, a, b);
  std::fputc('\n', stderr);
  std::exit(code);
}

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) die(20, "%s: %s", what, cudaGetErrorString(e));
}

// The driver API, opened at run time so that the harness starts (and checks
// its arguments and inputs) on a machine without a driver.
struct Driver {
  CUresult (*get_error_string)(CUresult, const char**) = nullptr;
  CUresult (*module_load)(CUmodule*, const char*) = nullptr;
  CUresult (*module_get_function)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*module_unload)(CUmodule) = nullptr;
  CUresult (*launch_kernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                            CUstream, void**, void**) = nullptr;
  bool open() {
    void* lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!lib) return false;
    get_error_string = reinterpret_cast<decltype(get_error_string)>(dlsym(lib, "cuGetErrorString"));
    module_load = reinterpret_cast<decltype(module_load)>(dlsym(lib, "cuModuleLoad"));
    module_get_function = reinterpret_cast<decltype(module_get_function)>(dlsym(lib, "cuModuleGetFunction"));
    module_unload = reinterpret_cast<decltype(module_unload)>(dlsym(lib, "cuModuleUnload"));
    launch_kernel = reinterpret_cast<decltype(launch_kernel)>(dlsym(lib, "cuLaunchKernel"));
    return get_error_string && module_load && module_get_function && module_unload && launch_kernel;
  }
};
Driver drv;

void drv_ok(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    const char* s = nullptr;
    drv.get_error_string(r, &s);
    die(20, "%s: %s", what, s ? s : "?");
  }
}

bool read_file(const std::string& path, std::vector<uint8_t>* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  std::vector<uint8_t> buf;
  uint8_t chunk[1 << 16];
  size_t n;
  while ((n = std::fread(chunk, 1, sizeof(chunk), f)) > 0) buf.insert(buf.end(), chunk, chunk + n);
  const bool ok = !std::ferror(f);
  std::fclose(f);
  *out = std::move(buf);
  return ok;
}

// Weight file of `rows` rows, or of 64 rows repeated up to `rows`.
bool load_rows(const std::string& path, size_t row_bytes, int rows, std::vector<uint8_t>* w) {
  std::vector<uint8_t> raw;
  if (!read_file(path, &raw) || raw.empty() || raw.size() % row_bytes) return false;
  const size_t have = raw.size() / row_bytes;
  if (have == static_cast<size_t>(rows)) {
    *w = std::move(raw);
    return true;
  }
  if (have != 64 || rows % 64) return false;
  w->resize(static_cast<size_t>(rows) * row_bytes);
  for (int t = 0; t < rows / 64; ++t) std::memcpy(w->data() + t * raw.size(), raw.data(), raw.size());
  return true;
}

double half_to_double(uint16_t h) {
  const int sign = h >> 15, exp = (h >> 10) & 31, man = h & 1023;
  double v;
  if (exp == 0) v = std::ldexp(static_cast<double>(man), -24);
  else if (exp == 31) v = man ? NAN : INFINITY;
  else v = std::ldexp(static_cast<double>(man | 1024), exp - 25);
  return sign ? -v : v;
}

// fp64 row dot of the Q4_K x Q8_1 format (every product exact in fp64; the
// sum rounds at ~1e-16 relative, far inside the harness tolerance).
double host_row(const uint8_t* row, const uint8_t* act, int nb) {
  double total = 0.0;
  for (int b = 0; b < nb; ++b) {
    const uint8_t* blk = row + b * kBlockBytes;
    const double d = half_to_double(static_cast<uint16_t>(blk[0] | blk[1] << 8));
    const double dmin = half_to_double(static_cast<uint16_t>(blk[2] | blk[3] << 8));
    const uint8_t* sm = blk + 4;
    for (int g = 0; g < 8; ++g) {
      int sc, mn;
      if (g < 4) {
        sc = sm[g] & 63;
        mn = sm[g + 4] & 63;
      } else {
        sc = (sm[g + 4] & 15) | ((sm[g - 4] >> 6) << 4);
        mn = (sm[g + 4] >> 4) | ((sm[g] >> 6) << 4);
      }
      const uint8_t* q8 = act + (b * 8 + g) * kQ8Bytes;
      const double delta = half_to_double(static_cast<uint16_t>(q8[0] | q8[1] << 8));
      long dot = 0, sum = 0;
      for (int l = 0; l < 32; ++l) {
        const int a = static_cast<int8_t>(q8[4 + l]);
        const int w = (blk[16 + (g / 2) * 32 + l] >> (4 * (g % 2))) & 15;
        dot += static_cast<long>(w) * a;
        sum += a;
      }
      total += delta * (d * sc * static_cast<double>(dot) - dmin * mn * static_cast<double>(sum));
    }
  }
  return total;
}

// NVML, opened at run time (query calls only).
struct Nvml {
  void* lib = nullptr;
  void* dev = nullptr;
  int (*clock)(void*, int, unsigned*) = nullptr;
  // The NVML device of the CUDA device in use, matched by PCI bus id (NVML
  // numbers the GPUs without regard to CUDA_VISIBLE_DEVICES).
  bool open(const char* pci_bus_id) {
    lib = dlopen("libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!lib) return false;
    auto init = reinterpret_cast<int (*)()>(dlsym(lib, "nvmlInit_v2"));
    auto handle = reinterpret_cast<int (*)(const char*, void**)>(dlsym(lib, "nvmlDeviceGetHandleByPciBusId_v2"));
    clock = reinterpret_cast<int (*)(void*, int, unsigned*)>(dlsym(lib, "nvmlDeviceGetClockInfo"));
    return init && handle && clock && init() == 0 && handle(pci_bus_id, &dev) == 0;
  }
  unsigned read(int which) {  // 0 graphics, 1 SM, 2 memory
    unsigned mhz = 0;
    if (clock(dev, which, &mhz) != 0) die(14, "NVML clock query failed");
    return mhz;
  }
};

double now(clockid_t id) {
  timespec t;
  clock_gettime(id, &t);
  return t.tv_sec + t.tv_nsec * 1e-9;
}

struct Arm {
  const char* name;
  cudaGraphExec_t exec = nullptr;
  cudaEvent_t start = nullptr, stop = nullptr;
  uint8_t* out_buf = nullptr;  // [red zone | outputs | red zone]
};

void usage() {
  die(2, "usage: mllb200_harness FIXTURE_DIR [--op matvec|gate_up] [--rows N] [--reps R] [--rounds N] "
         "[--cubin PATH]%s%s");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2 || argv[1][0] == '-') usage();
  std::string dir = argv[1], op = "matvec", cubin;
  int rows = 9728, reps = 32, rounds = 8, warmup_pairs = 2;
  for (int i = 2; i < argc; ++i) {
    const std::string a = argv[i];
    if (i + 1 >= argc) usage();
    if (a == "--op") op = argv[++i];
    else if (a == "--rows") rows = std::atoi(argv[++i]);
    else if (a == "--reps") reps = std::atoi(argv[++i]);
    else if (a == "--rounds") rounds = std::atoi(argv[++i]);
    else if (a == "--cubin") cubin = argv[++i];
    else usage();
  }
  if ((op != "matvec" && op != "gate_up") || rows <= 0 || rows % 64 || reps <= 0 || rounds <= 0) usage();
  const bool dual = op == "gate_up";

  // ---- inputs (exit 4 on anything malformed, before touching the GPU)
  std::vector<uint8_t> act, up, gate;
  if (!read_file(dir + "/activations.bin", &act) || act.empty() || act.size() % kQ8Bytes)
    die(4, "%s/activations.bin: missing or not whole Q8_1 blocks%s", dir.c_str());
  const int k = static_cast<int>(act.size() / kQ8Bytes * 32);
  if (k % 256 || (k != 2560 && k != 2048)) die(4, "input width %s is not 2560 or 2048%s", std::to_string(k).c_str());
  const int nb = k / 256;
  const size_t row_bytes = static_cast<size_t>(nb) * kBlockBytes;
  if (!load_rows(dir + "/weights.bin", row_bytes, rows, &up)) die(4, "%s/weights.bin: bad size%s", dir.c_str());
  if (dual && !load_rows(dir + "/gate.bin", row_bytes, rows, &gate)) die(4, "%s/gate.bin: bad size%s", dir.c_str());
  if (cubin.empty()) {
    Dl_info info;
    if (dladdr(reinterpret_cast<void*>(&mllb_abi_version), &info) && info.dli_fname) {
      cubin = info.dli_fname;
      cubin = cubin.substr(0, cubin.rfind('/') + 1) + "mllb200_compat.cubin";
    }
  }
  const char* entry = dual ? (nb == 10 ? "q4_k_q8_1_gate_order" : "q4_k_q8_1_gate_order_2b") : "q4_k_q8_1_matvec_dp4a_128";
  if (!dual && nb != 10) die(4, "the compat matvec entry takes K = 2560 only%s%s");

  // ---- expected outputs, fp64 on the host
  std::vector<double> ref(rows);
  for (int r = 0; r < rows; ++r) {
    const double u = host_row(up.data() + r * row_bytes, act.data(), nb);
    if (dual) {
      const double g = host_row(gate.data() + r * row_bytes, act.data(), nb);
      ref[r] = u * (g / (1.0 + std::exp(-g)));
    } else {
      ref[r] = u;
    }
  }

  // ---- device, NVML, module
  cuda_ok(cudaSetDevice(0), "cudaSetDevice");
  cuda_ok(cudaFree(nullptr), "context");
  char bus_id[32] = {0};
  cuda_ok(cudaDeviceGetPCIBusId(bus_id, sizeof(bus_id), 0), "cudaDeviceGetPCIBusId");
  Nvml nvml;
  if (!nvml.open(bus_id)) die(14, "NVML unavailable for %s%s", bus_id);
  if (!drv.open()) die(20, "the CUDA driver (libcuda.so.1) is not available%s%s");
  CUmodule module;
  CUfunction fn;
  drv_ok(drv.module_load(&module, cubin.c_str()), "cuModuleLoad");
  if (drv.module_get_function(&fn, module, entry) != CUDA_SUCCESS) die(3, "missing %s in %s", entry, cubin.c_str());

  uint8_t *d_up, *d_gate = nullptr, *d_act;
  cuda_ok(cudaMalloc(&d_up, up.size()), "cudaMalloc");
  cuda_ok(cudaMemcpy(d_up, up.data(), up.size(), cudaMemcpyHostToDevice), "H2D");
  if (dual) {
    cuda_ok(cudaMalloc(&d_gate, gate.size()), "cudaMalloc");
    cuda_ok(cudaMemcpy(d_gate, gate.data(), gate.size(), cudaMemcpyHostToDevice), "H2D");
  }
  cuda_ok(cudaMalloc(&d_act, act.size()), "cudaMalloc");
  cuda_ok(cudaMemcpy(d_act, act.data(), act.size(), cudaMemcpyHostToDevice), "H2D");
  cudaStream_t stream;
  cuda_ok(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");

  const size_t out_bytes = static_cast<size_t>(rows) * 4 + 2 * 16;
  std::vector<uint32_t> zone(out_bytes / 4, kRedZone);
  Arm arms[2] = {{"native"}, {"compat"}};
  for (Arm& arm : arms) {
    cuda_ok(cudaMalloc(&arm.out_buf, out_bytes), "cudaMalloc");
    cuda_ok(cudaMemcpy(arm.out_buf, zone.data(), out_bytes, cudaMemcpyHostToDevice), "H2D");
    cuda_ok(cudaEventCreate(&arm.start), "event");
    cuda_ok(cudaEventCreate(&arm.stop), "event");
  }

  // One launch of each arm outside any capture (kernel attributes set), then
  // each captured as a graph of `reps` serialised launches between events.
  auto launch = [&](int which) {
    float* out = reinterpret_cast<float*>(arms[which].out_buf + 16);
    if (which == 0) {
      const int rc = dual ? mllb_q4k_gate_up_ex(d_up, d_gate, d_act, nullptr, nullptr, out, rows, k, MLLB_LAUNCH_PDL,
                                                stream)
                          : mllb_q4k_matvec_ex(d_up, d_act, out, rows, k, MLLB_LAUNCH_PDL, stream);
      if (rc != MLLB_OK) die(20, "native arm: %s%s", mllb_last_error());
    } else {
      void* args_dual[] = {&d_up, &d_gate, &d_act, &out};
      void* args_one[] = {&d_up, &d_act, &out};
      drv_ok(drv.launch_kernel(fn, rows, 1, 1, 128, 1, 1, 0, reinterpret_cast<CUstream>(stream),
                               dual ? args_dual : args_one, nullptr),
             "cuLaunchKernel");
    }
  };
  for (int which = 0; which < 2; ++which) {
    launch(which);
    cuda_ok(cudaStreamSynchronize(stream), "warm launch");
    cudaGraph_t graph;
    cuda_ok(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "capture");
    // External records: event nodes of the graph (a plain record inside a
    // capture only orders the captured work).
    cuda_ok(cudaEventRecordWithFlags(arms[which].start, stream, cudaEventRecordExternal), "event record");
    for (int i = 0; i < reps; ++i) launch(which);
    cuda_ok(cudaEventRecordWithFlags(arms[which].stop, stream, cudaEventRecordExternal), "event record");
    cuda_ok(cudaStreamEndCapture(stream, &graph), "end capture");
    cuda_ok(cudaGraphInstantiate(&arms[which].exec, graph, 0), "instantiate");
    cuda_ok(cudaGraphDestroy(graph), "graph destroy");
    cuda_ok(cudaGraphUpload(arms[which].exec, stream), "upload");
  }
  cuda_ok(cudaStreamSynchronize(stream), "upload");
  for (int p = 0; p < warmup_pairs; ++p)
    for (Arm& arm : arms) {
      cuda_ok(cudaGraphLaunch(arm.exec, stream), "graph launch");
      cuda_ok(cudaStreamSynchronize(stream), "warm-up");
    }

  std::printf("{\"op\":\"%s\",\"rows\":%d,\"input_width\":%d,\"repetitions_per_graph\":%d,\"rounds\":%d,"
              "\"warmup_pairs\":%d,\"compat_entry\":\"%s\",\"samples\":[",
              op.c_str(), rows, k, reps, rounds, warmup_pairs, entry);
  const int abba[4] = {0, 1, 1, 0};
  double sum_us[2] = {0, 0};
  int count[2] = {0, 0};
  bool first = true;
  for (int round = 0; round < rounds; ++round)
    for (int slot = 0; slot < 4; ++slot) {
      Arm& arm = arms[abba[slot]];
      const unsigned sm_before = nvml.read(1), mem_before = nvml.read(2);
      const double wall0 = now(CLOCK_MONOTONIC), cpu0 = now(CLOCK_PROCESS_CPUTIME_ID);
      cuda_ok(cudaGraphLaunch(arm.exec, stream), "graph launch");
      cuda_ok(cudaStreamSynchronize(stream), "timed graph");
      const double cpu = now(CLOCK_PROCESS_CPUTIME_ID) - cpu0, wall = now(CLOCK_MONOTONIC) - wall0;
      float ms = 0.0f;
      cuda_ok(cudaEventElapsedTime(&ms, arm.start, arm.stop), "elapsed");
      if (!(ms > 0.0f) || !std::isfinite(ms)) std::exit(12);
      const unsigned sm_after = nvml.read(1), mem_after = nvml.read(2);
      const double us = ms * 1000.0 / reps;
      sum_us[abba[slot]] += us;
      count[abba[slot]] += 1;
      std::printf("%s{\"round\":%d,\"arm\":\"%s\",\"gpu_us_per_operation\":%.6f,\"host_wall_us_per_operation\":%.6f,"
                  "\"host_cpu_us_per_operation\":%.6f,\"sm_clock_before_mhz\":%u,\"sm_clock_after_mhz\":%u,"
                  "\"memory_clock_before_mhz\":%u,\"memory_clock_after_mhz\":%u}",
                  first ? "" : ",", round, arm.name, us, wall * 1e6 / reps, cpu * 1e6 / reps, sm_before, sm_after,
                  mem_before, mem_after);
      first = false;
    }

  // ---- after timing: tolerance and red zones of both arms
  double worst[2] = {0, 0};
  for (int which = 0; which < 2; ++which) {
    std::vector<uint32_t> host(out_bytes / 4);
    cuda_ok(cudaMemcpy(host.data(), arms[which].out_buf, out_bytes, cudaMemcpyDeviceToHost), "D2H");
    for (int z = 0; z < 4; ++z)
      if (host[z] != kRedZone || host[host.size() - 1 - z] != kRedZone) {
        std::fflush(stdout);
        die(13, "red zone of the %s arm overwritten%s", arms[which].name);
      }
    for (int r = 0; r < rows; ++r) {
      float v;
      std::memcpy(&v, &host[4 + r], 4);
      const double err = std::fabs(static_cast<double>(v) - ref[r]);
      if (!std::isfinite(v) || err > 1e-5 + 1e-5 * std::fabs(ref[r])) {
        std::fflush(stdout);
        std::fprintf(stderr, "%s arm row %d: %.9g, expected %.9g\n", arms[which].name, r, v, ref[r]);
        return 25;
      }
      if (err / (1e-5 + 1e-5 * std::fabs(ref[r])) > worst[which]) worst[which] = err / (1e-5 + 1e-5 * std::fabs(ref[r]));
    }
  }
  std::printf("],\"native_us_per_operation\":%.6f,\"compat_us_per_operation\":%.6f,"
              "\"worst_error_over_tolerance\":{\"native\":%.3g,\"compat\":%.3g},\"correct\":true,"
              "\"red_zones\":\"intact\"}\n",
              sum_us[0] / count[0], sum_us[1] / count[1], worst[0], worst[1]);
  for (Arm& arm : arms) {
    cudaGraphExecDestroy(arm.exec);
    cudaEventDestroy(arm.start);
    cudaEventDestroy(arm.stop);
    cudaFree(arm.out_buf);
  }
  cudaFree(d_up);
  cudaFree(d_gate);
  cudaFree(d_act);
  cudaStreamDestroy(stream);
  drv.module_unload(module);
  return 0;
}
