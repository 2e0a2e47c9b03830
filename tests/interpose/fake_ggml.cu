// Test stand-in for a GGML CUDA build (test infrastructure): a kernel with the
// name, parameter list and launch shape of GGML's fused Q4_K x Q8_1 matvec
// (mul_mat_vec_q<GGML_TYPE_Q4_K, 1, true, false, false>, grid rows x 1 x 1,
// block 32 x 4), launched with <<<>>> through a shared libcudart so that an
// LD_PRELOAD library can intercept it.  Its own body only marks every output
// row NaN: correct outputs can only come from a replacement.
//
//   fake_ggml ROWS WIDTH UP GATE Q8 OUT [eager|graph] [LAUNCHES]
// reads the Q4_K matrices and the Q8_1 column from files, launches LAUNCHES
// times (default 1; `graph`: one eager launch, then the rest captured in a
// CUDA graph and replayed), and writes the fp32 output of the last launch.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

enum ggml_type { GGML_TYPE_Q4_K = 12 };

struct ggml_cuda_mm_fusion_args_device {
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

template <ggml_type type, int ncols_dst, bool has_fusion, bool is_multi_token_id, bool small_k>
__global__ void mul_mat_vec_q(const void* vx, const void* vy, const int* ids, const ggml_cuda_mm_fusion_args_device fusion,
                              float* dst, const unsigned int ncols_x, const uint3 nchannels_y,
                              const unsigned int stride_row_x, const unsigned int stride_col_y,
                              const unsigned int stride_col_dst, const uint3 channel_ratio,
                              const unsigned int stride_channel_x, const unsigned int stride_channel_y,
                              const unsigned int stride_channel_dst, const uint3 sample_ratio,
                              const unsigned int stride_sample_x, const unsigned int stride_sample_y,
                              const unsigned int stride_sample_dst, const unsigned int ids_stride) {
  if (threadIdx.x == 0 && threadIdx.y == 0) dst[blockIdx.x] = __int_as_float(0x7fc00000);
}

static std::vector<char> slurp(const char* path) {
  FILE* f = std::fopen(path, "rb");
  if (!f) { std::fprintf(stderr, "cannot open %s\n", path); std::exit(2); }
  std::fseek(f, 0, SEEK_END);
  const long n = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  std::vector<char> buf(n);
  if (std::fread(buf.data(), 1, n, f) != static_cast<size_t>(n)) std::exit(2);
  std::fclose(f);
  return buf;
}

#define CHECK(x)                                                                 \
  do {                                                                           \
    cudaError_t e_ = (x);                                                        \
    if (e_ != cudaSuccess) {                                                     \
      std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));              \
      return 3;                                                                  \
    }                                                                            \
  } while (0)

int main(int argc, char** argv) {
  if (argc < 7) { std::fprintf(stderr, "usage: fake_ggml ROWS WIDTH UP GATE Q8 OUT [eager|graph] [LAUNCHES]\n"); return 2; }
  const unsigned rows = std::atoi(argv[1]), width = std::atoi(argv[2]);
  const bool graph = argc > 7 && std::strcmp(argv[7], "graph") == 0;
  const int launches = argc > 8 ? std::atoi(argv[8]) : 1;
  const auto up = slurp(argv[3]), gate = slurp(argv[4]), q8 = slurp(argv[5]);
  void *d_up, *d_gate, *d_q8;
  float* d_out;
  CHECK(cudaMalloc(&d_up, up.size()));
  CHECK(cudaMalloc(&d_gate, gate.size()));
  CHECK(cudaMalloc(&d_q8, q8.size()));
  CHECK(cudaMalloc(&d_out, rows * sizeof(float)));
  CHECK(cudaMemcpy(d_up, up.data(), up.size(), cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(d_gate, gate.data(), gate.size(), cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(d_q8, q8.data(), q8.size(), cudaMemcpyHostToDevice));
  CHECK(cudaMemset(d_out, 0, rows * sizeof(float)));
  cudaStream_t s;
  CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  ggml_cuda_mm_fusion_args_device fusion = {};
  fusion.gate = d_gate;
  fusion.glu_op = std::getenv("FAKE_GLU") ? std::atoi(std::getenv("FAKE_GLU")) : 2;  // 2: SWIGLU
  const uint3 one = make_uint3(1, 1, 1);
  auto launch = [&] {
    mul_mat_vec_q<GGML_TYPE_Q4_K, 1, true, false, false><<<dim3(rows), dim3(32, 4), 0, s>>>(
        d_up, d_q8, nullptr, fusion, d_out, width, one, width / 256, width / 32, rows, one, 0, 0, 0, one, 0, 0, 0, 0);
  };
  const char* name = nullptr;
  CHECK(cudaFuncGetName(&name, reinterpret_cast<const void*>(mul_mat_vec_q<GGML_TYPE_Q4_K, 1, true, false, false>)));
  std::fprintf(stderr, "fake_ggml kernel %s\n", name);
  launch();
  CHECK(cudaGetLastError());
  CHECK(cudaStreamSynchronize(s));
  if (launches > 1) {
    if (graph) {
      cudaGraph_t g;
      cudaGraphExec_t ge;
      CHECK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      for (int i = 1; i < launches; ++i) launch();
      CHECK(cudaStreamEndCapture(s, &g));
      CHECK(cudaGraphInstantiate(&ge, g, 0));
      CHECK(cudaMemsetAsync(d_out, 0, rows * sizeof(float), s));
      CHECK(cudaGraphLaunch(ge, s));
      CHECK(cudaStreamSynchronize(s));
      CHECK(cudaGraphExecDestroy(ge));
      CHECK(cudaGraphDestroy(g));
    } else {
      for (int i = 1; i < launches; ++i) launch();
      CHECK(cudaGetLastError());
      CHECK(cudaStreamSynchronize(s));
    }
  }
  std::vector<float> out(rows);
  CHECK(cudaMemcpy(out.data(), d_out, rows * sizeof(float), cudaMemcpyDeviceToHost));
  FILE* f = std::fopen(argv[6], "wb");
  if (!f) return 2;
  std::fwrite(out.data(), sizeof(float), rows, f);
  std::fclose(f);
  return 0;
}
