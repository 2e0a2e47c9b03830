// Reference-ABI entry points, built into a standalone cubin
// (lib/mllb200_compat.cubin) for harnesses that drive kernels through the
// CUDA driver API the way the reference's do: cuModuleLoad(path) +
// cuModuleGetFunction(entry) + cuLaunchKernel / cuGraphAddKernelNode with a
// flat list of device pointers and no scalar parameters
// (benchmark/bench.c:240-258, benchmark/q4_compare.c:299-300,389-399,
// tools/q4_comparison_worker.py:29-31).
//
// Each entry keeps the reference kernel's name, parameter list and launch
// geometry so it can be swapped in without touching the harness.  Shapes are
// compile-time as there: K = 2560 (10 super-blocks per row) unless the name
// ends in _2b (K = 2048); rows = gridDim.x.  The bodies are blockDim-agnostic
// (any multiple of 32), so both the 32- and 128-thread launches work.  The
// native C ABI (include/mllb200.h) is the fast path; these entries trade speed
// for the exact reference calling convention.
#include "common.cuh"
#include "imrope.cuh"
#include "q4k.cuh"
#include "q6k.cuh"

extern "C" {

// kernels/fused_q_imrope_runtime_fastpow.mojo:8-14, grid 32 x block 128.
__global__ void fused_q_imrope_runtime_fastpow(float* q, float* gamma, int32_t* positions, float* output,
                                               float* theta_scale_input) {
  if (threadIdx.x >= 32) return;
  const int head = blockIdx.x;
  mllb::imrope_head_warp(q + head * mllb::kHeadDim, gamma, positions, static_cast<double>(*theta_scale_input),
                         output + head * mllb::kHeadDim, threadIdx.x & 31);
}

// kernels/q4_k_q8_1_matvec.mojo:7 (scalar) -- grid rows x block 32.
__global__ void q4_k_q8_1_matvec(uint8_t* weights, uint8_t* activations, float* output) {
  mllb::q4k_rowblock_body(weights, nullptr, activations, output, nullptr, nullptr, 10);
}

// kernels/q4_k_q8_1_matvec_dp4a.mojo:8 -- grid rows x block 32.
__global__ void q4_k_q8_1_matvec_dp4a(uint8_t* weights, uint8_t* activations, float* output) {
  mllb::q4k_rowblock_body(weights, nullptr, activations, output, nullptr, nullptr, 10);
}

// kernels/q4_k_q8_1_matvec_dp4a_128.mojo:8 -- grid rows x block 128.
__global__ void q4_k_q8_1_matvec_dp4a_128(uint8_t* weights, uint8_t* activations, float* output) {
  mllb::q4k_rowblock_body(weights, nullptr, activations, output, nullptr, nullptr, 10);
}

// kernels/q4_k_q8_1_gate_order.mojo:55 -- (up weights, gate weights,
// activations, output = up * silu(gate)), grid rows x block 128.
__global__ void q4_k_q8_1_gate_order(uint8_t* weights, uint8_t* gate_weights, uint8_t* activations, float* output) {
  mllb::q4k_rowblock_body(weights, gate_weights, activations, nullptr, nullptr, output, 10);
}

// kernels/q4_k_q8_1_gate_order_2b.mojo -- same at K = 2048.
__global__ void q4_k_q8_1_gate_order_2b(uint8_t* weights, uint8_t* gate_weights, uint8_t* activations,
                                        float* output) {
  mllb::q4k_rowblock_body(weights, gate_weights, activations, nullptr, nullptr, output, 8);
}

// Q6_K vocabulary projection at K = 2560 (no reference kernel; same ABI style).
__global__ void q6_k_q8_1_matvec(uint8_t* weights, uint8_t* activations, float* output) {
  mllb::q6k_rowblock_body(weights, activations, output, 10);
}

// kernels/stream_read_roofline.mojo:12-27: XOR of the 417,177,600-byte buffer
// in 8-byte words, thread g taking words g, g + stride, ... with
// stride = gridDim.x * 128, result per thread in output[g].
__global__ void stream_read_roofline(uint8_t* data, uint64_t* output) {
  constexpr int64_t kWords = 417177600 / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * 128;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * 128 + threadIdx.x;
  const uint64_t* words = reinterpret_cast<const uint64_t*>(data);
  uint64_t acc = 0;
  for (int64_t i = g; i < kWords; i += stride) acc ^= __ldg(words + i);
  output[g] = acc;
}

}  // extern "C"
