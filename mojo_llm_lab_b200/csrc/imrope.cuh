// Fused RMSNorm + learned gamma + IMROPE on the Q tensor, one warp per head.
//
// Replaces kernels/fused_q_imrope_runtime_fastpow.mojo:8-36 (and GGML's
// rms_norm -> mul -> rope_multi chain, benchmark/bench.c:205-211):
//   r      = 1 / sqrt(sum(x^2) / 128 + 1e-6)
//   y_i    = x_i * r * gamma_i
//   axis(p)= 1 if p%3==1 and p<60; 2 if p%3==2 and p<60; 0 if p%3==0 and p<72; else 3
//   theta  = pos[axis(p)] * theta_scale^p            (pairs p < 64)
//   out_p  = y_p cos(theta) - y_{p+64} sin(theta),  out_{p+64} = y_p sin(theta) + y_{p+64} cos(theta)
// Lane l of the head's warp owns pairs l and l+32 (coalesced 128-byte loads
// of x and gamma).  The norm and the angles are evaluated in fp64: at position
// 32768 an fp32 angle carries ~4e-3 rad of rounding, 250x the 1e-5 output
// tolerance, while pos * theta_scale^p in fp64 with fp64 sincos is accurate to
// ~1e-11 rad.  The op moves 33 KB; it is latency-bound, not HBM-bound.
#pragma once

#include "common.cuh"

namespace mllb {

constexpr int kHeadDim = 128;

__device__ __forceinline__ int imrope_axis(int pair) {
  if (pair % 3 == 1 && pair < 60) return 1;
  if (pair % 3 == 2 && pair < 60) return 2;
  if (pair % 3 == 0 && pair < 72) return 0;
  return 3;
}

// One head, computed by the 32 lanes of the calling warp: lane l returns
// o[0] = out[l], o[1] = out[l + 64] (pair l) and o[2] = out[l + 32],
// o[3] = out[l + 96] (pair l + 32), in fp64.  p0..p3 are the head's 4 axis
// positions.
__device__ __forceinline__ void imrope_head_values(const float* __restrict__ x, const float* __restrict__ gamma,
                                                   int32_t p0, int32_t p1, int32_t p2, int32_t p3,
                                                   double theta_scale, int lane, double (&o)[4]) {
  const float x0 = x[lane], x1 = x[lane + 32], x2 = x[lane + 64], x3 = x[lane + 96];
  double ss = static_cast<double>(x0) * x0;
  ss = fma(static_cast<double>(x1), static_cast<double>(x1), ss);
  ss = fma(static_cast<double>(x2), static_cast<double>(x2), ss);
  ss = fma(static_cast<double>(x3), static_cast<double>(x3), ss);
  ss = warp_sum_double(ss);
  const double r = 1.0 / sqrt(ss / kHeadDim + 1e-6);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int p = lane + 32 * half;
    const int axis = imrope_axis(p);
    const int32_t position = axis == 0 ? p0 : axis == 1 ? p1 : axis == 2 ? p2 : p3;
    const double angle = static_cast<double>(position) * pow(theta_scale, static_cast<double>(p));
    double s, c;
    sincos(angle, &s, &c);
    const double ya = static_cast<double>(half ? x1 : x0) * r * static_cast<double>(gamma[p]);
    const double yb = static_cast<double>(half ? x3 : x2) * r * static_cast<double>(gamma[p + 64]);
    o[2 * half] = ya * c - yb * s;
    o[2 * half + 1] = ya * s + yb * c;
  }
}

// (cos, sin) of pair p's angle pos[axis(p)] * theta_scale^p, fp64.
__device__ __forceinline__ double2 imrope_rotation(int p, int32_t p0, int32_t p1, int32_t p2, int32_t p3,
                                                   double theta_scale) {
  const int axis = imrope_axis(p);
  const int32_t position = axis == 0 ? p0 : axis == 1 ? p1 : axis == 2 ? p2 : p3;
  const double angle = static_cast<double>(position) * pow(theta_scale, static_cast<double>(p));
  double s, c;
  sincos(angle, &s, &c);
  return make_double2(c, s);
}

// imrope_head_values with the 64 rotations precomputed (rot[p] = (cos, sin)),
// from values already in registers: lane l holds x[l + 32 i] and gamma[l + 32 i].
__device__ __forceinline__ void imrope_head_regs(float x0, float x1, float x2, float x3, float g0, float g1,
                                                 float g2, float g3, const double2* rot, int lane,
                                                 double (&o)[4]) {
  double ss = static_cast<double>(x0) * x0;
  ss = fma(static_cast<double>(x1), static_cast<double>(x1), ss);
  ss = fma(static_cast<double>(x2), static_cast<double>(x2), ss);
  ss = fma(static_cast<double>(x3), static_cast<double>(x3), ss);
  ss = warp_sum_double(ss);
  const double r = 1.0 / sqrt(ss / kHeadDim + 1e-6);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const double2 cs = rot[lane + 32 * half];
    const double ya = static_cast<double>(half ? x1 : x0) * r * static_cast<double>(half ? g1 : g0);
    const double yb = static_cast<double>(half ? x3 : x2) * r * static_cast<double>(half ? g3 : g2);
    o[2 * half] = ya * cs.x - yb * cs.y;
    o[2 * half + 1] = ya * cs.y + yb * cs.x;
  }
}

// imrope_head_regs with gamma already in fp64 (gd[i] = gamma[i], shared by
// the CTA's heads, converted once per CTA).
__device__ __forceinline__ void imrope_head_regs_gd(float x0, float x1, float x2, float x3, const double* gd,
                                                    const double2* rot, int lane, double (&o)[4]) {
  const double xd[4] = {static_cast<double>(x0), static_cast<double>(x1), static_cast<double>(x2),
                        static_cast<double>(x3)};
  double ss = xd[0] * xd[0];
  ss = fma(xd[1], xd[1], ss);
  ss = fma(xd[2], xd[2], ss);
  ss = fma(xd[3], xd[3], ss);
  ss = warp_sum_double(ss);
  const double r = 1.0 / sqrt(ss / kHeadDim + 1e-6);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const double2 cs = rot[lane + 32 * half];
    const double ya = xd[half] * r * gd[lane + 32 * half];
    const double yb = xd[2 + half] * r * gd[lane + 64 + 32 * half];
    o[2 * half] = ya * cs.x - yb * cs.y;
    o[2 * half + 1] = ya * cs.y + yb * cs.x;
  }
}

// imrope_head_regs loading the head's values itself.
__device__ __forceinline__ void imrope_head_table(const float* __restrict__ x, const float* __restrict__ gamma,
                                                  const double2* rot, int lane, double (&o)[4]) {
  imrope_head_regs(x[lane], x[lane + 32], x[lane + 64], x[lane + 96], gamma[lane], gamma[lane + 32],
                   gamma[lane + 64], gamma[lane + 96], rot, lane, o);
}

// One head, computed by the 32 lanes of the calling warp, stored as fp32.
__device__ __forceinline__ void imrope_head_warp(const float* __restrict__ x, const float* __restrict__ gamma,
                                                 const int32_t* __restrict__ pos, double theta_scale,
                                                 float* __restrict__ out, int lane) {
  double o[4];
  imrope_head_values(x, gamma, pos[0], pos[1], pos[2], pos[3], theta_scale, lane, o);
  out[lane] = static_cast<float>(o[0]);
  out[lane + 64] = static_cast<float>(o[1]);
  out[lane + 32] = static_cast<float>(o[2]);
  out[lane + 96] = static_cast<float>(o[3]);
}

// One CTA per (token, group of up to 8 heads), one warp per head (the
// launcher sizes the CTA to min(heads per token, 8) warps: small CTAs, so that
// several per SM overlap their latency chains in the many-token form).  Every
// head of a token shares its 4 positions, so the CTA first builds the 64
// rotations (one fp64 pow + sincos per thread) and the warps then only
// normalise and rotate.  Head h belongs to token h / heads_per_token and uses
// that token's 4 positions.  The theta scale comes from device memory (fp32,
// the reference ABI) unless theta_ptr is null, in which case theta_value is
// used.  early_aux (MLLB_LAUNCH_CONST_AUX): positions, theta and gamma are not
// written by the preceding kernel, so the rotation table (the pow / sincos
// chain) and gamma are built and loaded before the dependency wait; only q
// waits for the preceding kernel.
constexpr int kImropeMaxHeadsPerCta = 8;

// kGammaShared (the many-token form): gamma converted to fp64 once per CTA
// into shared memory, which takes a third of the conversion-unit work (that
// form's limit) off the heads; one token keeps gamma in each lane's
// registers, loaded before the wait, so nothing is added after it.
template <bool kGammaShared>
__global__ void __launch_bounds__(kImropeMaxHeadsPerCta * 32) imrope_q_kernel(
    const float* __restrict__ q, const float* __restrict__ gamma, const int32_t* __restrict__ positions,
    const float* __restrict__ theta_ptr, double theta_value, float* __restrict__ out, int64_t tokens,
    int64_t heads_per_token, int early_aux) {
  __shared__ double2 rot[kHeadDim / 2];
  __shared__ double gd[kGammaShared ? kHeadDim : 1];  // gamma in fp64, converted once per CTA
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int heads_per_cta = static_cast<int>(blockDim.x >> 5);
  const int64_t ctas_per_token = (heads_per_token + heads_per_cta - 1) / heads_per_cta;
  const int64_t token = blockIdx.x / ctas_per_token;
  const int64_t h = (blockIdx.x % ctas_per_token) * heads_per_cta + warp;
  const bool active = token < tokens && h < heads_per_token;
  const size_t head = static_cast<size_t>(token * heads_per_token + (active ? h : 0));
  float g0 = 0.0f, g1 = 0.0f, g2 = 0.0f, g3 = 0.0f;
  auto build_table = [&] {
    if (token < tokens) {
      if constexpr (kGammaShared) {
        for (int i = threadIdx.x; i < kHeadDim; i += blockDim.x) gd[i] = static_cast<double>(gamma[i]);
      } else {
        g0 = gamma[lane], g1 = gamma[lane + 32], g2 = gamma[lane + 64], g3 = gamma[lane + 96];
      }
      for (int p = threadIdx.x; p < kHeadDim / 2; p += blockDim.x) {
        const double theta = theta_ptr ? static_cast<double>(*theta_ptr) : theta_value;
        const int32_t* pos = positions + 4 * token;
        rot[p] = imrope_rotation(p, pos[0], pos[1], pos[2], pos[3], theta);
      }
    }
  };
  if (early_aux) build_table();
  pdl_wait_prerequisite();
  pdl_launch_dependents();
  if (token >= tokens) return;
  // The head's values are loaded first, so their latency overlaps the
  // rotation table's pow / sincos when that is built after the wait.
  const float* x = q + head * kHeadDim;
  const float x0 = x[lane], x1 = x[lane + 32], x2 = x[lane + 64], x3 = x[lane + 96];
  if (!early_aux) build_table();
  __syncthreads();
  if (!active) return;
  double o[4];
  if constexpr (kGammaShared) imrope_head_regs_gd(x0, x1, x2, x3, gd, rot, lane, o);
  else imrope_head_regs(x0, x1, x2, x3, g0, g1, g2, g3, rot, lane, o);
  float* dst = out + head * kHeadDim;
  dst[lane] = static_cast<float>(o[0]);
  dst[lane + 64] = static_cast<float>(o[1]);
  dst[lane + 32] = static_cast<float>(o[2]);
  dst[lane + 96] = static_cast<float>(o[3]);
}

}  // namespace mllb
