// Shared device helpers of libmround_b200 (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/mround_b200.h"

namespace mr {

constexpr int kSMs = 148;  // B200: 2 dies x 74 SMs

// Record the last CUDA error string for mr_last_cuda_error().
void set_cuda_error(cudaError_t e);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_LAUNCH;
  }
  return MR_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid size: a multiple of the SM count, capped by the work available.
inline int grid_for(int64_t work_items, int threads, int per_sm = 8) {
  int64_t want = (work_items + threads - 1) / threads;
  int64_t cap = int64_t(kSMs) * per_sm;
  if (want < 1) want = 1;
  return int(want < cap ? want : cap);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(uint32_t(b) << 16);
}

// float32 -> bfloat16, round to nearest even (finite inputs).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// float32 -> tf32 value (round to nearest, ties away from zero; the low 13
// bits cleared), the form the tf32 GEMM consumes exactly.
__device__ __forceinline__ float tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

// Unpack 8 bf16 held in a uint4 into floats (exact).
__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const uint16_t (&h)[8]) {
  uint4 u;
  u.x = uint32_t(h[0]) | (uint32_t(h[1]) << 16);
  u.y = uint32_t(h[2]) | (uint32_t(h[3]) << 16);
  u.z = uint32_t(h[4]) | (uint32_t(h[5]) << 16);
  u.w = uint32_t(h[6]) | (uint32_t(h[7]) << 16);
  return u;
}

// Correctly rounded a / b from y = RN(1/b) (one __frcp_rn per quantization
// group instead of a full division per element).  Markstein's correction
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Develop. 34(1), 1990, Theorem 1): when y
// is within half an ulp of 1/b and q = RN(a*y) is within one ulp of a/b, the
// remainder r = a - q*b is exact in one FMA and RN(q + r*y) is a/b correctly
// rounded, provided nothing overflows or underflows.  The quantizer divides
// weights by a scale bounded below by eps = 1e-8 and by span/255 of their own
// group, so quotients stay within a few thousand in magnitude; a quotient in
// the subnormal range (a denormal weight) only ever feeds rint(q + v) with
// |v| <= 0.5 or q == 0, where a last-bit difference cannot change the code.
// A zero numerator returns a * y, which carries the IEEE quotient's sign of
// zero (the correction step would turn -0 into +0; the zero point rint(-0/s)
// = -0 reaches the stored bias through its sign).
// mr_selftest_division compares it against __fdiv_rn on the device.
__device__ __forceinline__ float div_rcp(float a, float b, float y) {
  const float q = __fmul_rn(a, y);
  const float r = __fmaf_rn(-q, b, a);
  return a == 0.f ? q : __fmaf_rn(r, y, q);
}

// Streaming loads/stores: the weight-sized tensors are touched once per pass.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }

}  // namespace mr
