// Library-level entry points: version, status strings, device check, and the
// float32 -> (bf16 hi, bf16 lo) operand split used by the split-precision GEMMs.

#include <string.h>

#include "common.cuh"

namespace mr {

static thread_local char g_last_error[256] = "";

void set_cuda_error(cudaError_t e) {
  const char* s = cudaGetErrorString(e);
  strncpy(g_last_error, s ? s : "unknown", sizeof(g_last_error) - 1);
  g_last_error[sizeof(g_last_error) - 1] = '\0';
}

namespace {

constexpr int kThreads = 256;

// hi = bf16(x), lo = bf16(x - hi): hi + lo carries 16 significant bits of x.
__global__ void __launch_bounds__(kThreads) split_kernel(const float* __restrict__ x, int64_t n,
                                                         uint16_t* __restrict__ hi,
                                                         uint16_t* __restrict__ lo) {
  const int64_t n8 = n / 8;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n8; i += stride) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(x) + 2 * i);
    const float4 b = __ldcs(reinterpret_cast<const float4*>(x) + 2 * i + 1);
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint16_t h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h[j] = f32_to_bf16(f[j]);
      l[j] = f32_to_bf16(__fsub_rn(f[j], bf16_to_f32(h[j])));
    }
    reinterpret_cast<uint4*>(hi)[i] = pack8(h);
    if (lo) reinterpret_cast<uint4*>(lo)[i] = pack8(l);
  }
  for (int64_t i = n8 * 8 + int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride) {
    const uint16_t h = f32_to_bf16(x[i]);
    hi[i] = h;
    if (lo) lo[i] = f32_to_bf16(__fsub_rn(x[i], bf16_to_f32(h)));
  }
}

// Bit comparison of div_rcp (reciprocal + Markstein correction) with __fdiv_rn.
__global__ void selftest_division_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                         int64_t n, unsigned int* __restrict__ mismatches) {
  unsigned int bad = 0;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float y = __frcp_rn(b[i]);
    const float q1 = div_rcp(a[i], b[i], y);
    const float q2 = __fdiv_rn(a[i], b[i]);
    bad += __float_as_uint(q1) != __float_as_uint(q2) ? 1u : 0u;
  }
  if (bad) atomicAdd(mismatches, bad);
}

}  // namespace
}  // namespace mr

using namespace mr;

extern "C" int mr_selftest_division(const float* a, const float* b, int64_t n,
                                    unsigned int* mismatches, void* stream) {
  if (!a || !b || !mismatches || n < 0) return MR_ERR_ARGUMENT;
  if (n == 0) return MR_OK;
  selftest_division_kernel<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a, b, n, mismatches);
  return launch_status();
}

extern "C" int mr_version(void) { return 100; }  // 0.1.0

extern "C" const char* mr_status_string(int status) {
  switch (status) {
    case MR_OK: return "ok";
    case MR_ERR_ARGUMENT: return "invalid argument (shape, bits, group or size)";
    case MR_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
    case MR_ERR_LAUNCH: return "CUDA launch or runtime call failed";
    case MR_ERR_DEVICE: return "no usable sm_100 device";
    case MR_ERR_TIMEOUT: return "a bounded device-side wait gave up";
    case MR_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

extern "C" const char* mr_last_cuda_error(void) { return g_last_error; }

extern "C" int mr_device_check(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_DEVICE;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return (major == 10 && minor == 0) ? MR_OK : MR_ERR_DEVICE;
}

extern "C" int mr_split_bf16(const float* x, int64_t n, uint16_t* hi, uint16_t* lo,
                             void* stream) {
  if (!x || !hi || n < 0) return MR_ERR_ARGUMENT;
  if (n == 0) return MR_OK;
  if (!aligned16(x) || !aligned16(hi) || (lo && !aligned16(lo))) return MR_ERR_ALIGNMENT;
  const int grid = grid_for((n + 7) / 8, kThreads);
  split_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, n, hi, lo);
  return launch_status();
}
