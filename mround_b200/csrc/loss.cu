// K4 -- block-output loss with the exact global outlier threshold.
//
// The reference sorts |r| every step to find the k-th largest error
// (mround/core/losses.py:96-107).  Here the threshold is found by a three-pass
// MSB-first radix select on the bit patterns of |r| (non-negative floats order
// like their bit patterns): each pass histograms one digit of the candidates
// that still match the selected prefix, and a one-block kernel picks the
// digit that holds the k-th largest.  The result is the exact order
// statistic, and the histograms are small enough (2048 counters) to be summed
// across data-parallel ranks between passes, which makes the threshold global
// without gathering any residuals.
//
// The loss sum is deterministic: per-block float64 partials are reduced by a
// single block in a fixed order.

#include <mutex>

#include "common.cuh"

namespace mr {
namespace {

constexpr int kThreads = 256;
constexpr int kBins = 2048;
constexpr int kApplyBlocks = kSMs * 4;

// Digit layout of the 31 magnitude bits: [21,31), [10,21), [0,10).
__host__ __device__ constexpr int digit_shift(int pass) { return pass == 0 ? 21 : (pass == 1 ? 10 : 0); }
__host__ __device__ constexpr uint32_t digit_mask(int pass) { return pass == 1 ? 0x7FFu : 0x3FFu; }

struct SelectState {
  uint32_t prefix;    // selected high bits so far
  uint32_t mask;      // which bits of the key are selected
  int64_t k_left;     // rank still to find inside the prefix
  float thr;          // final threshold (valid after pass 2)
  uint32_t pad[3];
};

struct Workspace {
  SelectState state;
  uint32_t hist[kBins];
  double partial[kApplyBlocks];
};

__device__ __forceinline__ uint32_t key_of(float r) { return __float_as_uint(r) & 0x7FFFFFFFu; }

__global__ void __launch_bounds__(kThreads) hist_kernel(const float* __restrict__ pred,
                                                        const float* __restrict__ tgt, int64_t n,
                                                        int pass, const SelectState* state,
                                                        uint32_t* __restrict__ hist) {
  __shared__ uint32_t sh[kBins];
  for (int i = threadIdx.x; i < kBins; i += kThreads) sh[i] = 0;
  __syncthreads();
  const uint32_t prefix = pass == 0 ? 0u : state->prefix;
  const uint32_t mask = pass == 0 ? 0u : state->mask;
  const int shift = digit_shift(pass);
  const uint32_t dmask = digit_mask(pass);
  const int64_t n4 = n / 4;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
    const float4 p = __ldcs(reinterpret_cast<const float4*>(pred) + i);
    const float4 t = __ldcs(reinterpret_cast<const float4*>(tgt) + i);
    const float r[4] = {__fsub_rn(p.x, t.x), __fsub_rn(p.y, t.y), __fsub_rn(p.z, t.z),
                        __fsub_rn(p.w, t.w)};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t key = key_of(r[j]);
      if ((key & mask) != prefix) continue;
      const uint32_t bin = (key >> shift) & dmask;
      // aggregate lanes that hit the same bin before touching shared memory
      const uint32_t peers = __match_any_sync(__activemask(), bin);
      const int leader = __ffs(peers) - 1;
      if ((threadIdx.x & 31) == leader) atomicAdd(&sh[bin], __popc(peers));
    }
  }
  for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride) {
    const uint32_t key = key_of(__fsub_rn(pred[i], tgt[i]));
    if ((key & mask) == prefix) atomicAdd(&sh[(key >> shift) & dmask], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kBins; i += kThreads)
    if (sh[i]) atomicAdd(&hist[i], sh[i]);
}

// One block: find the digit holding the k-th largest, narrow the state.
__global__ void select_kernel(const uint32_t* __restrict__ hist, int64_t k, int pass,
                              SelectState* state, float* thr_out) {
  __shared__ uint32_t counts[kBins];
  const int bins = int(digit_mask(pass)) + 1;
  for (int i = threadIdx.x; i < bins; i += blockDim.x) counts[i] = hist[i];
  __syncthreads();
  if (threadIdx.x != 0) return;
  SelectState s = *state;
  if (pass == 0) {
    s.prefix = 0;
    s.mask = 0;
    s.k_left = k;
  }
  int64_t above = 0;
  int chosen = 0;
  for (int b = bins - 1; b >= 0; --b) {
    if (above + counts[b] >= s.k_left) {
      chosen = b;
      break;
    }
    above += counts[b];
  }
  s.k_left -= above;
  s.prefix |= uint32_t(chosen) << digit_shift(pass);
  s.mask |= digit_mask(pass) << digit_shift(pass);
  if (pass == 2) {
    s.thr = __uint_as_float(s.prefix);
    if (thr_out) *thr_out = s.thr;
  }
  *state = s;
}

__device__ __forceinline__ double kept_term(float r, uint32_t thr_key, bool suppress, float denom,
                                            float& g) {
  const bool keep = !suppress || key_of(r) < thr_key;
  const float kept = keep ? r : 0.f;
  g = __fdiv_rn(__fmul_rn(2.f, kept), denom);
  return double(kept) * double(kept);
}

__global__ void __launch_bounds__(kThreads) apply_kernel(
    const float* __restrict__ pred, const float* __restrict__ tgt, int64_t n, float denom,
    const float* thr_dev, float thr_val, int suppress, float* __restrict__ grad,
    double* __restrict__ partial) {
  const uint32_t thr_key = suppress ? key_of(thr_dev ? *thr_dev : thr_val) : 0u;
  const bool sup = suppress != 0;
  double acc = 0.0;
  const int64_t n4 = n / 4;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
    const float4 p = __ldcs(reinterpret_cast<const float4*>(pred) + i);
    const float4 t = __ldcs(reinterpret_cast<const float4*>(tgt) + i);
    float4 g;
    acc += kept_term(__fsub_rn(p.x, t.x), thr_key, sup, denom, g.x);
    acc += kept_term(__fsub_rn(p.y, t.y), thr_key, sup, denom, g.y);
    acc += kept_term(__fsub_rn(p.z, t.z), thr_key, sup, denom, g.z);
    acc += kept_term(__fsub_rn(p.w, t.w), thr_key, sup, denom, g.w);
    if (grad) __stcs(reinterpret_cast<float4*>(grad) + i, g);
  }
  for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride) {
    float g;
    acc += kept_term(__fsub_rn(pred[i], tgt[i]), thr_key, sup, denom, g);
    if (grad) grad[i] = g;
  }
  // fixed-order block reduction
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  __shared__ double warp_sums[kThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) s += warp_sums[w];
    partial[blockIdx.x] = s;
  }
}

__global__ void finish_kernel(const double* __restrict__ partial, int count, double denom,
                              double* loss) {
  __shared__ double sh[kThreads];
  double s = 0.0;
  for (int i = threadIdx.x; i < count; i += kThreads) s += partial[i];
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int w = kThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) sh[threadIdx.x] += sh[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = sh[0] / denom;
}

int check_vec(const void* p) { return aligned16(p) ? MR_OK : MR_ERR_ALIGNMENT; }

}  // namespace
}  // namespace mr

using namespace mr;

extern "C" size_t mr_loss_workspace_bytes(void) { return sizeof(Workspace); }

// The histogram bins count with 32-bit integers: inputs of 2^32 elements or
// more are refused rather than miscounted (every entry point that selects a
// threshold checks this).
constexpr int64_t kMaxSelectElements = int64_t(0xFFFFFFFFll);

extern "C" int mr_loss_hist_pass(const float* pred, const float* target, int64_t n, int pass,
                                 const void* state, uint32_t* hist, void* stream) {
  if (!pred || !target || !hist || n <= 0 || pass < 0 || pass > 2) return MR_ERR_ARGUMENT;
  if (n > kMaxSelectElements) return MR_ERR_ARGUMENT;
  if (pass > 0 && !state) return MR_ERR_WORKSPACE;
  if (check_vec(pred) || check_vec(target)) return MR_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(hist, 0, kBins * sizeof(uint32_t), s);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_LAUNCH;
  }
  const int grid = grid_for((n + 3) / 4, kThreads, 4);
  hist_kernel<<<grid, kThreads, 0, s>>>(pred, target, n, pass,
                                        static_cast<const SelectState*>(state), hist);
  return launch_status();
}

extern "C" int mr_loss_select_digit(const uint32_t* hist, int64_t k, int pass, void* state,
                                    float* thr_out, void* stream) {
  if (!hist || !state || k < 1 || pass < 0 || pass > 2) return MR_ERR_ARGUMENT;
  select_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      hist, k, pass, static_cast<SelectState*>(state), thr_out);
  return launch_status();
}

extern "C" int mr_loss_apply(const float* pred, const float* target, int64_t n, double denom,
                             const float* thr_dev, int suppress, float* grad, double* loss,
                             void* workspace, void* stream) {
  if (!pred || !target || !loss || n <= 0 || !(denom > 0.0)) return MR_ERR_ARGUMENT;
  if (!workspace) return MR_ERR_WORKSPACE;
  if (suppress && !thr_dev) return MR_ERR_ARGUMENT;
  if (check_vec(pred) || check_vec(target) || (grad && check_vec(grad))) return MR_ERR_ALIGNMENT;
  Workspace* ws = static_cast<Workspace*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  apply_kernel<<<kApplyBlocks, kThreads, 0, s>>>(pred, target, n, float(denom), thr_dev, 0.f,
                                                 suppress, grad, ws->partial);
  finish_kernel<<<1, kThreads, 0, s>>>(ws->partial, kApplyBlocks, denom, loss);
  return launch_status();
}

extern "C" int mr_loss_outlier(const float* pred, const float* target, int64_t n, int64_t k,
                               int suppress, double denom, float thr_in, float* grad,
                               double* loss, float* thr_out, void* workspace, void* stream) {
  if (!pred || !target || !loss || n <= 0 || !(denom > 0.0)) return MR_ERR_ARGUMENT;
  if (n > kMaxSelectElements) return MR_ERR_ARGUMENT;
  if (!workspace) return MR_ERR_WORKSPACE;
  if (check_vec(pred) || check_vec(target) || (grad && check_vec(grad))) return MR_ERR_ALIGNMENT;
  Workspace* ws = static_cast<Workspace*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float* thr_dev = nullptr;
  float thr_val = 0.f;
  if (suppress) {
    if (thr_in >= 0.f) {
      thr_val = thr_in;
    } else {
      if (k < 1 || k > n) return MR_ERR_ARGUMENT;
      for (int pass = 0; pass < 3; ++pass) {
        int st = mr_loss_hist_pass(pred, target, n, pass, &ws->state, ws->hist, stream);
        if (st) return st;
        st = mr_loss_select_digit(ws->hist, k, pass, &ws->state, thr_out, stream);
        if (st) return st;
      }
      thr_dev = &ws->state.thr;
    }
  }
  apply_kernel<<<kApplyBlocks, kThreads, 0, s>>>(pred, target, n, float(denom), thr_dev, thr_val,
                                                 suppress, grad, ws->partial);
  finish_kernel<<<1, kThreads, 0, s>>>(ws->partial, kApplyBlocks, denom, loss);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Allocation-free variant of mr_loss_outlier.
//
// Some callers of this library cannot hand it device memory: a host that
// binds the plain C ABI through an FFI and owns no device allocator, or a
// pipeline that must not call cudaMalloc because cudaMalloc may synchronize
// the device in the middle of its asynchronous work.  For them the loss
// kernels' scratch (selection state, one histogram, per-block partial sums:
// sizeof(Workspace) bytes) lives in a fixed array compiled into the library.
// Every GPU that loads the library holds this array until the process exits.
namespace mr {
namespace {

constexpr size_t kNoAllocScratchBytes = 16384;  // stated maximum: 16 KiB
static_assert(sizeof(Workspace) <= kNoAllocScratchBytes, "loss scratch exceeds the static array");

static __device__ __align__(256) unsigned char g_loss_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the array on the current device.  Host code may not use
// the symbol itself as a pointer (it names a host-side stand-in), so the
// address is looked up once per device, with that device current.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return MR_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_loss_scratch);
    if (e != cudaSuccess || !p) {
      set_cuda_error(e);
      return MR_ERR_DEVICE;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MR_OK;
}

}  // namespace
}  // namespace mr

extern "C" size_t mr_loss_noalloc_scratch_bytes(void) { return mr::kNoAllocScratchBytes; }

extern "C" int mr_loss_outlier_noalloc(const float* pred, const float* target, int64_t n,
                                       int64_t k, int suppress, double denom, float thr_in,
                                       float* grad, double* loss, float* thr_out, void* stream) {
  // histogram counters are 32-bit: larger inputs are refused rather than miscounted
  if (n > kMaxSelectElements) return MR_ERR_ARGUMENT;
  void* scratch = nullptr;
  int st = mr::scratch_for_current_device(&scratch);
  if (st) return st;
  // the scratch address belongs to the current device: a stream of another
  // device would have its kernels read a different GPU's array
  if (stream) {
    int dev = 0, sdev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MR_ERR_DEVICE;
    cudaError_t e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return MR_ERR_ARGUMENT;
    }
    if (sdev != dev) return MR_ERR_DEVICE;
  }
  // Every field of the scratch that is read is first written by this call:
  // the histogram is cleared by each pass, the selection state is reset by
  // pass 0, and the partial sums are overwritten -- stale contents from an
  // earlier call are never read.
  return mr_loss_outlier(pred, target, n, k, suppress, denom, thr_in, grad, loss, thr_out,
                         scratch, stream);
}
