// Peer memory for the fused GEMM -> reduce-scatter of the data-parallel step.
//
// mr_peer_send: the copy-engine source side -- one cudaMemcpyAsync of a rank's
// rows into their owner's slot, then a one-thread kernel that releases the
// step's epoch into the owner's flag.
//
// mr_ipc_export / mr_ipc_import: CUDA IPC handles of device buffers, so every
// rank (one process per GPU) can store into every other rank's slot buffers
// over NVLink; the handle names the allocation that holds the buffer and the
// offset locates the buffer inside it.  Imported peer memory is mapped with
// cudaIpcMemLazyEnablePeerAccess into the importing device's address space
// (no context on the peer device).  No multicast object is created.
//
// mr_reduce_slots: the owner's side of the exchange.  Every block first waits
// (bounded, acquire at system scope) until each source rank has released the
// step's epoch into its flag, then sums the world source slots in rank order
// (so the result does not depend on arrival order) into the output.  A wait
// that exceeds 2 s sets the status word (mr_peer_status) and skips the sum.
// Slot loads bypass L1 (ld.global.cg): the peers' stores land in this GPU's
// memory behind L2.

#include <cuda.h>
#include <string.h>

#include "common.cuh"

namespace mr {
namespace {

constexpr int kThreads = 256;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ int g_peer_status = 0;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) reduce_slots_kernel(
    const float* __restrict__ slots, int64_t slot_stride, int64_t n, int world,
    const unsigned long long* __restrict__ flags, unsigned long long epoch,
    float* __restrict__ out) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    bool ok = true;
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < world && ok; ++r) {
      for (uint32_t i = 0; ld_acquire_sys(flags + r) < epoch; ++i) {
        if ((i & 255u) == 255u) {
          if (globaltimer() - t0 > kWaitLimitNs) {
            atomicExch(&g_peer_status, MR_ERR_TIMEOUT);
            ok = false;
            break;
          }
          if (*reinterpret_cast<volatile int*>(&g_peer_status) != 0) {
            ok = false;
            break;
          }
        }
      }
    }
    ready = ok ? 1 : 0;
  }
  __syncthreads();
  if (!ready) return;
  const int64_t n4 = n / 4;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
    float4 s = __ldcg(reinterpret_cast<const float4*>(slots) + i);
    for (int r = 1; r < world; ++r) {
      const float4 q = __ldcg(reinterpret_cast<const float4*>(slots + r * slot_stride) + i);
      s.x = __fadd_rn(s.x, q.x);
      s.y = __fadd_rn(s.y, q.y);
      s.z = __fadd_rn(s.z, q.z);
      s.w = __fadd_rn(s.w, q.w);
    }
    reinterpret_cast<float4*>(out)[i] = s;
  }
}

// Publishes ``epoch`` to one owner's flag after the stream's preceding copy:
// the copy has completed when this kernel starts (stream order), the fence
// orders the flag after it at system scope.
__global__ void release_flag_kernel(unsigned long long* flag, unsigned long long epoch) {
  __threadfence_system();
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(epoch) : "memory");
}

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetRangeFn range_fn() {
  static GetRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(p);
  }
  return fn;
}

}  // namespace
}  // namespace mr

using namespace mr;

extern "C" size_t mr_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int mr_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return MR_ERR_ARGUMENT;
  GetRangeFn range = range_fn();
  if (!range) return MR_ERR_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return MR_ERR_LAUNCH;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_LAUNCH;
  }
  memcpy(handle, &h, sizeof(h));
  *offset = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return MR_OK;
}

extern "C" int mr_ipc_import(const void* handle, int64_t offset, void** base, void** ptr) {
  if (!handle || !base || !ptr || offset < 0) return MR_ERR_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_LAUNCH;
  }
  *base = b;
  *ptr = static_cast<char*>(b) + offset;
  return MR_OK;
}

extern "C" int mr_ipc_close(void* base) {
  if (!base) return MR_ERR_ARGUMENT;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_LAUNCH;
  }
  return MR_OK;
}

extern "C" int mr_reduce_slots(const float* slots, int64_t slot_stride, int64_t n, int world,
                               const unsigned long long* flags, unsigned long long epoch,
                               float* out, void* stream) {
  if (!slots || !flags || !out || n <= 0 || world < 1 || slot_stride < n || epoch == 0)
    return MR_ERR_ARGUMENT;
  if (n % 4 || slot_stride % 4 || !aligned16(slots) || !aligned16(out)) return MR_ERR_ALIGNMENT;
  const int grid = grid_for(n / 4, kThreads, 4);
  reduce_slots_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      slots, slot_stride, n, world, flags, epoch, out);
  return launch_status();
}

extern "C" int mr_peer_send(void* dst, const void* src, int64_t bytes, unsigned long long* flag,
                            unsigned long long epoch, void* stream) {
  if (!dst || !src || !flag || bytes < 0 || epoch == 0) return MR_ERR_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(flag) & 7u) return MR_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bytes > 0) {
    cudaError_t e = cudaMemcpyAsync(dst, src, size_t(bytes), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return MR_ERR_LAUNCH;
    }
  }
  release_flag_kernel<<<1, 1, 0, s>>>(flag, epoch);
  return launch_status();
}

// Device status word of the peer exchange (0 ok, MR_ERR_TIMEOUT after a wait
// gave up).  Synchronizes the device; `reset` clears the word.
extern "C" int mr_peer_status(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_peer_status, sizeof(int));
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_LAUNCH;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_peer_status, &zero, sizeof(int));
  }
  return v;
}
