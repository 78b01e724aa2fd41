// K8 -- the v2 candidate scale grid search, and the importance statistics it
// weighs by.
//
// search_kernel: the weight is a flat stream of rows*cols bf16 values in which
// every group is `group` consecutive elements (groups run along the input
// axis).  A warp owns a 256-element tile, each lane 8 consecutive elements,
// so a group spans group/8 adjacent lanes.  Per group the anchor is the signed
// largest-magnitude element, the first on ties (reference
// mround/reference/scale_search.py:178-186, MLX port
// mround/core/scale_search.py:152-157).  Every candidate's loss is evaluated
// from registers: each lane sums its 8 squared residuals left to right in
// float32 and the lanes of a group combine by xor-butterfly, so every lane of
// the group holds the same loss and the selection (strict improvement, in
// candidate order: the anchor first) is uniform across them.  The float32
// operations are those of the MLX port (scale_search.py:159-168):
//   inverse = -eff * recip(anchor), codes = clip(rint(inverse * w), lo, hi),
//   scale = recip(inverse), loss += (scale * codes - w)^2 [* importance]
// with recip(0) = 0, each one correctly rounded and none contracted into FMA.
//
// colsumsq_kernel: out[c] += sum_r (hi + lo)[r, c]^2 -- the summed squared
// activation each input channel sees (runner.py:359-363).  A block owns 64
// consecutive columns over all rows: 8 threads span a row (8 columns each, one
// 16-byte load per part) and 32 such row lanes stride the rows; the row lanes'
// partial sums are combined in shared memory in a fixed order and each column
// is written by one thread, so the result does not depend on scheduling.

#include "common.cuh"

namespace mr {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 256;
constexpr int kMaxCands = 256;

struct Cands {
  int n;
  float eff[kMaxCands];
};

__device__ __forceinline__ float recip0(float x) { return x != 0.f ? __frcp_rn(x) : 0.f; }

template <int LPG, bool WEIGHTED>
__global__ void __launch_bounds__(kThreads) search_kernel(const uint16_t* __restrict__ w,
                                                          int64_t n, int64_t cols, int group,
                                                          float lo, float hi,
                                                          const float* __restrict__ importance,
                                                          const Cands cands,
                                                          float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int sub = lane & (LPG - 1);  // lane index within its group
  const int64_t tiles = (n + kTile - 1) / kTile;
  for (int64_t t = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < tiles;
       t += int64_t(gridDim.x) * kWarps) {
    const int64_t e = t * kTile + lane * 8;
    const bool in = e < n;
    float wf[8], qw[8];
    if (in) {
      unpack8(__ldcs(reinterpret_cast<const uint4*>(w + e)), wf);
      if constexpr (WEIGHTED) {
        const int64_t c = e % cols;
        const float4 a = __ldg(reinterpret_cast<const float4*>(importance + c));
        const float4 b = __ldg(reinterpret_cast<const float4*>(importance + c) + 1);
        qw[0] = a.x; qw[1] = a.y; qw[2] = a.z; qw[3] = a.w;
        qw[4] = b.x; qw[5] = b.y; qw[6] = b.z; qw[7] = b.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) wf[i] = qw[i] = 0.f;
    }
    // anchor: largest |w|, first index on ties
    float best_abs = fabsf(wf[0]), anchor = wf[0];
    int best_idx = sub * 8;
#pragma unroll
    for (int i = 1; i < 8; ++i) {
      const float a = fabsf(wf[i]);
      if (a > best_abs) {
        best_abs = a;
        anchor = wf[i];
        best_idx = sub * 8 + i;
      }
    }
#pragma unroll
    for (int off = 1; off < LPG; off <<= 1) {
      const float oa = __shfl_xor_sync(0xffffffffu, best_abs, off);
      const float ov = __shfl_xor_sync(0xffffffffu, anchor, off);
      const int oi = __shfl_xor_sync(0xffffffffu, best_idx, off);
      if (oa > best_abs || (oa == best_abs && oi < best_idx)) {
        best_abs = oa;
        anchor = ov;
        best_idx = oi;
      }
    }
    const float rg = recip0(anchor);
    float best_loss = 0.f, best_scale = 0.f;
    for (int c = 0; c < cands.n; ++c) {
      const float inv = __fmul_rn(-cands.eff[c], rg);
      const float sc = recip0(inv);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float code = fminf(fmaxf(rintf(__fmul_rn(inv, wf[i])), lo), hi);
        const float r = __fsub_rn(__fmul_rn(sc, code), wf[i]);
        float sq = __fmul_rn(r, r);
        if constexpr (WEIGHTED) sq = __fmul_rn(sq, qw[i]);
        acc = __fadd_rn(acc, sq);
      }
#pragma unroll
      for (int off = 1; off < LPG; off <<= 1)
        acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
      if (c == 0 || acc < best_loss) {
        best_loss = acc;
        best_scale = sc;
      }
    }
    if (in && sub == 0) out[e / group] = best_scale;
  }
}

constexpr int kColThreads = 256;
constexpr int kColsPerBlock = 64;
constexpr int kRowLanes = kColThreads / (kColsPerBlock / 8);  // 32

__global__ void __launch_bounds__(kColThreads) colsumsq_kernel(const uint16_t* __restrict__ hi,
                                                               const uint16_t* __restrict__ lo,
                                                               int64_t rows, int64_t cols,
                                                               float* __restrict__ out) {
  const int chunk = threadIdx.x % (kColsPerBlock / 8);
  const int rlane = threadIdx.x / (kColsPerBlock / 8);
  const int64_t c0 = int64_t(blockIdx.x) * kColsPerBlock + chunk * 8;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  if (c0 < cols) {
    for (int64_t r = rlane; r < rows; r += kRowLanes) {
      float h[8];
      unpack8(__ldcs(reinterpret_cast<const uint4*>(hi + r * cols + c0)), h);
      if (lo) {
        float l[8];
        unpack8(__ldcs(reinterpret_cast<const uint4*>(lo + r * cols + c0)), l);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = __fadd_rn(h[i], l[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(h[i], h[i]));
    }
  }
  __shared__ float sh[kRowLanes][kColsPerBlock + 1];
#pragma unroll
  for (int i = 0; i < 8; ++i) sh[rlane][chunk * 8 + i] = acc[i];
  __syncthreads();
  if (threadIdx.x < kColsPerBlock) {
    const int col = threadIdx.x;
    float s = 0.f;
    for (int q = 0; q < kRowLanes; ++q) s = __fadd_rn(s, sh[q][col]);
    const int64_t c = int64_t(blockIdx.x) * kColsPerBlock + col;
    if (c < cols) out[c] = __fadd_rn(out[c], s);
  }
}

}  // namespace
}  // namespace mr

using namespace mr;

extern "C" int mr_scale_search(const uint16_t* w_bf16, int64_t rows, int64_t cols, int group,
                               int bits, const float* cands, int n_cands,
                               const float* importance, float* out, void* stream) {
  if (!w_bf16 || !cands || !out || rows <= 0 || cols <= 0) return MR_ERR_ARGUMENT;
  if (bits < 2 || bits > 8 || n_cands < 1 || n_cands > kMaxCands) return MR_ERR_ARGUMENT;
  if (group != 8 && group != 16 && group != 32 && group != 64 && group != 128 && group != 256)
    return MR_ERR_ARGUMENT;
  if (cols % group) return MR_ERR_ARGUMENT;
  if (!aligned16(w_bf16) || (importance && !aligned16(importance))) return MR_ERR_ALIGNMENT;
  Cands c{};
  c.n = n_cands;
  for (int i = 0; i < n_cands; ++i) c.eff[i] = cands[i];
  const float nmax = float(1 << (bits - 1));
  const float lo = -nmax, hi = nmax - 1.f;
  const int64_t n = rows * cols;
  const int grid = grid_for((n + kTile - 1) / kTile, kWarps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define MR_SEARCH_LAUNCH(W)                                                                      \
  switch (group / 8) {                                                                           \
    case 1: search_kernel<1, W><<<grid, kThreads, 0, s>>>(w_bf16, n, cols, group, lo, hi, importance, c, out); break;   \
    case 2: search_kernel<2, W><<<grid, kThreads, 0, s>>>(w_bf16, n, cols, group, lo, hi, importance, c, out); break;   \
    case 4: search_kernel<4, W><<<grid, kThreads, 0, s>>>(w_bf16, n, cols, group, lo, hi, importance, c, out); break;   \
    case 8: search_kernel<8, W><<<grid, kThreads, 0, s>>>(w_bf16, n, cols, group, lo, hi, importance, c, out); break;   \
    case 16: search_kernel<16, W><<<grid, kThreads, 0, s>>>(w_bf16, n, cols, group, lo, hi, importance, c, out); break; \
    case 32: search_kernel<32, W><<<grid, kThreads, 0, s>>>(w_bf16, n, cols, group, lo, hi, importance, c, out); break; \
    default: return MR_ERR_ARGUMENT;                                                              \
  }
  if (importance) {
    MR_SEARCH_LAUNCH(true)
  } else {
    MR_SEARCH_LAUNCH(false)
  }
#undef MR_SEARCH_LAUNCH
  return launch_status();
}

extern "C" int mr_colsumsq_split(const uint16_t* hi, const uint16_t* lo, int64_t rows,
                                 int64_t cols, float* out, void* stream) {
  if (!hi || !out || rows < 0 || cols <= 0) return MR_ERR_ARGUMENT;
  if (rows == 0) return MR_OK;
  if (cols % 8) return MR_ERR_ARGUMENT;
  if (!aligned16(hi) || (lo && !aligned16(lo))) return MR_ERR_ALIGNMENT;
  const int64_t col_blocks = (cols + kColsPerBlock - 1) / kColsPerBlock;
  if (col_blocks > (1ll << 31) - 1) return MR_ERR_ARGUMENT;
  colsumsq_kernel<<<unsigned(col_blocks), kColThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      hi, lo, rows, cols, out);
  return launch_status();
}
