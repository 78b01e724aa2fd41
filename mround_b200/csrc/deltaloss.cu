// K6 -- DeltaLoss sensitivity reduction: out[j] += sum |g * (RTN_bits[j](w) - w)|.
//
// One pass over the layer's gradient (float32) and weight (bf16) evaluates
// every candidate width in registers: the round-to-nearest quantize-dequantize
// at width b is the asymmetric quantizer with v = 0 and unit clipping
// coefficients (reference mround/pipeline/scoring.py:213-221), recomputed from
// the group extremes rather than stored.  The per-element term is float32, as
// the reference's ``mx.sum(mx.abs(gradient * perturbation))``
// (mround/pipeline/scoring.py:262) forms it; accumulation is float64
// (mround/planner/sensitivity.py:190-229).  Same warp-tile layout as the
// quantizer kernels: 8 elements per lane, a group over group/8 lanes.
// Symmetric schemes: the observed-range scale opposite to the dominant extreme
// over 2^(b-1), or the searched grid of each width; codes in
// [-2^(b-1), 2^(b-1)-1], reconstruction scale * code (mround/core/quantizer.py:
// 216-251, 319-339).

#include "common.cuh"

namespace mr {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 256;
constexpr int kMaxWidths = 8;

struct Widths {
  int n;
  float maxq[kMaxWidths];          // 2^b - 1 (asymmetric) or 2^(b-1) (symmetric)
  float rmaxq[kMaxWidths];         // RN(1 / maxq), formed on the host
  const float* grid[kMaxWidths];   // searched scale per group, or NULL
};

// sign(s) * max(|s|, eps), sign(0) = +1
__device__ __forceinline__ float clamp_mag(float s, float eps) {
  const float m = fmaxf(fabsf(s), eps);
  return s < 0.f ? -m : m;
}

// Two elements at a time with the paired float32 instructions of sm_100
// (__fmul2_rn / __ffma2_rn / __fadd2_rn: IEEE round-to-nearest per component,
// the same results as the scalar operations, half the instructions).
__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }

// a / b correctly rounded for a pair, from y = RN(1/b) (div_rcp, two lanes).
// For a = 0 the result is a zero whose sign may differ from IEEE division's
// (div_rcp keeps it); here only |g * (q - w)| is used, where the sign of a
// zero quotient cannot show.
__device__ __forceinline__ float2 div_rcp2(float2 a, float2 b, float2 y) {
  const float2 q = __fmul2_rn(a, y);
  const float2 r = __ffma2_rn(neg2(q), b, a);
  return __ffma2_rn(r, y, q);
}

template <int LPG, int SYM>
__global__ void __launch_bounds__(kThreads) deltaloss_kernel(const float* __restrict__ g,
                                                             const uint16_t* __restrict__ w,
                                                             int64_t n, Widths widths, float eps,
                                                             double* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  double acc[kMaxWidths];
#pragma unroll
  for (int j = 0; j < kMaxWidths; ++j) acc[j] = 0.0;
  const int64_t tiles = (n + kTile - 1) / kTile;
  for (int64_t t = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < tiles;
       t += int64_t(gridDim.x) * kWarps) {
    const int64_t e = t * kTile + lane * 8;
    const bool in = e < n;
    float wf[8], gf[8];
    if (in) {
      unpack8(__ldcs(reinterpret_cast<const uint4*>(w + e)), wf);
      const float4 a = __ldcs(reinterpret_cast<const float4*>(g + e));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(g + e) + 1);
      gf[0] = a.x; gf[1] = a.y; gf[2] = a.z; gf[3] = a.w;
      gf[4] = b.x; gf[5] = b.y; gf[6] = b.z; gf[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) wf[i] = gf[i] = 0.f;
    }
    float gmax = wf[0], gmin = wf[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) {
      gmax = fmaxf(gmax, wf[i]);
      gmin = fminf(gmin, wf[i]);
    }
#pragma unroll
    for (int off = 1; off < LPG; off <<= 1) {
      gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, off));
      gmin = fminf(gmin, __shfl_xor_sync(0xffffffffu, gmin, off));
    }
    if (!in) continue;
    const float w_max = gmax > 0.f ? gmax : 0.f;
    const float w_min = gmin < 0.f ? gmin : 0.f;
    const int64_t gi = e / (LPG * 8);
#pragma unroll
    for (int j = 0; j < kMaxWidths; ++j) {
      if (j >= widths.n) break;
      const float maxq = widths.maxq[j];
      const float rmaxq = widths.rmaxq[j];
      float part = 0.f;
      if constexpr (SYM) {
        float scale;
        if (widths.grid[j]) {
          scale = clamp_mag(widths.grid[j][gi], eps);
        } else {
          const float neg = -w_min;
          const bool pos = w_max >= neg;
          const float dom = pos ? w_max : neg;
          scale = clamp_mag(div_rcp(pos ? -dom : dom, maxq, rmaxq), eps);
        }
        const float rcp = __frcp_rn(scale);
        const float hi = __fsub_rn(maxq, 1.f);
        const float2 s2 = make_float2(scale, scale), y2 = make_float2(rcp, rcp);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 wv = make_float2(wf[i], wf[i + 1]);
          const float2 d = div_rcp2(wv, s2, y2);
          const float2 c = make_float2(fminf(fmaxf(rintf(d.x), -maxq), hi),
                                       fminf(fmaxf(rintf(d.y), -maxq), hi));
          const float2 q = __fmul2_rn(s2, c);
          const float2 t = __fmul2_rn(make_float2(gf[i], gf[i + 1]), __fadd2_rn(q, neg2(wv)));
          part = __fadd_rn(part, fabsf(t.x));
          part = __fadd_rn(part, fabsf(t.y));
        }
      } else {
        const float scale = fmaxf(div_rcp(__fsub_rn(w_max, w_min), maxq, rmaxq), eps);
        const float rcp = __frcp_rn(scale);
        const float zp = rintf(div_rcp(-w_min, scale, rcp));
        // clamp(rint(w / s) + zp, 0, maxq) - zp == clamp(rint(w / s), -zp, maxq - zp):
        // every operand is an integer-valued float of magnitude <= maxq (|w| is at
        // most the group's range, s at least range / maxq), so both sides are exact.
        const float lo_c = -zp, hi_c = __fsub_rn(maxq, zp);
        const float2 s2 = make_float2(scale, scale), y2 = make_float2(rcp, rcp);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 wv = make_float2(wf[i], wf[i + 1]);
          const float2 d = div_rcp2(wv, s2, y2);
          const float2 c = make_float2(fminf(fmaxf(rintf(d.x), lo_c), hi_c),
                                       fminf(fmaxf(rintf(d.y), lo_c), hi_c));
          const float2 q = __fmul2_rn(s2, c);
          const float2 t = __fmul2_rn(make_float2(gf[i], gf[i + 1]), __fadd2_rn(q, neg2(wv)));
          part = __fadd_rn(part, fabsf(t.x));
          part = __fadd_rn(part, fabsf(t.y));
        }
      }
      acc[j] += double(part);
    }
  }
  __shared__ double sh[kWarps][kMaxWidths];
#pragma unroll
  for (int j = 0; j < kMaxWidths; ++j) {
    double a = acc[j];
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    if (lane == 0) sh[threadIdx.x >> 5][j] = a;
  }
  __syncthreads();
  if (threadIdx.x < widths.n) {
    double s = 0.0;
    for (int wi = 0; wi < kWarps; ++wi) s += sh[wi][threadIdx.x];
    atomicAdd(&out[threadIdx.x], s);
  }
}

}  // namespace
}  // namespace mr

using namespace mr;

extern "C" int mr_deltaloss(const float* g, const uint16_t* w_bf16, int64_t rows, int64_t cols,
                            int group, const int* bits, int n_bits, int symmetric,
                            const float* const* grids, float eps, double* out, void* stream) {
  if (!g || !w_bf16 || !bits || !out || rows <= 0 || cols <= 0) return MR_ERR_ARGUMENT;
  if (n_bits < 1 || n_bits > kMaxWidths) return MR_ERR_ARGUMENT;
  if (group != 8 && group != 16 && group != 32 && group != 64 && group != 128 && group != 256)
    return MR_ERR_ARGUMENT;
  if (cols % group) return MR_ERR_ARGUMENT;
  if (grids && !symmetric) return MR_ERR_ARGUMENT;
  if (!aligned16(g) || !aligned16(w_bf16)) return MR_ERR_ALIGNMENT;
  Widths widths{};
  widths.n = n_bits;
  for (int j = 0; j < n_bits; ++j) {
    if (bits[j] < 2 || bits[j] > 8) return MR_ERR_ARGUMENT;
    widths.maxq[j] = symmetric ? float(1 << (bits[j] - 1)) : float((1 << bits[j]) - 1);
    widths.rmaxq[j] = 1.0f / widths.maxq[j];  // host float division: correctly rounded
    widths.grid[j] = grids ? grids[j] : nullptr;
    if (grids && !grids[j]) return MR_ERR_ARGUMENT;
  }
  const int64_t n = rows * cols;
  const int grid = grid_for((n + kTile - 1) / kTile, kWarps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define MR_DL_LAUNCH(SYM)                                                                       \
  switch (group / 8) {                                                                          \
    case 1: deltaloss_kernel<1, SYM><<<grid, kThreads, 0, s>>>(g, w_bf16, n, widths, eps, out); break;   \
    case 2: deltaloss_kernel<2, SYM><<<grid, kThreads, 0, s>>>(g, w_bf16, n, widths, eps, out); break;   \
    case 4: deltaloss_kernel<4, SYM><<<grid, kThreads, 0, s>>>(g, w_bf16, n, widths, eps, out); break;   \
    case 8: deltaloss_kernel<8, SYM><<<grid, kThreads, 0, s>>>(g, w_bf16, n, widths, eps, out); break;   \
    case 16: deltaloss_kernel<16, SYM><<<grid, kThreads, 0, s>>>(g, w_bf16, n, widths, eps, out); break; \
    case 32: deltaloss_kernel<32, SYM><<<grid, kThreads, 0, s>>>(g, w_bf16, n, widths, eps, out); break; \
    default: return MR_ERR_ARGUMENT;                                                             \
  }
  if (symmetric) {
    MR_DL_LAUNCH(1)
  } else {
    MR_DL_LAUNCH(0)
  }
#undef MR_DL_LAUNCH
  return launch_status();
}
