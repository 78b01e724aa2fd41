// K1 (fake-quant forward), K2 (straight-through backward + signSGD +
// projection, optionally fused with the next step's K1) and K5 (codes + MLX
// uint32 packing + affine scales/biases).
//
// Work decomposition, shared by the three kernels: the weight is a flat
// stream of rows*cols elements in which every quantization group is `group`
// consecutive elements.  A warp owns a 256-element tile; each lane owns 8
// consecutive elements (one 16-byte bf16 load of W, two 16-byte float loads
// of V or of the gradient), so a group spans group/8 adjacent lanes and its
// extremes and gradient sums are warp-shuffle reductions over those lanes.
// Groups never straddle a tile because group divides 256.
//
// Arithmetic follows the float32 operation order of the reference quantizer
// (mround/core/quantizer.py:185-195, 254-266, 341-347, 395-398) with correctly
// rounded division (a reciprocal and Markstein's correction, div_rcp in
// common.cuh, bit-identical to IEEE division) and ties-to-even rounding
// (rintf), and no contraction into FMA on the code path, so codes and
// reconstructions are bit-exact against a float32 implementation of the same
// formulas.

#include <cstring>
#include <type_traits>

#include "common.cuh"

namespace mr {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 256;  // elements per warp tile

// Scheme of a launch, fixed at compile time:
//   kAsym      codes in [0, 2^b - 1], scale from the clipped extremes, zero point
//              (reference asymmetric_scale, mround/core/quantizer.py:254-266);
//   kSym       codes in [-2^(b-1), 2^(b-1) - 1], signed scale opposite to the
//              dominant clipped extreme (symmetric_scale, quantizer.py:228-251);
//   kSearched  symmetric codes, scale = searched per-group value times beta,
//              alpha inert (the searched branch, quantizer.py:319-331).
// ``maxq`` is 2^b - 1 under kAsym and 2^(b-1) otherwise.
enum Mode { kAsym = 0, kSym = 1, kSearched = 2 };

struct GroupQ {
  float scale, rcp, zp, w_min, wmax_raw, wmin_raw, base;
  bool live;  // scale above the eps floor, i.e. a function of alpha/beta
  bool pos;   // kSym: the positive side dominates (alpha carries the gradient)
};

template <int LPG>
__device__ __forceinline__ void group_extremes(const float (&w)[8], float& gmax, float& gmin) {
  gmax = w[0];
  gmin = w[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    gmax = fmaxf(gmax, w[i]);
    gmin = fminf(gmin, w[i]);
  }
#pragma unroll
  for (int off = 1; off < LPG; off <<= 1) {
    gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, off));
    gmin = fminf(gmin, __shfl_xor_sync(0xffffffffu, gmin, off));
  }
}

template <int LPG>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int off = 1; off < LPG; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// sign(s) * max(|s|, eps) with sign(0) = +1 (reference _clamp_magnitude,
// quantizer.py:216-225).
__device__ __forceinline__ float clamp_magnitude(float s, float eps, bool& live) {
  const float mag = fabsf(s);
  live = mag > eps;
  const float m = fmaxf(mag, eps);
  return s < 0.f ? -m : m;
}

// Scale (and zero point under kAsym) of one group.  ``base`` is the searched
// scale (kSearched only).
template <int MODE>
__device__ __forceinline__ GroupQ group_params(float gmax, float gmin, float alpha, float beta,
                                               float base, float maxq, float eps) {
  GroupQ q;
  q.wmax_raw = gmax > 0.f ? gmax : 0.f;
  q.wmin_raw = gmin < 0.f ? gmin : 0.f;
  q.base = base;
  q.pos = false;
  q.zp = 0.f;
  q.w_min = 0.f;
  if constexpr (MODE == kAsym) {
    const float w_max = __fmul_rn(q.wmax_raw, alpha);
    const float w_min = __fmul_rn(q.wmin_raw, beta);
    const float span = div_rcp(__fsub_rn(w_max, w_min), maxq, __frcp_rn(maxq));
    q.live = span > eps;
    q.scale = fmaxf(span, eps);
    q.rcp = __frcp_rn(q.scale);
    q.zp = rintf(div_rcp(-w_min, q.scale, q.rcp));
    q.w_min = w_min;
  } else if constexpr (MODE == kSym) {
    const float w_max = __fmul_rn(q.wmax_raw, alpha);
    const float neg = -__fmul_rn(q.wmin_raw, beta);
    q.pos = w_max >= neg;
    const float dominant = q.pos ? w_max : neg;
    q.scale = clamp_magnitude(div_rcp(q.pos ? -dominant : dominant, maxq, __frcp_rn(maxq)), eps,
                              q.live);
  } else {
    q.scale = clamp_magnitude(__fmul_rn(base, beta), eps, q.live);
  }
  q.rcp = __frcp_rn(q.scale);
  return q;
}

// w / scale, correctly rounded (see div_rcp).
__device__ __forceinline__ float over_scale(float w, const GroupQ& q) {
  return div_rcp(w, q.scale, q.rcp);
}

// The code before the clamp from ws = w/scale: rint(ws + v) (+ zp under kAsym).
template <int MODE>
__device__ __forceinline__ float code_from(float ws, float v, const GroupQ& q) {
  const float r = rintf(__fadd_rn(ws, v));
  if constexpr (MODE == kAsym) return __fadd_rn(r, q.zp);
  return r;
}

template <int MODE>
__device__ __forceinline__ float unclamped_code(float w, float v, const GroupQ& q) {
  return code_from<MODE>(over_scale(w, q), v, q);
}

template <int MODE>
__device__ __forceinline__ float code_lo(float maxq) {
  return MODE == kAsym ? 0.f : -maxq;
}

template <int MODE>
__device__ __forceinline__ float code_hi(float maxq) {
  return MODE == kAsym ? maxq : __fsub_rn(maxq, 1.f);
}

template <int MODE>
__device__ __forceinline__ float clamp_code(float x, float maxq) {
  return fminf(fmaxf(x, code_lo<MODE>(maxq)), code_hi<MODE>(maxq));
}

template <int MODE>
__device__ __forceinline__ float dequant(float code, const GroupQ& q) {
  if constexpr (MODE == kAsym) return __fmul_rn(q.scale, __fsub_rn(code, q.zp));
  return __fmul_rn(q.scale, code);
}

__device__ __forceinline__ float signf(float x) {
  return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
}

__device__ __forceinline__ void load_f8(const float* p, float (&x)[8]) {
  const float4 a = ld_stream(reinterpret_cast<const float4*>(p));
  const float4 b = ld_stream(reinterpret_cast<const float4*>(p) + 1);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

__device__ __forceinline__ void store_f8(float* p, const float (&x)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
}

// Operand values are written with zeros as +0 (x + 0 under round-to-nearest):
// a product's sign of zero (rint(-0.3) * scale = -0) cannot survive the
// exchange of integer codes, and the operands rebuilt from codes
// (mr_dequant_split) must equal these bit for bit.  Only the sign of a zero
// changes; no product or nonzero sum can see it.
__device__ __forceinline__ float operand_value(float x) { return __fadd_rn(x, 0.f); }

// The tf32-rounded copy of 8 values (the backward GEMMs' float32 operand).
__device__ __forceinline__ void store_t8(float* p, const float (&x)[8]) {
  float t[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) t[i] = tf32_rna(operand_value(x[i]));
  reinterpret_cast<float4*>(p)[0] = make_float4(t[0], t[1], t[2], t[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(t[4], t[5], t[6], t[7]);
}

__device__ __forceinline__ void store_split(const float (&wq)[8], int64_t e, uint16_t* hi,
                                            uint16_t* lo) {
  uint16_t h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = operand_value(wq[i]);
    h[i] = f32_to_bf16(x);
    l[i] = f32_to_bf16(__fsub_rn(x, bf16_to_f32(h[i])));
  }
  if (hi) *reinterpret_cast<uint4*>(hi + e) = pack8(h);
  if (lo) *reinterpret_cast<uint4*>(lo + e) = pack8(l);
}

// Group extremes (not needed under kSearched) and the per-group inputs.
template <int LPG, int MODE>
__device__ __forceinline__ void extremes_for(const float (&wf)[8], float& gmax, float& gmin) {
  if constexpr (MODE != kSearched) {
    group_extremes<LPG>(wf, gmax, gmin);
  } else {
    gmax = gmin = 0.f;
  }
}

// ---------------------------------------------------------------- K1
template <int LPG, int MODE>
__global__ void __launch_bounds__(kThreads) fq_forward_kernel(
    const uint16_t* __restrict__ w, const float* __restrict__ v, const float* __restrict__ alpha,
    const float* __restrict__ beta, const float* __restrict__ init_scale, int64_t n, int group,
    float maxq, float eps, uint16_t* __restrict__ wq_hi, uint16_t* __restrict__ wq_lo,
    float* __restrict__ wq_f32, float* __restrict__ wq_t32, float* __restrict__ scale_out,
    float* __restrict__ zp_out) {
  const int lane = threadIdx.x & 31;
  const int64_t tiles = (n + kTile - 1) / kTile;
  for (int64_t t = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < tiles;
       t += int64_t(gridDim.x) * kWarps) {
    const int64_t e = t * kTile + lane * 8;
    const bool in = e < n;
    float wf[8], vf[8];
    // the group's coefficients are loaded with the tile, not after its reductions
    const int64_t gi = in ? e / group : 0;
    float ga = 1.f, gb = 1.f, gs = 0.f;
    if (in) {
      unpack8(ld_stream(reinterpret_cast<const uint4*>(w + e)), wf);
      load_f8(v + e, vf);
      ga = alpha[gi];
      gb = beta[gi];
      if (MODE == kSearched) gs = init_scale[gi];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) wf[i] = vf[i] = 0.f;
    }
    float gmax, gmin;
    extremes_for<LPG, MODE>(wf, gmax, gmin);
    if (!in) continue;  // whole groups lie past the end together
    const GroupQ q = group_params<MODE>(gmax, gmin, ga, gb, gs, maxq, eps);
    float wq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      wq[i] = dequant<MODE>(clamp_code<MODE>(unclamped_code<MODE>(wf[i], vf[i], q), maxq), q);
    store_split(wq, e, wq_hi, wq_lo);
    if (wq_f32) store_f8(wq_f32 + e, wq);
    if (wq_t32) store_t8(wq_t32 + e, wq);
    if ((lane & (LPG - 1)) == 0) {
      if (scale_out) scale_out[gi] = q.scale;
      if (zp_out) zp_out[gi] = q.zp;
    }
  }
}

// ---------------------------------------------------------------- K2
// Straight-through gradients per group (reference hand derivation
// mround/reference/quantize.py:370-397, 465-520; the chain MLX autodiff forms):
//   gV = g * scale * inside
//   kAsym:     d(wq)/d(scale) = (code - zp) - w/scale inside the clamp,
//              (code - zp) - w_min/scale outside; galpha = gs * w_max_raw,
//              gbeta = (sum_out g - gs) * w_min_raw, gs = sum g*d / maxq
//   kSym:      d(wq)/d(scale) = code - inside * w/scale; only the dominant
//              side's coefficient moves the scale: galpha = -gs * w_max_raw or
//              gbeta = -gs * w_min_raw, gs = sum g*d / 2^(b-1)
//   kSearched: same d; galpha = 0, gbeta = sum g*d * searched scale
// with gs zeroed where the eps floor holds the scale.
//
// One launch steps up to kMaxK2Segs matrices of one scheme and group size
// (the members of a block): their warp tiles form one list, segment s owning
// tiles [tile0, tile0 + ceil(n / kTile)), so small matrices share one
// launch's ramp and tail instead of paying one each.
struct K2Seg {
  const float* gq;
  const uint16_t* w;
  float* v;
  float* alpha;
  float* beta;
  const float* init_scale;
  float* gv_out;  // gradients (update = 0)
  float* ga_out;
  float* gb_out;
  uint16_t* wq_hi;  // next operands (update = 1)
  uint16_t* wq_lo;
  float* wq_t32;
  uint8_t* codes_out;  // or next codes, scale and zero point (update = 1)
  float* qscale_out;
  float* qzp_out;
  int64_t n;
  int64_t tile0;
  float maxq, lr, lo, hi;
};
constexpr int kMaxK2Segs = 8;
struct K2Launch {
  K2Seg seg[kMaxK2Segs];
  int64_t tiles;
  int count;
  int update;
  float eps;
};

template <int LPG, int MODE>
__global__ void __launch_bounds__(kThreads)
    ste_signsgd_kernel(const __grid_constant__ K2Launch L, int group) {
  const int lane = threadIdx.x & 31;
  const float eps = L.eps;
  for (int64_t t = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < L.tiles;
       t += int64_t(gridDim.x) * kWarps) {
    int s = 0;
#pragma unroll 1
    while (s + 1 < L.count && t >= L.seg[s + 1].tile0) ++s;
    const K2Seg& S = L.seg[s];
    const float* __restrict__ gq = S.gq;
    const uint16_t* __restrict__ w = S.w;
    float* __restrict__ v = S.v;
    float* __restrict__ alpha = S.alpha;
    float* __restrict__ beta = S.beta;
    const float* __restrict__ init_scale = S.init_scale;
    const int64_t n = S.n;
    const float maxq = S.maxq, lr = S.lr, lo = S.lo, hi = S.hi;
    const int64_t e = (t - S.tile0) * kTile + lane * 8;
    const bool in = e < n;
    float wf[8], vf[8], g[8];
    const int64_t gi = in ? e / group : 0;
    float a = 1.f, b = 1.f, base = 1.f;
    if (in) {
      unpack8(ld_stream(reinterpret_cast<const uint4*>(w + e)), wf);
      load_f8(v + e, vf);
      load_f8(gq + e, g);
      a = alpha[gi];
      b = beta[gi];
      if (MODE == kSearched) base = init_scale[gi];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) wf[i] = vf[i] = g[i] = 0.f;
    }
    float gmax, gmin;
    extremes_for<LPG, MODE>(wf, gmax, gmin);
    const GroupQ q = group_params<MODE>(gmax, gmin, a, b, base, maxq, eps);

    float gv[8];
    float sum_t = 0.f, sum_out = 0.f;
    const float wmin_s = MODE == kAsym ? div_rcp(q.w_min, q.scale, q.rcp) : 0.f;  // per group
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float ws = over_scale(wf[i], q);
      const float x = code_from<MODE>(ws, vf[i], q);
      const bool inside = (x >= code_lo<MODE>(maxq)) && (x <= code_hi<MODE>(maxq));
      const float code = clamp_code<MODE>(x, maxq);
      float d;
      if constexpr (MODE == kAsym) {
        const float cz = __fsub_rn(code, q.zp);
        d = inside ? __fsub_rn(cz, ws) : __fsub_rn(cz, wmin_s);
        if (!inside) sum_out = __fadd_rn(sum_out, g[i]);
      } else {
        d = inside ? __fsub_rn(code, ws) : code;
      }
      sum_t = __fadd_rn(sum_t, __fmul_rn(g[i], d));
      gv[i] = inside ? __fmul_rn(g[i], q.scale) : 0.f;
    }
    sum_t = group_sum<LPG>(sum_t);
    if constexpr (MODE == kAsym) sum_out = group_sum<LPG>(sum_out);
    if (!in) continue;
    float ga, gb;
    if constexpr (MODE == kAsym) {
      const float gs = q.live ? div_rcp(sum_t, maxq, __frcp_rn(maxq)) : 0.f;
      ga = __fmul_rn(gs, q.wmax_raw);
      gb = __fmul_rn(__fsub_rn(sum_out, gs), q.wmin_raw);
    } else if constexpr (MODE == kSym) {
      const float gs = q.live ? div_rcp(sum_t, maxq, __frcp_rn(maxq)) : 0.f;  // 2^(b-1): exact
      ga = q.pos ? -__fmul_rn(gs, q.wmax_raw) : 0.f;
      gb = q.pos ? 0.f : -__fmul_rn(gs, q.wmin_raw);
    } else {
      ga = 0.f;
      gb = q.live ? __fmul_rn(sum_t, q.base) : 0.f;
    }
    const bool leader = (lane & (LPG - 1)) == 0;
    if (S.gv_out) store_f8(S.gv_out + e, gv);
    if (leader) {
      if (S.ga_out) S.ga_out[gi] = ga;
      if (S.gb_out) S.gb_out[gi] = gb;
    }
    if (!L.update) continue;
    float vn[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      vn[i] = fminf(fmaxf(__fsub_rn(vf[i], __fmul_rn(lr, signf(gv[i]))), -0.5f), 0.5f);
    const float an = fminf(fmaxf(__fsub_rn(a, __fmul_rn(lr, signf(ga))), lo), hi);
    const float bn = fminf(fmaxf(__fsub_rn(b, __fmul_rn(lr, signf(gb))), lo), hi);
    store_f8(v + e, vn);
    if (leader) {
      alpha[gi] = an;
      beta[gi] = bn;
    }
    uint16_t* __restrict__ wq_hi = S.wq_hi;
    uint16_t* __restrict__ wq_lo = S.wq_lo;
    float* __restrict__ wq_t32 = S.wq_t32;
    uint8_t* __restrict__ codes_out = S.codes_out;
    if (wq_hi || wq_lo || wq_t32 || codes_out) {
      const GroupQ qn = group_params<MODE>(gmax, gmin, an, bn, base, maxq, eps);
      float wq[8], code[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        code[i] = clamp_code<MODE>(unclamped_code<MODE>(wf[i], vn[i], qn), maxq);
        wq[i] = dequant<MODE>(code[i], qn);
      }
      store_split(wq, e, wq_hi, wq_lo);
      if (wq_t32) store_t8(wq_t32 + e, wq);
      if (codes_out) {
        // one byte per code: unsigned under kAsym, two's complement otherwise
        uint32_t lo4 = 0, hi4 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          lo4 |= (uint32_t(int(code[i])) & 0xFFu) << (8 * i);
          hi4 |= (uint32_t(int(code[i + 4])) & 0xFFu) << (8 * i);
        }
        *reinterpret_cast<uint2*>(codes_out + e) = make_uint2(lo4, hi4);
        if (leader) {
          if (S.qscale_out) S.qscale_out[gi] = qn.scale;
          if (S.qzp_out) S.qzp_out[gi] = qn.zp;
        }
      }
    }
  }
}

// ---------------------------------------------------------------- K5
// Stored codes are unsigned: the code itself under kAsym, code + 2^(b-1) under
// the symmetric schemes (reference mround/formats/mlx_export.py:215-222).
// Affine form W = scales * q_u + biases with scales = bf16(scale) and
// biases = bf16(-scales * zp), zp the zero point or the fixed 2^(b-1)
// (mlx_export.py:159-195).  ``codes_out`` receives the codes one byte each:
// uint8 under kAsym, int8 (two's complement) under the symmetric schemes.
// The code width is a template parameter: the lane's 8 codes form a chunk of
// 8 * BITS bits with constant shifts (one 32-bit word for BITS <= 4).
template <int LPG, int MODE, int BITS>
__global__ void __launch_bounds__(kThreads) pack_mlx_kernel(
    const uint16_t* __restrict__ w, const float* __restrict__ v, const float* __restrict__ alpha,
    const float* __restrict__ beta, const float* __restrict__ init_scale, int64_t n, int group,
    float maxq, float eps, uint32_t* __restrict__ packed, uint16_t* __restrict__ scales,
    uint16_t* __restrict__ biases, uint8_t* __restrict__ codes_out) {
  constexpr int bits = BITS;
  using Chunk = typename std::conditional<(8 * BITS <= 32), uint32_t, uint64_t>::type;
  const int lane = threadIdx.x & 31;
  const int64_t tiles = (n + kTile - 1) / kTile;
  const int64_t total_words = n * bits / 32;
  constexpr int chunk_bits = 8 * bits;  // bits one lane contributes, 16..64
  const float offset = MODE == kAsym ? 0.f : maxq;
  for (int64_t t = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < tiles;
       t += int64_t(gridDim.x) * kWarps) {
    const int64_t e = t * kTile + lane * 8;
    const bool in = e < n;
    float wf[8], vf[8];
    const int64_t gi = in ? e / group : 0;
    float ga = 1.f, gb = 1.f, gs = 0.f;
    if (in) {
      unpack8(ld_stream(reinterpret_cast<const uint4*>(w + e)), wf);
      load_f8(v + e, vf);
      ga = alpha[gi];
      gb = beta[gi];
      if (MODE == kSearched) gs = init_scale[gi];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) wf[i] = vf[i] = 0.f;
    }
    float gmax, gmin;
    extremes_for<LPG, MODE>(wf, gmax, gmin);
    Chunk chunk = 0;
    if (in) {
      const GroupQ q = group_params<MODE>(gmax, gmin, ga, gb, gs, maxq, eps);
      uint8_t c8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float code = clamp_code<MODE>(unclamped_code<MODE>(wf[i], vf[i], q), maxq);
        c8[i] = uint8_t(int(code));
        chunk |= Chunk(uint32_t(__fadd_rn(code, offset))) << (i * bits);
      }
      if (codes_out) {
        uint2 u;
        u.x = uint32_t(c8[0]) | (uint32_t(c8[1]) << 8) | (uint32_t(c8[2]) << 16) | (uint32_t(c8[3]) << 24);
        u.y = uint32_t(c8[4]) | (uint32_t(c8[5]) << 8) | (uint32_t(c8[6]) << 16) | (uint32_t(c8[7]) << 24);
        *reinterpret_cast<uint2*>(codes_out + e) = u;
      }
      if ((lane & (LPG - 1)) == 0) {
        const uint16_t sb = f32_to_bf16(q.scale);
        const float zb = MODE == kAsym ? bf16_to_f32(f32_to_bf16(q.zp)) : offset;
        scales[gi] = sb;
        biases[gi] = f32_to_bf16(__fmul_rn(-bf16_to_f32(sb), zb));
      }
    }
    // Widths dividing 32 need no cross-lane assembly beyond a pair of lanes:
    // 4 bits -> one word per lane, 8 bits -> two, 2 bits -> half a word.
    if constexpr (BITS == 4) {
      if (in) packed[e / 8] = uint32_t(chunk);
      continue;
    } else if constexpr (BITS == 8) {
      if (in) *reinterpret_cast<uint2*>(packed + e / 4) = make_uint2(uint32_t(chunk), uint32_t(uint64_t(chunk) >> 32));
      continue;
    } else if constexpr (BITS == 2) {
      const uint32_t other = __shfl_xor_sync(0xffffffffu, uint32_t(chunk), 1);
      if (in && (lane & 1) == 0) packed[e / 16] = (uint32_t(chunk) & 0xFFFFu) | (other << 16);
      continue;
    }
    // Word j of this tile takes its bits from lane j*32/chunk_bits and the
    // next one; a tile holds 8*bits words (24 for 3 bits: one pass, 32-bit
    // chunks; 40-56 for 5-7 bits: two passes over 64-bit chunks).
    constexpr int kWords = 8 * BITS;
#pragma unroll
    for (int j0 = 0; j0 < kWords; j0 += 32) {
      const int j = j0 + lane;
      const int bitpos = j * 32;
      const int src = bitpos / chunk_bits;
      const int off = bitpos - src * chunk_bits;
      const int up = chunk_bits - off;
      const uint32_t lo0 = __shfl_sync(0xffffffffu, uint32_t(chunk), src & 31);
      const uint32_t lo1 = __shfl_sync(0xffffffffu, uint32_t(chunk), (src + 1) & 31);
      uint32_t word;
      if constexpr (8 * BITS <= 32) {
        const uint32_t c1 = src + 1 < 32 ? lo1 : 0u;
        word = (lo0 >> off) | (up < 32 ? c1 << up : 0u);
      } else {
        const uint32_t hi0 = __shfl_sync(0xffffffffu, uint32_t(uint64_t(chunk) >> 32), src & 31);
        const uint32_t hi1 = __shfl_sync(0xffffffffu, uint32_t(uint64_t(chunk) >> 32), (src + 1) & 31);
        const uint64_t c0 = (uint64_t(hi0) << 32) | lo0;
        const uint64_t c1 = (src + 1 < 32) ? ((uint64_t(hi1) << 32) | lo1) : 0ull;
        uint64_t w64 = c0 >> off;
        if (up < 64) w64 |= c1 << up;
        word = uint32_t(w64);
      }
      if (j < kWords) {
        const int64_t wi = t * (kTile * bits / 32) + j;
        if (wi < total_words) packed[wi] = word;
      }
    }
  }
}

int check_common(const void* w, const void* v, int64_t rows, int64_t cols, int group, int bits) {
  if (rows <= 0 || cols <= 0) return MR_ERR_ARGUMENT;
  if (bits < 2 || bits > 8) return MR_ERR_ARGUMENT;
  if (group != 8 && group != 16 && group != 32 && group != 64 && group != 128 && group != 256)
    return MR_ERR_ARGUMENT;
  if (cols % group) return MR_ERR_ARGUMENT;
  if (!w || !v) return MR_ERR_ARGUMENT;
  if (!aligned16(w) || !aligned16(v)) return MR_ERR_ALIGNMENT;
  return MR_OK;
}

}  // namespace
}  // namespace mr

using namespace mr;

#define MR_LAUNCH_LPG(MODE, group, KERNEL, GRID, STREAM, ...)                            \
  switch ((group) / 8) {                                                                 \
    case 1: KERNEL<1, MODE><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;          \
    case 2: KERNEL<2, MODE><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;          \
    case 4: KERNEL<4, MODE><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;          \
    case 8: KERNEL<8, MODE><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;          \
    case 16: KERNEL<16, MODE><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;        \
    case 32: KERNEL<32, MODE><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;        \
    default: return MR_ERR_ARGUMENT;                                                     \
  }

#define MR_DISPATCH(mode, group, KERNEL, GRID, STREAM, ...)                                \
  switch (mode) {                                                                        \
    case kAsym: MR_LAUNCH_LPG(kAsym, group, KERNEL, GRID, STREAM, __VA_ARGS__) break;    \
    case kSym: MR_LAUNCH_LPG(kSym, group, KERNEL, GRID, STREAM, __VA_ARGS__) break;      \
    default: MR_LAUNCH_LPG(kSearched, group, KERNEL, GRID, STREAM, __VA_ARGS__) break;   \
  }

namespace {

// Scheme mode from the ABI arguments; -1 for an invalid combination.
int scheme_mode(int symmetric, const float* init_scale) {
  if (init_scale) return symmetric ? kSearched : -1;
  return symmetric ? kSym : kAsym;
}

float mode_maxq(int mode, int bits) {
  return mode == kAsym ? float((1 << bits) - 1) : float(1 << (bits - 1));
}

}  // namespace

extern "C" int mr_fq_forward(const uint16_t* w_bf16, const float* v, const float* alpha,
                             const float* beta, int64_t rows, int64_t cols, int group, int bits,
                             int symmetric, const float* init_scale, float eps, uint16_t* wq_hi,
                             uint16_t* wq_lo, float* wq_f32, float* wq_t32, float* scale,
                             float* zp, void* stream) {
  int st = check_common(w_bf16, v, rows, cols, group, bits);
  if (st) return st;
  const int mode = scheme_mode(symmetric, init_scale);
  if (!alpha || !beta || mode < 0) return MR_ERR_ARGUMENT;
  if ((wq_hi && !aligned16(wq_hi)) || (wq_lo && !aligned16(wq_lo)) || (wq_f32 && !aligned16(wq_f32)) ||
      (wq_t32 && !aligned16(wq_t32)))
    return MR_ERR_ALIGNMENT;
  const int64_t n = rows * cols;
  const int grid = grid_for((n + kTile - 1) / kTile, kWarps);
  const float maxq = mode_maxq(mode, bits);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  MR_DISPATCH(mode, group, fq_forward_kernel, grid, s, w_bf16, v, alpha, beta, init_scale, n,
              group, maxq, eps, wq_hi, wq_lo, wq_f32, wq_t32, scale, zp);
  return launch_status();
}

namespace {

// Checks one K2 matrix and appends it to a launch; the scheme mode of every
// matrix of one launch must agree.
int add_k2(K2Launch& L, int* mode, const float* gq, const uint16_t* w_bf16, float* v,
           float* alpha, float* beta, int64_t rows, int64_t cols, int group, int bits,
           int symmetric, const float* init_scale, float lr, float coef_lo, float coef_hi,
           float* gv, float* galpha, float* gbeta, uint16_t* wq_hi, uint16_t* wq_lo,
           float* wq_t32, uint8_t* codes, float* qscale, float* qzp) {
  int st = check_common(w_bf16, v, rows, cols, group, bits);
  if (st) return st;
  const int m = scheme_mode(symmetric, init_scale);
  if (!gq || !alpha || !beta || m < 0) return MR_ERR_ARGUMENT;
  if (L.count && m != *mode) return MR_ERR_ARGUMENT;
  if (L.count >= kMaxK2Segs) return MR_ERR_ARGUMENT;
  if (codes && (!qscale || (m == kAsym && !qzp))) return MR_ERR_ARGUMENT;
  if (!aligned16(gq) || (gv && !aligned16(gv)) || (wq_hi && !aligned16(wq_hi)) ||
      (wq_lo && !aligned16(wq_lo)) || (wq_t32 && !aligned16(wq_t32)) ||
      (reinterpret_cast<uintptr_t>(codes) & 7u))
    return MR_ERR_ALIGNMENT;
  *mode = m;
  K2Seg& S = L.seg[L.count++];
  memset(&S, 0, sizeof(S));
  S.gq = gq; S.w = w_bf16; S.v = v; S.alpha = alpha; S.beta = beta; S.init_scale = init_scale;
  S.gv_out = gv; S.ga_out = galpha; S.gb_out = gbeta;
  S.wq_hi = wq_hi; S.wq_lo = wq_lo; S.wq_t32 = wq_t32;
  S.codes_out = codes; S.qscale_out = codes ? qscale : nullptr;
  S.qzp_out = codes && m == kAsym ? qzp : nullptr;
  S.n = rows * cols;
  S.tile0 = L.tiles;
  S.maxq = mode_maxq(m, bits);
  S.lr = lr; S.lo = coef_lo; S.hi = coef_hi;
  L.tiles += (S.n + kTile - 1) / kTile;
  return MR_OK;
}

int launch_k2(const K2Launch& L, int mode, int group, cudaStream_t s) {
  if (L.count == 0 || L.tiles <= 0) return MR_ERR_ARGUMENT;
  const int grid = grid_for(L.tiles, kWarps);
  MR_DISPATCH(mode, group, ste_signsgd_kernel, grid, s, L, group);
  return launch_status();
}

K2Launch k2_launch(int update, float eps) {
  K2Launch L;
  memset(&L, 0, sizeof(L));
  L.update = update;
  L.eps = eps;
  return L;
}

}  // namespace

extern "C" int mr_ste_signsgd(const float* gq, const uint16_t* w_bf16, float* v, float* alpha,
                              float* beta, int64_t rows, int64_t cols, int group, int bits,
                              int symmetric, const float* init_scale, float eps, float lr,
                              float coef_lo, float coef_hi, int update, float* gv, float* galpha,
                              float* gbeta, uint16_t* wq_hi, uint16_t* wq_lo, float* wq_t32,
                              void* stream) {
  K2Launch L = k2_launch(update ? 1 : 0, eps);
  int mode = 0;
  int st = add_k2(L, &mode, gq, w_bf16, v, alpha, beta, rows, cols, group, bits, symmetric,
                  init_scale, lr, coef_lo, coef_hi, gv, galpha, gbeta, wq_hi, wq_lo, wq_t32,
                  nullptr, nullptr, nullptr);
  if (st) return st;
  return launch_k2(L, mode, group, static_cast<cudaStream_t>(stream));
}

extern "C" int mr_ste_signsgd_codes(const float* gq, const uint16_t* w_bf16, float* v,
                                    float* alpha, float* beta, int64_t rows, int64_t cols,
                                    int group, int bits, int symmetric, const float* init_scale,
                                    float eps, float lr, float coef_lo, float coef_hi,
                                    uint8_t* codes, float* qscale, float* qzp, void* stream) {
  if (!codes) return MR_ERR_ARGUMENT;
  K2Launch L = k2_launch(1, eps);
  int mode = 0;
  int st = add_k2(L, &mode, gq, w_bf16, v, alpha, beta, rows, cols, group, bits, symmetric,
                  init_scale, lr, coef_lo, coef_hi, nullptr, nullptr, nullptr, nullptr, nullptr,
                  nullptr, codes, qscale, qzp);
  if (st) return st;
  return launch_k2(L, mode, group, static_cast<cudaStream_t>(stream));
}

extern "C" int mr_ste_signsgd_segments(const mr_k2_segment* segs, int count, int group,
                                       int symmetric, float eps, void* stream) {
  if (!segs || count < 1 || count > kMaxK2Segs) return MR_ERR_ARGUMENT;
  K2Launch L = k2_launch(1, eps);
  int mode = 0;
  for (int i = 0; i < count; ++i) {
    const mr_k2_segment& g = segs[i];
    int st = add_k2(L, &mode, g.gq, g.w_bf16, g.v, g.alpha, g.beta, g.rows, g.cols, group,
                    g.bits, symmetric, g.init_scale, g.lr, g.coef_lo, g.coef_hi, nullptr,
                    nullptr, nullptr, g.wq_hi, g.wq_lo, g.wq_t32, g.codes, g.qscale, g.qzp);
    if (st) return st;
  }
  return launch_k2(L, mode, group, static_cast<cudaStream_t>(stream));
}

namespace mr {
namespace {

// Operands from codes: wq = scale * (code - zp) (asymmetric) or scale * code
// (symmetric, codes as two's complement bytes) -- the same float32 operations
// as dequant<MODE> -- written as bf16 hi/lo and the tf32 copy.
template <bool SYM>
__global__ void __launch_bounds__(kThreads) dequant_split_kernel(
    const uint8_t* __restrict__ codes, const float* __restrict__ scale,
    const float* __restrict__ zp, int64_t n, int group, uint16_t* __restrict__ hi,
    uint16_t* __restrict__ lo, float* __restrict__ t32) {
  for (int64_t e = (int64_t(blockIdx.x) * kThreads + threadIdx.x) * 8; e < n;
       e += int64_t(gridDim.x) * kThreads * 8) {
    const uint2 u = *reinterpret_cast<const uint2*>(codes + e);
    const int64_t gi = e / group;
    const float sc = scale[gi];
    const float z = SYM ? 0.f : zp[gi];
    float wq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t byte = ((i < 4 ? u.x : u.y) >> (8 * (i & 3))) & 0xFFu;
      const float code = SYM ? float(int(int8_t(byte))) : float(byte);
      wq[i] = SYM ? __fmul_rn(sc, code) : __fmul_rn(sc, __fsub_rn(code, z));
    }
    store_split(wq, e, hi, lo);
    if (t32) store_t8(t32 + e, wq);
  }
}

}  // namespace
}  // namespace mr

extern "C" int mr_dequant_split(const uint8_t* codes, const float* qscale, const float* qzp,
                                int64_t rows, int64_t cols, int group, int symmetric,
                                uint16_t* wq_hi, uint16_t* wq_lo, float* wq_t32, void* stream) {
  if (!codes || !qscale || rows <= 0 || cols <= 0 || (!symmetric && !qzp)) return MR_ERR_ARGUMENT;
  if (group != 8 && group != 16 && group != 32 && group != 64 && group != 128 && group != 256)
    return MR_ERR_ARGUMENT;
  if (cols % group) return MR_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(codes) & 7u) || (wq_hi && !aligned16(wq_hi)) ||
      (wq_lo && !aligned16(wq_lo)) || (wq_t32 && !aligned16(wq_t32)))
    return MR_ERR_ALIGNMENT;
  const int64_t n = rows * cols;
  const int grid = grid_for((n + 7) / 8, kThreads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (symmetric)
    dequant_split_kernel<true><<<grid, kThreads, 0, s>>>(codes, qscale, qzp, n, group, wq_hi, wq_lo,
                                                          wq_t32);
  else
    dequant_split_kernel<false><<<grid, kThreads, 0, s>>>(codes, qscale, qzp, n, group, wq_hi,
                                                           wq_lo, wq_t32);
  return launch_status();
}

extern "C" int mr_pack_mlx(const uint16_t* w_bf16, const float* v, const float* alpha,
                           const float* beta, int64_t rows, int64_t cols, int group, int bits,
                           int symmetric, const float* init_scale, float eps, uint32_t* packed,
                           uint16_t* scales_bf16, uint16_t* biases_bf16, uint8_t* codes,
                           void* stream) {
  int st = check_common(w_bf16, v, rows, cols, group, bits);
  if (st) return st;
  const int mode = scheme_mode(symmetric, init_scale);
  if (!alpha || !beta || !packed || !scales_bf16 || !biases_bf16 || mode < 0)
    return MR_ERR_ARGUMENT;
  if (32 % bits == 0 ? (cols % (32 / bits)) : (cols % 32)) return MR_ERR_ARGUMENT;
  if (codes && (reinterpret_cast<uintptr_t>(codes) & 7u)) return MR_ERR_ALIGNMENT;
  if (reinterpret_cast<uintptr_t>(packed) & (bits == 8 ? 7u : 3u)) return MR_ERR_ALIGNMENT;
  const int64_t n = rows * cols;
  const int grid = grid_for((n + kTile - 1) / kTile, kWarps);
  const float maxq = mode_maxq(mode, bits);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define MR_PACK_LPG(MODE, B)                                                                 \
  switch (group / 8) {                                                                       \
    case 1: pack_mlx_kernel<1, MODE, B><<<grid, kThreads, 0, s>>>(MR_PACK_ARGS); break;      \
    case 2: pack_mlx_kernel<2, MODE, B><<<grid, kThreads, 0, s>>>(MR_PACK_ARGS); break;      \
    case 4: pack_mlx_kernel<4, MODE, B><<<grid, kThreads, 0, s>>>(MR_PACK_ARGS); break;      \
    case 8: pack_mlx_kernel<8, MODE, B><<<grid, kThreads, 0, s>>>(MR_PACK_ARGS); break;      \
    case 16: pack_mlx_kernel<16, MODE, B><<<grid, kThreads, 0, s>>>(MR_PACK_ARGS); break;    \
    case 32: pack_mlx_kernel<32, MODE, B><<<grid, kThreads, 0, s>>>(MR_PACK_ARGS); break;    \
    default: return MR_ERR_ARGUMENT;                                                         \
  }
#define MR_PACK_ARGS \
  w_bf16, v, alpha, beta, init_scale, n, group, maxq, eps, packed, scales_bf16, biases_bf16, codes
#define MR_PACK_BITS(B)                                                                      \
  case B: {                                                                                  \
    if (mode == kAsym) {                                                                     \
      MR_PACK_LPG(kAsym, B)                                                                  \
    } else if (mode == kSym) {                                                               \
      MR_PACK_LPG(kSym, B)                                                                   \
    } else {                                                                                 \
      MR_PACK_LPG(kSearched, B)                                                              \
    }                                                                                        \
    break;                                                                                   \
  }
  switch (bits) {
    MR_PACK_BITS(2)
    MR_PACK_BITS(3)
    MR_PACK_BITS(4)
    MR_PACK_BITS(5)
    MR_PACK_BITS(6)
    MR_PACK_BITS(7)
    MR_PACK_BITS(8)
    default: return MR_ERR_ARGUMENT;
  }
#undef MR_PACK_BITS
#undef MR_PACK_ARGS
#undef MR_PACK_LPG
  return launch_status();
}
