// Fused element-wise kernels of the decoder block (forward and backward).
//
// Each kernel reads float32 activations once and writes the next GEMM's
// operand directly as a bf16 hi/lo pair (hi = bf16(y), lo = bf16(y - hi)),
// so no float32 intermediate is materialised between an element-wise op and
// the tcgen05 GEMM that consumes it.  The math is the mlx-lm decoder layer's
// (the layer the reference runs in block_output,
// mround/pipeline/blocks.py:578-606): RMSNorm, non-interleaved RoPE, causal
// softmax, SwiGLU, and their derivatives.  All HBM-bound.
//
// Layouts: token t = b*S + s; qkv rows are [q heads | k heads | v heads] x D;
// attention operands are (B, H, S, D) contiguous.

#include "common.cuh"

namespace mr {
namespace {

__device__ __forceinline__ void put_split(uint16_t* hi, uint16_t* lo, int64_t i, float v) {
  const uint16_t h = f32_to_bf16(v);
  hi[i] = h;
  lo[i] = f32_to_bf16(__fsub_rn(v, bf16_to_f32(h)));
}

__device__ __forceinline__ void put_split4(uint16_t* hi, uint16_t* lo, int64_t i, float4 v) {
  const float f[4] = {v.x, v.y, v.z, v.w};
  uint16_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    h[j] = f32_to_bf16(f[j]);
    l[j] = f32_to_bf16(__fsub_rn(f[j], bf16_to_f32(h[j])));
  }
  *reinterpret_cast<uint2*>(hi + i) = make_uint2(uint32_t(h[0]) | (uint32_t(h[1]) << 16),
                                                 uint32_t(h[2]) | (uint32_t(h[3]) << 16));
  *reinterpret_cast<uint2*>(lo + i) = make_uint2(uint32_t(l[0]) | (uint32_t(l[1]) << 16),
                                                 uint32_t(l[2]) | (uint32_t(l[3]) << 16));
}

// Operand outputs of one element-wise kernel: the bf16 hi/lo pair (when hi is
// given) and/or the tf32-rounded float32 copy (when t32 is given).
__device__ __forceinline__ void put_out(uint16_t* hi, uint16_t* lo, float* t32, int64_t i,
                                        float v) {
  if (hi) put_split(hi, lo, i, v);
  if (t32) t32[i] = tf32_rna(v);
}

__device__ __forceinline__ void put_out4(uint16_t* hi, uint16_t* lo, float* t32, int64_t i,
                                         float4 v) {
  if (hi) put_split4(hi, lo, i, v);
  if (t32)
    *reinterpret_cast<float4*>(t32 + i) =
        make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
}

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) s += sh[i];
  __syncthreads();
  return s;
}

template <int THREADS>
__device__ __forceinline__ float block_max(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  float s = -INFINITY;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) s = fmaxf(s, sh[i]);
  __syncthreads();
  return s;
}

constexpr int kRowThreads = 128;
constexpr int kMaxVec = 16;  // float4 per thread: rows up to 8192

// y = x * rsqrt(mean(x^2) + eps) * w  -> hi/lo, and rstd per row.
__global__ void __launch_bounds__(kRowThreads) rmsnorm_split_kernel(
    const float* __restrict__ x, const uint16_t* __restrict__ w, int h, float eps,
    uint16_t* __restrict__ hi, uint16_t* __restrict__ lo, float* __restrict__ t32,
    float* __restrict__ rstd) {
  __shared__ float sh[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * h);
  const int n4 = h / 4;
  float4 v[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < n4) {
      v[i] = xr[c];
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
  }
  ss = block_sum<kRowThreads>(ss, sh);
  const float r = rsqrtf(ss / float(h) + eps);
  if (threadIdx.x == 0) rstd[row] = r;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < n4) {
      const int e = c * 4;
      float4 y;
      y.x = __fmul_rn(__fmul_rn(v[i].x, r), bf16_to_f32(w[e]));
      y.y = __fmul_rn(__fmul_rn(v[i].y, r), bf16_to_f32(w[e + 1]));
      y.z = __fmul_rn(__fmul_rn(v[i].z, r), bf16_to_f32(w[e + 2]));
      y.w = __fmul_rn(__fmul_rn(v[i].w, r), bf16_to_f32(w[e + 3]));
      put_out4(hi, lo, t32, row * h + e, y);
    }
  }
}

// dx = resid + rstd * (g - xhat * mean(g * xhat)),  g = dy * w,  xhat = x * rstd.
// Written as hi/lo (when hi is given), tf32-rounded float32 (when t32 is
// given) and/or float32 (when out is given); resid may be NULL (no residual
// term).
__global__ void __launch_bounds__(kRowThreads) rmsnorm_bwd_split_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, const uint16_t* __restrict__ w,
    const float* __restrict__ rstd, const float* __restrict__ resid, int h,
    uint16_t* __restrict__ hi, uint16_t* __restrict__ lo, float* __restrict__ t32,
    float* __restrict__ out) {
  __shared__ float sh[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const float r = rstd[row];
  const float4* dyr = reinterpret_cast<const float4*>(dy + row * h);
  const float4* xr = reinterpret_cast<const float4*>(x + row * h);
  const int n4 = h / 4;
  float4 g[kMaxVec], xh[kMaxVec];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < n4) {
      const int e = c * 4;
      const float4 a = dyr[c], b = xr[c];
      g[i] = make_float4(a.x * bf16_to_f32(w[e]), a.y * bf16_to_f32(w[e + 1]),
                         a.z * bf16_to_f32(w[e + 2]), a.w * bf16_to_f32(w[e + 3]));
      xh[i] = make_float4(b.x * r, b.y * r, b.z * r, b.w * r);
      dot += g[i].x * xh[i].x + g[i].y * xh[i].y + g[i].z * xh[i].z + g[i].w * xh[i].w;
    }
  }
  dot = block_sum<kRowThreads>(dot, sh) / float(h);
  const float4* rr = reinterpret_cast<const float4*>(resid + row * h);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < n4) {
      const float4 q = resid ? rr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 d;
      d.x = q.x + r * (g[i].x - xh[i].x * dot);
      d.y = q.y + r * (g[i].y - xh[i].y * dot);
      d.z = q.z + r * (g[i].z - xh[i].z * dot);
      d.w = q.w + r * (g[i].w - xh[i].w * dot);
      put_out4(hi, lo, t32, row * h + c * 4, d);
      if (out) reinterpret_cast<float4*>(out + row * h)[c] = d;
    }
  }
}

// qkv (T, (Hq+2Hkv)*D) -> rope(q), rope(k), v as (B,H,S,D) hi/lo.
__global__ void rope_split_kernel(const float* __restrict__ qkv, const float* __restrict__ cosv,
                                  const float* __restrict__ sinv, int B, int S, int Hq, int Hkv,
                                  int D, uint16_t* __restrict__ q_hi, uint16_t* __restrict__ q_lo,
                                  uint16_t* __restrict__ k_hi, uint16_t* __restrict__ k_lo,
                                  uint16_t* __restrict__ v_hi, uint16_t* __restrict__ v_lo) {
  const int half = D / 2;
  const int H = Hq + 2 * Hkv;
  const int64_t total = int64_t(B) * S * H * half;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int j = int(idx % half);
    const int head = int((idx / half) % H);
    const int64_t t = idx / (int64_t(half) * H);
    const int s = int(t % S);
    const int b = int(t / S);
    const float* src = qkv + t * int64_t(H) * D + int64_t(head) * D;
    const float x1 = src[j], x2 = src[j + half];
    float o1 = x1, o2 = x2;
    uint16_t *dh, *dl;
    int64_t base;
    if (head < Hq + Hkv) {
      const float c = cosv[int64_t(s) * half + j], sn = sinv[int64_t(s) * half + j];
      o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
      o2 = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, c));
    }
    if (head < Hq) {
      dh = q_hi; dl = q_lo;
      base = ((int64_t(b) * Hq + head) * S + s) * D;
    } else if (head < Hq + Hkv) {
      dh = k_hi; dl = k_lo;
      base = ((int64_t(b) * Hkv + (head - Hq)) * S + s) * D;
    } else {
      dh = v_hi; dl = v_lo;
      base = ((int64_t(b) * Hkv + (head - Hq - Hkv)) * S + s) * D;
    }
    put_split(dh, dl, base + j, o1);
    put_split(dh, dl, base + j + half, o2);
  }
}

// dq, dk, dv (B,H,S,D) -> dqkv (T, (Hq+2Hkv)*D) hi/lo, undoing the rotation.
__global__ void rope_bwd_split_kernel(const float* __restrict__ dq, const float* __restrict__ dk,
                                      const float* __restrict__ dv, const float* __restrict__ cosv,
                                      const float* __restrict__ sinv, int B, int S, int Hq, int Hkv,
                                      int D, uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                                      float* __restrict__ t32) {
  const int half = D / 2;
  const int H = Hq + 2 * Hkv;
  const int64_t total = int64_t(B) * S * H * half;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int j = int(idx % half);
    const int head = int((idx / half) % H);
    const int64_t t = idx / (int64_t(half) * H);
    const int s = int(t % S);
    const int b = int(t / S);
    const float* src;
    if (head < Hq) src = dq + ((int64_t(b) * Hq + head) * S + s) * D;
    else if (head < Hq + Hkv) src = dk + ((int64_t(b) * Hkv + (head - Hq)) * S + s) * D;
    else src = dv + ((int64_t(b) * Hkv + (head - Hq - Hkv)) * S + s) * D;
    const float d1 = src[j], d2 = src[j + half];
    float g1 = d1, g2 = d2;
    if (head < Hq + Hkv) {
      const float c = cosv[int64_t(s) * half + j], sn = sinv[int64_t(s) * half + j];
      g1 = d1 * c + d2 * sn;
      g2 = d2 * c - d1 * sn;
    }
    const int64_t o = t * int64_t(H) * D + int64_t(head) * D;
    put_out(hi, lo, t32, o + j, g1);
    put_out(hi, lo, t32, o + j + half, g2);
  }
}

// (B,H,S,D) float32 <-> (T, H*D): merge=1 reads heads and writes token rows.
__global__ void heads_kernel(const float* __restrict__ src, int B, int S, int H, int D, int merge,
                             uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                             float* __restrict__ t32) {
  const int64_t total4 = int64_t(B) * S * H * D / 4;
  for (int64_t i4 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i4 < total4;
       i4 += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i4 * 4;
    // e indexes the destination
    int64_t s_idx;
    if (merge) {  // dest (t, h, d)
      const int d = int(e % D);
      const int h = int((e / D) % H);
      const int64_t t = e / (int64_t(D) * H);
      const int s = int(t % S), b = int(t / S);
      s_idx = ((int64_t(b) * H + h) * S + s) * D + d;
    } else {  // dest (b, h, s, d) from (t, h, d)
      const int d = int(e % D);
      const int s = int((e / D) % S);
      const int h = int((e / (int64_t(D) * S)) % H);
      const int b = int(e / (int64_t(D) * S * H));
      s_idx = ((int64_t(b) * S + s) * H + h) * D + d;
    }
    put_out4(hi, lo, t32, e, *reinterpret_cast<const float4*>(src + s_idx));
  }
}

// Token-row forms of the three kernels above for head dims divisible by 8:
// one block walks one token's row (all heads), each thread 4 columns of a
// head's first half and the matching 4 of its second half, with 16-byte loads
// and 8-byte hi/lo stores; the index arithmetic is 32-bit inside the row
// (the per-element 64-bit divisions of the forms above made them issue-bound).
__device__ __forceinline__ float4 ldv4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

__device__ __forceinline__ float4 rot_fwd1(float4 x1, float4 x2, float4 c, float4 sn) {
  return make_float4(__fsub_rn(__fmul_rn(x1.x, c.x), __fmul_rn(x2.x, sn.x)),
                     __fsub_rn(__fmul_rn(x1.y, c.y), __fmul_rn(x2.y, sn.y)),
                     __fsub_rn(__fmul_rn(x1.z, c.z), __fmul_rn(x2.z, sn.z)),
                     __fsub_rn(__fmul_rn(x1.w, c.w), __fmul_rn(x2.w, sn.w)));
}

__device__ __forceinline__ float4 rot_fwd2(float4 x1, float4 x2, float4 c, float4 sn) {
  return make_float4(__fadd_rn(__fmul_rn(x1.x, sn.x), __fmul_rn(x2.x, c.x)),
                     __fadd_rn(__fmul_rn(x1.y, sn.y), __fmul_rn(x2.y, c.y)),
                     __fadd_rn(__fmul_rn(x1.z, sn.z), __fmul_rn(x2.z, c.z)),
                     __fadd_rn(__fmul_rn(x1.w, sn.w), __fmul_rn(x2.w, c.w)));
}

__global__ void __launch_bounds__(256) rope_row_kernel(
    const float* __restrict__ qkv, const float* __restrict__ cosv, const float* __restrict__ sinv,
    int B, int S, int Hq, int Hkv, int D, uint16_t* __restrict__ q_hi, uint16_t* __restrict__ q_lo,
    uint16_t* __restrict__ k_hi, uint16_t* __restrict__ k_lo, uint16_t* __restrict__ v_hi,
    uint16_t* __restrict__ v_lo) {
  const int half = D / 2, per_head = half / 4;
  const int H = Hq + 2 * Hkv;
  const int units = H * per_head;
  const int64_t T = int64_t(B) * S;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const int s = int(t % S), b = int(t / S);
    const float* row = qkv + t * int64_t(H) * D;
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      const int head = u / per_head;
      const int j = (u - head * per_head) * 4;
      const float4 x1 = ldv4(row + head * D + j), x2 = ldv4(row + head * D + half + j);
      float4 o1 = x1, o2 = x2;
      if (head < Hq + Hkv) {
        const float4 c = ldv4(cosv + int64_t(s) * half + j), sn = ldv4(sinv + int64_t(s) * half + j);
        o1 = rot_fwd1(x1, x2, c, sn);
        o2 = rot_fwd2(x1, x2, c, sn);
      }
      uint16_t *dh, *dl;
      int64_t base;
      if (head < Hq) {
        dh = q_hi; dl = q_lo;
        base = ((int64_t(b) * Hq + head) * S + s) * D;
      } else if (head < Hq + Hkv) {
        dh = k_hi; dl = k_lo;
        base = ((int64_t(b) * Hkv + (head - Hq)) * S + s) * D;
      } else {
        dh = v_hi; dl = v_lo;
        base = ((int64_t(b) * Hkv + (head - Hq - Hkv)) * S + s) * D;
      }
      put_split4(dh, dl, base + j, o1);
      put_split4(dh, dl, base + half + j, o2);
    }
  }
}

__global__ void __launch_bounds__(256) rope_bwd_row_kernel(
    const float* __restrict__ dq, const float* __restrict__ dk, const float* __restrict__ dv,
    const float* __restrict__ cosv, const float* __restrict__ sinv, int B, int S, int Hq, int Hkv,
    int D, uint16_t* __restrict__ hi, uint16_t* __restrict__ lo, float* __restrict__ t32) {
  const int half = D / 2, per_head = half / 4;
  const int H = Hq + 2 * Hkv;
  const int units = H * per_head;
  const int64_t T = int64_t(B) * S;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const int s = int(t % S), b = int(t / S);
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      const int head = u / per_head;
      const int j = (u - head * per_head) * 4;
      const float* src;
      if (head < Hq) src = dq + ((int64_t(b) * Hq + head) * S + s) * D;
      else if (head < Hq + Hkv) src = dk + ((int64_t(b) * Hkv + (head - Hq)) * S + s) * D;
      else src = dv + ((int64_t(b) * Hkv + (head - Hq - Hkv)) * S + s) * D;
      const float4 d1 = ldv4(src + j), d2 = ldv4(src + half + j);
      float4 g1 = d1, g2 = d2;
      if (head < Hq + Hkv) {
        const float4 c = ldv4(cosv + int64_t(s) * half + j), sn = ldv4(sinv + int64_t(s) * half + j);
        g1 = make_float4(d1.x * c.x + d2.x * sn.x, d1.y * c.y + d2.y * sn.y,
                         d1.z * c.z + d2.z * sn.z, d1.w * c.w + d2.w * sn.w);
        g2 = make_float4(d2.x * c.x - d1.x * sn.x, d2.y * c.y - d1.y * sn.y,
                         d2.z * c.z - d1.z * sn.z, d2.w * c.w - d1.w * sn.w);
      }
      const int64_t o = t * int64_t(H) * D + int64_t(head) * D;
      put_out4(hi, lo, t32, o + j, g1);
      put_out4(hi, lo, t32, o + half + j, g2);
    }
  }
}

// heads (B,H,S,D) <-> token rows (T, H*D), one token's row per block iteration
__global__ void __launch_bounds__(256) heads_row_kernel(const float* __restrict__ src, int B, int S,
                                                        int H, int D, int merge,
                                                        uint16_t* __restrict__ hi,
                                                        uint16_t* __restrict__ lo,
                                                        float* __restrict__ t32) {
  const int per_head = D / 4;
  const int units = H * per_head;
  const int64_t T = int64_t(B) * S;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const int s = int(t % S), b = int(t / S);
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      const int h = u / per_head;
      const int d = (u - h * per_head) * 4;
      const int64_t row_idx = t * int64_t(H) * D + int64_t(u) * 4;
      const int64_t head_idx = ((int64_t(b) * H + h) * S + s) * D + d;
      if (merge)
        put_out4(hi, lo, t32, row_idx, ldv4(src + head_idx));
      else
        put_out4(hi, lo, t32, head_idx, ldv4(src + row_idx));
    }
  }
}

__device__ __forceinline__ float silu_of(float g) { return g / (1.f + expf(-g)); }

// act = silu(g) * u, gu = [g | u] per row -> hi/lo (T, I), and a tf32 copy
// when t32 is given.
__global__ void swiglu_split_kernel(const float* __restrict__ gu, int64_t T, int I,
                                    uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                                    float* __restrict__ t32) {
  const int64_t total4 = T * I / 4;
  for (int64_t i4 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i4 < total4;
       i4 += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i4 * 4;
    const int64_t t = e / I;
    const int c = int(e % I);
    const float4 g = *reinterpret_cast<const float4*>(gu + t * 2 * I + c);
    const float4 u = *reinterpret_cast<const float4*>(gu + t * 2 * I + I + c);
    float4 a;
    a.x = silu_of(g.x) * u.x;
    a.y = silu_of(g.y) * u.y;
    a.z = silu_of(g.z) * u.z;
    a.w = silu_of(g.w) * u.w;
    put_out4(hi, lo, t32, e, a);
  }
}

// dgu = [dact * u * silu'(g) | dact * silu(g)] -> hi/lo and/or tf32 (T, 2I).
__global__ void swiglu_bwd_split_kernel(const float* __restrict__ dact,
                                        const float* __restrict__ gu, int64_t T, int I,
                                        uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                                        float* __restrict__ t32) {
  const int64_t total4 = T * I / 4;
  for (int64_t i4 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i4 < total4;
       i4 += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i4 * 4;
    const int64_t t = e / I;
    const int c = int(e % I);
    const float4 d = *reinterpret_cast<const float4*>(dact + e);
    const float4 g = *reinterpret_cast<const float4*>(gu + t * 2 * I + c);
    const float4 u = *reinterpret_cast<const float4*>(gu + t * 2 * I + I + c);
    const float gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {u.x, u.y, u.z, u.w};
    const float ds[4] = {d.x, d.y, d.z, d.w};
    float dg[4], du[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float sg = 1.f / (1.f + expf(-gs[j]));
      const float sl = gs[j] * sg;
      dg[j] = ds[j] * us[j] * (sg * (1.f + gs[j] * (1.f - sg)));
      du[j] = ds[j] * sl;
    }
    put_out4(hi, lo, t32, t * 2 * I + c, make_float4(dg[0], dg[1], dg[2], dg[3]));
    put_out4(hi, lo, t32, t * 2 * I + I + c, make_float4(du[0], du[1], du[2], du[3]));
  }
}

constexpr int kSoftThreads = 256;
constexpr int kSoftVec = 8;  // float4 per thread: rows up to 256 * 4 * 8 = 8192 columns

// Causal softmax rows, row r at position r % S.  With ``band`` set, columns
// from the end of the next 128-column block on are left unwritten: the causal
// GEMM modes never read them.
__device__ __forceinline__ int write_limit(int pos, int S, int band) {
  return band ? min(S, (pos / 128 + 2) * 128) : S;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ void unpack4(const uint2 u, float (&x)[4]) {
  x[0] = __uint_as_float(u.x << 16);
  x[1] = __uint_as_float(u.x & 0xFFFF0000u);
  x[2] = __uint_as_float(u.y << 16);
  x[3] = __uint_as_float(u.y & 0xFFFF0000u);
}

// P = softmax(scale * scores) over columns <= pos, written as bf16 hi/lo only
// (scores are not modified).  The row lives in registers: one float4 per
// thread and 1024-column chunk, read once with 16-byte loads.
__global__ void __launch_bounds__(kSoftThreads) softmax_causal_kernel(
    const float* __restrict__ scores, int S, float scale, int band, uint16_t* __restrict__ hi,
    uint16_t* __restrict__ lo) {
  __shared__ float sh[kSoftThreads / 32];
  const int64_t row = blockIdx.x;
  const int pos = int(row % S);
  const float* r = scores + row * S;
  float v[kSoftVec][4];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kSoftVec; ++i) {
    const int c = (i * kSoftThreads + threadIdx.x) * 4;
    if (c <= pos) {
      const float4 q = ld4(r + c);
      v[i][0] = __fmul_rn(q.x, scale);
      v[i][1] = c + 1 <= pos ? __fmul_rn(q.y, scale) : -INFINITY;
      v[i][2] = c + 2 <= pos ? __fmul_rn(q.z, scale) : -INFINITY;
      v[i][3] = c + 3 <= pos ? __fmul_rn(q.w, scale) : -INFINITY;
    } else {
      v[i][0] = v[i][1] = v[i][2] = v[i][3] = -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) m = fmaxf(m, v[i][j]);
  }
  m = block_max<kSoftThreads>(m, sh);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kSoftVec; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[i][j] = v[i][j] == -INFINITY ? 0.f : expf(v[i][j] - m);
      sum += v[i][j];
    }
  }
  sum = block_sum<kSoftThreads>(sum, sh);
  const float inv = 1.f / sum;
  const int lim = write_limit(pos, S, band);
#pragma unroll
  for (int i = 0; i < kSoftVec; ++i) {
    const int c = (i * kSoftThreads + threadIdx.x) * 4;
    if (c < lim)
      put_split4(hi, lo, row * S + c,
                 make_float4(v[i][0] * inv, v[i][1] * inv, v[i][2] * inv, v[i][3] * inv));
  }
}

// dS = scale * P * (dP - sum(dP * P)) -> hi/lo, with P = p_hi + p_lo.
__global__ void __launch_bounds__(kSoftThreads) softmax_bwd_kernel(
    const float* __restrict__ dp, const uint16_t* __restrict__ p_hi,
    const uint16_t* __restrict__ p_lo, int S, float scale, int band, uint16_t* __restrict__ hi,
    uint16_t* __restrict__ lo) {
  __shared__ float sh[kSoftThreads / 32];
  const int64_t row = blockIdx.x;
  const int pos = int(row % S);
  const float* dr = dp + row * S;
  float pv[kSoftVec][4], dv[kSoftVec][4];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < kSoftVec; ++i) {
    const int c = (i * kSoftThreads + threadIdx.x) * 4;
    if (c <= pos) {
      const float4 d = ld4(dr + c);
      float ph[4], pl[4];
      unpack4(*reinterpret_cast<const uint2*>(p_hi + row * S + c), ph);
      unpack4(*reinterpret_cast<const uint2*>(p_lo + row * S + c), pl);
      dv[i][0] = d.x; dv[i][1] = d.y; dv[i][2] = d.z; dv[i][3] = d.w;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        pv[i][j] = c + j <= pos ? __fadd_rn(ph[j], pl[j]) : 0.f;
        dot += pv[i][j] * dv[i][j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) pv[i][j] = dv[i][j] = 0.f;
    }
  }
  dot = block_sum<kSoftThreads>(dot, sh);
  const int lim = write_limit(pos, S, band);
#pragma unroll
  for (int i = 0; i < kSoftVec; ++i) {
    const int c = (i * kSoftThreads + threadIdx.x) * 4;
    if (c < lim) {
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = scale * pv[i][j] * (dv[i][j] - dot);
      put_split4(hi, lo, row * S + c, make_float4(o[0], o[1], o[2], o[3]));
    }
  }
}

// Rows up to 2048 columns: one warp per row, NV float4 per lane (columns
// 128 i + 4 lane .. +3); the reductions stay inside the warp (the block kernels
// above take longer rows).  Lanes past the causal position do not load.
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Four rows per block: the row stays in registers (86 per thread at 2048
// columns, 164 in the backward), and small blocks let more of them share an
// SM (measured at 8 x 28 x 2048 rows: 256-thread blocks 1.16 ms, 128-thread
// 0.98 ms for the forward).
constexpr int kSoftWarpThreads = 128;

template <int NV>
__global__ void __launch_bounds__(kSoftWarpThreads) softmax_causal_warp_kernel(
    const float* __restrict__ scores, int64_t rows, int S, float scale, int band,
    uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * (kSoftWarpThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int pos = int(row % S);
  const float* r = scores + row * S;
  float v[NV][4];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c <= pos) {
      const float4 q = __ldcs(reinterpret_cast<const float4*>(r + c));
      v[i][0] = __fmul_rn(q.x, scale);
      v[i][1] = c + 1 <= pos ? __fmul_rn(q.y, scale) : -INFINITY;
      v[i][2] = c + 2 <= pos ? __fmul_rn(q.z, scale) : -INFINITY;
      v[i][3] = c + 3 <= pos ? __fmul_rn(q.w, scale) : -INFINITY;
    } else {
      v[i][0] = v[i][1] = v[i][2] = v[i][3] = -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) m = fmaxf(m, v[i][j]);
  }
  m = warp_max(m);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[i][j] = v[i][j] == -INFINITY ? 0.f : expf(v[i][j] - m);
      sum += v[i][j];
    }
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  const int lim = write_limit(pos, S, band);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c < lim)
      put_split4(hi, lo, row * S + c,
                 make_float4(v[i][0] * inv, v[i][1] * inv, v[i][2] * inv, v[i][3] * inv));
  }
}


template <int NV>
__global__ void __launch_bounds__(kSoftWarpThreads) softmax_bwd_warp_kernel(
    const float* __restrict__ dp, const uint16_t* __restrict__ p_hi,
    const uint16_t* __restrict__ p_lo, int64_t rows, int S, float scale, int band,
    uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * (kSoftWarpThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int pos = int(row % S);
  const float* dr = dp + row * S;
  float dv[NV][4];
  uint2 ph[NV], pl[NV];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c <= pos) {
      const float4 d = __ldcs(reinterpret_cast<const float4*>(dr + c));
      ph[i] = __ldcs(reinterpret_cast<const uint2*>(p_hi + row * S + c));
      pl[i] = __ldcs(reinterpret_cast<const uint2*>(p_lo + row * S + c));
      dv[i][0] = d.x; dv[i][1] = d.y; dv[i][2] = d.z; dv[i][3] = d.w;
    } else {
      ph[i] = pl[i] = make_uint2(0u, 0u);
      dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    float a[4], b[4];
    unpack4(ph[i], a);
    unpack4(pl[i], b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a[j] = c + j <= pos ? __fadd_rn(a[j], b[j]) : 0.f;
      dot += a[j] * dv[i][j];
    }
  }
  dot = warp_sum(dot);
  const int lim = write_limit(pos, S, band);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c < lim) {
      float a[4], b[4], o[4];
      unpack4(ph[i], a);
      unpack4(pl[i], b);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = c + j <= pos ? __fadd_rn(a[j], b[j]) : 0.f;
        o[j] = scale * p * (dv[i][j] - dot);
      }
      put_split4(hi, lo, row * S + c, make_float4(o[0], o[1], o[2], o[3]));
    }
  }
}

// float4 per lane for the warp-per-row kernels (0: the row needs the block kernels)
int soft_vec(int s) {
  for (int nv = 1; nv <= 16; nv *= 2)
    if (s <= nv * 128) return nv;
  return 0;
}

int grid_elems(int64_t n, int threads = 256) { return grid_for(n, threads, 8); }

// one block per token row, at most 2^31 - 1 blocks (the kernels stride beyond)
unsigned row_grid(int64_t tokens) { return unsigned(tokens < 0x7fffffff ? tokens : 0x7fffffff); }

bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

}  // namespace
}  // namespace mr

using namespace mr;

extern "C" int mr_rmsnorm_split(const float* x, const uint16_t* w, int64_t rows, int h, float eps,
                                uint16_t* hi, uint16_t* lo, float* t32, float* rstd,
                                void* stream) {
  if (!x || !w || !hi || !lo || !rstd || rows <= 0 || h <= 0 || h % 4 || h > 4 * kMaxVec * kRowThreads)
    return MR_ERR_ARGUMENT;
  if (!aligned16(x) || (t32 && !aligned16(t32))) return MR_ERR_ALIGNMENT;
  rmsnorm_split_kernel<<<unsigned(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, w, h, eps, hi, lo, t32, rstd);
  return launch_status();
}

extern "C" int mr_rmsnorm_bwd_split(const float* dy, const float* x, const uint16_t* w,
                                    const float* rstd, const float* resid, int64_t rows, int h,
                                    uint16_t* hi, uint16_t* lo, float* t32, float* out,
                                    void* stream) {
  if (!dy || !x || !w || !rstd || rows <= 0 || h <= 0 || h % 4 ||
      h > 4 * kMaxVec * kRowThreads)
    return MR_ERR_ARGUMENT;
  if ((hi == nullptr) != (lo == nullptr) || (!hi && !out && !t32)) return MR_ERR_ARGUMENT;
  if (!aligned16(dy) || !aligned16(x) || (resid && !aligned16(resid)) || (out && !aligned16(out)) ||
      (t32 && !aligned16(t32)))
    return MR_ERR_ALIGNMENT;
  rmsnorm_bwd_split_kernel<<<unsigned(rows), kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      dy, x, w, rstd, resid, h, hi, lo, t32, out);
  return launch_status();
}

extern "C" int mr_rope_split(const float* qkv, const float* cosv, const float* sinv, int b, int s,
                             int hq, int hkv, int d, uint16_t* q_hi, uint16_t* q_lo,
                             uint16_t* k_hi, uint16_t* k_lo, uint16_t* v_hi, uint16_t* v_lo,
                             void* stream) {
  if (!qkv || !cosv || !sinv || b <= 0 || s <= 0 || hq <= 0 || hkv <= 0 || d <= 0 || d % 2)
    return MR_ERR_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool rows = d % 8 == 0 && aligned16(qkv) && aligned16(cosv) && aligned16(sinv) &&
                    aligned8(q_hi) && aligned8(q_lo) && aligned8(k_hi) && aligned8(k_lo) &&
                    aligned8(v_hi) && aligned8(v_lo);
  if (rows) {
    rope_row_kernel<<<row_grid(int64_t(b) * s), 256, 0, st>>>(qkv, cosv, sinv, b, s, hq, hkv, d,
                                                               q_hi, q_lo, k_hi, k_lo, v_hi, v_lo);
  } else {
    const int64_t total = int64_t(b) * s * (hq + 2 * hkv) * (d / 2);
    rope_split_kernel<<<grid_elems(total), 256, 0, st>>>(qkv, cosv, sinv, b, s, hq, hkv, d, q_hi,
                                                         q_lo, k_hi, k_lo, v_hi, v_lo);
  }
  return launch_status();
}

extern "C" int mr_rope_bwd_split(const float* dq, const float* dk, const float* dv,
                                 const float* cosv, const float* sinv, int b, int s, int hq,
                                 int hkv, int d, uint16_t* hi, uint16_t* lo, float* t32,
                                 void* stream) {
  if (!dq || !dk || !dv || !cosv || !sinv || b <= 0 || s <= 0 || d % 2) return MR_ERR_ARGUMENT;
  if ((hi == nullptr) != (lo == nullptr) || (!hi && !t32)) return MR_ERR_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool rows = d % 8 == 0 && aligned16(dq) && aligned16(dk) && aligned16(dv) &&
                    aligned16(cosv) && aligned16(sinv) && aligned8(hi) && aligned8(lo) &&
                    aligned16(t32);
  if (rows) {
    rope_bwd_row_kernel<<<row_grid(int64_t(b) * s), 256, 0, st>>>(dq, dk, dv, cosv, sinv, b, s, hq,
                                                                   hkv, d, hi, lo, t32);
  } else {
    const int64_t total = int64_t(b) * s * (hq + 2 * hkv) * (d / 2);
    rope_bwd_split_kernel<<<grid_elems(total), 256, 0, st>>>(dq, dk, dv, cosv, sinv, b, s, hq, hkv,
                                                             d, hi, lo, t32);
  }
  return launch_status();
}

extern "C" int mr_heads_split(const float* src, int b, int s, int h, int d, int merge,
                              uint16_t* hi, uint16_t* lo, float* t32, void* stream) {
  if (!src || !hi || !lo || b <= 0 || s <= 0 || h <= 0 || d % 4) return MR_ERR_ARGUMENT;
  if (!aligned16(src) || !aligned16(t32)) return MR_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (aligned8(hi) && aligned8(lo)) {
    heads_row_kernel<<<row_grid(int64_t(b) * s), 256, 0, st>>>(src, b, s, h, d, merge, hi, lo,
                                                                t32);
  } else {
    const int64_t total4 = int64_t(b) * s * h * d / 4;
    heads_kernel<<<grid_elems(total4), 256, 0, st>>>(src, b, s, h, d, merge, hi, lo, t32);
  }
  return launch_status();
}

extern "C" int mr_swiglu_split(const float* gu, int64_t t, int i, uint16_t* hi, uint16_t* lo,
                               float* t32, void* stream) {
  if (!gu || !hi || !lo || t <= 0 || i <= 0 || i % 4) return MR_ERR_ARGUMENT;
  if (!aligned16(gu) || !aligned16(t32)) return MR_ERR_ALIGNMENT;
  swiglu_split_kernel<<<grid_elems(t * i / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      gu, t, i, hi, lo, t32);
  return launch_status();
}

extern "C" int mr_swiglu_bwd_split(const float* dact, const float* gu, int64_t t, int i,
                                   uint16_t* hi, uint16_t* lo, float* t32, void* stream) {
  if (!dact || !gu || t <= 0 || i <= 0 || i % 4) return MR_ERR_ARGUMENT;
  if ((hi == nullptr) != (lo == nullptr) || (!hi && !t32)) return MR_ERR_ARGUMENT;
  if (!aligned16(dact) || !aligned16(gu) || !aligned16(t32)) return MR_ERR_ALIGNMENT;
  swiglu_bwd_split_kernel<<<grid_elems(t * i / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      dact, gu, t, i, hi, lo, t32);
  return launch_status();
}

extern "C" int mr_softmax_causal_split(const float* scores, int64_t rows, int s, float scale,
                                       int band, uint16_t* hi, uint16_t* lo, void* stream) {
  if (!scores || !hi || !lo || rows <= 0 || s <= 0 || rows % s) return MR_ERR_ARGUMENT;
  if (s % 4 || s > 4 * kSoftVec * kSoftThreads) return MR_ERR_ARGUMENT;
  if (!aligned16(scores) || (reinterpret_cast<uintptr_t>(hi) & 7u) ||
      (reinterpret_cast<uintptr_t>(lo) & 7u))
    return MR_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned warp_grid = unsigned((rows + kSoftWarpThreads / 32 - 1) / (kSoftWarpThreads / 32));
  switch (soft_vec(s)) {
#define MR_SOFT(NV)                                                                  \
    case NV:                                                                         \
      softmax_causal_warp_kernel<NV><<<warp_grid, kSoftWarpThreads, 0, st>>>(scores, rows, s, scale, \
                                                                          band, hi, lo);         \
      break;
    MR_SOFT(1) MR_SOFT(2) MR_SOFT(4) MR_SOFT(8) MR_SOFT(16)
#undef MR_SOFT
    default:
      softmax_causal_kernel<<<unsigned(rows), kSoftThreads, 0, st>>>(scores, s, scale, band, hi, lo);
  }
  return launch_status();
}

extern "C" int mr_softmax_bwd_split(const float* dp, const uint16_t* p_hi, const uint16_t* p_lo,
                                    int64_t rows, int s, float scale, int band, uint16_t* hi,
                                    uint16_t* lo, void* stream) {
  if (!dp || !p_hi || !p_lo || !hi || !lo || rows <= 0 || s <= 0 || rows % s)
    return MR_ERR_ARGUMENT;
  if (s % 4 || s > 4 * kSoftVec * kSoftThreads) return MR_ERR_ARGUMENT;
  if (!aligned16(dp) || ((reinterpret_cast<uintptr_t>(p_hi) | reinterpret_cast<uintptr_t>(p_lo) |
                          reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 7u))
    return MR_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned warp_grid = unsigned((rows + kSoftWarpThreads / 32 - 1) / (kSoftWarpThreads / 32));
  switch (soft_vec(s)) {
#define MR_SOFT(NV)                                                                        \
    case NV:                                                                               \
      softmax_bwd_warp_kernel<NV><<<warp_grid, kSoftWarpThreads, 0, st>>>(dp, p_hi, p_lo, rows, s,  \
                                                                       scale, band, hi, lo);    \
      break;
    MR_SOFT(1) MR_SOFT(2) MR_SOFT(4) MR_SOFT(8) MR_SOFT(16)
#undef MR_SOFT
    default:
      softmax_bwd_kernel<<<unsigned(rows), kSoftThreads, 0, st>>>(dp, p_hi, p_lo, s, scale, band,
                                                                  hi, lo);
  }
  return launch_status();
}

namespace mr {
namespace {

__global__ void round_tf32_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
  const int64_t n4 = n / 4;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    reinterpret_cast<float4*>(out)[i] =
        make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
  }
  for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    out[i] = tf32_rna(x[i]);
}

}  // namespace
}  // namespace mr

extern "C" int mr_round_tf32(const float* x, int64_t n, float* out, void* stream) {
  if (!x || !out || n <= 0) return MR_ERR_ARGUMENT;
  if (!aligned16(x) || !aligned16(out)) return MR_ERR_ALIGNMENT;
  round_tf32_kernel<<<grid_elems((n + 3) / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n,
                                                                                             out);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Cross-entropy gradient of the scoring backward: for each of `rows` logit
// rows of `vocab` float32 values and its label,
//   g = (softmax(x) - onehot(label)) * scale
// written as bf16 hi/lo (the next GEMM's operand).  One block per row: an
// online max / sum of exponentials over the row (16-byte loads), then a
// second pass that writes g.  The row is read twice (the second read mostly
// from L2) and nothing else is materialised.
namespace mr {
namespace {

constexpr int kCeThreads = 512;

__device__ __forceinline__ void lse_combine(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * expf(m - m2) + s2;
    m = m2;
  } else if (m2 != -INFINITY) {
    s += s2 * expf(m2 - m);
  }
}

__global__ void __launch_bounds__(kCeThreads) ce_grad_split_kernel(
    const float* __restrict__ logits, const int64_t* __restrict__ labels, int vocab, float scale,
    uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
  __shared__ float sm[kCeThreads / 32], ss[kCeThreads / 32];
  const int64_t row = blockIdx.x;
  const float4* x4 = reinterpret_cast<const float4*>(logits + row * vocab);
  const int n4 = vocab / 4;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < n4; i += kCeThreads) {
    const float4 v = x4[i];
    const float mv = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
    if (mv > m) {
      s *= expf(m - mv);
      m = mv;
    }
    s += expf(v.x - m) + expf(v.y - m) + expf(v.z - m) + expf(v.w - m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    lse_combine(m, s, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  float M = sm[0], S = ss[0];
  for (int i = 1; i < kCeThreads / 32; ++i) lse_combine(M, S, sm[i], ss[i]);
  const float inv = 1.f / S;
  const int64_t label = labels[row];
  for (int i = threadIdx.x; i < n4; i += kCeThreads) {
    const float4 v = x4[i];
    float4 g = make_float4(expf(v.x - M) * inv, expf(v.y - M) * inv, expf(v.z - M) * inv,
                           expf(v.w - M) * inv);
    const int64_t c = int64_t(i) * 4;
    if (label >= c && label < c + 4) {
      const int j = int(label - c);
      if (j == 0) g.x -= 1.f;
      if (j == 1) g.y -= 1.f;
      if (j == 2) g.z -= 1.f;
      if (j == 3) g.w -= 1.f;
    }
    put_split4(hi, lo, row * vocab + c,
               make_float4(g.x * scale, g.y * scale, g.z * scale, g.w * scale));
  }
}

}  // namespace
}  // namespace mr

extern "C" int mr_ce_grad_split(const float* logits, const int64_t* labels, int64_t rows,
                                int vocab, float scale, uint16_t* hi, uint16_t* lo,
                                void* stream) {
  if (!logits || !labels || !hi || !lo || rows <= 0 || rows > 0x7fffffff || vocab <= 0 ||
      vocab % 4)
    return MR_ERR_ARGUMENT;
  if (!aligned16(logits) || !aligned8(hi) || !aligned8(lo)) return MR_ERR_ALIGNMENT;
  ce_grad_split_kernel<<<unsigned(rows), kCeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, labels, vocab, scale, hi, lo);
  return launch_status();
}
