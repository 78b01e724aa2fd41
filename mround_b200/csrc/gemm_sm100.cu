// K3 -- tcgen05/TMEM GEMM for the decoder-block linears (sm_100a).
//
//   C[m, n] (+)= sum_k A[m, k] * B[n, k]  (+ bias[n]),  float32 accumulate.
//
// Operands are bf16 and may carry a second "lo" part (x = hi + lo, lo =
// bf16(x - hi)), so float32 activations and fake-quantized weights reach the
// tensor cores with 16 significant bits: precision 3 issues hi*hi + hi*lo +
// lo*hi into one TMEM accumulator, precision 2 hi*hi + lo*hi (B exact in
// bf16), precision 1 hi*hi.  Precision 4 is one tf32 product
// (tcgen05.mma kind::tf32): both operands are float32 tensors whose values
// the producer has already rounded to tf32 (10 explicit mantissa bits, round
// to nearest), so the tensor core's reading of the upper 19 bits is exact.
// A tf32 product costs two bf16 products of tensor time and carries 11
// significant bits per operand.
//
// Structure: a persistent kernel, one CTA (192 threads) per SM, walking the
// flattened (batch, M-tile, N-tile) list of 128 x BN output tiles with stride
// gridDim.x (grouped rasterization: 16 M-tiles share each sweep over N):
//   warp 0, one lane : TMA producer.  Loads 32- or 64-wide K slices of A and B (hi
//                      and lo parts) into a ring of up to 8 swizzled
//                      shared-memory stages, continuing across tiles; completion is
//                      tracked by the stage's "full" mbarrier (transaction bytes).
//   warp 1           : allocates two TMEM accumulators (2 x BN columns); one
//                      lane issues tcgen05.mma (M=128, N=BN, K=16) per 16-wide K
//                      step and per product into accumulator (tile & 1),
//                      tcgen05.commit to the stage's "empty" mbarrier so the
//                      producer can refill it, and to "tmem_full" at tile end.
//   warps 2-5        : epilogue.  Each warp reads the 32 TMEM lanes (rows) it
//                      may access with tcgen05.ld 32x32b.x32, adds bias / the
//                      previous C, stores float32 rows, and arrives on
//                      "tmem_empty" -- while the MMAs of the next tile run in
//                      the other accumulator.
// Operand majorness: K-major tiles are TMA boxes {BK (K), rows} whose rows of
// BK elements (64 or 128 bytes) are swizzled at their width; MN-major tiles
// are boxes {128 bytes of M or N, BK (K)}, one per MN chunk (64 bf16 or 32
// float32 values).  The UMMA shared-memory descriptors describe the canonical
// layouts of both (K-major: 8-row groups 8 rows apart; bf16 MN-major: 128-byte
// swizzle, 8-K-row groups 1024 B apart; float32 MN-major: the 128-byte
// swizzle of 32-byte atoms that kind::tf32 requires, 4-K-row groups 512 B
// apart; MN chunks one box apart).
// K slices are 32 wide (64-byte rows) when an operand is K-major: a stage is
// then 48 KB for three products at BN = 256, four stages fit, and the loads
// run several MMA groups ahead.  With both operands MN-major the slices are 64
// wide (128-byte rows), keeping each TMA box at 8 KB.
// Every mbarrier wait is bounded in time: a wait that exceeds the limit sets
// the device status word (read with mr_gemm_status), and all roles skip their
// remaining work, wait (bounded) for their own issued copies and MMAs, and
// free TMEM before returning.  Loads are plain tiled TMA (no multicast).

#include <cuda.h>
#include <string.h>

#include <atomic>
#include <cmath>

#include "common.cuh"

namespace mr {
namespace {

constexpr int BM = 128;
// K per stage (BK): 32 (K-major rows of 64 B, SWIZZLE_64B) or 64 (128 B rows,
// SWIZZLE_128B); MN-major tiles always have 128-byte rows (64 M or N values).
constexpr int kThreads = 192;
// K slice of the tf32 GEMM (float32 operands): 32 -- four 48 KB stages at
// BN = 256, four MMAs per stage, each operand part one TMA instruction.
constexpr int kTf32BK = 32;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait

__device__ int g_gemm_status = 0;

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; returns false (and raises the status word) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        atomicExch(&g_gemm_status, MR_ERR_TIMEOUT);
        return false;
      }
      if (*reinterpret_cast<volatile int*>(&g_gemm_status) != 0) return false;
    }
  }
}

// Tiled 3-D TMA load (x innermost, z = batch); no multicast.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Tiled 4-D TMA load (x innermost, w = batch); no multicast.  The chunked
// operand maps put a 128-byte chunk of the contiguous dimension in x, so one
// instruction fills a whole operand tile of a stage.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t addr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(cols));
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 columns of float32 from TMEM: thread i gets row (lane base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- descriptors
// UMMA shared-memory descriptor for a swizzled canonical layout
// (layout type 2 = SWIZZLE_128B, 4 = SWIZZLE_64B, 1 = SWIZZLE_128B with
// 32-byte atoms).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;  // descriptor version (sm_100)
  d |= uint64_t(layout) << 61;
  return d;
}

// Instruction descriptor: bf16 x bf16 (or tf32 x tf32) -> f32, M=128, N=BN,
// given majorness.
__host__ __device__ constexpr uint32_t instr_desc(int n, bool a_mn, bool b_mn, bool tf32) {
  return (1u << 4)                       // D format f32
         | ((tf32 ? 2u : 1u) << 7)       // A bf16 (1) or tf32 (2)
         | ((tf32 ? 2u : 1u) << 10)      // B bf16 (1) or tf32 (2)
         | (uint32_t(a_mn) << 15)        // A major
         | (uint32_t(b_mn) << 16)        // B major
         | (uint32_t(n >> 3) << 17)      // N
         | (uint32_t(BM >> 4) << 24);    // M
}

// MP: M parts per tile.  1: a 128 x BN tile, two TMEM accumulators (the
// epilogue of one tile overlaps the next tile's MMAs).  2 (tf32 only, BN of
// 224 or 256): a 256 x BN tile as two 128-row MMAs per K step sharing one B
// tile -- 1.5x the flops per staged byte of the 128 x 256 tile -- in the two
// halves of TMEM, so one tile is in flight and its epilogue does not overlap.
template <int BN, int BK, int PREC, int MP = 1>
struct Cfg {
  static constexpr bool kTf32 = PREC == 4;
  static constexpr int kElt = kTf32 ? 4 : 2;              // operand element bytes
  static constexpr int kMmaK = 32 / kElt;                 // K of one MMA (32 bytes)
  static constexpr int kA = BM * BK * kElt;               // bytes of one A part per stage
  static constexpr int kB = BN * BK * kElt;               // bytes of one B part per stage
  static constexpr int kAParts = (PREC == 2 || PREC == 3) ? 2 : 1;
  static constexpr int kBParts = PREC == 3 ? 2 : 1;
  static constexpr int kStage = kA * kAParts * MP + kB * kBParts;
  static constexpr int kStages = (200 * 1024) / kStage > 8 ? 8 : (200 * 1024) / kStage;
  // per epilogue warp, a 32 x 32 float32 block (padded rows) through which the
  // fused reduce-scatter turns row-per-lane values into row-contiguous stores
  static constexpr int kStaging = 4 * 32 * 33 * 4;
  static constexpr int kSmem = kStages * kStage + 1024 /* align */ + 256 /* barriers */ + kStaging;
  // TMEM: two accumulators of BN columns, the second at column kAccCols; the
  // allocation is a power of two (224 -> 256 per accumulator, 512 in all)
  static constexpr int kAccCols = BN <= 128 ? 128 : 256;
  static constexpr int kTmemCols = 2 * kAccCols;
  static constexpr int kBufs = MP == 2 ? 1 : 2;  // tiles whose accumulators are in flight
  static_assert(BN % 32 == 0 && BN <= kAccCols && kTmemCols <= 512,
                "two accumulators must fit the 512 TMEM columns");
  static_assert(MP == 1 || (MP == 2 && kTf32 && kAccCols == 256),
                "two M parts: tf32 with 224- or 256-wide tiles");
};

// Operand maps of one launch.  a_chunked / b_chunked: the map is 4-D with a
// 128-byte chunk of the contiguous dimension innermost (one TMA instruction
// per operand part and stage); otherwise 3-D (K-major: one box; MN-major: one
// box per 128-byte MN chunk).
struct Maps {
  CUtensorMap a_hi, a_lo, b_hi, b_lo;
  int a_chunked, b_chunked;
};

// Fused reduce-scatter epilogue (mr_gemm_rs): row r of C belongs to rank
// r / rows_per_rank and is stored, over NVLink, into that rank's slot for this
// source rank (dst[owner] + (r % rows_per_rank) * ldd).  When every CTA has
// stored its tiles, the last one releases ``epoch`` into flag[owner] on every
// rank (system scope); the owner waits for all flags before reading its slots.
constexpr int kMaxRanks = 8;
struct RemoteOut {
  float* dst[kMaxRanks];
  unsigned long long* flag[kMaxRanks];
  unsigned int* done;  // local CTA counter, zero between launches
  unsigned long long epoch;
  long long rows_per_rank;
  long long ldd;
  int world;
  int active;
};

// Shared-memory tile of one operand part (ROWS x BK):
//   K-major:  [BK*ELT/128 K-chunks][ROWS][one K-chunk of 64 or 128 bytes]
//   MN-major: [ROWS*ELT/128 MN-chunks][BK][128 bytes of MN]
template <int BK, int ELT>
struct KRow {
  static constexpr int kBytes = BK * ELT > 128 ? 128 : BK * ELT;  // K-major row width
  static constexpr int kElems = kBytes / ELT;
};

// Load one operand part of a stage.  Chunked maps: one instruction.  3-D maps:
// K-major one box {BK, ROWS}; MN-major one box {128 / ELT, BK} per MN chunk.
template <int ROWS, int BK, int ELT>
__device__ __forceinline__ void load_part(uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                          bool kmajor, int chunked, int row0, int k0, int z) {
  constexpr int kChunkMN = 128 / ELT;
  if (kmajor) {
    if (chunked)
      tma_load_4d(dst, map, bar, 0, row0, k0 / KRow<BK, ELT>::kElems, z);
    else
      tma_load_3d(dst, map, bar, k0, row0, z);
  } else if (chunked) {
    tma_load_4d(dst, map, bar, 0, k0, row0 / kChunkMN, z);
  } else {
#pragma unroll
    for (int c = 0; c < ROWS / kChunkMN; ++c)
      tma_load_3d(dst + c * 128 * BK, map, bar, row0 + c * kChunkMN, k0, z);
  }
}

template <int ROWS, int BK, int ELT>
__device__ __forceinline__ uint64_t part_desc(uint32_t base, bool kmajor, int kstep) {
  // K-major: +32 B per MMA K step inside the swizzled row of a K-chunk, the
  // next chunk ROWS rows further; 8-row groups 8 rows apart (SBO);
  // SWIZZLE_64B or SWIZZLE_128B by row width.
  // bf16 MN-major: +2048 B (two 8-row K groups of 1024 B) per 16-deep K step;
  // LBO = one MN chunk.  float32 MN-major (SWIZZLE_128B, 32-byte atoms):
  // +1024 B (two 4-row K groups of 512 B) per 8-deep K step; LBO = one MN chunk.
  if (kmajor) {
    constexpr int rb = KRow<BK, ELT>::kBytes;
    const int off = kstep * 32;
    return smem_desc(base + (off / rb) * ROWS * rb + (off % rb), 16, 8 * rb, rb == 64 ? 4 : 2);
  }
  if (ELT == 2) return smem_desc(base + kstep * 2048, 128 * BK, 1024, 2);
  return smem_desc(base + kstep * 1024, 128 * BK, 512, 1);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One output tile of the flattened (batch, M-tile, N-tile) space and its K range.
struct Tile {
  int m0, n0, z;
  int kt_end;    // K-tiles [0, kt_end) are visited (fewer under causal mode 2)
  int n_active;  // K-tiles that issue MMAs (0: the tile is written as zeros)
  bool skip;     // causal mode 1: the tile lies wholly above the diagonal, not written
};

struct Shape {
  int m, n, k, m_tiles, n_tiles, k_tiles, causal, clen;
};

// Causal attention products (rows of a batch entry stack heads of clen
// positions; a 128-row tile lies within one head because clen % 128 == 0):
//  1: C = Q K^T or dO V^T -- tiles wholly above the diagonal are skipped;
//  2: C = P V or dS K     -- K (key positions) stops after the tile's last row;
//  3: C = dS^T Q or P^T dO -- K-tiles whose rows all precede the tile's first
//     key are skipped.
template <int BK>
__device__ __forceinline__ bool k_active(const Shape& sh, int m0, int kt) {
  return sh.causal != 3 || ((kt * BK) % sh.clen) + BK - 1 >= m0;
}

// Grouped rasterization inside each batch entry: 16 M-tiles share a sweep over N.
template <int BN, int BK, int MP = 1>
__device__ __forceinline__ Tile tile_at(const Shape& sh, int t) {
  constexpr int G = 16;
  const int per_batch = sh.m_tiles * sh.n_tiles;
  Tile tl;
  tl.z = t / per_batch;
  const int tt = t - tl.z * per_batch;
  const int group = tt / (G * sh.n_tiles);
  const int first_m = group * G;
  const int gm = min(G, sh.m_tiles - first_m);
  const int r = tt - group * G * sh.n_tiles;
  tl.m0 = (first_m + r % gm) * BM * MP;
  tl.n0 = (r / gm) * BN;
  tl.kt_end = sh.k_tiles;
  tl.skip = sh.causal == 1 && tl.n0 > (tl.m0 % sh.clen) + BM - 1;
  if (sh.causal == 2) tl.kt_end = min(sh.k_tiles, ((tl.m0 % sh.clen) + BM + BK - 1) / BK);
  if (tl.skip) tl.kt_end = 0;
  tl.n_active = tl.kt_end;
  if (sh.causal == 3) {
    tl.n_active = 0;
    for (int kt = 0; kt < tl.kt_end; ++kt) tl.n_active += k_active<BK>(sh, tl.m0, kt) ? 1 : 0;
  }
  return tl;
}

// Persistent kernel: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...
// Roles (192 threads):
//   warp 0, one lane : TMA producer over the shared-memory ring, continuing
//                      across tiles.
//   warp 1           : allocates 2 x BN TMEM columns (two accumulators); one
//                      lane issues the tile's MMAs into accumulator (j & 1)
//                      and commits to tmem_full[j & 1].
//   warps 2-5        : epilogue of tile j from accumulator (j & 1) while the
//                      MMAs of tile j + 1 run in the other; each warp reads the
//                      32 TMEM lanes (warp % 4) it may access, stores float32
//                      rows, then arrives on tmem_empty[j & 1].
template <int BN, int BK, int PREC, int MP>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ Maps maps, float* __restrict__ c, int64_t ldc,
                int64_t stride_c, const float* __restrict__ bias, int accumulate, int m, int n,
                int k, int a_kmajor, int b_kmajor, int causal, int clen, int total_tiles,
                const __grid_constant__ RemoteOut remote) {
  using C = Cfg<BN, BK, PREC, MP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStage);
  uint64_t* empty = full + C::kStages;
  uint64_t* tmem_full = empty + C::kStages;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;      // [2]
  uint64_t* done = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  Shape sh;
  sh.m = m; sh.n = n; sh.k = k;
  sh.m_tiles = (m + BM * MP - 1) / (BM * MP);
  sh.n_tiles = (n + BN - 1) / BN;
  sh.k_tiles = (k + BK - 1) / BK;
  sh.causal = causal;
  sh.clen = clen;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.a_hi)));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.b_hi)));
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ producer
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const Tile tl = tile_at<BN, BK, MP>(sh, t);
        for (int kt = 0; kt < tl.kt_end; ++kt) {
          if (!k_active<BK>(sh, tl.m0, kt)) continue;
          const int s = it % C::kStages;
          const uint32_t round = it / C::kStages;
          if (it >= C::kStages) ok = mbar_wait(&empty[s], (round - 1) & 1);
          if (!ok) break;
          ++it;
          uint8_t* st = smem + s * C::kStage;
          mbar_expect_tx(&full[s], C::kStage);
          const int k0 = kt * BK;
          load_part<BM, BK, C::kElt>(st, &maps.a_hi, &full[s], a_kmajor, maps.a_chunked, tl.m0,
                                     k0, tl.z);
          if (C::kAParts == 2)
            load_part<BM, BK, C::kElt>(st + C::kA, &maps.a_lo, &full[s], a_kmajor,
                                       maps.a_chunked, tl.m0, k0, tl.z);
          if (MP == 2)  // the tile's second 128 rows (zero-filled past m)
            load_part<BM, BK, C::kElt>(st + C::kA, &maps.a_hi, &full[s], a_kmajor,
                                       maps.a_chunked, tl.m0 + BM, k0, tl.z);
          uint8_t* sb = st + C::kA * C::kAParts * MP;
          load_part<BN, BK, C::kElt>(sb, &maps.b_hi, &full[s], b_kmajor, maps.b_chunked, tl.n0,
                                     k0, tl.z);
          if (C::kBParts == 2)
            load_part<BN, BK, C::kElt>(sb + C::kB, &maps.b_lo, &full[s], b_kmajor,
                                       maps.b_chunked, tl.n0, k0, tl.z);
        }
      }
      if (!ok) {
        // let issued copies land before the CTA exits (bounded)
        for (int s = 0; s < C::kStages; ++s) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&full[s], 0) && !mbar_try_wait(&full[s], 1) &&
                 globaltimer() - t0 < kWaitLimitNs / 4) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = instr_desc(BN, !a_kmajor, !b_kmajor, C::kTf32);
      bool ok = true;
      int it = 0, j = 0;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++j) {
        const Tile tl = tile_at<BN, BK, MP>(sh, t);
        const int b = j % C::kBufs;
        const int use = j / C::kBufs;
        if (j >= C::kBufs) ok = mbar_wait(&tmem_empty[b], (use - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(b * C::kAccCols);  // MP = 2: b = 0, halves at 0, 256
        bool first = true;
        for (int kt = 0; kt < tl.kt_end; ++kt) {
          if (!k_active<BK>(sh, tl.m0, kt)) continue;
          const int s = it % C::kStages;
          ok = mbar_wait(&full[s], (it / C::kStages) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * C::kStage);
          const uint32_t a_hi = st;
          const uint32_t a_lo = st + C::kA;
          const uint32_t b_hi = st + C::kA * C::kAParts * MP;
          const uint32_t b_lo = b_hi + C::kB;
#pragma unroll
          for (int ks = 0; ks < BK / C::kMmaK; ++ks) {
            const uint32_t acc0 = (!first || ks > 0) ? 1u : 0u;
            const uint64_t dah = part_desc<BM, BK, C::kElt>(a_hi, a_kmajor, ks);
            const uint64_t dbh = part_desc<BN, BK, C::kElt>(b_hi, b_kmajor, ks);
            if constexpr (C::kTf32) {
              umma_tf32(d, dah, dbh, idesc, acc0);
              if constexpr (MP == 2)  // the second 128 rows on the same B tile
                umma_tf32(d + uint32_t(C::kAccCols),
                          part_desc<BM, BK, C::kElt>(a_hi + C::kA, a_kmajor, ks), dbh, idesc,
                          acc0);
            } else {
              umma_bf16(d, dah, dbh, idesc, acc0);
              if (PREC == 3)
                umma_bf16(d, dah, part_desc<BN, BK, 2>(b_lo, b_kmajor, ks), idesc, 1u);
              if (PREC >= 2)
                umma_bf16(d, part_desc<BM, BK, 2>(a_lo, a_kmajor, ks), dbh, idesc, 1u);
            }
          }
          umma_commit(&empty[s]);
          ++it;
          first = false;
        }
        if (!ok) break;
        umma_commit(&tmem_full[b]);  // fires when this tile's MMAs have completed
      }
      // every MMA issued above has completed before TMEM is released
      umma_commit(done);
      mbar_wait(done, 0);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2-5)
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    float* stage = reinterpret_cast<float*>(smem + C::kStages * C::kStage + 256) + quarter * 32 * 33;
    bool ok = true;
    int j = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++j) {
      const Tile tl = tile_at<BN, BK, MP>(sh, t);
      const int b = j % C::kBufs;
      ok = mbar_wait(&tmem_full[b], (j / C::kBufs) & 1);
      tc_fence_after();
      ok = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int*>(&g_gemm_status) == 0);
      if (!ok) break;
      if (!tl.skip) {
        float* cz = c + int64_t(tl.z) * stride_c;
#pragma unroll 1
        for (int h = 0; h < MP; ++h) {  // MP = 2: rows m0 .. +127 at column 0, +128 .. at 256
          const int m0 = tl.m0 + h * BM;
          const int row = m0 + quarter * 32 + lane;
          const uint32_t lane_base =
              tmem + uint32_t((b + h) * C::kAccCols) + (uint32_t(quarter * 32) << 16);
#pragma unroll 1
          for (int col = 0; col < BN; col += 32) {
            float v[32];
            tmem_ld32(lane_base + col, v);
            if (tl.n_active == 0) {
#pragma unroll
              for (int q = 0; q < 32; ++q) v[q] = 0.f;
            }
            const int gc = tl.n0 + col;
            if (remote.active) {
              // Peer stores: lane i holds row i's 32 columns; through the staging
              // block, each store instruction writes 4 rows x 128 contiguous bytes
              // (8 lanes per row) instead of 32 scattered 16-byte pieces, so
              // NVLink carries full-line writes.
#pragma unroll
              for (int q = 0; q < 32; ++q) stage[lane * 33 + q] = v[q];
              __syncwarp();
              const int sub = lane >> 3, c4 = (lane & 7) * 4;
#pragma unroll 2
              for (int p = 0; p < 8; ++p) {
                const int r = p * 4 + sub;
                const int grow = m0 + quarter * 32 + r;
                const int gcol = gc + c4;
                if (grow < m && gcol < n) {
                  const int owner = int(grow / remote.rows_per_rank);
                  float* dst = remote.dst[owner] +
                               (grow - owner * remote.rows_per_rank) * remote.ldd + gcol;
                  const float* src = stage + r * 33 + c4;
                  if (gcol + 4 <= n) {
                    *reinterpret_cast<float4*>(dst) = make_float4(src[0], src[1], src[2], src[3]);
                  } else {
                    for (int i = 0; gcol + i < n; ++i) dst[i] = src[i];
                  }
                }
              }
              __syncwarp();
              continue;
            }
            if (row < m && gc < n) {
              float* dst = cz + int64_t(row) * ldc + gc;
              const bool full_chunk =
                  gc + 32 <= n && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
              if (full_chunk) {
#pragma unroll
                for (int q = 0; q < 32; q += 4) {
                  float4 o = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
                  if (bias) {
                    o.x += bias[gc + q]; o.y += bias[gc + q + 1];
                    o.z += bias[gc + q + 2]; o.w += bias[gc + q + 3];
                  }
                  if (accumulate) {
                    const float4 p = *reinterpret_cast<const float4*>(dst + q);
                    o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
                  }
                  *reinterpret_cast<float4*>(dst + q) = o;
                }
              } else {
                for (int q = 0; q < 32 && gc + q < n; ++q) {
                  float o = v[q];
                  if (bias) o += bias[gc + q];
                  if (accumulate) o += dst[q];
                  dst[q] = o;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[b]);
    }
    if (remote.active) {
      // every epilogue thread's peer stores are ordered before the CTA's
      // arrival; the last CTA publishes the epoch to every owner
      __threadfence_system();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (warp == 2 && lane == 0) {
        const unsigned int prev = atomicAdd(remote.done, 1u);
        if (prev == gridDim.x - 1) {
          __threadfence_system();
          for (int r = 0; r < remote.world; ++r)
            asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(remote.flag[r]),
                         "l"(remote.epoch)
                         : "memory");
          atomicExch(remote.done, 0u);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
// cuTensorMapEncodeTiled, resolved through the runtime so that the library
// does not link libcuda (it must load on hosts without a driver).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D tiled map (inner, outer, batch) of bf16 (elt 2) or float32 (elt 4) values.
bool make_map(CUtensorMap* map, const void* base, int elt, int64_t inner, int64_t outer,
              int64_t ld, int64_t batch, int64_t batch_stride, uint32_t box_inner,
              uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn encode = encode_fn();
  if (!encode) return false;
  const cuuint64_t dims[3] = {cuuint64_t(inner), cuuint64_t(outer), cuuint64_t(batch)};
  const cuuint64_t strides[2] = {cuuint64_t(ld) * elt,
                                 cuuint64_t(batch > 1 ? batch_stride : ld * outer) * elt};
  const cuuint32_t box[3] = {box_inner, box_outer, 1};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  CUresult r = encode(map, elt == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                      3, const_cast<void*>(base), dims, strides, box, elem_strides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D chunked map: x = a 128-byte chunk of the contiguous dimension, then the
// other matrix dimension (stride ld), then the chunk index (stride 128 bytes),
// then the batch.  One box {chunk, y_box, chunks, 1} lands in shared memory as
// [chunks][y_box][128 bytes] -- the tile layout the UMMA descriptors describe.
bool make_chunked_map(CUtensorMap* map, const void* base, int elt, int64_t contiguous,
                      int64_t other, int64_t ld, int64_t batch, int64_t batch_stride,
                      uint32_t box_other, uint32_t box_chunks, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn encode = encode_fn();
  if (!encode) return false;
  const int64_t chunk = 128 / elt;
  const cuuint64_t dims[4] = {cuuint64_t(chunk), cuuint64_t(other), cuuint64_t(contiguous / chunk),
                              cuuint64_t(batch)};
  const cuuint64_t strides[3] = {cuuint64_t(ld) * elt, 128,
                                 cuuint64_t(batch > 1 ? batch_stride : ld * other) * elt};
  const cuuint32_t box[4] = {uint32_t(chunk), box_other, box_chunks, 1};
  const cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  CUresult r = encode(map, elt == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                      4, const_cast<void*>(base), dims, strides, box, elem_strides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Map for an operand with `rows` logical rows (M or N) and K columns, and
// whether it is chunked (one TMA instruction per stage).  K-major rows of up
// to 128 bytes: one box {bk, tile_rows} swizzled at its row width; wider rows
// (float32 at bk = 64): chunked, two 128-byte K-chunks (K a multiple of 32).
// MN-major: chunked when the rows divide into 128-byte chunks, else one box
// {128 bytes, bk} per chunk; 128-byte swizzle for bf16, the 32-byte-atom form
// of it for float32 (the layout kind::tf32 reads MN-major).
bool operand_map(CUtensorMap* map, int* chunked, const void* p, int elt, bool kmajor,
                 int64_t rows, int64_t k, int64_t ld, int64_t batch, int64_t batch_stride,
                 int tile_rows, int bk) {
  const int chunk = 128 / elt;
  if (kmajor) {
    if (bk * elt <= 128) {
      *chunked = 0;
      return make_map(map, p, elt, k, rows, ld, batch, batch_stride, uint32_t(bk),
                      uint32_t(tile_rows),
                      bk * elt == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (k % chunk) return false;
    *chunked = 1;
    return make_chunked_map(map, p, elt, k, rows, ld, batch, batch_stride, uint32_t(tile_rows),
                            uint32_t(bk / chunk), CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const CUtensorMapSwizzle swz =
      elt == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  if (rows % chunk) {
    *chunked = 0;
    return make_map(map, p, elt, rows, k, ld, batch, batch_stride, uint32_t(chunk), uint32_t(bk),
                    swz);
  }
  *chunked = 1;
  return make_chunked_map(map, p, elt, rows, k, ld, batch, batch_stride, uint32_t(bk),
                          uint32_t(tile_rows / chunk), swz);
}

// Per-device caches (a process may drive several GPUs from one or more host
// threads): the SM count and, per kernel instantiation, whether its dynamic
// shared-memory limit has been raised on that device.  Racing first calls
// only repeat an idempotent query or attribute call.
constexpr int kMaxDevices = 64;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

int sm_count() {
  static std::atomic<int> counts[kMaxDevices];
  const int dev = current_device();
  if (dev < 0) return kSMs;
  int count = counts[dev].load(std::memory_order_relaxed);
  if (!count) {
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        count <= 0)
      count = kSMs;
    counts[dev].store(count, std::memory_order_relaxed);
  }
  return count;
}

template <int BN, int BK, int PREC, int MP = 1>
int launch(const Maps& maps, float* c, int64_t ldc, int64_t stride_c, const float* bias,
           int accumulate, int m, int n, int k, int a_kmajor, int b_kmajor, int batch,
           int causal, int clen, const RemoteOut& remote, cudaStream_t stream) {
  using C = Cfg<BN, BK, PREC, MP>;
  static std::atomic<bool> configured[kMaxDevices];
  const int dev = current_device();
  if (dev < 0) return MR_ERR_DEVICE;
  if (!configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN, BK, PREC, MP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return MR_ERR_LAUNCH;
    }
    configured[dev].store(true, std::memory_order_release);
  }
  const int64_t tiles = int64_t((m + BM * MP - 1) / (BM * MP)) * ((n + BN - 1) / BN) * batch;
  if (tiles > (1ll << 31) - 1) return MR_ERR_ARGUMENT;
  const int grid = int(tiles < sm_count() ? tiles : sm_count());
  gemm_kernel<BN, BK, PREC, MP><<<grid, kThreads, C::kSmem, stream>>>(
      maps, c, ldc, stride_c, bias, accumulate, m, n, k, a_kmajor, b_kmajor, causal, clen,
      int(tiles), remote);
  return launch_status();
}

}  // namespace
}  // namespace mr

using namespace mr;

namespace {

// Output tile shape.  128 x 128 for narrow outputs (attention's head
// dimension); 128 x 256 for the bf16 products; for the tf32 products (no
// batch, no causal mode) the shape of 128 or 256 rows (MP = 1 or 2) by 224 or
// 256 columns whose persistent schedule is shortest.  CTA i takes tiles i,
// i + grid, ..., so a launch lasts ceil(tiles / SMs) tile-times; a tile's time
// is modelled as the larger of its staged operand bytes at one SM's share of
// L2 bandwidth and its flops at one SM's tf32 rate (ratio ~55 flop/byte):
// the 128 x 256 tile stages 384 rows of K per 2 x 128 x 256 flops (43.7
// flop/byte) and is bandwidth-bound; the 256 x 256 tile, 512 rows for twice
// the flops (65.5), is not.  224 needs every B chunk whole (MN-major tf32: 7
// chunks of 32; K-major: any).  Measured 224 against 256 at MP = 1 (same box,
// CUDA events): tf32 dW through qkv 0.95x the time, dX through o at 2048
// tokens 0.97x, the long-K shapes unchanged; the bf16 split's forward at 224
// ran up to 6 % slower, so it keeps 256.
struct TileChoice {
  int bn;
  int mp;
};

TileChoice select_tile(int64_t m, int64_t n, int64_t k, int64_t batch, int precision,
                       int causal) {
  if (n <= 128) return {128, 1};
  if (!(batch == 1 && causal == 0 && precision == 4)) return {256, 1};
  const double sms = double(sm_count());
  constexpr double kFlopPerByte = 55.0;
  // a 256-row tile's epilogue does not overlap MMAs: measured as ~640 K
  // elements of its main loop (dW through o at 2048 tokens, K = 2048, ran
  // 1.14x slower with 256-row tiles; at K >= 3584 they won)
  constexpr double kEpilogueK = 640.0;
  TileChoice best{256, 1};
  double best_cost = -1.0;
  for (int mp = 1; mp <= 2; ++mp) {
    for (int bn : {256, 224}) {
      const double rows = double(BM) * mp;
      const double tiles = std::ceil(double(m) / rows) * std::ceil(double(n) / bn);
      const double waves = std::ceil(tiles / sms);
      const double staged = (rows + bn) * 4.0 * kFlopPerByte;
      const double flops = rows * bn * 2.0;
      const double per_k = staged > flops ? staged : flops;
      const double cost = waves * (double(k) + (mp == 2 ? kEpilogueK : 0.0)) * per_k;
      // a later shape must be at least 3 % cheaper
      if (best_cost < 0.0 || cost <= 0.97 * best_cost) {
        best = {bn, mp};
        best_cost = cost;
      }
    }
  }
  return best;
}

int select_bk(int64_t k, int tf32, int a_kmajor, int b_kmajor) {
  const bool k_chunks = k % 32 == 0 || (!a_kmajor && !b_kmajor);
  return tf32 ? (k_chunks ? kTf32BK : 32) : (!a_kmajor && !b_kmajor) ? 64 : 32;
}

// precision 1..3: bf16 operands (hi, optional lo); 4: one tf32 product of
// float32 operands (a_hi / b_hi point at float32 data; the lo parts are unused).
int gemm_impl(const void* a_hi, const void* a_lo, int64_t lda, int64_t stride_a,
              int a_kmajor, const void* b_hi, const void* b_lo, int64_t ldb,
              int64_t stride_b, int b_kmajor, float* c, int64_t ldc, int64_t stride_c,
              const float* bias, int accumulate, int64_t m, int64_t n, int64_t k, int64_t batch,
              int precision, int causal, int64_t seq, const RemoteOut& remote, void* stream) {
  if (!a_hi || !b_hi || !c || m <= 0 || n <= 0 || k <= 0 || batch <= 0) return MR_ERR_ARGUMENT;
  if (m > (1ll << 31) - 1 || n > (1ll << 31) - 1 || k > (1ll << 31) - 1 || batch > 65535)
    return MR_ERR_ARGUMENT;
  if (precision < 1 || precision > 4) return MR_ERR_ARGUMENT;
  const bool tf32 = precision == 4;
  const int elt = tf32 ? 4 : 2;
  if (tf32) a_lo = b_lo = nullptr;
  if ((precision == 2 || precision == 3) && !a_lo) return MR_ERR_ARGUMENT;
  if (precision == 3 && !b_lo) return MR_ERR_ARGUMENT;
  if (!aligned16(a_hi) || !aligned16(b_hi) || (a_lo && !aligned16(a_lo)) ||
      (b_lo && !aligned16(b_lo)))
    return MR_ERR_ALIGNMENT;
  // TMA: global strides are multiples of 16 bytes
  const int per16 = 16 / elt;
  if ((lda % per16) || (ldb % per16)) return MR_ERR_ALIGNMENT;
  if (batch > 1 && ((stride_a % per16) || (stride_b % per16))) return MR_ERR_ALIGNMENT;
  if (a_kmajor ? lda < k : lda < m) return MR_ERR_ARGUMENT;
  if (b_kmajor ? ldb < k : ldb < n) return MR_ERR_ARGUMENT;
  if (ldc < n) return MR_ERR_ARGUMENT;
  if (causal < 0 || causal > 3) return MR_ERR_ARGUMENT;
  if (causal) {
    if (seq <= 0 || seq % BM || m % seq) return MR_ERR_ARGUMENT;
    if (causal == 1 && n != seq) return MR_ERR_ARGUMENT;
    if (causal == 2 && k != seq) return MR_ERR_ARGUMENT;
    if (causal == 3 && (m != seq || k % seq)) return MR_ERR_ARGUMENT;
  }
  // narrow outputs (attention's head dimension) use 128-wide tiles; 32-wide K
  // slices (deeper pipelines) unless both operands are MN-major, whose 64-wide
  // boxes would then be split into many small TMA copies
  // float32 (tf32) operands: kTf32BK-wide K slices (a 64-wide slice takes
  // K-major rows as two 128-byte chunks, so it needs K a multiple of 32),
  // else 32-wide.
  const int BKsel = select_bk(k, tf32, a_kmajor, b_kmajor);
  const TileChoice tile = select_tile(m, n, k, batch, precision, causal);
  const int BNsel = tile.bn;
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  int a_lo_chunked = 0, b_lo_chunked = 0;
  bool good = operand_map(&maps.a_hi, &maps.a_chunked, a_hi, elt, a_kmajor, m, k, lda, batch,
                          stride_a, BM, BKsel) &&
              operand_map(&maps.b_hi, &maps.b_chunked, b_hi, elt, b_kmajor, n, k, ldb, batch,
                          stride_b, BNsel, BKsel);
  if (good && (precision == 2 || precision == 3))
    good = operand_map(&maps.a_lo, &a_lo_chunked, a_lo, elt, a_kmajor, m, k, lda, batch, stride_a,
                       BM, BKsel);
  if (good && precision == 3)
    good = operand_map(&maps.b_lo, &b_lo_chunked, b_lo, elt, b_kmajor, n, k, ldb, batch, stride_b,
                       BNsel, BKsel);
  if (!good) return MR_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int bt = int(batch);
  const int M = int(m), N = int(n), Kk = int(k);
#define MR_GEMM_LAUNCH(BN_, BK_)                                                               \
  switch (precision) {                                                                         \
    case 1: return launch<BN_, BK_, 1>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk,     \
                                       a_kmajor, b_kmajor, bt, causal, int(seq), remote, s);   \
    case 2: return launch<BN_, BK_, 2>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk,     \
                                       a_kmajor, b_kmajor, bt, causal, int(seq), remote, s);   \
    default: return launch<BN_, BK_, 3>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk,    \
                                        a_kmajor, b_kmajor, bt, causal, int(seq), remote, s);  \
  }
  if (tf32) {
    static_assert(kTf32BK == 32, "one tf32 instantiation per tile shape serves both K slices");
    if (tile.mp == 2) {
      if (BNsel == 224)
        return launch<224, 32, 4, 2>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk,
                                     a_kmajor, b_kmajor, bt, causal, int(seq), remote, s);
      return launch<256, 32, 4, 2>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk, a_kmajor,
                                   b_kmajor, bt, causal, int(seq), remote, s);
    }
    if (BNsel == 224)
      return launch<224, 32, 4>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk, a_kmajor,
                                b_kmajor, bt, causal, int(seq), remote, s);
    if (BKsel == kTf32BK) {
      if (BNsel == 128)
        return launch<128, kTf32BK, 4>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk,
                                       a_kmajor, b_kmajor, bt, causal, int(seq), remote, s);
      return launch<256, kTf32BK, 4>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk,
                                     a_kmajor, b_kmajor, bt, causal, int(seq), remote, s);
    }
    if (BNsel == 128)
      return launch<128, 32, 4>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk, a_kmajor,
                                b_kmajor, bt, causal, int(seq), remote, s);
    return launch<256, 32, 4>(maps, c, ldc, stride_c, bias, accumulate, M, N, Kk, a_kmajor,
                              b_kmajor, bt, causal, int(seq), remote, s);
  }
  if (BNsel == 128) {
    if (BKsel == 64) { MR_GEMM_LAUNCH(128, 64) }
    MR_GEMM_LAUNCH(128, 32)
  }
  if (BKsel == 64) { MR_GEMM_LAUNCH(256, 64) }
  MR_GEMM_LAUNCH(256, 32)
#undef MR_GEMM_LAUNCH
}

}  // namespace

extern "C" int mr_gemm_batched(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda,
                               int64_t stride_a, int a_kmajor, const uint16_t* b_hi,
                               const uint16_t* b_lo, int64_t ldb, int64_t stride_b, int b_kmajor,
                               float* c, int64_t ldc, int64_t stride_c, const float* bias,
                               int accumulate, int64_t m, int64_t n, int64_t k, int64_t batch,
                               int precision, int causal, int64_t seq, void* stream) {
  if (precision < 1 || precision > 3) return MR_ERR_ARGUMENT;  // tf32: mr_gemm_tf32
  RemoteOut none;
  memset(&none, 0, sizeof(none));
  return gemm_impl(a_hi, a_lo, lda, stride_a, a_kmajor, b_hi, b_lo, ldb, stride_b, b_kmajor, c,
                   ldc, stride_c, bias, accumulate, m, n, k, batch, precision, causal, seq, none,
                   stream);
}

namespace {

int gemm_rs_impl(const void* a_hi, const void* a_lo, int64_t lda, int a_kmajor, const void* b_hi,
                 const void* b_lo, int64_t ldb, int b_kmajor, int64_t m, int64_t n, int64_t k,
                 int precision, float* const* dst, int64_t ldd, int64_t rows_per_rank,
                 unsigned long long* const* flags, int world, unsigned int* done,
                 unsigned long long epoch, void* stream) {
  if (!dst || !flags || !done || world < 1 || world > kMaxRanks || rows_per_rank <= 0 ||
      m != rows_per_rank * world || ldd < n || epoch == 0)
    return MR_ERR_ARGUMENT;
  RemoteOut remote;
  memset(&remote, 0, sizeof(remote));
  for (int r = 0; r < world; ++r) {
    if (!dst[r] || !flags[r]) return MR_ERR_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(dst[r]) & 15u) return MR_ERR_ALIGNMENT;
    remote.dst[r] = dst[r];
    remote.flag[r] = flags[r];
  }
  if ((ldd % 4) != 0) return MR_ERR_ALIGNMENT;
  remote.done = done;
  remote.epoch = epoch;
  remote.rows_per_rank = rows_per_rank;
  remote.ldd = ldd;
  remote.world = world;
  remote.active = 1;
  // c is unused (every row goes to its owner); dst[0] stands in for the checks
  return gemm_impl(a_hi, a_lo, lda, 0, a_kmajor, b_hi, b_lo, ldb, 0, b_kmajor, dst[0], n, 0,
                   nullptr, 0, m, n, k, 1, precision, 0, 0, remote, stream);
}

}  // namespace

extern "C" int mr_gemm_rs(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda, int a_kmajor,
                          const uint16_t* b_hi, const uint16_t* b_lo, int64_t ldb, int b_kmajor,
                          int64_t m, int64_t n, int64_t k, int precision, float* const* dst,
                          int64_t ldd, int64_t rows_per_rank, unsigned long long* const* flags,
                          int world, unsigned int* done, unsigned long long epoch, void* stream) {
  if (precision < 1 || precision > 3) return MR_ERR_ARGUMENT;  // tf32: mr_gemm_rs_tf32
  return gemm_rs_impl(a_hi, a_lo, lda, a_kmajor, b_hi, b_lo, ldb, b_kmajor, m, n, k, precision,
                      dst, ldd, rows_per_rank, flags, world, done, epoch, stream);
}

extern "C" int mr_gemm(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda, int a_kmajor,
                       const uint16_t* b_hi, const uint16_t* b_lo, int64_t ldb, int b_kmajor,
                       float* c, int64_t ldc, const float* bias, int accumulate, int64_t m,
                       int64_t n, int64_t k, int precision, void* stream) {
  return mr_gemm_batched(a_hi, a_lo, lda, 0, a_kmajor, b_hi, b_lo, ldb, 0, b_kmajor, c, ldc, 0,
                         bias, accumulate, m, n, k, 1, precision, 0, 0, stream);
}

extern "C" int mr_gemm_tf32(const float* a, int64_t lda, int a_kmajor, const float* b,
                            int64_t ldb, int b_kmajor, float* c, int64_t ldc, const float* bias,
                            int accumulate, int64_t m, int64_t n, int64_t k, void* stream) {
  RemoteOut none;
  memset(&none, 0, sizeof(none));
  return gemm_impl(a, nullptr, lda, 0, a_kmajor, b, nullptr, ldb, 0, b_kmajor, c, ldc, 0, bias,
                   accumulate, m, n, k, 1, 4, 0, 0, none, stream);
}

extern "C" int mr_gemm_rs_tf32(const float* a, int64_t lda, int a_kmajor, const float* b,
                               int64_t ldb, int b_kmajor, int64_t m, int64_t n, int64_t k,
                               float* const* dst, int64_t ldd, int64_t rows_per_rank,
                               unsigned long long* const* flags, int world, unsigned int* done,
                               unsigned long long epoch, void* stream) {
  return gemm_rs_impl(a, nullptr, lda, a_kmajor, b, nullptr, ldb, b_kmajor, m, n, k, 4, dst, ldd,
                      rows_per_rank, flags, world, done, epoch, stream);
}

// The output tile width (128, 224 or 256) and height (128 or 256) a launch
// of this shape uses.
extern "C" int mr_gemm_tile_n(int64_t m, int64_t n, int64_t k, int64_t batch, int precision,
                              int a_kmajor, int b_kmajor, int causal) {
  if (m <= 0 || n <= 0 || k <= 0 || batch <= 0 || precision < 1 || precision > 4)
    return MR_ERR_ARGUMENT;
  (void)a_kmajor;
  (void)b_kmajor;
  return select_tile(m, n, k, batch, precision, causal).bn;
}

extern "C" int mr_gemm_tile_m(int64_t m, int64_t n, int64_t k, int64_t batch, int precision,
                              int a_kmajor, int b_kmajor, int causal) {
  if (m <= 0 || n <= 0 || k <= 0 || batch <= 0 || precision < 1 || precision > 4)
    return MR_ERR_ARGUMENT;
  (void)a_kmajor;
  (void)b_kmajor;
  return BM * select_tile(m, n, k, batch, precision, causal).mp;
}

// Device status word of the GEMM (0 ok, MR_ERR_TIMEOUT after a wait gave up).
// Synchronizes the device; `reset` clears the word.
extern "C" int mr_gemm_status(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int));
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return MR_ERR_LAUNCH;
  }
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
  }
  return v;
}
