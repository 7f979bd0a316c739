// strassen_gemm.cu -- tile-local one-level Strassen GEMM for B200 (sm_100a).
//
// Algorithm (reference: strassen_pallas.py:156-880).  The reference splits
// every (bm, bk) A tile and (bk, bn) B tile into 2x2 quadrants, forms ten
// bf16 operand sums, runs seven half-size products P1..P7 and accumulates four
// fp32 quadrant accumulators over the K panels.  Because the quadrant
// recombination is linear, the same result (up to fp32 summation order) is
// obtained by accumulating each product over the whole K range first and
// recombining once at the end.  Seen that way, each product Pi is an ordinary
// GEMM of size (M/2) x (N/2) x (K/2) over "product coordinates": product row t
// is row r' of block I = t / (bm/2), product column u is column c' of block
// J = u / (bn/2), and product depth kappa is column k' of panel
// P = kappa / (bk/2).  The reference's quadrant q of block (I, J) is the
// matrix element (I*bm + qr*bm/2 + r', J*bn + qc*bn/2 + c').
//
// This file holds two layouts of that computation and the C ABI over both.
//
// The planes path (strassen_planes.cuh; the default for large products):
// operand passes write the seven A and seven B operands of every block as
// planes in a caller workspace, one persistent kernel runs the seven product
// GEMMs on CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles) into fp32
// products, and a recombination pass applies the fused epilogue; two halves
// of the product rows run on two streams.  sb_workspace_bytes asks for its
// workspace where a cost model predicts it wins.
//
// The one-CTA fused kernel below (small products, the research options,
// narrow tiles, the no-allocation entry point), one CTA per SM and one output
// tile per CTA:
//   * CTA tile: 128 product rows x 64 product columns, i.e. a 256 x 128 patch
//     of C made of four 128 x 64 quadrant pieces.
//   * TMEM: seven fp32 accumulators M1..M7 of 128 lanes x 64 columns
//     (448 of the 512 columns) plus a two-step ring of A sums (448..511).
//   * Warp 0: TMA producer.  Per 16-deep K step ONE copy lands the four raw A
//     quadrant tiles (128 x 16, 32-byte swizzle) and ONE copy the four raw B
//     quadrant tiles (16 x 64, 128-byte swizzle), through tensor maps whose
//     extra dimensions are the quadrant offsets.
//   * Warps 4..11: two sets of four operand-sum warps on alternate K steps.
//     They form the A and B sums with bf16x2 adds (round-to-nearest-even,
//     exactly the reference's bf16 pre-add rounding): a0+a1 and the five B
//     sums in place in shared memory, the other four A sums into the TMEM
//     ring for A-from-TMEM MMAs.
//   * Warp 1: TMEM allocator and single-thread tcgen05.mma issuer: per step
//     one wait, seven 128x64x16 MMAs and one commit that frees the stage.
//   * Warps 4..11 again, after the K loop: epilogue.  Each thread owns one
//     TMEM lane (= one product row), reads M1..M7 with tcgen05.ld, recombines
//     C11 = M1+M4-M5+M7, C12 = M3+M5, C21 = M2+M4, C22 = M1-M2+M3+M6 in fp32,
//     applies the fused epilogue and stores bf16 (or fp32).
//
// The opt-in two-CTA (strassen_pair.cuh) and four-CTA (strassen_quad.cuh)
// kernels split the seven products over the CTAs of a cluster.
//
// The same skeleton also runs the matched-tile classical control (eight
// sub-block products into four accumulators, no operand sums), which mirrors
// the reference's blocked cubic Pallas control
// (experiments/qwen3/benchmark_cubic_control.py:57-237).

#include "sm100_primitives.cuh"
#include "strassen_b200.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

namespace sb {

// ------------------------------------------------------------------ shape
constexpr int kBlockM = 128;  // product rows per CTA = TMEM lanes
constexpr int kBlockN = 64;   // product columns per CTA = TMEM columns per product
#ifndef SB_BLOCK_K
#define SB_BLOCK_K 16
#endif
#ifndef SB_STAGES
#define SB_STAGES 5
#endif
#ifndef SB_TS_STAGES
#define SB_TS_STAGES 6
#endif
#ifndef SB_TMEM_A
#define SB_TMEM_A 1
#endif
#ifndef SB_C_BLOCK_K
#define SB_C_BLOCK_K 64
#endif
#ifndef SB_C_STAGES
#define SB_C_STAGES 2
#endif
constexpr int kFirstSumWarp = 4;
constexpr int kSumWarps = 8;
constexpr int kSumThreads = kSumWarps * 32;
constexpr int kThreads = (kFirstSumWarp + kSumWarps) * 32;  // 384
constexpr uint32_t kTmemCols = 512;
#ifndef SB_BARRIER_BYTES
#define SB_BARRIER_BYTES 256
#endif
constexpr int kBarrierBytes = SB_BARRIER_BYTES;
constexpr int kRasterGroup = 16;  // product-row tiles per column sweep (L2 reuse)
static_assert(7 * kBlockN <= (int)kTmemCols, "seven accumulators must fit in TMEM");

// Pipeline geometry.  A stage holds `kASlots` A tiles (128 x BK, K-major) and
// `kBSlots` B tiles (BK x 64, N-major): the four raw quadrants first, then
// (Strassen only) the operand sums formed in shared memory.
template <int kBK, int kNumStages, int kASlots, int kBSlots>
struct PipeCfg {
  static constexpr int BK = kBK;
  static constexpr int STAGES = kNumStages;
  static constexpr int A_SLOT = kBlockM * kBK * 2;
  static constexpr int B_SLOT = kBK * kBlockN * 2;
  static constexpr int B_OFFSET = kASlots * A_SLOT;  // B tiles follow the A tiles
  static constexpr int STAGE_BYTES = kASlots * A_SLOT + kBSlots * B_SLOT;
  static constexpr int A_STAGES = 0;  // A shares the stage with B
  static constexpr int A_STAGE_BYTES = 0;
  static constexpr int B_BASE = 0;
  static constexpr int DATA_BYTES = kNumStages * STAGE_BYTES;
  static constexpr int RAW_TX = 4 * (A_SLOT + B_SLOT);
  static constexpr int SMEM = STAGES * STAGE_BYTES + kBarrierBytes + 1024;  // + alignment slack
  // A: K-major, one BK-wide row per swizzle row (32/64/128 bytes); 8-row core
  // groups 8*row bytes apart; LBO unused for swizzled K-major.
  static constexpr uint32_t A_ROW = kBK * 2;
  static constexpr uint32_t A_LAYOUT = A_ROW == 32 ? kLayoutSwizzle32B
                                       : A_ROW == 64 ? kLayoutSwizzle64B : kLayoutSwizzle128B;
  static constexpr uint32_t A_SBO = 8 * A_ROW;
  static constexpr uint32_t A_LBO = 16;
  // B: N-major 128-byte rows (64 columns), 128B swizzle, 8 k-rows per 1024 B; the
  // LBO (next 64-column chunk) is never used because the N tile is 64.
  static constexpr uint32_t B_LAYOUT = kLayoutSwizzle128B;
  static constexpr uint32_t B_SBO = 1024;
  static constexpr uint32_t B_LBO = kBK * 128;
  static_assert(kBK == 16 || kBK == 32 || kBK == 64, "K chunk must be one swizzle row");
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(kNumStages <= 8, "barrier area holds at most 8 stages");
};
using StrassenPipe = PipeCfg<SB_BLOCK_K, SB_STAGES, 7, 7>;
using ClassicalPipe = PipeCfg<SB_C_BLOCK_K, SB_C_STAGES, 4, 4>;

// Geometry of the default Strassen kernel (see uses_tmem_a).  A stage holds one
// 16-deep K step: the four raw A quadrant tiles (128 x 16, K-major, 32-byte
// swizzle; a1's slot is overwritten with a0+a1) and the four raw B quadrant
// tiles plus the five B sums (16 x 64, N-major, 128-byte swizzle).  The other
// four A sums live in TMEM, so a stage is 30 KB and the ring is seven deep.
// Each operand arrives in one TMA copy per step (make_ts_maps) instead of one
// copy per quadrant.
template <int kNumStages>
struct TsPipeCfg {
  static constexpr int BK = 16;
  static constexpr int STAGES = kNumStages;
  static constexpr int A_STAGES = 0;
  static constexpr int A_STAGE_BYTES = 0;
  static constexpr int B_BASE = 0;
  static constexpr int A_SLOT = kBlockM * 16 * 2;
  static constexpr int B_SLOT = 16 * kBlockN * 2;
  static constexpr int B_OFFSET = 4 * A_SLOT;
  static constexpr int STAGE_BYTES = 4 * A_SLOT + 7 * B_SLOT;
  static constexpr int RAW_TX = 4 * (A_SLOT + B_SLOT);
  static constexpr int DATA_BYTES = kNumStages * STAGE_BYTES;
  static constexpr int SMEM = DATA_BYTES + kBarrierBytes + 1024;
  static constexpr uint32_t A_ROW = 32;
  static constexpr uint32_t A_LAYOUT = kLayoutSwizzle32B;
  static constexpr uint32_t A_SBO = 8 * A_ROW;
  static constexpr uint32_t A_LBO = 16;
  static constexpr uint32_t B_LAYOUT = kLayoutSwizzle128B;
  static constexpr uint32_t B_SBO = 1024;
  static constexpr uint32_t B_LBO = 16 * 128;
  static_assert(STAGE_BYTES % 1024 == 0 && B_OFFSET % 1024 == 0, "1024-byte stage alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert((3 * kNumStages + 2) * 8 + 8 <= kBarrierBytes, "barrier area");
};
using StrassenTsPipe = TsPipeCfg<SB_TS_STAGES>;

// Strassen launches with A stored row-major (the default and the research
// options) keep four of the five A operand sums in TMEM: a ring of kRingSlots
// slots of 128 lanes x 8 columns (one 128 x 16 bf16 operand) after the seven
// accumulators, two K steps deep, and issue those four products as
// A-from-TMEM MMAs, which takes their A operand off shared memory.  The
// transposed-A launch (strassen_matmul_lhs_transposed) keeps the earlier layout
// with all ten sums in shared memory.
// kOpts: 0 = the default instantiation; 1, 2, 3 = research options with the
// classical, dual and power-of-two formula, compiled separately so the
// formula's operand tables fold to constants.
template <int kOpts>
__host__ __device__ constexpr int kFormula() { return kOpts > 0 ? kOpts - 1 : 0; }

template <bool kStrassen, int kOpts, bool kATrans>
constexpr bool uses_tmem_a() { return SB_TMEM_A && kStrassen && !kATrans; }
constexpr int kRingSlots = 8;
constexpr uint32_t kRingCol0 = 7 * kBlockN;  // 448
static_assert(kRingCol0 + 8 * kRingSlots <= kTmemCols, "operand ring must fit in TMEM");

template <bool kStrassen, bool kTs = false>
using PipeFor = typename std::conditional<
    kStrassen, typename std::conditional<kTs, StrassenTsPipe, StrassenPipe>::type,
    ClassicalPipe>::type;

constexpr uint32_t kIdesc = umma_idesc_bf16_f32(kBlockM, kBlockN, false, true);
constexpr uint32_t kIdescNegA = kIdesc | (1u << 13);  // D (+)= -A * B
constexpr uint32_t kIdescAT = umma_idesc_bf16_f32(kBlockM, kBlockN, true, true);  // A MN-major

// Operand slots inside a stage.  Raw tiles land in slots 0..3
// (a0=A[top,left] a1=A[top,right] a2=A[bottom,left] a3=A[bottom,right];
//  b0=B[top,left] b1=B[top,right] b2=B[bottom,left] b3=B[bottom,right]).
// The sum warps then overwrite a1/a2/b1/b2 (not needed raw) and fill 4..6:
//   A: s1 <- a0+a1 (P5)  s2 <- a2-a0 (P6)  s4 <- a0+a3 (P1)  s5 <- a2+a3 (P2)  s6 <- a1-a3 (P7)
//   B: s1 <- b1-b3 (P3)  s2 <- b2-b0 (P4)  s4 <- b0+b3 (P1)  s5 <- b0+b1 (P6)  s6 <- b2+b3 (P7)
// Product Pi (strassen_pallas.py:324-379) reads A slot kASlot[i-1], B slot kBSlot[i-1]:
//   P1=(a0+a3)(b0+b3)  P2=(a2+a3)b0  P3=a0(b1-b3)  P4=a3(b2-b0)
//   P5=(a0+a1)b3       P6=(a2-a0)(b0+b1)           P7=(a1-a3)(b2+b3)
__constant__ int kASlot[7] = {4, 5, 0, 3, 1, 2, 6};
__constant__ int kBSlot[7] = {4, 0, 1, 2, 3, 5, 6};
// Exact classical panel (strassen_pallas.py:575-586) expressed in the seven
// accumulators, so the unchanged recombination yields C0 += a0b0+a1b2,
// C1 += a0b1+a1b3, C2 += a2b0+a3b2, C3 += a2b1+a3b3:
//   classical: acc6 += E0, acc2 += E1, acc1 += E2, acc5 += E3 - E1 + E2
//   dual:      acc6 += E0, acc1 += E1, acc2 += E2, acc5 += E3 + E1 - E2
// Entries: accumulator, A raw slot, B raw slot, negate (for the two formulas).
__device__ constexpr int kExactAcc[2][12] = {{6, 6, 2, 2, 1, 1, 5, 5, 5, 5, 5, 5}, {6, 6, 1, 1, 2, 2, 5, 5, 5, 5, 5, 5}};
__device__ constexpr int kExactA[12] = {0, 1, 0, 1, 2, 3, 2, 3, 0, 1, 2, 3};
__device__ constexpr int kExactB[12] = {0, 2, 1, 3, 0, 2, 1, 3, 1, 3, 0, 2};
__device__ constexpr int kExactNeg[2][12] = {{0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 0, 0}, {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1}};
// TMEM-ring layout, per formula (classical, dual, powers) and product: the ring
// slot of its A operand (-1: shared memory), its shared-memory A slot, its B
// slot.  Slots 0-3 of the classical/dual rows are quadrant positions, which the
// block permutation remaps; powers operands sit in fixed slots.
__device__ constexpr int kProdRing[3][7] = {{0, 1, -1, -1, -1, 2, 3}, {0, -1, 1, -1, -1, 2, 3}, {0, 1, -1, -1, -1, 2, 3}};
__device__ constexpr int kProdA[3][7] = {{0, 0, 0, 3, 1, 0, 0}, {0, 0, 0, 1, 3, 0, 0}, {0, 0, 0, 1, 2, 0, 0}};
__device__ constexpr int kProdB[3][7] = {{4, 0, 1, 2, 3, 5, 6}, {4, 1, 0, 3, 2, 5, 6}, {0, 1, 2, 3, 4, 5, 6}};
// Classical control: C0+=a0b0, C0+=a1b2, C1+=a0b1, C1+=a1b3, C2+=a2b0, C2+=a3b2,
// C3+=a2b1, C3+=a3b3 (strassen_pallas.py:575-586 order).
__constant__ int kCAslot[8] = {0, 1, 0, 1, 2, 3, 2, 3};
__constant__ int kCBslot[8] = {0, 2, 1, 3, 0, 2, 1, 3};

struct GemmParams {
  int32_t M, N, K;
  int32_t bm, bn, bk;
  int32_t half_bm, half_bn, half_bk;
  int32_t Mp, Np;
  int32_t num_chunks;
  int32_t tiles_m, tiles_n;
  void* C;
  int64_t ldc;
  const void* residual;
  int64_t ldr;
  int32_t residual_f32;
  int32_t aux_f32;
  const void* bias;
  const void* rope_cos;
  const void* rope_sin;
  int64_t ld_rope;
  const void* rope_scale;
  int32_t half_head;
  float inv_head_dim;
  float eps;
  int* err;
  // Research options (strassen_pallas.py:205-226, 466-517, 575-586).
  int32_t formula;                 // 0 classical, 1 dual
  int32_t swap_m, swap_k, swap_n;  // block_permutation bits
  const int32_t* panel_schedule;   // device [num_panels], nonzero = exact panel; may be null
  int32_t num_panels;
  int32_t raster;                  // four-CTA kernel: tile rows per column sweep (0 = its default)
};

// Whether K chunk c lies in an exact classical panel.
__device__ __forceinline__ bool exact_chunk(const GemmParams& p, int c, int chunk_k) {
  if (p.panel_schedule == nullptr) return false;
  const int panel = (c * chunk_k) / p.half_bk;
  return __ldg(p.panel_schedule + panel) != 0;
}

// True when every K panel is exact: then accumulators 0, 3 and 4 are never
// written (the exact schedule below only uses 1, 2, 5 and 6).
__device__ __forceinline__ bool all_panels_exact(const GemmParams& p) {
  if (p.panel_schedule == nullptr) return false;
  for (int i = 0; i < p.num_panels; ++i)
    if (__ldg(p.panel_schedule + i) == 0) return false;
  return true;
}

__device__ int g_device_error = 0;

enum : int {
  kErrWaitRaw = 1,
  kErrWaitSums = 2,
  kErrWaitEmpty = 3,
  kErrWaitAcc = 4,
  kErrSelfTest = SB_SELFTEST_ERROR_CODE,
};

__device__ __forceinline__ float load_aux(const void* p, int64_t idx, int f32) {
  if (f32) return __ldg(reinterpret_cast<const float*>(p) + idx);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
}

__device__ __forceinline__ void load8(const void* base, int64_t idx, int f32, float (&v)[8]) {
  if (f32) {
    const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    float4 x = q[0], y = q[1];
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
  } else {
    uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + idx);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <bool kOutF32>
__device__ __forceinline__ void store8(void* base, int64_t idx, const float (&v)[8]) {
  if (kOutF32) {
    float4* q = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + idx);
    q[0] = make_float4(v[0], v[1], v[2], v[3]);
    q[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                         pack_bf16x2(v[6], v[7]));
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + idx) = u;
  }
}

__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float gelu_tanh_f32(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

// Recombined quadrant values for 8 consecutive product columns of this
// thread's product row.
struct Quad8 {
  float c[4][8];
};

template <bool kStrassen, int kOpts>
__device__ __forceinline__ void read_quadrants(uint32_t tmem_row, int col, Quad8& out,
                                               const GemmParams& p, bool all_exact) {
  if constexpr (kStrassen) {
    float m[7][8];
#pragma unroll
    for (int i = 0; i < 7; ++i) tmem_load_8(tmem_row + i * kBlockN + col, m[i]);
    if (kOpts && all_exact) {
#pragma unroll
      for (int e = 0; e < 8; ++e) m[0][e] = m[3][e] = m[4][e] = 0.f;
    }
    if (kFormula<kOpts>() == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // strassen_pallas.py:324-379 quadrant updates, summed once.
        out.c[0][e] = ((m[0][e] + m[3][e]) - m[4][e]) + m[6][e];
        out.c[1][e] = m[2][e] + m[4][e];
        out.c[2][e] = m[1][e] + m[3][e];
        out.c[3][e] = ((m[0][e] - m[1][e]) + m[2][e]) + m[5][e];
      }
    } else if (kFormula<kOpts>() == 2) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // Power-of-two formula: basis updates (strassen_pallas.py:398-464) then
        // the decode of strassen_pallas.py:744-761.
        const float z0 = m[2][e] + m[4][e];
        const float z1 = m[5][e] + m[6][e];
        const float z2 = m[1][e] - m[3][e];
        const float z3 = ((m[0][e] - m[2][e]) + m[3][e]) + m[6][e];
        out.c[3][e] = z0;
        out.c[2][e] = z3 + z0 * 0.5f;
        out.c[0][e] = (z1 + z2) * 0.5f + z0 * 0.25f;
        out.c[1][e] = ((z2 - z1) + z3) + z0 * 0.5f;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // Dual formula, strassen_pallas.py:466-517.
        out.c[0][e] = ((m[0][e] + m[3][e]) - m[4][e]) + m[6][e];
        out.c[1][e] = m[1][e] + m[3][e];
        out.c[2][e] = m[2][e] + m[4][e];
        out.c[3][e] = ((m[0][e] - m[1][e]) + m[2][e]) + m[5][e];
      }
    }
    // block_permutation: the quadrant computed at (r, c) belongs at (r^swap_m, c^swap_n).
    if (kOpts && p.swap_m) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float t0 = out.c[0][e], t1 = out.c[1][e];
        out.c[0][e] = out.c[2][e];
        out.c[1][e] = out.c[3][e];
        out.c[2][e] = t0;
        out.c[3][e] = t1;
      }
    }
    if (kOpts && p.swap_n) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float t0 = out.c[0][e], t2 = out.c[2][e];
        out.c[0][e] = out.c[1][e];
        out.c[2][e] = out.c[3][e];
        out.c[1][e] = t0;
        out.c[3][e] = t2;
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) tmem_load_8(tmem_row + q * kBlockN + col, out.c[q]);
  }
}

// Epilogue of one 128 x 64 product tile, run by the eight epilogue warps once
// the accumulators are final: reads M1..M7 (or the quadrant accumulators) per
// TMEM lane, recombines the quadrants and applies the fused epilogue
// (strassen_pallas.py:739-879).  Product rows start at t0, columns at u0.
template <bool kStrassen, int kEpi, bool kOutF32, int kOpts>
__device__ __forceinline__ void tile_epilogue(const GemmParams& p, uint32_t tmem_base, int t0, int u0,
                                              int warp, int lane, uint8_t* smem, uint32_t qss_bar,
                                              volatile int* abort_flag) {
  const int q = warp & 3;                  // TMEM lane quarter this warp may read
  const int h = (warp - kFirstSumWarp) >> 2;  // which 32-column half of the tile
  const int row_in_tile = 32 * q + lane;
  const int t = t0 + row_in_tile;
  const bool row_ok = t < p.Mp;
  const int blk_i = t / p.half_bm;
  const int rp = t - blk_i * p.half_bm;
  const int64_t row_top = (int64_t)blk_i * p.bm + rp;
  const int64_t row_bot = row_top + p.half_bm;
  const int j_block = u0 / p.half_bn;
  const int cp_base = u0 - j_block * p.half_bn;  // column inside the half block
  const int64_t col_left0 = (int64_t)j_block * p.bn + cp_base;
  const uint32_t tmem_row = tmem_base + ((uint32_t)(32 * q) << 16);
  const bool all_exact = kStrassen && kOpts && all_panels_exact(p);

  if constexpr (kEpi == SB_EPI_QK_NORM_ROPE) {
    // Per-head sum of squares over both halves of every head
    // (strassen_pallas.py:793-835).  A head's a-half lies in quadrant 0/2,
    // its b-half at the same offset in quadrant 1/3.  Pass 1 writes this
    // thread's partial sums per head slot, pass 2 normalises and rotates.
    float* qss = reinterpret_cast<float*>(smem);  // stage memory is idle now
    bool return_early = false;
    auto qidx = [&](int hh, int tb, int slot) { return ((hh * 2 + tb) * kBlockM + row_in_tile) * 8 + slot; };
#pragma unroll
    for (int slot = 0; slot < 8; ++slot) {
      qss[qidx(h, 0, slot)] = 0.f;
      qss[qidx(h, 1, slot)] = 0.f;
    }
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      const int col = 32 * h + 8 * j;
      Quad8 v;
      read_quadrants<kStrassen, kOpts>(tmem_row, col, v, p, all_exact);
      const int slot = col / p.half_head;
      float st = 0.f, sbm = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        st += v.c[0][e] * v.c[0][e] + v.c[1][e] * v.c[1][e];
        sbm += v.c[2][e] * v.c[2][e] + v.c[3][e] * v.c[3][e];
      }
      qss[qidx(h, 0, slot)] += st;
      qss[qidx(h, 1, slot)] += sbm;
    }
    // Exchange partial sums between the two column halves (bounded wait).
    __syncwarp();
    if (lane == 0) mbar_arrive(qss_bar);
    if (!warp_wait(qss_bar, 0, abort_flag, p.err, kErrWaitAcc)) return_early = true;
    if (!return_early) {
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      const int col = 32 * h + 8 * j;
      Quad8 v;
      read_quadrants<kStrassen, kOpts>(tmem_row, col, v, p, all_exact);
      const int slot = col / p.half_head;
      const int cp = cp_base + col;
#pragma unroll
      for (int tb = 0; tb < 2; ++tb) {
        const float sums = qss[qidx(0, tb, slot)] + qss[qidx(1, tb, slot)];
        const float recip = 1.0f / sqrtf(sums * p.inv_head_dim + p.eps);
        const int64_t row = tb ? row_bot : row_top;
        float outa[8], outb[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float sa = load_aux(p.rope_scale, cp + e, p.aux_f32);
          const float sbv = load_aux(p.rope_scale, p.half_bn + cp + e, p.aux_f32);
          const float cs = row_ok ? load_aux(p.rope_cos, row * p.ld_rope + cp + e, p.aux_f32) : 0.f;
          const float sn = row_ok ? load_aux(p.rope_sin, row * p.ld_rope + cp + e, p.aux_f32) : 0.f;
          const float na = v.c[2 * tb][e] * recip * sa;
          const float nb = v.c[2 * tb + 1][e] * recip * sbv;
          outa[e] = na * cs - nb * sn;
          outb[e] = nb * cs + na * sn;
        }
        if (row_ok) {
          store8<kOutF32>(p.C, row * p.ldc + col_left0 + col, outa);
          store8<kOutF32>(p.C, row * p.ldc + col_left0 + p.half_bn + col, outb);
        }
      }
    }
    }
  } else {
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      const int col = 32 * h + 8 * j;
      Quad8 v;
      read_quadrants<kStrassen, kOpts>(tmem_row, col, v, p, all_exact);
      if (!row_ok) continue;
      const int64_t cl = col_left0 + col;
      const int64_t cr = cl + p.half_bn;
      if constexpr (kEpi == SB_EPI_SWIGLU || kEpi == SB_EPI_GEGLU) {
        // strassen_pallas.py:762-777: quadrants 0/2 gate, 1/3 up; output
        // column J*bn/2 + c'.
        float top[8], bot[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if constexpr (kEpi == SB_EPI_SWIGLU) {
            top[e] = silu_f32(v.c[0][e]) * v.c[1][e];
            bot[e] = silu_f32(v.c[2][e]) * v.c[3][e];
          } else {
            top[e] = gelu_tanh_f32(v.c[0][e]) * v.c[1][e];
            bot[e] = gelu_tanh_f32(v.c[2][e]) * v.c[3][e];
          }
        }
        const int64_t oc = (int64_t)j_block * p.half_bn + cp_base + col;
        store8<kOutF32>(p.C, row_top * p.ldc + oc, top);
        store8<kOutF32>(p.C, row_bot * p.ldc + oc, bot);
      } else {
        if constexpr (kEpi == SB_EPI_RESIDUAL_ADD) {
          // strassen_pallas.py:778-792
          float r[8];
          load8(p.residual, row_top * p.ldr + cl, p.residual_f32, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) v.c[0][e] += r[e];
          load8(p.residual, row_top * p.ldr + cr, p.residual_f32, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) v.c[1][e] += r[e];
          load8(p.residual, row_bot * p.ldr + cl, p.residual_f32, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) v.c[2][e] += r[e];
          load8(p.residual, row_bot * p.ldr + cr, p.residual_f32, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) v.c[3][e] += r[e];
        } else if constexpr (kEpi == SB_EPI_BIAS_ADD) {
          // strassen_pallas.py:867-874
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float bl = load_aux(p.bias, cl + e, p.aux_f32);
            const float br = load_aux(p.bias, cr + e, p.aux_f32);
            v.c[0][e] += bl;
            v.c[2][e] += bl;
            v.c[1][e] += br;
            v.c[3][e] += br;
          }
        }
        store8<kOutF32>(p.C, row_top * p.ldc + cl, v.c[0]);
        store8<kOutF32>(p.C, row_top * p.ldc + cr, v.c[1]);
        store8<kOutF32>(p.C, row_bot * p.ldc + cl, v.c[2]);
        store8<kOutF32>(p.C, row_bot * p.ldc + cr, v.c[3]);
      }
    }
  }
}

// kOpts compiles in the research options (dual and power-of-two formulas,
// block permutation, exact panels); the default launch uses the lean classical
// instantiation.
// kATrans: A is stored transposed, (K, M) row-major (strassen_matmul_lhs_transposed);
// its tiles arrive M-major and feed the MMA as an MN-major operand.
template <bool kStrassen, int kEpi, bool kOutF32, int kOpts, bool kATrans = false>
__global__ void __launch_bounds__(kThreads, 1)
    strassen_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b, const GemmParams p) {
  constexpr bool kTs = uses_tmem_a<kStrassen, kOpts, kATrans>();
  static_assert(!kOpts || kTs, "research options run on the TMEM-ring layout");
  using P = PipeFor<kStrassen, kTs>;
  constexpr int kStages = P::STAGES;
  constexpr int kStageBytes = P::STAGE_BYTES;
  constexpr int kASlotBytes = P::A_SLOT;
  constexpr int kBSlotBytes = P::B_SLOT;
  constexpr int kBlockK = P::BK;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t smem_base = smem_addr(smem);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::DATA_BYTES);
  const uint32_t full_bar = smem_addr(bars);                 // [kStages] TMA landed
  const uint32_t sums_bar = smem_addr(bars + kStages);       // [kStages] operand sums ready
  const uint32_t empty_bar = smem_addr(bars + 2 * kStages);  // [kStages] MMAs done reading
  const uint32_t acc_bar = smem_addr(bars + 3 * kStages);    // accumulators final
  const uint32_t qss_bar = smem_addr(bars + 3 * kStages + 1);  // q/k partial sums written
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3 * kStages + 2);
  static_assert((3 * kStages + 2) * 8 + 8 <= kBarrierBytes, "barrier area");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Grouped rasterisation: walk 8 product-row tiles per column sweep for L2 reuse.
  const int tile = blockIdx.x;
  const int group_rows = kRasterGroup;
  const int per_group = group_rows * p.tiles_n;
  const int group = tile / per_group;
  const int first_m = group * group_rows;
  const int rows_in_group = min(p.tiles_m - first_m, group_rows);
  const int in_group = tile - group * per_group;
  const int tm = first_m + in_group % rows_in_group;
  const int tn = in_group / rows_in_group;
  const int t0 = tm * kBlockM;  // first product row
  const int u0 = tn * kBlockN;  // first product column

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(sums_bar + 8 * s, kTs ? 4 : kSumWarps);  // kTs: the set owning the step
      mbar_init(empty_bar + 8 * s, 1);
    }
    mbar_init(acc_bar, 1);
    mbar_init(qss_bar, kSumWarps);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) tmem_alloc<kTmemCols>(smem_addr(tmem_holder));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if constexpr (kTs) {
     if (lane == 0) {
      int last_issued[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) last_issued[s] = -1;
      const int a_row_base = t0 % p.half_bm;
      const int a_block = t0 / p.half_bm;
      const int j_block = u0 / p.half_bn;
      const int b_col0 = j_block * p.bn + (u0 % p.half_bn);
      for (int c = 0; c < p.num_chunks; ++c) {
        const int s = c % kStages;
        if (!mbar_wait(empty_bar + 8 * s, ((c / kStages) & 1u) ^ 1u, abort_flag, p.err, kErrWaitEmpty)) break;
        const int kap = c * 16;
        const int panel = kap / p.half_bk;
        const int kcol = panel * p.bk + (kap - panel * p.half_bk);
        const uint32_t fb = full_bar + 8 * s;
        const uint32_t stage = smem_base + s * kStageBytes;
        mbar_arrive_expect_tx(fb, P::RAW_TX);
        // One copy per operand lands all four quadrants in slot order (make_ts_maps).
        tma_load_5d(stage, &tmap_a, fb, kcol, a_row_base, a_block, 0, 0);
        tma_load_4d(stage + P::B_OFFSET, &tmap_b, fb, b_col0, kcol, 0, 0);
        last_issued[s] = c;
      }
      // Drain: never leave a TMA write in flight past teardown.
#pragma unroll
      for (int s = 0; s < kStages; ++s)
        if (last_issued[s] >= 0) mbar_wait_drain(full_bar + 8 * s, (last_issued[s] / kStages) & 1u);
     }
    } else if (lane == 0) {
      int last_issued[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) last_issued[s] = -1;
      const int a_row_base = t0 % p.half_bm;  // 0 when a tile spans several blocks
      const int a_block = t0 / p.half_bm;
      const int j_block = u0 / p.half_bn;
      const int b_col0 = j_block * p.bn + (u0 % p.half_bn);
      for (int c = 0; c < p.num_chunks; ++c) {
        const int s = c % kStages;
        const uint32_t ph = (c / kStages) & 1u;
        if (!mbar_wait(empty_bar + 8 * s, ph ^ 1u, abort_flag, p.err, kErrWaitEmpty)) break;
        const uint32_t fb = full_bar + 8 * s;
        mbar_arrive_expect_tx(fb, P::RAW_TX);
        const int kap = c * kBlockK;
        const int panel = kap / p.half_bk;
        const int kin = kap - panel * p.half_bk;
        const uint32_t stage = smem_base + s * kStageBytes;
        // Slot (2*qr + qk) of A holds the block's quadrant (qr, qk), slot
        // (2*qk + qc) of B its quadrant (qk, qc).
#pragma unroll
        for (int qk = 0; qk < 2; ++qk) {
          const int kcol = panel * p.bk + qk * p.half_bk + kin;
#pragma unroll
          for (int qr = 0; qr < 2; ++qr) {
            if constexpr (kATrans) {
              // Two 64-row halves of the 128-row product tile, each a (16 k x 64 m)
              // box of A^T; half h lands 2 KB after half 0 (the MN-major LBO).
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int t = t0 + 64 * h;
                const int blk = t / p.half_bm;
                const int m_coord = blk * p.bm + qr * p.half_bm + (t - blk * p.half_bm);
                tma_load_2d(stage + (2 * qr + qk) * kASlotBytes + h * 2048, &tmap_a, fb, m_coord, kcol);
              }
            } else {
              tma_load_3d(stage + (2 * qr + qk) * kASlotBytes, &tmap_a, fb, kcol,
                          qr * p.half_bm + a_row_base, a_block);
            }
          }
#pragma unroll
          for (int qc = 0; qc < 2; ++qc) {
            tma_load_2d(stage + P::B_OFFSET + (2 * qk + qc) * kBSlotBytes, &tmap_b, fb,
                        b_col0 + qc * p.half_bn, kcol);
          }
        }
        last_issued[s] = c;
      }
      // Drain: never leave a TMA write in flight past teardown.
#pragma unroll
      for (int s = 0; s < kStages; ++s) {
        if (last_issued[s] >= 0) mbar_wait_drain(full_bar + 8 * s, (last_issued[s] / kStages) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if constexpr (kTs) {
     if (lane == 0) {
      // One wait per K step: the sum warps arrive on sums_bar only after the
      // stage's TMA copies landed, so it also covers the raw tiles.  The issue
      // queue is shallow, so every synchronisation in this thread idles the
      // tensor pipe: one wait and one commit per step, descriptors advanced by
      // adding (byte offset >> 4) to precomputed stage-0 descriptors.
      constexpr uint64_t kA = kASlotBytes >> 4, kB = kBSlotBytes >> 4;
      const uint64_t a_d0 = umma_smem_desc(smem_base, P::A_LBO, P::A_SBO, P::A_LAYOUT);
      const uint64_t b_d0 = umma_smem_desc(smem_base + P::B_OFFSET, P::B_LBO, P::B_SBO, P::B_LAYOUT);
      // Research options: per product, the A operand (ring columns, or a shared-
      // memory descriptor offset) and the B descriptor offset, resolved once into
      // registers for the formula and block permutation; likewise the exact-step
      // schedule.  The loop then only adds them to the stage descriptors.
      uint32_t r_off[7], e_acc[12], e_neg[12];
      uint64_t a_off[7], b_off[7], ea_off[12], eb_off[12];
      bool from_ring[7];
      uint32_t written = 0;  // accumulators holding a product (exact steps skip some)
      bool exact_step = false;
      if constexpr (kOpts) {
        constexpr int f = kFormula<kOpts>();
        const int xa = 2 * p.swap_m + p.swap_k, xb = 2 * p.swap_k + p.swap_n;
#pragma unroll
        for (int i = 0; i < 7; ++i) {
          const int rr = f == 0 ? kProdRing[0][i] : f == 1 ? kProdRing[1][i] : kProdRing[2][i];
          int as = f == 0 ? kProdA[0][i] : f == 1 ? kProdA[1][i] : kProdA[2][i];
          int bs = f == 0 ? kProdB[0][i] : f == 1 ? kProdB[1][i] : kProdB[2][i];
          if (f != 2) {
            as ^= xa;
            if (bs < 4) bs ^= xb;
          }
          from_ring[i] = rr >= 0;
          r_off[i] = rr >= 0 ? 8 * rr : 0;
          a_off[i] = (uint64_t)as * kA;
          b_off[i] = (uint64_t)bs * kB;
        }
#pragma unroll
        for (int e = 0; e < 12; ++e) {
          e_acc[e] = f == 1 ? kExactAcc[1][e] : kExactAcc[0][e];
          e_neg[e] = f == 1 ? kExactNeg[1][e] : kExactNeg[0][e];
          ea_off[e] = (uint64_t)(kExactA[e] ^ xa) * kA;
          eb_off[e] = (uint64_t)(kExactB[e] ^ xb) * kB;
        }
      }
      int s = 0;
      uint32_t ph = 0;
      for (int c = 0; c < p.num_chunks; ++c) {
        if (!mbar_wait(sums_bar + 8 * s, ph, abort_flag, p.err, kErrWaitSums)) break;
        tc_fence_after();
        const uint64_t ad = a_d0 + (uint32_t)((s * kStageBytes) >> 4);
        const uint64_t bd = b_d0 + (uint32_t)((s * kStageBytes) >> 4);
        const uint32_t acc = c != 0 ? 1u : 0u;
        const uint32_t ring = tmem_base + kRingCol0 + 32 * (c & 1);
        if constexpr (kOpts) {
          // The schedule entry changes only at K-panel boundaries.
          if (p.panel_schedule != nullptr && (c * 16) % p.half_bk == 0) exact_step = exact_chunk(p, c, 16);
          if (exact_step) {
            // Exact classical step on the raw quadrants (see kExactAcc).
#pragma unroll
            for (int e = 0; e < 12; ++e) {
              umma_bf16_ss(tmem_base + e_acc[e] * kBlockN, ad + ea_off[e], bd + eb_off[e],
                           e_neg[e] ? kIdescNegA : kIdesc, (written >> e_acc[e]) & 1u);
              written |= 1u << e_acc[e];
            }
          } else {
#pragma unroll
            for (int i = 0; i < 7; ++i) {
              const uint32_t a_acc = (written >> i) & 1u;
              if (from_ring[i])
                umma_bf16_ts(tmem_base + i * kBlockN, ring + r_off[i], bd + b_off[i], kIdesc, a_acc);
              else
                umma_bf16_ss(tmem_base + i * kBlockN, ad + a_off[i], bd + b_off[i], kIdesc, a_acc);
            }
            written = 0x7Fu;
          }
          umma_commit(empty_bar + 8 * s);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
          continue;
        }
        umma_bf16_ts(tmem_base + 0 * kBlockN, ring + 0, bd + 4 * kB, kIdesc, acc);        // (a0+a3)(b0+b3)
        umma_bf16_ts(tmem_base + 1 * kBlockN, ring + 8, bd, kIdesc, acc);                 // (a2+a3) b0
        umma_bf16_ss(tmem_base + 2 * kBlockN, ad, bd + 1 * kB, kIdesc, acc);              // a0 (b1-b3)
        umma_bf16_ss(tmem_base + 3 * kBlockN, ad + 3 * kA, bd + 2 * kB, kIdesc, acc);     // a3 (b2-b0)
        umma_bf16_ss(tmem_base + 4 * kBlockN, ad + 1 * kA, bd + 3 * kB, kIdesc, acc);     // (a0+a1) b3
        umma_bf16_ts(tmem_base + 5 * kBlockN, ring + 16, bd + 5 * kB, kIdesc, acc);       // (a2-a0)(b0+b1)
        umma_bf16_ts(tmem_base + 6 * kBlockN, ring + 24, bd + 6 * kB, kIdesc, acc);       // (a1-a3)(b2+b3)
        // Frees stage s and, for the A-sum warps, ring half c & 1 (two steps on).
        umma_commit(empty_bar + 8 * s);
        if (++s == kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      // Always commit: the epilogue (or the teardown drain) waits on it.
      umma_commit(acc_bar);
     }
    } else if (lane == 0) {
      // Operand slot byte offsets of the seven products, resolved once.
      uint32_t a_off[7], b_off[7];
#pragma unroll
      for (int i = 0; i < 7; ++i) {
        a_off[i] = kASlot[i] * kASlotBytes;
        b_off[i] = kBSlot[i] * kBSlotBytes;
      }
      for (int c = 0; c < p.num_chunks; ++c) {
        const int s = c % kStages;
        const uint32_t ph = (c / kStages) & 1u;
        if (!mbar_wait(full_bar + 8 * s, ph, abort_flag, p.err, kErrWaitRaw)) break;
        if constexpr (kStrassen) {
          if (!mbar_wait(sums_bar + 8 * s, ph, abort_flag, p.err, kErrWaitSums)) break;
        }
        tc_fence_after();
        const uint32_t a_stage = smem_base + s * kStageBytes;
        const uint32_t b_stage = a_stage + P::B_OFFSET;
#pragma unroll
        for (int kk = 0; kk < kBlockK / 16; ++kk) {
          if constexpr (kStrassen) {
#pragma unroll
            for (int i = 0; i < 7; ++i) {
              const uint64_t ad = kATrans
                  ? umma_smem_desc(a_stage + a_off[i] + kk * 2048, 2048, 1024, kLayoutSwizzle128B)
                  : umma_smem_desc(a_stage + a_off[i] + kk * 32, P::A_LBO, P::A_SBO, P::A_LAYOUT);
              const uint64_t bd = umma_smem_desc(b_stage + b_off[i] + kk * 2048,
                                                 P::B_LBO, P::B_SBO, P::B_LAYOUT);
              umma_bf16_ss(tmem_base + i * kBlockN, ad, bd, kATrans ? kIdescAT : kIdesc,
                           (c | kk) != 0 ? 1u : 0u);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint64_t ad = umma_smem_desc(a_stage + kCAslot[i] * kASlotBytes + kk * 32, P::A_LBO,
                                                 P::A_SBO, P::A_LAYOUT);
              const uint64_t bd = umma_smem_desc(b_stage + kCBslot[i] * kBSlotBytes + kk * 2048,
                                                 P::B_LBO, P::B_SBO, P::B_LAYOUT);
              const bool first = (c == 0) && (kk == 0) && ((i & 1) == 0);
              umma_bf16_ss(tmem_base + (i >> 1) * kBlockN, ad, bd, kIdesc, first ? 0u : 1u);
            }
          }
        }
        umma_commit(empty_bar + 8 * s);
      }
      // Always commit: the epilogue (or the teardown drain) waits on it.
      umma_commit(acc_bar);
    }
  } else if (warp >= kFirstSumWarp) {
    const int sum_tid = threadIdx.x - kFirstSumWarp * 32;  // 0..255
    bool ok = true;
    // ------------------------------------------------------------ operand sums
    if constexpr (kTs) {
      // Two sets of four warps take alternate K steps (set = step & 1), so each
      // warp's per-step chain (loads, ring wait, TMEM stores, fences) has two
      // steps of time.  Within a set, warp w owns TMEM lane quarter w % 4.
      // A sums: each thread owns one product row and reads that row's two
      // 16-byte chunks from the four raw A quadrants, conflict-free (8 rows per
      // wavefront); one A operand goes back to shared memory, four to ring half
      // (step & 1) in TMEM.  B sums: one 16-byte chunk of every B slot per
      // thread, in place in shared memory.
      static_assert(kBSlotBytes == 128 * 16, "one B chunk per thread of a set");
      const int set = (warp - kFirstSumWarp) >> 2;
      const int q = warp & 3;
      const uint32_t row = 32 * q + lane;
      // Row `row` of a 32-byte-swizzled A tile: its two 16-byte chunks swap
      // places on rows with bit 2 set.
      const uint32_t sw = (row >> 2) & 1u;
      const uint32_t lo_off = 32 * row + 16 * sw;
      const uint32_t hi_off = 32 * row + 16 * (sw ^ 1u);
      const uint32_t tmem_lane = tmem_base + ((uint32_t)(32 * q) << 16) + kRingCol0;
      const uint32_t b_off = 16 * row;
      const uint32_t xa = kOpts ? 2 * p.swap_m + p.swap_k : 0;  // block permutation
      const uint32_t xb = kOpts ? 2 * p.swap_k + p.swap_n : 0;
      bool exact = false;  // this step lies in an exact classical panel
      for (int c = set; c < p.num_chunks; c += 2) {
        const int s = c % kStages;
        // Every lane waits itself: cheaper than a lane-0 poll and broadcast.
        if (!__all_sync(0xffffffffu, mbar_wait(full_bar + 8 * s, (c / kStages) & 1u, abort_flag, p.err,
                                               kErrWaitRaw))) {
          ok = false;
          break;
        }
        const uint32_t a_stage = smem_base + s * kStageBytes;
        const uint32_t b_stage = a_stage + P::B_OFFSET;
        // Research options: operand a_j / b_j of the block permutation sits in
        // slot j ^ xa / j ^ xb; an exact classical step multiplies the raw
        // quadrants and needs no sums.
        // The schedule entry changes only at K-panel boundaries (a set sees a
        // boundary step or the step after it, hence the two-step window).
        if (kOpts && p.panel_schedule != nullptr && (c * 16) % p.half_bk < 32) exact = exact_chunk(p, c, 16);
        uint4 rlo[4], rhi[4];  // the four A operands for the TMEM ring
        if (!exact) {
          uint4 lo[4], hi[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            lo[t] = lds128(a_stage + (t ^ xa) * kASlotBytes + lo_off);
            hi[t] = lds128(a_stage + (t ^ xa) * kASlotBytes + hi_off);
          }
          uint4 b[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) b[t] = lds128(b_stage + (t ^ xb) * kBSlotBytes + b_off);
          constexpr int formula = kFormula<kOpts>();
          if (formula == 0) {
            // Classical (strassen_pallas.py:324-379): a0+a1 over a1; ring
            // a0+a3, a2+a3, a2-a0, a1-a3.
            sts128(a_stage + (1 ^ xa) * kASlotBytes + lo_off, add4(lo[0], lo[1]));
            sts128(a_stage + (1 ^ xa) * kASlotBytes + hi_off, add4(hi[0], hi[1]));
            rlo[0] = add4(lo[0], lo[3]); rhi[0] = add4(hi[0], hi[3]);
            rlo[1] = add4(lo[2], lo[3]); rhi[1] = add4(hi[2], hi[3]);
            rlo[2] = sub4(lo[2], lo[0]); rhi[2] = sub4(hi[2], hi[0]);
            rlo[3] = sub4(lo[1], lo[3]); rhi[3] = sub4(hi[1], hi[3]);
            sts128(b_stage + 4 * kBSlotBytes + b_off, add4(b[0], b[3]));
            sts128(b_stage + 5 * kBSlotBytes + b_off, add4(b[0], b[1]));
            sts128(b_stage + 6 * kBSlotBytes + b_off, add4(b[2], b[3]));
            sts128(b_stage + (1 ^ xb) * kBSlotBytes + b_off, sub4(b[1], b[3]));
            sts128(b_stage + (2 ^ xb) * kBSlotBytes + b_off, sub4(b[2], b[0]));
          } else if (formula == 1) {
            // Dual (strassen_pallas.py:466-517): a1-a0 over a1; ring a0+a3,
            // a2-a3, a0+a2, a1+a3.
            sts128(a_stage + (1 ^ xa) * kASlotBytes + lo_off, sub4(lo[1], lo[0]));
            sts128(a_stage + (1 ^ xa) * kASlotBytes + hi_off, sub4(hi[1], hi[0]));
            rlo[0] = add4(lo[0], lo[3]); rhi[0] = add4(hi[0], hi[3]);
            rlo[1] = sub4(lo[2], lo[3]); rhi[1] = sub4(hi[2], hi[3]);
            rlo[2] = add4(lo[0], lo[2]); rhi[2] = add4(hi[0], hi[2]);
            rlo[3] = add4(lo[1], lo[3]); rhi[3] = add4(hi[1], hi[3]);
            sts128(b_stage + 4 * kBSlotBytes + b_off, add4(b[0], b[3]));
            sts128(b_stage + 5 * kBSlotBytes + b_off, sub4(b[1], b[0]));
            sts128(b_stage + 6 * kBSlotBytes + b_off, sub4(b[2], b[3]));
            sts128(b_stage + (1 ^ xb) * kBSlotBytes + b_off, add4(b[1], b[3]));
            sts128(b_stage + (2 ^ xb) * kBSlotBytes + b_off, add4(b[0], b[2]));
          } else {
            // Power-of-two formula (strassen_pallas.py:398-464), each bf16 op
            // rounded in the reference's order: A3, A4, A5 into slots 0-2, ring
            // A1, A2, A6, A7; B1..B7 into B slots 0-6.
            const uint4 h1l = half4(lo[1]), h2l = half4(lo[2]), h3l = half4(lo[3]), q3l = quarter4(lo[3]);
            const uint4 h1h = half4(hi[1]), h2h = half4(hi[2]), h3h = half4(hi[3]), q3h = quarter4(hi[3]);
            rlo[0] = sub4(lo[2], lo[1]); rhi[0] = sub4(hi[2], hi[1]);
            rlo[1] = add4(sub4(lo[0], h2l), sub4(h1l, q3l)); rhi[1] = add4(sub4(hi[0], h2h), sub4(h1h, q3h));
            rlo[2] = add4(sub4(lo[0], h1l), sub4(h2l, q3l)); rhi[2] = add4(sub4(hi[0], h1h), sub4(h2h, q3h));
            rlo[3] = add4(lo[1], h3l); rhi[3] = add4(hi[1], h3h);
            sts128(a_stage + 0 * kASlotBytes + lo_off, sub4(lo[2], h3l));
            sts128(a_stage + 0 * kASlotBytes + hi_off, sub4(hi[2], h3h));
            sts128(a_stage + 1 * kASlotBytes + lo_off, sub4(lo[1], h3l));
            sts128(a_stage + 1 * kASlotBytes + hi_off, sub4(hi[1], h3h));
            sts128(a_stage + 2 * kASlotBytes + lo_off, add4(lo[2], h3l));
            sts128(a_stage + 2 * kASlotBytes + hi_off, add4(hi[2], h3h));
            const uint4 h0 = half4(b[0]), h1 = half4(b[1]), h3 = half4(b[3]), q1 = quarter4(b[1]);
            sts128(b_stage + 0 * kBSlotBytes + b_off, sub4(b[0], b[3]));
            sts128(b_stage + 1 * kBSlotBytes + b_off, add4(b[0], h1));
            sts128(b_stage + 2 * kBSlotBytes + b_off, sub4(h1, b[3]));
            sts128(b_stage + 3 * kBSlotBytes + b_off, add4(sub4(h0, b[2]), sub4(q1, h3)));
            sts128(b_stage + 4 * kBSlotBytes + b_off, add4(h1, b[3]));
            sts128(b_stage + 5 * kBSlotBytes + b_off, sub4(b[0], h1));
            sts128(b_stage + 6 * kBSlotBytes + b_off, sub4(add4(h0, b[2]), add4(q1, h3)));
          }
        }
        // Shared-memory sums are complete: order them for the tensor core now,
        // so only the TMEM stores follow the ring wait.
        fence_proxy_async_smem();
        if (!exact) {
          // Ring half c & 1 is free once the MMAs of step c - 2 completed: the
          // commit that frees stage (c - 2) % kStages.  Every lane waits itself
          // (no lane-0 poll and broadcast on this path).
          if (c >= 2) {
            const bool waited = mbar_wait(empty_bar + 8 * ((c - 2) % kStages), ((c - 2) / kStages) & 1u,
                                          abort_flag, p.err, kErrWaitEmpty);
            if (!__all_sync(0xffffffffu, waited)) {
              ok = false;
              break;
            }
          }
          tc_fence_after();
          const uint32_t ring = tmem_lane + 32 * (c & 1);
#pragma unroll
          for (int j = 0; j < 4; ++j) tmem_store_8(ring + 8 * j, rlo[j], rhi[j]);
          tmem_store_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sums_bar + 8 * s);
      }
    } else if constexpr (kStrassen) {
      for (int c = 0; c < p.num_chunks; ++c) {
        const int s = c % kStages;
        const uint32_t ph = (c / kStages) & 1u;
        if (!warp_wait(full_bar + 8 * s, ph, abort_flag, p.err, kErrWaitRaw)) {
          ok = false;
          break;
        }
        const uint32_t a_stage = smem_base + s * kStageBytes;
        const uint32_t b_stage = a_stage + P::B_OFFSET;
        {
#pragma unroll
        for (int idx = sum_tid; idx < kASlotBytes / 16; idx += kSumThreads) {
          const uint32_t off = idx * 16;
          const uint4 a0 = lds128(a_stage + 0 * kASlotBytes + off);
          const uint4 a1 = lds128(a_stage + 1 * kASlotBytes + off);
          const uint4 a2 = lds128(a_stage + 2 * kASlotBytes + off);
          const uint4 a3 = lds128(a_stage + 3 * kASlotBytes + off);
          sts128(a_stage + 4 * kASlotBytes + off, add4(a0, a3));
          sts128(a_stage + 5 * kASlotBytes + off, add4(a2, a3));
          sts128(a_stage + 6 * kASlotBytes + off, sub4(a1, a3));
          sts128(a_stage + 1 * kASlotBytes + off, add4(a0, a1));
          sts128(a_stage + 2 * kASlotBytes + off, sub4(a2, a0));
        }
#pragma unroll
        for (int idx = sum_tid; idx < kBSlotBytes / 16; idx += kSumThreads) {
          const uint32_t off = idx * 16;
          const uint4 b0 = lds128(b_stage + 0 * kBSlotBytes + off);
          const uint4 b1 = lds128(b_stage + 1 * kBSlotBytes + off);
          const uint4 b2 = lds128(b_stage + 2 * kBSlotBytes + off);
          const uint4 b3 = lds128(b_stage + 3 * kBSlotBytes + off);
          sts128(b_stage + 4 * kBSlotBytes + off, add4(b0, b3));
          sts128(b_stage + 5 * kBSlotBytes + off, add4(b0, b1));
          sts128(b_stage + 6 * kBSlotBytes + off, add4(b2, b3));
          sts128(b_stage + 1 * kBSlotBytes + off, sub4(b1, b3));
          sts128(b_stage + 2 * kBSlotBytes + off, sub4(b2, b0));
        }
        }
        // Make the generic-proxy writes visible to the tensor core, then signal.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(sums_bar + 8 * s);
      }
    }

    // ------------------------------------------------------------ epilogue
    if (ok && warp_wait(acc_bar, 0, abort_flag, p.err, kErrWaitAcc)) {
      tc_fence_after();
      tile_epilogue<kStrassen, kEpi, kOutF32, kOpts>(p, tmem_base, t0, u0, warp, lane, smem, qss_bar,
                                                     abort_flag);
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (lane == 0) mbar_wait_drain(acc_bar, 0);  // every issued MMA has retired
    __syncwarp();
    tmem_dealloc<kTmemCols>(tmem_base);
  }
}

// The two-CTA product-split kernel (sb_strassen_gemm_pair).
#include "strassen_pair.cuh"
// The four-CTA kernel on CTA pairs (sb_strassen_gemm_quad).
#include "strassen_quad.cuh"
// Seven full-width product GEMMs on CTA pairs (sb_strassen_gemm_planes).
#include "strassen_planes.cuh"

// Failure-detection self-test (sb_wait_selftest): warp 0 waits on a barrier
// nobody arrives on and gives up after the bounded-wait limit, raising the abort
// flag; warp 1 starts waiting on another such barrier half a limit later, so it
// leaves through the abort flag before its own limit.
__global__ void __launch_bounds__(64, 1) wait_selftest_kernel(int* err) {
  __shared__ uint64_t bars[2];
  __shared__ int abort_word;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bars[0]), 1);
    mbar_init(smem_addr(&bars[1]), 1);
    abort_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort_flag = &abort_word;
  if (threadIdx.x == 0) mbar_wait(smem_addr(&bars[0]), 0, abort_flag, err, kErrSelfTest);
  if (threadIdx.x == 32) {
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < kWaitTimeoutNs / 2) {
    }
    mbar_wait(smem_addr(&bars[1]), 0, abort_flag, err, kErrWaitRaw);
  }
  __syncthreads();
}

// Row pass of norm_residual_add (strassen_pallas.py:836-866): the GEMM has
// written fp32 pre-norm rows to `x`; one CTA normalises one row:
// out = bf16(x * rsqrt((sum(left^2) + sum(right^2)) / n + eps) * scale + residual).
//
// Block reduction of the two half-row sums; every thread receives both totals.
__device__ __forceinline__ float2 block_sum2(float sl, float sr) {
  __shared__ float red[2][32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sl += __shfl_xor_sync(0xffffffffu, sl, o);
    sr += __shfl_xor_sync(0xffffffffu, sr, o);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    red[0][w] = sl;
    red[1][w] = sr;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    sl = l < nw ? red[0][l] : 0.f;
    sr = l < nw ? red[1][l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sl += __shfl_xor_sync(0xffffffffu, sl, o);
      sr += __shfl_xor_sync(0xffffffffu, sr, o);
    }
    if (l == 0) {
      red[0][0] = sl;
      red[1][0] = sr;
    }
  }
  __syncthreads();
  return make_float2(red[0][0], red[1][0]);
}

// Eight consecutive values of a bf16 or fp32 vector as fp32 (16- or 32-byte loads).
__device__ __forceinline__ void load8_f32(const void* base, bool f32, int64_t off, float* f) {
  if (f32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
    const float4 u = q[0], v = q[1];
    f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
    f[4] = v.x; f[5] = v.y; f[6] = v.z; f[7] = v.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + off);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(h[j]);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
}

// Vector form: each thread keeps up to kChunks 8-wide pieces of the row in
// registers between the two passes (one read of `x`), with 32-byte fp32 and
// 16-byte bf16 loads and 16-byte bf16 stores.  Needs n % 16 == 0 (a piece never
// straddles the two halves), n <= 8 * 256 * kChunks, 16-byte aligned rows
// (x, residual, out and scale), launched with 256 threads.
template <int kChunks>
__global__ void __launch_bounds__(256) norm_residual_rows_kernel(
    const float* __restrict__ x, int64_t n, const void* __restrict__ scale, int scale_f32,
    const void* __restrict__ residual, int64_t ldr, int residual_f32, float eps,
    __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t row = blockIdx.x;
  const float* xr = x + row * n;
  const int pieces = (int)(n / 8), half = pieces / 2;
  float v[kChunks][8];
  float sl = 0.f, sr = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int p = threadIdx.x + c * 256;
    if (p < pieces) {
      load8_f32(xr, true, (int64_t)p * 8, v[c]);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[c][j] * v[c][j];
      if (p < half) sl += s; else sr += s;
    }
  }
  const float2 sums = block_sum2(sl, sr);
  const float recip = 1.0f / sqrtf((sums.x + sums.y) * (1.0f / (float)n) + eps);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int p = threadIdx.x + c * 256;
    if (p < pieces) {
      float sc[8], r[8], o[8];
      load8_f32(scale, scale_f32, (int64_t)p * 8, sc);
      load8_f32(residual, residual_f32, row * ldr + (int64_t)p * 8, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[c][j] * recip * sc[j] + r[j];
      *reinterpret_cast<uint4*>(out + row * ldo + (int64_t)p * 8) =
          make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                     pack_bf16x2(o[6], o[7]));
    }
  }
}

// Scalar form for rows the vector form cannot take (odd widths, unaligned
// residual or output rows, n above 8192): the same arithmetic, reading `x` twice.
__global__ void __launch_bounds__(256) norm_residual_rows_scalar_kernel(
    const float* __restrict__ x, int64_t n, const void* __restrict__ scale, int scale_f32,
    const void* __restrict__ residual, int64_t ldr, int residual_f32, float eps,
    __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t row = blockIdx.x;
  const float* xr = x + row * n;
  const int64_t half = n / 2;
  float sl = 0.f, sr = 0.f;
  for (int64_t i = threadIdx.x; i < half; i += blockDim.x) {
    const float a = xr[i], b = xr[half + i];
    sl += a * a;
    sr += b * b;
  }
  const float2 sums = block_sum2(sl, sr);
  const float recip = 1.0f / sqrtf((sums.x + sums.y) * (1.0f / (float)n) + eps);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float s = scale_f32 ? reinterpret_cast<const float*>(scale)[i]
                              : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(scale)[i]);
    const float r = residual_f32
                        ? reinterpret_cast<const float*>(residual)[row * ldr + i]
                        : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(residual)[row * ldr + i]);
    out[row * ldo + i] = __float2bfloat16_rn(xr[i] * recip * s + r);
  }
}

// norm_residual_add on the planes path in one pass over the products: one CTA
// per product row t, whose seven fp32 products give both of its output rows
// whole (bn == n: C row I*bm + r' = [C11 | C12], row + bm/2 = [C21 | C22]).
// Each thread recombines up to kChunks 8-column pieces in registers
// (C11 = M1 + M4 - M5 + M7, C12 = M3 + M5, C21 = M2 + M4, C22 = M1 - M2 + M3 + M6,
// the one-CTA kernel's order), the block reduces both rows' sums of squares,
// and the normalised rows plus the residual are stored as bf16
// (strassen_pallas.py:836-866).  No fp32 pre-norm row goes to memory.  Needs
// nh = N/2 <= 8 * 256 * kChunks and 16-byte aligned residual, scale and C rows.
template <int kChunks>
__global__ void __launch_bounds__(256) planes_norm_rows_kernel(const float* __restrict__ prod, int32_t mh, int32_t nh,
                                                               int32_t bm, const void* __restrict__ scale,
                                                               int scale_f32, const void* __restrict__ residual,
                                                               int64_t ldr, int residual_f32, float eps,
                                                               __nv_bfloat16* __restrict__ out, int64_t ldo,
                                                               int64_t t0) {
  const int64_t t = t0 + blockIdx.x;
  const int64_t plane = (int64_t)mh * nh;
  const int64_t hbm = bm / 2;
  const int64_t blk = t / hbm;
  const int64_t row_top = blk * bm + (t - blk * hbm), row_bot = row_top + hbm;
  const int pieces = nh / 8;
  float q[kChunks][4][8];
  float s_top = 0.f, s_bot = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int pc = threadIdx.x + c * 256;
    if (pc < pieces) {
      float mv[7][8];
#pragma unroll
      for (int i = 0; i < 7; ++i) load8_f32(prod + i * plane, true, t * nh + 8 * (int64_t)pc, mv[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        q[c][0][e] = ((mv[0][e] + mv[3][e]) - mv[4][e]) + mv[6][e];
        q[c][1][e] = mv[2][e] + mv[4][e];
        q[c][2][e] = mv[1][e] + mv[3][e];
        q[c][3][e] = ((mv[0][e] - mv[1][e]) + mv[2][e]) + mv[5][e];
        s_top += q[c][0][e] * q[c][0][e] + q[c][1][e] * q[c][1][e];
        s_bot += q[c][2][e] * q[c][2][e] + q[c][3][e] * q[c][3][e];
      }
    }
  }
  const float2 sums = block_sum2(s_top, s_bot);
  const float inv_n = 1.0f / (2.0f * (float)nh);
  const float rt = 1.0f / sqrtf(sums.x * inv_n + eps), rb = 1.0f / sqrtf(sums.y * inv_n + eps);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int pc = threadIdx.x + c * 256;
    if (pc < pieces) {
      const int64_t cl = 8 * (int64_t)pc, cr = cl + nh;
      float sl[8], sr[8], r[8], o[8];
      load8_f32(scale, scale_f32, cl, sl);
      load8_f32(scale, scale_f32, cr, sr);
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        const int64_t row = qd < 2 ? row_top : row_bot;
        const int64_t col = (qd & 1) ? cr : cl;
        const float rec = qd < 2 ? rt : rb;
        load8_f32(residual, residual_f32, row * ldr + col, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = q[c][qd][e] * rec * ((qd & 1) ? sr[e] : sl[e]) + r[e];
        *reinterpret_cast<uint4*>(out + row * ldo + col) =
            make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                       pack_bf16x2(o[6], o[7]));
      }
    }
  }
}

// Standalone RMSNorm (experiments/qwen3/benchmark_qwen3_32b_layer.py:270-276):
// y = bf16(x * rsqrt(mean(x^2) + eps) * w), fp32 math.  One CTA per row,
// 16-byte vector loads.
__global__ void __launch_bounds__(256) rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const void* __restrict__ w, int w_f32,
                                                       __nv_bfloat16* __restrict__ y, int64_t n,
                                                       float eps) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * n;
  float ss = 0.f;
  const int64_t nvec = n / 8;
  for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 u = reinterpret_cast<const uint4*>(xr)[v];
    const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(hp[i]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int wi = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[wi] = ss;
  __syncthreads();
  if (wi == 0) {
    ss = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (l == 0) red[0] = ss;
  }
  __syncthreads();
  const float recip = 1.0f / sqrtf(red[0] / (float)n + eps);
  for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 u = reinterpret_cast<const uint4*>(xr)[v];
    const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&u);
    float o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(hp[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t c = v * 8 + i;
      const float wv = w_f32 ? reinterpret_cast<const float*>(w)[c]
                             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[c]);
      o[i] = (o[i] * recip) * wv;
    }
    uint4 r = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                         pack_bf16x2(o[6], o[7]));
    reinterpret_cast<uint4*>(y + row * n)[v] = r;
  }
}

// ====================================================================== host
namespace {

thread_local std::string t_last_error;

int fail(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }
bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

template <bool kStrassen, int kEpi, bool kOutF32, int kOpts, bool kATrans = false>
int launch_typed(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tb,
                 const GemmParams& p) {
  auto kernel = strassen_gemm_kernel<kStrassen, kEpi, kOutF32, kOpts, kATrans>;
  constexpr int kSmem = PipeFor<kStrassen, uses_tmem_a<kStrassen, kOpts, kATrans>()>::SMEM;
  // The attribute is per device: set it once for each device this kernel runs on.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(SB_ERR_DEVICE, "no usable current device");
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev], [&]() {
    attr_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (attr_err[dev] != cudaSuccess)
    return fail(SB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(attr_err[dev]));
  const unsigned grid = (unsigned)(p.tiles_m * p.tiles_n);
  kernel<<<grid, kThreads, kSmem, stream>>>(ta, tb, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

template <int kOpts>
int dispatch_strassen(int epi, bool out_f32, cudaStream_t stream, const CUtensorMap& ta,
                      const CUtensorMap& tb, const GemmParams& p) {
  switch (epi) {
    case SB_EPI_NONE:
      return out_f32 ? launch_typed<true, SB_EPI_NONE, true, kOpts>(stream, ta, tb, p)
                     : launch_typed<true, SB_EPI_NONE, false, kOpts>(stream, ta, tb, p);
    case SB_EPI_SWIGLU: return launch_typed<true, SB_EPI_SWIGLU, false, kOpts>(stream, ta, tb, p);
    case SB_EPI_GEGLU: return launch_typed<true, SB_EPI_GEGLU, false, kOpts>(stream, ta, tb, p);
    case SB_EPI_RESIDUAL_ADD:
      return launch_typed<true, SB_EPI_RESIDUAL_ADD, false, kOpts>(stream, ta, tb, p);
    case SB_EPI_BIAS_ADD: return launch_typed<true, SB_EPI_BIAS_ADD, false, kOpts>(stream, ta, tb, p);
    case SB_EPI_QK_NORM_ROPE:
      return launch_typed<true, SB_EPI_QK_NORM_ROPE, false, kOpts>(stream, ta, tb, p);
    default: return fail(SB_ERR_EPILOGUE, "unknown epilogue kind");
  }
}

int dispatch(bool strassen, int epi, bool out_f32, cudaStream_t stream, const CUtensorMap& ta,
             const CUtensorMap& tb, const GemmParams& p) {
  if (!strassen) {
    return out_f32 ? launch_typed<false, SB_EPI_NONE, true, false>(stream, ta, tb, p)
                   : launch_typed<false, SB_EPI_NONE, false, false>(stream, ta, tb, p);
  }
  const bool opts = p.formula != 0 || p.swap_m || p.swap_k || p.swap_n || p.panel_schedule;
  if (!opts) return dispatch_strassen<0>(epi, out_f32, stream, ta, tb, p);
  switch (p.formula) {
    case 0: return dispatch_strassen<1>(epi, out_f32, stream, ta, tb, p);
    case 1: return dispatch_strassen<2>(epi, out_f32, stream, ta, tb, p);
    default: return dispatch_strassen<3>(epi, out_f32, stream, ta, tb, p);
  }
}

// Device address of g_device_error in the current context, resolved by
// check_device() on every call (so a cudaDeviceReset or a new primary context
// never leaves a stale pointer) and read by base_params() on the same host
// thread.
thread_local int* t_error_word = nullptr;

// Checks that the current device is an sm_100 part (the compute capability is
// cached per device) and resolves the address of the bounded-wait error word
// the kernels write to.
int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  static int cached_major[64];
  static int cached_minor[64];
  static std::once_flag flags[64];
  if (dev < 0 || dev >= 64) return fail(SB_ERR_DEVICE, "device ordinal out of range");
  std::call_once(flags[dev], [&]() {
    cudaDeviceGetAttribute(&cached_major[dev], cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&cached_minor[dev], cudaDevAttrComputeCapabilityMinor, dev);
  });
  if (cached_major[dev] != 10 || cached_minor[dev] != 0)
    return fail(SB_ERR_DEVICE, "the Strassen kernel is built for sm_100a (B200); device is sm_" +
                                   std::to_string(cached_major[dev]) + std::to_string(cached_minor[dev]));
  void* addr = nullptr;
  e = cudaGetSymbolAddress(&addr, g_device_error);
  if (e != cudaSuccess || addr == nullptr) {
    t_error_word = nullptr;
    return fail(SB_ERR_CUDA, std::string("cudaGetSymbolAddress(device error word): ") + cudaGetErrorString(e));
  }
  t_error_word = static_cast<int*>(addr);
  return SB_OK;
}

// Validation shared by the Strassen and classical entry points; mirrors the
// reference's host-side checks (strassen_pallas.py:927-1047, :127-140).
int validate_core(const void* a, const void* b, const void* c, int64_t m, int64_t n, int64_t k,
                  int64_t lda, int64_t ldb, int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
                  int32_t out_dtype, int32_t bn_align = 256) {
  if (!a || !b || !c) return fail(SB_ERR_RANK, "null matrix pointer");
  if (m <= 0 || n <= 0 || k <= 0) return fail(SB_ERR_RANK, "matrix dimensions must be positive");
  if (bm <= 0 || bn <= 0 || bk <= 0) return fail(SB_ERR_TILING, "tile sizes must be positive");
  const char* names[3] = {"M", "N", "K"};
  const int64_t dims[3] = {m, n, k};
  const int32_t blocks[3] = {bm, bn, bk};
  for (int i = 0; i < 3; ++i) {
    if (dims[i] % blocks[i])
      return fail(SB_ERR_DIVISIBILITY, std::string(names[i]) + "=" + std::to_string(dims[i]) +
                                           " is not divisible by " + std::to_string(blocks[i]));
  }
  std::string tiling;
  if (bm % 16) tiling += "\n  bm=" + std::to_string(bm) + " must be a multiple of 16";
  if (bn % bn_align) tiling += "\n  bn=" + std::to_string(bn) + " must be a multiple of " + std::to_string(bn_align);
  if (bk % 256) tiling += "\n  bk=" + std::to_string(bk) + " must be a multiple of 256";
  if (!tiling.empty()) return fail(SB_ERR_TILING, "tile breaks TPU v5e alignment:" + tiling);
  if (out_dtype != SB_BF16 && out_dtype != SB_F32)
    return fail(SB_ERR_OUTPUT_DTYPE, "output_dtype must be BF16 or FP32");
  const int half_bm = bm / 2;
  if (!(half_bm % kBlockM == 0 || (is_pow2(half_bm) && half_bm < kBlockM)))
    return fail(SB_ERR_UNSUPPORTED,
                "bm=" + std::to_string(bm) +
                    ": the B200 kernel needs bm/2 to be a multiple of 128 or a power of two below 128");
  if (m > (int64_t)INT32_MAX || n > (int64_t)INT32_MAX || k > (int64_t)INT32_MAX)
    return fail(SB_ERR_UNSUPPORTED, "dimensions above 2^31-1 are not supported");
  if (!aligned16(a) || !aligned16(b) || !aligned16(c))
    return fail(SB_ERR_ALIGNMENT, "A, B and C must be 16-byte aligned");
  if (lda % 8 || ldb % 8 || ldc % 8 || lda < k || ldb < n)
    return fail(SB_ERR_ALIGNMENT,
                "leading dimensions must be multiples of 8 elements and cover the rows");
  return SB_OK;
}

int make_maps(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int64_t lda,
              int64_t ldb, int32_t bm, int bk_chunk, CUtensorMap* ta, CUtensorMap* tb) {
  const int a_row_bytes = bk_chunk * 2;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int half_bm = bm / 2;
  const uint32_t rows = half_bm >= kBlockM ? kBlockM : half_bm;
  const uint32_t blocks = half_bm >= kBlockM ? 1 : kBlockM / half_bm;
  {
    // A viewed as [M/bm][bm][K]; a box is kBlockK columns of `rows` rows in each
    // of `blocks` consecutive Strassen blocks = one 128-row product tile.
    cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)bm, (cuuint64_t)(m / bm)};
    cuuint64_t strides[2] = {(cuuint64_t)lda * 2, (cuuint64_t)lda * 2 * bm};
    cuuint32_t box[3] = {(cuuint32_t)bk_chunk, rows, blocks};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(a), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     a_row_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                     : a_row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled(A) failed: " + std::to_string((int)r));
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)k};
    cuuint64_t strides[1] = {(cuuint64_t)ldb * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBlockN, (cuuint32_t)bk_chunk};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(b), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled(B) failed: " + std::to_string((int)r));
  }
  return SB_OK;
}

// Row pass of norm_residual_add over M rows of fp32 pre-norm values `x` [M, n]:
// the register-resident vector kernel when the row fits 8 * 256 * 4 values and
// every row start is 16-byte aligned, else the scalar kernel.
int launch_norm_rows(cudaStream_t stream, const float* x, int64_t m, int64_t n, const sb_epilogue* ep,
                     __nv_bfloat16* c, int64_t ldc) {
  const bool res_f32 = ep->residual_dtype == SB_F32, scale_f32 = ep->aux_dtype == SB_F32;
  const int64_t pieces = n / 8;
  const bool vec = n % 16 == 0 && pieces <= 4 * 256 && aligned16(x) && aligned16(c) && ldc % 8 == 0 &&
                   aligned16(ep->norm_scale) && aligned16(ep->residual) &&
                   ep->ld_residual % (res_f32 ? 4 : 8) == 0;
  const int chunks = (int)((pieces + 255) / 256);
  auto args = [&](auto kernel) {
    kernel<<<(unsigned)m, 256, 0, stream>>>(x, n, ep->norm_scale, scale_f32, ep->residual, ep->ld_residual,
                                            res_f32, ep->norm_eps, c, ldc);
  };
  if (!vec) args(norm_residual_rows_scalar_kernel);
  else if (chunks <= 1) args(norm_residual_rows_kernel<1>);
  else if (chunks == 2) args(norm_residual_rows_kernel<2>);
  else if (chunks == 3) args(norm_residual_rows_kernel<3>);
  else args(norm_residual_rows_kernel<4>);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("norm rows launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

// Tensor maps of the TMEM-ring Strassen kernel: one TMA copy per operand and
// K step.  The quadrant offsets become tensor dimensions (strides need not
// grow with the dimension index), ordered so the copy lays the four quadrant
// tiles out contiguously in slot order:
//   A: dims (k, row in half-block, block, qk, qr), strides (1, lda, bm*lda,
//      half_bk, half_bm*lda) elements; box {16, rows, blocks, 2, 2} -> slot
//      2*qr + qk, each tile `blocks` x `rows` = 128 rows of 16 columns.
//   B: dims (n, k, qc, qk), strides (1, ldb, half_bn, half_bk*ldb); box
//      {64, 16, 2, 2} -> slot 2*qk + qc, each 16 rows of 64 columns.
int make_ts_maps(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int64_t lda,
                 int64_t ldb, int32_t bm, int32_t bn, int32_t bk, CUtensorMap* ta, CUtensorMap* tb) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t half_bm = bm / 2, half_bn = bn / 2, half_bk = bk / 2;
  const uint32_t rows = half_bm >= kBlockM ? kBlockM : (uint32_t)half_bm;
  const uint32_t blocks = half_bm >= kBlockM ? 1 : (uint32_t)(kBlockM / half_bm);
  {
    cuuint64_t dims[5] = {(cuuint64_t)k, (cuuint64_t)half_bm, (cuuint64_t)(m / bm), 2, 2};
    cuuint64_t strides[4] = {(cuuint64_t)(lda * 2), (cuuint64_t)(bm * lda * 2), (cuuint64_t)(half_bk * 2),
                             (cuuint64_t)(half_bm * lda * 2)};
    cuuint32_t box[5] = {16, rows, blocks, 2, 2};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = enc(ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(a), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_32B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled(A, 5-D) failed: " + std::to_string((int)r));
  }
  {
    cuuint64_t dims[4] = {(cuuint64_t)n, (cuuint64_t)k, 2, 2};
    cuuint64_t strides[3] = {(cuuint64_t)(ldb * 2), (cuuint64_t)(half_bn * 2), (cuuint64_t)(half_bk * ldb * 2)};
    cuuint32_t box[4] = {(cuuint32_t)kBlockN, 16, 2, 2};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(b), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled(B, 4-D) failed: " + std::to_string((int)r));
  }
  return SB_OK;
}

// Tensor maps for a Strassen launch: the default kernel's (make_ts_maps) unless
// research options select the 16-wide-chunk kernel.
int make_strassen_maps(bool options, const void* a, const void* b, int64_t m, int64_t n, int64_t k,
                       int64_t lda, int64_t ldb, int32_t bm, int32_t bn, int32_t bk, CUtensorMap* ta,
                       CUtensorMap* tb) {
  (void)options;
  if (SB_TMEM_A) return make_ts_maps(a, b, m, n, k, lda, ldb, bm, bn, bk, ta, tb);
  return make_maps(a, b, m, n, k, lda, ldb, bm, StrassenPipe::BK, ta, tb);
}

GemmParams base_params(int64_t m, int64_t n, int64_t k, int32_t bm, int32_t bn, int32_t bk, void* c,
                       int64_t ldc, int bk_chunk) {
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = (int32_t)m;
  p.N = (int32_t)n;
  p.K = (int32_t)k;
  p.bm = bm;
  p.bn = bn;
  p.bk = bk;
  p.half_bm = bm / 2;
  p.half_bn = bn / 2;
  p.half_bk = bk / 2;
  p.Mp = (int32_t)(m / 2);
  p.Np = (int32_t)(n / 2);
  p.num_chunks = (int32_t)(k / 2 / bk_chunk);
  p.tiles_m = (p.Mp + kBlockM - 1) / kBlockM;
  p.tiles_n = p.Np / kBlockN;
  p.C = c;
  p.ldc = ldc;
  p.eps = 1e-6f;
  p.half_head = 64;
  p.inv_head_dim = 1.0f / 128.0f;
  // check_device(), called first by every entry point on this thread, has
  // resolved the error word of the current context.
  p.err = t_error_word;
  return p;
}

// Tensor maps of the two-CTA kernel (strassen_pair.cuh); KD = the stage depth
// of the mode (16 for raw B, pair::Geo<true>::KD for the planes).  Both B
// modes share the two A maps:
//   a:  dims (k, row in half-block, block, qk, qr) as make_ts_maps; box
//       {KD, rows, blocks, 2, 1} -> quadrants (r, 0), (r, 1) at qr = r
//       (KD = 16: 32-byte rows, 32-byte swizzle; KD = 32: 64-byte rows and swizzle);
//   a1: the same dims, box {KD, rows, blocks, 1, 1} -> one quadrant.
// Raw B (b_planes == nullptr): dims (column in a 64-column chunk, k, chunk,
// qc, qk), strides (1, ldb, 64, half_bn, half_bk*ldb) elements;
//   b:  box {64, 16, 2, 1, 2} -> quadrants (0, qc), (1, qc), 16 x 128 each;
//   b1: box {64, 16, 2, 1, 1} -> one 16 x 128 quadrant;
//   bh: box {64, 16, 1, 1, 1} -> one 64-column chunk of a quadrant.
// B operand planes ([7][K/2][N/2], from b_operand_planes_kernel): dims
// (column in a chunk, kappa, chunk, plane);
//   b:  box {64, KD, 2, 3} -> three planes of KD x 128;  bh: box {64, KD, 1, 1}.
struct PairMaps {
  CUtensorMap a, a1, b, b1, bh;
};

int make_pair_maps(const void* a, const void* b, const void* b_planes, int64_t m, int64_t n, int64_t k,
                   int64_t lda, int64_t ldb, int32_t bm, int32_t bn, int32_t bk, PairMaps* maps) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t half_bm = bm / 2, half_bn = bn / 2, half_bk = bk / 2;
  const uint32_t rows = half_bm >= kBlockM ? kBlockM : (uint32_t)half_bm;
  const uint32_t blocks = half_bm >= kBlockM ? 1 : (uint32_t)(kBlockM / half_bm);
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const uint32_t kd = b_planes ? (uint32_t)pair::Geo<true>::KD : 16u;
  const CUtensorMapSwizzle a_sw = kd == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
  auto encode = [&](CUtensorMap* map, const void* base, cuuint32_t rank, const cuuint64_t* dims,
                    const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw,
                    const char* what) -> int {
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(SB_ERR_CUDA, std::string("cuTensorMapEncodeTiled(") + what + ") failed: " + std::to_string((int)r));
    return SB_OK;
  };
  {
    cuuint64_t dims[5] = {(cuuint64_t)k, (cuuint64_t)half_bm, (cuuint64_t)(m / bm), 2, 2};
    cuuint64_t strides[4] = {(cuuint64_t)(lda * 2), (cuuint64_t)(bm * lda * 2), (cuuint64_t)(half_bk * 2),
                             (cuuint64_t)(half_bm * lda * 2)};
    cuuint32_t box[5] = {kd, rows, blocks, 2, 1};
    int st = encode(&maps->a, a, 5, dims, strides, box, a_sw, "A, pair");
    if (st != SB_OK) return st;
    box[3] = 1;
    st = encode(&maps->a1, a, 5, dims, strides, box, a_sw, "A, one quadrant");
    if (st != SB_OK) return st;
  }
  if (b_planes == nullptr) {
    cuuint64_t dims[5] = {64, (cuuint64_t)k, (cuuint64_t)(n / 64), 2, 2};
    cuuint64_t strides[4] = {(cuuint64_t)(ldb * 2), 128, (cuuint64_t)(half_bn * 2), (cuuint64_t)(half_bk * ldb * 2)};
    cuuint32_t box[5] = {64, 16, 2, 1, 2};
    int st = encode(&maps->b, b, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "B, pair");
    if (st != SB_OK) return st;
    box[4] = 1;
    st = encode(&maps->b1, b, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "B, one quadrant");
    if (st != SB_OK) return st;
    box[2] = 1;
    return encode(&maps->bh, b, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "B, half quadrant");
  }
  const int64_t kh = k / 2, nh = n / 2;
  cuuint64_t dims[4] = {64, (cuuint64_t)kh, (cuuint64_t)(nh / 64), 7};
  cuuint64_t strides[3] = {(cuuint64_t)(nh * 2), 128, (cuuint64_t)(kh * nh * 2)};
  cuuint32_t box[4] = {64, kd, 2, 3};
  int st = encode(&maps->b, b_planes, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "B planes");
  if (st != SB_OK) return st;
  box[2] = 1;
  box[3] = 1;
  st = encode(&maps->bh, b_planes, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "B plane, half");
  if (st != SB_OK) return st;
  maps->b1 = maps->bh;  // unused with planes
  return SB_OK;
}

// Launches the two-CTA kernel: clusters of two consecutive CTAs, one cluster
// per 128 x 128 product tile.
template <bool kOutF32, bool kPreB>
int launch_pair(cudaStream_t stream, const PairMaps& m, const GemmParams& p) {
  auto kernel = strassen_pair_kernel<kOutF32, kPreB>;
  constexpr int kSmem = pair::Geo<kPreB>::SMEM;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(SB_ERR_DEVICE, "no usable current device");
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev], [&]() {
    attr_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (attr_err[dev] != cudaSuccess)
    return fail(SB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(attr_err[dev]));
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(2 * p.tiles_m * p.tiles_n), 1, 1);
  cfg.blockDim = dim3(pair::kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, m.a, m.a1, m.b, m.b1, m.bh, p);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("pair kernel launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

// Shared body of sb_strassen_gemm_pair (raw B) and sb_strassen_gemm_pair_planes.
int run_pair(cudaStream_t stream, const void* a, const void* b, const void* b_planes, void* c, int64_t m,
             int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
             int32_t out_dtype) {
  if (ldc < n) return fail(SB_ERR_ALIGNMENT, "ldc must be >= N");
  int st = check_device();
  if (st != SB_OK) return st;
  PairMaps maps;
  st = make_pair_maps(a, b, b_planes, m, n, k, lda, ldb, bm, bn, bk, &maps);
  if (st != SB_OK) return st;
  GemmParams p = base_params(m, n, k, bm, bn, bk, c, ldc, 16);
  p.tiles_n = p.Np / pair::kCols;  // bn % 256 == 0, so Np is a multiple of 128
  if (b_planes)
    return out_dtype == SB_F32 ? launch_pair<true, true>(stream, maps, p) : launch_pair<false, true>(stream, maps, p);
  return out_dtype == SB_F32 ? launch_pair<true, false>(stream, maps, p) : launch_pair<false, false>(stream, maps, p);
}

// Tensor maps of the four-CTA kernel (strassen_quad.cuh):
//   a:  the A operand array [M/2][4K] of a_operand_pass_kernel, 2-D, box {64, 128},
//       128-byte swizzle (one 128-byte row = a pair's four operands, 16 deep);
//   b:  the B operand planes [7][K/2][N/2] as dims (column in a 64-column
//       chunk, kappa, chunk, plane), box {64, 16, 1, 3}, 128-byte swizzle;
//   bh: the planes as dims (column, kappa, plane), box {32, 16, 1}, 64-byte
//       swizzle (a CTA's 32 columns of P1's half tile).
struct QuadMaps {
  CUtensorMap a, b, bh;
};

int make_quad_maps(const void* ops, const void* planes, int64_t m, int64_t n, int64_t k, QuadMaps* maps) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint32_t estr[4] = {1, 1, 1, 1};
  auto encode = [&](CUtensorMap* map, const void* base, cuuint32_t rank, const cuuint64_t* dims,
                    const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw,
                    const char* what) -> int {
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(SB_ERR_CUDA, std::string("cuTensorMapEncodeTiled(") + what + ") failed: " + std::to_string((int)r));
    return SB_OK;
  };
  const int64_t kh = k / 2, nh = n / 2;
  {
    cuuint64_t dims[2] = {(cuuint64_t)(4 * k), (cuuint64_t)(m / 2)};
    cuuint64_t strides[1] = {(cuuint64_t)(4 * k * 2)};
    cuuint32_t box[2] = {64, 128};
    int st = encode(&maps->a, ops, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "A operands, quad");
    if (st != SB_OK) return st;
  }
  {
    cuuint64_t dims[4] = {64, (cuuint64_t)kh, (cuuint64_t)(nh / 64), 7};
    cuuint64_t strides[3] = {(cuuint64_t)(nh * 2), 128, (cuuint64_t)(kh * nh * 2)};
    cuuint32_t box[4] = {64, 16, 1, 3};
    int st = encode(&maps->b, planes, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "B planes, quad");
    if (st != SB_OK) return st;
  }
  cuuint64_t dims[3] = {(cuuint64_t)nh, (cuuint64_t)kh, 7};
  cuuint64_t strides[2] = {(cuuint64_t)(nh * 2), (cuuint64_t)(kh * nh * 2)};
  cuuint32_t box[3] = {32, 16, 1};
  return encode(&maps->bh, planes, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B, "B plane half, quad");
}

// Launches the four-CTA kernel: clusters of four consecutive CTAs (two CTA
// pairs), one cluster per 256 x 128 product tile.
template <bool kOutF32>
int launch_quad(cudaStream_t stream, const QuadMaps& m, const GemmParams& p) {
  auto kernel = strassen_quad_kernel<kOutF32>;
  constexpr int kSmem = quad::Geo::SMEM;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(SB_ERR_DEVICE, "no usable current device");
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev], [&]() {
    attr_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (attr_err[dev] != cudaSuccess)
    return fail(SB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(attr_err[dev]));
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(4 * p.tiles_m * p.tiles_n), 1, 1);
  cfg.blockDim = dim3(quad::kThreadsQ, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 4;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, m.a, m.b, m.bh, p);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("quad kernel launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

// Bytes of the A operand array and of the B planes the four-CTA path forms.
size_t quad_ops_bytes(int64_t m, int64_t k) { return (size_t)(m / 2) * (size_t)(4 * k) * 2u; }
size_t quad_planes_bytes(int64_t k, int64_t n) { return (size_t)7 * (size_t)(k / 2) * (size_t)(n / 2) * 2u; }

// Shape rules of the four-CTA kernel beyond validate_core: 256-row product
// tiles (M % 512), 128-column product tiles inside one block half (bn % 256),
// the B planes' tile rule (bk % 256).
int check_quad_shape(int64_t m, int32_t bn, int32_t bk) {
  if (m % 512)
    return fail(SB_ERR_TILING, "the four-CTA kernel needs M divisible by 512 (256-row product tiles), got M=" +
                                   std::to_string(m));
  if (bn % 256 || bk % 256) return fail(SB_ERR_TILING, "the four-CTA kernel needs bn and bk multiples of 256");
  return SB_OK;
}

// A operand pass, B planes (unless given) and the GEMM, in stream order.
int run_quad(cudaStream_t stream, const void* a, const void* b, const void* b_planes, void* c, int64_t m,
             int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
             int32_t out_dtype, void* workspace, size_t workspace_bytes, int32_t raster) {
  if (ldc < n) return fail(SB_ERR_ALIGNMENT, "ldc must be >= N");
  if (raster < 0) return fail(SB_ERR_UNSUPPORTED, "raster must be >= 0 (0 = the kernel's default)");
  int st = check_quad_shape(m, bn, bk);
  if (st != SB_OK) return st;
  const size_t need = quad_ops_bytes(m, k) + (b_planes ? 0 : quad_planes_bytes(k, n));
  if (!workspace || workspace_bytes < need)
    return fail(SB_ERR_WORKSPACE, "the four-CTA path needs a workspace of " + std::to_string(need) +
                                      " bytes (sb_quad_workspace_bytes), got " + std::to_string(workspace_bytes));
  if (!aligned16(workspace)) return fail(SB_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  st = check_device();
  if (st != SB_OK) return st;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* ops = reinterpret_cast<__nv_bfloat16*>(ws);
  const void* planes = b_planes;
  if (!planes) {
    void* pl = ws + quad_ops_bytes(m, k);
    st = sb_strassen_b_operands(reinterpret_cast<sb_stream_t>(stream), b, pl, k, n, ldb, bn, bk);
    if (st != SB_OK) return st;
    planes = pl;
  }
  const int64_t items = (m / 2) * (k / 16);
  const unsigned grid = (unsigned)std::min<int64_t>((items + 255) / 256, 148 * 16);
  a_operand_pass_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(a), lda, (int32_t)m,
                                                  (int32_t)k, bm, bk, ops);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("A operand pass launch: ") + cudaGetErrorString(e));
  QuadMaps maps;
  st = make_quad_maps(ops, planes, m, n, k, &maps);
  if (st != SB_OK) return st;
  GemmParams p = base_params(m, n, k, bm, bn, bk, c, ldc, 16);
  p.tiles_m = (int32_t)(p.Mp / quad::kTileRows);
  p.tiles_n = (int32_t)(p.Np / quad::kCols);
  p.raster = raster;
  return out_dtype == SB_F32 ? launch_quad<true>(stream, maps, p) : launch_quad<false>(stream, maps, p);
}

// ---------------------------------------------------------------- planes path
// Workspace of sb_strassen_gemm_planes: A operand planes [7][M/2][K/2] bf16,
// B operand planes [7][K/2][N/2] bf16, products [7][M/2][N/2] fp32.
size_t planes_a_bytes(int64_t m, int64_t k) { return (size_t)7 * (size_t)(m / 2) * (size_t)(k / 2) * 2u; }
size_t planes_prod_bytes(int64_t m, int64_t n) { return (size_t)7 * (size_t)(m / 2) * (size_t)(n / 2) * 4u; }

// Tensor maps of the product GEMM:
//   a: A operand planes as dims (kappa, t, plane), box {64, 128, 1}, 128-byte
//      swizzle (a CTA's 128 product rows, 64 deep);
//   b: B operand planes as dims (column in a 64-column chunk, kappa, chunk,
//      plane), box {64, 64, 2, 1}, 128-byte swizzle (a CTA's 128 columns as two
//      MN-major chunks, 64 deep).
int make_planes_maps(const void* aop, const void* bop, int64_t m, int64_t n, int64_t k, CUtensorMap* ta,
                     CUtensorMap* tb) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t mh = m / 2, nh = n / 2, kh = k / 2;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  {
    cuuint64_t dims[3] = {(cuuint64_t)kh, (cuuint64_t)mh, 7};
    cuuint64_t strides[2] = {(cuuint64_t)(kh * 2), (cuuint64_t)(mh * kh * 2)};
    cuuint32_t box[3] = {(cuuint32_t)planes::kBK, 128, 1};
    CUresult r = enc(ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(aop), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled(A planes) failed: " + std::to_string((int)r));
  }
  cuuint64_t dims[4] = {64, (cuuint64_t)kh, (cuuint64_t)(nh / 64), 7};
  cuuint64_t strides[3] = {(cuuint64_t)(nh * 2), 128, (cuuint64_t)(kh * nh * 2)};
  cuuint32_t box[4] = {64, (cuuint32_t)planes::kBK, 2, 1};
  CUresult r = enc(tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(bop), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled(B planes) failed: " + std::to_string((int)r));
  return SB_OK;
}

size_t planes_workspace(int64_t m, int64_t n, int64_t k) {
  return planes_a_bytes(m, k) + quad_planes_bytes(k, n) + planes_prod_bytes(m, n);
}

// Shapes the planes path takes (256 x 256 product tiles, 64-deep steps, at
// least two tiles per CTA pair of a B200) and where it is expected to beat the
// one-CTA kernel.  The estimate uses rates measured on B200: the product GEMM
// runs 1.36 PFLOP/s of raw tensor work, the one-CTA kernel 0.67, and the extra
// passes move their bytes at 6 TB/s -- operand planes (7/4 of A and of B
// written, A and B read), the fp32 products written and read back, C written.
// Small K loses: at 8192 x 4096 x 512 the products' round trip (0.47 GB) costs
// twice the one-CTA kernel's whole GEMM.
bool planes_preferred(int64_t m, int64_t n, int64_t k) {
  if (m % 512 || n % 512 || k % 128 || 7 * (m / 512) * (n / 512) < 148) return false;
  const double md = (double)m, nd = (double)n, kd = (double)k;
  const double raw_flops = 1.75 * md * nd * kd;
  const double bytes = 2.75 * 2.0 * (md * kd + kd * nd) + 7.0 * (md / 2) * (nd / 2) * 8.0 + md * nd * 2.0;
  const double t_planes = raw_flops / 1.36e15 + bytes / 6.0e12;
  const double t_one_cta = raw_flops / 0.67e15;
  return t_planes < 0.9 * t_one_cta;
}

// The fused epilogue's operands, as both GEMM layouts read them.
void fill_epilogue(GemmParams& p, const sb_epilogue* ep, int epi) {
  if (!ep) return;
  p.residual = ep->residual;
  p.ldr = ep->ld_residual;
  p.residual_f32 = ep->residual_dtype == SB_F32;
  p.aux_f32 = ep->aux_dtype == SB_F32;
  p.bias = ep->bias;
  p.rope_cos = ep->rope_cos;
  p.rope_sin = ep->rope_sin;
  p.ld_rope = ep->ld_rope;
  p.rope_scale = ep->rope_scale;
  if (epi == SB_EPI_QK_NORM_ROPE) {
    p.half_head = ep->rope_head_dim / 2;
    p.inv_head_dim = 1.0f / (float)ep->rope_head_dim;
    p.eps = ep->rope_eps;
  }
}

// Epilogues the planes path applies in its recombination pass.
bool planes_epilogue(int epi) {
  return epi == SB_EPI_NONE || epi == SB_EPI_RESIDUAL_ADD || epi == SB_EPI_BIAS_ADD || epi == SB_EPI_SWIGLU ||
         epi == SB_EPI_GEGLU || epi == SB_EPI_QK_NORM_ROPE || epi == SB_EPI_NORM_RESIDUAL_ADD;
}

// norm_residual_add on the planes path keeps a row's pieces in registers:
// N/2 <= 8 * 256 * 2 (planes_norm_rows_kernel<2>).
constexpr int64_t kPlanesNormMaxN = 2 * 8 * 256 * 2;

// Persistent launch: one cluster (CTA pair) per two SMs, each walking its tiles.
int launch_planes_gemm(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tb, const PlanesParams& p) {
  auto kernel = strassen_planes_gemm_kernel;
  constexpr int kSmem = planes::kSmem;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(SB_ERR_DEVICE, "no usable current device");
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  static int sms[64];
  std::call_once(once[dev], [&]() {
    attr_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  });
  if (attr_err[dev] != cudaSuccess)
    return fail(SB_ERR_CUDA, std::string("planes kernel setup: ") + cudaGetErrorString(attr_err[dev]));
  const int clusters = std::max(1, std::min(sms[dev] / 2, p.num_tiles));
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  cfg.blockDim = dim3(planes::kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, p);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("planes kernel launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

// One row range [t0, t1) of product rows (multiples of 256) through one step
// of the planes path, on `stream`.
int planes_a_pass(cudaStream_t stream, const void* a, int64_t lda, int64_t m, int64_t k, int32_t bm, int32_t bk,
                  __nv_bfloat16* aop, int64_t t0, int64_t t1) {
  const int64_t items = (t1 - t0) * (k / 2 / 8);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, 148 * 16));
  a_operand_planes_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(a), lda, (int32_t)m,
                                                    (int32_t)k, bm, bk, aop, t0, t1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("A planes launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

int planes_gemm(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tb, int64_t m, int64_t n, int64_t k,
                int32_t raster, float* prod, int64_t t0, int64_t t1) {
  PlanesParams p;
  std::memset(&p, 0, sizeof(p));
  p.mh = (int32_t)(m / 2);
  p.nh = (int32_t)(n / 2);
  p.kh = (int32_t)(k / 2);
  p.tile_m0 = (int32_t)(t0 / planes::kTileM);
  p.tiles_m = (int32_t)((t1 - t0) / planes::kTileM);
  p.tiles_n = p.nh / planes::kTileN;
  p.num_tiles = 7 * p.tiles_m * p.tiles_n;
  p.k_steps = p.kh / planes::kBK;
  p.raster = raster;
  p.prod = prod;
  p.err = t_error_word;
  return launch_planes_gemm(stream, ta, tb, p);
}

int planes_recombine(cudaStream_t stream, const float* prod, int64_t m, int64_t n, int64_t k, int32_t bm, int32_t bn,
                     int32_t bk, void* c, int64_t ldc, int32_t out_dtype, int epi, const sb_epilogue* ep, int64_t t0,
                     int64_t t1) {
  const int32_t mh = (int32_t)(m / 2), nh = (int32_t)(n / 2);
  const int64_t items = (t1 - t0) * (nh / 8);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, 148 * 16));
  GemmParams ep_p = base_params(m, n, k, bm, bn, bk, c, ldc, 16);
  fill_epilogue(ep_p, ep, epi);
  if (epi == SB_EPI_NORM_RESIDUAL_ADD) {
    const bool vec = aligned16(ep->norm_scale) && aligned16(ep->residual) && aligned16(c) && ldc % 8 == 0 &&
                     ep->ld_residual % (ep->residual_dtype == SB_F32 ? 4 : 8) == 0;
    if (!vec || n > kPlanesNormMaxN)
      return fail(SB_ERR_ALIGNMENT, "norm_residual_add on the planes path needs N <= 8192 and 16-byte aligned "
                                    "scale, residual and output rows");
    auto kernel = (nh / 8 <= 256) ? planes_norm_rows_kernel<1> : planes_norm_rows_kernel<2>;
    kernel<<<(unsigned)(t1 - t0), 256, 0, stream>>>(prod, mh, nh, bm, ep->norm_scale, ep->aux_dtype == SB_F32,
                                                    ep->residual, ep->ld_residual, ep->residual_dtype == SB_F32,
                                                    ep->norm_eps, reinterpret_cast<__nv_bfloat16*>(c), ldc, t0);
  } else {
    switch (epi) {
      case SB_EPI_RESIDUAL_ADD:
        planes_recombine_kernel<SB_EPI_RESIDUAL_ADD, false><<<grid, 256, 0, stream>>>(prod, mh, nh, ep_p, t0, t1);
        break;
      case SB_EPI_BIAS_ADD:
        planes_recombine_kernel<SB_EPI_BIAS_ADD, false><<<grid, 256, 0, stream>>>(prod, mh, nh, ep_p, t0, t1);
        break;
      case SB_EPI_SWIGLU:
        planes_recombine_kernel<SB_EPI_SWIGLU, false><<<grid, 256, 0, stream>>>(prod, mh, nh, ep_p, t0, t1);
        break;
      case SB_EPI_GEGLU:
        planes_recombine_kernel<SB_EPI_GEGLU, false><<<grid, 256, 0, stream>>>(prod, mh, nh, ep_p, t0, t1);
        break;
      case SB_EPI_QK_NORM_ROPE:
        planes_recombine_kernel<SB_EPI_QK_NORM_ROPE, false><<<grid, 256, 0, stream>>>(prod, mh, nh, ep_p, t0, t1);
        break;
      default:
        if (out_dtype == SB_F32)
          planes_recombine_kernel<SB_EPI_NONE, true><<<grid, 256, 0, stream>>>(prod, mh, nh, ep_p, t0, t1);
        else
          planes_recombine_kernel<SB_EPI_NONE, false><<<grid, 256, 0, stream>>>(prod, mh, nh, ep_p, t0, t1);
    }
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("recombination launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

// A second stream and fork/join events per device and host thread, created on
// first use and kept for the thread's life (not destroyed at thread exit, where
// the CUDA runtime may already be shutting down): the planes path runs its
// second row half there.
struct PlanesSide {
  cudaStream_t aux = nullptr;
  cudaEvent_t fork = nullptr, b_done = nullptr, join = nullptr;
};

// *out stays null (the caller runs the halves in sequence) when the side
// stream does not exist yet and `stream` is being captured into a CUDA graph,
// where creating streams and events may be refused.
int planes_side(cudaStream_t stream, PlanesSide** out) {
  *out = nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(SB_ERR_DEVICE, "no usable current device");
  thread_local PlanesSide side[64];
  PlanesSide& s = side[dev];
  if (!s.aux) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return SB_OK;
    cudaError_t e = cudaStreamCreateWithFlags(&s.aux, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.b_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      // Release whatever was created so the next call starts from scratch.
      for (cudaEvent_t* ev : {&s.fork, &s.b_done, &s.join}) {
        if (*ev) cudaEventDestroy(*ev);
        *ev = nullptr;
      }
      if (s.aux) cudaStreamDestroy(s.aux);
      s.aux = nullptr;
      return fail(SB_ERR_CUDA, std::string("planes side stream: ") + cudaGetErrorString(e));
    }
  }
  *out = &s;
  return SB_OK;
}

// Operand passes, the seven product GEMMs and the recombination.  `stages`
// selects them (bit 0 the operand passes, bit 1 the product GEMM, bit 2 the
// recombination) so a caller can time the GEMM alone; the workspace carries
// the intermediate results between separate calls.  The whole product
// (stages 7) runs in two halves of product rows: the second half's A pass,
// GEMM and recombination on a second stream, so the passes and the
// recombination of one half overlap the other half's GEMM (their kernels need
// no shared memory and fit on an SM beside a GEMM CTA) and the two GEMMs fill
// each other's last wave.  `timing` (optional, four cudaEvent_t): recorded
// around the two GEMM launches, on the stream each runs on.
int run_planes(cudaStream_t stream, const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k,
               int64_t lda, int64_t ldb, int64_t ldc, int32_t bm, int32_t bn, int32_t bk, int32_t out_dtype,
               void* workspace, size_t workspace_bytes, int32_t raster, int32_t stages = 7,
               int epi = SB_EPI_NONE, const sb_epilogue* ep = nullptr, void* const* timing = nullptr) {
  const bool gated = epi == SB_EPI_SWIGLU || epi == SB_EPI_GEGLU;  // output [M, N/2]
  if (ldc < (gated ? n / 2 : n)) return fail(SB_ERR_ALIGNMENT, gated ? "ldc must be >= N/2" : "ldc must be >= N");
  if (raster < 0) return fail(SB_ERR_UNSUPPORTED, "raster must be >= 0 (0 = the kernel's default)");
  if (stages <= 0 || stages > 7) return fail(SB_ERR_UNSUPPORTED, "stages must be a nonzero mask of bits 0-2");
  if (m % 512 || n % 512 || k % 128)
    return fail(SB_ERR_TILING, "the planes path needs M and N divisible by 512 and K by 128 (256 x 256 product "
                               "tiles, 64-deep steps), got M=" + std::to_string(m) + " N=" + std::to_string(n) +
                               " K=" + std::to_string(k));
  const size_t a_bytes = planes_a_bytes(m, k), b_bytes = quad_planes_bytes(k, n);
  const size_t need = planes_workspace(m, n, k);
  if (!workspace || workspace_bytes < need)
    return fail(SB_ERR_WORKSPACE, "the planes path needs a workspace of " + std::to_string(need) +
                                      " bytes (sb_planes_workspace_bytes), got " + std::to_string(workspace_bytes));
  if (!aligned16(workspace)) return fail(SB_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  int st = check_device();
  if (st != SB_OK) return st;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* aop = reinterpret_cast<__nv_bfloat16*>(ws);
  void* bop = ws + a_bytes;
  float* prod = reinterpret_cast<float*>(ws + a_bytes + b_bytes);
  const int64_t mh = m / 2;
  CUtensorMap ta, tb;
  if (stages & 2) {
    st = make_planes_maps(aop, bop, m, n, k, &ta, &tb);
    if (st != SB_OK) return st;
  }
  auto ev = [&](int i) { return timing ? static_cast<cudaEvent_t>(timing[i]) : nullptr; };
  auto chk = [&](cudaError_t e, const char* what) {
    return e == cudaSuccess ? SB_OK : fail(SB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  };

  PlanesSide* side = nullptr;
  if (stages == 7 && mh >= 2 * planes::kTileM) {
    st = planes_side(stream, &side);
    if (st != SB_OK) return st;
  }
  if (side) {
    const int64_t half = (mh / planes::kTileM / 2) * planes::kTileM;  // first half's product rows
    cudaStream_t aux = side->aux;
    if ((st = chk(cudaEventRecord(side->fork, stream), "fork")) != SB_OK) return st;
    if ((st = chk(cudaStreamWaitEvent(aux, side->fork, 0), "fork wait")) != SB_OK) return st;
    // Everything issued to the side stream is joined back into `stream`, on
    // failure too, so no later call overlaps this one's work.
    auto halves = [&]() -> int {
      int s2 = sb_strassen_b_operands(reinterpret_cast<sb_stream_t>(stream), b, bop, k, n, ldb, bn, bk);
      if (s2 != SB_OK) return s2;
      if ((s2 = chk(cudaEventRecord(side->b_done, stream), "B planes event")) != SB_OK) return s2;
      if ((s2 = planes_a_pass(stream, a, lda, m, k, bm, bk, aop, 0, half)) != SB_OK) return s2;
      if ((s2 = planes_a_pass(aux, a, lda, m, k, bm, bk, aop, half, mh)) != SB_OK) return s2;
      if ((s2 = chk(cudaStreamWaitEvent(aux, side->b_done, 0), "B planes wait")) != SB_OK) return s2;
      if (ev(0) && (s2 = chk(cudaEventRecord(ev(0), stream), "timing event")) != SB_OK) return s2;
      if ((s2 = planes_gemm(stream, ta, tb, m, n, k, raster, prod, 0, half)) != SB_OK) return s2;
      if (ev(1) && (s2 = chk(cudaEventRecord(ev(1), stream), "timing event")) != SB_OK) return s2;
      if (ev(2) && (s2 = chk(cudaEventRecord(ev(2), aux), "timing event")) != SB_OK) return s2;
      if ((s2 = planes_gemm(aux, ta, tb, m, n, k, raster, prod, half, mh)) != SB_OK) return s2;
      if (ev(3) && (s2 = chk(cudaEventRecord(ev(3), aux), "timing event")) != SB_OK) return s2;
      if ((s2 = planes_recombine(stream, prod, m, n, k, bm, bn, bk, c, ldc, out_dtype, epi, ep, 0, half)) != SB_OK)
        return s2;
      return planes_recombine(aux, prod, m, n, k, bm, bn, bk, c, ldc, out_dtype, epi, ep, half, mh);
    };
    st = halves();
    const int joined = chk(cudaEventRecord(side->join, aux), "join");
    const int waited = joined == SB_OK ? chk(cudaStreamWaitEvent(stream, side->join, 0), "join wait") : joined;
    return st != SB_OK ? st : waited;
  }
  if (stages & 1) {
    st = sb_strassen_b_operands(reinterpret_cast<sb_stream_t>(stream), b, bop, k, n, ldb, bn, bk);
    if (st != SB_OK) return st;
    if ((st = planes_a_pass(stream, a, lda, m, k, bm, bk, aop, 0, mh)) != SB_OK) return st;
  }
  if (stages & 2) {
    if (ev(0) && (st = chk(cudaEventRecord(ev(0), stream), "timing event")) != SB_OK) return st;
    if ((st = planes_gemm(stream, ta, tb, m, n, k, raster, prod, 0, mh)) != SB_OK) return st;
    if (ev(1) && (st = chk(cudaEventRecord(ev(1), stream), "timing event")) != SB_OK) return st;
    // One launch: events 2 and 3 mark the same end, so every span stays defined.
    if (ev(2) && (st = chk(cudaEventRecord(ev(2), stream), "timing event")) != SB_OK) return st;
    if (ev(3) && (st = chk(cudaEventRecord(ev(3), stream), "timing event")) != SB_OK) return st;
  }
  if (stages & 4) return planes_recombine(stream, prod, m, n, k, bm, bn, bk, c, ldc, out_dtype, epi, ep, 0, mh);
  return SB_OK;
}

void apply_options(GemmParams& p, int formula, int perm, const int32_t* schedule) {
  p.formula = formula == SB_FORMULA_DUAL ? 1 : formula == SB_FORMULA_POWERS ? 2 : 0;
  p.swap_m = perm & 1;
  p.swap_k = (perm >> 1) & 1;
  p.swap_n = (perm >> 2) & 1;
  p.panel_schedule = schedule;
  p.num_panels = p.K / p.bk;
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" {

size_t sb_workspace_bytes(int64_t m, int64_t n, int64_t k, int32_t epilogue_kind) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const bool planes = planes_epilogue(epilogue_kind) && planes_preferred(m, n, k) &&
                      (epilogue_kind != SB_EPI_NORM_RESIDUAL_ADD || n <= kPlanesNormMaxN);
  if (planes) return std::max(planes_workspace(m, n, k), epilogue_kind == SB_EPI_NORM_RESIDUAL_ADD
                                                             ? (size_t)m * (size_t)n * 4u : (size_t)0);
  if (epilogue_kind == SB_EPI_NORM_RESIDUAL_ADD) return (size_t)m * (size_t)n * 4u;
  return 0;
}

int sb_strassen_gemm(sb_stream_t stream_, const void* a, const void* b, void* c, int64_t m,
                     int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm,
                     int32_t bn, int32_t bk, int32_t out_dtype, const sb_epilogue* ep,
                     void* workspace, size_t workspace_bytes) {
  return sb_strassen_gemm_ex(stream_, a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype, ep,
                             nullptr, workspace, workspace_bytes);
}

int sb_strassen_gemm_ex(sb_stream_t stream_, const void* a, const void* b, void* c, int64_t m,
                        int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm,
                        int32_t bn, int32_t bk, int32_t out_dtype, const sb_epilogue* ep,
                        const sb_options* opt, void* workspace, size_t workspace_bytes) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int epi = ep ? ep->kind : SB_EPI_NONE;
  const bool narrow = opt && opt->narrow_bn;  // B200 extension: bn a multiple of 128
  int st = validate_core(a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype, narrow ? 128 : 256);
  if (st != SB_OK) return st;
  if (epi < SB_EPI_NONE || epi > SB_EPI_NORM_RESIDUAL_ADD)
    return fail(SB_ERR_EPILOGUE, "unknown epilogue kind " + std::to_string(epi));
  const int formula = opt ? opt->formula_variant : SB_FORMULA_CLASSICAL;
  const int perm = opt ? opt->block_permutation : 0;
  const int32_t* schedule = opt ? opt->panel_schedule : nullptr;
  if (formula == SB_FORMULA_POWERS && epi != SB_EPI_NONE)
    return fail(SB_ERR_EPILOGUE, "fused epilogues require a quadrant-basis formula");
  if (formula == SB_FORMULA_POWERS && schedule)
    return fail(SB_ERR_UNSUPPORTED, "exact classical panels need a quadrant-basis formula");
  if (formula != SB_FORMULA_CLASSICAL && formula != SB_FORMULA_DUAL && formula != SB_FORMULA_POWERS)
    return fail(SB_ERR_RANK, "formula_variant must be 'classical', 'dual', or 'powers'");
  if (perm < 0 || perm > 7) return fail(SB_ERR_RANK, "block_permutation must be an integer from 0 through 7");
  if (schedule && (reinterpret_cast<uintptr_t>(schedule) & 3u))
    return fail(SB_ERR_ALIGNMENT, "panel_schedule must be a 4-byte aligned int32 device array");
  if (epi != SB_EPI_NONE && out_dtype != SB_BF16)
    return fail(SB_ERR_OUTPUT_DTYPE, "fused epilogues write a BF16 output tile");
  if ((epi == SB_EPI_SWIGLU || epi == SB_EPI_GEGLU) && (bn % 2))
    return fail(SB_ERR_EPILOGUE, "gated epilogue needs an even bn");
  if ((epi == SB_EPI_RESIDUAL_ADD || epi == SB_EPI_NORM_RESIDUAL_ADD) &&
      (!ep->residual || !aligned16(ep->residual) || ep->ld_residual % 8 || ep->ld_residual < n))
    return fail(SB_ERR_EPILOGUE, "residual must be a 16-byte aligned [M, N] array with ld % 8 == 0");
  if (epi == SB_EPI_BIAS_ADD && !ep->bias) return fail(SB_ERR_EPILOGUE, "bias_add epilogue requires bias=");
  if (epi == SB_EPI_NORM_RESIDUAL_ADD) {
    if (!ep->norm_scale) return fail(SB_ERR_EPILOGUE, "norm_residual_add requires residual= and norm_scale=");
    if (bn != n)
      return fail(SB_ERR_EPILOGUE, "norm_residual_add normalises over the whole output row, so the tile must "
                                   "span it: bn=" + std::to_string(bn) + " must equal n=" + std::to_string(n));
    // The fp32 rows of the one-CTA kernel's two passes at least; the planes
    // path (sb_workspace_bytes) runs when the caller passes its larger workspace.
    const size_t rows_bytes = (size_t)m * (size_t)n * 4u;
    if (!workspace || workspace_bytes < rows_bytes || !aligned16(workspace))
      return fail(SB_ERR_WORKSPACE, "norm_residual_add needs a 16-byte aligned workspace of at least " +
                                        std::to_string(rows_bytes) + " bytes (" +
                                        std::to_string(sb_workspace_bytes(m, n, k, epi)) +
                                        " for the planes path)");
  }
  if (epi == SB_EPI_QK_NORM_ROPE) {
    if (!ep->rope_cos || !ep->rope_sin || !ep->rope_scale)
      return fail(SB_ERR_EPILOGUE, "qk_norm_rope epilogue requires rope_cos=, rope_sin= and rope_scale= "
                                   "(use rope_layout_tables and rope_scale_layout)");
    const int hd = ep->rope_head_dim;
    if (narrow ? (hd <= 0 || bn % hd) : (hd <= 0 || bn % (2 * hd)))
      return fail(SB_ERR_EPILOGUE,
                  narrow ? "qk_norm_rope with narrow tiles needs bn a multiple of head_dim=" + std::to_string(hd) +
                               " so a tile half holds whole half-heads, got bn=" + std::to_string(bn)
                         : "qk_norm_rope needs bn a multiple of 2*head_dim=" + std::to_string(2 * hd) +
                               " so a tile half holds whole heads, got bn=" + std::to_string(bn));
    if (!(hd / 2 == 8 || hd / 2 == 16 || hd / 2 == 32 || hd / 2 == 64))
      return fail(SB_ERR_UNSUPPORTED, "qk_norm_rope on B200 supports head_dim in {16, 32, 64, 128}");
    if (ep->ld_rope < bn / 2) return fail(SB_ERR_EPILOGUE, "rope tables must have bn/2 columns");
  }
  if (epi == SB_EPI_SWIGLU || epi == SB_EPI_GEGLU) {
    if (ldc < n / 2 || ldc % 8) return fail(SB_ERR_ALIGNMENT, "swiglu output leading dimension must be >= N/2 and a multiple of 8");
  } else if (ldc < n) {
    return fail(SB_ERR_ALIGNMENT, "ldc must be >= N");
  }
  // A product with room for the planes workspace runs as seven full-width
  // product GEMMs (same products, rounding and recombination order; the fused
  // epilogue applied to the recombined fp32 values as the one-CTA kernel does).
  const bool norm_ok = epi != SB_EPI_NORM_RESIDUAL_ADD ||
                       (n <= kPlanesNormMaxN && aligned16(ep->norm_scale) && aligned16(ep->residual) &&
                        aligned16(c) && ldc % 8 == 0 &&
                        ep->ld_residual % (ep->residual_dtype == SB_F32 ? 4 : 8) == 0);
  if (planes_epilogue(epi) && norm_ok && formula == SB_FORMULA_CLASSICAL && perm == 0 && !schedule && !narrow &&
      planes_preferred(m, n, k) && workspace && aligned16(workspace) &&
      workspace_bytes >= planes_workspace(m, n, k))
    return run_planes(stream, a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype, workspace, workspace_bytes,
                      0, 7, epi, ep);
  st = check_device();
  if (st != SB_OK) return st;

  CUtensorMap ta, tb;
  st = make_strassen_maps(formula != 0 || perm != 0 || schedule, a, b, m, n, k, lda, ldb, bm, bn, bk, &ta,
                          &tb);
  if (st != SB_OK) return st;

  if (epi == SB_EPI_NORM_RESIDUAL_ADD) {
    // Pass 1: fp32 pre-norm rows into the caller's workspace; pass 2: row norm.
    GemmParams p = base_params(m, n, k, bm, bn, bk, workspace, n, StrassenPipe::BK);
    apply_options(p, formula, perm, schedule);
    st = dispatch(true, SB_EPI_NONE, true, stream, ta, tb, p);
    if (st != SB_OK) return st;
    return launch_norm_rows(stream, reinterpret_cast<const float*>(workspace), m, n, ep,
                            reinterpret_cast<__nv_bfloat16*>(c), ldc);
  }

  GemmParams p = base_params(m, n, k, bm, bn, bk, c, ldc, StrassenPipe::BK);
  apply_options(p, formula, perm, schedule);
  fill_epilogue(p, ep, epi);
  return dispatch(true, epi, out_dtype == SB_F32, stream, ta, tb, p);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// No-allocation variant of the norm_residual_add path.
//
// Some callers cannot hand this library a scratch buffer or let it call
// cudaMalloc: a custom-call handler inside a framework that owns the device
// memory (XLA reserves most of it up front and cudaMalloc would both compete
// with its allocator and synchronise the device), or a serving process that
// runs with a fixed, pre-planned memory budget.  For them the fp32 pre-norm
// rows live in this file-scope device array instead of a caller workspace.
//
// Limits and sharing rules:
//   * capacity kNoAllocScratchFloats fp32 values (32 MiB): M * N must not
//     exceed it, otherwise the call returns SB_ERR_WORKSPACE before launching;
//   * every GPU that loads the library holds this array until the process
//     exits;
//   * all calls share the one array and it keeps the previous call's
//     contents; nothing needs clearing, because the GEMM pass overwrites all
//     M * N values before the row pass reads them;
//   * calls whose kernels overlap on the GPU (different streams, or several
//     host threads) race on the array -- serialise them;
//   * every call resolves the array's device address in the current context
//     with cudaGetSymbolAddress (the first call on a device also loads the
//     module there); make that first call before any stream capture.
// ---------------------------------------------------------------------------
namespace sb {
namespace {
constexpr size_t kNoAllocScratchFloats = size_t(32) << 20 >> 2;  // 32 MiB of fp32
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// The array's device address in the current context, looked up on every call
// (cheap next to a GEMM) so that it stays valid after a cudaDeviceReset or in a
// new primary context.
int noalloc_scratch_address(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return fail(SB_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
  *out = static_cast<float*>(p);
  return SB_OK;
}
}  // namespace
}  // namespace sb

extern "C" int sb_strassen_gemm_norm_residual_noalloc(sb_stream_t stream_, const void* a, const void* b,
                                                      void* c, int64_t m, int64_t n, int64_t k,
                                                      int64_t lda, int64_t ldb, int64_t ldc, int32_t bm,
                                                      int32_t bn, int32_t bk, const sb_epilogue* ep) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!ep || ep->kind != SB_EPI_NORM_RESIDUAL_ADD)
    return fail(SB_ERR_EPILOGUE, "the no-allocation entry point runs the norm_residual_add epilogue only");
  int st = validate_core(a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, SB_BF16);
  if (st != SB_OK) return st;
  if (!ep->residual || !aligned16(ep->residual) || ep->ld_residual % 8 || ep->ld_residual < n)
    return fail(SB_ERR_EPILOGUE, "residual must be a 16-byte aligned [M, N] array with ld % 8 == 0");
  if (!ep->norm_scale) return fail(SB_ERR_EPILOGUE, "norm_residual_add requires residual= and norm_scale=");
  if (bn != n)
    return fail(SB_ERR_EPILOGUE, "norm_residual_add normalises over the whole output row, so the tile must "
                                 "span it: bn=" + std::to_string(bn) + " must equal n=" + std::to_string(n));
  if (ldc < n) return fail(SB_ERR_ALIGNMENT, "ldc must be >= N");
  if ((uint64_t)m * (uint64_t)n > kNoAllocScratchFloats)
    return fail(SB_ERR_WORKSPACE, "M*N=" + std::to_string((uint64_t)m * (uint64_t)n) +
                                      " exceeds the no-allocation scratch capacity of " +
                                      std::to_string(kNoAllocScratchFloats) + " fp32 values (32 MiB)");
  st = check_device();
  if (st != SB_OK) return st;
  float* scratch = nullptr;
  st = noalloc_scratch_address(&scratch);
  if (st != SB_OK) return st;
  CUtensorMap ta, tb;
  st = make_strassen_maps(false, a, b, m, n, k, lda, ldb, bm, bn, bk, &ta, &tb);
  if (st != SB_OK) return st;
  GemmParams p = base_params(m, n, k, bm, bn, bk, scratch, n, StrassenPipe::BK);
  st = dispatch(true, SB_EPI_NONE, true, stream, ta, tb, p);
  if (st != SB_OK) return st;
  return launch_norm_rows(stream, scratch, m, n, ep, reinterpret_cast<__nv_bfloat16*>(c), ldc);
}

extern "C" {

int sb_classical_gemm(sb_stream_t stream_, const void* a, const void* b, void* c, int64_t m,
                      int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm,
                      int32_t bn, int32_t bk, int32_t out_dtype) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  int st = validate_core(a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype);
  if (st != SB_OK) return st;
  if (ldc < n) return fail(SB_ERR_ALIGNMENT, "ldc must be >= N");
  st = check_device();
  if (st != SB_OK) return st;
  CUtensorMap ta, tb;
  st = make_maps(a, b, m, n, k, lda, ldb, bm, ClassicalPipe::BK, &ta, &tb);
  if (st != SB_OK) return st;
  GemmParams p = base_params(m, n, k, bm, bn, bk, c, ldc, ClassicalPipe::BK);
  return dispatch(false, SB_EPI_NONE, out_dtype == SB_F32, stream, ta, tb, p);
}

int sb_strassen_gemm_pair(sb_stream_t stream_, const void* a, const void* b, void* c, int64_t m, int64_t n,
                          int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
                          int32_t out_dtype) {
  int st = validate_core(a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype);
  if (st != SB_OK) return st;
  return run_pair(reinterpret_cast<cudaStream_t>(stream_), a, b, nullptr, c, m, n, k, lda, ldb, ldc, bm, bn, bk,
                  out_dtype);
}

size_t sb_b_operands_bytes(int64_t k, int64_t n) {
  if (k <= 0 || n <= 0) return 0;
  return (size_t)7 * (size_t)(k / 2) * (size_t)(n / 2) * 2u;
}

int sb_strassen_b_operands(sb_stream_t stream_, const void* b, void* planes, int64_t k, int64_t n, int64_t ldb,
                           int32_t bn, int32_t bk) {
  if (!b || !planes) return fail(SB_ERR_RANK, "null matrix pointer");
  if (k <= 0 || n <= 0) return fail(SB_ERR_RANK, "matrix dimensions must be positive");
  if (bn <= 0 || bk <= 0 || n % bn || k % bk)
    return fail(SB_ERR_DIVISIBILITY, "K=" + std::to_string(k) + ", N=" + std::to_string(n) +
                                         " must be divisible by bk=" + std::to_string(bk) + ", bn=" + std::to_string(bn));
  if (bn % 256 || bk % 256) return fail(SB_ERR_TILING, "bn and bk must be multiples of 256");
  if (k > (int64_t)INT32_MAX || n > (int64_t)INT32_MAX)
    return fail(SB_ERR_UNSUPPORTED, "dimensions above 2^31-1 are not supported");
  if (!aligned16(b) || !aligned16(planes) || ldb % 8 || ldb < n)
    return fail(SB_ERR_ALIGNMENT, "B and the planes must be 16-byte aligned; ldb a multiple of 8 covering N");
  const int64_t chunks = (k / 2) * (n / 16);
  const unsigned grid = (unsigned)std::min<int64_t>((chunks + 255) / 256, 148 * 16);
  b_operand_planes_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      reinterpret_cast<const __nv_bfloat16*>(b), ldb, (int32_t)k, (int32_t)n, bn, bk,
      reinterpret_cast<__nv_bfloat16*>(planes));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("B operand planes launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

int sb_strassen_gemm_pair_planes(sb_stream_t stream_, const void* a, const void* b_planes, void* c, int64_t m,
                                 int64_t n, int64_t k, int64_t lda, int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
                                 int32_t out_dtype) {
  // The planes stand in for B [K, N] (ldb = N) in the shared validation.
  int st = validate_core(a, b_planes, c, m, n, k, lda, n, ldc, bm, bn, bk, out_dtype);
  if (st != SB_OK) return st;
  return run_pair(reinterpret_cast<cudaStream_t>(stream_), a, nullptr, b_planes, c, m, n, k, lda, n, ldc, bm, bn,
                  bk, out_dtype);
}

int sb_strassen_gemm_lhs_transposed(sb_stream_t stream_, const void* at, const void* b, void* c,
                                    int64_t m, int64_t n, int64_t k, int64_t ldat, int64_t ldb,
                                    int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
                                    int32_t out_dtype) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  // validate_core checks lda >= k for a row-major A; A^T needs ldat >= m instead.
  int st = validate_core(at, b, c, m, n, k, k, ldb, ldc, bm, bn, bk, out_dtype);
  if (st != SB_OK) return st;
  if (ldat < m || ldat % 8)
    return fail(SB_ERR_ALIGNMENT, "A^T leading dimension must cover M and be a multiple of 8");
  if ((bm / 2) % 64)
    return fail(SB_ERR_UNSUPPORTED, "strassen_matmul_lhs_transposed on B200 needs bm a multiple of 128, got " +
                                        std::to_string(bm));
  if (ldc < n) return fail(SB_ERR_ALIGNMENT, "ldc must be >= N");
  st = check_device();
  if (st != SB_OK) return st;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap ta, tb, unused;
  {
    cuuint64_t dims[2] = {(cuuint64_t)m, (cuuint64_t)k};
    cuuint64_t strides[1] = {(cuuint64_t)ldat * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)StrassenPipe::BK};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(at), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled(A^T) failed: " + std::to_string((int)r));
  }
  // B map exactly as for the ordinary GEMM (the A map it builds alongside is discarded).
  st = make_maps(b, b, m, n, k, ldb, ldb, bm, StrassenPipe::BK, &unused, &tb);
  if (st != SB_OK) return st;
  GemmParams p = base_params(m, n, k, bm, bn, bk, c, ldc, StrassenPipe::BK);
  return out_dtype == SB_F32 ? launch_typed<true, SB_EPI_NONE, true, false, true>(stream, ta, tb, p)
                             : launch_typed<true, SB_EPI_NONE, false, false, true>(stream, ta, tb, p);
}

int sb_rms_norm(sb_stream_t stream_, const void* x, const void* w, void* y, int64_t rows, int64_t n,
                int32_t w_dtype, float eps) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!x || !w || !y) return fail(SB_ERR_RANK, "null pointer");
  if (rows <= 0 || n <= 0) return fail(SB_ERR_RANK, "rows and n must be positive");
  if (n % 8 || !aligned16(x) || !aligned16(y))
    return fail(SB_ERR_ALIGNMENT, "rms_norm needs n % 8 == 0 and 16-byte aligned rows");
  if (rows > (int64_t)INT32_MAX) return fail(SB_ERR_UNSUPPORTED, "too many rows");
  rms_norm_kernel<<<(unsigned)rows, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), w,
                                                      w_dtype == SB_F32,
                                                      reinterpret_cast<__nv_bfloat16*>(y), n, eps);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("rms_norm launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

void sb_query_tile(int32_t* block_m, int32_t* block_n, int32_t* block_k) {
  if (block_m) *block_m = kBlockM;
  if (block_n) *block_n = kBlockN;
  if (block_k) *block_k = StrassenPipe::BK;
}

const char* sb_status_string(int32_t status) {
  switch (status) {
    case SB_OK: return "ok";
    case SB_ERR_RANK: return "bad rank or shape";
    case SB_ERR_INNER_DIM: return "inner dimensions disagree";
    case SB_ERR_DTYPE: return "unsupported input dtype";
    case SB_ERR_DIVISIBILITY: return "dimension not divisible by tile";
    case SB_ERR_TILING: return "tile breaks alignment";
    case SB_ERR_EPILOGUE: return "epilogue argument error";
    case SB_ERR_OUTPUT_DTYPE: return "unsupported output dtype";
    case SB_ERR_UNSUPPORTED: return "not supported by the B200 kernel";
    case SB_ERR_ALIGNMENT: return "pointer or leading-dimension alignment";
    case SB_ERR_WORKSPACE: return "workspace missing or too small";
    case SB_ERR_CUDA: return "CUDA runtime error";
    case SB_ERR_DEVICE: return "device is not an sm_100 B200";
    case SB_ERR_DEVICE_TIMEOUT: return "bounded device wait timed out";
    case SB_ERR_P2P: return "peer group argument error";
    default: return "unknown status";
  }
}

const char* sb_last_error_message(void) { return t_last_error.c_str(); }

int sb_device_status(int32_t* device_error, int32_t reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaDeviceSynchronize: ") + cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaMemcpyFromSymbol: ") + cudaGetErrorString(e));
  if (device_error) *device_error = v;
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaMemcpyToSymbol: ") + cudaGetErrorString(e));
  }
  return v ? SB_ERR_DEVICE_TIMEOUT : SB_OK;
}

int sb_wait_selftest(sb_stream_t stream) {
  int st = check_device();
  if (st != SB_OK) return st;
  int* err = nullptr;
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_device_error);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(err);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("selftest launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

size_t sb_quad_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return quad_ops_bytes(m, k) + quad_planes_bytes(k, n);
}

size_t sb_planes_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return planes_workspace(m, n, k);
}

int sb_strassen_gemm_planes(sb_stream_t stream_, const void* a, const void* b, void* c, int64_t m, int64_t n,
                            int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
                            int32_t out_dtype, void* workspace, size_t workspace_bytes, int32_t raster,
                            int32_t stages, void* const* timing_events) {
  int st = validate_core(a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype);
  if (st != SB_OK) return st;
  return run_planes(reinterpret_cast<cudaStream_t>(stream_), a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype,
                    workspace, workspace_bytes, raster, stages, SB_EPI_NONE, nullptr, timing_events);
}

int sb_strassen_gemm_quad(sb_stream_t stream_, const void* a, const void* b, void* c, int64_t m, int64_t n,
                          int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t bm, int32_t bn, int32_t bk,
                          int32_t out_dtype, void* workspace, size_t workspace_bytes, int32_t raster) {
  int st = validate_core(a, b, c, m, n, k, lda, ldb, ldc, bm, bn, bk, out_dtype);
  if (st != SB_OK) return st;
  return run_quad(reinterpret_cast<cudaStream_t>(stream_), a, b, nullptr, c, m, n, k, lda, ldb, ldc, bm, bn, bk,
                  out_dtype, workspace, workspace_bytes, raster);
}

const char* sb_version(void) { return "strassen_b200 0.1.0 (sm_100a, tcgen05)"; }

}  // extern "C"

#include "p2p_reduce.cuh"
