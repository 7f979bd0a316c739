// strassen_quad.cuh -- the four-CTA ("two SM pairs") Strassen kernel.
//
// Same algorithm, product coordinates and product split as the two-CTA kernel
// (strassen_pair.cuh; strassen_pallas.py:324-379 restated per product and
// recombined once), on B200's paired tensor cores: a thread-block cluster of
// four CTAs shares one 256 x 128 product tile (a 512 x 256 patch of C).
//
//   pair 0 (CTA ranks 0, 1): P3, P5, P7 and the left 64 columns of P1;
//   pair 1 (CTA ranks 2, 3): P2, P4, P6 and the right 64 columns of P1.
//
// Each pair runs tcgen05.mma.cta_group::2 with M = 256: CTA (pair, half) holds
// product rows 128*half .. +127 in its TMEM lanes and in its A tiles, and the
// 64-column half `half` of every B tile; the even CTA issues one 256 x 128 x 16
// MMA per full product and one 256 x 64 x 16 for P1's half.  Per SM and K step
// that is the two-CTA kernel's math with half its B bytes and half its MMA
// instructions.
//
// Operands arrive ready-made, so the K loop is a pure TMA -> MMA pipeline with
// no operand sums and no software hand-off between SMs:
//   * A operands (a_operand_pass_kernel): per product row and 16-deep chunk of
//     product depth, the four A operands of each pair side by side --
//     pair 0: a0, a0+a1, a1-a3, a0+a3;  pair 1: a2+a3, a3, a2-a0, a0+a3 --
//     64 elements = one 128-byte row, so one TMA box (128 rows x 128 bytes)
//     lands a CTA's four A operand tiles and MMA operand j starts 32 j bytes
//     into each 128-byte-swizzled row.  Each sum is one RNE bf16 rounding, the
//     reference's pre-add rounding.
//   * B operands: the seven B operand planes of b_operand_planes_kernel.
// Both CTAs of a pair issue .cta_group::2 TMA copies that complete on the even
// CTA's full barrier (armed by the even CTA with both CTAs' bytes); the even
// CTA's MMA warp commits each stage to the empty barrier of both CTAs.
//
// Recombination: as the two-CTA kernel, between CTA r and CTA r ^ 2 (the same
// rows in the other pair): pair 0 finishes C11/C12, pair 1 C21/C22, after one
// fp32 128 x 128 partial exchange through distributed shared memory.
//
// Roles per CTA (14 warps): warps 0, 2, 12, 13 TMA producers (round robin over
// K steps, lanes 0-2 one copy each); warp 1 TMEM allocation and, in the even
// CTA, the MMA issue; warp 3 (even CTA) waits on the full barriers and hands
// groups of steps to the MMA warp through a named barrier; warps 4-11 epilogue.
//
// Included by strassen_gemm.cu inside namespace sb after strassen_pair.cuh.

namespace quad {

constexpr int kCols = 128;       // product columns per cluster tile
constexpr int kTileRows = 256;   // product rows per cluster tile (128 per CTA)
constexpr int kProducers = 4;
constexpr int kProducerWarp[kProducers] = {0, 2, 12, 13};
constexpr int kThreadsQ = 14 * 32;
#ifndef SB_QUAD_GROUP
#define SB_QUAD_GROUP 2
#endif
constexpr int kGroup = SB_QUAD_GROUP;  // K steps per hand-off to the MMA warp
#ifndef SB_QUAD_RASTER
#define SB_QUAD_RASTER 2
#endif
// Default product-row tiles per column sweep (GemmParams::raster overrides it).
// Two keeps A' (the larger operand stream) in L2 across the column tiles in
// flight: 2.7 GB of DRAM reads per 8192^3 launch against 6.8 GB at 16.
constexpr int kRaster = SB_QUAD_RASTER;

// Stage layout (bytes, the same in every CTA).
struct Geo {
  static constexpr int A = 0;                       // 128 rows x 128 B: the pair's four A operands
  static constexpr int ABYTES = 128 * 128;
  static constexpr int B3 = ABYTES;                 // three planes x 16 k-rows x 64 columns (128 B rows)
  static constexpr int BPLANE = 16 * 64 * 2;
  static constexpr int BH = B3 + 3 * BPLANE;        // P1's 32 columns x 16 k-rows (64 B rows)
  static constexpr int BHBYTES = 16 * 32 * 2;
  static constexpr int STAGE = BH + BHBYTES;        // 23 KB
  static constexpr int STAGES = 9;
  static constexpr int DATA = STAGES * STAGE;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = DATA + BAR_BYTES + 1024;  // + alignment slack
  static constexpr int FULL = 0, EMPTY = STAGES, ACC = 2 * STAGES, XFREE = ACC + 1, XDATA = ACC + 2,
                       WORDS = ACC + 3;
  static_assert(STAGE % 1024 == 0 && B3 % 1024 == 0 && BH % 512 == 0, "swizzle atom alignment");
  static_assert(WORDS * 8 + 16 <= BAR_BYTES, "barrier area");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(kBlockM * pair::kXRowBytes <= DATA, "exchange buffer fits in the idle stages");
};

// M = 256 (a CTA pair), B MN-major.
constexpr uint32_t kIdesc128 = umma_idesc_bf16_f32(256, 128, false, true);
constexpr uint32_t kIdesc64 = umma_idesc_bf16_f32(256, 64, false, true);

}  // namespace quad

// A operands of both pairs for every product row t and product depth kappa:
//   ops[t][kappa / 16][g][16 j + kappa % 16] = operand j of pair g, with
//   a_q = A[I*bm + qr*bm/2 + r', P*bk + qk*bk/2 + k'] (t = I*bm/2 + r',
//   kappa = P*bk/2 + k', q = 2 qr + qk) and
//   pair 0: a0, a0+a1, a1-a3, a0+a3;  pair 1: a2+a3, a3, a2-a0, a0+a3.
// ops is [M/2][4K] bf16, contiguous.  One thread per 8 consecutive kappa.
__global__ void __launch_bounds__(256) a_operand_pass_kernel(const __nv_bfloat16* __restrict__ a, int64_t lda,
                                                             int32_t m, int32_t k, int32_t bm, int32_t bk,
                                                             __nv_bfloat16* __restrict__ ops) {
  const int64_t mh = m / 2, kh = k / 2, hbm = bm / 2, hbk = bk / 2;
  const int64_t per_row = kh / 8;  // 8-wide kappa chunks per product row
  const int64_t items = mh * per_row;
  const int64_t ld_ops = 4 * (int64_t)k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_row;
    const int64_t kap = (i - t * per_row) * 8;
    const int64_t blk = t / hbm, pnl = kap / hbk;
    const int64_t row0 = blk * bm + (t - blk * hbm);
    const int64_t col0 = pnl * bk + (kap - pnl * hbk);
    const uint4 a0 = *reinterpret_cast<const uint4*>(a + row0 * lda + col0);
    const uint4 a1 = *reinterpret_cast<const uint4*>(a + row0 * lda + col0 + hbk);
    const uint4 a2 = *reinterpret_cast<const uint4*>(a + (row0 + hbm) * lda + col0);
    const uint4 a3 = *reinterpret_cast<const uint4*>(a + (row0 + hbm) * lda + col0 + hbk);
    const uint4 s03 = add4(a0, a3);
    // Element offset of operand j of pair g for this chunk: (2 c + g) * 64 + 16 j + e.
    const int64_t c = kap / 16, e = kap % 16;
    __nv_bfloat16* row = ops + t * ld_ops + (2 * c) * 64 + e;
    uint4* g0 = reinterpret_cast<uint4*>(row);
    uint4* g1 = reinterpret_cast<uint4*>(row + 64);
    g0[0] = a0;
    g0[2] = add4(a0, a1);
    g0[4] = sub4(a1, a3);
    g0[6] = s03;
    g1[0] = add4(a2, a3);
    g1[2] = a3;
    g1[4] = sub4(a2, a0);
    g1[6] = s03;
  }
}

// ---------------------------------------------------------------- cta_group::2
__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder_smem) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem),
               "r"(kTmemCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kTmemCols) : "memory");
}
// D[tmem] (+)= A * B over the CTA pair (M = 256), issued by the even CTA.
__device__ __forceinline__ void umma2_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on one mbarrier (this CTA's or, by its shared::cluster address, the
// peer's) once every tcgen05.mma the pair's issuing thread has issued completed.
__device__ __forceinline__ void umma2_commit(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
// TMA tile loads into this CTA's shared memory whose transaction bytes complete
// on an mbarrier of either CTA of the pair (shared::cluster address).
__device__ __forceinline__ void tma2_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t c0,
                                             int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma2_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t c0,
                                             int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma2_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t c0,
                                             int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

template <bool kOutF32>
__global__ void __launch_bounds__(quad::kThreadsQ, 1)
    strassen_quad_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_bh, const GemmParams p) {
  using namespace quad;
  using G = Geo;
  constexpr int kStages = G::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t smem_base = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::DATA);
  const uint32_t bar0 = smem_addr(bars);
  auto bar = [&](int slot) -> uint32_t { return bar0 + 8u * (uint32_t)slot; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + G::WORDS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0..3
  const uint32_t pr = rank >> 1;            // product set (pair)
  const uint32_t half = rank & 1u;          // rows 128*half of the tile; B column half
  const bool even = half == 0;              // the pair's MMA-issuing CTA
  const uint32_t leader = rank & ~1u;
  const uint32_t xpeer = rank ^ 2u;         // same rows, other product set

  // Grouped rasterisation over cluster tiles (as the other kernels).
  const int tile = blockIdx.x >> 2;
  const int raster = p.raster > 0 ? p.raster : kRaster;
  const int per_group = raster * p.tiles_n;
  const int group = tile / per_group;
  const int first_m = group * raster;
  const int rows_in_group = min(p.tiles_m - first_m, raster);
  const int in_group = tile - group * per_group;
  const int tt0 = (first_m + in_group % rows_in_group) * kTileRows;  // first product row of the tile
  const int t0 = tt0 + 128 * (int)half;                               // this CTA's first product row
  const int u0 = (in_group / rows_in_group) * kCols;                  // first product column

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(G::FULL + s), 1);
      mbar_init(bar(G::EMPTY + s), 1);
    }
    mbar_init(bar(G::ACC), 1);
    mbar_init(bar(G::XFREE), kSumWarps);
    mbar_init(bar(G::XDATA), kSumThreads);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  const int producer = warp == kProducerWarp[0] ? 0 : warp == kProducerWarp[1] ? 1
                     : warp == kProducerWarp[2] ? 2 : warp == kProducerWarp[3] ? 3 : -1;
  if (producer >= 0 && lane < 3) tma_prefetch_desc(lane == 0 ? &tmap_a : lane == 1 ? &tmap_b : &tmap_bh);
  if (warp == 1) tmem_alloc_pair(smem_addr(tmem_holder));
  tc_fence_before();
  // Every CTA's barriers and TMEM must exist before a peer's copies, commits or
  // exchange can reach them.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  bool ok = true;
  if (producer >= 0) {
    // ------------------------------------------------------------ TMA producers
    for (int c = producer; c < p.num_chunks; c += kProducers) {
      const int s = c % kStages;
      const bool freed = mbar_wait_hint(bar(G::EMPTY + s), ((c / kStages) & 1u) ^ 1u, abort_flag, p.err,
                                        kErrWaitEmpty);
      if (!__all_sync(0xffffffffu, freed)) break;
      const uint32_t stage = smem_base + s * G::STAGE;
      const uint32_t fb = mapa_shared(bar(G::FULL + s), leader);
      if (even && lane == 0) mbar_arrive_expect_tx(bar(G::FULL + s), 2 * G::STAGE);
      __syncwarp();
      const int kap = c * 16;
      if (lane == 0) {
        tma2_load_2d(stage + G::A, &tmap_a, fb, (2 * c + (int)pr) * 64, t0);
      } else if (lane == 1) {
        tma2_load_4d(stage + G::B3, &tmap_b, fb, 0, kap, u0 / 64 + (int)half,
                     pr ? pair::kPlaneP2 : pair::kPlaneP3);
      } else if (lane == 2) {
        tma2_load_3d(stage + G::BH, &tmap_bh, fb, u0 + 64 * (int)pr + 32 * (int)half, kap, pair::kPlaneP1);
      }
      __syncwarp();
    }
    // Drain (the even CTA: its full barriers count both CTAs' bytes): no TMA
    // write may land after teardown.  Bounded; in normal runs every phase has
    // completed long before.
    if (even && lane == 0) {
      const int first = p.num_chunks > kStages ? p.num_chunks - kStages : 0;
      for (int c = producer; c < p.num_chunks; c += kProducers)
        if (c >= first) mbar_wait_drain(bar(G::FULL + c % kStages), (c / kStages) & 1u);
    }
  } else if (warp == 3 && even) {
    // ------------------------------------------------------------ step hand-off
    for (int g0 = 0; g0 < p.num_chunks; g0 += kGroup) {
      const int cnt = min(kGroup, p.num_chunks - g0);
      bool waited = true;
      for (int i = 0; i < cnt && waited; ++i) {
        const int g = g0 + i;
        waited = mbar_wait_hint(bar(G::FULL + g % kStages), (g / kStages) & 1u, abort_flag, p.err, kErrWaitRaw);
      }
      __syncwarp();  // bar.red is warp-aligned
      if (named_bar_red_or(1, 64, !waited)) break;
    }
  } else if (warp == 1 && even) {
    // ------------------------------------------------------------ MMA issuer
    // Accumulators (TMEM columns, both CTAs): 0, 128, 256 the pair's three full
    // products (pair 0: M3, M5, M7; pair 1: M2, M4, M6), 384 P1's 64-column
    // half.  A operand j is 32 j bytes into each 128-byte row of the A tile.
    const uint64_t a_d0 = umma_smem_desc(smem_base + G::A, 16, 1024, kLayoutSwizzle128B);
    const uint64_t b_d0 = umma_smem_desc(smem_base + G::B3, 2048, 1024, kLayoutSwizzle128B);
    const uint64_t bh_d0 = umma_smem_desc(smem_base + G::BH, 1024, 512, kLayoutSwizzle64B);
    const uint64_t bp = (uint64_t)(G::BPLANE >> 4);
    for (int g0 = 0; g0 < p.num_chunks; g0 += kGroup) {
      __syncwarp();  // bar.red is warp-aligned
      if (named_bar_red_or(1, 64, false)) break;
      if (lane == 0) {
        tc_fence_after();
        const int cnt = min(kGroup, p.num_chunks - g0);
        for (int i = 0; i < cnt; ++i) {
          const int g = g0 + i;
          const int s = g % kStages;
          const uint64_t so = (uint64_t)((s * G::STAGE) >> 4);
          const uint32_t acc = g != 0 ? 1u : 0u;
          umma2_bf16_ss(tmem_base + 0, a_d0 + so + 0, b_d0 + so + 0 * bp, kIdesc128, acc);
          umma2_bf16_ss(tmem_base + 128, a_d0 + so + 2, b_d0 + so + 1 * bp, kIdesc128, acc);
          umma2_bf16_ss(tmem_base + 256, a_d0 + so + 4, b_d0 + so + 2 * bp, kIdesc128, acc);
          umma2_bf16_ss(tmem_base + 384, a_d0 + so + 6, bh_d0 + so, kIdesc64, acc);
          // The stage is free in both CTAs once these MMAs have read it.
          umma2_commit(bar(G::EMPTY + s));
          umma2_commit(mapa_shared(bar(G::EMPTY + s), rank | 1u));
        }
      }
    }
    // Always commit: both CTAs' epilogues (or teardown drains) wait on it.
    if (lane == 0) {
      umma2_commit(bar(G::ACC));
      umma2_commit(mapa_shared(bar(G::ACC), rank | 1u));
    }
    __syncwarp();
  } else if (warp >= kFirstSumWarp && warp < kFirstSumWarp + kSumWarps) {
    // ------------------------------------------------------------ epilogue
    const int set = (warp - kFirstSumWarp) >> 2;
    const int q = warp & 3;
    const uint32_t row = 32 * q + lane;  // product row t0 + row = TMEM lane
    if (warp_wait(bar(G::ACC), 0, abort_flag, p.err, kErrWaitAcc)) {
      tc_fence_after();
      // Every MMA retired, every copy consumed: our stages may take the peer's partial.
      if (lane == 0) mbar_remote_arrive(mapa_shared(bar(G::XFREE), xpeer));
      const int h = set;                      // columns [64h, 64h + 64) of the product tile
      const bool mine = (uint32_t)h == pr;    // this half holds our 64 columns of P1
      const uint32_t tmem_row = tmem_base + ((uint32_t)(32 * q) << 16);
      const uint32_t xrow = smem_base + row * pair::kXRowBytes;
      if (pair::warp_wait_cluster(bar(G::XFREE), 0, abort_flag, p.err, pair::kErrPairExchange)) {
#pragma unroll 1
        for (int j = 0; j < 8; ++j) {
          const int col = 64 * h + 8 * j;
          float y[8], m1[8];
          tmem_load_8(tmem_row + (pr ? 128u : 0u) + col, y);  // pair 0: M3, pair 1: M4
          if (mine) {
            tmem_load_8(tmem_row + 384u + (col - 64 * (int)pr), m1);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] += m1[e];
          }
          st_cluster_f32x4(mapa_shared(xrow + col * 4, xpeer), y[0], y[1], y[2], y[3]);
          st_cluster_f32x4(mapa_shared(xrow + col * 4 + 16, xpeer), y[4], y[5], y[6], y[7]);
        }
        mbar_remote_arrive(mapa_shared(bar(G::XDATA), xpeer));
        if (pair::warp_wait_cluster(bar(G::XDATA), 0, abort_flag, p.err, pair::kErrPairExchange)) {
          const int t = t0 + (int)row;
          const bool row_ok = t < p.Mp;
          const int blk_i = t / p.half_bm;
          const int64_t out_row = (int64_t)blk_i * p.bm + (t - blk_i * p.half_bm) + (pr ? p.half_bm : 0);
          const int j_block = u0 / p.half_bn;
          const int64_t col_left0 = (int64_t)j_block * p.bn + (u0 - j_block * p.half_bn);
#pragma unroll 1
          for (int j = 0; j < 8; ++j) {
            const int col = 64 * h + 8 * j;
            float d0[8], d1[8], d2[8], m1[8], left[8], right[8];
            tmem_load_8(tmem_row + col, d0);
            tmem_load_8(tmem_row + 128u + col, d1);
            tmem_load_8(tmem_row + 256u + col, d2);
            if (mine) tmem_load_8(tmem_row + 384u + (col - 64 * (int)pr), m1);
            const float4 ya = lds_f32x4(xrow + col * 4), yb = lds_f32x4(xrow + col * 4 + 16);
            const float yin[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float z = mine ? yin[e] + m1[e] : yin[e];
              if (pr == 0) {
                left[e] = (z - d1[e]) + d2[e];  // C11 = M1 + M4 - M5 + M7
                right[e] = d0[e] + d1[e];       // C12 = M3 + M5
              } else {
                left[e] = d0[e] + d1[e];        // C21 = M2 + M4
                right[e] = (z - d0[e]) + d2[e]; // C22 = M1 - M2 + M3 + M6
              }
            }
            if (row_ok) {
              store8<kOutF32>(p.C, out_row * p.ldc + col_left0 + col, left);
              store8<kOutF32>(p.C, out_row * p.ldc + col_left0 + p.half_bn + col, right);
            }
          }
        }
      }
    } else {
      ok = false;
    }
  }
  (void)ok;

  // ------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  // No CTA leaves while a peer may still write into its shared memory, arrive
  // on its barriers, or (the even CTA's MMAs) use its TMEM.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if (lane == 0) mbar_wait_drain(bar(G::ACC), 0);  // every MMA of the pair has retired
    __syncwarp();
    tmem_dealloc_pair(tmem_base);
  }
}
