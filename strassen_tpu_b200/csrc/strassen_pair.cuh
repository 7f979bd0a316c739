// strassen_pair.cuh -- the two-CTA ("product split") Strassen kernel.
//
// Same algorithm and product coordinates as strassen_gemm_kernel
// (strassen_pallas.py:156-880 restated per product, recombined once), but a
// thread-block cluster of two CTAs shares one 128 x 128 product tile (a
// 256 x 256 patch of C) and splits the seven products between them:
//
//   CTA 0: P3 = a0 (b1-b3), P5 = (a0+a1) b3, P7 = (a1-a3)(b2+b3), and the left
//          64 columns of P1 = (a0+a3)(b0+b3);
//   CTA 1: P2 = (a2+a3) b0, P4 = a3 (b2-b0), P6 = (a2-a0)(b0+b1), and the
//          right 64 columns of P1.
//
// Each CTA accumulates 3 x 128 + 64 = 448 TMEM columns, so three of its four
// tcgen05.mma per 16-deep K step are 128 x 128 x 16 instead of 128 x 64 x 16:
// about half the MMA instructions per unit of work of the one-CTA kernel.
//
// Operands.  Each CTA TMA-loads the three A quadrants its products use (CTA 0:
// a0, a1, a3; CTA 1: a2, a3, a0) and its B operands, in one of two forms:
//   * kPreB = false (sb_strassen_gemm_pair): the raw B quadrants it needs
//     (CTA 0: b1, b3, b2, b0's left half; CTA 1: b0, b2, b1, b3's right
//     half); the sum warps form the B sums in shared memory -- CTA 0 b1-b3
//     into the sum slot, b2+b3 over b2, (b0+b3)L over b0L; CTA 1 b2-b0 into
//     the sum slot, b0+b1 over b1, (b0+b3)R over b3R.
//   * kPreB = true (sb_strassen_gemm_pair_planes): the seven B operands were
//     formed once by b_operand_planes_kernel (the same bf16 sums, the same
//     rounding) and each CTA loads its three and a half operand planes as they
//     are: no B sums in the K loop, so the step's shared-memory traffic is the
//     TMA fill, the A-row reads of the sum warps and the MMA operand reads.
// Four producer warps (0, 2, 12, 13) take the steps round robin; four lanes of
// the step's warp issue its copies.  The A sums (CTA 0: a0+a1, a1-a3, a0+a3; CTA 1: a2+a3,
// a2-a0, a0+a3) are written back into the stage (two over raw quadrants that
// are no longer needed, one into a fourth A slot), so every MMA reads both
// operands from shared memory and a stage is recycled only through the stage
// ring: no operand ring in TMEM, whose two-step depth made every step wait on
// the MMAs of the step before last.  Every pre-add is one RNE bf16 rounding,
// the reference's pre-add rounding.
//
// Recombination.  C11 = M1+M4-M5+M7 and C12 = M3+M5 belong to CTA 0 (top
// rows of each block), C21 = M2+M4 and C22 = M1-M2+M3+M6 to CTA 1 (bottom
// rows).  After the K loop each CTA sends its peer one fp32 128 x 128 partial
// through distributed shared memory -- CTA 0: M3 + [M1L | 0], CTA 1:
// M4 + [0 | M1R] -- then finishes its two quadrants:
//   CTA 0: C11 = ((Y1 + [M1L | 0]) - M5) + M7, C12 = M3 + M5;
//   CTA 1: C21 = M2 + M4, C22 = ((Y0 + [0 | M1R]) - M2) + M6.
//
// Synchronisation (all waits bounded, as in the one-CTA kernel):
//   full[s]  the producer's arrival + the stage's TMA bytes;
//   sums[s]  the four sum warps of the step's set; empty[s] local MMA commit;
//   named barrier 1: warp 3 waits on sums[] for a group of kGroup steps and
//            meets the MMA warp there, so the issuing thread never polls an
//            mbarrier (that stalls it behind its queued MMAs on B200);
//   xfree / xdata  the epilogue exchange: remote arrivals from the peer, waited
//            with cluster-scope acquire.
// The K loop never waits on the peer.  Both CTAs end with a cluster barrier,
// so neither leaves while the other may still write into its shared memory.
//
// Roles: warps 0, 2, 12, 13 TMA producers, warp 1 TMEM allocation + MMA issue,
// warp 3 hands each sub-step to the MMA warp (named barrier), warps 4-11
// operand sums then epilogue (as in the one-CTA kernel).
//
// Included by strassen_gemm.cu inside namespace sb, after the one-CTA kernel
// (it uses its constants, GemmParams and store helpers).

namespace pair {

constexpr int kCols = 128;  // product columns per CTA pair
// Steps handed from warp 3 to the MMA warp per named-barrier meeting.
#ifndef SB_PAIR_GROUP
#define SB_PAIR_GROUP 2
#endif
constexpr int kGroup = SB_PAIR_GROUP;
// Stage geometry: one 16-deep K step of every operand.  Byte offsets, the same
// in both CTAs:
//   AOWN  A quadrants (r, 0), (r, 1)           ARECV the third A quadrant
//   ASUM  the third A operand sum              B0..B2 three B tiles (128 columns)
//   BH    the 64-column half tile for P1       BSUM  (raw B only) the B sum slot
// Raw B (kPreB = false): B0/B1 own quadrants (0, 1-r), (1, 1-r), B2 the other
// full quadrant.  Planes (kPreB = true): B0..B2 the operand planes of the CTA's
// three full products (CTA 0: P3, P5, P7; CTA 1: P2, P4, P6), BH P1's.
template <bool kPreB>
struct Geo {
  static constexpr int KD = 16;
  static constexpr int ATILE = kBlockM * KD * 2;         // 128 rows x 16, K-major, 32-byte rows
  static constexpr int BTILE = KD * kCols * 2;           // 16 rows x 128 columns, two 64-column chunks
  static constexpr int BHALF = BTILE / 2;
  static constexpr int AOWN = 0, ARECV = 2 * ATILE, ASUM = 3 * ATILE, B0 = 4 * ATILE, B1 = B0 + BTILE,
                       B2 = B1 + BTILE, BH = B2 + BTILE, BSUM = BH + BHALF;
  static constexpr int STAGE = kPreB ? BSUM : BSUM + BTILE;  // 30 KB (planes), 34 KB (raw)
  static constexpr int STAGES = kPreB ? 7 : 6;
  static constexpr int DATA = STAGES * STAGE;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = DATA + BAR_BYTES + 1024;  // + alignment slack
  // Bytes each producer warp lands per stage (roles, see the kernel).
  static constexpr int TX_A_OWN = 2 * ATILE, TX_A_RECV = ATILE;  // per stage, all four copies together
  static constexpr int TX_B = (kPreB ? 3 : 2) * BTILE, TX_BH = (kPreB ? 0 : BTILE) + BHALF;
  static constexpr uint32_t A_LAYOUT = kLayoutSwizzle32B;
  static constexpr uint32_t A_SBO = 8 * KD * 2;
  static constexpr uint32_t B_LBO = KD * 128;  // MN-major 128-byte swizzle: next 64-column chunk
  // Barrier slots (8 bytes each) after the stages.
  static constexpr int FULL = 0, SUMS = STAGES, EMPTY = 2 * STAGES, ACC = 3 * STAGES, XFREE = ACC + 1,
                       XDATA = ACC + 2, WORDS = ACC + 3;
  static_assert(STAGE % 1024 == 0 && B0 % 1024 == 0 && BH % 1024 == 0 && BSUM % 1024 == 0,
                "128-byte swizzle atoms need 1024-byte aligned tiles");
  static_assert(WORDS * 8 + 16 <= BAR_BYTES, "barrier area");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};
// Four producer warps take the K steps round robin (warp i: steps i, i + 4,
// ...); within a step lanes 0-3 issue its four TMA copies.  A B200 thread that
// streams copies through a ring sustains only about one copy per 500-800
// cycles however deep the ring or large the copy (measured), so each thread
// issues one copy per four steps.
constexpr int kProducers = 4;
constexpr int kProducerWarp[kProducers] = {0, 2, 12, 13};
constexpr int kCopies = 4;  // TMA copies per stage (lanes 0..3 of the step's producer warp)
constexpr int kPairThreads = 14 * 32;  // warps 0-13
constexpr int kXRowBytes = kCols * 4 + 16;  // exchange row: 128 fp32 + 16 B (bank spread)
static_assert(kBlockM * kXRowBytes <= Geo<true>::DATA && kBlockM * kXRowBytes <= Geo<false>::DATA,
              "exchange buffer fits in the idle stages");
constexpr uint32_t kIdesc128 = umma_idesc_bf16_f32(kBlockM, 128, false, true);
constexpr uint32_t kIdesc64 = umma_idesc_bf16_f32(kBlockM, 64, false, true);
constexpr uint32_t kBSbo = 1024;  // next 8 k-rows of a 128-byte-swizzled B tile
constexpr uint32_t kALbo = 16;    // unused for swizzled K-major A
// Operand planes of the B side, in the order the CTAs load them.
constexpr int kPlaneP3 = 0, kPlaneP5 = 1, kPlaneP7 = 2, kPlaneP1 = 3, kPlaneP2 = 4, kPlaneP4 = 5, kPlaneP6 = 6;

enum : int {
  kErrPairExchange = 6,  // epilogue exchange with the peer timed out
};

// Every lane waits itself with cluster-scope acquire (the peer's writes into
// this CTA's shared memory must be visible to each lane afterwards).
__device__ __forceinline__ bool warp_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err, int code) {
  return __all_sync(0xffffffffu, mbar_wait_cluster(bar, parity, abort_flag, err, code));
}

}  // namespace pair

// The seven B operands of every Strassen block, formed once (the reference's
// B pre-adds, strassen_pallas.py:324-379, each rounded once to bf16):
//   planes[i][kappa][u] = operand i at product depth kappa = P*bk/2 + k' and
//   product column u = J*bn/2 + c', in the order P3 (b1-b3), P5 (b3),
//   P7 (b2+b3), P1 (b0+b3), P2 (b0), P4 (b2-b0), P6 (b0+b1).
// planes is [7][K/2][N/2] bf16, contiguous.  One thread per 8 columns.
__global__ void __launch_bounds__(256) b_operand_planes_kernel(const __nv_bfloat16* __restrict__ b, int64_t ldb,
                                                               int32_t k, int32_t n, int32_t bn, int32_t bk,
                                                               __nv_bfloat16* __restrict__ planes) {
  const int64_t kh = k / 2, nh = n / 2, hbn = bn / 2, hbk = bk / 2;
  const int64_t chunks = kh * (nh / 8);
  const int64_t plane = kh * nh;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kappa = i / (nh / 8);
    const int64_t u = (i - kappa * (nh / 8)) * 8;
    const int64_t pnl = kappa / hbk, blk = u / hbn;
    const int64_t row0 = pnl * bk + (kappa - pnl * hbk);
    const int64_t col0 = blk * bn + (u - blk * hbn);
    const uint4 b0 = *reinterpret_cast<const uint4*>(b + row0 * ldb + col0);
    const uint4 b1 = *reinterpret_cast<const uint4*>(b + row0 * ldb + col0 + hbn);
    const uint4 b2 = *reinterpret_cast<const uint4*>(b + (row0 + hbk) * ldb + col0);
    const uint4 b3 = *reinterpret_cast<const uint4*>(b + (row0 + hbk) * ldb + col0 + hbn);
    uint4* out = reinterpret_cast<uint4*>(planes + kappa * nh + u);
    const int64_t step = plane / 8;  // one plane, in uint4 units
    out[pair::kPlaneP3 * step] = sub4(b1, b3);
    out[pair::kPlaneP5 * step] = b3;
    out[pair::kPlaneP7 * step] = add4(b2, b3);
    out[pair::kPlaneP1 * step] = add4(b0, b3);
    out[pair::kPlaneP2 * step] = b0;
    out[pair::kPlaneP4 * step] = sub4(b2, b0);
    out[pair::kPlaneP6 * step] = add4(b0, b1);
  }
}

template <bool kOutF32, bool kPreB>
__global__ void __launch_bounds__(pair::kPairThreads, 1)
    strassen_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_a1,
                         const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_b1,
                         const __grid_constant__ CUtensorMap tmap_bh, const GemmParams p) {
  using namespace pair;
  using G = Geo<kPreB>;
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
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;

  // Grouped rasterisation over pair tiles (the one-CTA kernel's order).
  const int tile = blockIdx.x >> 1;
  const int per_group = kRasterGroup * p.tiles_n;
  const int group = tile / per_group;
  const int first_m = group * kRasterGroup;
  const int rows_in_group = min(p.tiles_m - first_m, kRasterGroup);
  const int in_group = tile - group * per_group;
  const int t0 = (first_m + in_group % rows_in_group) * kBlockM;  // first product row
  const int u0 = (in_group / rows_in_group) * kCols;               // first product column

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(G::FULL + s), 1);
      mbar_init(bar(G::SUMS + s), 4);
      mbar_init(bar(G::EMPTY + s), 1);
    }
    mbar_init(bar(G::ACC), 1);
    mbar_init(bar(G::XFREE), kSumWarps);
    mbar_init(bar(G::XDATA), kSumThreads);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  // Index of this producer warp (-1: not a producer); lane `role` < kCopies
  // issues one copy of each of the warp's steps: 0 A own quadrants, 1 the third
  // A quadrant, 2 the B tiles, 3 P1's half tile (raw B: also the third B tile).
  const int producer = warp == kProducerWarp[0] ? 0 : warp == kProducerWarp[1] ? 1
                     : warp == kProducerWarp[2] ? 2 : warp == kProducerWarp[3] ? 3 : -1;
  const int role = lane;
  if (producer >= 0 && role < kCopies) {
    tma_prefetch_desc(role == 0 ? &tmap_a : role == 1 ? &tmap_a1 : role == 2 ? &tmap_b : &tmap_bh);
    if (!kPreB && role == 3) tma_prefetch_desc(&tmap_b1);
  }
  if (warp == 1) tmem_alloc<kTmemCols>(smem_addr(tmem_holder));
  tc_fence_before();
  // The peer's barriers must be initialised before its epilogue exchange can
  // reach them.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  bool ok = true;
  if (producer >= 0) {
    // ------------------------------------------------------------ TMA producers
    const int a_row_base = t0 % p.half_bm;
    const int a_block = t0 / p.half_bm;
    const int j_block = u0 / p.half_bn;
    const int b_chunk0 = (j_block * p.bn + (u0 - j_block * p.half_bn)) / 64;  // raw-B column chunk
    for (int c = producer; c < p.num_chunks; c += kProducers) {
      const int s = c % kStages;
      const bool freed = mbar_wait_hint(bar(G::EMPTY + s), ((c / kStages) & 1u) ^ 1u, abort_flag, p.err,
                                        kErrWaitEmpty);
      if (!__all_sync(0xffffffffu, freed)) break;
      const uint32_t stage = smem_base + s * G::STAGE;
      const uint32_t fb = bar(G::FULL + s);
      const int kap = c * G::KD;
      const int panel = kap / p.half_bk;
      const int kcol = panel * p.bk + (kap - panel * p.half_bk);
      if (lane == 0) mbar_arrive_expect_tx(fb, G::TX_A_OWN + G::TX_A_RECV + G::TX_B + G::TX_BH);
      __syncwarp();
      if (role == 0) {
        tma_load_5d(stage + G::AOWN, &tmap_a, fb, kcol, a_row_base, a_block, 0, (int)rank);
      } else if (role == 1) {
        tma_load_5d(stage + G::ARECV, &tmap_a1, fb, kcol, a_row_base, a_block, (int)peer, (int)peer);
      } else if (role == 2) {
        if constexpr (kPreB) {
          tma_load_4d(stage + G::B0, &tmap_b, fb, 0, kap, u0 / 64, rank ? kPlaneP2 : kPlaneP3);
        } else {
          tma_load_5d(stage + G::B0, &tmap_b, fb, 0, kcol, b_chunk0, (int)peer, 0);
        }
      } else if (role == 3) {
        if constexpr (kPreB) {
          tma_load_4d(stage + G::BH, &tmap_bh, fb, 0, kap, u0 / 64 + (int)rank, kPlaneP1);
        } else {
          tma_load_5d(stage + G::B2, &tmap_b1, fb, 0, kcol, b_chunk0, (int)rank, (int)peer);
          tma_load_5d(stage + G::BH, &tmap_bh, fb, 0, kcol, b_chunk0 + (int)rank, (int)rank, (int)rank);
        }
      }
      __syncwarp();
    }
    // Drain: no TMA write may land after teardown.  Every step this warp armed
    // in the last kStages steps is waited for (bounded: a phase that never
    // completes gives up after the wait limit).
    if (lane == 0) {
      const int first = p.num_chunks > kStages ? p.num_chunks - kStages : 0;
      for (int c = producer; c < p.num_chunks; c += kProducers)
        if (c >= first) mbar_wait_drain(bar(G::FULL + c % kStages), (c / kStages) & 1u);
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ step hand-off
    // Waits on the sums barriers of a group of kGroup steps and meets the MMA
    // warp at named barrier 1 (ORing in the abort verdict), so the issuing
    // thread itself never polls an mbarrier: that would stall it behind its
    // queued MMAs and idle the tensor pipe.
    for (int g0 = 0; g0 < p.num_chunks; g0 += kGroup) {
      const int cnt = min(kGroup, p.num_chunks - g0);
      bool waited = true;
      for (int i = 0; i < cnt && waited; ++i) {
        const int g = g0 + i;
        waited = mbar_wait_hint(bar(G::SUMS + g % kStages), (g / kStages) & 1u, abort_flag, p.err, kErrWaitSums);
      }
      __syncwarp();  // bar.red is warp-aligned
      if (named_bar_red_or(1, 64, !waited)) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Accumulators (TMEM columns): 0 and 128 two full products, 256 the third,
    // 384 the 64-column half of P1 (CTA 0: M3, M5, M7, M1L; CTA 1: M2, M4, M6,
    // M1R).  A operand of each, by slot (after the sum warps): x0, x1, ARECV,
    // ASUM -- CTA 0: a0, a0+a1, a1-a3, a0+a3; CTA 1: a2+a3, a3, a2-a0, a0+a3.
    // B tiles: planes B0, B1, B2, BH; raw B: CTA 0 BSUM (b1-b3), B1 (b3),
    // B2 (b2+b3), BH; CTA 1 B0 (b0), BSUM (b2-b0), B2 (b0+b1), BH.
    const uint64_t a_d0 = umma_smem_desc(smem_base, kALbo, G::A_SBO, G::A_LAYOUT);
    const uint64_t b_d0 = umma_smem_desc(smem_base, G::B_LBO, kBSbo, kLayoutSwizzle128B);
    const uint64_t a0_o = (uint64_t)(G::AOWN >> 4), a1_o = (uint64_t)((G::AOWN + G::ATILE) >> 4);
    const uint64_t a2_o = (uint64_t)(G::ARECV >> 4), a3_o = (uint64_t)(G::ASUM >> 4);
    const int b0_bo = kPreB ? G::B0 : (rank ? G::B0 : G::BSUM);
    const int b1_bo = kPreB ? G::B1 : (rank ? G::BSUM : G::B1);
    const uint64_t b0_o = (uint64_t)(b0_bo >> 4), b1_o = (uint64_t)(b1_bo >> 4);
    const uint64_t b2_o = (uint64_t)(G::B2 >> 4), bh_o = (uint64_t)(G::BH >> 4);
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
          umma_bf16_ss(tmem_base + 0, a_d0 + so + a0_o, b_d0 + so + b0_o, kIdesc128, acc);
          umma_bf16_ss(tmem_base + 128, a_d0 + so + a1_o, b_d0 + so + b1_o, kIdesc128, acc);
          umma_bf16_ss(tmem_base + 256, a_d0 + so + a2_o, b_d0 + so + b2_o, kIdesc128, acc);
          umma_bf16_ss(tmem_base + 384, a_d0 + so + a3_o, b_d0 + so + bh_o, kIdesc64, acc);
          umma_commit(bar(G::EMPTY + s));  // frees the stage once these MMAs have read it
        }
      }
    }
    // Always commit: the epilogue (or the teardown drain) waits on it.
    if (lane == 0) umma_commit(bar(G::ACC));
    __syncwarp();
  } else if (warp >= kFirstSumWarp && warp < kFirstSumWarp + kSumWarps) {
    // ------------------------------------------------------------ operand sums
    const int set = (warp - kFirstSumWarp) >> 2;
    const int q = warp & 3;
    const uint32_t row = 32 * q + lane;  // 0..127 within the set
    // The A operand tiles of a stage share one layout (same swizzle, same row
    // order), so the sums are elementwise over byte offsets: thread `row` takes
    // the 16-byte chunks row and row + 128 of each tile, a warp reading 512
    // contiguous bytes per load (no bank conflicts).
    const uint32_t lo_off = 16 * row;
    const uint32_t hi_off = 16 * row + 2048;
    const uint32_t o1 = 16 * row, o2 = o1 + G::BHALF;
    // Steps g = set, set + 2, ...
    for (int g = set; g < p.num_chunks; g += 2) {
      const int s = g % kStages;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_hint(bar(G::FULL + s), (g / kStages) & 1u, abort_flag, p.err, kErrWaitRaw))) {
        ok = false;
        break;
      }
      const uint32_t st = smem_base + s * G::STAGE;
      // A: x0, x1 = quadrants (r, 0), (r, 1); x2 = the third quadrant.
      const uint32_t x0a = st + G::AOWN, x1a = st + G::AOWN + G::ATILE, x2a = st + G::ARECV, xsa = st + G::ASUM;
      const uint4 x0l = lds128(x0a + lo_off), x0h = lds128(x0a + hi_off);
      const uint4 x1l = lds128(x1a + lo_off), x1h = lds128(x1a + hi_off);
      const uint4 x2l = lds128(x2a + lo_off), x2h = lds128(x2a + hi_off);
      if (rank == 0) {
        sts128(x1a + lo_off, add4(x0l, x1l));  // a0+a1 over a1
        sts128(x1a + hi_off, add4(x0h, x1h));
        sts128(x2a + lo_off, sub4(x1l, x2l));  // a1-a3 over a3
        sts128(x2a + hi_off, sub4(x1h, x2h));
        sts128(xsa + lo_off, add4(x0l, x2l));  // a0+a3
        sts128(xsa + hi_off, add4(x0h, x2h));
      } else {
        sts128(x0a + lo_off, add4(x0l, x1l));  // a2+a3 over a2
        sts128(x0a + hi_off, add4(x0h, x1h));
        sts128(x2a + lo_off, sub4(x0l, x2l));  // a2-a0 over a0
        sts128(x2a + hi_off, sub4(x0h, x2h));
        sts128(xsa + lo_off, add4(x1l, x2l));  // a3+a0
        sts128(xsa + hi_off, add4(x1h, x2h));
      }
      if constexpr (!kPreB) {
        // B: d, e = own quadrants (0, 1-r), (1, 1-r); f = the other full quadrant, h = P1's half.
        const uint4 d1 = lds128(st + G::B0 + o1), d2 = lds128(st + G::B0 + o2);
        const uint4 e1 = lds128(st + G::B1 + o1), e2 = lds128(st + G::B1 + o2);
        const uint4 f1 = lds128(st + G::B2 + o1), f2 = lds128(st + G::B2 + o2);
        const uint4 h1 = lds128(st + G::BH + o1);
        if (rank == 0) {
          sts128(st + G::BSUM + o1, sub4(d1, e1));  // b1 - b3
          sts128(st + G::BSUM + o2, sub4(d2, e2));
          sts128(st + G::B2 + o1, add4(f1, e1));    // b2 + b3
          sts128(st + G::B2 + o2, add4(f2, e2));
          sts128(st + G::BH + o1, add4(h1, e1));    // (b0 + b3) left chunk
        } else {
          sts128(st + G::BSUM + o1, sub4(e1, d1));  // b2 - b0
          sts128(st + G::BSUM + o2, sub4(e2, d2));
          sts128(st + G::B2 + o1, add4(d1, f1));    // b0 + b1
          sts128(st + G::B2 + o2, add4(d2, f2));
          sts128(st + G::BH + o1, add4(d2, h1));    // (b0 + b3) right chunk
        }
      }
      // Make the generic-proxy writes visible to the tensor core, then signal.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(G::SUMS + s));
    }

    // ------------------------------------------------------------ epilogue
    if (ok && warp_wait(bar(G::ACC), 0, abort_flag, p.err, kErrWaitAcc)) {
      tc_fence_after();
      // Our stages are idle now (every MMA retired, every copy consumed): let
      // the peer write its partial into them.
      if (lane == 0) mbar_remote_arrive(mapa_shared(bar(G::XFREE), peer));
      const int h = set;                        // columns [64h, 64h + 64) of the product tile
      const bool mine = (uint32_t)h == rank;    // this half holds our 64 columns of P1
      const uint32_t tmem_row = tmem_base + ((uint32_t)(32 * q) << 16);
      const uint32_t xrow = smem_base + row * kXRowBytes;
      if (warp_wait_cluster(bar(G::XFREE), 0, abort_flag, p.err, kErrPairExchange)) {
#pragma unroll 1
        for (int j = 0; j < 8; ++j) {
          const int col = 64 * h + 8 * j;
          float y[8], m1[8];
          tmem_load_8(tmem_row + (rank ? 128u : 0u) + col, y);  // CTA 0: M3, CTA 1: M4
          if (mine) {
            tmem_load_8(tmem_row + 384u + (col - 64 * (int)rank), m1);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] += m1[e];
          }
          st_cluster_f32x4(mapa_shared(xrow + col * 4, peer), y[0], y[1], y[2], y[3]);
          st_cluster_f32x4(mapa_shared(xrow + col * 4 + 16, peer), y[4], y[5], y[6], y[7]);
        }
        mbar_remote_arrive(mapa_shared(bar(G::XDATA), peer));
        if (warp_wait_cluster(bar(G::XDATA), 0, abort_flag, p.err, kErrPairExchange)) {
          const int t = t0 + (int)row;
          const bool row_ok = t < p.Mp;
          const int blk_i = t / p.half_bm;
          const int64_t out_row = (int64_t)blk_i * p.bm + (t - blk_i * p.half_bm) + (rank ? p.half_bm : 0);
          const int j_block = u0 / p.half_bn;
          const int64_t col_left0 = (int64_t)j_block * p.bn + (u0 - j_block * p.half_bn);
#pragma unroll 1
          for (int j = 0; j < 8; ++j) {
            const int col = 64 * h + 8 * j;
            float d0[8], d1[8], d2[8], m1[8], left[8], right[8];
            tmem_load_8(tmem_row + col, d0);
            tmem_load_8(tmem_row + 128u + col, d1);
            tmem_load_8(tmem_row + 256u + col, d2);
            if (mine) tmem_load_8(tmem_row + 384u + (col - 64 * (int)rank), m1);
            const float4 ya = lds_f32x4(xrow + col * 4), yb = lds_f32x4(xrow + col * 4 + 16);
            const float yin[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float z = mine ? yin[e] + m1[e] : yin[e];
              if (rank == 0) {
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
    }
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  // Neither CTA leaves while the other may still write into its shared memory
  // or arrive on its barriers.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if (lane == 0) mbar_wait_drain(bar(G::ACC), 0);  // every issued MMA has retired
    __syncwarp();
    tmem_dealloc<kTmemCols>(tmem_base);
  }
}
