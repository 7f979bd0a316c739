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
// Two producer threads (warps 0 and 2) issue the copies and arm the stage's
// barrier together.  The A sums (CTA 0: a0+a1, a1-a3, a0+a3; CTA 1: a2+a3,
// a2-a0, a0+a3) go to a two-step TMEM ring and feed A-from-TMEM MMAs; the raw
// a0 (CTA 0) or a3 (CTA 1) is read from shared memory.  Every pre-add is one
// RNE bf16 rounding, the reference's pre-add rounding.
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
//   full[s]  both producers' arrivals + the stage's TMA bytes;
//   sums[s]  the four sum warps of the step's set; empty[s] local MMA commit;
//   xfree / xdata  the epilogue exchange: remote arrivals from the peer, waited
//            with cluster-scope acquire.
// The K loop never waits on the peer.  Both CTAs end with a cluster barrier,
// so neither leaves while the other may still write into its shared memory.
//
// Roles: warps 0 and 2 TMA producers, warp 1 TMEM allocation + MMA issue,
// warps 4-11 operand sums then epilogue (as in the one-CTA kernel).
//
// Included by strassen_gemm.cu inside namespace sb, after the one-CTA kernel
// (it uses its constants, GemmParams and store helpers).

namespace pair {

constexpr int kCols = 128;  // product columns per CTA pair
// Stage depth of the planes mode: 16 (eight 26 KB stages, the default) or 32
// (four 52 KB stages with 64-byte A rows: half the TMA requests per byte,
// measured 2-6 % slower at 8192^3 -- depth in stages matters more).
#ifndef SB_PAIR_PLANES_KD
#define SB_PAIR_PLANES_KD 16
#endif
// Stage geometry.  A stage holds KD (16 or 32) product-depth columns of every
// operand; the MMAs and the A-sum ring work in 16-deep sub-steps (two per stage
// when KD = 32).  Byte offsets, the same in both CTAs:
//   AOWN  A quadrants (r, 0), (r, 1)           ARECV the third A quadrant
//   B0..B2 three B tiles (128 columns)          BH    the 64-column half tile for P1
//   BSUM  (raw B only) the B sum slot
// Raw B (kPreB = false, KD = 16): B0/B1 own quadrants (0, 1-r), (1, 1-r), B2 the
// other full quadrant.  Planes (kPreB = true): B0..B2 the operand planes of the
// CTA's three full products (CTA 0: P3, P5, P7; CTA 1: P2, P4, P6), BH P1's.
// KD = 32 gives the A tiles 64-byte rows (half the TMA requests of 32-byte rows).
template <bool kPreB>
struct Geo {
  static constexpr int KD = kPreB ? SB_PAIR_PLANES_KD : 16;
  static constexpr int SUB = KD / 16;                    // 16-deep sub-steps per stage
  static constexpr int ATILE = kBlockM * KD * 2;         // 128 rows x KD, K-major
  static constexpr int BTILE = KD * kCols * 2;           // KD rows x 128 columns, two 64-column chunks
  static constexpr int BHALF = BTILE / 2;
  static constexpr int AOWN = 0, ARECV = 2 * ATILE, B0 = 3 * ATILE, B1 = B0 + BTILE, B2 = B1 + BTILE,
                       BH = B2 + BTILE, BSUM = BH + BHALF;
  static constexpr int STAGE = kPreB ? BSUM : BSUM + BTILE;  // 26 or 52 KB (planes), 30 KB (raw)
  static constexpr int STAGES = kPreB ? (KD == 32 ? 4 : 8) : 7;
  static constexpr int DATA = STAGES * STAGE;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = DATA + BAR_BYTES + 1024;  // + alignment slack
  static constexpr int TX0 = 2 * ATILE + (kPreB ? 3 : 2) * BTILE;   // producer 0 (warp 0)
  static constexpr int TX1 = ATILE + (kPreB ? 0 : BTILE) + BHALF;   // producer 1 (warp 2)
  // A tiles: 32- or 64-byte rows (swizzle span); 8-row core groups.
  static constexpr uint32_t A_LAYOUT = KD == 32 ? kLayoutSwizzle64B : kLayoutSwizzle32B;
  static constexpr uint32_t A_SBO = 8 * KD * 2;
  static constexpr uint32_t B_LBO = KD * 128;  // MN-major 128-byte swizzle: next 64-column chunk
  // Barrier slots (8 bytes each) after the stages.  RING0: the commit after a
  // stage's first sub-step (KD = 32), which frees ring half 0.
  static constexpr int FULL = 0, SUMS = STAGES, EMPTY = STAGES * (1 + SUB), RING0 = EMPTY + STAGES,
                       ACC = RING0 + STAGES, XFREE = ACC + 1, XDATA = ACC + 2, WORDS = ACC + 3;
  static_assert(KD == 16 || (KD == 32 && kPreB), "32-deep stages need the B operand planes");
  static_assert(STAGE % 1024 == 0 && B0 % 1024 == 0 && BH % 1024 == 0 && BSUM % 1024 == 0,
                "128-byte swizzle atoms need 1024-byte aligned tiles");
  static_assert(WORDS * 8 + 16 <= BAR_BYTES, "barrier area");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};
constexpr int kXRowBytes = kCols * 4 + 16;  // exchange row: 128 fp32 + 16 B (bank spread)
static_assert(kBlockM * kXRowBytes <= Geo<true>::DATA && kBlockM * kXRowBytes <= Geo<false>::DATA,
              "exchange buffer fits in the idle stages");
constexpr uint32_t kIdesc128 = umma_idesc_bf16_f32(kBlockM, 128, false, true);
constexpr uint32_t kIdesc64 = umma_idesc_bf16_f32(kBlockM, 64, false, true);
constexpr uint32_t kBSbo = 1024;  // next 8 k-rows of a 128-byte-swizzled B tile
constexpr uint32_t kALbo = 16;    // unused for swizzled K-major A
static_assert(kRingCol0 + 32 + 24 <= kTmemCols, "two-step ring of three A operands");
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
__global__ void __launch_bounds__(kThreads, 1)
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
      mbar_init(bar(G::FULL + s), 2);
      for (int h = 0; h < G::SUB; ++h) mbar_init(bar(G::SUMS + s * G::SUB + h), 4);
      mbar_init(bar(G::EMPTY + s), 1);
      mbar_init(bar(G::RING0 + s), 1);
    }
    mbar_init(bar(G::ACC), 1);
    mbar_init(bar(G::XFREE), kSumWarps);
    mbar_init(bar(G::XDATA), kSumThreads);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if ((warp == 0 || warp == 2) && lane == 0) {
    tma_prefetch_desc(warp == 0 ? &tmap_a : &tmap_a1);
    tma_prefetch_desc(warp == 0 ? &tmap_b : &tmap_bh);
  }
  if (warp == 1) tmem_alloc<kTmemCols>(smem_addr(tmem_holder));
  tc_fence_before();
  // The peer's barriers must be initialised before its epilogue exchange can
  // reach them.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  bool ok = true;
  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ TMA producers
    if (lane == 0) {
      const bool first = warp == 0;
      int last_armed[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) last_armed[s] = -1;
      const int a_row_base = t0 % p.half_bm;
      const int a_block = t0 / p.half_bm;
      const int j_block = u0 / p.half_bn;
      const int b_chunk0 = (j_block * p.bn + (u0 - j_block * p.half_bn)) / 64;  // raw-B column chunk
      const int num_stages = p.num_chunks / G::SUB;  // num_chunks counts 16-deep steps
      for (int c = 0; c < num_stages; ++c) {
        const int s = c % kStages;
        if (!mbar_wait(bar(G::EMPTY + s), ((c / kStages) & 1u) ^ 1u, abort_flag, p.err, kErrWaitEmpty)) break;
        const uint32_t stage = smem_base + s * G::STAGE;
        const uint32_t fb = bar(G::FULL + s);
        const int kap = c * G::KD;  // a stage never straddles a K panel: half_bk is a multiple of 128
        const int panel = kap / p.half_bk;
        const int kcol = panel * p.bk + (kap - panel * p.half_bk);
        if (first) {
          mbar_arrive_expect_tx(fb, G::TX0);
          tma_load_5d(stage + G::AOWN, &tmap_a, fb, kcol, a_row_base, a_block, 0, (int)rank);
          if constexpr (kPreB) {
            tma_load_4d(stage + G::B0, &tmap_b, fb, 0, kap, u0 / 64, rank ? kPlaneP2 : kPlaneP3);
          } else {
            tma_load_5d(stage + G::B0, &tmap_b, fb, 0, kcol, b_chunk0, (int)peer, 0);
          }
        } else {
          mbar_arrive_expect_tx(fb, G::TX1);
          tma_load_5d(stage + G::ARECV, &tmap_a1, fb, kcol, a_row_base, a_block, (int)peer, (int)peer);
          if constexpr (kPreB) {
            tma_load_4d(stage + G::BH, &tmap_bh, fb, 0, kap, u0 / 64 + (int)rank, kPlaneP1);
          } else {
            tma_load_5d(stage + G::B2, &tmap_b1, fb, 0, kcol, b_chunk0, (int)rank, (int)peer);
            tma_load_5d(stage + G::BH, &tmap_bh, fb, 0, kcol, b_chunk0 + (int)rank, (int)rank, (int)rank);
          }
        }
        last_armed[s] = c;
      }
      // Drain: no TMA write may land after teardown (bounded: a phase the
      // other producer never armed gives up after the wait limit).
#pragma unroll
      for (int s = 0; s < kStages; ++s)
        if (last_armed[s] >= 0) mbar_wait_drain(bar(G::FULL + s), (last_armed[s] / kStages) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint64_t a_d0 = umma_smem_desc(smem_base, kALbo, G::A_SBO, G::A_LAYOUT);
      const uint64_t b_d0 = umma_smem_desc(smem_base, G::B_LBO, kBSbo, kLayoutSwizzle128B);
      // Accumulators 0 and 1: one with A in shared memory, one from the A ring
      // (CTA 0: M3 = a0 x B0 ss, M5 = ring0 x B1; CTA 1: M2 = ring0 x B0,
      // M4 = a3 x B1 ss).  B tile of each accumulator per mode (see Geo).
      const uint64_t ss_a = (uint64_t)((G::AOWN + (rank ? G::ATILE : 0)) >> 4);  // a0 or a3
      int ss_bo, ts_bo;
      if (kPreB) {
        ss_bo = rank ? G::B1 : G::B0;
        ts_bo = rank ? G::B0 : G::B1;
      } else {
        ss_bo = G::BSUM;               // b1-b3 or b2-b0
        ts_bo = rank ? G::B0 : G::B1;  // b0 (own quadrant 0 of CTA 1) or b3 (own quadrant 1 of CTA 0)
      }
      const uint64_t ss_b = (uint64_t)(ss_bo >> 4), ts_b = (uint64_t)(ts_bo >> 4);
      const uint64_t b2_b = (uint64_t)(G::B2 >> 4), bh_b = (uint64_t)(G::BH >> 4);
      const uint32_t ss_d = tmem_base + (rank ? 128u : 0u);
      const uint32_t ts_d = tmem_base + (rank ? 0u : 128u);
      // One pass per 16-deep sub-step g: stage g / SUB, half h = g % SUB.  Within
      // a stage, sub-step h starts 16 K columns in: +32 bytes along a K-major A
      // row, +16 rows (2048 bytes) of an MN-major B tile.
      int s = 0, h = 0;
      uint32_t ph = 0;
      for (int g = 0; g < p.num_chunks; ++g) {
        if (!mbar_wait(bar(G::SUMS + s * G::SUB + h), ph, abort_flag, p.err, kErrWaitSums)) break;
        tc_fence_after();
        const uint64_t so = (uint64_t)((s * G::STAGE) >> 4);
        const uint64_t ka = (uint64_t)(h * 2), kb = (uint64_t)(h * 128);
        const uint32_t acc = g != 0 ? 1u : 0u;
        const uint32_t ring = tmem_base + kRingCol0 + 32u * (uint32_t)(g & 1);
        umma_bf16_ss(ss_d, a_d0 + so + ss_a + ka, b_d0 + so + ss_b + kb, kIdesc128, acc);
        umma_bf16_ts(ts_d, ring + 0, b_d0 + so + ts_b + kb, kIdesc128, acc);
        umma_bf16_ts(tmem_base + 256, ring + 8, b_d0 + so + b2_b + kb, kIdesc128, acc);
        umma_bf16_ts(tmem_base + 384, ring + 16, b_d0 + so + bh_b + kb, kIdesc64, acc);
        // The last sub-step of a stage frees the stage (and its ring half); an
        // earlier one frees ring half 0 only.
        if (h == G::SUB - 1) {
          umma_commit(bar(G::EMPTY + s));
        } else {
          umma_commit(bar(G::RING0 + s));
        }
        if (++h == G::SUB) {
          h = 0;
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Always commit: the epilogue (or the teardown drain) waits on it.
      umma_commit(bar(G::ACC));
    }
  } else if (warp >= kFirstSumWarp) {
    // ------------------------------------------------------------ operand sums
    const int set = (warp - kFirstSumWarp) >> 2;
    const int q = warp & 3;
    const uint32_t row = 32 * q + lane;  // product row = TMEM lane; also the B chunk index
    // The two 16-byte chunks of this row's 16-deep slice in a swizzled A tile.
    // 32-byte rows (KD = 16): the chunks swap on row bit 2.  64-byte rows
    // (KD = 32): chunk j sits at j ^ ((row >> 1) & 3); a set always takes the
    // same half h = set of a stage, so its offsets are fixed.
    uint32_t lo_off, hi_off;
    if constexpr (G::KD == 32) {
      const uint32_t sw = (row >> 1) & 3u;
      lo_off = 64 * row + 16 * ((2u * set) ^ sw);
      hi_off = 64 * row + 16 * ((2u * set + 1u) ^ sw);
    } else {
      const uint32_t sw = (row >> 2) & 1u;
      lo_off = 32 * row + 16 * sw;
      hi_off = 32 * row + 16 * (sw ^ 1u);
    }
    const uint32_t tmem_lane = tmem_base + ((uint32_t)(32 * q) << 16) + kRingCol0;
    const uint32_t o1 = 16 * row, o2 = o1 + G::BHALF;
    // Sub-steps g = set, set + 2, ...: stage g / SUB, half g % SUB.
    for (int g = set; g < p.num_chunks; g += 2) {
      const int stage_i = g / G::SUB, h = g % G::SUB;
      const int s = stage_i % kStages;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(bar(G::FULL + s), (stage_i / kStages) & 1u, abort_flag, p.err, kErrWaitRaw))) {
        ok = false;
        break;
      }
      const uint32_t st = smem_base + s * G::STAGE;
      // A: x0, x1 = quadrants (r, 0), (r, 1); x2 = the third quadrant.
      const uint4 x0l = lds128(st + G::AOWN + lo_off), x0h = lds128(st + G::AOWN + hi_off);
      const uint4 x1l = lds128(st + G::AOWN + G::ATILE + lo_off), x1h = lds128(st + G::AOWN + G::ATILE + hi_off);
      const uint4 x2l = lds128(st + G::ARECV + lo_off), x2h = lds128(st + G::ARECV + hi_off);
      uint4 r0l, r0h, r1l, r1h, r2l, r2h;
      r0l = add4(x0l, x1l);  // CTA 0: a0+a1   CTA 1: a2+a3
      r0h = add4(x0h, x1h);
      if (rank == 0) {
        r1l = sub4(x1l, x2l); r1h = sub4(x1h, x2h);  // a1-a3
        r2l = add4(x0l, x2l); r2h = add4(x0h, x2h);  // a0+a3
      } else {
        r1l = sub4(x0l, x2l); r1h = sub4(x0h, x2h);  // a2-a0
        r2l = add4(x1l, x2l); r2h = add4(x1h, x2h);  // a3+a0
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
        fence_proxy_async_smem();
      }
      // Ring half g & 1 is free once the MMAs of sub-step g - 2 completed: the
      // stage commit if that was its stage's last sub-step, else RING0.
      if (g >= 2) {
        const int ps = (g - 2) / G::SUB, ph_ = (g - 2) % G::SUB;
        const uint32_t free_bar = bar((ph_ == G::SUB - 1 ? G::EMPTY : G::RING0) + ps % kStages);
        const bool waited = mbar_wait(free_bar, (ps / kStages) & 1u, abort_flag, p.err, kErrWaitEmpty);
        if (!__all_sync(0xffffffffu, waited)) {
          ok = false;
          break;
        }
      }
      tc_fence_after();
      const uint32_t ring = tmem_lane + 32u * (uint32_t)(g & 1);
      tmem_store_8(ring + 0, r0l, r0h);
      tmem_store_8(ring + 8, r1l, r1h);
      tmem_store_8(ring + 16, r2l, r2h);
      tmem_store_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(G::SUMS + s * G::SUB + h));
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
