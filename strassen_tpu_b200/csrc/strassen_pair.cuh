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
// half the instructions per unit of work of the one-CTA kernel.
//
// Operands.  CTA r TMA-loads only half of what the pair needs -- the A
// quadrants of row half r (a0, a1 or a2, a3) and the B quadrants of column
// half 1 - r (b1, b3 or b0, b2) -- and forwards the part its peer also needs
// (CTA 0: a0, b1, b3's right half; CTA 1: a3, b2, b0's left half) from its own
// shared memory into the peer's with one shared-to-shared bulk copy per tile
// (one source, one destination CTA per copy).
// Every operand crosses the L2 once per pair instead of once per CTA.
//
// Operand sums, formed by the sum warps with one RNE bf16 rounding each (the
// reference's pre-add rounding):
//   A (into a two-step TMEM ring): CTA 0 a0+a1, a1-a3, a0+a3; CTA 1 a2+a3,
//     a2-a0, a0+a3.
//   B (shared memory; never over a tile that is forwarded): CTA 0 b1-b3 into
//     the sum slot, b2+b3 over the received b2, (b0+b3)L over the received
//     b0L; CTA 1 b2-b0 into the sum slot, b0+b1 over the received b1,
//     (b0+b3)R over the received b3R.
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
//   own[s]   own TMA landed (16 KB per step);
//   full[s]  own data landed (the forwarder's arrival) + the producer's
//            arrival expecting the peer's 10 KB + those bytes;
//   sums[s]  the four sum warps of the step's set; empty[s] local MMA commit;
//   pfree[s] the peer's producer: its stage s may be overwritten by our
//            forward (remote arrival, cluster scope);
//   xfree / xdata  the epilogue exchange (remote arrivals, cluster scope).
// Both CTAs end with a cluster barrier, so neither leaves while the other may
// still touch its shared memory.
//
// Roles: warp 0 TMA producer, warp 1 TMEM allocation + MMA issue, warp 2
// forwarder, warps 4-11 operand sums then epilogue (as in the one-CTA kernel).
//
// Included by strassen_gemm.cu inside namespace sb, after the one-CTA kernel
// (it uses its constants, GemmParams and store helpers).

namespace pair {

constexpr int kCols = 128;                         // product columns per CTA pair
constexpr int kATile = kBlockM * 16 * 2;           // 4 KB: 128 x 16 A quadrant tile (32-byte swizzle)
constexpr int kBTile = 16 * kCols * 2;             // 4 KB: 16 x 128 B quadrant tile (two 64-column chunks)
constexpr int kBHalf = kBTile / 2;                 // 2 KB: one 64-column chunk
// Stage layout (byte offsets), the same in both CTAs.
constexpr int kAOwn = 0;                           // A quadrants (r, 0), (r, 1)
constexpr int kARecv = 2 * kATile;                 // A quadrant from the peer (CTA 0: a3, CTA 1: a0)
constexpr int kBOwn = 3 * kATile;                  // B quadrants (0, 1-r), (1, 1-r)
constexpr int kBRecvF = kBOwn + 2 * kBTile;        // full B tile from the peer (CTA 0: b2, CTA 1: b1)
constexpr int kBRecvH = kBRecvF + kBTile;          // half B tile from the peer (CTA 0: b0L, CTA 1: b3R)
constexpr int kBSum = kBRecvH + kBHalf;            // B sum slot (CTA 0: b1-b3, CTA 1: b2-b0)
constexpr int kStageBytes = kBSum + kBTile;        // 30 KB
constexpr int kOwnTx = 2 * kATile + 2 * kBTile;    // bytes landed by the CTA's own TMA per step
constexpr int kRecvTx = kATile + kBTile + kBHalf;  // bytes forwarded by the peer per step
#ifndef SB_PAIR_STAGES
#define SB_PAIR_STAGES 7
#endif
constexpr int kStages = SB_PAIR_STAGES;
constexpr int kBarBytes = 512;
constexpr int kDataBytes = kStages * kStageBytes;
constexpr int kSmem = kDataBytes + kBarBytes + 1024;  // + alignment slack
constexpr int kXRowBytes = kCols * 4 + 16;            // exchange row: 128 fp32 + 16 B (bank spread)
constexpr uint32_t kIdesc128 = umma_idesc_bf16_f32(kBlockM, 128, false, true);
constexpr uint32_t kIdesc64 = umma_idesc_bf16_f32(kBlockM, 64, false, true);
constexpr uint32_t kBLbo = 2048;  // MN-major 128-byte swizzle: offset of the next 64-column chunk
constexpr uint32_t kBSbo = 1024;  // next 8 k-rows
constexpr uint32_t kALbo = 16, kASbo = 256;  // K-major 32-byte swizzle rows (LBO unused)
// Barrier slots (8 bytes each) after the stages.
constexpr int kBarFull = 0, kBarOwn = kStages, kBarSums = 2 * kStages, kBarEmpty = 3 * kStages,
              kBarPfree = 4 * kStages, kBarAcc = 5 * kStages, kBarXfree = kBarAcc + 1,
              kBarXdata = kBarAcc + 2, kBarWords = kBarAcc + 3;
static_assert(kStageBytes % 1024 == 0 && kBOwn % 1024 == 0 && kBRecvF % 1024 == 0 && kBRecvH % 1024 == 0 &&
                  kBSum % 1024 == 0,
              "128-byte swizzle atoms need 1024-byte aligned tiles");
static_assert(kBarWords * 8 + 16 <= kBarBytes, "barrier area");
static_assert(kBlockM * kXRowBytes <= kDataBytes, "exchange buffer fits in the idle stages");
static_assert(kSmem <= 227 * 1024, "shared memory budget");
static_assert(kRingCol0 + 32 + 24 <= kTmemCols, "two-step ring of three A operands");

enum : int {
  kErrPairForward = 5,   // forwarder: own TMA or the peer's stage release never came
  kErrPairExchange = 6,  // epilogue exchange with the peer timed out
};

// Every lane waits itself with cluster-scope acquire (the peer's writes into
// this CTA's shared memory must be visible to each lane afterwards).
__device__ __forceinline__ bool warp_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err, int code) {
  return __all_sync(0xffffffffu, mbar_wait_cluster(bar, parity, abort_flag, err, code));
}

}  // namespace pair

template <bool kOutF32>
__global__ void __launch_bounds__(kThreads, 1)
    strassen_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const GemmParams p) {
  using namespace pair;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t smem_base = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDataBytes);
  const uint32_t bar0 = smem_addr(bars);
  auto bar = [&](int slot) -> uint32_t { return bar0 + 8u * (uint32_t)slot; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kBarWords);
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
      mbar_init(bar(kBarFull + s), 2);
      mbar_init(bar(kBarOwn + s), 1);
      mbar_init(bar(kBarSums + s), 4);
      mbar_init(bar(kBarEmpty + s), 1);
      mbar_init(bar(kBarPfree + s), 1);
    }
    mbar_init(bar(kBarAcc), 1);
    mbar_init(bar(kBarXfree), kSumWarps);
    mbar_init(bar(kBarXdata), kSumThreads);
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
  // The peer's barriers must be initialised before the first remote arrival
  // or forwarded byte reaches them.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  bool ok = true;
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int last_armed[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) last_armed[s] = -1;
      const int a_row_base = t0 % p.half_bm;
      const int a_block = t0 / p.half_bm;
      const int j_block = u0 / p.half_bn;
      const int b_chunk0 = (j_block * p.bn + (u0 - j_block * p.half_bn)) / 64;
      for (int c = 0; c < p.num_chunks; ++c) {
        const int s = c % kStages;
        if (!mbar_wait(bar(kBarEmpty + s), ((c / kStages) & 1u) ^ 1u, abort_flag, p.err, kErrWaitEmpty)) break;
        // Our stage s is free: the peer may forward this phase's tiles into it.
        mbar_remote_arrive(mapa_shared(bar(kBarPfree + s), peer));
        const int kap = c * 16;
        const int panel = kap / p.half_bk;
        const int kcol = panel * p.bk + (kap - panel * p.half_bk);
        const uint32_t stage = smem_base + s * kStageBytes;
        mbar_arrive_expect_tx(bar(kBarOwn + s), kOwnTx);
        tma_load_5d(stage + kAOwn, &tmap_a, bar(kBarOwn + s), kcol, a_row_base, a_block, 0, (int)rank);
        tma_load_5d(stage + kBOwn, &tmap_b, bar(kBarOwn + s), 0, kcol, b_chunk0, (int)peer, 0);
        mbar_arrive_expect_tx(bar(kBarFull + s), kRecvTx);
        last_armed[s] = c;
      }
      // Drain: no TMA write may land after teardown.
#pragma unroll
      for (int s = 0; s < kStages; ++s)
        if (last_armed[s] >= 0) mbar_wait_drain(bar(kBarOwn + s), (last_armed[s] / kStages) & 1u);
      // After a failure, give the peer's forwards into our stages time to land
      // (a phase we armed and never consumed; bounded).
      if (*abort_flag) {
#pragma unroll
        for (int s = 0; s < kStages; ++s)
          if (last_armed[s] >= 0) mbar_wait_drain(bar(kBarFull + s), (last_armed[s] / kStages) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint64_t a_d0 = umma_smem_desc(smem_base, kALbo, kASbo, kLayoutSwizzle32B);
      const uint64_t b_d0 = umma_smem_desc(smem_base, kBLbo, kBSbo, kLayoutSwizzle128B);
      // Per rank: accumulator 0 and 1 -- one from the A ring, one with A in
      // shared memory (CTA 0: P3 ss, P5 ts; CTA 1: P2 ts, P4 ss).
      const uint64_t ss_a = (uint64_t)((kAOwn + (rank ? kATile : 0)) >> 4);    // a0 or a3
      const uint64_t ss_b = (uint64_t)(kBSum >> 4);
      const uint64_t ts_b = (uint64_t)((kBOwn + (rank ? 0 : kBTile)) >> 4);     // b3 or b0
      const uint32_t ss_d = tmem_base + (rank ? 128u : 0u);
      const uint32_t ts_d = tmem_base + (rank ? 0u : 128u);
      int s = 0;
      uint32_t ph = 0;
      for (int c = 0; c < p.num_chunks; ++c) {
        if (!mbar_wait(bar(kBarSums + s), ph, abort_flag, p.err, kErrWaitSums)) break;
        tc_fence_after();
        const uint64_t so = (uint64_t)((s * kStageBytes) >> 4);
        const uint32_t acc = c != 0 ? 1u : 0u;
        const uint32_t ring = tmem_base + kRingCol0 + 32u * (uint32_t)(c & 1);
        umma_bf16_ss(ss_d, a_d0 + so + ss_a, b_d0 + so + ss_b, kIdesc128, acc);
        umma_bf16_ts(ts_d, ring + 0, b_d0 + so + ts_b, kIdesc128, acc);
        umma_bf16_ts(tmem_base + 256, ring + 8, b_d0 + so + (uint64_t)(kBRecvF >> 4), kIdesc128, acc);
        umma_bf16_ts(tmem_base + 384, ring + 16, b_d0 + so + (uint64_t)(kBRecvH >> 4), kIdesc64, acc);
        umma_commit(bar(kBarEmpty + s));
        if (++s == kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      // Always commit: the epilogue (or the teardown drain) waits on it.
      umma_commit(bar(kBarAcc));
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ forwarder
    if (lane == 0) {
      const uint32_t a_src = kAOwn + (rank ? kATile : 0);                 // CTA 0: a0, CTA 1: a3
      const uint32_t f_src = kBOwn + (rank ? kBTile : 0);                 // CTA 0: b1, CTA 1: b2
      const uint32_t h_src = kBOwn + (rank ? 0 : kBTile + kBHalf);        // CTA 0: b3R, CTA 1: b0L
      for (int c = 0; c < p.num_chunks; ++c) {
        const int s = c % kStages;
        const uint32_t ph = (c / kStages) & 1u;
        if (!mbar_wait(bar(kBarOwn + s), ph, abort_flag, p.err, kErrPairForward)) break;
        if (!mbar_wait_cluster(bar(kBarPfree + s), ph, abort_flag, p.err, kErrPairForward)) break;
        const uint32_t so = (uint32_t)(s * kStageBytes);
        const uint32_t peer_full = mapa_shared(bar(kBarFull + s), peer);
        const uint32_t local = smem_base + so;
        bulk_copy_to_peer(mapa_shared(local + kARecv, peer), local + a_src, kATile, peer_full);
        bulk_copy_to_peer(mapa_shared(local + kBRecvF, peer), local + f_src, kBTile, peer_full);
        bulk_copy_to_peer(mapa_shared(local + kBRecvH, peer), local + h_src, kBHalf, peer_full);
        mbar_arrive(bar(kBarFull + s));  // our own half of stage s has landed
      }
    }
  } else if (warp >= kFirstSumWarp) {
    // ------------------------------------------------------------ operand sums
    const int set = (warp - kFirstSumWarp) >> 2;
    const int q = warp & 3;
    const uint32_t row = 32 * q + lane;  // product row = TMEM lane; also the B chunk index
    const uint32_t sw = (row >> 2) & 1u;  // 32-byte swizzle: the row's two chunks swap on bit 2
    const uint32_t lo_off = 32 * row + 16 * sw;
    const uint32_t hi_off = 32 * row + 16 * (sw ^ 1u);
    const uint32_t tmem_lane = tmem_base + ((uint32_t)(32 * q) << 16) + kRingCol0;
    const uint32_t o1 = 16 * row, o2 = o1 + kBHalf;
    for (int c = set; c < p.num_chunks; c += 2) {
      const int s = c % kStages;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(bar(kBarFull + s), (c / kStages) & 1u, abort_flag, p.err, kErrWaitRaw))) {
        ok = false;
        break;
      }
      const uint32_t st = smem_base + s * kStageBytes;
      // A: x0, x1 own (quadrants (r,0), (r,1)), x2 received.
      const uint4 x0l = lds128(st + kAOwn + lo_off), x0h = lds128(st + kAOwn + hi_off);
      const uint4 x1l = lds128(st + kAOwn + kATile + lo_off), x1h = lds128(st + kAOwn + kATile + hi_off);
      const uint4 x2l = lds128(st + kARecv + lo_off), x2h = lds128(st + kARecv + hi_off);
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
      // B: d = own quadrant (0, 1-r), e = own (1, 1-r), f = received full, h = received half.
      const uint32_t bo = st + kBOwn;
      const uint4 d1 = lds128(bo + o1), d2 = lds128(bo + o2);
      const uint4 e1 = lds128(bo + kBTile + o1), e2 = lds128(bo + kBTile + o2);
      const uint4 f1 = lds128(st + kBRecvF + o1), f2 = lds128(st + kBRecvF + o2);
      const uint4 h1 = lds128(st + kBRecvH + o1);
      if (rank == 0) {
        sts128(st + kBSum + o1, sub4(d1, e1));    // b1 - b3
        sts128(st + kBSum + o2, sub4(d2, e2));
        sts128(st + kBRecvF + o1, add4(f1, e1));  // b2 + b3
        sts128(st + kBRecvF + o2, add4(f2, e2));
        sts128(st + kBRecvH + o1, add4(h1, e1));  // (b0 + b3) left chunk
      } else {
        sts128(st + kBSum + o1, sub4(e1, d1));    // b2 - b0
        sts128(st + kBSum + o2, sub4(e2, d2));
        sts128(st + kBRecvF + o1, add4(d1, f1));  // b0 + b1
        sts128(st + kBRecvF + o2, add4(d2, f2));
        sts128(st + kBRecvH + o1, add4(d2, h1));  // (b0 + b3) right chunk
      }
      fence_proxy_async_smem();
      // Ring half c & 1 is free once the MMAs of step c - 2 completed.
      if (c >= 2) {
        const bool waited = mbar_wait(bar(kBarEmpty + (c - 2) % kStages), ((c - 2) / kStages) & 1u, abort_flag,
                                      p.err, kErrWaitEmpty);
        if (!__all_sync(0xffffffffu, waited)) {
          ok = false;
          break;
        }
      }
      tc_fence_after();
      const uint32_t ring = tmem_lane + 32u * (uint32_t)(c & 1);
      tmem_store_8(ring + 0, r0l, r0h);
      tmem_store_8(ring + 8, r1l, r1h);
      tmem_store_8(ring + 16, r2l, r2h);
      tmem_store_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarSums + s));
    }

    // ------------------------------------------------------------ epilogue
    if (ok && warp_wait(bar(kBarAcc), 0, abort_flag, p.err, kErrWaitAcc)) {
      tc_fence_after();
      // Our stages are idle now: let the peer write its partial into them.
      if (lane == 0) mbar_remote_arrive(mapa_shared(bar(kBarXfree), peer));
      const int h = set;                        // columns [64h, 64h + 64) of the product tile
      const bool mine = (uint32_t)h == rank;    // this half holds our 64 columns of P1
      const uint32_t tmem_row = tmem_base + ((uint32_t)(32 * q) << 16);
      const uint32_t xrow = smem_base + row * kXRowBytes;
      if (warp_wait_cluster(bar(kBarXfree), 0, abort_flag, p.err, kErrPairExchange)) {
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
        mbar_remote_arrive(mapa_shared(bar(kBarXdata), peer));
        if (warp_wait_cluster(bar(kBarXdata), 0, abort_flag, p.err, kErrPairExchange)) {
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
    if (lane == 0) mbar_wait_drain(bar(kBarAcc), 0);  // every issued MMA has retired
    __syncwarp();
    tmem_dealloc<kTmemCols>(tmem_base);
  }
}
