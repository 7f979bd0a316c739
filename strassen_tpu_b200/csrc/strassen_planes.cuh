// strassen_planes.cuh -- Strassen as seven full-width product GEMMs on paired
// tensor cores (sb_strassen_gemm_planes).
//
// Same algorithm, product coordinates, operand values and recombination as the
// one-CTA kernel (strassen_pallas.py:324-379 restated per product over the
// whole K range, recombined once in fp32), organised the way B200's tensor
// cores run fastest: instead of holding all seven product accumulators of a
// small tile in one SM's TMEM (which caps the MMA at N = 64), every product is
// a plain GEMM in product coordinates,
//
//   M_i[t][u] = sum_kappa Aop_i[t][kappa] * Bop_i[kappa][u],   i = 1..7,
//
// run with 256 x 256 tiles on a CTA pair (tcgen05.mma.cta_group::2, M = 256,
// N = 256, 128-byte operand rows) and two TMEM accumulators per SM, so a
// tile's epilogue overlaps the next tile's K loop.  The operands come from
// two passes (A operand planes [7][M/2][K/2], B operand planes [7][K/2][N/2],
// each pre-add rounded once to bf16 as the reference rounds them); the
// products land in an fp32 workspace [7][M/2][N/2]; a last pass recombines
// C11 = M1 + M4 - M5 + M7, C12 = M3 + M5, C21 = M2 + M4,
// C22 = M1 - M2 + M3 + M6 and writes C.  The extra HBM traffic (operand planes
// and fp32 products) is what this layout pays for full-width MMAs.
//
// Roles (256 threads per CTA, one CTA per SM, persistent: a cluster walks the
// tiles cluster_id, cluster_id + clusters, ...):
//   warp 0 lane 0 (both CTAs): TMA producer -- per 64-deep step one A copy (its
//     128 product rows) and one B copy (its 128 of the tile's 256 columns,
//     MN-major, two 64-column chunks); both CTAs' bytes complete on the even
//     CTA's full barrier (.cta_group::2 loads, no multicast);
//   warp 1 lane 0 (even CTA): MMA issuer -- four 256x256x16 MMAs per step into
//     accumulator buffer (tile & 1), one commit per step freeing the stage in
//     both CTAs, one commit per tile to both CTAs' accumulator-full barriers;
//   warps 4-7 (both CTAs): epilogue -- each thread one product row: TMEM ->
//     registers -> fp32 stores, then the buffer is released to the issuer
//     (an arrival on the even CTA's accumulator-empty barrier).
// Every wait is bounded (the library's 1 s rule); a timeout raises the abort
// flag, records an error code and the kernel winds down.

namespace planes {

constexpr int kTileM = 256;   // product rows per cluster tile (128 per CTA)
constexpr int kTileN = 256;   // product columns per cluster tile
constexpr int kBK = 64;       // product depth per pipeline step
constexpr int kStages = 6;
constexpr int kThreads = 256;
constexpr int kFirstEpiWarp = 4;
constexpr int kABytes = 128 * kBK * 2;            // 16 KB: 128 rows x 128 bytes
constexpr int kBBytes = (kTileN / 2) * kBK * 2;   // 16 KB: two 64-column chunks x 64 k-rows
constexpr int kStage = kABytes + kBBytes;
constexpr int kData = kStages * kStage;           // 192 KB
constexpr int kBarBytes = 256;
constexpr int kSmem = kData + kBarBytes + 1024;   // + alignment slack
// Barrier slots.
constexpr int FULL = 0, EMPTY = kStages, ACCF = 2 * kStages, ACCE = ACCF + 2, DRAIN = ACCE + 2, WORDS = DRAIN + 1;
static_assert(WORDS * 8 + 16 <= kBarBytes, "barrier area");
static_assert(kSmem <= 227 * 1024, "shared memory budget");
// M = 256 over the pair, N = 256, A K-major, B MN-major.
constexpr uint32_t kIdesc = umma_idesc_bf16_f32(256, 256, false, true);
constexpr uint32_t kBLbo = kBK * 128;  // next 64-column chunk of the B tile
constexpr uint32_t kSbo = 1024;        // next 8 rows (A) / 8 k-rows (B) of a 128-byte-swizzled tile
// Raster default: product-row tiles per column sweep.
constexpr int kRaster = 8;

// Error codes (sb_device_status) of this kernel's bounded waits.
constexpr int kErrEmpty = 41, kErrFull = 42, kErrAccFull = 43, kErrAccEmpty = 44;

// Order of the B operand planes sb_strassen_b_operands writes (P3, P5, P7, P1,
// P2, P4, P6): plane index of product i (0 = P1 .. 6 = P7).
__host__ __device__ constexpr int b_plane_of(int i) {
  return i == 0 ? 3 : i == 1 ? 4 : i == 2 ? 0 : i == 3 ? 5 : i == 4 ? 1 : i == 5 ? 6 : 2;
}

}  // namespace planes

struct PlanesParams {
  int32_t mh, nh, kh;        // M/2, N/2, K/2
  int32_t tiles_m, tiles_n;  // product tiles of one product
  int32_t num_tiles;         // 7 * tiles_m * tiles_n
  int32_t k_steps;           // kh / kBK
  int32_t raster;
  int32_t tile_m0;           // first product-row tile of this launch (tiles_m tiles from there)
  float* prod;               // [7][mh][nh] fp32
  int* err;
};

// The A operand planes of every Strassen block: aop[i][t][kappa] with
// t = I*bm/2 + r', kappa = P*bk/2 + k' and a_q = A[I*bm + qr*bm/2 + r',
// P*bk + qk*bk/2 + k'] (q = 2 qr + qk):
//   P1 a0+a3, P2 a2+a3, P3 a0, P4 a3, P5 a0+a1, P6 a2-a0, P7 a1-a3,
// each sum rounded once to bf16 (strassen_pallas.py:324-379).  aop is
// [7][M/2][K/2] bf16, contiguous.  One thread per 8 consecutive kappa.
// Product rows t0 <= t < t1 only (the whole array when t0 = 0, t1 = M/2).
__global__ void __launch_bounds__(256) a_operand_planes_kernel(const __nv_bfloat16* __restrict__ a, int64_t lda,
                                                               int32_t m, int32_t k, int32_t bm, int32_t bk,
                                                               __nv_bfloat16* __restrict__ aop, int64_t t0,
                                                               int64_t t1) {
  const int64_t mh = m / 2, kh = k / 2, hbm = bm / 2, hbk = bk / 2;
  const int64_t per_row = kh / 8;
  const int64_t items = (t1 - t0) * per_row;
  const int64_t plane = mh * kh / 8;  // one plane, in uint4 units
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tl = i / per_row;
    const int64_t t = t0 + tl;
    const int64_t kap = (i - tl * per_row) * 8;
    const int64_t blk = t / hbm, pnl = kap / hbk;
    const int64_t row0 = blk * bm + (t - blk * hbm);
    const int64_t col0 = pnl * bk + (kap - pnl * hbk);
    const uint4 a0 = *reinterpret_cast<const uint4*>(a + row0 * lda + col0);
    const uint4 a1 = *reinterpret_cast<const uint4*>(a + row0 * lda + col0 + hbk);
    const uint4 a2 = *reinterpret_cast<const uint4*>(a + (row0 + hbm) * lda + col0);
    const uint4 a3 = *reinterpret_cast<const uint4*>(a + (row0 + hbm) * lda + col0 + hbk);
    uint4* out = reinterpret_cast<uint4*>(aop) + (t * kh + kap) / 8;
    out[0 * plane] = add4(a0, a3);
    out[1 * plane] = add4(a2, a3);
    out[2 * plane] = a0;
    out[3 * plane] = a3;
    out[4 * plane] = add4(a0, a1);
    out[5 * plane] = sub4(a2, a0);
    out[6 * plane] = sub4(a1, a3);
  }
}

// C from the seven fp32 products (product coordinates -> matrix quadrants):
// C11 = M1 + M4 - M5 + M7, C12 = M3 + M5, C21 = M2 + M4, C22 = M1 - M2 + M3 + M6,
// summed left to right in fp32 (the one-CTA kernel's order), then the fused
// epilogue on the fp32 quadrant values exactly as the one-CTA kernel applies
// it (strassen_pallas.py:739-879): residual_add, bias_add, swiglu / geglu
// (quadrants 0/2 gate, 1/3 up; output [M, N/2]) or qk_norm_rope (a head's
// a-half in quadrant 0/2, its b-half at the same offset in 1/3), stored as bf16
// (round to nearest even) or, without an epilogue, fp32.  One thread per 8
// product columns of one product row; a warp covers 256 consecutive columns
// of one row (nh % 256 == 0), so a head slot's sum of squares is a shuffle
// reduction over half_head / 8 neighbouring lanes.  p: C, ldc, bm, bn,
// half_bm, half_bn and the epilogue operands as the one-CTA kernel takes them.
template <int kEpi, bool kOutF32>
__global__ void __launch_bounds__(256) planes_recombine_kernel(const float* __restrict__ prod, int32_t mh, int32_t nh,
                                                               const GemmParams p, int64_t t0, int64_t t1) {
  const int64_t plane = (int64_t)mh * nh;
  const int64_t per_row = nh / 8;
  const int64_t items = (t1 - t0) * per_row;
  const int64_t hbm = p.half_bm, hbn = p.half_bn;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tl = i / per_row;
    const int64_t t = t0 + tl;
    const int64_t u = (i - tl * per_row) * 8;
    const int64_t off = t * nh + u;
    float mv[7][8];
#pragma unroll
    for (int q = 0; q < 7; ++q) {
      const float4 x = *reinterpret_cast<const float4*>(prod + q * plane + off);
      const float4 y = *reinterpret_cast<const float4*>(prod + q * plane + off + 4);
      mv[q][0] = x.x; mv[q][1] = x.y; mv[q][2] = x.z; mv[q][3] = x.w;
      mv[q][4] = y.x; mv[q][5] = y.y; mv[q][6] = y.z; mv[q][7] = y.w;
    }
    Quad8 v;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v.c[0][e] = ((mv[0][e] + mv[3][e]) - mv[4][e]) + mv[6][e];  // C11
      v.c[1][e] = mv[2][e] + mv[4][e];                            // C12
      v.c[2][e] = mv[1][e] + mv[3][e];                            // C21
      v.c[3][e] = ((mv[0][e] - mv[1][e]) + mv[2][e]) + mv[5][e];  // C22
    }
    const int64_t blk_i = t / hbm, blk_j = u / hbn;
    const int64_t cp = u - blk_j * hbn;  // column inside the half block
    const int64_t row_top = blk_i * p.bm + (t - blk_i * hbm), row_bot = row_top + hbm;
    const int64_t cl = blk_j * p.bn + cp, cr = cl + hbn;
    if constexpr (kEpi == SB_EPI_SWIGLU || kEpi == SB_EPI_GEGLU) {
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
      const int64_t oc = blk_j * hbn + cp;
      store8<kOutF32>(p.C, row_top * p.ldc + oc, top);
      store8<kOutF32>(p.C, row_bot * p.ldc + oc, bot);
    } else if constexpr (kEpi == SB_EPI_QK_NORM_ROPE) {
      // Per-head sums of squares over both halves (strassen_pallas.py:793-835):
      // this thread's 8 columns, then the lanes of the same head slot.
      float st = 0.f, sb2 = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        st += v.c[0][e] * v.c[0][e] + v.c[1][e] * v.c[1][e];
        sb2 += v.c[2][e] * v.c[2][e] + v.c[3][e] * v.c[3][e];
      }
      for (int w = 1; w < p.half_head / 8; w <<= 1) {
        st += __shfl_xor_sync(0xffffffffu, st, w);
        sb2 += __shfl_xor_sync(0xffffffffu, sb2, w);
      }
#pragma unroll
      for (int tb = 0; tb < 2; ++tb) {
        const float sums = tb ? sb2 : st;
        const float recip = 1.0f / sqrtf(sums * p.inv_head_dim + p.eps);
        const int64_t row = tb ? row_bot : row_top;
        float outa[8], outb[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float sa = load_aux(p.rope_scale, cp + e, p.aux_f32);
          const float sbv = load_aux(p.rope_scale, hbn + cp + e, p.aux_f32);
          const float cs = load_aux(p.rope_cos, row * p.ld_rope + cp + e, p.aux_f32);
          const float sn = load_aux(p.rope_sin, row * p.ld_rope + cp + e, p.aux_f32);
          const float na = v.c[2 * tb][e] * recip * sa;
          const float nb = v.c[2 * tb + 1][e] * recip * sbv;
          outa[e] = na * cs - nb * sn;
          outb[e] = nb * cs + na * sn;
        }
        store8<kOutF32>(p.C, row * p.ldc + cl, outa);
        store8<kOutF32>(p.C, row * p.ldc + cr, outb);
      }
    } else {
      if constexpr (kEpi == SB_EPI_RESIDUAL_ADD) {
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

__global__ void __launch_bounds__(planes::kThreads, 1)
    strassen_planes_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                                const PlanesParams p) {
  using namespace planes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t smem_base = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kData);
  const uint32_t bar0 = smem_addr(bars);
  auto bar = [&](int slot) -> uint32_t { return bar0 + 8u * (uint32_t)slot; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + WORDS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 or 1
  const bool even = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;
  const int raster = p.raster > 0 ? p.raster : kRaster;

  // Tile index -> (product, first product row, first product column).
  auto decode = [&](int tile, int& prod, int& row0, int& col0) {
    const int per_prod = p.tiles_m * p.tiles_n;
    prod = tile / per_prod;
    const int rem = tile - prod * per_prod;
    const int per_group = raster * p.tiles_n;
    const int group = rem / per_group;
    const int first_m = group * raster;
    const int rows_in_group = min(p.tiles_m - first_m, raster);
    const int in_group = rem - group * per_group;
    row0 = (p.tile_m0 + first_m + in_group % rows_in_group) * kTileM;
    col0 = (in_group / rows_in_group) * kTileN;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(ACCF + b), 1);
      mbar_init(bar(ACCE + b), 2 * (planes::kThreads / 32 - kFirstEpiWarp));  // every epilogue warp of both CTAs
    }
    mbar_init(bar(DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane < 2) tma_prefetch_desc(lane == 0 ? &tmap_a : &tmap_b);
  if (warp == 1) tmem_alloc_pair(smem_addr(tmem_holder));
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers and TMEM exist before any copy, commit or arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t leader = rank & ~1u;
      int it = 0;
      bool ok = true;
      for (int tile = cluster; tile < p.num_tiles && ok; tile += clusters) {
        int prod, row0, col0;
        decode(tile, prod, row0, col0);
        const int a_row = row0 + 128 * (int)rank;
        const int b_chunk = (col0 + 128 * (int)rank) / 64;
        const int b_plane = b_plane_of(prod);
        for (int ks = 0; ks < p.k_steps; ++ks, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(bar(EMPTY + s), ((it / kStages) & 1u) ^ 1u, abort_flag, p.err, kErrEmpty)) {
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(bar(FULL + s), leader);
          if (even) mbar_arrive_expect_tx(bar(FULL + s), 2 * kStage);
          const uint32_t stage = smem_base + s * kStage;
          tma2_load_3d(stage, &tmap_a, fb, ks * kBK, a_row, prod);
          tma2_load_4d(stage + kABytes, &tmap_b, fb, 0, ks * kBK, b_chunk, b_plane);
        }
      }
      // No TMA write may land after teardown (the even CTA's full barriers
      // count both CTAs' bytes).  Bounded.
      if (even) {
        const int first = it > kStages ? it - kStages : 0;
        for (int j = first; j < it; ++j) mbar_wait_drain(bar(FULL + j % kStages), (j / kStages) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1 && even) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint64_t a_d0 = umma_smem_desc(smem_base, 16, kSbo, kLayoutSwizzle128B);
      const uint64_t b_d0 = umma_smem_desc(smem_base + kABytes, kBLbo, kSbo, kLayoutSwizzle128B);
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = cluster; tile < p.num_tiles && ok; tile += clusters, ++lt) {
        const int b = lt & 1;
        // Both CTAs' epilogues arrive from the cluster: acquire at cluster scope.
        if (!mbar_wait_cluster(bar(ACCE + b), ((lt >> 1) & 1u) ^ 1u, abort_flag, p.err, kErrAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(b * 256);
        for (int ks = 0; ks < p.k_steps; ++ks, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(bar(FULL + s), (it / kStages) & 1u, abort_flag, p.err, kErrFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = (uint64_t)((s * kStage) >> 4);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            // K-major A: 32 bytes further along each 128-byte row; MN-major B:
            // 16 k-rows (2048 bytes) further down each 64-column chunk.
            umma2_bf16_ss(d, a_d0 + so + (uint64_t)(2 * j), b_d0 + so + (uint64_t)(128 * j), planes::kIdesc,
                                (ks > 0 || j > 0) ? 1u : 0u);
          }
          umma2_commit(bar(EMPTY + s));
          umma2_commit(mapa_shared(bar(EMPTY + s), 1u));
        }
        if (!ok) break;
        umma2_commit(bar(ACCF + b));
        umma2_commit(mapa_shared(bar(ACCF + b), 1u));
      }
      // Always: both CTAs free their TMEM only after every MMA of the pair retired.
      umma2_commit(bar(DRAIN));
      umma2_commit(mapa_shared(bar(DRAIN), 1u));
    }
    __syncwarp();
  } else if (warp >= kFirstEpiWarp) {
    // ------------------------------------------------------------ epilogue
    const int q = warp - kFirstEpiWarp;           // TMEM lane quarter
    const uint32_t row = 32 * q + lane;           // product row within this CTA's 128
    const uint32_t acce0 = mapa_shared(bar(ACCE), 0u);
    int lt = 0;
    for (int tile = cluster; tile < p.num_tiles; tile += clusters, ++lt) {
      const int b = lt & 1;
      if (!warp_wait(bar(ACCF + b), (lt >> 1) & 1u, abort_flag, p.err, kErrAccFull)) break;
      tc_fence_after();
      int prod, row0, col0;
      decode(tile, prod, row0, col0);
      const int64_t t = row0 + 128 * (int)rank + (int)row;
      float* out = p.prod + ((int64_t)prod * p.mh + t) * p.nh + col0;
      const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * 256);
#pragma unroll 1
      for (int c = 0; c < kTileN; c += 8) {
        float v[8];
        tmem_load_8(taddr + (uint32_t)c, v);
        reinterpret_cast<float4*>(out + c)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(out + c)[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_remote_arrive(acce0 + 8u * (uint32_t)b);  // the even CTA's ACCE[b]
    }
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still arrive on it or use its TMEM
  if (warp == 1) {
    tc_fence_after();
    if (lane == 0) mbar_wait_drain(bar(DRAIN), 0);
    __syncwarp();
    tmem_dealloc_pair(tmem_base);
  }
}
