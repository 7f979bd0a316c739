/*
 * strassen_b200.h -- C ABI of the B200 (sm_100a) tile-local Strassen GEMM.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream and
 * returns an sb_status code; nothing throws and nothing traps.  Argument
 * errors are detected on the host before any launch.  The caller owns every
 * buffer: the library allocates device memory only in sb_p2p_buffer_alloc,
 * whose job that is.  Scratch space is passed in as `workspace`, sized by
 * sb_workspace_bytes(): the fp32 rows of norm_residual_add, and for large
 * products the operand planes and fp32 products of the planes path (a caller
 * that passes less gets the one-CTA kernel, which needs none); the one
 * exception is
 * sb_strassen_gemm_norm_residual_noalloc, whose scratch is a fixed 32 MiB
 * device array built into the library (see its declaration).  Besides
 * memory, the planes path creates one side stream and three events per device
 * and host thread on first use and keeps them for the thread's life.
 *
 * The single operator mirrors strassen_pallas.strassen_matmul
 * (reference: strassen_pallas.py:882-1221).  Matrix semantics follow the
 * reference exactly: C = A·B with A row-major [M,K], B row-major [K,N], and a
 * one-level Strassen split applied inside every (bm, bn, bk) block, i.e. the
 * ten operand sums pair element (r, c) of a block with (r + bm/2, c + bk/2)
 * and (r + bk/2, c + bn/2) exactly as the reference's in-VMEM quadrant split
 * does (strassen_pallas.py:188-204).
 */
#ifndef STRASSEN_B200_H_
#define STRASSEN_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SB_API __attribute__((visibility("default")))
#else
#define SB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef void* sb_stream_t;

/* ---- status codes (map 1:1 onto the reference's ValueError conditions) --- */
typedef enum sb_status {
  SB_OK = 0,
  SB_ERR_RANK = 1,            /* strassen_pallas.py:927-928 rank-2 inputs       */
  SB_ERR_INNER_DIM = 2,       /* :931-932 inner dimensions disagree              */
  SB_ERR_DTYPE = 3,           /* :933-936 input dtype must be BF16 (B200 path)   */
  SB_ERR_DIVISIBILITY = 4,    /* :1044-1046 M/N/K not divisible by bm/bn/bk      */
  SB_ERR_TILING = 5,          /* :127-140 check_tiling alignment                  */
  SB_ERR_EPILOGUE = 6,        /* :944-1002 epilogue argument contract            */
  SB_ERR_OUTPUT_DTYPE = 7,    /* :955-958, :1048-1050 output dtype                */
  SB_ERR_UNSUPPORTED = 8,     /* valid for the reference, not built for B200     */
  SB_ERR_ALIGNMENT = 9,       /* pointer / leading-dimension alignment (TMA)     */
  SB_ERR_WORKSPACE = 10,      /* workspace missing or too small                  */
  SB_ERR_CUDA = 11,           /* a CUDA runtime call failed                      */
  SB_ERR_DEVICE = 12,         /* device is not sm_100 (B200)                     */
  SB_ERR_DEVICE_TIMEOUT = 13, /* a bounded in-kernel wait gave up                */
  SB_ERR_P2P = 14             /* peer-group argument error (sb_p2p_*)            */
} sb_status;

/* ---- dtypes ------------------------------------------------------------- */
typedef enum sb_dtype { SB_BF16 = 0, SB_F32 = 1 } sb_dtype;

/* ---- fused epilogues (strassen_pallas.py:739-879) ------------------------ */
typedef enum sb_epilogue_kind {
  SB_EPI_NONE = 0,
  SB_EPI_SWIGLU = 1,            /* :762-777, silu(gate)*up, output [M, N/2]   */
  SB_EPI_GEGLU = 2,             /* :143-153, gelu_tanh(gate)*up               */
  SB_EPI_RESIDUAL_ADD = 3,      /* :778-792                                   */
  SB_EPI_BIAS_ADD = 4,          /* :867-874                                   */
  SB_EPI_QK_NORM_ROPE = 5,      /* :793-835, per-head RMSNorm + RoPE          */
  SB_EPI_NORM_RESIDUAL_ADD = 6  /* :836-866, row RMSNorm * scale + residual   */
} sb_epilogue_kind;

typedef struct sb_epilogue {
  int32_t kind;               /* sb_epilogue_kind                                  */
  /* residual_add / norm_residual_add: [M, N], leading dimension ld_residual     */
  const void* residual;
  int64_t ld_residual;
  int32_t residual_dtype;     /* sb_dtype                                          */
  /* dtype of bias, rope tables, rope scale and norm scale                       */
  int32_t aux_dtype;          /* sb_dtype                                          */
  const void* bias;           /* bias_add: [N]                                     */
  const void* rope_cos;       /* qk_norm_rope: [M, bn/2] (rope_layout_tables)      */
  const void* rope_sin;       /* qk_norm_rope: [M, bn/2]                           */
  int64_t ld_rope;            /* leading dimension of rope_cos / rope_sin          */
  const void* rope_scale;     /* qk_norm_rope: [bn] (rope_scale_layout)            */
  int32_t rope_head_dim;      /* default 128                                       */
  float rope_eps;             /* default 1e-6                                      */
  const void* norm_scale;     /* norm_residual_add: [N]                            */
  float norm_eps;             /* default 1e-6                                      */
} sb_epilogue;

/* ---- research options (strassen_pallas.py:205-226, 381-517, 575-586) ------ */
typedef enum sb_formula {
  SB_FORMULA_CLASSICAL = 0,  /* Strassen's P1..P7, strassen_pallas.py:324-379   */
  SB_FORMULA_DUAL = 1,       /* the dual rank-7 formula Q1..Q7, :466-517         */
  SB_FORMULA_POWERS = 2      /* power-of-two formula R1..R7, :381-464; no epilogue,
                                no exact panels                                   */
} sb_formula;

typedef struct sb_options {
  int32_t formula_variant;        /* sb_formula                                     */
  int32_t block_permutation;      /* bit 0 swaps M halves, bit 1 K halves, bit 2 N   */
  /* Exact classical K panels: device int32 array [K/bk], nonzero = run that panel
   * as eight exact sub-block products instead of Strassen (the reference's
   * classical_panels / panel_schedule).  NULL = none. */
  const int32_t* panel_schedule;
  /* B200 extension (no counterpart in the reference, whose TPU lane rule asks
   * bn % 256 == 0): nonzero accepts any bn that is a multiple of 128, and
   * qk_norm_rope then needs bn % head_dim == 0 (each half block holds whole
   * half-heads).  The tensor-parallel decoder uses it for one-head k/v shards
   * (128 columns).  0 = the reference's rules. */
  int32_t narrow_bn;
} sb_options;

/*
 * sb_strassen_gemm -- C = epilogue(A·B) with one tile-local Strassen level.
 *
 * Replaces strassen_pallas.strassen_matmul (strassen_pallas.py:882-1221) for
 * bf16 inputs.  bm/bn/bk are the reference's tile arguments and define the
 * Strassen block, so results follow the reference's pairing of operands.
 * Shapes: A [M,K] (lda), B [K,N] (ldb), C [M,N] (ldc) -- or [M, N/2] for the
 * swiglu/geglu epilogues.  out_dtype: SB_BF16 or SB_F32 (SB_F32 only without
 * an epilogue, as in the reference).  `ep` may be NULL for no epilogue.
 * workspace / workspace_bytes: caller-owned scratch.  norm_residual_add
 * requires sb_workspace_bytes() bytes.  For other products a non-zero
 * sb_workspace_bytes() is the planes path's workspace (see
 * sb_strassen_gemm_planes): passing at least that much, 16-byte aligned, runs
 * the product there; passing less (or NULL) runs the one-CTA kernel.  Same
 * result either way up to fp32 summation order.  Asynchronous on `stream`.
 */
SB_API int sb_strassen_gemm(sb_stream_t stream,
                     const void* a, const void* b, void* c,
                     int64_t m, int64_t n, int64_t k,
                     int64_t lda, int64_t ldb, int64_t ldc,
                     int32_t bm, int32_t bn, int32_t bk,
                     int32_t out_dtype, const sb_epilogue* ep,
                     void* workspace, size_t workspace_bytes);

/*
 * sb_strassen_gemm_ex -- sb_strassen_gemm with the reference's research options
 * (formula_variant, block_permutation, classical_panels / panel_schedule of
 * strassen_matmul, strassen_pallas.py:882-911).  opt == NULL is sb_strassen_gemm.
 */
SB_API int sb_strassen_gemm_ex(sb_stream_t stream,
                               const void* a, const void* b, void* c,
                               int64_t m, int64_t n, int64_t k,
                               int64_t lda, int64_t ldb, int64_t ldc,
                               int32_t bm, int32_t bn, int32_t bk,
                               int32_t out_dtype, const sb_epilogue* ep,
                               const sb_options* opt,
                               void* workspace, size_t workspace_bytes);

/* Scratch bytes sb_strassen_gemm wants for this problem: the norm_residual_add
 * rows, the planes path's workspace where a cost model with rates measured on
 * B200 expects it to beat the one-CTA kernel (no epilogue or residual_add /
 * bias_add / swiglu / geglu / qk_norm_rope; M, N % 512, K % 128), else 0.
 * Replaces the reference's VMEM scratch_shapes sizing (strassen_pallas.py:1074-1078). */
SB_API size_t sb_workspace_bytes(int64_t m, int64_t n, int64_t k, int32_t epilogue_kind);

/*
 * sb_classical_gemm -- the matched-tile cubic control: the same kernel
 * skeleton, tile and pipeline as sb_strassen_gemm but eight classical
 * sub-block products and no operand sums.  Replaces the reference's Pallas
 * cubic control (experiments/qwen3/benchmark_cubic_control.py:57-237,
 * variant="blocked").  bf16 in, bf16/f32 out, no epilogue.
 */
SB_API int sb_classical_gemm(sb_stream_t stream,
                      const void* a, const void* b, void* c,
                      int64_t m, int64_t n, int64_t k,
                      int64_t lda, int64_t ldb, int64_t ldc,
                      int32_t bm, int32_t bn, int32_t bk, int32_t out_dtype);

/*
 * sb_strassen_gemm_pair -- C = A·B, no epilogue, on the two-CTA kernel: a
 * thread-block cluster of two CTAs shares each 128 x 128 product tile and
 * splits the seven Strassen products between them (3.5 each, 128-wide
 * tensor-core products); the two quadrant halves of every output tile are
 * finished after one fp32 partial exchange through distributed shared memory.
 * Same contract as sb_strassen_gemm with ep == NULL (strassen_pallas.py:882-1221,
 * no epilogue): same arguments, validation and Strassen block semantics; the
 * fp32 order of the final recombination differs, so results agree with
 * sb_strassen_gemm to fp32 rounding, not bit for bit.
 */
SB_API int sb_strassen_gemm_pair(sb_stream_t stream,
                                 const void* a, const void* b, void* c,
                                 int64_t m, int64_t n, int64_t k,
                                 int64_t lda, int64_t ldb, int64_t ldc,
                                 int32_t bm, int32_t bn, int32_t bk, int32_t out_dtype);

/*
 * sb_strassen_b_operands -- the seven B operands of every Strassen block of
 * B [K, N] (ldb) for the tile (bn, bk), formed once: the reference's B
 * pre-adds (strassen_pallas.py:324-379), each rounded once to bf16, written as
 * planes [7][K/2][N/2] bf16 (contiguous, sb_b_operands_bytes(k, n) bytes) in
 * the order P3 (b1-b3), P5 (b3), P7 (b2+b3), P1 (b0+b3), P2 (b0),
 * P4 (b2-b0), P6 (b0+b1).  For a weight used many times this is an offline
 * relayout, like the reference's swiglu_weight_layout (strassen_pallas.py:1381-1411).
 */
SB_API size_t sb_b_operands_bytes(int64_t k, int64_t n);
SB_API int sb_strassen_b_operands(sb_stream_t stream, const void* b, void* planes,
                                  int64_t k, int64_t n, int64_t ldb, int32_t bn, int32_t bk);

/*
 * sb_strassen_gemm_pair_planes -- sb_strassen_gemm_pair with B given as its
 * operand planes (sb_strassen_b_operands, built for the same bn and bk): the
 * kernel loads each product's B operand as it is and forms no B sums.  The
 * operand values are the ones the in-kernel sums produce, so the result
 * equals sb_strassen_gemm_pair on the raw B bit for bit.
 */
SB_API int sb_strassen_gemm_pair_planes(sb_stream_t stream,
                                        const void* a, const void* b_planes, void* c,
                                        int64_t m, int64_t n, int64_t k,
                                        int64_t lda, int64_t ldc,
                                        int32_t bm, int32_t bn, int32_t bk, int32_t out_dtype);

/*
 * sb_strassen_gemm_quad -- C = A·B, no epilogue, on the four-CTA kernel:
 * clusters of two CTA pairs (tcgen05 cta_group::2, M = 256) per 256 x 128
 * product tile, each pair 3.5 of the seven products.  Replaces
 * strassen_pallas.strassen_matmul(a, b, bm=, bn=, bk=, output_dtype=) without
 * an epilogue (strassen_pallas.py:882-1221); same operand pairing and
 * rounding, recombination in a different fp32 order.  The call forms A's
 * operands (a pass over A) and B's operand planes (sb_strassen_b_operands) in
 * `workspace` (sb_quad_workspace_bytes(m, n, k) bytes, 16-byte aligned) and
 * then runs the GEMM, all on `stream`.  Needs M % 512 == 0, bn % 256 == 0 and
 * bk % 256 == 0 (SB_ERR_TILING otherwise).  `raster`: product-row tiles the
 * cluster tiles walk per column sweep (L2 reuse; 0 = the kernel's default of 2).
 */
SB_API size_t sb_quad_workspace_bytes(int64_t m, int64_t n, int64_t k);
SB_API int sb_strassen_gemm_quad(sb_stream_t stream,
                                 const void* a, const void* b, void* c,
                                 int64_t m, int64_t n, int64_t k,
                                 int64_t lda, int64_t ldb, int64_t ldc,
                                 int32_t bm, int32_t bn, int32_t bk, int32_t out_dtype,
                                 void* workspace, size_t workspace_bytes, int32_t raster);

/*
 * sb_strassen_gemm_planes -- C = A·B, no epilogue, as seven full-width product
 * GEMMs (sb_strassen_gemm runs the same path, with its fused epilogues applied
 * in the recombination, when given this workspace): two passes form the A operand planes [7][M/2][K/2] and the B operand
 * planes [7][K/2][N/2] (the reference's pre-adds, strassen_pallas.py:324-379,
 * each rounded once to bf16), a persistent kernel on CTA pairs (tcgen05
 * cta_group::2, 256 x 256 product tiles) writes the seven fp32 products, and a
 * last pass recombines C11 = M1+M4-M5+M7, C12 = M3+M5, C21 = M2+M4,
 * C22 = M1-M2+M3+M6 into C.  Replaces strassen_pallas.strassen_matmul(a, b,
 * bm=, bn=, bk=, output_dtype=) without an epilogue (strassen_pallas.py:882-1221);
 * same operand pairing, rounding and recombination order as sb_strassen_gemm.
 * `workspace`: sb_planes_workspace_bytes(m, n, k) bytes, 16-byte aligned.
 * Needs M % 512 == 0, N % 512 == 0 and K % 128 == 0 (SB_ERR_TILING otherwise).
 * `raster`: product-row tiles per column sweep (0 = the kernel's default).
 * `stages`: which steps run (bit 0 the operand passes, bit 1 the product GEMM,
 * bit 2 the recombination; 7 = the whole product); the workspace carries the
 * intermediate results between calls, so a caller can time the GEMM alone.
 * The whole product runs in two halves of product rows, the second on a
 * stream of the library's (forked from and joined back into `stream`), so each
 * half's passes and recombination overlap the other half's GEMM.
 * `timing_events`: NULL, or four cudaEvent_t the call records around its GEMM
 * launches: 0/1 around the first half's on `stream`, 2/3 around the second
 * half's on the side stream; when the GEMM runs as one launch (`stages` 2, a
 * product under two 256-row tiles, or a first use inside a graph capture)
 * 0/1 around it and 2/3 at its end.
 * sb_strassen_gemm / sb_strassen_gemm_ex take this path (no research option;
 * no epilogue or residual_add / bias_add / swiglu / geglu / qk_norm_rope) when
 * sb_workspace_bytes asks for the planes workspace and the caller passes it.
 */
SB_API size_t sb_planes_workspace_bytes(int64_t m, int64_t n, int64_t k);
SB_API int sb_strassen_gemm_planes(sb_stream_t stream,
                                   const void* a, const void* b, void* c,
                                   int64_t m, int64_t n, int64_t k,
                                   int64_t lda, int64_t ldb, int64_t ldc,
                                   int32_t bm, int32_t bn, int32_t bk, int32_t out_dtype,
                                   void* workspace, size_t workspace_bytes, int32_t raster,
                                   int32_t stages, void* const* timing_events);

/*
 * sb_strassen_gemm_norm_residual_noalloc -- the norm_residual_add epilogue of
 * sb_strassen_gemm, with its fp32 scratch in a device array built into the
 * library instead of a caller workspace.  No counterpart in the reference.
 *
 * For callers that cannot provide or allocate scratch memory: a custom-call
 * handler in a framework that owns device memory (cudaMalloc would compete with
 * its allocator and synchronise the device), or a service with a fixed memory
 * budget.  It allocates nothing.  Limit: M*N <= 8,388,608 (32 MiB of fp32),
 * else SB_ERR_WORKSPACE.  Every GPU that loads the library holds the 32 MiB
 * until exit; all calls share it, so calls that overlap on the GPU race.  Every
 * call looks up the array's address in the current context (the first call on
 * a device also loads the module there: make it before any stream capture).
 * `ep->kind` must be SB_EPI_NORM_RESIDUAL_ADD and bn == n.
 */
SB_API int sb_strassen_gemm_norm_residual_noalloc(sb_stream_t stream,
                                                  const void* a, const void* b, void* c,
                                                  int64_t m, int64_t n, int64_t k,
                                                  int64_t lda, int64_t ldb, int64_t ldc,
                                                  int32_t bm, int32_t bn, int32_t bk,
                                                  const sb_epilogue* ep);

/*
 * sb_strassen_gemm_lhs_transposed -- C = A^T·B with A stored (K, M) row-major
 * (leading dimension ldat >= M), without materialising the transpose.
 * Replaces strassen_pallas.strassen_matmul_lhs_transposed
 * (strassen_pallas.py:1224-1312): classical formula, no epilogue, bf16 or fp32
 * output.  B200 restriction: bm must be a multiple of 128.
 */
SB_API int sb_strassen_gemm_lhs_transposed(sb_stream_t stream,
                                           const void* at, const void* b, void* c,
                                           int64_t m, int64_t n, int64_t k,
                                           int64_t ldat, int64_t ldb, int64_t ldc,
                                           int32_t bm, int32_t bn, int32_t bk,
                                           int32_t out_dtype);

/*
 * sb_rms_norm -- y = bf16(x * rsqrt(mean(x^2) + eps) * w), fp32 math.
 * Replaces the reference's rms_norm
 * (experiments/qwen3/benchmark_qwen3_32b_layer.py:270-276).  x, y: [rows, n]
 * bf16 (ld = n), w: [n] in w_dtype.
 */
SB_API int sb_rms_norm(sb_stream_t stream, const void* x, const void* w, void* y,
                int64_t rows, int64_t n, int32_t w_dtype, float eps);

/* Internal tile shape of the kernel (product rows, product cols, k-chunk). */
SB_API void sb_query_tile(int32_t* block_m, int32_t* block_n, int32_t* block_k);

/* Human-readable text for a status code (static storage). */
SB_API const char* sb_status_string(int32_t status);

/* Detailed message of the last failing call on this host thread. */
SB_API const char* sb_last_error_message(void);

/*
 * Reads (and with reset != 0 clears) the device-side error word that bounded
 * in-kernel waits set when they give up.  Synchronises the current device.
 */
SB_API int sb_device_status(int32_t* device_error, int32_t reset);

/*
 * Failure-detection self-test (no counterpart in the reference): launches one
 * CTA on `stream` whose first warp waits, with the same bounded wait the GEMM
 * kernels use, on an mbarrier that nothing arrives on, while a second warp,
 * starting half a limit later, waits on another such barrier until the CTA
 * abort flag stops it.  After ~1 s the
 * first wait gives up, sets the error word to SB_SELFTEST_ERROR_CODE and both
 * warps return; sb_device_status then reports SB_ERR_DEVICE_TIMEOUT.  No fault,
 * no trap: the context stays usable.
 */
#define SB_SELFTEST_ERROR_CODE 9
SB_API int sb_wait_selftest(sb_stream_t stream);

/* ---- tensor-parallel row reduction over NVLink peer memory ------------- */
/*
 * The row-parallel projections of the tensor-parallel Qwen3 decoder (o and
 * down) end in a sum of every rank's partial product plus the residual.
 * sb_p2p_reduce computes that sum in one kernel over peer memory, in place of
 * an NCCL all-reduce and a residual add.  No counterpart in the reference
 * (its decoder runs on one device); its residual_add epilogue contract
 * (strassen_pallas.py:778-792: fp32 sum, one bf16 rounding) is kept.
 *
 * Buffers are symmetric: every rank allocates the same three buffers with
 * sb_p2p_buffer_alloc (zero-filled), ships the handles to the other ranks
 * (any host channel), and opens the peers' handles with sb_p2p_buffer_open.
 *   partial  bf16, >= offset + elems elements: this rank's partial product,
 *            written by its GEMM before the call (stream order);
 *   reduced  bf16, same size: the rank's reduced slice (internal);
 *   flags    sb_p2p_flag_bytes(): barrier words and this rank's call counter.
 */
#define SB_P2P_MAX_RANKS 8
#define SB_P2P_MAX_BLOCKS 256
#define SB_P2P_ERROR_CODE 10 /* device error word after a barrier wait gave up */

typedef struct sb_ipc_handle {
  unsigned char bytes[64]; /* a cudaIpcMemHandle_t */
} sb_ipc_handle;

/* cudaMalloc + zero fill + IPC handle.  Free with sb_p2p_buffer_free. */
SB_API int sb_p2p_buffer_alloc(size_t bytes, void** dev_ptr, sb_ipc_handle* handle);
/* Maps another process's buffer on the current device (peer access enabled). */
SB_API int sb_p2p_buffer_open(const sb_ipc_handle* handle, void** dev_ptr);
SB_API int sb_p2p_buffer_close(void* dev_ptr);
SB_API int sb_p2p_buffer_free(void* dev_ptr);
SB_API size_t sb_p2p_flag_bytes(void);

typedef struct sb_p2p_group {
  int32_t rank;                         /* this process's rank                 */
  int32_t world;                        /* 1 .. SB_P2P_MAX_RANKS               */
  void* partial[SB_P2P_MAX_RANKS];      /* rank q's buffers, mapped here       */
  void* reduced[SB_P2P_MAX_RANKS];
  void* flags[SB_P2P_MAX_RANKS];
} sb_p2p_group;

/*
 * out[i] = bf16( (sum over q = 0..world-1 of partial_q[offset + i]) + residual[i] )
 * for 0 <= i < elems, in fp32 with the ranks summed in order, identical on
 * every rank.  Two phases in one kernel: each rank reduces its slice of the
 * elements from every rank's partial buffer (plain peer loads) into its
 * reduced buffer, then gathers the other ranks' slices into `out`.  Each CTA
 * meets its counterparts on the other ranks at a flag barrier before each
 * phase; a wait gives up after 2 s, sets the device error word to
 * SB_P2P_ERROR_CODE and the kernel returns (sb_device_status reports it).
 * Every rank must make the same sequence of calls, with the same offset,
 * elems and blocks, each on one stream per rank; calls may be captured in a
 * CUDA graph (the call counter lives in device memory).  residual: bf16 or
 * f32 (residual_dtype) or NULL; out: bf16.  offset and elems are multiples of
 * 8; pointers 16-byte aligned; blocks in 1 .. SB_P2P_MAX_BLOCKS.
 */
SB_API int sb_p2p_reduce(sb_stream_t stream, const sb_p2p_group* group, int64_t offset,
                         int64_t elems, const void* residual, int32_t residual_dtype, void* out,
                         int32_t blocks);

/* Library version string. */
SB_API const char* sb_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* STRASSEN_B200_H_ */
