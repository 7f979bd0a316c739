// p2p_reduce.cuh -- the tensor-parallel row reduction over NVLink peer memory
// (sb_p2p_reduce and its symmetric buffers).  Included at the end of
// strassen_gemm.cu so it shares the device error word and the host helpers.
//
// The row-parallel o and down projections of the tensor-parallel decoder each
// produce one partial product per rank; the block output is their sum plus
// the residual.  One kernel does that sum over peer memory:
//   barrier A  every CTA meets its counterparts on the other ranks (the
//              partials, written by each rank's GEMM earlier on its stream,
//              are complete);
//   phase 1    rank r reduces slice r of the elements: plain 16-byte loads of
//              every rank's partial (ranks summed in order, fp32), + residual,
//              one bf16 rounding, into r's `reduced` buffer;
//   barrier B  the slices are complete;
//   phase 2    every rank copies all slices from the owners' `reduced`
//              buffers into its output.
// CTA b touches the same element set of every slice in both phases on every
// rank, so a per-CTA barrier (b meets b) orders each read after its write.
// Each barrier wait is bounded (kP2PWaitNs of %globaltimer); on timeout the
// kernel records SB_P2P_ERROR_CODE and returns.  Buffer reuse across calls:
// a rank's next call writes `partial` (by its GEMM) only after its previous
// reduce returned, which is after every peer passed barrier B, i.e. finished
// reading it; `reduced` is rewritten only after the next barrier A, i.e. after
// every peer finished the previous call.  The call counter (the barrier epoch)
// lives in the rank's flag buffer, so CUDA-graph replays stay in step.

namespace sb {

constexpr int kP2PThreads = 512;
constexpr uint64_t kP2PWaitNs = 2000ull * 1000ull * 1000ull;  // 2 s
// Flag buffer: [barrier 0..1][block][rank] epoch words, then this rank's
// state words [epoch, finished-CTA count] (padded to 128 bytes).
constexpr size_t kP2PFlagWords = 2ull * SB_P2P_MAX_BLOCKS * SB_P2P_MAX_RANKS;
constexpr size_t kP2PFlagBytes = (kP2PFlagWords + 32) * sizeof(uint32_t);

struct P2PParams {
  const __nv_bfloat16* partial[SB_P2P_MAX_RANKS];
  __nv_bfloat16* reduced[SB_P2P_MAX_RANKS];
  uint32_t* flags[SB_P2P_MAX_RANKS];
  int32_t rank, world;
  int64_t offset;  // elements
  int64_t vecs;    // elements / 8
  const void* residual;
  int32_t residual_f32;
  __nv_bfloat16* out;
  int* err;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Slice r of `vecs` 16-byte vectors: [vecs*r/world, vecs*(r+1)/world).
__device__ __forceinline__ int64_t p2p_slice_begin(int64_t vecs, int r, int world) {
  return vecs * r / world;
}

// CTA b signals its counterpart on every rank, then waits (bounded) until every
// rank's CTA b signalled this epoch.  Threads 0..world-1 do one peer each.
__device__ bool p2p_barrier(const P2PParams& p, int which, uint32_t epoch) {
  __threadfence_system();  // this thread's earlier writes before the signal
  __syncthreads();
  int ok = 1;
  const int t = threadIdx.x;
  if (t < p.world) {
    const size_t slot = ((size_t)which * SB_P2P_MAX_BLOCKS + blockIdx.x) * SB_P2P_MAX_RANKS;
    st_release_sys(p.flags[t] + slot + p.rank, epoch);
    const uint32_t* mine = p.flags[p.rank] + slot + t;
    const uint64_t t0 = global_timer_ns();
    while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
      if (global_timer_ns() - t0 > kP2PWaitNs) {
        atomicCAS(p.err, 0, SB_P2P_ERROR_CODE);
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ void add_bf16x8(const uint4& u, float (&acc)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

__global__ void __launch_bounds__(kP2PThreads) p2p_reduce_kernel(const P2PParams p) {
  __shared__ uint32_t s_epoch;
  uint32_t* state = p.flags[p.rank] + kP2PFlagWords;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(state) + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;

  if (p2p_barrier(p, 0, epoch)) {
    // Phase 1: this rank's slice, every rank's partial.
    const int64_t lo = p2p_slice_begin(p.vecs, p.rank, p.world);
    const int64_t hi = p2p_slice_begin(p.vecs, p.rank + 1, p.world);
    uint4* red = reinterpret_cast<uint4*>(p.reduced[p.rank] + p.offset);
    // Two vectors per thread per pass (v and v + stride) keep 2 x world peer
    // loads in flight per thread; remote loads are latency-bound.
    for (int64_t v = lo + first; v < hi; v += 2 * stride) {
      const bool second = v + stride < hi;
      uint4 u[2][SB_P2P_MAX_RANKS];
#pragma unroll
      for (int q = 0; q < SB_P2P_MAX_RANKS; ++q) {
        if (q < p.world) {
          const uint4* src = reinterpret_cast<const uint4*>(p.partial[q] + p.offset);
          u[0][q] = __ldcg(src + v);
          if (second) u[1][q] = __ldcg(src + v + stride);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 1 && !second) break;
        const int64_t w = v + h * stride;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < SB_P2P_MAX_RANKS; ++q)
          if (q < p.world) add_bf16x8(u[h][q], acc);
        if (p.residual != nullptr) {
          float r[8];
          load8(p.residual, w * 8, p.residual_f32, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += r[e];
        }
        red[w] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                            pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
      }
    }
    if (p2p_barrier(p, 1, epoch)) {
      // Phase 2: every slice from its owner, this CTA's elements of each.
      uint4* out = reinterpret_cast<uint4*>(p.out);
      for (int j = 0; j < p.world; ++j) {
        const int r = (p.rank + j) % p.world;  // stagger the owners read at once
        const int64_t slo = p2p_slice_begin(p.vecs, r, p.world);
        const int64_t shi = p2p_slice_begin(p.vecs, r + 1, p.world);
        const uint4* src = reinterpret_cast<const uint4*>(p.reduced[r] + p.offset);
        int64_t v = slo + first;
        for (; v + 3 * stride < shi; v += 4 * stride) {
          const uint4 x0 = __ldcg(src + v), x1 = __ldcg(src + v + stride);
          const uint4 x2 = __ldcg(src + v + 2 * stride), x3 = __ldcg(src + v + 3 * stride);
          out[v] = x0;
          out[v + stride] = x1;
          out[v + 2 * stride] = x2;
          out[v + 3 * stride] = x3;
        }
        for (; v < shi; v += stride) out[v] = __ldcg(src + v);
      }
    }
  }
  // Advance the call counter once every CTA of this launch is done (the last
  // CTA to finish; all CTAs read the counter at their start).
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(state + 1, 1u);
    if (done == gridDim.x - 1) {
      state[1] = 0u;
      *reinterpret_cast<volatile uint32_t*>(state) = epoch;
      __threadfence();
    }
  }
}

}  // namespace sb

extern "C" {

size_t sb_p2p_flag_bytes(void) { return sb::kP2PFlagBytes; }

int sb_p2p_buffer_alloc(size_t bytes, void** dev_ptr, sb_ipc_handle* handle) {
  using namespace sb;
  if (dev_ptr == nullptr || handle == nullptr || bytes == 0)
    return fail(SB_ERR_P2P, "sb_p2p_buffer_alloc needs a size and two output pointers");
  int st = check_device();
  if (st != SB_OK) return st;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer maps it
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == sizeof(handle->bytes), "IPC handle size");
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(SB_ERR_CUDA, std::string("p2p buffer: ") + cudaGetErrorString(e));
  }
  std::memcpy(handle->bytes, &h, sizeof(h));
  *dev_ptr = p;
  return SB_OK;
}

int sb_p2p_buffer_open(const sb_ipc_handle* handle, void** dev_ptr) {
  using namespace sb;
  if (dev_ptr == nullptr || handle == nullptr)
    return fail(SB_ERR_P2P, "sb_p2p_buffer_open needs a handle and an output pointer");
  int st = check_device();
  if (st != SB_OK) return st;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  return SB_OK;
}

int sb_p2p_buffer_close(void* dev_ptr) {
  using namespace sb;
  if (dev_ptr == nullptr) return fail(SB_ERR_P2P, "sb_p2p_buffer_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return SB_OK;
}

int sb_p2p_buffer_free(void* dev_ptr) {
  using namespace sb;
  if (dev_ptr == nullptr) return fail(SB_ERR_P2P, "sb_p2p_buffer_free: null pointer");
  cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaFree: ") + cudaGetErrorString(e));
  return SB_OK;
}

int sb_p2p_reduce(sb_stream_t stream, const sb_p2p_group* g, int64_t offset, int64_t elems,
                  const void* residual, int32_t residual_dtype, void* out, int32_t blocks) {
  using namespace sb;
  if (g == nullptr) return fail(SB_ERR_P2P, "sb_p2p_reduce: null group");
  if (g->world < 1 || g->world > SB_P2P_MAX_RANKS)
    return fail(SB_ERR_P2P, "world must be 1.." + std::to_string(SB_P2P_MAX_RANKS) + ", got " +
                                std::to_string(g->world));
  if (g->rank < 0 || g->rank >= g->world)
    return fail(SB_ERR_P2P, "rank " + std::to_string(g->rank) + " outside world " + std::to_string(g->world));
  for (int q = 0; q < g->world; ++q) {
    if (g->partial[q] == nullptr || g->reduced[q] == nullptr || g->flags[q] == nullptr)
      return fail(SB_ERR_P2P, "rank " + std::to_string(q) + " has a null buffer");
    if (!aligned16(g->partial[q]) || !aligned16(g->reduced[q]) || !aligned16(g->flags[q]))
      return fail(SB_ERR_ALIGNMENT, "rank " + std::to_string(q) + " buffers must be 16-byte aligned");
  }
  if (elems <= 0 || elems % 8 || offset < 0 || offset % 8)
    return fail(SB_ERR_P2P, "offset and elems must be multiples of 8 (elems > 0), got " +
                                std::to_string(offset) + ", " + std::to_string(elems));
  if (out == nullptr || !aligned16(out))
    return fail(SB_ERR_ALIGNMENT, "out must be a 16-byte aligned device pointer");
  if (residual != nullptr && !aligned16(residual))
    return fail(SB_ERR_ALIGNMENT, "residual must be 16-byte aligned");
  if (residual_dtype != SB_BF16 && residual_dtype != SB_F32)
    return fail(SB_ERR_DTYPE, "residual dtype must be bf16 or f32");
  if (blocks < 1 || blocks > SB_P2P_MAX_BLOCKS)
    return fail(SB_ERR_P2P, "blocks must be 1.." + std::to_string(SB_P2P_MAX_BLOCKS));
  int st = check_device();
  if (st != SB_OK) return st;
  P2PParams p;
  std::memset(&p, 0, sizeof(p));
  for (int q = 0; q < g->world; ++q) {
    p.partial[q] = static_cast<const __nv_bfloat16*>(g->partial[q]);
    p.reduced[q] = static_cast<__nv_bfloat16*>(g->reduced[q]);
    p.flags[q] = static_cast<uint32_t*>(g->flags[q]);
  }
  p.rank = g->rank;
  p.world = g->world;
  p.offset = offset;
  p.vecs = elems / 8;
  p.residual = residual;
  p.residual_f32 = residual_dtype == SB_F32 ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p.err), g_device_error);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  p2p_reduce_kernel<<<blocks, kP2PThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, std::string("p2p reduce launch: ") + cudaGetErrorString(e));
  return SB_OK;
}

}  // extern "C"
