// Shared helpers for the b200serve sm_100a kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define B200_CHECK_CUDA(expr)                                                        \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess) {                                                         \
      TORCH_CHECK(false, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__, ":", \
                  __LINE__);                                                         \
    }                                                                                \
  } while (0)

namespace b200 {

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over a block whose size is a multiple of 32 (<= 1024). `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

// 16-byte vector of 8 bf16
struct alignas(16) bf16x8 {
  uint32_t w[4];
};

__device__ __forceinline__ void unpack8(const bf16x8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16_lo(v.w[i]);
    f[2 * i + 1] = bf16_hi(v.w[i]);
  }
}

__device__ __forceinline__ bf16x8 pack8(const float* f) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.w[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// fp32 partial sums of a stream-K GEMM (EPI_PARTIAL) that a row kernel reduces: slot s of
// column c holds part[s][row][c]. Worker g of `ctas` (a CTA of the tcgen05 GEMM, a warp of the
// GGUF GEMV) streamed the flattened k-blocks [g*total/ctas, (g+1)*total/ctas) of the `tile`-wide
// column tiles (`kb` k-blocks per tile, total = tiles*kb); tile t's slots are the workers from
// the one holding k-block t*kb to the one holding k-block (t+1)*kb - 1, in that order.
struct PartialIn {
  const float* part;      // nullptr: not in use
  int kb, ctas;
  long long total;
  int rows, cols;
  int tile;               // columns per tile (128: tcgen05 GEMM, 16: GGUF GEMV)
};

// Slots holding a column: the CTAs first(t)..last(t) whose stream-K ranges touch its tile. The
// products stay below 2^32 (tiles x kb x ctas; checked by the host wrappers), so 32-bit unsigned
// division does.
__device__ __forceinline__ int partial_slots(const PartialIn& pi, int col) {
  const uint32_t t = (uint32_t)(col / pi.tile), kb = (uint32_t)pi.kb, ctas = (uint32_t)pi.ctas;
  const uint32_t total = (uint32_t)pi.total;
  const uint32_t first = ((t * kb + 1u) * ctas + total - 1u) / total - 1u;
  const uint32_t last = ((t + 1u) * kb * ctas + total - 1u) / total - 1u;
  return (int)(last - first + 1u);
}

// Sum of one column's slots, in slot order (no rounding).
__device__ __forceinline__ float partial_col(const PartialIn& pi, int row, int col) {
  const int n = partial_slots(pi, col);
  const float* src = pi.part + (size_t)row * pi.cols + col;
  const size_t slot = (size_t)pi.rows * pi.cols;
  float acc = 0.f;
  for (int s = 0; s < n; ++s) acc += __ldcg(src + s * slot);
  return acc;
}

// Sum of the slots for NE consecutive columns of one tile (NE even; 8-byte aligned, 16-byte
// when NE is a multiple of 4), in slot order, rounded to bf16 as a bf16 GEMM output would be.
// The reads of up to BATCH slots are issued together (slots past n read nothing and add zero), so
// a column costs one L2 round trip per batch rather than one per slot.
template <int NE, int BATCH = 8>
__device__ __forceinline__ void partial_sum(const PartialIn& pi, int row, int col, float* acc) {
  constexpr int kPartBatch = BATCH;
  const int n = partial_slots(pi, col);
  const float* src = pi.part + (size_t)row * pi.cols + col;
  const size_t slot = (size_t)pi.rows * pi.cols;
#pragma unroll
  for (int i = 0; i < NE; ++i) acc[i] = 0.f;
  for (int s0 = 0; s0 < n; s0 += kPartBatch) {
    float v[kPartBatch][NE];
#pragma unroll
    for (int u = 0; u < kPartBatch; ++u) {
      const bool live = s0 + u < n;
      const float* p = src + (size_t)(s0 + u) * slot;
      if constexpr (NE % 4 == 0) {
#pragma unroll
        for (int i = 0; i < NE; i += 4) {
          const float4 t = live ? __ldcg(reinterpret_cast<const float4*>(p + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[u][i] = t.x; v[u][i + 1] = t.y; v[u][i + 2] = t.z; v[u][i + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < NE; i += 2) {
          const float2 t = live ? __ldcg(reinterpret_cast<const float2*>(p + i)) : make_float2(0.f, 0.f);
          v[u][i] = t.x; v[u][i + 1] = t.y;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kPartBatch; ++u)          // slot order; an absent slot adds +0.0 (no change)
#pragma unroll
      for (int i = 0; i < NE; ++i) acc[i] += v[u][i];
  }
#pragma unroll
  for (int i = 0; i < NE; ++i) acc[i] = __bfloat162float(__float2bfloat16_rn(acc[i]));
}

}  // namespace b200

namespace b200 {

// Thread-block cluster helpers: a cluster-wide barrier (release / acquire), this CTA's rank in its
// cluster, and 32-bit reads of another CTA's shared memory (distributed shared memory).
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float cluster_ld_f32(const void* p, uint32_t rank) {
  uint32_t a, v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return __uint_as_float(v);
}
__device__ __forceinline__ int cluster_ld_i32(const void* p, uint32_t rank) {
  return (int)__float_as_uint(cluster_ld_f32(p, rank));
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Programmatic dependent launch (PDL). A kernel launched with
// launch_pdl() may start while the previous kernel on the stream is still
// running; it must call pdl_wait() before touching anything the previous
// kernel writes (or writing anything it reads). pdl_trigger() lets the next
// kernel start its own prologue early. Both are no-ops without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

// Bounds-checked builds (compiled with -DB200_BOUNDS_CHECK: the b200_ops_checked extension that
// ops loads when B200_BOUNDS_CHECK=1). B200_IN_RANGE(i, n, code) is false for an index outside
// [0, n): it records `code` in this translation unit's error word (the first one wins) and the
// caller skips the access, so a bad index shows up as an error code instead of a fault. Release
// builds compile the check to `true`. B200_BOUNDS_ACCESSOR(name) defines the host reader
// `int64_t bounds_error_<name>(bool reset)` of the unit's word (0 in release builds).
#ifdef B200_BOUNDS_CHECK
static __device__ int g_b200_bounds_err;
#define B200_IN_RANGE(i, n, code)                                                           \
  (((unsigned long long)(long long)(i) < (unsigned long long)(long long)(n)) ||             \
   (atomicCAS(&g_b200_bounds_err, 0, (int)(code)), false))
#define B200_BOUNDS_ACCESSOR(name)                                                          \
  int64_t bounds_error_##name(bool reset) {                                                 \
    int v = 0;                                                                              \
    B200_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_b200_bounds_err, sizeof(int)));              \
    if (reset) {                                                                            \
      const int z = 0;                                                                      \
      B200_CHECK_CUDA(cudaMemcpyToSymbol(g_b200_bounds_err, &z, sizeof(int)));              \
    }                                                                                       \
    return v;                                                                               \
  }
#else
#define B200_IN_RANGE(i, n, code) true
#define B200_BOUNDS_ACCESSOR(name) \
  int64_t bounds_error_##name(bool) { return 0; }
#endif

// Block id of table entry `idx` of a paged-KV block-table row: bt[idx] in release builds; in
// checked builds -1 when idx is outside [0, max_blocks) (recorded as code + 1) or the block id
// outside [0, nblocks) (recorded as code).
static __device__ __forceinline__ int table_block(const int* bt, int idx, int max_blocks, int nblocks, int code) {
  if (!B200_IN_RANGE(idx, max_blocks, code + 1)) return -1;
  const int blk = bt[idx];
  return B200_IN_RANGE(blk, nblocks, code) ? blk : -1;
}

// Deadline (ns) of every cross-GPU flag wait, passed to the kernels as an argument (so a CUDA
// graph keeps the value it was captured with). Default 2 s; B200_FLAG_WAIT_MS or
// set_flag_wait_ms() change it.
uint64_t flag_wait_ns();

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) TORCH_CHECK(false, "launch failed: ", cudaGetErrorString(e));
}

// launch_pdl with a thread-block cluster of `cluster_x` CTAs along x
template <typename... KArgs, typename... Args>
inline void launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                               int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) TORCH_CHECK(false, "cluster launch failed: ", cudaGetErrorString(e));
}

}  // namespace b200
