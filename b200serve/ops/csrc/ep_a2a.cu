// Expert-parallel all-to-all over NVLink for a token-sharded MoE step.
//
// Rank r owns Tw token rows (`valid` of them real) and the experts [r*per, (r+1)*per).
//  1. ep_count: for its valid rows, rank r counts the (token, expert) pairs per destination
//     expert, gives every pair its rank among the pairs of the same expert (pos), and stores its
//     whole [world dst][per] count matrix into cnt_all[r] on EVERY rank, then raises flag
//     [site][r] on every rank (one system fence, relaxed flag stores).
//  2. ep_dispatch: after every rank's counts arrived, rank r knows where each of its pairs goes:
//     owner d's receive buffer is sorted by local expert, and inside one expert by source rank
//     (base(d, e) + rows of lower source ranks + pos). It stores the token row there (P2P, 16-byte
//     vectors) with (source rank, pair index, routing weight) metadata, and raises the dispatch
//     flags. The owner's grouped gate_up GEMM waits for those flags inside the kernel.
//  3. The grouped down GEMM (gemm_grouped_ep, EPI_PUSH with combine metadata) scales each output
//     row by its routing weight and stores it back into the home rank's combine slot
//     [j][t] of pair p = t * k + j; the home rank's norm sums the k slots.
// Every wait is bounded by the flag-wait deadline and records an error code instead of hanging.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

struct EpPeers {
  int* cnt_all[8];            // [world src][world dst][per] int32 on each rank
  int* flag[8];               // this site's flag word for source `me` on each rank
  __nv_bfloat16* rows[8];     // receive rows [R_cap][H] on each rank
  int4* meta[8];              // receive metadata [R_cap] on each rank
  int* dflag[8];              // dispatch site's flag word for source `me` on each rank
};

__device__ __forceinline__ bool ep_wait_flags(const int* flags, int n, int e, uint64_t wait_ns, int* err, int code) {
  const uint64_t deadline = globaltimer_ns() + wait_ns;
  for (int r = 0; r < n; ++r) {
    uint32_t it = 0;
    while (true) {
      int v;
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
      if (v == e) break;
      if ((++it & 1023u) == 0 && globaltimer_ns() > deadline) {
        if (err) atomicExch(err, code + r);
        return false;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return true;
}

// One CTA. ids [Tw, k] int32 (global expert ids), valid rows < `valid`.
__global__ void __launch_bounds__(1024) ep_count_kernel(const int* __restrict__ ids, int valid, int k, int per,
                                                        int world, int me, int* __restrict__ pos,
                                                        const EpPeers peers, const int* epoch) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int cnt[];                       // [world][per]
  const int n = world * per;
  for (int i = threadIdx.x; i < n; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int pairs = valid * k;
  for (int p = threadIdx.x; p < pairs; p += blockDim.x)
    pos[p] = B200_IN_RANGE(ids[p], n, 0x601) ? atomicAdd(&cnt[ids[p]], 1) : 0;   // checked: skip the pair
  __syncthreads();
  // cnt_all[me] on every rank
  for (int i = threadIdx.x; i < world * n; i += blockDim.x) {
    const int r = i / n, c = i % n;
    peers.cnt_all[r][me * n + c] = cnt[c];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int e = *epoch;
    for (int r = 0; r < world; ++r)
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(peers.flag[r]), "r"(e) : "memory");
  }
}

// Grid of CTAs, one warp per pair. cnt_all: this rank's [world src][world dst][per] (filled by
// ep_count on every rank); wait_flags: the count site's flags on this rank.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(
    const __nv_bfloat16* __restrict__ x, const int* __restrict__ ids, const float* __restrict__ wts,
    const int* __restrict__ pos, int valid, int k, int per, int world, int me, int H, const int* cnt_all,
    const int* wait_flags, const EpPeers peers, const int* epoch, int* done, int* err, uint64_t wait_ns) {
  pdl_wait();
  pdl_trigger();
  __shared__ int off[8 * 64];                         // [dst][local expert] first slot of my rows
  __shared__ int ok;
  const int n = world * per;
  if (threadIdx.x == 0) ok = ep_wait_flags(wait_flags, world, *epoch, wait_ns, err, 180) ? 1 : 0;
  __syncthreads();
  if (ok) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int d = i / per, el = i % per;
      int base = 0;
      for (int e2 = 0; e2 < el; ++e2)
        for (int s = 0; s < world; ++s) base += __ldcg(cnt_all + s * n + d * per + e2);
      for (int s = 0; s < me; ++s) base += __ldcg(cnt_all + s * n + d * per + el);
      off[i] = base;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pairs = valid * k;
  if (ok) {
    for (int p = blockIdx.x * 8 + warp; p < pairs; p += gridDim.x * 8) {
      const int e = ids[p], d = e / per, el = e % per;
      if (!B200_IN_RANGE(e, n, 0x602)) continue;
      const int slot = off[d * per + el] + pos[p];
      const int t = p / k;
      const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
      uint4* dst = reinterpret_cast<uint4*>(peers.rows[d] + (size_t)slot * H);
      for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
      if (lane == 0) peers.meta[d][slot] = make_int4(me, p, __float_as_int(wts[p]), 0);
    }
  }
  // the last CTA raises the dispatch flags once every CTA's rows reached their owners
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(done, 1);
    if (old == (int)gridDim.x - 1) {
      *done = 0;
      __threadfence_system();
      const int e = *epoch;
      for (int r = 0; r < world; ++r)
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(peers.dflag[r]), "r"(e) : "memory");
    }
  }
}

}  // namespace b200

using namespace b200;

static EpPeers ep_peers(torch::Tensor cnt_ptrs, torch::Tensor flag_ptrs, torch::Tensor rows_ptrs,
                        torch::Tensor meta_ptrs, torch::Tensor dflag_ptrs) {
  EpPeers p{};
  const int world = cnt_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= 8, "1..8 ranks");
  for (int r = 0; r < world; ++r) {
    p.cnt_all[r] = reinterpret_cast<int*>(cnt_ptrs.data_ptr<int64_t>()[r]);
    p.flag[r] = reinterpret_cast<int*>(flag_ptrs.data_ptr<int64_t>()[r]);
    if (rows_ptrs.numel()) p.rows[r] = reinterpret_cast<__nv_bfloat16*>(rows_ptrs.data_ptr<int64_t>()[r]);
    if (meta_ptrs.numel()) p.meta[r] = reinterpret_cast<int4*>(meta_ptrs.data_ptr<int64_t>()[r]);
    if (dflag_ptrs.numel()) p.dflag[r] = reinterpret_cast<int*>(dflag_ptrs.data_ptr<int64_t>()[r]);
  }
  return p;
}

// pointer lists: host int64 [world] (per rank: its cnt_all base / this site's flag for source me)
void ep_count(torch::Tensor ids, int64_t valid, int64_t per, int64_t me, torch::Tensor pos, torch::Tensor cnt_ptrs,
              torch::Tensor flag_ptrs, int64_t epoch_ptr) {
  const int world = cnt_ptrs.numel(), k = ids.size(1);
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && pos.numel() >= valid * k);
  TORCH_CHECK(world * per <= 8 * 64, "at most 512 (rank, expert) counters");
  EpPeers p = ep_peers(cnt_ptrs, flag_ptrs, torch::empty({0}, torch::kInt64), torch::empty({0}, torch::kInt64),
                       torch::empty({0}, torch::kInt64));
  launch_pdl(ep_count_kernel, dim3(1), dim3(1024), (size_t)world * per * sizeof(int),
             at::cuda::getCurrentCUDAStream(), (const int*)ids.data_ptr<int>(), (int)valid, k, (int)per, world,
             (int)me, pos.data_ptr<int>(), p, reinterpret_cast<const int*>(epoch_ptr));
}

void ep_dispatch(torch::Tensor x, torch::Tensor ids, torch::Tensor wts, torch::Tensor pos, int64_t valid, int64_t per,
                 int64_t me, int64_t cnt_all_ptr, int64_t wait_flags_ptr, torch::Tensor cnt_ptrs,
                 torch::Tensor rows_ptrs, torch::Tensor meta_ptrs, torch::Tensor dflag_ptrs, int64_t epoch_ptr,
                 torch::Tensor done, int64_t err_ptr) {
  const int world = rows_ptrs.numel(), k = ids.size(1), H = x.size(1);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && H % 8 == 0);
  TORCH_CHECK(wts.scalar_type() == at::kFloat && wts.is_contiguous());
  EpPeers p = ep_peers(cnt_ptrs, rows_ptrs, rows_ptrs, meta_ptrs, dflag_ptrs);
  const int pairs = (int)valid * k;
  const int blocks = std::max(1, std::min(148 * 4, (pairs + 7) / 8));
  launch_pdl(ep_dispatch_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (const int*)ids.data_ptr<int>(),
             (const float*)wts.data_ptr<float>(), (const int*)pos.data_ptr<int>(), (int)valid, k, (int)per, world,
             (int)me, H, reinterpret_cast<const int*>(cnt_all_ptr), reinterpret_cast<const int*>(wait_flags_ptr), p,
             reinterpret_cast<const int*>(epoch_ptr), done.data_ptr<int>(), reinterpret_cast<int*>(err_ptr),
             flag_wait_ns());
}

B200_BOUNDS_ACCESSOR(ep_a2a)
