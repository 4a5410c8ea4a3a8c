// Mixture-of-experts routing and token permutation.
//
// topk_softmax restates the reference's CPU router (webgpu/src/engine/moe-cpu.ts:157
// topKSoftmax): softmax over all experts in fp32, keep the k largest
// probabilities (lowest expert id on ties), renormalise them when asked.
// One warp per token; experts are spread over the lanes (E <= 256).
//
// moe_permute builds the expert-sorted token order used by the grouped expert
// GEMM: counts per expert, exclusive offsets, and for every (token, k) slot its
// position in the sorted list (a deterministic counting sort: slots of one
// expert keep their token order).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

template <int EPL>  // experts per lane
__global__ void topk_softmax_kernel(const float* __restrict__ logits, int T, int E, int k, bool renorm,
                                    float* __restrict__ w_out, int* __restrict__ id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + (size_t)warp * E;
  float v[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? row[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __expf(v[i] - mx) : 0.f;
    sum += v[i];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  float picked_sum = 0.f;
  float wsel[16];
  int isel[16];
  for (int j = 0; j < k; ++j) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > bv || (v[i] == bv && e < bi)) { bv = v[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    // remove the winner from its owner lane
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i == bi) v[i] = -1.f;
    wsel[j] = bv * inv;
    isel[j] = bi;
    picked_sum += bv * inv;
  }
  if (lane == 0) {
    const float scale = renorm ? 1.f / picked_sum : 1.f;
    for (int j = 0; j < k; ++j) {
      w_out[(size_t)warp * k + j] = wsel[j] * scale;
      id_out[(size_t)warp * k + j] = isel[j];
    }
  }
}

// Single CTA: counting sort of the T*k expert ids that fall in this rank's
// experts [e0, e0+E). offsets [E+1] (local), pos [T*k] (sorted row of each slot,
// -1 for experts of other ranks), sorted_tok [T*k] (token of each sorted row;
// rows past offsets[E] unused). Slots of one expert keep their order.
__global__ void moe_permute_kernel(const int* __restrict__ ids, int n, int k, int e0, int E,
                                   int* __restrict__ offsets, int* __restrict__ pos, int* __restrict__ sorted_tok) {
  extern __shared__ int cnt[];  // [E]
  pdl_wait();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i] - e0;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      const int c = cnt[e];
      offsets[e] = run;
      cnt[e] = run;
      run += c;
    }
    offsets[E] = run;
    for (int i = 0; i < n; ++i) {
      const int e = ids[i] - e0;
      if (e >= 0 && e < E) {
        const int p = cnt[e]++;
        pos[i] = p;
        sorted_tok[p] = i / k;
      } else {
        pos[i] = -1;
      }
    }
  }
}

// out[t, :] = sum_j w[t, j] * y[pos[t*k + j], :] over this rank's slots (pos >= 0); bf16 out.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const float* __restrict__ w,
                                   const int* __restrict__ pos, int k, int H, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < k; ++j) {
      const int p = pos[t * k + j];
      if (p < 0) continue;
      const float wt = w[t * k + j];
      float f[8];
      unpack8(*reinterpret_cast<const bf16x8*>(y + (size_t)p * H + c), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += wt * f[i];
    }
    *reinterpret_cast<bf16x8*>(out + (size_t)t * H + c) = pack8(acc);
  }
}

// Combine fused with the expert-parallel reduction: like moe_combine_kernel, but every CTA
// stores its combined row into the receive slot of every rank (NVLink P2P); the CTA that
// finishes last publishes flag[r] = epoch on every rank (one system fence, relaxed stores).
struct CombinePush {
  __nv_bfloat16* dst[8];
  int* flag[8];
  int world;
  int* done;                 // local counter of finished CTAs, zero on entry and exit
  const int* epoch;
};

__global__ void moe_combine_push_kernel(const __nv_bfloat16* __restrict__ y, const float* __restrict__ w,
                                        const int* __restrict__ pos, int k, int H, const CombinePush cp) {
  pdl_wait();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < k; ++j) {
      const int p = pos[t * k + j];
      if (p < 0) continue;
      const float wt = w[t * k + j];
      float f[8];
      unpack8(*reinterpret_cast<const bf16x8*>(y + (size_t)p * H + c), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += wt * f[i];
    }
    const bf16x8 v = pack8(acc);
    for (int r = 0; r < cp.world; ++r) *reinterpret_cast<bf16x8*>(cp.dst[r] + (size_t)t * H + c) = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(cp.done, 1);
    if (old == (int)gridDim.x - 1) {
      *cp.done = 0;
      __threadfence_system();
      const int e = *cp.epoch;
      for (int r = 0; r < cp.world; ++r)
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(cp.flag[r]), "r"(e) : "memory");
    }
  }
}

__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ rows,
                                   const int* __restrict__ count, int H, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  if ((int)blockIdx.x >= *count) return;
  const int r = rows[blockIdx.x];
  const bf16x8* src = reinterpret_cast<const bf16x8*>(x + (size_t)r * H);
  bf16x8* dst = reinterpret_cast<bf16x8*>(out + (size_t)blockIdx.x * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

}  // namespace b200

using namespace b200;

void topk_softmax(torch::Tensor logits, int64_t k, bool renorm, torch::Tensor w_out, torch::Tensor id_out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous());
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= 256 && k <= 16 && k <= E);
  if (T == 0) return;
  const int threads = 128;
  const int blocks = (T * 32 + threads - 1) / threads;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int epl = (E + 31) / 32;
#define B200_TK(N) topk_softmax_kernel<N><<<blocks, threads, 0, stream>>>(logits.data_ptr<float>(), T, E, (int)k, renorm, \
                                                                         w_out.data_ptr<float>(), id_out.data_ptr<int>())
  if (epl <= 1) B200_TK(1);
  else if (epl <= 2) B200_TK(2);
  else if (epl <= 4) B200_TK(4);
  else B200_TK(8);
#undef B200_TK
  B200_CHECK_CUDA(cudaGetLastError());
}

void moe_permute(torch::Tensor ids, int64_t k, int64_t e0, int64_t E, torch::Tensor offsets, torch::Tensor pos,
                 torch::Tensor sorted_tok) {
  const int n = ids.numel();
  if (n == 0) return;
  moe_permute_kernel<<<1, 256, E * sizeof(int), at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int>(), n, (int)k, (int)e0, (int)E, offsets.data_ptr<int>(), pos.data_ptr<int>(),
      sorted_tok.data_ptr<int>());
  B200_CHECK_CUDA(cudaGetLastError());
}

// rows of x listed in rows[0:count] (count read on the device) -> out [max_rows, H]
void gather_rows(torch::Tensor x, torch::Tensor rows, torch::Tensor count, torch::Tensor out) {
  const int R = out.size(0), H = x.size(1);
  if (R == 0) return;
  gather_rows_kernel<<<R, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), rows.data_ptr<int>(), count.data_ptr<int>(), H,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  B200_CHECK_CUDA(cudaGetLastError());
}

void moe_combine(torch::Tensor y, torch::Tensor w, torch::Tensor pos, int64_t k, torch::Tensor out) {
  const int T = out.size(0), H = out.size(1);
  TORCH_CHECK(H % 8 == 0);
  if (T == 0) return;
  moe_combine_kernel<<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), w.data_ptr<float>(), pos.data_ptr<int>(), (int)k, H,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  B200_CHECK_CUDA(cudaGetLastError());
}

// y [rows, H] expert outputs, w/pos [T, k]; dst_ptrs/flag_ptrs host int64 [world]; done int32 [1].
void moe_combine_push(torch::Tensor y, torch::Tensor w, torch::Tensor pos, int64_t k, int64_t T, int64_t H,
                      torch::Tensor dst_ptrs, torch::Tensor flag_ptrs, int64_t epoch_ptr, torch::Tensor done) {
  const int world = dst_ptrs.numel();
  TORCH_CHECK(H % 8 == 0 && world >= 1 && world <= 8 && flag_ptrs.numel() == world && dst_ptrs.device().is_cpu());
  if (T == 0) return;
  CombinePush cp{};
  cp.world = world;
  cp.done = done.data_ptr<int>();
  cp.epoch = reinterpret_cast<const int*>(epoch_ptr);
  for (int r = 0; r < world; ++r) {
    cp.dst[r] = reinterpret_cast<__nv_bfloat16*>(dst_ptrs.data_ptr<int64_t>()[r]);
    cp.flag[r] = reinterpret_cast<int*>(flag_ptrs.data_ptr<int64_t>()[r]);
  }
  launch_pdl(moe_combine_push_kernel, dim3((unsigned)T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), w.data_ptr<float>(), pos.data_ptr<int>(), (int)k,
             (int)H, cp);
}
