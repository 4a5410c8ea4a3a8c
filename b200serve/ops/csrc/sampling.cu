// Greedy argmax over vocabulary rows (restates argmax.wgsl:58,80: maximum value,
// lowest index on ties), plus the merge step of a vocabulary-parallel argmax
// across tensor-parallel ranks.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

// One CTA (512 threads) per row; fp32 logits read as float4.
__global__ void __launch_bounds__(512) argmax_rows_kernel(const float* __restrict__ logits, int V, int ld,
                                                          int* __restrict__ out_idx, float* __restrict__ out_val,
                                                          int index_offset) {
  const float* row = logits + (size_t)blockIdx.x * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const int V4 = ((reinterpret_cast<uintptr_t>(row) & 15) == 0 && (ld & 3) == 0) ? V / 4 : 0;
  for (int i = threadIdx.x; i < V4; i += blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(row)[i];
    better(bv, bi, v.x, 4 * i);
    better(bv, bi, v.y, 4 * i + 1);
    better(bv, bi, v.z, 4 * i + 2);
    better(bv, bi, v.w, 4 * i + 3);
  }
  for (int i = V4 * 4 + threadIdx.x; i < V; i += blockDim.x) better(bv, bi, row[i], i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __shared__ float sv[16];
  __shared__ int si[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      better(bv, bi, ov, oi);
    }
    if (lane == 0) {
      out_idx[blockIdx.x] = bi + index_offset;
      if (out_val) out_val[blockIdx.x] = bv;
    }
  }
}

// Merge per-rank (value, index) candidates [R, B] -> index [B].
__global__ void argmax_merge_kernel(const float* __restrict__ vals, const int* __restrict__ idx, int R, int B,
                                    int* __restrict__ out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int r = 0; r < R; ++r) better(bv, bi, vals[r * B + b], idx[r * B + b]);
  out[b] = bi;
}

}  // namespace b200

using namespace b200;

void argmax_rows(torch::Tensor logits, torch::Tensor out_idx, torch::Tensor out_val, int64_t index_offset) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1);
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  argmax_rows_kernel<<<B, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), V, logits.stride(0), out_idx.data_ptr<int>(),
      out_val.numel() ? out_val.data_ptr<float>() : nullptr, (int)index_offset);
  B200_CHECK_CUDA(cudaGetLastError());
}

void argmax_merge(torch::Tensor vals, torch::Tensor idx, torch::Tensor out) {
  const int R = vals.size(0), B = vals.size(1);
  if (B == 0) return;
  argmax_merge_kernel<<<(B + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      vals.data_ptr<float>(), idx.data_ptr<int>(), R, B, out.data_ptr<int>());
  B200_CHECK_CUDA(cudaGetLastError());
}
