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
  pdl_wait();
  pdl_trigger();
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
  launch_pdl(argmax_rows_kernel, dim3(B), dim3(512), 0, at::cuda::getCurrentCUDAStream(),
             (const float*)logits.data_ptr<float>(), V, (int)logits.stride(0), out_idx.data_ptr<int>(),
             out_val.numel() ? out_val.data_ptr<float>() : (float*)nullptr, (int)index_offset);
}

void argmax_merge(torch::Tensor vals, torch::Tensor idx, torch::Tensor out) {
  const int R = vals.size(0), B = vals.size(1);
  if (B == 0) return;
  argmax_merge_kernel<<<(B + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      vals.data_ptr<float>(), idx.data_ptr<int>(), R, B, out.data_ptr<int>());
  B200_CHECK_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Full sampler: penalties, temperature, top-k, top-p, min-p, seeded draw.
// Semantics follow the reference CPU sampler (webgpu/src/engine/generate.ts:274-510)
// and HF logits processors; the draw is a Gumbel-max over the kept tokens,
// which samples exactly from the softmax restricted to them.
// ---------------------------------------------------------------------------
namespace b200 {

// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC 2011): 10 rounds of two 32x32->64
// multiplies with the paper's multipliers and Weyl key increments.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += W0;
    k.y += W1;
  }
  return c;
}

__device__ __forceinline__ uint32_t ordered_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct SampleRow {
  float temperature, top_p, min_p;
  int top_k;
  uint64_t seed;
  uint32_t step;
};

// Largest key K such that  sum over {key >= K} of weight  >= target  (weight = 1 for counts,
// = exp((x - m) / t) for probability mass). Radix select over 4 digits of 8 bits.
template <bool MASS>
__device__ uint32_t radix_select_desc(const float* row, int V, uint32_t floor_key, float m, float inv_t,
                                      float target, float* hist, float* sh) {
  uint32_t prefix = 0, mask = 0;
  float remaining = target;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0.f;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float x = row[i];
      const uint32_t key = ordered_key(x);
      if (key >= floor_key && (key & mask) == prefix) {
        const float wgt = MASS ? __expf((x - m) * inv_t) : 1.f;
        atomicAdd(&hist[(key >> shift) & 255u], wgt);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float cum = 0.f;
      int d = 255;
      for (; d > 0; --d) {
        if (cum + hist[d] >= remaining) break;
        cum += hist[d];
      }
      sh[0] = remaining - cum;
      sh[1] = __uint_as_float((uint32_t)d);
    }
    __syncthreads();
    remaining = sh[0];
    prefix |= __float_as_uint(sh[1]) << shift;
    mask |= 255u << shift;
    __syncthreads();
  }
  return prefix;
}

__global__ void __launch_bounds__(1024) sample_rows_kernel(float* __restrict__ logits, int V, int ld,
                                                           const SampleRow* __restrict__ params,
                                                           const int* __restrict__ pen_ids,
                                                           const float* __restrict__ pen_counts, int P,
                                                           const float* __restrict__ pen_vals,
                                                           int* __restrict__ out) {
  __shared__ float hist[256];
  __shared__ float red[32];
  __shared__ float sh[4];
  __shared__ int shi[32];
  float* row = logits + (size_t)blockIdx.x * ld;
  const SampleRow pr = params[blockIdx.x];
  // ---- penalties (ids unique per row): repetition, presence, frequency ----
  if (P > 0) {
    const float rp = pen_vals[blockIdx.x * 3 + 0], pres = pen_vals[blockIdx.x * 3 + 1],
                freq = pen_vals[blockIdx.x * 3 + 2];
    for (int j = threadIdx.x; j < P; j += blockDim.x) {
      const int id = pen_ids[blockIdx.x * P + j];
      if (id < 0 || id >= V) continue;
      float x = row[id];
      if (rp != 1.f) x = x > 0.f ? x / rp : x * rp;
      x -= pres + freq * pen_counts[blockIdx.x * P + j];
      row[id] = x;
    }
    __syncthreads();
  }
  // ---- row max (also the greedy answer) ----
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) better(bv, bi, row[i], i);
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) { red[warp] = bv; shi[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = lane < nw ? red[lane] : -INFINITY;
    bi = lane < nw ? shi[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      better(bv, bi, ov, oi);
    }
    if (lane == 0) { sh[2] = bv; shi[0] = bi; }
  }
  __syncthreads();
  const float m = sh[2];
  if (!(pr.temperature > 0.f)) {
    if (threadIdx.x == 0) out[blockIdx.x] = shi[0];
    return;
  }
  __syncthreads();
  const float inv_t = 1.f / pr.temperature;
  // ---- top-k threshold ----
  uint32_t floor_key = 0;
  if (pr.top_k > 0 && pr.top_k < V)
    floor_key = radix_select_desc<false>(row, V, 0, m, inv_t, (float)pr.top_k, hist, sh);
  // ---- min-p: keep p >= min_p * p_max  <=>  x >= m + t * ln(min_p) ----
  if (pr.min_p > 0.f) {
    const uint32_t k2 = ordered_key(m + pr.temperature * __logf(pr.min_p));
    floor_key = max(floor_key, k2);
  }
  // ---- top-p over the survivors ----
  if (pr.top_p < 1.f) {
    float z = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float x = row[i];
      if (ordered_key(x) >= floor_key) z += __expf((x - m) * inv_t);
    }
    z = block_sum(z, red);
    const uint32_t kp = radix_select_desc<true>(row, V, floor_key, m, inv_t, pr.top_p * z, hist, sh);
    floor_key = max(floor_key, kp);
  }
  // ---- Gumbel-max draw over kept tokens ----
  float best = -INFINITY;
  int best_i = 0x7fffffff;
  const uint2 key = make_uint2((uint32_t)pr.seed, (uint32_t)(pr.seed >> 32));
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = row[i];
    if (ordered_key(x) < floor_key) continue;
    const uint4 r = philox4x32_10(make_uint4((uint32_t)i, pr.step, blockIdx.x, 0x5A4D504Cu), key);
    const float u = ((float)(r.x >> 8) + 0.5f) * (1.f / 16777216.f);
    const float g = -__logf(-__logf(u));
    better(best, best_i, x * inv_t + g, i);
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    better(best, best_i, ov, oi);
  }
  __syncthreads();
  if (lane == 0) { red[warp] = best; shi[warp] = best_i; }
  __syncthreads();
  if (warp == 0) {
    best = lane < nw ? red[lane] : -INFINITY;
    best_i = lane < nw ? shi[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      better(best, best_i, ov, oi);
    }
    if (lane == 0) out[blockIdx.x] = best_i == 0x7fffffff ? shi[0] : best_i;
  }
}

}  // namespace b200

// logits [B, V] fp32 (modified in place by penalties); params: int64 [B, 6] packed as
// (temperature bits, top_p bits, min_p bits, top_k, seed, step); pen_ids [B, P] int32 (-1 pad),
// pen_counts [B, P] fp32, pen_vals [B, 3] fp32 (repeat, presence, frequency).
void sample_rows(torch::Tensor logits, torch::Tensor params, torch::Tensor pen_ids, torch::Tensor pen_counts,
                 torch::Tensor pen_vals, torch::Tensor out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1);
  TORCH_CHECK(params.scalar_type() == at::kByte && params.numel() == logits.size(0) * (int64_t)sizeof(b200::SampleRow));
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const int P = pen_ids.numel() ? pen_ids.size(1) : 0;
  b200::sample_rows_kernel<<<B, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), V, logits.stride(0), reinterpret_cast<const b200::SampleRow*>(params.data_ptr()),
      P ? pen_ids.data_ptr<int>() : nullptr, P ? pen_counts.data_ptr<float>() : nullptr, P,
      P ? pen_vals.data_ptr<float>() : nullptr, out.data_ptr<int>());
  B200_CHECK_CUDA(cudaGetLastError());
}
