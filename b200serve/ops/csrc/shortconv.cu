// LFM2 gated short convolution (reference behaviour: shaders/short_conv.wgsl:37,
// conv1d.wgsl:57-82). After the input projection y = [B | C | x] (C channels each):
//   out[t, c] = C[t, c] * sum_j w[c, j] * bx[t - (K-1) + j, c],   bx = B * x
// Taps before the batch's first token of a sequence come from the per-sequence conv
// state [slots][C][K-1] (zero when the sequence starts at position 0). Two launches: the
// output for every (token, channel) reads the old state; a second pass per (sequence,
// channel) then rolls the state to the last K-1 inputs.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace b200 {

namespace {
constexpr int kMaxTaps = 8;

__device__ __forceinline__ int sc_seq_of(const int* __restrict__ cu_q, int S, int t) {
  if (cu_q == nullptr) return t;
  int lo = 0, hi = S - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_q[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float bx_at(const __nv_bfloat16* __restrict__ y, int ystride, int t, int c, int C) {
  const __nv_bfloat16* row = y + (size_t)t * ystride;
  return __bfloat162float(__float2bfloat16_rn(__bfloat162float(row[c]) * __bfloat162float(row[2 * C + c])));
}
}  // namespace

__global__ void shortconv_out_kernel(const __nv_bfloat16* __restrict__ y, int ystride, const float* __restrict__ w,
                                     const float* __restrict__ state, const int* __restrict__ cu_q,
                                     const int* __restrict__ q_start, const int* __restrict__ slots,
                                     __nv_bfloat16* __restrict__ out, int T, int S, int C, int K, int nstates) {
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)T * C;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / C), c = (int)(i % C);
    const int s = sc_seq_of(cu_q, S, t);
    const int r = t - (cu_q ? cu_q[s] : s);
    const bool hist = q_start[s] > 0;
    if (!B200_IN_RANGE(slots[s], nstates, 0x511)) continue;
    const float* st = state + ((size_t)slots[s] * C + c) * (K - 1);
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
      const int m = K - 1 - j;
      float v = 0.f;
      if (r >= m) v = bx_at(y, ystride, t - m, c, C);
      else if (hist) v = st[(K - 1) - (m - r)];
      acc += w[c * K + j] * v;
    }
    const float gate = __bfloat162float(y[(size_t)t * ystride + C + c]);
    out[i] = __float2bfloat16_rn(gate * __bfloat162float(__float2bfloat16_rn(acc)));
  }
}

__global__ void shortconv_roll_kernel(const __nv_bfloat16* __restrict__ y, int ystride, float* __restrict__ state,
                                      const int* __restrict__ cu_q, const int* __restrict__ q_start,
                                      const int* __restrict__ slots, int S, int C, int K, int nstates) {
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)S * C;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int s = (int)(i / C), c = (int)(i % C);
    const int t0 = cu_q ? cu_q[s] : s;
    const int len = cu_q ? cu_q[s + 1] - t0 : 1;
    if (len <= 0) continue;
    const bool hist = q_start[s] > 0;
    if (!B200_IN_RANGE(slots[s], nstates, 0x512)) continue;
    float* st = state + ((size_t)slots[s] * C + c) * (K - 1);
    float old[kMaxTaps];
    for (int q = 0; q < K - 1; ++q) old[q] = hist ? st[q] : 0.f;
    for (int q = 0; q < K - 1; ++q) {
      const int p = len - (K - 1) + q;
      st[q] = p >= 0 ? bx_at(y, ystride, t0 + p, c, C) : old[(K - 1) + p];
    }
  }
}

}  // namespace b200

using namespace b200;

void shortconv_layer(torch::Tensor y, torch::Tensor conv_w, torch::Tensor conv_state,
                     c10::optional<torch::Tensor> cu_q, torch::Tensor q_start, torch::Tensor slots,
                     torch::Tensor out) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == torch::kBFloat16 && y.stride(1) == 1);
  TORCH_CHECK(conv_w.scalar_type() == torch::kFloat32 && conv_w.is_contiguous());
  TORCH_CHECK(conv_state.scalar_type() == torch::kFloat32 && conv_state.is_contiguous());
  TORCH_CHECK(q_start.scalar_type() == torch::kInt && slots.scalar_type() == torch::kInt);
  const int C = conv_w.size(0), K = conv_w.size(1);
  TORCH_CHECK(K >= 2 && K <= kMaxTaps, "conv taps must be 2..8");
  TORCH_CHECK(y.size(1) >= 3 * C && conv_state.size(1) == C && conv_state.size(2) == K - 1);
  TORCH_CHECK(out.is_contiguous() && out.size(1) == C);
  const int T = y.size(0);
  const int S = cu_q ? (int)cu_q->size(0) - 1 : T;
  TORCH_CHECK(slots.size(0) >= S && q_start.size(0) >= S);
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int* cu = cu_q ? cu_q->data_ptr<int>() : nullptr;
  const long n = (long)T * C;
  const int blocks = (int)std::min<long>((n + 255) / 256, 148L * 16);
  launch_pdl(shortconv_out_kernel, dim3(blocks), dim3(256), 0, stream, (const __nv_bfloat16*)y.data_ptr(),
             (int)y.stride(0), conv_w.data_ptr<float>(), (const float*)conv_state.data_ptr<float>(), cu,
             q_start.data_ptr<int>(), slots.data_ptr<int>(), (__nv_bfloat16*)out.data_ptr(), T, S, C, K,
             (int)conv_state.size(0));
  const long n2 = (long)S * C;
  const int blocks2 = (int)std::min<long>((n2 + 255) / 256, 148L * 16);
  launch_pdl(shortconv_roll_kernel, dim3(blocks2), dim3(256), 0, stream, (const __nv_bfloat16*)y.data_ptr(),
             (int)y.stride(0), conv_state.data_ptr<float>(), cu, q_start.data_ptr<int>(), slots.data_ptr<int>(), S,
             C, K, (int)conv_state.size(0));
  B200_CHECK_CUDA(cudaGetLastError());
}

B200_BOUNDS_ACCESSOR(shortconv)
