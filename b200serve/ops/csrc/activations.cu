// Gated activations other than SwiGLU (which the GEMM epilogue fuses).
// gelu_tanh_mul: act = gelu_tanh(gate) * up on the gate/up GEMM output, whose 64-column
// blocks interleave gate and up ([g(0..63) u(0..63) g(64..127) ...], see norm_rope.cu's
// silu_mul). GeGLU of the Gemma family (reference behaviour: elementwise.wgsl gate_gelu).
// gelu_tanh(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), the tanh approximation
// of Hendrycks & Gimpel.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace b200 {

__global__ void gelu_tanh_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ act, int T,
                                     int I) {
  pdl_wait();
  pdl_trigger();
  const size_t n8 = (size_t)T * I / 8;
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < n8; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    const size_t t = e / I;
    const int j = (int)(e % I);
    const int blk = j >> 6, within = j & 63;
    const __nv_bfloat16* row = gu + t * 2 * (size_t)I;
    float g[8], u[8], o[8];
    unpack8(*reinterpret_cast<const bf16x8*>(row + blk * 128 + within), g);
    unpack8(*reinterpret_cast<const bf16x8*>(row + blk * 128 + 64 + within), u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = g[i];
      const float gg = __bfloat162float(__float2bfloat16_rn(0.5f * x * (1.f + tanhf(k0 * (x + 0.044715f * x * x * x)))));
      o[i] = gg * u[i];
    }
    *reinterpret_cast<bf16x8*>(act + e) = pack8(o);
  }
}

// x[t, :] *= sigmoid(g[t]) (the sigmoid gate of a shared expert)
__global__ void row_sigmoid_scale_kernel(__nv_bfloat16* __restrict__ x, const float* __restrict__ g, int T, int H) {
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)T * H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float s = 1.f / (1.f + __expf(-g[i / H]));
    x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) * s);
  }
}

// x = cap * tanh(x / cap) in place (fp32 logits; Gemma 2's final logit softcapping)
__global__ void softcap_kernel(float* __restrict__ x, size_t n, float cap) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = cap * tanhf(x[i] / cap);
}

}  // namespace b200

using namespace b200;

void softcap_(torch::Tensor x, double cap) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == torch::kFloat32);
  const size_t n = x.numel();
  if (n == 0) return;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 16);
  launch_pdl(softcap_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(), x.data_ptr<float>(), n,
             (float)cap);
  B200_CHECK_CUDA(cudaGetLastError());
}

void row_sigmoid_scale(torch::Tensor x, torch::Tensor g) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == torch::kBFloat16 && g.scalar_type() == torch::kFloat32);
  TORCH_CHECK(g.numel() == x.size(0));
  const int T = x.size(0), H = x.size(1);
  if (T == 0) return;
  const long n = (long)T * H;
  const int blocks = (int)std::min<long>((n + 255) / 256, 148L * 16);
  launch_pdl(row_sigmoid_scale_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             (__nv_bfloat16*)x.data_ptr(), g.data_ptr<float>(), T, H);
  B200_CHECK_CUDA(cudaGetLastError());
}

void gelu_tanh_mul(torch::Tensor gu, torch::Tensor act) {
  const int I = act.size(-1);
  const int T = act.numel() / I;
  TORCH_CHECK(I % 64 == 0 && gu.size(-1) == 2 * I && gu.is_contiguous() && act.is_contiguous());
  TORCH_CHECK(gu.scalar_type() == torch::kBFloat16 && act.scalar_type() == torch::kBFloat16);
  if (T == 0) return;
  const long n8 = (long)T * I / 8;
  const int blocks = (int)std::min<long>((n8 + 255) / 256, 148L * 16);
  launch_pdl(gelu_tanh_mul_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)act.data_ptr(), T, I);
  B200_CHECK_CUDA(cudaGetLastError());
}
