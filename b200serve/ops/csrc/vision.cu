// Row and elementwise kernels of the vision tower (Qwen3-VL style ViT; the GEMMs are the tcgen05
// GEMM and the attention is the tcgen05 prefill attention):
//   layernorm_rows   out = (x - mean) / sqrt(var + eps) * w + b over rows of bf16 (fp32 statistics)
//   gelu_rows        x = gelu(x) in place, exact (erf) or the tanh approximation
//   vision_qkv_rope  qkv rows [N, 3 * heads * hd] -> rotary (rotate-half pairs (d, d + hd/2) with
//                    per-patch cos/sin of the 2-D patch position) on q and k, then q [N, heads, 128]
//                    and K/V scattered into a paged cache [blocks, heads, 16, 128], zero-padded from
//                    hd to 128 (the padding adds nothing to q.k and is dropped from the output)
// The vision math (LayerNorm eps 1e-6, GELU, 2-D rotary of the first half / second half of the
// rotary dims by row / column) is the checkpoint format's: the model definition the weights
// were trained with.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace b200 {

// One CTA per row; D up to 8192.
__global__ void __launch_bounds__(256) layernorm_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                             const __nv_bfloat16* __restrict__ w,
                                                             const __nv_bfloat16* __restrict__ b, int D, float eps,
                                                             __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const __nv_bfloat16* row = x + (size_t)blockIdx.x * D;
  float s = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) s += __bfloat162float(row[i]);
  const float mean = block_sum(s, red) / D;
  float v = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float d = __bfloat162float(row[i]) - mean;
    v += d * d;
  }
  const float rstd = rsqrtf(block_sum(v, red) / D + eps);
  __nv_bfloat16* o = out + (size_t)blockIdx.x * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float y = (__bfloat162float(row[i]) - mean) * rstd;
    o[i] = __float2bfloat16_rn(y * __bfloat162float(w[i]) + (b ? __bfloat162float(b[i]) : 0.f));
  }
}

__global__ void gelu_rows_kernel(__nv_bfloat16* __restrict__ x, size_t n, int tanh_approx) {
  pdl_wait();
  pdl_trigger();
  const float k0 = 0.7978845608028654f;   // sqrt(2 / pi)
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = __bfloat162float(x[i]);
    const float g = tanh_approx ? 0.5f * v * (1.f + tanhf(k0 * (v + 0.044715f * v * v * v)))
                                : 0.5f * v * (1.f + erff(v * 0.7071067811865476f));
    x[i] = __float2bfloat16_rn(g);
  }
}

// grid (N, heads), block 128 (one thread per padded dim). cs: [N, hd] fp32 cos then [N, hd] sin.
__global__ void vision_qkv_rope_kernel(const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ cosv,
                                       const float* __restrict__ sinv, int heads, int hd,
                                       const int* __restrict__ slots, __nv_bfloat16* __restrict__ q_out,
                                       __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                                       int cache_slots) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int H = heads * hd;
  const __nv_bfloat16* row = qkv + (size_t)t * 3 * H;
  const int half = hd / 2;
  float qv = 0.f, kv = 0.f, vv = 0.f;
  if (d < hd) {
    const float c = cosv[(size_t)t * hd + d], s = sinv[(size_t)t * hd + d];
    const int pd = d < half ? d + half : d - half;           // rotate-half partner
    const float sg = d < half ? -1.f : 1.f;
    const float q0 = __bfloat162float(row[h * hd + d]), q1 = __bfloat162float(row[h * hd + pd]);
    const float k0 = __bfloat162float(row[H + h * hd + d]), k1 = __bfloat162float(row[H + h * hd + pd]);
    qv = q0 * c + sg * q1 * s;
    kv = k0 * c + sg * k1 * s;
    vv = __bfloat162float(row[2 * H + h * hd + d]);
  }
  q_out[((size_t)t * heads + h) * 128 + d] = __float2bfloat16_rn(qv);
  const int slot = slots[t];
  if (!B200_IN_RANGE(slot, cache_slots, 0x801)) return;
  const size_t kvo = (((size_t)(slot >> 4) * heads + h) * 16 + (slot & 15)) * 128 + d;
  k_cache[kvo] = __float2bfloat16_rn(kv);
  v_cache[kvo] = __float2bfloat16_rn(vv);
}

}  // namespace b200

using namespace b200;

void layernorm_rows(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, double eps, torch::Tensor out) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && out.is_contiguous() && x.dim() == 2);
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(w.numel() == D && (!b || b->numel() == D), "weight / bias size");
  if (T == 0) return;
  launch_pdl(layernorm_rows_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
             b ? reinterpret_cast<const __nv_bfloat16*>(b->data_ptr()) : nullptr, D, (float)eps,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
}

void gelu_rows(torch::Tensor x, bool tanh_approx) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous());
  const size_t n = x.numel();
  if (n == 0) return;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 16);
  launch_pdl(gelu_rows_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), n, tanh_approx ? 1 : 0);
}

// qkv [N, 3 * heads * hd] bf16; cos_sin [2, N, hd] fp32; slots [N] int32 (paged slot of each patch);
// q_out [N, heads, 128]; k_cache / v_cache [blocks, heads, 16, 128] bf16.
void vision_qkv_rope(torch::Tensor qkv, torch::Tensor cos_sin, int64_t heads, int64_t hd, torch::Tensor slots,
                     torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache) {
  const int N = qkv.size(0);
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() && qkv.size(1) == 3 * heads * hd);
  TORCH_CHECK(hd <= 128 && hd % 2 == 0, "head_dim up to 128");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.numel() == 2LL * N * hd);
  TORCH_CHECK(k_cache.size(1) == heads && k_cache.size(2) == 16 && k_cache.size(3) == 128 && q_out.is_contiguous());
  TORCH_CHECK(slots.scalar_type() == at::kInt && slots.numel() == N);
  if (N == 0) return;
  launch_pdl(vision_qkv_rope_kernel, dim3(N, (unsigned)heads), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), cos_sin.data_ptr<float>(),
             cos_sin.data_ptr<float>() + (size_t)N * hd, (int)heads, (int)hd, slots.data_ptr<int>(),
             reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), (int)(k_cache.size(0) * 16));
}

B200_BOUNDS_ACCESSOR(vision)
