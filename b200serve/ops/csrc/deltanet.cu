// Gated DeltaNet (the linear-attention layers of the Qwen3.5 hybrid decoder).
//
// Reference behaviour: shaders/ssm_step.wgsl:1-12 (single-token delta-rule step),
// conv1d.wgsl:28-82 (causal depthwise conv with state), l2norm.wgsl:14, and the
// gated output norm of the hybrid layers (elementwise.wgsl gates, decay_compute).
//
// Per layer and rank the fused input projection y = x W_in^T holds, per token,
//   [ q (nk*D) | k (nk*D) | v (nv*D) | z (nv*D) | b (nv) | a (nv) ]
// (D = key = value head dim). Two kernels follow the GEMM:
//
//  dn_prep   one warp per (token, q/k/v head): causal depthwise conv over the
//            sequence (taps before the batch's first token come from the
//            per-sequence conv state, or are zero when the sequence starts at
//            position 0), SiLU, L2-normalisation of the q and k heads; the v-head
//            warps also turn (a, b) into the decay exp(A softplus(a + dt)) and
//            beta = sigmoid(b).
//  dn_scan   one CTA of 2D threads per (sequence, v head): the thread pair
//            (2j, 2j+1) keeps column j of the fp32 state S [D x D] in registers
//            (D/2 rows each) and runs the recurrence over the sequence's tokens
//            in order,
//               S <- decay S;  d = beta (v - S^T k);  S <- S + k d^T;  o = S^T q,
//            then the gated RMSNorm  out = w * norm(o) * silu(z)  over the head.
//            It also rolls the conv state forward (last K-1 inputs of the
//            sequence) after the prep kernel has read the old one.
//
// Sequences: decode passes cu_q = nullptr (token t is sequence t); prefill passes
// the token offsets cu_q [S+1]. q_start[s] is the absolute position of sequence s's
// first token in this batch; state_slots[s] indexes the state buffers
// (conv [slots][conv_dim][K-1] fp32, rec [slots][nv][D][D] fp32).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace b200 {

namespace {

__device__ __forceinline__ int seq_of(const int* __restrict__ cu_q, int S, int t) {
  if (cu_q == nullptr) return t;
  int lo = 0, hi = S - 1;
  while (lo < hi) {  // last s with cu_q[s] <= t
    const int mid = (lo + hi + 1) >> 1;
    if (cu_q[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

}  // namespace

template <int D, int K>
__global__ void __launch_bounds__(256) dn_prep_kernel(
    const __nv_bfloat16* __restrict__ y, int ystride, const float* __restrict__ conv_w,
    const float* __restrict__ A, const float* __restrict__ dt_bias, const float* __restrict__ conv_state,
    const int* __restrict__ cu_q, const int* __restrict__ q_start, const int* __restrict__ slots,
    __nv_bfloat16* __restrict__ xc, float* __restrict__ gb, int T, int S, int nk, int nv) {
  constexpr int E = D / 32;
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nheads = 2 * nk + nv;
  if (warp >= T * nheads) return;
  const int t = warp / nheads, hs = warp % nheads;
  const int conv_dim = nheads * D;
  const int s = seq_of(cu_q, S, t);
  const int r = t - (cu_q ? cu_q[s] : s);
  const bool hist = q_start[s] > 0;
  const float* st = conv_state + (size_t)slots[s] * conv_dim * (K - 1);
  float x[E];
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const int c = hs * D + lane * E + i;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int m = K - 1 - j;  // how many tokens back
      float v = 0.f;
      if (r >= m) v = __bfloat162float(y[(size_t)(t - m) * ystride + c]);
      else if (hist) v = st[(size_t)c * (K - 1) + (K - 1) - (m - r)];
      acc += conv_w[c * K + j] * v;
    }
    x[i] = bf16r(silu(acc));
  }
  if (hs < 2 * nk) {  // q or k head: L2-normalise over the head
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss += x[i] * x[i];
    const float inv = rsqrtf(warp_sum(ss) + 1e-6f);
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = bf16r(x[i] * inv);
  }
  __nv_bfloat16* dst = xc + (size_t)t * conv_dim + hs * D + lane * E;
#pragma unroll
  for (int i = 0; i < E; ++i) dst[i] = __float2bfloat16_rn(x[i]);
  if (hs >= 2 * nk && lane == 0) {
    const int h = hs - 2 * nk;
    const __nv_bfloat16* row = y + (size_t)t * ystride + conv_dim + nv * D;
    const float b = __bfloat162float(row[h]), a = __bfloat162float(row[nv + h]);
    const float g = A[h] * softplus(a + dt_bias[h]);
    gb[((size_t)t * nv + h) * 2 + 0] = __expf(g);
    gb[((size_t)t * nv + h) * 2 + 1] = 1.f / (1.f + __expf(-b));
  }
}

template <int D, int K>
__global__ void __launch_bounds__(2 * D) dn_scan_kernel(
    const __nv_bfloat16* __restrict__ y, int ystride, const __nv_bfloat16* __restrict__ xc,
    const float* __restrict__ gb, const __nv_bfloat16* __restrict__ norm_w, float* __restrict__ conv_state,
    float* __restrict__ rec_state, const int* __restrict__ cu_q, const int* __restrict__ q_start,
    const int* __restrict__ slots, __nv_bfloat16* __restrict__ out, int nk, int nv, float eps) {
  constexpr int R = D / 2;         // state rows per thread
  constexpr int NW = 2 * D / 32;   // warps
  __shared__ float qs[2][D], ks[2][D];
  __shared__ float red[2][NW];
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int j = tid >> 1, half = tid & 1, i0 = half * R;
  const int lane = tid & 31, warp = tid >> 5;
  const int ratio = nv / nk, kh = h / ratio;
  const int conv_dim = (2 * nk + nv) * D;
  const int t0 = cu_q ? cu_q[s] : s;
  const int n = cu_q ? cu_q[s + 1] - t0 : 1;
  const int slot = slots[s];
  const bool hist = q_start[s] > 0;
  const float scale = rsqrtf((float)D);
  float* rs = rec_state + ((size_t)slot * nv + h) * D * D;
  float Sc[R];  // Sc[i] = S[i0 + i][j]
#pragma unroll
  for (int i = 0; i < R; ++i) Sc[i] = hist ? rs[(size_t)(i0 + i) * D + j] : 0.f;
  const float wj = __bfloat162float(norm_w[j]);
  for (int tt = 0; tt < n; ++tt) {
    const int t = t0 + tt, buf = tt & 1;
    const __nv_bfloat16* xr = xc + (size_t)t * conv_dim;
    if (tid < D) qs[buf][tid] = __bfloat162float(xr[kh * D + tid]) * scale;
    else ks[buf][tid - D] = __bfloat162float(xr[nk * D + kh * D + tid - D]);
    const float v = __bfloat162float(xr[2 * nk * D + h * D + j]);
    const float z = __bfloat162float(y[(size_t)t * ystride + conv_dim + h * D + j]);
    const float decay = gb[((size_t)t * nv + h) * 2 + 0], beta = gb[((size_t)t * nv + h) * 2 + 1];
    __syncthreads();
    const float* kk = ks[buf] + i0;
    const float* qq = qs[buf] + i0;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int i = 0; i < R; i += 4) {
      Sc[i] *= decay; Sc[i + 1] *= decay; Sc[i + 2] *= decay; Sc[i + 3] *= decay;
      a0 += Sc[i] * kk[i];
      a1 += Sc[i + 1] * kk[i + 1];
      a2 += Sc[i + 2] * kk[i + 2];
      a3 += Sc[i + 3] * kk[i + 3];
    }
    float acc = (a0 + a1) + (a2 + a3);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    const float delta = beta * (v - acc);
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
    for (int i = 0; i < R; i += 4) {
      Sc[i] += kk[i] * delta;
      Sc[i + 1] += kk[i + 1] * delta;
      Sc[i + 2] += kk[i + 2] * delta;
      Sc[i + 3] += kk[i + 3] * delta;
      o0 += Sc[i] * qq[i];
      o1 += Sc[i + 1] * qq[i + 1];
      o2 += Sc[i + 2] * qq[i + 2];
      o3 += Sc[i + 3] * qq[i + 3];
    }
    float of = (o0 + o1) + (o2 + o3);
    of += __shfl_xor_sync(0xffffffffu, of, 1);
    const float o = bf16r(of);
    const float ss = warp_sum(half ? 0.f : o * o);
    if (lane == 0) red[buf][warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += red[buf][w];
    const float normed = bf16r(o * rsqrtf(tot / (float)D + eps));
    const float res = bf16r(wj * normed) * silu(z);
    if (!half) out[(size_t)t * nv * D + h * D + j] = __float2bfloat16_rn(res);
  }
#pragma unroll
  for (int i = 0; i < R; ++i) rs[(size_t)(i0 + i) * D + j] = Sc[i];
  if (half) return;
  // roll the conv state: the last K-1 inputs of (old state ++ this batch's tokens)
  auto roll = [&](int c) {
    float* cs = conv_state + ((size_t)slot * conv_dim + c) * (K - 1);
    float old[K - 1];
#pragma unroll
    for (int q = 0; q < K - 1; ++q) old[q] = hist ? cs[q] : 0.f;
#pragma unroll
    for (int q = 0; q < K - 1; ++q) {
      const int p = n - (K - 1) + q;   // index into this batch's tokens; < 0 -> old state
      cs[q] = p >= 0 ? __bfloat162float(y[(size_t)(t0 + p) * ystride + c]) : old[(K - 1) + p];
    }
  };
  roll(2 * nk * D + h * D + j);
  if (h % ratio == 0) {   // one v head per k head rolls the shared q/k channels
    roll(kh * D + j);
    roll(nk * D + kh * D + j);
  }
}

// out[t, c] = attn[t, c] * sigmoid(gate[t, c]); gate rows have stride gstride.
__global__ void sigmoid_gate_kernel(__nv_bfloat16* __restrict__ attn, const __nv_bfloat16* __restrict__ gate,
                                    int gstride, int T, int W) {
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)T * W;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / W;
    const int c = (int)(i % W);
    const float g = __bfloat162float(gate[t * gstride + c]);
    const float a = __bfloat162float(attn[i]);
    attn[i] = __float2bfloat16_rn(a / (1.f + __expf(-g)));
  }
}

}  // namespace b200

using namespace b200;

void deltanet_layer(torch::Tensor y, torch::Tensor conv_w, torch::Tensor A, torch::Tensor dt_bias,
                    torch::Tensor norm_w, torch::Tensor conv_state, torch::Tensor rec_state,
                    c10::optional<torch::Tensor> cu_q, torch::Tensor q_start, torch::Tensor slots, torch::Tensor xc,
                    torch::Tensor gb, torch::Tensor out, int64_t nk, int64_t nv, int64_t D, double eps) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == torch::kBFloat16 && y.stride(1) == 1);
  TORCH_CHECK(conv_w.scalar_type() == torch::kFloat32 && conv_w.is_contiguous());
  TORCH_CHECK(A.scalar_type() == torch::kFloat32 && dt_bias.scalar_type() == torch::kFloat32);
  TORCH_CHECK(norm_w.scalar_type() == torch::kBFloat16);
  TORCH_CHECK(conv_state.scalar_type() == torch::kFloat32 && rec_state.scalar_type() == torch::kFloat32);
  TORCH_CHECK(q_start.scalar_type() == torch::kInt && slots.scalar_type() == torch::kInt);
  TORCH_CHECK(nk > 0 && nv % nk == 0, "value heads must be a multiple of key heads");
  const int K = conv_w.size(1);
  TORCH_CHECK(K == 4, "conv kernel size 4 only");
  const int T = y.size(0);
  const int S = cu_q ? (int)cu_q->size(0) - 1 : T;
  const int conv_dim = (2 * nk + nv) * D;
  TORCH_CHECK(conv_w.size(0) == conv_dim && conv_state.size(1) == conv_dim && conv_state.size(2) == K - 1);
  TORCH_CHECK(rec_state.size(1) == nv && rec_state.size(2) == D && rec_state.size(3) == D);
  TORCH_CHECK(y.size(1) >= conv_dim + nv * D + 2 * nv, "input projection too narrow");
  TORCH_CHECK(xc.size(0) >= T && xc.size(1) == conv_dim && gb.size(0) >= T && out.size(1) == nv * D);
  TORCH_CHECK(slots.size(0) >= S && q_start.size(0) >= S);
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int* cu = cu_q ? cu_q->data_ptr<int>() : nullptr;
  const int warps = T * (2 * nk + nv);
  const int blocks = (warps * 32 + 255) / 256;
  const int ys = (int)y.stride(0);
#define B200_DN(DV)                                                                                            \
  launch_pdl(dn_prep_kernel<DV, 4>, dim3(blocks), dim3(256), 0, stream,                                         \
             (const __nv_bfloat16*)y.data_ptr(), ys, (const float*)conv_w.data_ptr(), (const float*)A.data_ptr(), \
             (const float*)dt_bias.data_ptr(), (const float*)conv_state.data_ptr(), cu, q_start.data_ptr<int>(),  \
             slots.data_ptr<int>(), (__nv_bfloat16*)xc.data_ptr(), gb.data_ptr<float>(), T, S, (int)nk, (int)nv);  \
  launch_pdl(dn_scan_kernel<DV, 4>, dim3(S, nv), dim3(2 * DV), 0, stream, (const __nv_bfloat16*)y.data_ptr(), ys, \
             (const __nv_bfloat16*)xc.data_ptr(), (const float*)gb.data_ptr(),                                  \
             (const __nv_bfloat16*)norm_w.data_ptr(), conv_state.data_ptr<float>(), rec_state.data_ptr<float>(),  \
             cu, q_start.data_ptr<int>(), slots.data_ptr<int>(), (__nv_bfloat16*)out.data_ptr(), (int)nk,        \
             (int)nv, (float)eps)
  if (D == 128) { B200_DN(128); }
  else if (D == 64) { B200_DN(64); }
  else if (D == 32) { B200_DN(32); }
  else TORCH_CHECK(false, "DeltaNet head dim must be 32, 64 or 128");
#undef B200_DN
  B200_CHECK_CUDA(cudaGetLastError());
}

void sigmoid_gate_mul(torch::Tensor attn, torch::Tensor gate) {
  TORCH_CHECK(attn.is_contiguous() && gate.stride(1) == 1 && attn.size(0) == gate.size(0) &&
              attn.size(1) == gate.size(1));
  TORCH_CHECK(attn.scalar_type() == torch::kBFloat16 && gate.scalar_type() == torch::kBFloat16);
  const int T = attn.size(0), W = attn.size(1);
  if (T == 0) return;
  const long n = (long)T * W;
  const int blocks = (int)std::min<long>((n + 255) / 256, 148L * 16);
  launch_pdl(sigmoid_gate_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             (__nv_bfloat16*)attn.data_ptr(), (const __nv_bfloat16*)gate.data_ptr(), (int)gate.stride(0), T, W);
  B200_CHECK_CUDA(cudaGetLastError());
}
