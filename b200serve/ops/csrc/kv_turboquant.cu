// TurboQuant KV cache kernels (head_dim 128): encode on write, query preparation, and page
// dequantisation for prefill. The codec is the one of the CPU TurboQuantCodec
// (reference core/turboquant_cache.py:41-200, webgpu/src/shaders/turboquant_encode.wgsl:51):
//   n = ||x||, u = H(x / n) with H the normalised Walsh-Hadamard transform,
//   code = Lloyd-Max bin of sqrt(d) * u_i plus its sign, u_hat = +-centroid / sqrt(d);
//   keys only: r = u - u_hat, one sign bit per row of S r (S = the fixed Gaussian JL matrix),
//   and gamma = alpha * ||r|| / ||S^T s||, so the key estimate is n * (u_hat + gamma * S^T s).
// The paged GPU layout keeps one 4-bit code per dimension (byte m = dims 2m | 2m+1 << 4) so a
// page dequantises with one table lookup per pair of dims; the 1..4-bit codebooks all fit.
//
// Work split: one warp per head vector, lane l owns dims 4l..4l+3. The transform runs in
// registers and over lane shuffles; S (64 KB fp32) is staged once per CTA in shared memory with a
// 129-float row pitch, and S r / S^T s are computed with lane l owning rows (or columns) l + 32j,
// which keeps every shared-memory access conflict free.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

constexpr int kTqW = 8;          // warps per CTA
constexpr int kSP = 129;         // shared-memory row pitch of S

struct TqCodec {
  float thr_k[8], thr_v[8];      // magnitude thresholds (levels - 1 used)
  int lev_k, lev_v;              // 2^(bits - 1)
  float alpha;                   // QJL shrinkage
};

__device__ __forceinline__ void fwht128(float (&u)[4], int lane) {
  float a, b;
  a = u[0]; b = u[1]; u[0] = a + b; u[1] = a - b;
  a = u[2]; b = u[3]; u[2] = a + b; u[3] = a - b;
  a = u[0]; b = u[2]; u[0] = a + b; u[2] = a - b;
  a = u[1]; b = u[3]; u[1] = a + b; u[3] = a - b;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float p = __shfl_xor_sync(0xffffffffu, u[e], m);
      u[e] = upper ? (p - u[e]) : (u[e] + p);
    }
  }
  const float inv = 0.08838834764831845f;   // 1 / sqrt(128)
#pragma unroll
  for (int e = 0; e < 4; ++e) u[e] *= inv;
}

__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&x)[4]) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  x[0] = bf16_lo(w.x); x[1] = bf16_hi(w.x); x[2] = bf16_lo(w.y); x[3] = bf16_hi(w.y);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&x)[4]) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
}

// quantise u (4 dims) -> 4-bit codes and u_hat
__device__ __forceinline__ void tq_quant(const float (&u)[4], const float* thr, int lev, const float* cent,
                                         int (&idx)[4], float (&uh)[4]) {
  const float sq = 11.313708498984761f;   // sqrt(128)
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float s = u[e] * sq;
    const float a = fabsf(s);
    int bin = 0;
    for (int t = 0; t < lev - 1; ++t) bin += a > thr[t] ? 1 : 0;
    idx[e] = s >= 0.f ? bin : bin + lev;
    uh[e] = (s >= 0.f ? cent[bin] : -cent[bin]) / sq;
  }
}

__device__ __forceinline__ void load_S(const float* __restrict__ S, float* sS) {
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) sS[(i >> 7) * kSP + (i & 127)] = S[i];
  __syncthreads();
}

// Vectors 0 .. T*nq-1: queries -> q_rot = H q, q_jl = S q_rot. Vectors T*nq ..: new K/V rows
// (read from the staging pages written by qkv_post, token t at row ((t/16)*nkv + h)*16 + t%16)
// encoded into the paged cache at slots[t].
__global__ void __launch_bounds__(kTqW * 32) tq_qkv_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kst, const __nv_bfloat16* __restrict__ vst,
    const int* __restrict__ slots, int T, int nq, int nkv, const float* __restrict__ S,
    __nv_bfloat16* __restrict__ q_rot, __nv_bfloat16* __restrict__ q_jl, uint8_t* __restrict__ kc,
    uint8_t* __restrict__ ksg, __half* __restrict__ kmeta, uint8_t* __restrict__ vc, __half* __restrict__ vmeta,
    const TqCodec cd, const float* __restrict__ cent_k, const float* __restrict__ cent_v, int cache_slots,
    __nv_bfloat16* __restrict__ win_k, __nv_bfloat16* __restrict__ win_v, const int* __restrict__ win_slots,
    int win_cap) {
  extern __shared__ float sS[];
  __shared__ float vec[kTqW][128];
  __shared__ float cent[2][8];
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x < 16) cent[threadIdx.x >> 3][threadIdx.x & 7] = (threadIdx.x < 8 ? cent_k : cent_v)[threadIdx.x & 7];
  load_S(S, sS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sv = vec[warp];
  const int nqv = T * nq, nkvv = T * nkv;
  for (int v = blockIdx.x * kTqW + warp; v < nqv + 2 * nkvv; v += gridDim.x * kTqW) {
    float x[4];
    if (v < nqv) {
      // ---- query: rotate, then project with S ----
      load4(q + (size_t)v * 128 + 4 * lane, x);
      fwht128(x, lane);
      store4(q_rot + (size_t)v * 128 + 4 * lane, x);
#pragma unroll
      for (int e = 0; e < 4; ++e) sv[4 * lane + e] = x[e];
      __syncwarp();
      float pj[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float* row = sS + (lane + 32 * j) * kSP;
        float a = 0.f;
#pragma unroll 8
        for (int k = 0; k < 128; ++k) a += row[k] * sv[k];
        pj[j] = a;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) q_jl[(size_t)v * 128 + lane + 32 * j] = __float2bfloat16_rn(pj[j]);
      __syncwarp();
      continue;
    }
    const int w = v - nqv;
    const bool is_v = w >= nkvv;
    const int tv = is_v ? w - nkvv : w;
    const int t = tv / nkv, h = tv % nkv;
    const int slot = slots[t];
    if (slot < 0 || !B200_IN_RANGE(slot, cache_slots, 0x401)) continue;
    const size_t src = ((size_t)(t >> 4) * nkv + h) * 16 + (t & 15);
    const size_t dst = ((size_t)(slot >> 4) * nkv + h) * 16 + (slot & 15);
    load4((is_v ? vst : kst) + src * 128 + 4 * lane, x);
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float n = fmaxf(sqrtf(ss), 1e-8f);
    float u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) u[e] = x[e] / n;
    fwht128(u, lane);
    if (win_slots != nullptr) {             // residual window: the rotated row n * u in bf16
      const int wsl = win_slots[t];
      if (wsl >= 0 && B200_IN_RANGE(wsl, win_cap, 0x403)) {
        __nv_bfloat16* wd = (is_v ? win_v : win_k) + (((size_t)(wsl >> 4) * nkv + h) * 16 + (wsl & 15)) * 128 + 4 * lane;
        *reinterpret_cast<uint2*>(wd) = make_uint2(pack_bf16x2(n * u[0], n * u[1]), pack_bf16x2(n * u[2], n * u[3]));
      }
    }
    int idx[4];
    float uh[4];
    tq_quant(u, is_v ? cd.thr_v : cd.thr_k, is_v ? cd.lev_v : cd.lev_k, cent[is_v ? 1 : 0], idx, uh);
    const uint32_t packed = (uint32_t)(idx[0] | (idx[1] << 4)) | ((uint32_t)(idx[2] | (idx[3] << 4)) << 8);
    *reinterpret_cast<uint16_t*>((is_v ? vc : kc) + dst * 64 + 2 * lane) = (uint16_t)packed;
    if (is_v) {
      if (lane == 0) vmeta[dst] = __float2half_rn(n);
      continue;
    }
    // ---- keys: QJL sign bits of S r and the folded correction scale ----
    float r[4], rs = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) { r[e] = u[e] - uh[e]; rs += r[e] * r[e]; sv[4 * lane + e] = r[e]; }
    const float rn = fmaxf(sqrtf(warp_sum(rs)), 1e-8f);
    __syncwarp();
    uint32_t bits[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float* row = sS + (lane + 32 * j) * kSP;
      float a = 0.f;
#pragma unroll 8
      for (int k = 0; k < 128; ++k) a += row[k] * sv[k];
      bits[j] = __ballot_sync(0xffffffffu, a >= 0.f);
    }
    if (lane == 0) *reinterpret_cast<uint4*>(ksg + dst * 16) = make_uint4(bits[0], bits[1], bits[2], bits[3]);
    float tsq = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = lane + 32 * j;
      float a = 0.f;
#pragma unroll 4
      for (int i = 0; i < 128; ++i) {
        const float sgn = ((bits[i >> 5] >> (i & 31)) & 1u) ? 1.f : -1.f;
        a += sS[i * kSP + col] * sgn;
      }
      tsq += a * a;
    }
    const float tn = fmaxf(sqrtf(warp_sum(tsq)), 1e-8f);
    if (lane == 0) {
      kmeta[dst * 2] = __float2half_rn(n);
      kmeta[dst * 2 + 1] = __float2half_rn(cd.alpha * rn / tn);
    }
    __syncwarp();
  }
}

// Prefill: pages block_ids[j] of the TurboQuant cache -> bf16 pages j of out_k / out_v in the rotated
// domain: K = n (u_hat + gamma S^T s), V = n u_hat. One warp per (page, head, token) row.
__global__ void __launch_bounds__(kTqW * 32) tq_dequant_kernel(
    const int* __restrict__ block_ids, int n_blocks, int nkv, const uint8_t* __restrict__ kc,
    const uint8_t* __restrict__ ksg, const __half* __restrict__ kmeta, const uint8_t* __restrict__ vc,
    const __half* __restrict__ vmeta, const float* __restrict__ S, const float* __restrict__ code_vals,
    __nv_bfloat16* __restrict__ out_k, __nv_bfloat16* __restrict__ out_v, int cache_blocks) {
  extern __shared__ float sS[];
  __shared__ float cv[32];
  __shared__ float vec[kTqW][128];
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x < 32) cv[threadIdx.x] = code_vals[threadIdx.x];
  load_S(S, sS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = n_blocks * nkv * 16;
  for (int rr = blockIdx.x * kTqW + warp; rr < rows; rr += gridDim.x * kTqW) {
    const int j = rr / (nkv * 16), rest = rr % (nkv * 16);
    int blk = block_ids[j];
    if (!B200_IN_RANGE(blk, cache_blocks, 0x402)) blk = 0;   // checked builds: read block 0 instead
    const size_t src = (size_t)blk * nkv * 16 + rest;
    const size_t dst = (size_t)rr;
    // values: dims 4l..4l+3 from code bytes 2l, 2l+1
    const uint32_t vb = *reinterpret_cast<const uint16_t*>(vc + src * 64 + 2 * lane);
    const float vn = __half2float(vmeta[src]);
    float xv[4] = {cv[16 + (vb & 15)] * vn, cv[16 + ((vb >> 4) & 15)] * vn, cv[16 + ((vb >> 8) & 15)] * vn,
                   cv[16 + ((vb >> 12) & 15)] * vn};
    store4(out_v + dst * 128 + 4 * lane, xv);
    const uint32_t kb = *reinterpret_cast<const uint16_t*>(kc + src * 64 + 2 * lane);
    const float kn = __half2float(kmeta[src * 2]), kg = __half2float(kmeta[src * 2 + 1]);
    const uint4 sw = *reinterpret_cast<const uint4*>(ksg + src * 16);
    const uint32_t bits[4] = {sw.x, sw.y, sw.z, sw.w};
    // S^T s: lane computes columns lane + 32j (conflict-free), exchanged through shared memory
    float* sv = vec[warp];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = lane + 32 * j;
      float a = 0.f;
#pragma unroll 4
      for (int i = 0; i < 128; ++i) {
        const float sgn = ((bits[i >> 5] >> (i & 31)) & 1u) ? 1.f : -1.f;
        a += sS[i * kSP + col] * sgn;
      }
      sv[col] = a;
    }
    __syncwarp();
    float xk[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) xk[e] = kn * (cv[(kb >> (4 * e)) & 15] + kg * sv[4 * lane + e]);
    __syncwarp();
    store4(out_k + dst * 128 + 4 * lane, xk);
  }
}

}  // namespace b200

using namespace b200;

static TqCodec make_codec(torch::Tensor thr, int64_t kbits, int64_t vbits, double alpha) {
  // thr: host float [2][8] (K, V magnitude thresholds)
  TORCH_CHECK(thr.device().is_cpu() && thr.numel() == 16, "thresholds: host float [2, 8]");
  auto t = thr.to(at::kFloat).contiguous();
  TqCodec cd{};
  for (int i = 0; i < 8; ++i) { cd.thr_k[i] = t.data_ptr<float>()[i]; cd.thr_v[i] = t.data_ptr<float>()[8 + i]; }
  TORCH_CHECK(kbits >= 1 && kbits <= 4 && vbits >= 1 && vbits <= 4, "TurboQuant bits must be 1..4");
  cd.lev_k = 1 << (kbits - 1);
  cd.lev_v = 1 << (vbits - 1);
  cd.alpha = (float)alpha;
  return cd;
}

static int tq_grid(int64_t work_warps) {
  const int64_t ctas = (work_warps + kTqW - 1) / kTqW;
  return (int)std::max<int64_t>(1, std::min<int64_t>(ctas, 2 * 148));
}

static const size_t kTqSmem = (size_t)128 * kSP * 4;

// q [T, nq, 128] bf16; k_stage / v_stage [ceil(T/16), nkv, 16, 128] bf16 (written by qkv_post with
// slots 0..T-1); slots [T] int32 (-1 = skip); S [128, 128] fp32; cents [2, 8] fp32 (device) centroids
// of K and V; thr host [2, 8]. Outputs: q_rot, q_jl [T, nq, 128]; the layer's cache slices.
void tq_qkv(torch::Tensor q, torch::Tensor k_stage, torch::Tensor v_stage, torch::Tensor slots, torch::Tensor S,
            torch::Tensor cents, torch::Tensor thr, int64_t kbits, int64_t vbits, double alpha, torch::Tensor q_rot,
            torch::Tensor q_jl, torch::Tensor k_codes, torch::Tensor k_sign, torch::Tensor k_meta,
            torch::Tensor v_codes, torch::Tensor v_meta, torch::Tensor win_k, torch::Tensor win_v,
            torch::Tensor win_slots) {
  const int T = q.size(0), nq = q.size(1), nkv = k_codes.size(1);
  const bool win = win_slots.numel() > 0;
  if (win)
    TORCH_CHECK(win_k.scalar_type() == at::kBFloat16 && win_k.is_contiguous() && win_v.is_contiguous() &&
                    win_k.size(1) == nkv && win_k.size(3) == 128 && win_slots.scalar_type() == at::kInt &&
                    win_slots.numel() == T,
                "window pages: bf16 [pages, nkv, 16, 128]; window slots: int32 [T]");
  TORCH_CHECK(q.size(2) == 128 && q.is_contiguous() && k_stage.size(3) == 128, "TurboQuant needs head_dim 128");
  TORCH_CHECK(S.scalar_type() == at::kFloat && S.numel() == 128 * 128 && cents.numel() == 16);
  if (T == 0) return;
  const TqCodec cd = make_codec(thr, kbits, vbits, alpha);
  static bool attr = false;
  if (!attr) {
    B200_CHECK_CUDA(cudaFuncSetAttribute(tq_qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTqSmem));
    attr = true;
  }
  const float* cp = cents.data_ptr<float>();
  launch_pdl(tq_qkv_kernel, dim3(tq_grid((int64_t)T * (nq + 2 * nkv))), dim3(kTqW * 32), kTqSmem,
             at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),
             reinterpret_cast<const __nv_bfloat16*>(k_stage.data_ptr()),
             reinterpret_cast<const __nv_bfloat16*>(v_stage.data_ptr()), (const int*)slots.data_ptr<int>(), T, nq,
             nkv, (const float*)S.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(q_rot.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(q_jl.data_ptr()), k_codes.data_ptr<uint8_t>(),
             k_sign.data_ptr<uint8_t>(), reinterpret_cast<__half*>(k_meta.data_ptr()), v_codes.data_ptr<uint8_t>(),
             reinterpret_cast<__half*>(v_meta.data_ptr()), cd, cp, cp + 8, (int)(k_codes.size(0) * 16),
             win ? reinterpret_cast<__nv_bfloat16*>(win_k.data_ptr()) : nullptr,
             win ? reinterpret_cast<__nv_bfloat16*>(win_v.data_ptr()) : nullptr,
             win ? (const int*)win_slots.data_ptr<int>() : nullptr, win ? (int)(win_k.size(0) * 16) : 0);
}

// block_ids [n] int32 (device); code_vals [2, 16] fp32 (device); out_k / out_v [n, nkv, 16, 128] bf16.
void tq_dequant(torch::Tensor block_ids, torch::Tensor k_codes, torch::Tensor k_sign, torch::Tensor k_meta,
                torch::Tensor v_codes, torch::Tensor v_meta, torch::Tensor S, torch::Tensor code_vals,
                torch::Tensor out_k, torch::Tensor out_v) {
  const int n = block_ids.numel(), nkv = k_codes.size(1);
  TORCH_CHECK(code_vals.is_cuda() && code_vals.numel() == 32 && out_k.size(0) >= n);
  if (n == 0) return;
  static bool attr = false;
  if (!attr) {
    B200_CHECK_CUDA(cudaFuncSetAttribute(tq_dequant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kTqSmem));
    attr = true;
  }
  launch_pdl(tq_dequant_kernel, dim3(tq_grid((int64_t)n * nkv * 16)), dim3(kTqW * 32), kTqSmem,
             at::cuda::getCurrentCUDAStream(), (const int*)block_ids.data_ptr<int>(), n, nkv,
             k_codes.data_ptr<uint8_t>(), k_sign.data_ptr<uint8_t>(),
             reinterpret_cast<const __half*>(k_meta.data_ptr()), v_codes.data_ptr<uint8_t>(),
             reinterpret_cast<const __half*>(v_meta.data_ptr()), (const float*)S.data_ptr<float>(),
             (const float*)code_vals.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out_k.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(out_v.data_ptr()), (int)k_codes.size(0));
}

B200_BOUNDS_ACCESSOR(kv_turboquant)
