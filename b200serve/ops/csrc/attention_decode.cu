// Paged GQA decode attention (split-KV flash-decoding) over 16-token KV pages.
//
// Restates the math of the reference's fused attention kernel
// (webgpu/src/shaders/attention.wgsl:63: QK^T, causal softmax, .V) for one new
// query token per sequence, reading K/V through a block table instead of a
// contiguous per-session buffer (forward-pass.ts:322-342 in the reference).
//
// Grid (nsplit, nkv, B); 4 warps per CTA. A CTA owns tokens
// [split*tps, min(len, (split+1)*tps)) of one (sequence, kv head) and all G
// query heads that share the kv head. Each warp streams whole 16-token pages:
//   QK: lane l takes token l&15 and half (l>>4) of the head dims, so every
//       16-byte load instruction of the warp covers 32 contiguous bytes of
//       each of the 16 key rows (full 32-byte sectors);
//   PV: lane l takes dims [l*E, l*E+E) of every value row (contiguous rows).
// Partial (m, l, acc) per CTA go to a workspace; a second kernel merges splits.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

constexpr int kPage = 16;
constexpr int kAttnWarps = 4;

template <int HD>
struct PageRegs {
  uint4 k[HD / 16];               // this lane's key chunks: 16-byte chunk (2c + half) of row (lane & 15)
  uint32_t v[16][HD / 64];        // this lane's value dims [lane*E, lane*E+E) of all 16 rows
};

template <int HD>
__device__ __forceinline__ void load_page(PageRegs<HD>& r, const __nv_bfloat16* __restrict__ k_cache,
                                          const __nv_bfloat16* __restrict__ v_cache, size_t page_off, int tok,
                                          int half, int lane) {
  constexpr int E = HD / 32;
  const __nv_bfloat16* krow = k_cache + page_off + (size_t)tok * HD;
#pragma unroll
  for (int c = 0; c < HD / 16; ++c) r.k[c] = __ldg(reinterpret_cast<const uint4*>(krow + (c * 2 + half) * 8));
  const __nv_bfloat16* vpage = v_cache + page_off + lane * E;
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    if constexpr (E == 8) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(vpage + (size_t)t * HD));
      r.v[t][0] = raw.x;
      r.v[t][1] = raw.y;
      r.v[t][2] = raw.z;
      r.v[t][3] = raw.w;
    } else if constexpr (E == 4) {
      const uint2 raw = __ldg(reinterpret_cast<const uint2*>(vpage + (size_t)t * HD));
      r.v[t][0] = raw.x;
      r.v[t][1] = raw.y;
    } else {
      r.v[t][0] = __ldg(reinterpret_cast<const uint32_t*>(vpage + (size_t)t * HD));
    }
  }
}

template <int HD, int G>
__global__ void __launch_bounds__(kAttnWarps * 32) paged_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
    const __nv_bfloat16* __restrict__ v_cache, const int* __restrict__ block_tables,
    const int* __restrict__ seq_lens, int max_blocks, int nkv, float scale_log2, int tps,
    float* __restrict__ part_acc, float* __restrict__ part_ml, __nv_bfloat16* __restrict__ out, int nsplit,
    int window = 0, float softcap = 0.f, int nblocks = 0x7fffffff) {
  constexpr int E = HD / 32;          // value dims per lane
  __shared__ float q_s[G][HD];
  __shared__ __align__(16) float p_s[kAttnWarps][kPage][G < 4 ? 4 : G];
  __shared__ float m_s[kAttnWarps][G], l_s[kAttnWarps][G];
  __shared__ float acc_s[kAttnWarps][G][HD];

  pdl_wait();
  pdl_trigger();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = seq_lens[b];
  const int nq = nkv * G;
  // sliding window: keys [len - window, len) only; pages wholly before it are skipped
  const int lo = window > 0 ? max(0, len - window) : 0;
  const int start = max(split * tps, lo & ~(kPage - 1));
  const int stop = min(len, split * tps + tps);

  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int g = i / HD, d = i % HD;
    q_s[g][d] = __bfloat162float(q[((size_t)b * nq + kvh * G + g) * HD + d]) * scale_log2;
  }
  __syncthreads();

  float m[G], l[G], acc[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
  }

  const int tok = lane & 15, half = lane >> 4;
  const int* bt = block_tables + (size_t)b * max_blocks;
  auto page_offset = [&](int page_start) {
    const int blk = max(table_block(bt, page_start / kPage, max_blocks, nblocks, 0x203), 0);   // checked: block 0
    return ((size_t)blk * nkv + kvh) * kPage * HD;
  };

  // one page: scores, online softmax, p.V
  auto consume = [&](const PageRegs<HD>& r, int page_start) {
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll
    for (int c = 0; c < HD / 16; ++c) {
      const int chunk = c * 2 + half;
      float kf[8];
      const uint4 kv = r.k[c];
      kf[0] = bf16_lo(kv.x); kf[1] = bf16_hi(kv.x); kf[2] = bf16_lo(kv.y); kf[3] = bf16_hi(kv.y);
      kf[4] = bf16_lo(kv.z); kf[5] = bf16_hi(kv.z); kf[6] = bf16_lo(kv.w); kf[7] = bf16_hi(kv.w);
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int j = 0; j < 8; ++j) s[g] = fmaf(q_s[g][chunk * 8 + j], kf[j], s[g]);
      }
    }
    const bool valid = page_start + tok < stop && page_start + tok >= lo;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] += __shfl_xor_sync(0xffffffffu, s[g], 16);
      if (softcap > 0.f) {   // logit softcapping c tanh(x / c) on the natural-scale score
        const float x = s[g] * 0.69314718055994531f;
        s[g] = softcap * tanhf(x / softcap) * 1.4426950408889634f;
      }
      if (!valid) s[g] = -INFINITY;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float bm = s[g];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float m_new = fmaxf(m[g], bm);
      const float p = exp2f(s[g] - m_new);
      float ps = p;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      const float alpha = exp2f(m[g] - m_new);
      l[g] = l[g] * alpha + ps;
      m[g] = m_new;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][e] *= alpha;
      if (half == 0) p_s[warp][tok][g] = p;
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < kPage; ++t) {
      float vf[E];
      if constexpr (E >= 4) {
#pragma unroll
        for (int w = 0; w < E / 2; ++w) { vf[2 * w] = bf16_lo(r.v[t][w]); vf[2 * w + 1] = bf16_hi(r.v[t][w]); }
      } else {
        vf[0] = bf16_lo(r.v[t][0]); vf[1] = bf16_hi(r.v[t][0]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = p_s[warp][t][g];
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][e] = fmaf(p, vf[e], acc[g][e]);
      }
    }
    __syncwarp();
  };

  // pages of this warp: start + warp*16, then every 4*16 tokens; keep the next page in flight
  constexpr int STRIDE = kAttnWarps * kPage;
  int pg = start + warp * kPage;
  if constexpr (HD > 128) {
    // a 256-dim page already takes 128 registers per lane: no second page in flight
    for (; pg < stop; pg += STRIDE) {
      PageRegs<HD> ra;
      load_page<HD>(ra, k_cache, v_cache, page_offset(pg), tok, half, lane);
      consume(ra, pg);
    }
  } else if (pg < stop) {
    PageRegs<HD> ra, rb;
    load_page<HD>(ra, k_cache, v_cache, page_offset(pg), tok, half, lane);
    while (true) {
      const int pn = pg + STRIDE;
      if (pn < stop) load_page<HD>(rb, k_cache, v_cache, page_offset(pn), tok, half, lane);
      consume(ra, pg);
      if (pn >= stop) break;
      pg = pn;
      const int pn2 = pg + STRIDE;
      if (pn2 < stop) load_page<HD>(ra, k_cache, v_cache, page_offset(pn2), tok, half, lane);
      consume(rb, pg);
      if (pn2 >= stop) break;
      pg = pn2;
    }
  }

  // ---- merge the 4 warps ----
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) { m_s[warp][g] = m[g]; l_s[warp][g] = l[g]; }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e) acc_s[warp][g][lane * E + e] = acc[g][e];
  __syncthreads();
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, m_s[w][g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = exp2f(m_s[w][g] - M);
        L += l_s[w][g] * f;
        A += acc_s[w][g][d] * f;
      }
    }
    if (nsplit == 1) {
      out[((size_t)b * nq + kvh * G + g) * HD + d] = __float2bfloat16_rn(L > 0.f ? A / L : 0.f);
    } else {
      const size_t slot = (((size_t)b * nkv + kvh) * nsplit + split) * G + g;
      part_acc[slot * HD + d] = A;
      if (d == 0) { part_ml[slot * 2] = M; part_ml[slot * 2 + 1] = L; }
    }
  }
}

// out[b, h] = sum_s w_s acc_s / sum_s w_s l_s with w_s = 2^(m_s - max m). One warp per (b, q head).
template <int HD>
__global__ void paged_decode_combine_kernel(const float* __restrict__ part_acc, const float* __restrict__ part_ml,
                                            const int* __restrict__ seq_lens, __nv_bfloat16* __restrict__ out,
                                            int B, int nkv, int G, int nsplit, int tps) {
  constexpr int E = HD / 32;
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nq = nkv * G;
  if (warp >= B * nq) return;
  const int b = warp / nq, h = warp % nq, kvh = h / G, g = h % G;
  // tps 0: every split holds a share (empty ones carry m = -inf, l = 0)
  const int used = tps > 0 ? min(nsplit, (seq_lens[b] + tps - 1) / tps) : nsplit;
  float M = -INFINITY;
  for (int s = 0; s < used; ++s) M = fmaxf(M, part_ml[((((size_t)b * nkv + kvh) * nsplit + s) * G + g) * 2]);
  float L = 0.f, A[E];
#pragma unroll
  for (int e = 0; e < E; ++e) A[e] = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < used; ++s) {
      const size_t slot = (((size_t)b * nkv + kvh) * nsplit + s) * G + g;
      const float f = exp2f(part_ml[slot * 2] - M);
      L += part_ml[slot * 2 + 1] * f;
#pragma unroll
      for (int e = 0; e < E; ++e) A[e] += part_acc[slot * HD + lane * E + e] * f;
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) out[((size_t)b * nq + h) * HD + lane * E + e] = __float2bfloat16_rn(A[e] * inv);
}

}  // namespace b200

using namespace b200;

// q [B, nq, HD]; caches [nblocks, nkv, 16, HD]; block_tables [B, max_blocks] int32; seq_lens [B] int32
// (length including the current token). workspace: part_acc [B*nkv*nsplit*G*HD], part_ml [B*nkv*nsplit*G*2].
void paged_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor out,
                            torch::Tensor part_acc, torch::Tensor part_ml, double scale, int64_t tps,
                            int64_t nsplit, int64_t window, double softcap) {
  const int B = q.size(0), nq = q.size(1), HD = q.size(2);
  const int nkv = k_cache.size(1);
  const int G = nq / nkv;
  TORCH_CHECK(k_cache.size(2) == kPage && tps % kPage == 0 && nsplit >= 1);
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt);
  if (nsplit > 1) {
    TORCH_CHECK(part_acc.numel() >= (int64_t)B * nkv * nsplit * G * HD, "attention workspace too small");
    TORCH_CHECK(part_ml.numel() >= (int64_t)B * nkv * nsplit * G * 2, "attention workspace too small");
  }
  if (B == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const float sl2 = (float)(scale * 1.4426950408889634);
  dim3 grid(nsplit, nkv, B);
  auto qp = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  auto kp = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  auto vp = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  float* pa = nsplit > 1 ? part_acc.data_ptr<float>() : nullptr;
  float* pm = nsplit > 1 ? part_ml.data_ptr<float>() : nullptr;
#define B200_DEC(HDV, GV)                                                                                    \
  launch_pdl(paged_decode_kernel<HDV, GV>, grid, dim3(kAttnWarps * 32), 0, stream, qp, kp, vp,                \
             (const int*)block_tables.data_ptr<int>(), (const int*)seq_lens.data_ptr<int>(),                  \
             (int)block_tables.size(1), nkv, sl2, (int)tps, pa, pm, op, (int)nsplit, (int)window, (float)softcap, \
             (int)k_cache.size(0))
  if (HD == 256 && G == 4) B200_DEC(256, 4);
  else if (HD == 256 && G == 2) B200_DEC(256, 2);
  else if (HD == 256 && G == 1) B200_DEC(256, 1);
  else if (HD == 256 && G == 8) B200_DEC(256, 8);
  else if (HD == 128 && G == 4) B200_DEC(128, 4);
  else if (HD == 128 && G == 8) B200_DEC(128, 8);
  else if (HD == 128 && G == 2) B200_DEC(128, 2);
  else if (HD == 128 && G == 1) B200_DEC(128, 1);
  else if (HD == 64 && G == 2) B200_DEC(64, 2);
  else if (HD == 64 && G == 1) B200_DEC(64, 1);
  else if (HD == 64 && G == 4) B200_DEC(64, 4);
  else TORCH_CHECK(false, "unsupported head_dim/group ", HD, "/", G);
#undef B200_DEC
  B200_CHECK_CUDA(cudaGetLastError());
  if (nsplit > 1) {
    const int warps = B * nq;
    const int threads = 128;
    const int blocks = (warps * 32 + threads - 1) / threads;
    auto comb = HD == 256 ? paged_decode_combine_kernel<256>
                : HD == 128 ? paged_decode_combine_kernel<128> : paged_decode_combine_kernel<64>;
    launch_pdl(comb, dim3(blocks), dim3(threads), 0, stream, (const float*)pa, (const float*)pm,
               (const int*)seq_lens.data_ptr<int>(), op, B, nkv, G, (int)nsplit, (int)tps);
  }
}

// Merge split-KV partials into out [B, nq, HD] (used by the tensor-core decode kernel); tps 0 merges
// all nsplit splits of every sequence.
void paged_decode_combine(torch::Tensor part_acc, torch::Tensor part_ml, torch::Tensor seq_lens, torch::Tensor out,
                          int64_t nkv, int64_t G, int64_t nsplit, int64_t tps) {
  const int B = out.size(0), nq = out.size(1), HD = out.size(2);
  const int threads = 128;
  const int blocks = (B * nq * 32 + threads - 1) / threads;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  TORCH_CHECK(HD == 128 || HD == 64, "paged_decode_combine supports head_dim 64 and 128, got ", HD);
  if (HD == 128)
    launch_pdl(paged_decode_combine_kernel<128>, dim3(blocks), dim3(threads), 0, stream,
               (const float*)part_acc.data_ptr<float>(), (const float*)part_ml.data_ptr<float>(),
               (const int*)seq_lens.data_ptr<int>(), op, B, (int)nkv, (int)G, (int)nsplit, (int)tps);
  else
    launch_pdl(paged_decode_combine_kernel<64>, dim3(blocks), dim3(threads), 0, stream,
               (const float*)part_acc.data_ptr<float>(), (const float*)part_ml.data_ptr<float>(),
               (const int*)seq_lens.data_ptr<int>(), op, B, (int)nkv, (int)G, (int)nsplit, (int)tps);
}

// ---------------------------------------------------------------------------
// Entry point without device allocation (declared in noalloc.h; no counterpart
// in the reference). The split-KV partials go to a fixed array compiled into
// this file instead of a caller- or framework-allocated workspace.
// ---------------------------------------------------------------------------
#include <mutex>
#include <stdio.h>
#include "noalloc.h"

namespace b200 {

static __device__ __align__(256) float g_noalloc_scratch[B200_NOALLOC_MAX_ACC_FLOATS + B200_NOALLOC_MAX_ML_FLOATS];

constexpr int kNoAllocMaxDevices = 64;
static float* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
static cudaError_t g_noalloc_setup_err[kNoAllocMaxDevices] = {cudaSuccess};
static std::once_flag g_noalloc_once[kNoAllocMaxDevices];
static thread_local char g_noalloc_msg[256] = "";

static int noalloc_fail(int code, const char* fmt, long a = 0, long b = 0) {
  snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), fmt, a, b);
  return code;
}

}  // namespace b200

extern "C" __attribute__((visibility("default"))) const char* b200_noalloc_last_error(void) {
  return b200::g_noalloc_msg;
}

extern "C" __attribute__((visibility("default"))) int b200_paged_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_tables, const int* seq_lens,
    void* out, int B, int nq, int nkv, int head_dim, int max_blocks, float scale, int tokens_per_split, int nsplit,
    cudaStream_t stream) {
  using namespace b200;
  g_noalloc_msg[0] = '\0';
  if (B < 0 || nq <= 0 || nkv <= 0 || nq % nkv != 0 || nsplit < 1 || tokens_per_split <= 0 ||
      tokens_per_split % kPage != 0)
    return noalloc_fail(1, "invalid shape (B=%ld, nsplit=%ld)", B, nsplit);
  const int G = nq / nkv;
  const long need_acc = (long)B * nkv * nsplit * G * head_dim;
  const long need_ml = (long)B * nkv * nsplit * G * 2;
  // one split writes straight to `out` and uses no scratch, so only split calls have a limit
  if (nsplit > 1 && need_acc > (long)B200_NOALLOC_MAX_ACC_FLOATS)
    return noalloc_fail(2, "scratch limit: needs %ld accumulator floats, maximum is %ld", need_acc,
                        (long)B200_NOALLOC_MAX_ACC_FLOATS);
  if (nsplit > 1 && need_ml > (long)B200_NOALLOC_MAX_ML_FLOATS)
    return noalloc_fail(2, "scratch limit: needs %ld max/sum floats, maximum is %ld", need_ml,
                        (long)B200_NOALLOC_MAX_ML_FLOATS);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(3, "cudaGetDevice failed (%ld)", (long)e);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return noalloc_fail(3, "device %ld out of range", dev);
  // once per device, with that device current: resolve the device address of the array
  std::call_once(g_noalloc_once[dev], [dev] {
    void* p = nullptr;
    g_noalloc_setup_err[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  });
  if (g_noalloc_setup_err[dev] != cudaSuccess || g_noalloc_ptr[dev] == nullptr)
    return noalloc_fail(4, "cudaGetSymbolAddress failed on device %ld (error %ld)", dev,
                        (long)g_noalloc_setup_err[dev]);
  if (B == 0) return 0;
  float* acc = g_noalloc_ptr[dev];
  float* ml = acc + B200_NOALLOC_MAX_ACC_FLOATS;
  const float sl2 = scale * 1.4426950408889634f;
  dim3 grid(nsplit, nkv, B);
  auto qp = reinterpret_cast<const __nv_bfloat16*>(q);
  auto kp = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  auto vp = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  auto op = reinterpret_cast<__nv_bfloat16*>(out);
  float* pa = nsplit > 1 ? acc : nullptr;
  float* pm = nsplit > 1 ? ml : nullptr;
#define B200_NA(HDV, GV)                                                                                \
  paged_decode_kernel<HDV, GV><<<grid, kAttnWarps * 32, 0, stream>>>(qp, kp, vp, block_tables, seq_lens, \
                                                                    max_blocks, nkv, sl2, tokens_per_split, pa, pm, op, nsplit)
  if (head_dim == 128 && G == 4) B200_NA(128, 4);
  else if (head_dim == 128 && G == 8) B200_NA(128, 8);
  else if (head_dim == 128 && G == 2) B200_NA(128, 2);
  else if (head_dim == 128 && G == 1) B200_NA(128, 1);
  else if (head_dim == 64 && G == 2) B200_NA(64, 2);
  else if (head_dim == 64 && G == 1) B200_NA(64, 1);
  else if (head_dim == 64 && G == 4) B200_NA(64, 4);
  else return noalloc_fail(5, "unsupported head_dim %ld with group %ld", head_dim, G);
#undef B200_NA
  e = cudaGetLastError();
  if (e != cudaSuccess) return noalloc_fail(6, "attention launch failed (error %ld)", (long)e);
  if (nsplit > 1) {
    const int threads = 128;
    const int blocks = (B * nq * 32 + threads - 1) / threads;
    if (head_dim == 128)
      paged_decode_combine_kernel<128><<<blocks, threads, 0, stream>>>(pa, pm, seq_lens, op, B, nkv, G, nsplit,
                                                                       tokens_per_split);
    else
      paged_decode_combine_kernel<64><<<blocks, threads, 0, stream>>>(pa, pm, seq_lens, op, B, nkv, G, nsplit,
                                                                      tokens_per_split);
    e = cudaGetLastError();
    if (e != cudaSuccess) return noalloc_fail(6, "combine launch failed (error %ld)", (long)e);
  }
  return 0;
}

B200_BOUNDS_ACCESSOR(attention_decode)
