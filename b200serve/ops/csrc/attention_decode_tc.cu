// Paged GQA decode attention, tensor-core version (head_dim 128).
//
// Same contract as paged_decode_kernel (attention_decode.cu): grid (splits,
// kv heads, sequences), one new query per sequence, split-KV partials merged by
// paged_decode_combine_kernel. The difference is how a 16-token page is
// processed: each warp owns a 3-deep ring of shared-memory stages; one lane
// fills a stage with four TMA tensor copies (K and V, two 64-dim boxes each,
// 128-byte swizzle) completing on the stage's mbarrier, so every warp keeps up
// to 24 KB of KV in flight. Scores S^T = Q K^T use mma.sync m16n8k16 with the
// G query heads of the kv head as the M rows (rows >= G are zero), K fragments
// read with ldmatrix from the swizzled stage; P from the score accumulators is
// re-packed in registers as the A operand of O += P V, whose B fragments come
// from ldmatrix.trans. About 200 instructions per page instead of ~1000 on
// CUDA cores, which keeps the kernel at the HBM stream rate.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <mutex>
#include "tc_primitives.cuh"

namespace b200 {

constexpr int kTcWarps = 4, kTcStages = 3, kHD = 128;
constexpr int kBoxBytes = 16 * 128;              // 16 rows x 64 bf16
constexpr int kStageBytes = 4 * kBoxBytes;       // K lo, K hi, V lo, V hi

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// byte offset of (row tok, 16-byte chunk c of 16) inside a K or V page stage
__device__ __forceinline__ uint32_t swz(int tok, int c) {
  return (uint32_t)((c >> 3) * kBoxBytes + tok * 128 + (((c & 7) ^ (tok & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(kTcWarps * 32, 2) paged_decode_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    const __nv_bfloat16* __restrict__ q, const int* __restrict__ block_tables, const int* __restrict__ seq_lens,
    int max_blocks, int nkv, float scale_log2, int tps, float* __restrict__ part_acc, float* __restrict__ part_ml,
    __nv_bfloat16* __restrict__ out, int nsplit, int* err) {
  static_assert(G >= 1 && G <= 16, "query heads per kv head");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  uint8_t* ring = smem + warp * kTcStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcWarps * kTcStages * kStageBytes) + warp * kTcStages;
  float* mrg = reinterpret_cast<float*>(smem);   // merge scratch, reuses the rings after the page loop

  pdl_wait();
  pdl_trigger();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int len = seq_lens[b];
  const int nq = nkv * G;
  const int start = split * tps;
  const int stop = min(len, start + tps);
  const int* bt = block_tables + (size_t)b * max_blocks;

  if (lane == 0) {
    for (int s = 0; s < kTcStages; ++s) tc::mbar_init(&bars[s], 1);
    tc::fence_barrier_init();
  }
  __syncwarp();

  // Q as the A operand: rows = query heads (>= G zero), k = head dims
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* qb = q + ((size_t)b * nq + kvh * G) * kHD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + 2 * t4;
      qa[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * kHD + d0) : 0u;
      qa[kk][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * kHD + d0) : 0u;
      qa[kk][2] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * kHD + d0 + 8) : 0u;
      qa[kk][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * kHD + d0 + 8) : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;   // rows g and g+8

  // this warp's pages: start + (warp + i*4)*16
  const int first = start + warp * 16;
  const int n_pages = first < stop ? (stop - first + kTcWarps * 16 - 1) / (kTcWarps * 16) : 0;
  auto issue = [&](int i) {
    const int s = i % kTcStages;
    const int tok0 = first + i * kTcWarps * 16;
    const int y = (bt[tok0 >> 4] * nkv + kvh) * 16;
    uint8_t* st = ring + s * kStageBytes;
    tc::mbar_arrive_expect_tx(&bars[s], kStageBytes);
    tc::tma_load_2d(st, &tm_k, &bars[s], 0, y, 0ull);
    tc::tma_load_2d(st + kBoxBytes, &tm_k, &bars[s], 64, y, 0ull);
    tc::tma_load_2d(st + 2 * kBoxBytes, &tm_v, &bars[s], 0, y, 0ull);
    tc::tma_load_2d(st + 3 * kBoxBytes, &tm_v, &bars[s], 64, y, 0ull);
  };
  if (lane == 0)
    for (int i = 0; i < min(n_pages, kTcStages); ++i) issue(i);
  __syncwarp();

  volatile int never = 0;
  for (int i = 0; i < n_pages; ++i) {
    const int s = i % kTcStages;
    const uint32_t phase = (uint32_t)((i / kTcStages) & 1);
    if (!tc::mbar_wait_bounded(&bars[s], phase, &never, err, 11)) break;
    const uint32_t kbase = tc::smem_u32(ring + s * kStageBytes);
    const uint32_t vbase = kbase + 2 * kBoxBytes;
    const int tok0 = first + i * kTcWarps * 16;
    // ---- S^T [heads x 16 tokens] ----
    float sc[2][4];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      // matrices: (tok 0-7, chunk 2kk), (tok 0-7, chunk 2kk+1), (tok 8-15, 2kk), (tok 8-15, 2kk+1)
      const int mi = lane >> 3, r = lane & 7;
      const int tok = (mi >> 1) * 8 + r;
      uint32_t kf[4];
      ldsm_x4(kf, kbase + swz(tok, kk * 2 + (mi & 1)));
      mma16816(sc[0], qa[kk], kf[0], kf[1]);
      mma16816(sc[1], qa[kk], kf[2], kf[3]);
    }
    // ---- online softmax over the 16 tokens (log2 domain) ----
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = tok0 + nb * 8 + 2 * t4 + e < stop;
        sc[nb][e] = ok ? sc[nb][e] * scale_log2 : -INFINITY;
        sc[nb][2 + e] = ok ? sc[nb][2 + e] * scale_log2 : -INFINITY;
        mx_a = fmaxf(mx_a, sc[nb][e]);
        mx_b = fmaxf(mx_b, sc[nb][2 + e]);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float base_a = mn_a == -INFINITY ? 0.f : mn_a, base_b = mn_b == -INFINITY ? 0.f : mn_b;
    const float al_a = exp2f(m_a - base_a), al_b = exp2f(m_b - base_b);
    m_a = mn_a;
    m_b = mn_b;
    float ps_a = 0.f, ps_b = 0.f;
    uint32_t pa[4];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      const float p0 = exp2f(sc[nb][0] - base_a), p1 = exp2f(sc[nb][1] - base_a);
      const float p2 = exp2f(sc[nb][2] - base_b), p3 = exp2f(sc[nb][3] - base_b);
      ps_a += p0 + p1;
      ps_b += p2 + p3;
      pa[nb * 2 + 0] = pack_bf16x2(p0, p1);
      pa[nb * 2 + 1] = pack_bf16x2(p2, p3);
    }
    ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 1);
    ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 2);
    ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 1);
    ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 2);
    l_a = l_a * al_a + ps_a;
    l_b = l_b * al_b + ps_b;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= al_a; o[j][1] *= al_a; o[j][2] *= al_b; o[j][3] *= al_b;
    }
    // ---- O [heads x 128] += P [heads x 16] . V [16 x 128] ----
#pragma unroll
    for (int j2 = 0; j2 < 8; ++j2) {
      // matrices: (tok 0-7, chunk 2j2), (tok 8-15, 2j2), (tok 0-7, 2j2+1), (tok 8-15, 2j2+1)
      const int mi = lane >> 3, r = lane & 7;
      const int tok = (mi & 1) * 8 + r;
      uint32_t vf[4];
      ldsm_x4_t(vf, vbase + swz(tok, j2 * 2 + (mi >> 1)));
      mma16816(o[j2 * 2], pa, vf[0], vf[1]);
      mma16816(o[j2 * 2 + 1], pa, vf[2], vf[3]);
    }
    __syncwarp();
    if (lane == 0 && i + kTcStages < n_pages) {
      tc::fence_proxy_async_smem();   // generic reads of this stage happen before the TMA overwrite
      issue(i + kTcStages);
    }
    __syncwarp();
  }

  // ---- merge the warps: per warp m, l [G] and O [G][128] in shared memory ----
  __syncthreads();
  float* wm = mrg;                         // [warps][16]
  float* wl = mrg + kTcWarps * 16;         // [warps][16]
  float* wo = mrg + kTcWarps * 32;         // [warps][G][128]
  if (t4 == 0) {
    if (g < G) { wm[warp * 16 + g] = m_a; wl[warp * 16 + g] = l_a; }
    if (g + 8 < G) { wm[warp * 16 + g + 8] = m_b; wl[warp * 16 + g + 8] = l_b; }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = j * 8 + 2 * t4;
    if (g < G) { wo[(warp * G + g) * kHD + d] = o[j][0]; wo[(warp * G + g) * kHD + d + 1] = o[j][1]; }
    if (g + 8 < G) {
      wo[(warp * G + g + 8) * kHD + d] = o[j][2];
      wo[(warp * G + g + 8) * kHD + d + 1] = o[j][3];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * kHD; idx += blockDim.x) {
    const int hh = idx / kHD, d = idx % kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, wm[w * 16 + hh]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kTcWarps; ++w) {
        const float f = exp2f(wm[w * 16 + hh] - M);
        L += wl[w * 16 + hh] * f;
        A += wo[(w * G + hh) * kHD + d] * f;
      }
    }
    if (nsplit == 1) {
      out[((size_t)b * nq + kvh * G + hh) * kHD + d] = __float2bfloat16_rn(L > 0.f ? A / L : 0.f);
    } else {
      const size_t slot = (((size_t)b * nkv + kvh) * nsplit + split) * G + hh;
      part_acc[slot * kHD + d] = A;
      if (d == 0) { part_ml[slot * 2] = M; part_ml[slot * 2 + 1] = L; }
    }
  }
}

size_t decode_tc_smem(int) { return 1024 + kTcWarps * kTcStages * kStageBytes + 256; }

typedef CUresult (*EncodeTiledFnKV)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// KV cache viewed as [rows = blocks * kv_heads * 16, 128] bf16; box 64 dims x 16 rows, 128-byte swizzle.
static CUtensorMap make_tmap_kv(const void* base, int64_t rows) {
  static EncodeTiledFnKV fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qr;
    B200_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr));
    TORCH_CHECK(qr == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFnKV>(ptr);
  });
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)kHD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kHD * 2};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (KV) failed: ", (int)r);
  return m;
}

static int* g_tc_err = nullptr;
static int* decode_tc_err_word() {
  if (!g_tc_err) {
    B200_CHECK_CUDA(cudaMalloc(&g_tc_err, sizeof(int)));
    B200_CHECK_CUDA(cudaMemset(g_tc_err, 0, sizeof(int)));
  }
  return g_tc_err;
}

}  // namespace b200

using namespace b200;

// defined in attention_decode.cu
void paged_decode_combine(torch::Tensor part_acc, torch::Tensor part_ml, torch::Tensor seq_lens, torch::Tensor out,
                          int64_t nkv, int64_t G, int64_t nsplit, int64_t tps);

void paged_decode_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                               torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor out,
                               torch::Tensor part_acc, torch::Tensor part_ml, double scale, int64_t tps,
                               int64_t nsplit) {
  const int B = q.size(0), nq = q.size(1), HD = q.size(2);
  const int nkv = k_cache.size(1);
  const int G = nq / nkv;
  TORCH_CHECK(HD == kHD && k_cache.size(2) == 16 && tps % 16 == 0 && nsplit >= 1);
  if (nsplit > 1) {
    TORCH_CHECK(part_acc.numel() >= (int64_t)B * nkv * nsplit * G * HD, "attention workspace too small");
    TORCH_CHECK(part_ml.numel() >= (int64_t)B * nkv * nsplit * G * 2, "attention workspace too small");
  }
  if (B == 0) return;
  const int64_t rows = k_cache.size(0) * (int64_t)nkv * 16;
  CUtensorMap tk = make_tmap_kv(k_cache.data_ptr(), rows);
  CUtensorMap tv = make_tmap_kv(v_cache.data_ptr(), rows);
  auto stream = at::cuda::getCurrentCUDAStream();
  const float sl2 = (float)(scale * 1.4426950408889634);
  dim3 grid(nsplit, nkv, B);
  float* pa = nsplit > 1 ? part_acc.data_ptr<float>() : nullptr;
  float* pm = nsplit > 1 ? part_ml.data_ptr<float>() : nullptr;
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const size_t smem = decode_tc_smem(G);
#define B200_TC(GV)                                                                                            \
  {                                                                                                            \
    static bool attr = false;                                                                                  \
    if (!attr) {                                                                                               \
      B200_CHECK_CUDA(cudaFuncSetAttribute(paged_decode_tc_kernel<GV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                           (int)smem));                                                       \
      attr = true;                                                                                             \
    }                                                                                                          \
    launch_pdl(paged_decode_tc_kernel<GV>, grid, dim3(kTcWarps * 32), smem, stream, tk, tv,                    \
               reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (const int*)block_tables.data_ptr<int>(),  \
               (const int*)seq_lens.data_ptr<int>(), (int)block_tables.size(1), nkv, sl2, (int)tps, pa, pm, op, \
               (int)nsplit, decode_tc_err_word());                                                             \
  }
  switch (G) {
    case 1: B200_TC(1) break;
    case 2: B200_TC(2) break;
    case 4: B200_TC(4) break;
    case 8: B200_TC(8) break;
    case 16: B200_TC(16) break;
    default: TORCH_CHECK(false, "unsupported GQA group ", G);
  }
#undef B200_TC
  if (nsplit > 1) paged_decode_combine(part_acc, part_ml, seq_lens, out, nkv, G, nsplit, tps);
}
