// Causal paged prefill attention (chunked prefill against the paged KV cache).
//
// Restates reference attention.wgsl:63 (causal GQA attention) and the
// online-softmax tiling of attention_stream.wgsl:160 for many query rows.
// This version runs the two products on mma.sync m16n8k16 (bf16 in, fp32
// accumulate); K/V tiles of 64 tokens (4 pages) are staged in shared memory
// with cp.async, double-buffered.
//
// Grid (q tiles of 64 rows, nq heads, sequences); 4 warps, 16 query rows each.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

constexpr int PF_BQ = 64, PF_BK = 64;

__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// KVQ = 1: int4g128 cache (codes [blocks][nkv][16][HD/2], fp16 scale per row); tiles are
// fetched as codes + scales and dequantised into the bf16 tiles before use.
template <int HD, int KVQ>
__global__ void __launch_bounds__(128) paged_prefill_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
    const __nv_bfloat16* __restrict__ v_cache, const int* __restrict__ block_tables, int max_blocks,
    const int* __restrict__ seq_lens, const int* __restrict__ q_start, const int* __restrict__ cu_q,
    __nv_bfloat16* __restrict__ out, int nq, int nkv, float scale_log2, const uint8_t* __restrict__ kq,
    const uint8_t* __restrict__ vq, const __half* __restrict__ ksc, const __half* __restrict__ vsc, int window,
    float softcap, int nblocks) {
  constexpr int LD = HD + 8;  // padded smem row (bf16) -> conflict-free 32-bit fragment loads
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem_raw);          // [2][64][LD]
  __nv_bfloat16* vs = ks + 2 * PF_BK * LD;                                  // [2][64][LD]
  uint8_t* qraw = reinterpret_cast<uint8_t*>(vs + 2 * PF_BK * LD);           // KVQ: [2][K|V][64][HD/2]
  __half* qscl = reinterpret_cast<__half*>(qraw + 2 * 2 * PF_BK * (HD / 2));  // KVQ: [2][K|V][64]

  pdl_wait();
  pdl_trigger();
  const int seq = blockIdx.z, h = blockIdx.y, qt = blockIdx.x;
  const int row0 = cu_q[seq], nrows = cu_q[seq + 1] - row0;
  if (qt * PF_BQ >= nrows) return;
  const int kvh = h / (nq / nkv);
  const int L = seq_lens[seq];
  const int pos0 = q_start[seq];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;

  // query rows of this warp: r_a = base + g, r_b = base + g + 8 (relative to the sequence)
  const int rbase = qt * PF_BQ + warp * 16;
  const int ra = rbase + g, rb = rbase + g + 8;
  const int qpos_a = pos0 + ra, qpos_b = pos0 + rb;
  uint32_t qf[HD / 16][4];
  {
    const __nv_bfloat16* qa = q + ((size_t)(row0 + min(ra, nrows - 1)) * nq + h) * HD;
    const __nv_bfloat16* qb = q + ((size_t)(row0 + min(rb, nrows - 1)) * nq + h) * HD;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      qf[kk][0] = *reinterpret_cast<const uint32_t*>(qa + kk * 16 + 2 * t4);
      qf[kk][1] = *reinterpret_cast<const uint32_t*>(qb + kk * 16 + 2 * t4);
      qf[kk][2] = *reinterpret_cast<const uint32_t*>(qa + kk * 16 + 8 + 2 * t4);
      qf[kk][3] = *reinterpret_cast<const uint32_t*>(qb + kk * 16 + 8 + 2 * t4);
    }
  }
  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

  // KV tokens needed by this CTA: [0, min(L, last query position + 1))
  const int last_pos = pos0 + min(nrows, (qt + 1) * PF_BQ) - 1;
  const int kv_end = min(L, last_pos + 1);
  const int n_tiles = (kv_end + PF_BK - 1) / PF_BK;
  // sliding window: a query at p sees keys (p - window, p]; tiles before the CTA's first
  // query row's window are skipped
  const int first_tile = window > 0 ? max(0, pos0 + qt * PF_BQ - window + 1) / PF_BK : 0;
  const int* bt = block_tables + (size_t)seq * max_blocks;

  auto load_tile = [&](int tile, int buf) {
    if constexpr (KVQ) {
      // codes: 64 rows x HD/2 bytes for K and V, plus one fp16 scale per row
      constexpr int CH = PF_BK * (HD / 2) / 16;
      for (int c = threadIdx.x; c < CH; c += 128) {
        const int tok = c / (HD / 32), part = c % (HD / 32);
        const int abs_tok = tile * PF_BK + tok;
        const int pg = abs_tok < kv_end ? table_block(bt, abs_tok >> 4, max_blocks, nblocks, 0x301) : -1;
        const bool ok = pg >= 0;
        const int page = ok ? pg : 0;
        const size_t row = ((size_t)page * nkv + kvh) * 16 + (abs_tok & 15);
        uint8_t* dk = qraw + ((buf * 2 + 0) * PF_BK + tok) * (HD / 2) + part * 16;
        uint8_t* dv = qraw + ((buf * 2 + 1) * PF_BK + tok) * (HD / 2) + part * 16;
        cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(dk)), kq + row * (HD / 2) + part * 16, ok);
        cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(dv)), vq + row * (HD / 2) + part * 16, ok);
        if (part == 0) {
          qscl[(buf * 2 + 0) * PF_BK + tok] = ok ? ksc[row] : __float2half(0.f);
          qscl[(buf * 2 + 1) * PF_BK + tok] = ok ? vsc[row] : __float2half(0.f);
        }
      }
      cp_async_commit();
      return;
    }
    // 64 tokens x HD dims for K and V: 64*HD/8 16-byte chunks each
    constexpr int CH = PF_BK * HD / 8;
    for (int c = threadIdx.x; c < CH; c += 128) {
      const int tok = c / (HD / 8), part = c % (HD / 8);
      const int abs_tok = tile * PF_BK + tok;
      const int pg = abs_tok < kv_end ? table_block(bt, abs_tok >> 4, max_blocks, nblocks, 0x301) : -1;
      const bool ok = pg >= 0;
      const int page = ok ? pg : 0;
      const size_t off = (((size_t)page * nkv + kvh) * 16 + (abs_tok & 15)) * HD + part * 8;
      const uint32_t dk = static_cast<uint32_t>(__cvta_generic_to_shared(ks + (buf * PF_BK + tok) * LD + part * 8));
      const uint32_t dv = static_cast<uint32_t>(__cvta_generic_to_shared(vs + (buf * PF_BK + tok) * LD + part * 8));
      cp_async16(dk, k_cache + off, ok);
      cp_async16(dv, v_cache + off, ok);
    }
    cp_async_commit();
  };

  if (n_tiles > first_tile) load_tile(first_tile, 0);
  for (int tile = first_tile; tile < n_tiles; ++tile) {
    const int buf = (tile - first_tile) & 1;
    if (tile + 1 < n_tiles) {
      load_tile(tile + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if constexpr (KVQ) {
      // dequantise this buffer's codes into the bf16 tiles (8 dims = one 32-bit word per step)
      for (int i = threadIdx.x; i < 2 * PF_BK * (HD / 8); i += 128) {
        const int kv = i / (PF_BK * (HD / 8)), rem = i % (PF_BK * (HD / 8));
        const int tok = rem / (HD / 8), grp = rem % (HD / 8);
        const uint32_t w = *reinterpret_cast<const uint32_t*>(qraw + ((buf * 2 + kv) * PF_BK + tok) * (HD / 2) + grp * 4);
        const float sc = __half2float(qscl[(buf * 2 + kv) * PF_BK + tok]);
        float f[8];
#pragma unroll
        for (int p2 = 0; p2 < 4; ++p2) {
          f[2 * p2] = (float)((int)((w >> (4 * p2)) & 15u) - 8) * sc;
          f[2 * p2 + 1] = (float)((int)((w >> (16 + 4 * p2)) & 15u) - 8) * sc;
        }
        __nv_bfloat16* dst = (kv ? vs : ks) + (buf * PF_BK + tok) * LD + grp * 8;
        *reinterpret_cast<bf16x8*>(dst) = pack8(f);
      }
      __syncthreads();
    }
    const __nv_bfloat16* kb = ks + buf * PF_BK * LD;
    const __nv_bfloat16* vb = vs + buf * PF_BK * LD;
    // ---- S = Q K^T : 16 rows x 64 tokens per warp ----
    float s[PF_BK / 8][4];
#pragma unroll
    for (int j = 0; j < PF_BK / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int j = 0; j < PF_BK / 8; ++j) {
        uint32_t bfr[2];
        const __nv_bfloat16* krow = kb + (j * 8 + g) * LD + kk * 16 + 2 * t4;
        bfr[0] = *reinterpret_cast<const uint32_t*>(krow);
        bfr[1] = *reinterpret_cast<const uint32_t*>(krow + 8);
        mma_16816(s[j], qf[kk], bfr);
      }
    }
    // ---- mask + online softmax (log2 domain) ----
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < PF_BK / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kpos = tile * PF_BK + j * 8 + 2 * t4 + e;
        const bool valid_k = kpos < kv_end;
        const bool in_a = kpos <= qpos_a && (window == 0 || kpos > qpos_a - window);
        const bool in_b = kpos <= qpos_b && (window == 0 || kpos > qpos_b - window);
        float xa = s[j][e] * scale_log2, xb = s[j][2 + e] * scale_log2;
        if (softcap > 0.f) {   // c tanh(x / c) on the natural-scale score, back to log2 units
          xa = softcap * tanhf(xa * 0.69314718055994531f / softcap) * 1.4426950408889634f;
          xb = softcap * tanhf(xb * 0.69314718055994531f / softcap) * 1.4426950408889634f;
        }
        s[j][e] = (valid_k && in_a) ? xa : -INFINITY;
        s[j][2 + e] = (valid_k && in_b) ? xb : -INFINITY;
        mx_a = fmaxf(mx_a, s[j][e]);
        mx_b = fmaxf(mx_b, s[j][2 + e]);
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
    float sum_a = 0.f, sum_b = 0.f;
    uint32_t pf[PF_BK / 16][4];
#pragma unroll
    for (int j = 0; j < PF_BK / 8; ++j) {
      const float p0 = exp2f(s[j][0] - base_a), p1 = exp2f(s[j][1] - base_a);
      const float p2 = exp2f(s[j][2] - base_b), p3 = exp2f(s[j][3] - base_b);
      sum_a += p0 + p1;
      sum_b += p2 + p3;
      const int kk = j >> 1, hi = j & 1;
      pf[kk][hi * 2 + 0] = pack_bf16x2(p0, p1);
      pf[kk][hi * 2 + 1] = pack_bf16x2(p2, p3);
    }
    sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 1);
    sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 2);
    sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 1);
    sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 2);
    l_a = l_a * al_a + sum_a;
    l_b = l_b * al_b + sum_b;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      o[j][0] *= al_a; o[j][1] *= al_a; o[j][2] *= al_b; o[j][3] *= al_b;
    }
    // ---- O += P V ----
#pragma unroll
    for (int kk = 0; kk < PF_BK / 16; ++kk) {
      // a-fragment order: (row g, k lo), (row g+8, k lo), (row g, k hi), (row g+8, k hi)
      uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int j2 = 0; j2 < HD / 16; ++j2) {
        uint32_t r[4];
        const int m = lane >> 3, rr = lane & 7;
        const int tok = kk * 16 + (m & 1) * 8 + rr;
        const int dim = j2 * 16 + (m >> 1) * 8;
        ldmatrix_x4_trans(r, static_cast<uint32_t>(__cvta_generic_to_shared(vb + tok * LD + dim)));
        uint32_t b0[2] = {r[0], r[1]}, b1[2] = {r[2], r[3]};
        mma_16816(o[j2 * 2], a, b0);
        mma_16816(o[j2 * 2 + 1], a, b1);
      }
    }
    __syncthreads();
  }
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  if (ra < nrows) {
    __nv_bfloat16* oa = out + ((size_t)(row0 + ra) * nq + h) * HD;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j)
      *reinterpret_cast<uint32_t*>(oa + j * 8 + 2 * t4) = pack_bf16x2(o[j][0] * inv_a, o[j][1] * inv_a);
  }
  if (rb < nrows) {
    __nv_bfloat16* ob = out + ((size_t)(row0 + rb) * nq + h) * HD;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j)
      *reinterpret_cast<uint32_t*>(ob + j * 8 + 2 * t4) = pack_bf16x2(o[j][2] * inv_b, o[j][3] * inv_b);
  }
}

// int4g128 pages -> bf16 pages (for the tensor-core prefill attention): pages block_ids[j] of
// codes [blocks][nkv][16][64] + fp16 scale [blocks][nkv][16] -> out [j][nkv][16][128]. Dims
// (2p, 2p+1) of each 8-dim group sit in nibbles (p, p + 4) of the group's 32-bit word.
__global__ void q4_dequant_pages_kernel(const int* __restrict__ block_ids, int n, int nkv,
                                        const uint32_t* __restrict__ codes, const __half* __restrict__ scales,
                                        __nv_bfloat16* __restrict__ out, int nblocks) {
  pdl_wait();
  pdl_trigger();
  const int64_t words = (int64_t)n * nkv * 16 * 16;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i >> 4;                      // (j, h, token) row of the output
    const int g = (int)(i & 15);
    const int j = (int)(row / (nkv * 16));
    int blk = block_ids[j];
    if (!B200_IN_RANGE(blk, nblocks, 0x303)) blk = 0;       // checked builds: read block 0 instead
    const int64_t src_row = (int64_t)blk * nkv * 16 + row % (nkv * 16);
    const uint32_t w = codes[src_row * 16 + g];
    const float sc = __half2float(scales[src_row]);
    uint32_t o[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float lo = (float)((int)((w >> (4 * p)) & 15u) - 8) * sc;
      const float hi = (float)((int)((w >> (4 * (p + 4))) & 15u) - 8) * sc;
      o[p] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4*>(out + row * 128 + g * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace b200

using namespace b200;

static void prefill_impl(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                         torch::Tensor seq_lens, torch::Tensor q_start, torch::Tensor cu_q, torch::Tensor out,
                         double scale, int64_t max_q, int kvq, const uint8_t* kq, const uint8_t* vq,
                         const __half* ksc, const __half* vsc, int window = 0, float softcap = 0.f) {
  const int T = q.size(0), nq = q.size(1), HD = q.size(2);
  const int nkv = k_cache.size(1);
  const int nseq = seq_lens.size(0);
  TORCH_CHECK(nq % nkv == 0);
  if (T == 0 || nseq == 0) return;
  dim3 grid((max_q + PF_BQ - 1) / PF_BQ, nq, nseq);
  auto stream = at::cuda::getCurrentCUDAStream();
  const float sl2 = (float)(scale * 1.4426950408889634);
#define B200_PF1(HDV, KQV)                                                                                      \
  {                                                                                                             \
    const size_t smem = 4 * PF_BK * (HDV + 8) * 2 + (KQV ? (2 * 2 * PF_BK * (HDV / 2) + 2 * 2 * PF_BK * 2) : 0); \
    static bool attr = false;                                                                                   \
    if (!attr) {                                                                                                \
      B200_CHECK_CUDA(cudaFuncSetAttribute(paged_prefill_kernel<HDV, KQV>,                                      \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));            \
      attr = true;                                                                                              \
    }                                                                                                           \
    launch_pdl(paged_prefill_kernel<HDV, KQV>, grid, dim3(128), smem, stream,                                   \
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()), \
        reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()), (const int*)block_tables.data_ptr<int>(),   \
        (int)block_tables.size(1), (const int*)seq_lens.data_ptr<int>(), (const int*)q_start.data_ptr<int>(),    \
        (const int*)cu_q.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nq, nkv, sl2,       \
        kq, vq, ksc, vsc, window, softcap, (int)k_cache.size(0));                                               \
  }
  if (kvq) {
    TORCH_CHECK(HD == 128, "int4 KV cache needs head_dim 128");
    B200_PF1(128, 1)
  } else if (HD == 128) B200_PF1(128, 0)
  else if (HD == 64) B200_PF1(64, 0)
  else if (HD == 256) B200_PF1(256, 0)
  else TORCH_CHECK(false, "head_dim must be 64, 128 or 256");
#undef B200_PF1
  B200_CHECK_CUDA(cudaGetLastError());
}

void paged_prefill_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                             torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start,
                             torch::Tensor cu_q, torch::Tensor out, double scale, int64_t max_q, int64_t window,
                             double softcap) {
  prefill_impl(q, k_cache, v_cache, block_tables, seq_lens, q_start, cu_q, out, scale, max_q, 0, nullptr, nullptr,
               nullptr, nullptr, (int)window, (float)softcap);
}

// int4g128 cache: k_codes/v_codes [blocks][nkv][16][64] uint8, k_scale/v_scale [blocks][nkv][16] fp16.
void paged_prefill_attention_q4(torch::Tensor q, torch::Tensor k_codes, torch::Tensor v_codes, torch::Tensor k_scale,
                                torch::Tensor v_scale, torch::Tensor block_tables, torch::Tensor seq_lens,
                                torch::Tensor q_start, torch::Tensor cu_q, torch::Tensor out, double scale,
                                int64_t max_q) {
  prefill_impl(q, k_codes, v_codes, block_tables, seq_lens, q_start, cu_q, out, scale, max_q, 1,
               k_codes.data_ptr<uint8_t>(), v_codes.data_ptr<uint8_t>(),
               reinterpret_cast<const __half*>(k_scale.data_ptr()), reinterpret_cast<const __half*>(v_scale.data_ptr()));
}

void q4_dequant_pages(torch::Tensor block_ids, torch::Tensor codes, torch::Tensor scales, torch::Tensor out) {
  const int n = block_ids.numel(), nkv = codes.size(1);
  TORCH_CHECK(codes.size(2) == 16 && codes.size(3) == 64 && out.size(0) >= n && out.size(3) == 128);
  if (n == 0) return;
  const int64_t words = (int64_t)n * nkv * 16 * 16;
  const int blocks = (int)std::min<int64_t>((words + 255) / 256, 148 * 8);
  launch_pdl(q4_dequant_pages_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             (const int*)block_ids.data_ptr<int>(), n, nkv, reinterpret_cast<const uint32_t*>(codes.data_ptr()),
             reinterpret_cast<const __half*>(scales.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
             (int)codes.size(0));
}

B200_BOUNDS_ACCESSOR(attention_prefill)
