// Causal paged prefill attention on the 5th-generation tensor cores (head_dim 128, bf16 KV).
//
// Same contract as paged_prefill_kernel (attention_prefill.cu): sequence i owns query rows
// cu_q[i]:cu_q[i+1] at absolute positions q_start[i] + j, its keys are the first seq_lens[i]
// rows of the paged cache [blocks][nkv][16][128]. Restates the causal GQA attention of the
// reference (attention.wgsl:63) with online softmax (attention_stream.wgsl:160).
//
// One CTA = one kv head x 128 MMA rows, the rows being 128/G query tokens x the G query heads
// of that kv head, so every K/V tile is read once for all G heads. Per 128-key tile:
//   S = Q K^T      tcgen05.mma, A = Q (smem, K-major), B = K (smem, K-major), S in TMEM;
//   softmax        4 warps, one TMEM lane (row) per thread, online max/sum in registers;
//                  P (bf16) is written to smem in the 128-byte-swizzled K-major layout;
//   O += P V       tcgen05.mma, A = P, B = V read MN-major straight from the TMA-loaded
//                  [key][dim] tile, O in TMEM.
// O is rescaled in TMEM only when a row maximum grows by more than 8 (log2 units); until then
// the stale maximum keeps exp2() <= 256, which fp32/bf16 absorb.
// Roles (320 threads): warp 0 lane 0 = TMA producer (K/V pages, 2 stages), warp 1 = TMEM
// allocator + MMA issuer, warps 2..9 = softmax and the output epilogue (two warps per TMEM lane
// quadrant, each taking half of the key and output columns). Every wait is bounded.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <mutex>
#include "tc_primitives.cuh"

namespace b200 {

constexpr int kPT_Rows = 128, kPT_Keys = 128, kPT_HD = 128;
constexpr int kPT_Half = kPT_Rows * 128;            // 128 rows x 64 bf16 = 16 KB
constexpr int kPT_Tile = 2 * kPT_Half;              // 128 x 128 bf16 = 32 KB
// smem: Q | K[2] | V[2] | P | barriers
constexpr int kPT_Q = 0, kPT_K = kPT_Tile, kPT_V = 3 * kPT_Tile, kPT_P = 5 * kPT_Tile, kPT_Bar = 6 * kPT_Tile;
constexpr size_t kPT_Smem = 1024 + 6 * kPT_Tile + 256 + 2048 + 64;   // + row max/sum exchange, flags

// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32, one MUFU instruction)
__device__ __forceinline__ float pt_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// byte offset of (row r, 16-byte chunk c of 16) in a 128-row SW128 K-major tile of two 64-col halves
__device__ __forceinline__ uint32_t pt_swz(int r, int c) {
  return (uint32_t)((c >> 3) * kPT_Half + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(320, 1) paged_prefill_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    const __nv_bfloat16* __restrict__ q, const int* __restrict__ block_tables, int max_blocks,
    const int* __restrict__ seq_lens, const int* __restrict__ q_start, const int* __restrict__ cu_q,
    __nv_bfloat16* __restrict__ out, int nq, int nkv, float scale_log2, int* err, int nblocks) {
  constexpr int QT = kPT_Rows / G;                  // query tokens per CTA
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPT_Bar);
  uint64_t* kfull = bars;          // [2]
  uint64_t* vfull = bars + 2;      // [2]
  uint64_t* kempty = bars + 4;     // [2]
  uint64_t* vempty = bars + 6;     // [2]
  uint64_t* s_full = bars + 8;     // [2]: S buffer b holds a finished Q K^T
  uint64_t* s_free = bars + 10;    // [2]: the softmax warps finished reading S buffer b
  uint64_t* p_full = bars + 12;
  uint64_t* pv_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = blockIdx.z, kvh = blockIdx.y;
  pdl_wait();
  pdl_trigger();
  const int row0 = cu_q[seq], nrows = cu_q[seq + 1] - row0;
  const int tq0 = blockIdx.x * QT;
  if (tq0 >= nrows) return;
  const int qs = q_start[seq], len = seq_lens[seq];
  const int tq_end = min(nrows, tq0 + QT);
  const int last_pos = qs + tq_end - 1;                             // highest query position here
  const int n_tiles = (min(len, last_pos + 1) + kPT_Keys - 1) / kPT_Keys;
  const int* bt = block_tables + (size_t)seq * max_blocks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 14; ++i) tc::mbar_init(&bars[i], (i == 10 || i == 11 || i == 12) ? 8 : 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tm_k);
    tc::prefetch_tmap(&tm_v);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  // ---- Q rows (token-major, G heads per token) -> swizzled K-major smem tile ----
  for (int i = threadIdx.x; i < kPT_Rows * 16; i += blockDim.x) {
    const int r = i >> 4, c = i & 15;
    const int t = tq0 + r / G;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t < nrows)
      v = *reinterpret_cast<const uint4*>(q + ((size_t)(row0 + t) * nq + kvh * G + r % G) * kPT_HD + c * 8);
    *reinterpret_cast<uint4*>(smem + kPT_Q + pt_swz(r, c)) = v;
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;                            // S buffers at columns 0 and 128

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: K and V pages of each 128-key tile ----------------
      for (int j = 0; j < n_tiles && !*abort_flag; ++j) {
        const int s = j & 1;
        const uint32_t ph = (uint32_t)((j >> 1) & 1);
        if (!tc::mbar_wait_bounded(&kempty[s], ph ^ 1, abort_flag, err, 31)) break;
        tc::mbar_arrive_expect_tx(&kfull[s], kPT_Tile);
        for (int pg = 0; pg < 8; ++pg) {
          const int blk = j * 8 + pg;
          const int b0 = blk < max_blocks ? bt[blk] : 0;   // -1 (no block) past the sequence reads block 0
          const int b = b0 < 0 || !B200_IN_RANGE(b0, nblocks, 0x311) ? 0 : b0;
          const int y = (b * nkv + kvh) * 16;
          uint8_t* dst = smem + kPT_K + s * kPT_Tile + pg * 2048;
          tc::tma_load_2d(dst, &tm_k, &kfull[s], 0, y, 0ull);
          tc::tma_load_2d(dst + kPT_Half, &tm_k, &kfull[s], 64, y, 0ull);
        }
        if (!tc::mbar_wait_bounded(&vempty[s], ph ^ 1, abort_flag, err, 32)) break;
        tc::mbar_arrive_expect_tx(&vfull[s], kPT_Tile);
        for (int pg = 0; pg < 8; ++pg) {
          const int blk = j * 8 + pg;
          const int b0 = blk < max_blocks ? bt[blk] : 0;   // -1 (no block) past the sequence reads block 0
          const int b = b0 < 0 || !B200_IN_RANGE(b0, nblocks, 0x311) ? 0 : b0;
          const int y = (b * nkv + kvh) * 16;
          uint8_t* dst = smem + kPT_V + s * kPT_Tile + pg * 2048;
          tc::tma_load_2d(dst, &tm_v, &vfull[s], 0, y, 0ull);
          tc::tma_load_2d(dst + kPT_Half, &tm_v, &vfull[s], 64, y, 0ull);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t IDESC_S = tc::idesc_bf16_f32(128, 128);
      constexpr uint32_t IDESC_PV = tc::idesc_bf16_f32_bmn(128, 128);
      const uint32_t q_addr = tc::smem_u32(smem + kPT_Q), p_addr = tc::smem_u32(smem + kPT_P);
      // S(j+1) is issued before PV(j), into the other S buffer, so the tensor core computes the
      // next scores while the softmax warps work on this tile
      auto issue_s = [&](int t) -> bool {
        const int b = t & 1;
        if (!tc::mbar_wait_bounded(&kfull[b], (uint32_t)((t >> 1) & 1), abort_flag, err, 33)) return false;
        if (t >= 2 && !tc::mbar_wait_bounded(&s_free[b], (uint32_t)(((t - 2) >> 1) & 1), abort_flag, err, 34))
          return false;
        tc::tc_fence_after();
        const uint32_t k_addr = tc::smem_u32(smem + kPT_K + b * kPT_Tile);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kPT_Half;
          const uint64_t a = tc::sw128_kmajor_desc(q_addr + off) + 2 * (kk & 3);
          const uint64_t bd = tc::sw128_kmajor_desc(k_addr + off) + 2 * (kk & 3);
          tc::mma_bf16(tmem + b * 128, a, bd, IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(&s_full[b]);
        tc::mma_commit(&kempty[b]);
        return true;
      };
      bool live = n_tiles > 0 && issue_s(0);
      for (int j = 0; j < n_tiles && live && !*abort_flag; ++j) {
        const int s = j & 1;
        const uint32_t ph = (uint32_t)((j >> 1) & 1);
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        // O += P V once the softmax warps have written P of this tile
        if (!tc::mbar_wait_bounded(p_full, (uint32_t)(j & 1), abort_flag, err, 35)) break;
        if (!tc::mbar_wait_bounded(&vfull[s], ph, abort_flag, err, 36)) break;
        tc::tc_fence_after();
        const uint32_t v_addr = tc::smem_u32(smem + kPT_V + s * kPT_Tile);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = tc::sw128_kmajor_desc(p_addr + (kk >> 2) * kPT_Half) + 2 * (kk & 3);
          // 16 keys = two 8-row groups (1024 B apart); the 128 dims span the two 64-dim halves
          const uint64_t bd = tc::sw128_mnmajor_desc(v_addr + kk * 2048, kPT_Half, 1024);
          tc::mma_bf16(tO, a, bd, IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc::mma_commit(pv_done);
        tc::mma_commit(&vempty[s]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue: 8 warps, thread = (row, half of the columns) ----------
    // Warps 2..5 and 6..9 cover the four TMEM lane quadrants twice; the first set handles key
    // (and output) columns 0..63 of its rows, the second 64..127. Row maxima and sums are
    // combined through shared memory under named barrier 2 (the 256 softmax threads).
    const int quad = warp & 3, half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int cbase = half * 64;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    float* xmax = reinterpret_cast<float*>(smem + kPT_Bar + 256);   // [2][128]
    float* xsum = xmax + 256;                                        // [2][128]
    const int t = tq0 + r / G;
    const int pos = t < nrows ? qs + t : -1;                  // -1: padding row, attends nothing
    float m = -INFINITY, l = 0.f;
    // lane 0 waits, the warp follows: keeps every later warp-collective TMEM access uniform
    auto warp_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      int ok = 1;
      if (lane == 0) ok = tc::mbar_wait_bounded(bar, parity, abort_flag, err, code) ? 1 : 0;
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    // Named barriers: 1 = all 8 softmax warps (once per tile, `agree`); 2 + quad = the two warps
    // of one lane quadrant (the row max / sum exchange, whose pass count can differ between
    // quadrants but never between the two halves of the same rows).
    const int pair_bar = 2 + quad;
    auto pair_sync = [pair_bar] { asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory"); };
    int* xok = reinterpret_cast<int*>(xsum + 256);                   // [8]
    // every softmax warp calls agree() the same number of times: a timed-out wait in any of
    // them makes all eight leave together
    auto agree = [&](bool v) -> bool {
      if (lane == 0) xok[warp - 2] = v ? 1 : 0;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      int all = 1;
#pragma unroll
      for (int i = 0; i < 8; ++i) all &= xok[i];
      asm volatile("bar.sync 1, 256;" ::: "memory");
      return all != 0;
    };
    int j = 0;
    bool ok = true;
    for (; j < n_tiles; ++j) {
      ok = warp_wait(&s_full[j & 1], (uint32_t)((j >> 1) & 1), 37);
      if (ok && j > 0) ok = warp_wait(pv_done, (uint32_t)((j - 1) & 1), 38);
      ok = agree(ok);
      if (!ok) break;
      tc::tc_fence_after();
      const int key0 = j * kPT_Keys;
      const uint32_t tSj = tmem + (uint32_t)(j & 1) * 128;    // this tile's S buffer
      const int lim = min(len - 1, pos);                       // last key this row may see
      // one pass over S in the common case: p = exp2(s - m) with the running (possibly stale)
      // maximum m; the pass is repeated only when a row sees its first visible key here or its
      // maximum grows by more than 8, after O is rescaled
      float rs = 0.f;
      int lim_min = lim;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lim_min = min(lim_min, __shfl_xor_sync(0xffffffffu, lim_min, o));
      const bool full_tile = key0 + cbase + 63 <= lim_min;      // warp-uniform: no per-key mask
      for (int pass = 0; pass < 2; ++pass) {
        rs = 0.f;
        float mxr = -INFINITY;                                 // max of the raw (unscaled) scores
        const float mref = m == -INFINITY ? 0.f : m;
        uint32_t raw[64];
#pragma unroll
        for (int u = 0; u < 4; ++u) tc::tmem_ld16_async(tSj + lane_off + cbase + 16 * u, raw + 16 * u);
        tc::tmem_wait_ld();
        uint32_t pk[32];
        if (full_tile) {
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const float s0 = __uint_as_float(raw[i]), s1 = __uint_as_float(raw[i + 1]);
            mxr = fmaxf(mxr, fmaxf(s0, s1));
            const float p0 = pt_ex2(fmaf(s0, scale_log2, -mref)), p1 = pt_ex2(fmaf(s1, scale_log2, -mref));
            rs += p0 + p1;
            pk[i >> 1] = pack_bf16x2(p0, p1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const int kk = key0 + cbase + i;
            const float s0 = kk <= lim ? __uint_as_float(raw[i]) : -INFINITY;
            const float s1 = kk + 1 <= lim ? __uint_as_float(raw[i + 1]) : -INFINITY;
            mxr = fmaxf(mxr, fmaxf(s0, s1));
            const float p0 = kk <= lim ? pt_ex2(fmaf(s0, scale_log2, -mref)) : 0.f;
            const float p1 = kk + 1 <= lim ? pt_ex2(fmaf(s1, scale_log2, -mref)) : 0.f;
            rs += p0 + p1;
            pk[i >> 1] = pack_bf16x2(p0, p1);
          }
        }
#pragma unroll
        for (int cc = 0; cc < 8; ++cc)
          *reinterpret_cast<uint4*>(smem + kPT_P + pt_swz(r, (cbase >> 3) + cc)) =
              make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
        xmax[half * 128 + r] = mxr == -INFINITY ? -INFINITY : mxr * scale_log2;
        pair_sync();
        const float mx = fmaxf(xmax[r], xmax[128 + r]);
        pair_sync();                                           // both halves read before reuse
        // decisions are identical for the two warps of a row set and warp-uniform: the TMEM
        // loads/stores below are warp-collective and must never run in a partial warp
        const bool redo = mx != -INFINITY && (m == -INFINITY || mx > m + 8.f);
        if (pass == 1 || !__any_sync(0xffffffffu, redo)) break;
        const bool grow = redo && m != -INFINITY;
        const float alpha = grow ? exp2f(m - mx) : 1.f;
        if (__any_sync(0xffffffffu, grow)) {
          l *= alpha;
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 16) {
            float v[16];
            tc::tmem_ld16(tO + lane_off + cbase + c0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= alpha;
            tc::tmem_st16(tO + lane_off + cbase + c0, v);
          }
        }
        if (redo) m = mx;
      }
      l += rs;
      tc::tc_fence_before();
      tc::fence_proxy_async_smem();                            // P (generic writes) -> MMA (async proxy)
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&s_free[j & 1]);
        tc::mbar_arrive(p_full);
      }
    }
    // ---- epilogue: O / (l_lo + l_hi) -> out rows, each half its 64 dims ----
    if (ok && n_tiles > 0) ok = warp_wait(pv_done, (uint32_t)((n_tiles - 1) & 1), 39);
    ok = agree(ok);
    xsum[half * 128 + r] = l;
    pair_sync();
    const float lt = xsum[r] + xsum[128 + r];
    if (ok) {
      tc::tc_fence_after();
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      __nv_bfloat16* dst = out + ((size_t)(row0 + t) * nq + kvh * G + r % G) * kPT_HD + cbase;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 16) {
        float v[16];
        tc::tmem_ld16(tO + lane_off + cbase + c0, v);
        if (t < nrows) {
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) pk[i >> 1] = pack_bf16x2(v[i] * inv, v[i + 1] * inv);
          *reinterpret_cast<uint4*>(dst + c0) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(dst + c0 + 8) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    }
    tc::tc_fence_before();
  }
  __syncthreads();
  if (*abort_flag) {
    // error path: let TMA copies still in flight land before the CTA's shared memory is reused
    const uint64_t until = globaltimer_ns() + 100000ull;
    while (globaltimer_ns() < until) {
    }
  }
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFnPT)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// KV cache viewed as [rows = blocks * kv_heads * 16, 128] bf16; box 64 dims x 16 rows, 128-byte swizzle.
static CUtensorMap pt_tmap(const void* base, int64_t rows) {
  static EncodeTiledFnPT fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qr;
    B200_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr));
    TORCH_CHECK(qr == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFnPT>(ptr);
  });
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)kPT_HD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kPT_HD * 2};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (prefill KV) failed: ", (int)r);
  return m;
}

static int* g_pt_err = nullptr;

}  // namespace b200

using namespace b200;

int64_t prefill_tc_error(bool reset) {
  if (!g_pt_err) return 0;
  int v = 0;
  B200_CHECK_CUDA(cudaMemcpy(&v, g_pt_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) B200_CHECK_CUDA(cudaMemset(g_pt_err, 0, sizeof(int)));
  return v;
}

// q [T, nq, 128] bf16 (rows of all sequences back to back), caches [blocks][nkv][16][128] bf16.
void paged_prefill_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start,
                                torch::Tensor cu_q, torch::Tensor out, double scale, int64_t max_q) {
  const int nq = q.size(1), nkv = k_cache.size(1), S = seq_lens.size(0);
  TORCH_CHECK(q.size(2) == kPT_HD && k_cache.size(3) == kPT_HD && k_cache.size(2) == 16 &&
                  k_cache.scalar_type() == at::kBFloat16 && q.is_contiguous() && out.is_contiguous(),
              "tcgen05 prefill attention: bf16 paged KV [blocks][nkv][16][128]");
  const int G = nq / nkv;
  if (S == 0 || q.size(0) == 0) return;
  if (!g_pt_err) {
    B200_CHECK_CUDA(cudaMalloc(&g_pt_err, sizeof(int)));
    B200_CHECK_CUDA(cudaMemset(g_pt_err, 0, sizeof(int)));
  }
  const int64_t rows = k_cache.size(0) * (int64_t)nkv * 16;
  const CUtensorMap tk = pt_tmap(k_cache.data_ptr(), rows), tv = pt_tmap(v_cache.data_ptr(), rows);
  const int QT = kPT_Rows / G;
  const dim3 grid((unsigned)((max_q + QT - 1) / QT), nkv, S);
  const float sl2 = (float)(scale * 1.4426950408889634);
  auto stream = at::cuda::getCurrentCUDAStream();
#define B200_PT(GV)                                                                                          \
  {                                                                                                          \
    static bool attr = false;                                                                                \
    if (!attr) {                                                                                             \
      B200_CHECK_CUDA(cudaFuncSetAttribute(paged_prefill_tc_kernel<GV>,                                      \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPT_Smem));     \
      attr = true;                                                                                           \
    }                                                                                                        \
    launch_pdl(paged_prefill_tc_kernel<GV>, grid, dim3(320), kPT_Smem, stream, tk, tv,                       \
               reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (const int*)block_tables.data_ptr<int>(), \
               (int)block_tables.size(1), (const int*)seq_lens.data_ptr<int>(),                              \
               (const int*)q_start.data_ptr<int>(), (const int*)cu_q.data_ptr<int>(),                       \
               reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nq, nkv, sl2, g_pt_err, (int)k_cache.size(0)); \
  }
  switch (G) {
    case 1: B200_PT(1) break;
    case 2: B200_PT(2) break;
    case 4: B200_PT(4) break;
    case 8: B200_PT(8) break;
    default: TORCH_CHECK(false, "unsupported GQA group ", G);
  }
#undef B200_PT
}

B200_BOUNDS_ACCESSOR(attention_prefill_tc)
