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

// int4g128 page stage: raw codes K (1 KB) | V (1 KB) | K scales (32 B) | V scales (32 B), padded
constexpr int kQ4Raw = 2 * 1024 + 2 * 32 + 64;

// Dequantise one int4g128 page (raw stage) into the swizzled bf16 stage layout.
// Lane l converts row l/2, dims [64*(l&1), +64): 8 words of 8 interleaved nibbles.
__device__ __forceinline__ void dequant_q4_page(const uint8_t* raw, uint8_t* work, int lane) {
  const int row = lane >> 1, half = lane & 1;
#pragma unroll
  for (int kv = 0; kv < 2; ++kv) {
    const uint4* src = reinterpret_cast<const uint4*>(raw + kv * 1024 + row * 64 + half * 32);
    const __half sh = reinterpret_cast<const __half*>(raw + 2048 + kv * 32)[row];
    const __nv_bfloat16 sb = __float2bfloat16_rn(__half2float(sh));
    const uint32_t s2 = (uint32_t)__bfloat16_as_ushort(sb) * 0x00010001u;
    const uint32_t off = 0x43084308u;   // bf16 (136, 136): 128 (magic) + 8 (offset binary)
    uint8_t* dst_base = work + kv * 2 * kBoxBytes;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 c = src[j];
      const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t r[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const uint32_t qq = ((wv[w] >> (4 * p)) & 0x000F000Fu) | 0x43004300u;   // (128+q, 128+q')
          uint32_t d;
          asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(qq), "r"(off));      // q - 8 (exact)
          asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r[p]) : "r"(d), "r"(s2));
        }
        const int chunk = half * 8 + j * 4 + w;   // 16-byte chunk = 8 dims
        *reinterpret_cast<uint4*>(dst_base + swz(row, chunk)) = make_uint4(r[0], r[1], r[2], r[3]);
      }
    }
  }
}

// TurboQuant page stage (KVQ == 2), per (page, kv head):
//   K codes [16][64] (one 4-bit index per dim, byte m = dims 2m | 2m+1 << 4) | K QJL signs [16][16]
//   (bit i = sign of row i of S r) | K (norm, gamma) [16][2] fp16 | V codes [16][64] | V norm [16] fp16.
// Scores run in the rotated domain over a 256-dim virtual key: [u_hat | s] against the query
// [H q | S H q]; the two halves accumulate separately and combine per token as
// n (q.u_hat) + n gamma (qj.s), so the per-token norms never touch the tiles. V tiles hold the
// unscaled code values; each token's V norm scales its softmax weight instead.
constexpr int kTqKCodes = 0, kTqKSign = 1024, kTqKMeta = 1280, kTqVCodes = 1344, kTqVMeta = 2368;
constexpr int kTqRaw = 2400;
// pair tables (bf16x2 per code byte) for K and V
constexpr int kTqLut = 2 * 256 * 4;

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Expand one TurboQuant page into the work stage: code values of K (boxes 0-1), +-1 signs of K
// (boxes 2-3), code values of V (4-5). Codes go through the pair tables, signs are set with bit
// operations; every access names shared memory explicitly. Lane l converts row l/2, dims
// [64*(l&1), +64).
__device__ __forceinline__ void dequant_tq_page(uint32_t raw, uint32_t work, int lane, uint32_t lutk, uint32_t lutv) {
  const int row = lane >> 1, half = lane & 1;
#pragma unroll
  for (int kv = 0; kv < 2; ++kv) {
    const uint32_t src = raw + (kv ? kTqVCodes : kTqKCodes) + row * 64 + half * 32;
    const uint32_t lut = kv ? lutv : lutk;
    const uint32_t dst = work + (kv ? 4 : 0) * kBoxBytes;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 c = lds128(src + j * 16);
      const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint4 r = make_uint4(lds32(lut + (wv[w] & 255u) * 4), lds32(lut + ((wv[w] >> 8) & 255u) * 4),
                                   lds32(lut + ((wv[w] >> 16) & 255u) * 4), lds32(lut + (wv[w] >> 24) * 4));
        sts128(dst + swz(row, half * 8 + j * 4 + w), r);
      }
    }
  }
  // signs: bit 1 -> +1 (0x3F80), bit 0 -> -1 (0xBF80)
  const uint32_t s0 = lds32(raw + kTqKSign + row * 16 + half * 8), s1 = lds32(raw + kTqKSign + row * 16 + half * 8 + 4);
#pragma unroll
  for (int by = 0; by < 8; ++by) {    // dims 8*by .. 8*by+7 of this half
    const uint32_t bits = ((by < 4 ? s0 : s1) >> (8 * (by & 3))) & 255u;
    uint32_t r[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t neg_lo = ((bits >> (2 * p)) & 1u) ^ 1u, neg_hi = ((bits >> (2 * p + 1)) & 1u) ^ 1u;
      r[p] = 0x3F803F80u | (neg_lo << 15) | (neg_hi << 31);
    }
    sts128(work + swz(row, 16 + half * 8 + by), make_uint4(r[0], r[1], r[2], r[3]));
  }
}

struct TqArgs {
  const uint8_t* ksign;             // [pages][16][16]
  const __nv_bfloat16* qj;          // [B, nq, 128]: S H q
  float cbk[16], cbv[16];           // value of each 4-bit code (sign and 1/sqrt(d) folded in)
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   tc::smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(tc::smem_u32(bar))
               : "memory");
}

template <int G, int KVQ>
__global__ void __launch_bounds__(kTcWarps * 32, 2) paged_decode_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    const __nv_bfloat16* __restrict__ q, const int* __restrict__ block_tables, const int* __restrict__ seq_lens,
    int max_blocks, int nkv, float scale_log2, int tps, float* __restrict__ part_acc, float* __restrict__ part_ml,
    __nv_bfloat16* __restrict__ out, int nsplit, int* err, const uint8_t* __restrict__ kq,
    const uint8_t* __restrict__ vq, const __half* __restrict__ ks, const __half* __restrict__ vs, const TqArgs tq,
    int nblocks, const int* __restrict__ tok_lo, int split_base, int nsplit_total) {
  static_assert(G >= 1 && G <= 16, "query heads per kv head");
  constexpr int KSTEPS = KVQ == 2 ? 16 : 8;        // 16-dim MMA k-steps of the (virtual) key
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  // bf16 pages: ring of kTcStages swizzled stages per warp. int4 pages: ring of raw stages plus
  // one swizzled work stage per warp.
  constexpr int kRaw = KVQ == 2 ? kTqRaw : kQ4Raw;
  constexpr int kWarpBytes = KVQ == 2 ? (kTcStages * kTqRaw + 6 * kBoxBytes)
                             : KVQ ? (kTcStages * kQ4Raw + kStageBytes) : kTcStages * kStageBytes;
  uint8_t* ring = smem + warp * kWarpBytes;
  uint8_t* work = ring + kTcStages * kRaw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcWarps * kWarpBytes) + warp * kTcStages;
  uint32_t* lutk = reinterpret_cast<uint32_t*>(smem + kTcWarps * kWarpBytes + kTcWarps * kTcStages * 8);
  uint32_t* lutv = lutk + 256;
  if constexpr (KVQ == 2) {
    for (int e = threadIdx.x; e < 512; e += blockDim.x) {
      const float* cb = e < 256 ? tq.cbk : tq.cbv;
      const int i = e & 255;
      lutk[e] = pack_bf16x2(cb[i & 15], cb[i >> 4]);
    }
    __syncthreads();
  }
  float* mrg = reinterpret_cast<float*>(smem);   // merge scratch, reuses the rings after the page loop

  pdl_wait();
  pdl_trigger();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int len = seq_lens[b];
  const int nq = nkv * G;
  // tokens [tok_lo[b], len) when given (a multiple of 16), split into chunks of tps
  const int start = (tok_lo ? tok_lo[b] : 0) + split * tps;
  const int stop = min(len, start + tps);
  const int* bt = block_tables + (size_t)b * max_blocks;

  if (lane == 0) {
    for (int s = 0; s < kTcStages; ++s) tc::mbar_init(&bars[s], 1);
    tc::fence_barrier_init();
  }
  __syncwarp();

  // Q as the A operand: rows = query heads (>= G zero), k = head dims
  uint32_t qa[KSTEPS][4];
#pragma unroll
  for (int kk = 0; kk < KSTEPS; ++kk) {
    const __nv_bfloat16* qsrc = (KVQ == 2 && kk >= 8) ? tq.qj : q;
    const __nv_bfloat16* qb = qsrc + ((size_t)b * nq + kvh * G) * kHD;
    {
      const int d0 = (kk & 7) * 16 + 2 * t4;
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
    const int blk = max(table_block(bt, tok0 >> 4, max_blocks, nblocks, 0x201), 0);   // checked: block 0
    const int page = blk * nkv + kvh;
    if constexpr (KVQ == 0) {
      const int y = page * 16;
      uint8_t* st = ring + s * kStageBytes;
      tc::mbar_arrive_expect_tx(&bars[s], kStageBytes);
      tc::tma_load_2d(st, &tm_k, &bars[s], 0, y, 0ull);
      tc::tma_load_2d(st + kBoxBytes, &tm_k, &bars[s], 64, y, 0ull);
      tc::tma_load_2d(st + 2 * kBoxBytes, &tm_v, &bars[s], 0, y, 0ull);
      tc::tma_load_2d(st + 3 * kBoxBytes, &tm_v, &bars[s], 64, y, 0ull);
    } else if constexpr (KVQ == 2) {
      uint8_t* st = ring + s * kTqRaw;
      tc::mbar_arrive_expect_tx(&bars[s], kTqRaw);
      bulk_load(st + kTqKCodes, kq + (size_t)page * 1024, 1024, &bars[s]);
      bulk_load(st + kTqKSign, tq.ksign + (size_t)page * 256, 256, &bars[s]);
      bulk_load(st + kTqKMeta, reinterpret_cast<const uint8_t*>(ks) + (size_t)page * 64, 64, &bars[s]);
      bulk_load(st + kTqVCodes, vq + (size_t)page * 1024, 1024, &bars[s]);
      bulk_load(st + kTqVMeta, reinterpret_cast<const uint8_t*>(vs) + (size_t)page * 32, 32, &bars[s]);
    } else {
      uint8_t* st = ring + s * kQ4Raw;
      tc::mbar_arrive_expect_tx(&bars[s], 2 * 1024 + 2 * 32);
      bulk_load(st, kq + (size_t)page * 1024, 1024, &bars[s]);
      bulk_load(st + 1024, vq + (size_t)page * 1024, 1024, &bars[s]);
      bulk_load(st + 2048, ks + (size_t)page * 16, 32, &bars[s]);
      bulk_load(st + 2080, vs + (size_t)page * 16, 32, &bars[s]);
    }
  };
  if (lane == 0)
    for (int i = 0; i < min(n_pages, kTcStages); ++i) issue(i);
  __syncwarp();

  volatile int never = 0;
  for (int i = 0; i < n_pages; ++i) {
    const int s = i % kTcStages;
    const uint32_t phase = (uint32_t)((i / kTcStages) & 1);
    if (!tc::mbar_wait_bounded(&bars[s], phase, &never, err, 11)) break;
    uint32_t kbase;
    if constexpr (KVQ == 0) {
      kbase = tc::smem_u32(ring + s * kStageBytes);
    } else if constexpr (KVQ == 2) {
      dequant_tq_page(tc::smem_u32(ring + s * kTqRaw), tc::smem_u32(work), lane, tc::smem_u32(lutk),
                      tc::smem_u32(lutv));
      __syncwarp();
      kbase = tc::smem_u32(work);
    } else {
      dequant_q4_page(ring + s * kQ4Raw, work, lane);
      __syncwarp();
      kbase = tc::smem_u32(work);
    }
    const uint32_t vbase = kbase + (KVQ == 2 ? 4 : 2) * kBoxBytes;
    const int tok0 = first + i * kTcWarps * 16;
    // ---- S^T [heads x 16 tokens] ----
    float sc[2][4], sg[2][4];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
      sg[nb][0] = sg[nb][1] = sg[nb][2] = sg[nb][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      // matrices: (tok 0-7, chunk 2kk), (tok 0-7, chunk 2kk+1), (tok 8-15, 2kk), (tok 8-15, 2kk+1)
      const int mi = lane >> 3, r = lane & 7;
      const int tok = (mi >> 1) * 8 + r;
      uint32_t kf[4];
      ldsm_x4(kf, kbase + swz(tok, kk * 2 + (mi & 1)));
      float (*acc)[4] = (KVQ == 2 && kk >= 8) ? sg : sc;      // TurboQuant: QJL half apart
      mma16816(acc[0], qa[kk], kf[0], kf[1]);
      mma16816(acc[1], qa[kk], kf[2], kf[3]);
    }
    float vn[2][2];                                           // TurboQuant: V norm of this lane's tokens
    if constexpr (KVQ == 2) {
      const uint32_t mb = tc::smem_u32(ring + s * kTqRaw);
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        const uint32_t v2 = lds32(mb + kTqVMeta + (nb * 8 + 2 * t4) * 2);       // V norms of both tokens
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = nb * 8 + 2 * t4 + e;
          const uint32_t ng2 = lds32(mb + kTqKMeta + tk * 4);                   // (norm, gamma) fp16
          const float n = __half2float(__ushort_as_half((unsigned short)(ng2 & 0xffffu)));
          const float ng = n * __half2float(__ushort_as_half((unsigned short)(ng2 >> 16)));
          sc[nb][e] = n * sc[nb][e] + ng * sg[nb][e];
          sc[nb][2 + e] = n * sc[nb][2 + e] + ng * sg[nb][2 + e];
          vn[nb][e] = __half2float(__ushort_as_half((unsigned short)(e ? (v2 >> 16) : (v2 & 0xffffu))));
        }
      }
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
      if constexpr (KVQ == 2) {      // V rows hold code values: the token's V norm scales its weight
        pa[nb * 2 + 0] = pack_bf16x2(p0 * vn[nb][0], p1 * vn[nb][1]);
        pa[nb * 2 + 1] = pack_bf16x2(p2 * vn[nb][0], p3 * vn[nb][1]);
      } else {
        pa[nb * 2 + 0] = pack_bf16x2(p0, p1);
        pa[nb * 2 + 1] = pack_bf16x2(p2, p3);
      }
    }
    ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 1);
    ps_a += __shfl_xor_sync(0xffffffffu, ps_a, 2);
    ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 1);
    ps_b += __shfl_xor_sync(0xffffffffu, ps_b, 2);
    l_a = l_a * al_a + ps_a;
    l_b = l_b * al_b + ps_b;
    if (__any_sync(0xffffffffu, al_a != 1.f || al_b != 1.f)) {   // skipped while the maxima hold
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= al_a; o[j][1] *= al_a; o[j][2] *= al_b; o[j][3] *= al_b;
      }
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
    if (nsplit_total == 1) {
      out[((size_t)b * nq + kvh * G + hh) * kHD + d] = __float2bfloat16_rn(L > 0.f ? A / L : 0.f);
    } else {
      const size_t slot = (((size_t)b * nkv + kvh) * nsplit_total + split_base + split) * G + hh;
      part_acc[slot * kHD + d] = A;
      if (d == 0) { part_ml[slot * 2] = M; part_ml[slot * 2 + 1] = L; }
    }
  }
}

size_t decode_tc_smem(int kvq) {
  const size_t per_warp = kvq == 2 ? (kTcStages * kTqRaw + 6 * kBoxBytes)
                          : kvq ? (kTcStages * kQ4Raw + kStageBytes) : kTcStages * kStageBytes;
  return 1024 + kTcWarps * per_warp + 256 + (kvq == 2 ? kTqLut : 0);
}

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

static void decode_tc_impl(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                           torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_acc, torch::Tensor part_ml,
                           double scale, int64_t tps, int64_t nsplit, int kvq, const uint8_t* kq, const uint8_t* vq,
                           const __half* ksc, const __half* vsc, int nkv, const TqArgs& tq,
                           const int* tok_lo = nullptr, int split_base = 0, int nsplit_total = 0) {
  // nsplit_total 0: this launch covers every split and combines them itself
  const bool own = nsplit_total == 0;
  if (own) nsplit_total = (int)nsplit;
  const int B = q.size(0), nq = q.size(1), HD = q.size(2);
  const int G = nq / nkv;
  TORCH_CHECK(HD == kHD && k_cache.size(2) == 16 && tps % 16 == 0 && nsplit >= 1);
  TORCH_CHECK(split_base >= 0 && split_base + nsplit <= nsplit_total, "splits out of range");
  if (nsplit_total > 1) {
    TORCH_CHECK(part_acc.numel() >= (int64_t)B * nkv * nsplit_total * G * HD, "attention workspace too small");
    TORCH_CHECK(part_ml.numel() >= (int64_t)B * nkv * nsplit_total * G * 2, "attention workspace too small");
  }
  if (B == 0) return;
  CUtensorMap tk, tv;
  if (!kvq) {
    const int64_t rows = k_cache.size(0) * (int64_t)nkv * 16;
    tk = make_tmap_kv(k_cache.data_ptr(), rows);
    tv = make_tmap_kv(v_cache.data_ptr(), rows);
  } else {
    memset(&tk, 0, sizeof(tk));
    memset(&tv, 0, sizeof(tv));
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  const float sl2 = (float)(scale * 1.4426950408889634);
  dim3 grid(nsplit, nkv, B);
  float* pa = nsplit_total > 1 ? part_acc.data_ptr<float>() : nullptr;
  float* pm = nsplit_total > 1 ? part_ml.data_ptr<float>() : nullptr;
  auto op = (out.defined() && out.numel()) ? reinterpret_cast<__nv_bfloat16*>(out.data_ptr()) : nullptr;
  const size_t smem = decode_tc_smem(kvq);
#define B200_TC1(GV, KQ)                                                                                       \
  {                                                                                                            \
    static bool attr = false;                                                                                  \
    if (!attr) {                                                                                               \
      B200_CHECK_CUDA(cudaFuncSetAttribute(paged_decode_tc_kernel<GV, KQ>,                                     \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));          \
      attr = true;                                                                                             \
    }                                                                                                          \
    launch_pdl(paged_decode_tc_kernel<GV, KQ>, grid, dim3(kTcWarps * 32), smem, stream, tk, tv,                \
               reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (const int*)block_tables.data_ptr<int>(),  \
               (const int*)seq_lens.data_ptr<int>(), (int)block_tables.size(1), nkv, sl2, (int)tps, pa, pm, op, \
               (int)nsplit, decode_tc_err_word(), kq, vq, ksc, vsc, tq, (int)k_cache.size(0), tok_lo,         \
               split_base, nsplit_total);                                                                   \
  }
#define B200_TC(GV) { if (kvq == 2) B200_TC1(GV, 2) else if (kvq) B200_TC1(GV, 1) else B200_TC1(GV, 0) }
  switch (G) {
    case 1: B200_TC(1) break;
    case 2: B200_TC(2) break;
    case 4: B200_TC(4) break;
    case 8: B200_TC(8) break;
    case 16: B200_TC(16) break;
    default: TORCH_CHECK(false, "unsupported GQA group ", G);
  }
#undef B200_TC
#undef B200_TC1
  if (own && nsplit > 1) paged_decode_combine(part_acc, part_ml, seq_lens, out, nkv, G, nsplit, tps);
}

// Splits [split_base, split_base + nsplit) of a decode attention whose partials the caller merges
// (paged_decode_combine over nsplit_total splits, tps 0): bf16 pages over tokens [tok_lo[b], len).
void paged_decode_attention_tc_part(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                    torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor tok_lo,
                                    torch::Tensor part_acc, torch::Tensor part_ml, double scale, int64_t tps,
                                    int64_t nsplit, int64_t split_base, int64_t nsplit_total) {
  TORCH_CHECK(nsplit_total >= 2 && tok_lo.scalar_type() == at::kInt && tok_lo.numel() == q.size(0));
  TqArgs none{};
  decode_tc_impl(q, k_cache, v_cache, block_tables, seq_lens, torch::Tensor(), part_acc, part_ml, scale, tps, nsplit,
                 0, nullptr, nullptr, nullptr, nullptr, k_cache.size(1), none, (const int*)tok_lo.data_ptr<int>(),
                 (int)split_base, (int)nsplit_total);
}

void paged_decode_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                               torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor out,
                               torch::Tensor part_acc, torch::Tensor part_ml, double scale, int64_t tps,
                               int64_t nsplit) {
  TqArgs none{};
  decode_tc_impl(q, k_cache, v_cache, block_tables, seq_lens, out, part_acc, part_ml, scale, tps, nsplit, 0, nullptr,
                 nullptr, nullptr, nullptr, k_cache.size(1), none);
}

// int4g128 KV: codes [blocks][nkv][16][64] uint8, scales [blocks][nkv][16] fp16.
void paged_decode_attention_q4(torch::Tensor q, torch::Tensor k_codes, torch::Tensor v_codes, torch::Tensor k_scale,
                               torch::Tensor v_scale, torch::Tensor block_tables, torch::Tensor seq_lens,
                               torch::Tensor out, torch::Tensor part_acc, torch::Tensor part_ml, double scale,
                               int64_t tps, int64_t nsplit) {
  TORCH_CHECK(k_codes.size(3) == 64 && k_codes.scalar_type() == at::kByte, "int4g128 codes must be [*, nkv, 16, 64] uint8");
  decode_tc_impl(q, k_codes, v_codes, block_tables, seq_lens, out, part_acc, part_ml, scale, tps, nsplit, 1,
                 k_codes.data_ptr<uint8_t>(), v_codes.data_ptr<uint8_t>(),
                 reinterpret_cast<const __half*>(k_scale.data_ptr()), reinterpret_cast<const __half*>(v_scale.data_ptr()),
                 k_codes.size(1), TqArgs{});
}

// TurboQuant KV: codes [blocks][nkv][16][64] uint8 (one 4-bit code per dim), k_sign [blocks][nkv][16][16]
// uint8, k_meta [blocks][nkv][16][2] fp16 (norm, gamma), v_meta [blocks][nkv][16] fp16 (norm).
// q_rot = H q and q_jl = S H q, [B, nq, 128] bf16; the output is in the rotated domain (H o).
// code_vals: float [2][16] = value of each K / V code.
void paged_decode_attention_tq(torch::Tensor q_rot, torch::Tensor q_jl, torch::Tensor k_codes, torch::Tensor k_sign,
                               torch::Tensor k_meta, torch::Tensor v_codes, torch::Tensor v_meta,
                               torch::Tensor code_vals, torch::Tensor block_tables, torch::Tensor seq_lens,
                               torch::Tensor out, torch::Tensor part_acc, torch::Tensor part_ml, double scale,
                               int64_t tps, int64_t nsplit) {
  TORCH_CHECK(k_codes.size(3) == 64 && k_codes.scalar_type() == at::kByte && k_sign.size(3) == 16,
              "turboquant codes must be [*, nkv, 16, 64] and signs [*, nkv, 16, 16] uint8");
  TORCH_CHECK(q_jl.sizes() == q_rot.sizes() && q_jl.is_contiguous() && q_rot.is_contiguous());
  TORCH_CHECK(code_vals.device().is_cpu(), "code_vals is a host tensor (baked into the launch parameters)");
  auto cv = code_vals.to(at::kFloat).contiguous();
  TORCH_CHECK(cv.numel() == 32, "code_vals must hold 2 x 16 values");
  TqArgs tq{};
  tq.ksign = k_sign.data_ptr<uint8_t>();
  tq.qj = reinterpret_cast<const __nv_bfloat16*>(q_jl.data_ptr());
  for (int i = 0; i < 16; ++i) { tq.cbk[i] = cv.data_ptr<float>()[i]; tq.cbv[i] = cv.data_ptr<float>()[16 + i]; }
  decode_tc_impl(q_rot, k_codes, v_codes, block_tables, seq_lens, out, part_acc, part_ml, scale, tps, nsplit, 2,
                 k_codes.data_ptr<uint8_t>(), v_codes.data_ptr<uint8_t>(),
                 reinterpret_cast<const __half*>(k_meta.data_ptr()), reinterpret_cast<const __half*>(v_meta.data_ptr()),
                 k_codes.size(1), tq);
}

// The TurboQuant splits [split_base, split_base + nsplit) of a decode attention merged by the caller
// (the residual window adds a bf16 split after them).
void paged_decode_attention_tq_part(torch::Tensor q_rot, torch::Tensor q_jl, torch::Tensor k_codes,
                                    torch::Tensor k_sign, torch::Tensor k_meta, torch::Tensor v_codes,
                                    torch::Tensor v_meta, torch::Tensor code_vals, torch::Tensor block_tables,
                                    torch::Tensor seq_lens, torch::Tensor part_acc, torch::Tensor part_ml, double scale,
                                    int64_t tps, int64_t nsplit, int64_t split_base, int64_t nsplit_total) {
  TORCH_CHECK(k_codes.size(3) == 64 && k_codes.scalar_type() == at::kByte && k_sign.size(3) == 16,
              "turboquant codes must be [*, nkv, 16, 64] and signs [*, nkv, 16, 16] uint8");
  TORCH_CHECK(q_jl.sizes() == q_rot.sizes() && q_jl.is_contiguous() && q_rot.is_contiguous() && nsplit_total >= 2);
  TORCH_CHECK(code_vals.device().is_cpu(), "code_vals is a host tensor (baked into the launch parameters)");
  auto cv = code_vals.to(at::kFloat).contiguous();
  TORCH_CHECK(cv.numel() == 32, "code_vals must hold 2 x 16 values");
  TqArgs tq{};
  tq.ksign = k_sign.data_ptr<uint8_t>();
  tq.qj = reinterpret_cast<const __nv_bfloat16*>(q_jl.data_ptr());
  for (int i = 0; i < 16; ++i) { tq.cbk[i] = cv.data_ptr<float>()[i]; tq.cbv[i] = cv.data_ptr<float>()[16 + i]; }
  decode_tc_impl(q_rot, k_codes, v_codes, block_tables, seq_lens, torch::Tensor(), part_acc, part_ml, scale, tps,
                 nsplit, 2, k_codes.data_ptr<uint8_t>(), v_codes.data_ptr<uint8_t>(),
                 reinterpret_cast<const __half*>(k_meta.data_ptr()), reinterpret_cast<const __half*>(v_meta.data_ptr()),
                 k_codes.size(1), tq, nullptr, (int)split_base, (int)nsplit_total);
}

B200_BOUNDS_ACCESSOR(attention_decode_tc)
