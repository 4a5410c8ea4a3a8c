// GGUF block-quantised GEMV for decode batches of 1..16 tokens: a persistent, stream-K kernel
// that keeps the weight stream in flight with bulk copies into shared memory.
//
// Work: a group of matrices that share the input (each N % 128 == 0) is cut into 128-row tiles
// (8 slices of 16 rows in the fragment order of models/gguf.py: one 32-bit word of 4-bit codes
// or two of 8-bit codes per lane per 16-column k-step) and 256-column chunks; `items` = tiles x
// chunks, tile-major. CTA g owns the contiguous items [g*items/G, (g+1)*items/G), so every CTA
// streams the same number of bytes whatever the shapes. Two CTAs per SM, each with one producer
// warp and eight consumer warps:
//   producer  fills a ring of stages with cp.async.bulk copies into this CTA only: per item the
//             codes and scales of the 8 slices plus the item's 256 activation columns of every
//             token (rows padded by 16 bytes so the B-fragment reads hit 32 distinct banks);
//             the weights of the first stages are requested before the dependency wait
//   consumer  warp w dequantises slice w of each landed item in registers (gguf_common.cuh)
//             and runs mma.sync m16n8k16 with the staged activations as the B operand
// Code types: 4-bit (Q4_K: scale and -min per 32), 8-bit (Q6_K / Q8_0: scale per 16 or 32), 4-bit
// indices into the 16-value IQ4 table (bits 5: a 256-entry pair table in shared memory, scale per
// 32), and E8 lattice vectors (bits 2: one byte per 8 weights, a 256 x 8 codebook in shared memory,
// scale and offset per group; the MMA k-slots are permuted so each lane reads half a vector).
// All waits are bounded (error 190 in the last counter word, then the CTA drains and exits).
//
// A CTA's range starts and ends inside tiles, so a tile's rows are summed over the CTAs
// first(t)..last(t) that hold its items:
//   GS_PARTIAL      fp32 part[g - first(t)][tok][col] (PartialIn with 128-column tiles: the
//                   same contract as the tcgen05 stream-K GEMM), summed by the consuming row
//                   kernel (RMSNorm, qkv_post, silu_mul_partial)
//   GS_BF16/GS_F32  out[tok][col]; a tile shared by several CTAs is finished by the last to
//   GS_PUSH         arrive (per-tile counter; partials summed in CTA order, so the result does not
//                   depend on timing); GS_PUSH stores the bf16 tile into every rank's flag-free
//                   all-reduce slot (P2P, or one multimem store through an NVLink multicast object)
//
// Reference kernels restated: webgpu/src/shaders/matmul_gguf.wgsl:2103-3310 (q4_k / q6_k / q8_0
// matmuls), with the weight repack of webgpu/src/model/gguf-dequant.ts:152-406.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "gguf_common.cuh"
#include "tc_primitives.cuh"

namespace b200 {

enum GsMode : int { GS_BF16 = 0, GS_F32 = 1, GS_PARTIAL = 2, GS_PUSH = 4 };

constexpr int kGsConsumers = 8;             // consumer warps = slices per tile
constexpr int kGsThreads = (kGsConsumers + 1) * 32;
constexpr int kGsMaxParts = 4;
// bf16 per staged activation row: 256 + padding so that the B-fragment reads of a warp hit distinct
// banks (32-bit reads: a row stride of 4 words mod 32; the E8 path's 64-bit reads: 8 words)
template <int BITS>
struct GsX {
  static constexpr int row = BITS == 2 ? 272 : 264;
};
constexpr int kGsXBytes = 16 * 272 * 2;     // activation rows of one stage (up to 16 tokens)
constexpr int kGsSmemBudget = 110 * 1024;   // per CTA: two CTAs per SM
constexpr int kGsCtl = 6144;                // barriers and flags (128 B) + push staging (8 x 512 B) + IQ4 table (1 KB)
constexpr int kGsNlTab = 5120;              // offset of the IQ4 pair table in the control block

// Stage geometry for codes of `bits` (8 also covers groups mixing 4- and 8-bit parts; 2 is the
// E8 vector code: one byte per 8 weights, and a 4 KB codebook table after the control block).
template <int BITS>
struct GsGeom {
  static constexpr int code = BITS == 4 ? 2048 : BITS == 8 ? 4096 : 512;   // codes of one slice-chunk
  static constexpr int meta = 1024;                             // scales of one slice-chunk (max)
  static constexpr int codes_off = 0;
  static constexpr int meta_off = kGsConsumers * code;
  static constexpr int x_off = meta_off + kGsConsumers * meta;
  static constexpr int bytes = x_off + kGsXBytes;
  static constexpr int table = BITS == 2 ? 4096 : 0;
  static constexpr int fit = (kGsSmemBudget - kGsCtl - table) / bytes;
  static constexpr int stages = fit < 4 ? fit : 4;
  static constexpr size_t smem = (size_t)stages * bytes + kGsCtl + table;
  static_assert(stages >= 2 && stages <= 4, "stage too large or too small");
};

// E8 meta: (s, s) and (o, o) as bf16x2 per (group, row); bytes of one slice-chunk
__device__ __forceinline__ uint32_t gs_e8_meta_bytes(int group) { return (uint32_t)(256 / group) * 128u; }

struct GsPart {
  const uint32_t* codes;
  const uint32_t* meta;
  int tile0;                                // first 128-row tile of this matrix in the group
  int slices;                               // N / 16 (the last tile may hold fewer than 8 slices)
  int col0;                                 // first output column of this matrix in the group
  int bits, group;
};

struct GsArgs {
  GsPart parts[kGsMaxParts];
  int nparts;
  const __nv_bfloat16* x;
  int ldx, M, K, nchunks, tiles;
  int items;
  int ctas;
  void* out;                                // GS_BF16 / GS_F32 output, GS_PARTIAL slots
  int ldo;                                  // output row stride (= group width for partials)
  long long part_slot;                      // floats per partial slot
  float* ws;                                // [ctas][2][16 tokens][128 rows] fp32 shared-tile partials
  int* counters;                            // [tiles] arrival counters (zero between launches)
  __nv_bfloat16* push[8];                   // GS_PUSH: this rank's slot base on every rank
  int world;
  __nv_bfloat16* mc;                        // GS_PUSH through a multicast object
  const uint32_t* table;                    // E8 parts: codebook as bf16 pairs [256][4]; IQ4 parts (bits 5):
                                            // bf16 pairs of the 16-value table for every code byte [256]
  int* err;
  uint64_t wait_ns;
};

// items * ctas < 2^32 (checked on the host), so the share arithmetic stays in 32 bits
__device__ __forceinline__ int gs_begin(const GsArgs& a, int c) {
  return (int)((uint32_t)c * (uint32_t)a.items / (uint32_t)a.ctas);
}
// the CTA holding item i: the largest c with gs_begin(c) <= i
__device__ __forceinline__ int gs_owner(const GsArgs& a, int i) {
  return (int)(((uint32_t)(i + 1) * (uint32_t)a.ctas + (uint32_t)a.items - 1) / (uint32_t)a.items) - 1;
}

__device__ __forceinline__ int gs_part_of(const GsArgs& a, int tile) {
  int p = 0;
#pragma unroll
  for (int q = 1; q < kGsMaxParts; ++q)
    if (q < a.nparts && tile >= a.parts[q].tile0) p = q;
  return p;
}

__device__ __forceinline__ bool gs_wait(uint64_t* bar, uint32_t parity, const GsArgs& a, volatile int* abort_flag) {
  if (tc::mbar_try_wait(bar, parity)) return true;
  const uint64_t deadline = globaltimer_ns() + a.wait_ns;
  for (uint32_t it = 1;; ++it) {
    if (tc::mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if ((it & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() > deadline) {
        if (a.err) atomicExch(a.err, 190);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Producer, all 32 lanes. `what`: GS_ANNOUNCE (lane 0 tells the stage's barrier to expect all of
// the item's bytes), GS_W (lane l < 8 copies slice l's codes, 8 <= l < 16 its scales), GS_X
// (lane 16 + t copies the item's 256 activation columns of token t). The weights of the first
// stages go out (announced) before the dependency wait, their activations after it.
enum : int { GS_ANNOUNCE = 1, GS_W = 2, GS_X = 4 };

template <int BITS>
__device__ __forceinline__ void gs_issue(const GsArgs& a, int tile, int c, uint8_t* st, uint64_t* bar, int lane,
                                         int what) {
  using Gm = GsGeom<BITS>;
  const GsPart& p = a.parts[gs_part_of(a, tile)];
  const int ksteps = a.K / 16;
  const bool b4 = p.bits == 4 || p.bits == 5;                   // 5: 4-bit codes through the IQ4 table
  const uint32_t cbytes = b4 ? 2048u : p.bits == 8 ? 4096u : 512u;
  const uint32_t mbytes = b4 ? 1024u : p.bits == 8 ? (uint32_t)(256 / p.group) * 64u : gs_e8_meta_bytes(p.group);
  const int nvalid = min(kGsConsumers, p.slices - (tile - p.tile0) * kGsConsumers);
  if ((what & GS_ANNOUNCE) && lane == 0)
    tc::mbar_arrive_expect_tx(bar, (uint32_t)nvalid * (cbytes + mbytes) + (uint32_t)a.M * 512u);
  __syncwarp();
  if ((what & GS_W) && lane < 2 * kGsConsumers && (lane & 7) < nvalid) {
    const size_t ls = (size_t)(tile - p.tile0) * kGsConsumers + (lane & 7);
    if (lane < kGsConsumers) {
      const uint32_t* src = p.codes + (ls * ksteps + (size_t)c * 16) * (b4 ? 32 : p.bits == 8 ? 64 : 8);
      tc::bulk_g2s(st + Gm::codes_off + (lane & 7) * Gm::code, src, cbytes, bar);
    } else {
      const uint32_t* src = b4 ? p.meta + (ls * (a.K / 32) + (size_t)c * 8) * 32
                            : p.meta + (ls * (a.K / p.group) + (size_t)c * (256 / p.group)) * (p.bits == 8 ? 16 : 32);
      tc::bulk_g2s(st + Gm::meta_off + (lane & 7) * Gm::meta, src, mbytes, bar);
    }
  }
  if ((what & GS_X) && lane >= 16 && lane < 16 + a.M) {
    const int tok = lane - 16;
    tc::bulk_g2s(st + Gm::x_off + tok * GsX<BITS>::row * 2, a.x + (size_t)tok * a.ldx + (size_t)c * 256, 512u, bar);
  }
}

// Consumer warp w: slice w of the staged item (codes of `bits`) into acc (C fragments: rows g,
// g, g+8, g+8 of the slice x tokens j*8 + 2*t4, +1, +0, +1).
template <int BITS, int NB>
__device__ __forceinline__ void gs_compute(const uint8_t* st, int bits, int group, int w, int lane,
                                           float (&acc)[NB][4], uint32_t cbt, uint32_t nlt) {
  using Gm = GsGeom<BITS>;
  constexpr int kGsXRow = GsX<BITS>::row;
  const int g = lane >> 2, t4 = lane & 3;
  const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(st + Gm::x_off) + g * kGsXRow + 2 * t4;
  const uint8_t* cb = st + Gm::codes_off + w * Gm::code;
  const uint8_t* mb = st + Gm::meta_off + w * Gm::meta;
  // odd k-steps accumulate separately: two independent MMA chains per item
  float odd[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j) odd[j][0] = odd[j][1] = odd[j][2] = odd[j][3] = 0.f;
  if constexpr (BITS == 2) {
    // The 16 k-slots of each MMA are permuted: lane t4's slots (2t4, 2t4+1, 2t4+8, 2t4+9) carry
    // columns 4t4 .. 4t4+3, i.e. half (t4 & 1) of the k-step's 8-column vector (t4 >> 1). The
    // staged activations are read in the same order (one 64-bit read per token), and each row's
    // four weights are one 64-bit codebook read.
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(cb);          // [16 k-steps][8 row pairs]
    const uint2* mt = reinterpret_cast<const uint2*>(mb);                 // [256 / group][16 rows] (s, o)
    const int gsh = group == 32 ? 1 : group == 64 ? 2 : group == 128 ? 3 : 4;   // k-steps per group, log2
    const int vsh = 16 * (t4 >> 1);                                       // this lane's vector in the word
    const uint32_t half = cbt + 8u * (uint32_t)(t4 & 1);
    const __nv_bfloat16* xp = xs + 2 * t4;                                // columns 4t4 .. 4t4+3
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      const int gi = ks >> gsh;
      const uint2 ma = mt[gi * 16 + g], mc = mt[gi * 16 + g + 8];
      const uint32_t q = cw[ks * 8 + g] >> vsh;
      const uint2 ra = lds_u64(half + ((q & 255u) << 4)), rb = lds_u64(half + (((q >> 8) & 255u) << 4));
      uint32_t wv[4];
      wv[0] = bf2_fma(ra.x, ma.x, ma.y);
      wv[1] = bf2_fma(rb.x, mc.x, mc.y);
      wv[2] = bf2_fma(ra.y, ma.x, ma.y);
      wv[3] = bf2_fma(rb.y, mc.x, mc.y);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const uint2 bx = *reinterpret_cast<const uint2*>(xp + j * 8 * kGsXRow + ks * 16);
        qmma((ks & 1) ? odd[j] : acc[j], wv, bx.x, bx.y);
      }
    }
  } else if (bits == 5) {
    // IQ4: byte i of the lane's word is register i's pair of table indices; w = s * table[q]
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(cb);
    const uint2* mt = reinterpret_cast<const uint2*>(mb);                 // [8 sub-blocks][16 rows] (s, 0)
#pragma unroll
    for (int sb = 0; sb < 8; ++sb) {
      const uint32_t sa = mt[sb * 16 + g].x, sc = mt[sb * 16 + g + 8].x;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int ks = sb * 2 + h;
        const uint32_t q = cw[ks * 32 + lane];
        uint32_t wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          wv[i] = bf2_fma(lds_u32(nlt + (((q >> (8 * i)) & 255u) << 2)), (i & 1) ? sc : sa, 0u);
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const __nv_bfloat16* r = xs + j * 8 * kGsXRow + ks * 16;
          qmma(h ? odd[j] : acc[j], wv, *reinterpret_cast<const uint32_t*>(r), *reinterpret_cast<const uint32_t*>(r + 8));
        }
      }
    }
  } else if (BITS == 4 || bits == 4) {
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(cb);
    const uint2* mt = reinterpret_cast<const uint2*>(mb);                 // [8 sub-blocks][16 rows] (s, -m)
#pragma unroll
    for (int sb = 0; sb < 8; ++sb) {
      const uint2 ma = mt[sb * 16 + g], mc = mt[sb * 16 + g + 8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int ks = sb * 2 + h;
        uint32_t wv[4];
        dequant_u4(cw[ks * 32 + lane], ma.x, ma.y, mc.x, mc.y, wv);
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const __nv_bfloat16* r = xs + j * 8 * kGsXRow + ks * 16;
          qmma(h ? odd[j] : acc[j], wv, *reinterpret_cast<const uint32_t*>(r), *reinterpret_cast<const uint32_t*>(r + 8));
        }
      }
    }
  } else {
    const uint2* cw = reinterpret_cast<const uint2*>(cb);
    const uint32_t* sc = reinterpret_cast<const uint32_t*>(mb);          // [groups][16 rows]
    const int gsh = group == 16 ? 0 : 1;
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      const int gi = ks >> gsh;
      uint32_t wv[4];
      const uint2 q = cw[ks * 32 + lane];
      dequant_s8(q.x, q.y, sc[gi * 16 + g], sc[gi * 16 + g + 8], wv);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const __nv_bfloat16* r = xs + j * 8 * kGsXRow + ks * 16;
        qmma((ks & 1) ? odd[j] : acc[j], wv, *reinterpret_cast<const uint32_t*>(r),
             *reinterpret_cast<const uint32_t*>(r + 8));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NB; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] += odd[j][e];
}

// Store the finished 16 rows x M tokens of a slice at output column n0 (values in the C-fragment
// layout).
template <int NB>
__device__ __forceinline__ void gs_store(const GsArgs& a, int mode, int n0, const float (&v)[NB][4], int lane,
                                         __nv_bfloat16* stage) {
  const int g = lane >> 2, t4 = lane & 3;
  if (mode == GS_PUSH) {
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = j * 8 + 2 * t4 + (e & 1), row = g + (e >> 1) * 8;
        __nv_bfloat16 h = __float2bfloat16_rn(v[j][e]);
        // 0xFFFF marks an empty flag-free slot; a NaN with that payload is stored as 0x7FFF
        if (__bfloat16_as_ushort(h) == 0xFFFFu) h = __ushort_as_bfloat16((unsigned short)0x7FFFu);
        stage[tok * 16 + row] = h;
      }
    }
    __syncwarp();
    if (lane < 2 * a.M) {                                  // 16 columns = two 16-byte pieces per token
      const int tok = lane >> 1, half = lane & 1;
      const uint4 q = *reinterpret_cast<const uint4*>(stage + tok * 16 + half * 8);
      const size_t off = (size_t)tok * a.ldo + n0 + half * 8;
      if (a.mc) {
        asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};"
                     ::"l"(a.mc + off), "r"(q.x), "r"(q.y), "r"(q.z), "r"(q.w) : "memory");
      } else {
        for (int r = 0; r < a.world; ++r) *reinterpret_cast<uint4*>(a.push[r] + off) = q;
      }
    }
    __syncwarp();
    return;
  }
#pragma unroll
  for (int j = 0; j < NB; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = j * 8 + 2 * t4 + (e & 1), n = n0 + g + (e >> 1) * 8;
      if (tok >= a.M) continue;
      if (mode == GS_F32)
        reinterpret_cast<float*>(a.out)[(size_t)tok * a.ldo + n] = v[j][e];
      else
        reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)tok * a.ldo + n] = __float2bfloat16_rn(v[j][e]);
    }
  }
}

__device__ __forceinline__ void gs_consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kGsConsumers * 32) : "memory"); }

// The CTA's items of `tile` are done: warp w writes slice w's share (partial slot, direct store,
// or the shared-tile fix-up through the workspace and the tile's arrival counter). Every consumer
// warp calls this in the same order, aborted or not, so the named barriers always pair up.
template <int NB>
__device__ __forceinline__ void gs_tile_done(const GsArgs& a, int mode, int cta, int tile, float (&acc)[NB][4],
                                             int w, int lane, volatile int* abort_flag, int* bcast,
                                             __nv_bfloat16* stage) {
  const int g = lane >> 2, t4 = lane & 3;
  const int i_first = tile * a.nchunks;
  const int first = gs_owner(a, i_first), last = gs_owner(a, i_first + a.nchunks - 1);
  const GsPart& p = a.parts[gs_part_of(a, tile)];
  const int local = (tile - p.tile0) * kGsConsumers + w;
  const bool valid = local < p.slices;                     // a ragged last tile has idle warps
  const int n0 = p.col0 + local * 16;
  if (mode == GS_PARTIAL) {
    if (*abort_flag || !valid) return;
    float* part = reinterpret_cast<float*>(a.out) + (size_t)(cta - first) * a.part_slot;
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = j * 8 + 2 * t4 + (e & 1);
        if (tok < a.M) part[(size_t)tok * a.ldo + n0 + g + (e >> 1) * 8] = acc[j][e];
      }
    return;
  }
  if (first == last) {
    if (!*abort_flag && valid) gs_store<NB>(a, mode, n0, acc, lane, stage);
    return;
  }
  // shared tile: a CTA's head tile goes to its workspace slot 0, its tail tile to slot 1
  auto slot_of = [&](int c) { return (gs_begin(a, c) / a.nchunks == tile) ? 0 : 1; };
  if (!*abort_flag) {
    float* mine = a.ws + ((size_t)cta * 2 + slot_of(cta)) * (16 * 128);
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        mine[(j * 8 + 2 * t4 + (e & 1)) * 128 + w * 16 + g + (e >> 1) * 8] = acc[j][e];
  }
  __threadfence();
  gs_consumer_sync();
  if (threadIdx.x == 0) *bcast = *abort_flag ? -1 : atomicAdd(a.counters + tile, 1);
  gs_consumer_sync();
  if (*bcast != last - first) return;
  __threadfence();
  // sum the contributions in CTA order; four CTAs' loads in flight at a time
  float v[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j) v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f;
  for (int c = first; c <= last; c += 4) {
    float ld[4][NB][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (c + u > last) break;
      const float* src = a.ws + ((size_t)(c + u) * 2 + slot_of(c + u)) * (16 * 128) + w * 16;
#pragma unroll
      for (int j = 0; j < NB; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) ld[u][j][e] = __ldcg(src + (j * 8 + 2 * t4 + (e & 1)) * 128 + g + (e >> 1) * 8);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (c + u > last) break;
#pragma unroll
      for (int j = 0; j < NB; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) v[j][e] += ld[u][j][e];
    }
  }
  if (threadIdx.x == 0) a.counters[tile] = 0;                 // ready for the next launch
  if (valid) gs_store<NB>(a, mode, n0, v, lane, stage);
}

template <int BITS, int NB>
__global__ void __launch_bounds__(kGsThreads, 2) gguf_stream_kernel(const GsArgs a, int mode) {
  using Gm = GsGeom<BITS>;
  constexpr int S = Gm::stages;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ctl = smem + (size_t)S * Gm::bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctl);
  uint64_t* empty = full + 4;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + 4);
  int* bcast = reinterpret_cast<int*>(empty + 4) + 1;
  volatile int* issued = reinterpret_cast<volatile int*>(empty + 4) + 2;     // producer: items issued, -1 while running
  __nv_bfloat16* pstage = reinterpret_cast<__nv_bfloat16*>(ctl + 128);
  uint32_t* cbt = reinterpret_cast<uint32_t*>(ctl + kGsCtl);              // E8 codebook (BITS == 2)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int i0 = gs_begin(a, cta), n = gs_begin(a, cta + 1) - i0;
  const int t0 = i0 / a.nchunks, c0 = i0 % a.nchunks;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], kGsConsumers);
    }
    *abort_flag = 0;
    *issued = -1;
    tc::fence_barrier_init();
  }
  uint32_t* nlt = reinterpret_cast<uint32_t*>(ctl + kGsNlTab);           // IQ4 pair table (bits 5 parts)
  if constexpr (BITS == 2) {          // weights: read before the dependency wait
    for (int i = threadIdx.x; i < 1024; i += kGsThreads) cbt[i] = __ldg(a.table + i);
  } else {
    if (a.table != nullptr)
      for (int i = threadIdx.x; i < 256; i += kGsThreads) nlt[i] = __ldg(a.table + i);
  }
  __syncthreads();
  if (warp == kGsConsumers) {
    // ---------------- producer warp (tile, chunk) advance without divisions
    const int pro = min(n, S);
    int tile = t0, c = c0;
    for (int j = 0; j < pro; ++j) {
      gs_issue<BITS>(a, tile, c, smem + j * Gm::bytes, &full[j], lane, GS_ANNOUNCE | GS_W);
      if (++c == a.nchunks) c = 0, ++tile;
    }
    pdl_wait();
    pdl_trigger();
    tile = t0, c = c0;
    for (int j = 0; j < pro; ++j) {
      gs_issue<BITS>(a, tile, c, smem + j * Gm::bytes, &full[j], lane, GS_X);
      if (++c == a.nchunks) c = 0, ++tile;
    }
    int j = pro, s = 0;
    uint32_t ph = 0;
    for (; j < n; ++j) {
      int ok = 1;
      if (lane == 0) ok = gs_wait(&empty[s], ph, a, abort_flag) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      gs_issue<BITS>(a, tile, c, smem + s * Gm::bytes, &full[s], lane, GS_ANNOUNCE | GS_W | GS_X);
      if (++c == a.nchunks) c = 0, ++tile;
      if (++s == S) s = 0, ph ^= 1u;
    }
    if (lane == 0) *issued = j;
    return;
  }
  // ---------------- consumer warps
  pdl_wait();
  pdl_trigger();
  float acc[NB][4];
#pragma unroll
  for (int q = 0; q < NB; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
  int cur = t0, c = c0, s = 0;
  uint32_t ph = 0;
  const GsPart* pp = &a.parts[gs_part_of(a, cur)];
  bool mine = (cur - pp->tile0) * kGsConsumers + warp < pp->slices;
  for (int j = 0; j < n; ++j) {
    if (j > 0 && c == 0) {                              // a new tile starts with this item
      gs_tile_done<NB>(a, mode, cta, cur, acc, warp, lane, abort_flag, bcast, pstage + warp * 256);
#pragma unroll
      for (int q = 0; q < NB; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
      ++cur;
      pp = &a.parts[gs_part_of(a, cur)];
      mine = (cur - pp->tile0) * kGsConsumers + warp < pp->slices;
    }
    if (!*abort_flag && gs_wait(&full[s], ph, a, abort_flag)) {
      if (mine)
        gs_compute<BITS, NB>(smem + s * Gm::bytes, pp->bits, pp->group, warp, lane, acc, tc::smem_u32(cbt),
                             tc::smem_u32(nlt));
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
    if (++c == a.nchunks) c = 0;
    if (++s == S) s = 0, ph ^= 1u;
  }
  if (n > 0) gs_tile_done<NB>(a, mode, cta, cur, acc, warp, lane, abort_flag, bcast, pstage + warp * 256);
  if (*abort_flag && threadIdx.x == 0) {
    // a copy did not land in time: before the CTA exits, wait (bounded) for the producer and for
    // the last copy it issued into every stage
    const uint64_t deadline = globaltimer_ns() + a.wait_ns;
    while (*issued < 0 && globaltimer_ns() < deadline) {
    }
    const int done = *issued;
    for (int s = 0; s < S && done > 0; ++s) {
      const int lastj = done - 1 - ((done - 1 - s) % S + S) % S;
      if (lastj < 0) continue;
      while (!tc::mbar_try_wait(&full[s], (uint32_t)(lastj / S) & 1u) && globaltimer_ns() < deadline) {
      }
    }
  }
}

// act[t][i] = silu(gate) * up from the fp32 partial slots (PartialIn) of a gate/up output of
// width 2I, each rounded to bf16 first as a bf16 gate/up projection would be. inter == 0: the
// columns are [gate | up]; inter == 64: blocks of 64 gate columns then 64 up columns (the
// interleaved gate/up weight of the tcgen05 GEMM).
// Eight consecutive outputs per thread (I % 8 == 0): their gate and up columns are eight
// consecutive columns of one tile each, summed with 16-byte reads.
__global__ void silu_mul_partial_kernel(const PartialIn pi, int M, int I, int inter, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int per = I / 8;
  if (idx >= M * per) return;
  const int t = idx / per, i = (idx % per) * 8;
  const int gc = inter ? (i / inter) * 2 * inter + i % inter : i;
  const int uc = inter ? gc + inter : I + i;
  float g[8], u[8], o[8];
  partial_sum<8>(pi, t, gc, g);             // rounded to bf16 as a bf16 projection output would be
  partial_sum<8>(pi, t, uc, u);
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = __bfloat162float(__float2bfloat16_rn(g[k] / (1.f + __expf(-g[k])))) * u[k];
  *reinterpret_cast<bf16x8*>(out + (size_t)t * I + i) = pack8(o);
}

}  // namespace b200

using namespace b200;

// Stream-K plan of a group of matrices (N: 128 x the tiles over the parts, shared K): {kb, ctas, items}.
std::vector<int64_t> gguf_stream_plan(int64_t N, int64_t K, int64_t num_sms) {
  const int64_t tiles = N / 128, nchunks = K / 256, items = tiles * nchunks;
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(2 * num_sms, items));   // two CTAs per SM
  return {nchunks, ctas, items};
}

template <int BITS, int NB>
static void gs_launch(const GsArgs& a, int mode, int grid, cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    B200_CHECK_CUDA(cudaFuncSetAttribute(gguf_stream_kernel<BITS, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)GsGeom<BITS>::smem));
    attr = true;
  }
  launch_pdl(gguf_stream_kernel<BITS, NB>, dim3(grid), dim3(kGsThreads), GsGeom<BITS>::smem, stream, a, mode);
}

// x [M, K] bf16 (M <= 16); parts share K, each N % 16 == 0 (% 128 for partial outputs); the
// group's columns are the parts' rows in order. mode 0 bf16 / 1 fp32 into out[t][ldo]; 2 fp32 partial slots into out
// ([slots][M][ldo], 128-column tiles); 4 bf16 push into the flag-free slots at push_ptrs (host
// int64 [world]) or through mc_ptr. ws / counters: per-device scratch (fp32 >= ctas * 4096;
// int32 >= tiles + 1, zero on first use, the last word records error 190 when a copy did not
// land within the wait deadline: wait_ms, or the process-wide flag deadline when 0).
std::vector<int64_t> gguf_stream(torch::Tensor x, std::vector<torch::Tensor> codes, std::vector<torch::Tensor> metas,
                                 std::vector<int64_t> ns, std::vector<int64_t> bits, std::vector<int64_t> groups,
                                 int64_t mode, torch::Tensor out, int64_t ldo, torch::Tensor ws, torch::Tensor counters,
                                 torch::Tensor push_ptrs, int64_t mc_ptr, int64_t num_sms, int64_t wait_ms,
                                 int64_t table) {
  const int M = x.size(0), K = x.size(1);
  const int np = (int)codes.size();
  TORCH_CHECK(np >= 1 && np <= kGsMaxParts && metas.size() == codes.size() && ns.size() == codes.size() &&
                  bits.size() == codes.size() && groups.size() == codes.size(),
              "1..4 parts with codes, scales, N, bits and group each");
  TORCH_CHECK(M >= 1 && M <= 16, "gguf_stream serves decode batches of 1..16 tokens");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && (x.stride(0) % 8) == 0 &&
                  (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) == 0,
              "x: bf16 rows, 16-byte aligned");
  TORCH_CHECK(K % 256 == 0, "K must be a multiple of 256");
  GsArgs a{};
  int64_t ntot = 0;
  int tiles = 0;
  bool any8 = false;
  for (int p = 0; p < np; ++p) {
    TORCH_CHECK(ns[p] % 16 == 0, "N must be a multiple of 16");
    TORCH_CHECK(mode != GS_PARTIAL || ns[p] % 128 == 0, "partial outputs need N % 128 == 0 (128-column tiles)");
    TORCH_CHECK(bits[p] == 4 || bits[p] == 5 || (bits[p] == 8 && (groups[p] == 16 || groups[p] == 32)) ||
                    (bits[p] == 2 && (groups[p] == 32 || groups[p] == 64 || groups[p] == 128 || groups[p] == 256)),
                "4-bit codes (group 32; 5: through the IQ4 table), 8-bit codes with group 16 or 32, or E8 codes "
                "with group 32..256");
    TORCH_CHECK((bits[p] == 2) == (bits[0] == 2), "E8 parts cannot share a launch with other code types");
    const auto cp = reinterpret_cast<uintptr_t>(codes[p].data_ptr()), mp = reinterpret_cast<uintptr_t>(metas[p].data_ptr());
    TORCH_CHECK(cp % 16 == 0 && mp % 16 == 0, "codes and scales must be 16-byte aligned for the bulk copies");
    TORCH_CHECK(codes[p].numel() * codes[p].element_size() >= ns[p] * K / (bits[p] == 2 ? 8 : bits[p] == 8 ? 1 : 2),
                "codes too small");
    if (bits[p] == 2)
      TORCH_CHECK(metas[p].numel() * metas[p].element_size() >= ns[p] * (K / groups[p]) * 8, "E8 scales too small");
    a.parts[p].codes = reinterpret_cast<const uint32_t*>(cp);
    a.parts[p].meta = reinterpret_cast<const uint32_t*>(mp);
    a.parts[p].tile0 = tiles;
    a.parts[p].slices = (int)(ns[p] / 16);
    a.parts[p].col0 = (int)ntot;
    a.parts[p].bits = (int)bits[p];
    a.parts[p].group = (int)groups[p];
    any8 = any8 || bits[p] == 8;
    ntot += ns[p];
    tiles += (int)((ns[p] + 127) / 128);
  }
  auto plan = gguf_stream_plan((int64_t)tiles * 128, K, num_sms);
  a.nparts = np;
  bool any5 = false;
  for (int p = 0; p < np; ++p) any5 = any5 || bits[p] == 5;
  if (bits[0] == 2 || any5) {
    TORCH_CHECK(table != 0 && table % 16 == 0,
                "E8 parts need the codebook table ([256][4] bf16 pairs), IQ4 parts the pair table ([256])");
    a.table = reinterpret_cast<const uint32_t*>(table);
  }
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = (int)x.stride(0);
  a.M = M;
  a.K = K;
  a.nchunks = (int)plan[0];
  a.ctas = (int)plan[1];
  a.items = (int)plan[2];
  TORCH_CHECK((uint64_t)a.items * (uint64_t)(a.ctas + 1) < (1ull << 32), "matrix group too large for one launch");
  a.tiles = tiles;
  a.ldo = (int)ldo;
  a.out = out.numel() ? out.data_ptr() : nullptr;
  a.wait_ns = wait_ms > 0 ? (uint64_t)wait_ms * 1000000ull : flag_wait_ns();
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= (int64_t)a.ctas * 4096, "workspace too small");
  TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= a.tiles + 1, "counters too small");
  a.ws = ws.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.err = counters.data_ptr<int>() + (counters.numel() - 1);     // the last word: error code
  if (mode == GS_PARTIAL) {
    // slots per 128-column tile: at most ceil(kb * ctas / items) + 1
    const int64_t slots = (a.nchunks * (int64_t)a.ctas + a.items - 1) / a.items + 1;
    TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() >= slots * M * ldo && ldo >= ntot,
                "partial buffer too small");
    a.part_slot = (long long)M * ldo;
  } else if (mode == GS_PUSH) {
    const int world = push_ptrs.numel();
    TORCH_CHECK(world >= 1 && world <= 8 && push_ptrs.device().is_cpu(), "push pointers: host int64 [world]");
    for (int r = 0; r < world; ++r) {
      a.push[r] = reinterpret_cast<__nv_bfloat16*>(push_ptrs.data_ptr<int64_t>()[r]);
      TORCH_CHECK(reinterpret_cast<uintptr_t>(a.push[r]) % 16 == 0, "push slots must be 16-byte aligned");
    }
    a.world = world;
    a.mc = reinterpret_cast<__nv_bfloat16*>(mc_ptr);
    TORCH_CHECK(ldo % 8 == 0, "push row stride must be a multiple of 8");
  } else {
    TORCH_CHECK(mode == GS_BF16 || mode == GS_F32, "mode: 0 bf16, 1 fp32, 2 partial, 4 push");
    TORCH_CHECK(out.scalar_type() == (mode == GS_F32 ? at::kFloat : at::kBFloat16) && out.numel() >= (int64_t)M * ldo &&
                    ldo >= ntot,
                "output type or size");
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  if (bits[0] == 2) {
    if (M <= 8) gs_launch<2, 1>(a, (int)mode, a.ctas, stream);
    else gs_launch<2, 2>(a, (int)mode, a.ctas, stream);
  } else if (any8) {
    if (M <= 8) gs_launch<8, 1>(a, (int)mode, a.ctas, stream);
    else gs_launch<8, 2>(a, (int)mode, a.ctas, stream);
  } else {
    if (M <= 8) gs_launch<4, 1>(a, (int)mode, a.ctas, stream);
    else gs_launch<4, 2>(a, (int)mode, a.ctas, stream);
  }
  return plan;
}

// out [M, I] = silu(gate) * up from the fp32 partial slots of a gate/up output (width 2I; inter
// 0: [gate | up], 64: 64-column gate/up blocks).
void silu_mul_partial(torch::Tensor part, int64_t kb, int64_t ctas, int64_t total, int64_t tile, int64_t M, int64_t I,
                      torch::Tensor out, int64_t inter) {
  TORCH_CHECK(part.scalar_type() == at::kFloat && out.scalar_type() == at::kBFloat16 && out.is_contiguous());
  TORCH_CHECK(tile == 16 || tile == 128, "partial tiles are 16 or 128 columns wide");
  TORCH_CHECK(inter == 0 || (inter == 64 && I % 64 == 0), "inter: 0 or 64 (I % 64 == 0)");
  TORCH_CHECK(I % 8 == 0, "I must be a multiple of 8");
  TORCH_CHECK((uint64_t)((2 * I + tile - 1) / tile) * (uint64_t)kb * (uint64_t)ctas < (1ull << 32),
              "stream-K plan too large for 32-bit slot arithmetic");
  PartialIn pi{part.data_ptr<float>(), (int)kb, (int)ctas, (long long)total, (int)M, (int)(2 * I), (int)tile};
  const int n = (int)(M * I / 8);
  launch_pdl(silu_mul_partial_kernel, dim3((n + 127) / 128), dim3(128), 0, at::cuda::getCurrentCUDAStream(), pi, (int)M,
             (int)I, (int)inter, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
}
