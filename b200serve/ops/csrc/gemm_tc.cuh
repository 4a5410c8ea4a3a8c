// Persistent tcgen05/TMEM GEMM for the decoder's linear layers:
//   out[m, n] = sum_k act[m, k] * W[n, k]  (+ bias[n]) (+ residual[m, n])
// with fused epilogues (bf16 store, fp32 store for logits, SwiGLU on the
// 64-row interleaved gate/up layout).
//
// The weight is the MMA "A" operand (128 output features per tile = the 128
// TMEM lanes) and the activations are the MMA "B" operand (BN tokens per tile =
// BN TMEM columns), so a decode batch of 16..256 tokens maps onto the MMA N
// dimension and every CTA streams weight tiles at full width.
//
// Roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA
// issuer (one elected thread), warps 2..5 = epilogue (warp w reads TMEM lanes
// 32*(w%4) .. 32*(w%4)+31). Shared memory holds STAGES stages of
// [W tile 128x64 | act tile BNx64] in the 128-byte-swizzled K-major layout
// written by TMA; the accumulator is double-buffered in TMEM so the epilogue of
// one work unit overlaps the main loop of the next.
//
// Work units are (n tile, m tile, k split). With fewer tiles than SMs the K
// loop is split; every split writes an fp32 partial tile to a workspace and
// the last CTA to finish a tile (counter per tile) sums the partials and runs
// the epilogue.
//
// Reference kernels restated: matmul.wgsl:133,201 (matmul_bt_bf16, C = A B^T).
#pragma once
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "tc_primitives.cuh"

namespace b200 {

enum GemmEpi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2, EPI_PUSH = 3, EPI_QKV = 4, EPI_PARTIAL = 5 };

constexpr int kMaxPeers = 8;

struct GemmParams {
  int M, N, K;                  // tokens, output features, reduction
  int w_packed;                 // 1: W stored tile-contiguous [n_tile][k_block][128][64]
  // grouped (mixture-of-experts) mode: expert e owns A rows [g_offsets[e], g_offsets[e+1]) of the
  // expert-sorted activations and output rows with the same indices; its weight is the e-th
  // [N, K] block of a packed [E][n_tiles][k_blocks][128][64] tensor. Units = E x m_tiles x n_tiles x splits.
  int grouped;
  const int* g_offsets;
  int g_E;
  int n_tiles, m_tiles, splits, kb_per_split, kb_total, units;
  int stages;                   // shared-memory ring depth (set by the host launcher)
  int cluster_red;              // 1: the splits of a tile form one cluster and reduce through DSMEM
  // EPI_QKV: the fused QKV projection's tile n is head slot n (head_dim 128): bias, per-head
  // q/k RMSNorm, rotate-half RoPE, then q -> q_out [T][nq][128], k/v -> paged bf16 caches
  int qkv_nq, qkv_nkv;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* cos_sin;         // [max_pos][128] = cos(64) | sin(64)
  const int* positions;
  const int* slots;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;       // [blocks][nkv][16][128]
  __nv_bfloat16* v_cache;
  float qkv_eps;
  // EPI_PUSH as reduce-scatter: token row t goes only to rank t / rs_rows, at row t % rs_rows
  int rs_rows;
  // all-gather -> GEMM: the activation rows arrive from peers; the producer waits until
  // ag_flags[0..ag_n) all hold *ag_epoch before loading any activation tile
  const int* ag_flags;
  int ag_n;
  const int* ag_epoch;
  unsigned long long ag_wait_ns;  // deadline of the all-gather flag wait
  const uint8_t* w_ptr;         // packed weight base (L2 prefetch), or null
  int l2_prefetch_blocks;       // weight tiles per CTA prefetched into L2 before the dependency wait
  void* out;                    // bf16 or fp32, row stride ldo (elements)
  int ldo;
  const __nv_bfloat16* bias;    // [N] or null
  const __nv_bfloat16* residual;  // [M, ldr] or null
  int ldr;
  float* ws;                    // [splits, m_tiles*BN, N] fp32 (splits > 1)
  int* counters;                // [m_tiles * n_tiles], zero on entry and on exit
  int* err;
  // EPI_PUSH: bf16 tile stored to every rank's receive slot, then per-rank flags raised
  int world;
  __nv_bfloat16* push_dst[kMaxPeers];   // slot base on rank r (row stride ldo)
  int* push_flag[kMaxPeers];            // flag word on rank r for (site, this rank)
  const int* epoch;                     // this step's epoch (device)
  int* tile_done;                       // local counter of pushed tiles, zero on entry and exit
  // EPI_PUSH without flags: the receive slots hold the sentinel bf16 pattern 0xFFFF until data
  // lands, and the consumer polls the data itself (no system fence, no tile counter, no flag
  // stores). The kernel lets its dependent launch only after its own prerequisites completed,
  // so a consumer that skips griddepcontrol.wait still runs after everything before this GEMM.
  int lamport;
  // flag-free push through an NVLink multicast object (NVLS): one multimem.st per 16 bytes reaches
  // this rank's slot on every GPU of the group (row stride ldo); null = one P2P store per rank
  __nv_bfloat16* mc_dst;
  // EPI_PUSH as the expert-parallel combine: output row r carries comb_meta[r] = (home rank,
  // pair p = t * comb_k + j, routing weight bits); the row is scaled by the weight and stored at
  // row j * comb_rows + t of the home rank's slot (push_dst[home]). push_tiles: number of tiles
  // that publish (the grouped GEMM's non-empty tiles); 0 = m_tiles * n_tiles.
  const int4* comb_meta;
  int comb_k, comb_rows, push_tiles;
  // stream-K with partial sums reduced by the consumer (EPI_PARTIAL, m_tiles == 1): CTA c streams the
  // flattened k-blocks [c*sk_total/G, (c+1)*sk_total/G) of the n tiles (sk_total = n_tiles*kb_total,
  // G = gridDim.x), cut at tile boundaries; each piece's fp32 partial goes to
  // part[slot][M][N] with slot = c - (first CTA touching the tile). No counters, no fixup pass.
  int streamk;
  long long sk_total;
  float* part;
  // > 1: raster the (m tile, n tile) grid in bands of `raster` m tiles (prefill): consecutive
  // units walk down a band for one n tile, so a wave of CTAs shares its activation and weight
  // tiles in L2 instead of sweeping every weight tile once per m tile
  int raster;
  // optional per-CTA timeline (globaltimer ns): [cta][8] = entry, setup done, first TMA issued,
  // first stage landed, last MMA committed, epilogue done, exit (thread 0), exit (thread 32)
  unsigned long long* trace;
};

__device__ __forceinline__ void trace_mark(const GemmParams& p, int slot) {
  if (p.trace && blockIdx.x < 2048) p.trace[blockIdx.x * 8 + slot] = globaltimer_ns();
}


template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int W_BYTES = BM * BK * 2;
  static constexpr int A_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = W_BYTES + A_BYTES;
  // the ring depth is a launch parameter (GemmParams::stages, 2..MAX_STAGES); the barrier
  // block is sized for MAX_STAGES so its layout does not depend on it
  static constexpr int MAX_STAGES = 12;
  static constexpr int TMEM_COLS = (2 * BN) < 32 ? 32 : 2 * BN;
  // epilogue exchange buffer: 64 rows x 17 (SwiGLU, push staging); the QKV epilogue needs 128 rows
  static constexpr int xchg_floats(int epi) { return epi == 4 ? 128 * 17 : 64 * 17; }
  static constexpr size_t smem(int stages, int epi) {
    return 1024 + (size_t)stages * STAGE_BYTES + xchg_floats(epi) * 4 + 256;
  }
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Final epilogue for 16 consecutive tokens [t0, t0+16) of this thread's feature row.
template <int EPI>
__device__ __forceinline__ void epilogue_store(const GemmParams& p, float* v, int row, int n_tile, int t0, int t_end,
                                               float* xchg, int quad, int lane) {
  if constexpr (EPI == EPI_SWIGLU) {
    // rows 0..63 hold gate features, rows 64..127 the up features of the same 64 columns
    if (quad >= 2) {
#pragma unroll
      for (int j = 0; j < 16; ++j) xchg[((quad - 2) * 32 + lane) * 17 + j] = v[j];
    }
    epi_bar();
    if (quad < 2) {
      const int col = n_tile * 64 + quad * 32 + lane;
      const int half_n = p.N / 2;
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = t0 + j;
        if (t < t_end && col < half_n) {
          const float g = v[j];
          const float u = xchg[(quad * 32 + lane) * 17 + j];
          const float sg = __bfloat162float(__float2bfloat16_rn(g / (1.f + __expf(-g))));
          // gate and up are rounded to bf16 first, as a bf16 framework would store them
          out[(size_t)t * p.ldo + col] =
              __float2bfloat16_rn(sg * __bfloat162float(__float2bfloat16_rn(u)));
        }
      }
    }
    epi_bar();
  } else if constexpr (EPI == EPI_PUSH) {
    // stage the 16-token x 128-feature chunk as bf16 rows, then push 16-byte vectors:
    // consecutive threads cover consecutive 16-byte pieces of a token row on every peer
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(xchg);      // [16][136]
    {
      const int col = n_tile * 128 + row;
      const float b = (p.bias && col < p.N) ? __bfloat162float(p.bias[col]) : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float scale = p.comb_meta ? (t0 + j < t_end ? __int_as_float(p.comb_meta[t0 + j].z) : 0.f) : 1.f;
        __nv_bfloat16 h = __float2bfloat16_rn((v[j] + b) * scale);
        // 0xFFFF marks an empty receive slot; a NaN with that payload is stored as 0x7FFF
        if (__bfloat16_as_ushort(h) == 0xFFFFu) h = __ushort_as_bfloat16((unsigned short)0x7FFFu);
        xs[j * 136 + row] = h;
      }
    }
    epi_bar();
    const int tid = threadIdx.x - 64;                                    // 0..127 over the epilogue warps
#pragma unroll
    for (int rep = 0; rep < 2; ++rep) {
      const int piece = tid + rep * 128;                                 // 16 tokens x 16 pieces of 8 features
      const int tok = piece >> 4, chunk = piece & 15;
      const int t = t0 + tok, col = n_tile * 128 + chunk * 8;
      if (t < t_end && col < p.N) {
        const uint4 val = *reinterpret_cast<const uint4*>(xs + tok * 136 + chunk * 8);
        if (p.comb_meta) {
          const int4 m = p.comb_meta[t];
          const int home = m.x, pair = m.y;
          const size_t r = (size_t)(pair % p.comb_k) * p.comb_rows + pair / p.comb_k;
          *reinterpret_cast<uint4*>(p.push_dst[home] + r * p.ldo + col) = val;
        } else if (p.mc_dst) {
          __nv_bfloat16* d = p.mc_dst + (size_t)t * p.ldo + col;
          asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};"
                       ::"l"(d), "r"(val.x), "r"(val.y), "r"(val.z), "r"(val.w) : "memory");
        } else if (p.rs_rows > 0) {
          const int owner = t / p.rs_rows;
          *reinterpret_cast<uint4*>(p.push_dst[owner] + (size_t)(t - owner * p.rs_rows) * p.ldo + col) = val;
        } else {
          for (int r = 0; r < p.world; ++r)
            *reinterpret_cast<uint4*>(p.push_dst[r] + (size_t)t * p.ldo + col) = val;
        }
      }
    }
    epi_bar();
  } else if constexpr (EPI == EPI_QKV) {
    // this thread: dim `row` of head slot n_tile, 16 tokens; xchg holds [128 rows][17]
    const int h = n_tile, d = row;
    const bool is_q = h < p.qkv_nq, is_k = !is_q && h < p.qkv_nq + p.qkv_nkv;
    float x[16];
    const float b = p.bias ? __bfloat162float(p.bias[h * 128 + d]) : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = __bfloat162float(__float2bfloat16_rn(v[j] + b));
    if (is_q || is_k) {
      const __nv_bfloat16* nw = is_q ? p.q_norm : p.k_norm;
      if (nw) {
        // per-token sum of squares over the 128 dims: warp sums, then the 4 warps through xchg
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float s2 = warp_sum(x[j] * x[j]);
          if (lane == 0) xchg[quad * 16 + j] = s2;
        }
        epi_bar();
        const float wd = __bfloat162float(nw[d]);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float tot = xchg[j] + xchg[16 + j] + xchg[32 + j] + xchg[48 + j];
          const float inv = rsqrtf(tot / 128.f + p.qkv_eps);
          x[j] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(x[j] * inv)) * wd));
        }
        epi_bar();
      }
      // rotate-half RoPE: dim d pairs with d ^ 64 (thread row ^ 64). The 16 positions and
      // their cos/sin are loaded up front (independent loads, one round trip).
      const int f = d & 63;
      float cv[16], sv[16];
      {
        int pos[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pos[j] = p.positions[min(t0 + j, t_end - 1)];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float* cs = p.cos_sin + (size_t)pos[j] * 128;
          cv[j] = cs[f];
          sv[j] = cs[64 + f];
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) xchg[d * 17 + j] = x[j];
      epi_bar();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float partner = xchg[(d ^ 64) * 17 + j];
        x[j] = d < 64 ? x[j] * cv[j] - partner * sv[j] : x[j] * cv[j] + partner * sv[j];
      }
      epi_bar();
    }
    if (is_q) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (t0 + j < t_end) p.q_out[((size_t)(t0 + j) * p.qkv_nq + h) * 128 + d] = __float2bfloat16_rn(x[j]);
    } else {
      int sl[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) sl[j] = t0 + j < t_end ? p.slots[t0 + j] : -1;
      const int kvh = is_k ? h - p.qkv_nq : h - p.qkv_nq - p.qkv_nkv;
      __nv_bfloat16* cache = is_k ? p.k_cache : p.v_cache;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (sl[j] >= 0) {
          const size_t r = ((size_t)(sl[j] >> 4) * p.qkv_nkv + kvh) * 16 + (sl[j] & 15);
          cache[r * 128 + d] = __float2bfloat16_rn(x[j]);
        }
      }
    }
  } else {
    const int col = n_tile * 128 + row;
    if (col >= p.N) return;
    const float b = p.bias ? __bfloat162float(p.bias[col]) : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int t = t0 + j;
      if (t >= t_end) break;
      float x = v[j] + b;
      if constexpr (EPI == EPI_F32) {
        reinterpret_cast<float*>(p.out)[(size_t)t * p.ldo + col] = x;
      } else {
        if (p.residual) x = __bfloat162float(__float2bfloat16_rn(x)) + __bfloat162float(p.residual[(size_t)t * p.ldr + col]);
        reinterpret_cast<__nv_bfloat16*>(p.out)[(size_t)t * p.ldo + col] = __float2bfloat16_rn(x);
      }
    }
  }
}

struct Unit {
  int n_tile, m_tile, split, tile;   // tile: index for split-K counters / push accounting
  int a_row0, m_lim, w_tile_base;    // first activation row, rows valid, packed weight tile row base
  bool empty;
};

__device__ __forceinline__ Unit decode_unit(const GemmParams& p, int u, int BN) {
  Unit x;
  x.split = u % p.splits;
  x.tile = u / p.splits;
  x.n_tile = x.tile % p.n_tiles;
  const int rest = x.tile / p.n_tiles;
  if (!p.grouped && p.raster > 1) {
    const int band = p.raster * p.n_tiles;                 // tiles per band of `raster` m tiles
    const int b = x.tile / band, in = x.tile % band;
    const int rows = min(p.raster, p.m_tiles - b * p.raster);
    x.m_tile = b * p.raster + in % rows;
    x.n_tile = in / rows;
    x.a_row0 = x.m_tile * BN;
    x.m_lim = p.M - x.a_row0;
    x.w_tile_base = x.n_tile;
    x.empty = false;
  } else if (!p.grouped) {
    x.m_tile = rest;
    x.a_row0 = x.m_tile * BN;
    x.m_lim = p.M - x.a_row0;
    x.w_tile_base = x.n_tile;
    x.empty = false;
  } else {
    x.m_tile = rest % p.m_tiles;
    const int e = rest / p.m_tiles;
    const int r0 = __ldg(p.g_offsets + e), r1 = __ldg(p.g_offsets + e + 1);
    x.a_row0 = r0 + x.m_tile * BN;
    x.m_lim = r1 - x.a_row0;
    x.w_tile_base = e * p.n_tiles + x.n_tile;
    x.empty = x.m_lim <= 0;
  }
  return x;
}

// One piece of work of a CTA: a (tile, k-range) with the partial-sum slot (stream-K) or the split.
struct Work {
  Unit x;
  int kb0, kb1, slot;
};

__device__ __forceinline__ long long sk_begin(const GemmParams& p, long long c) {
  return c * p.sk_total / (long long)gridDim.x;
}
// first CTA whose range touches tile t: the largest c with sk_begin(c) <= t * kb_total
__device__ __forceinline__ int sk_first_cta(const GemmParams& p, int t) {
  const long long x = ((long long)t * p.kb_total + 1) * (long long)gridDim.x;
  return (int)((x + p.sk_total - 1) / p.sk_total) - 1;
}

// The sequence of work pieces of this CTA; every role (producer, MMA issuer, epilogue) walks
// the same sequence, so they agree on stage and accumulator order.
struct WorkIter {
  int u;
  long long g, g_end;
  __device__ __forceinline__ explicit WorkIter(const GemmParams& p) {
    u = blockIdx.x;
    g = p.streamk ? sk_begin(p, blockIdx.x) : 0;
    g_end = p.streamk ? sk_begin(p, (long long)blockIdx.x + 1) : 0;
  }
  __device__ __forceinline__ bool next(const GemmParams& p, int BN, Work& w) {
    if (p.streamk) {
      if (g >= g_end) return false;
      const int t = (int)(g / p.kb_total);
      const long long seg_end = min(g_end, (long long)(t + 1) * p.kb_total);
      w.x.n_tile = t; w.x.m_tile = 0; w.x.split = 0; w.x.tile = t;
      w.x.a_row0 = 0; w.x.m_lim = p.M; w.x.w_tile_base = t; w.x.empty = false;
      w.kb0 = (int)(g - (long long)t * p.kb_total);
      w.kb1 = (int)(seg_end - (long long)t * p.kb_total);
      w.slot = (int)blockIdx.x - sk_first_cta(p, t);
      g = seg_end;
      return true;
    }
    if (u >= p.units) return false;
    w.x = decode_unit(p, u, BN);
    w.kb0 = w.x.split * p.kb_per_split;
    w.kb1 = min(p.kb_total, w.kb0 + p.kb_per_split);
    w.slot = w.x.split;
    u += gridDim.x;
    return true;
  }
};

// TMA coordinates of the weight tile (n_tile, k block kb) in the plain [N, K]
// layout or the tile-contiguous packed layout (each 128x64 tile one 16 KB run).
__device__ __forceinline__ int w_x(const GemmParams& p, int kb) { return p.w_packed ? 0 : kb * 64; }
__device__ __forceinline__ int w_y(const GemmParams& p, int w_tile, int kb) {
  return p.w_packed ? (w_tile * p.kb_total + kb) * 128 : w_tile * 128;
}

// All-gather -> GEMM: spin (bounded by ag_wait_ns) until every rank published this step's epoch
// for the gathered activation rows, then order the async proxy (TMA) after those acquires.
__device__ __forceinline__ bool wait_ag_flags(const GemmParams& p, volatile int* abort_flag, int* err) {
  const int e = *p.ag_epoch;
  const uint64_t deadline = globaltimer_ns() + p.ag_wait_ns;
  for (int r = 0; r < p.ag_n; ++r) {
    uint32_t it = 0;
    while (true) {
      int v;
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.ag_flags + r) : "memory");
      if (v == e) break;
      if ((++it & 1023u) == 0 && globaltimer_ns() > deadline) {
        atomicExch(err, 120 + r);
        *abort_flag = 1;
        return false;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");   // acquire side of the writers' fence + relaxed flags
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// EPI_PUSH: after a tile's stores reached every peer, count it; the CTA that
// completes the last tile raises flag[r] = epoch on every rank (after a system-scope fence).
__device__ __forceinline__ void publish_tile(const GemmParams& p, int* scratch) {
  __threadfence_system();
  epi_bar();
  if (threadIdx.x == 64) {
    const int total = p.push_tiles > 0 ? p.push_tiles : p.m_tiles * p.n_tiles;
    const int old = atomicAdd(p.tile_done, 1);
    if (old == total - 1) {
      *p.tile_done = 0;
      __threadfence_system();
      const int e = *p.epoch;
      // one system-scope fence above orders every pushed tile before the flags; the flag
      // stores themselves are relaxed so they pipeline instead of each waiting for the
      // previous one's acknowledgement (a release store per peer serialises ~2.5 us each)
      for (int r = 0; r < p.world; ++r)
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p.push_flag[r]), "r"(e) : "memory");
    }
  }
  epi_bar();
}

// Cluster split-K: every CTA of the cluster (one K split of the same tile) has staged its fp32
// partial tile [BN][128] at the start of its shared memory. CTA rank r sums token columns
// [r*ceil(BN/S), ...) over the S partials through distributed shared memory and runs the final
// epilogue for them, so the tile is reduced in parallel without a global workspace round trip.
template <int BN, int EPI>
__device__ __forceinline__ void cluster_reduce_store(const GemmParams& p, const uint8_t* red_smem, float* xchg,
                                                     int row, int quad, int lane) {
  const Unit x = decode_unit(p, blockIdx.x, BN);
  const int S = p.splits;
  const int r = (int)tc::cluster_ctarank();
  const int cpc = (BN + S - 1) / S;
  const int c_lo = r * cpc, c_hi = min(BN, c_lo + cpc);
  const int t_tile_end = x.a_row0 + min(x.m_lim, BN);
  const uint32_t base = tc::smem_u32(red_smem);
  for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
    for (int sp = 0; sp < S; ++sp) {
      const uint32_t rb = tc::map_shared_rank(base, (uint32_t)sp);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c0 + j < c_hi) v[j] += tc::ld_shared_cluster_f32(rb + (uint32_t)(((c0 + j) * 128 + row) * 4));
    }
    epilogue_store<EPI>(p, v, row, x.n_tile, x.a_row0 + c0, min(t_tile_end, x.a_row0 + c_hi), xchg, quad, lane);
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 2)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                   const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  const int STAGES = p.stages;
  constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_w = smem;
  uint8_t* s_a = smem + STAGES * Cfg::W_BYTES;
  float* xchg = reinterpret_cast<float*>(s_a + STAGES * Cfg::A_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(xchg + Cfg::xchg_floats(EPI));
  uint64_t* empty = full + Cfg::MAX_STAGES;
  uint64_t* tfull = empty + Cfg::MAX_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_slot + 2));
  (void)last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = p.err;  // never null: the host passes its error word
  if (threadIdx.x == 0) trace_mark(p, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { tc::mbar_init(&full[s], 1); tc::mbar_init(&empty[s], 1); }
    for (int i = 0; i < 2; ++i) { tc::mbar_init(&tfull[i], 1); tc::mbar_init(&tempty[i], 4); }
    tc::mbar_init(mma_done, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tm_w);
    tc::prefetch_tmap(&tm_a);
  }
  __syncwarp();
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) trace_mark(p, 1);
  if (!p.lamport) pdl_trigger();
  if (warp != 0) {
    pdl_wait();
    if (p.lamport) pdl_trigger();   // the dependent may start only after our prerequisites completed
  }

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const uint64_t pol_w = tc::policy_evict_first(), pol_a = tc::policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      // Weights never depend on the previous kernel: stream the first stages of W
      // while that kernel finishes, then wait for it before loading activations.
      WorkIter it(p);
      Work w;
      bool have = it.next(p, BN, w);
      int pre = 0;
      if (have && !p.grouped && !w.x.empty) {
        pre = min(w.kb1 - w.kb0, STAGES);
        for (int i = 0; i < pre; ++i) {
          tc::mbar_arrive_expect_tx(&full[i], Cfg::STAGE_BYTES);
          tc::tma_load_2d(s_w + i * Cfg::W_BYTES, &tm_w, &full[i], w_x(p, w.kb0 + i),
                          w_y(p, w.x.w_tile_base, w.kb0 + i), pol_w);
        }
        // Stream further weight tiles of this CTA's work into L2 while the previous kernel
        // finishes (tile-packed weights: each 128 x 64 tile is one contiguous 16 KB run).
        if (p.w_ptr && p.l2_prefetch_blocks > 0) {
          int budget = p.l2_prefetch_blocks;
          WorkIter it2(p);
          Work y;
          bool first_piece = true;
          while (budget > 0 && it2.next(p, BN, y)) {
            for (int kb = y.kb0 + (first_piece ? pre : 0); kb < y.kb1 && budget > 0; ++kb, --budget)
              tc::prefetch_l2(p.w_ptr + ((size_t)y.x.w_tile_base * p.kb_total + kb) * (size_t)Cfg::W_BYTES,
                              Cfg::W_BYTES);
            first_piece = false;
          }
        }
        pdl_wait();
        if (p.ag_flags) wait_ag_flags(p, abort_flag, err);
        for (int i = 0; i < pre; ++i)
          tc::tma_load_2d(s_a + i * Cfg::A_BYTES, &tm_a, &full[i], (w.kb0 + i) * 64, w.x.a_row0, pol_a);
        trace_mark(p, 2);
        stage = pre % STAGES;
        phase = pre == STAGES ? 1 : 0;
      } else {
        pdl_wait();
        if (p.ag_flags) wait_ag_flags(p, abort_flag, err);
      }
      bool first_piece = true;
      for (; have && !*abort_flag; have = it.next(p, BN, w)) {
        const int kb_start = w.kb0 + (first_piece ? pre : 0);
        first_piece = false;
        if (w.x.empty) continue;
        for (int kb = kb_start; kb < w.kb1; ++kb) {
          if (!tc::mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, err, 1)) break;
          tc::mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tc::tma_load_2d(s_w + stage * Cfg::W_BYTES, &tm_w, &full[stage], w_x(p, kb), w_y(p, w.x.w_tile_base, kb), pol_w);
          tc::tma_load_2d(s_a + stage * Cfg::A_BYTES, &tm_a, &full[stage], kb * 64, w.x.a_row0, pol_a);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();   // lanes 1..31 wait for the producer lane: the CTA barrier below is warp-aligned
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase[2] = {0, 0};
      int acc = 0;
      bool first = true;
      WorkIter it(p);
      Work w;
      while (!*abort_flag && it.next(p, BN, w)) {
        if (w.x.empty) continue;
        const int kb0 = w.kb0, kb1 = w.kb1;
        if (!tc::mbar_wait_bounded(&tempty[acc], acc_phase[acc] ^ 1, abort_flag, err, 2)) break;
        if (first) {
          tc::mbar_wait_bounded(&full[stage], phase, abort_flag, err, 3);
          trace_mark(p, 3);
          first = false;
        }
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!tc::mbar_wait_bounded(&full[stage], phase, abort_flag, err, 3)) break;
          tc::tc_fence_after();
          const uint64_t a0 = tc::sw128_kmajor_desc(tc::smem_u32(s_w + stage * Cfg::W_BYTES));
          const uint64_t b0 = tc::sw128_kmajor_desc(tc::smem_u32(s_a + stage * Cfg::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // 16 bf16 = 32 bytes along K per MMA: +2 in the 16-byte-unit address field
            tc::mma_bf16(d_tmem, a0 + 2 * kk, b0 + 2 * kk, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc::mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        tc::mma_commit(&tfull[acc]);
        acc_phase[acc] ^= 1;
        acc ^= 1;
      }
      trace_mark(p, 4);
      // no tcgen05.mma may still be running when TMEM is released below
      tc::mma_commit(mma_done);
      volatile int never = 0;
      tc::mbar_wait_bounded(mma_done, 0, &never, err, 5);
    }
    __syncwarp();   // reconverge before the warp-aligned CTA barrier
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    uint32_t acc_phase[2] = {0, 0};
    int acc = 0;
    const int total_tiles = p.units / p.splits;
    WorkIter it(p);
    Work w;
    while (!*abort_flag && it.next(p, BN, w)) {
      const Unit& x = w.x;
      if (x.empty) continue;
      const int t_end = x.a_row0 + min(x.m_lim, BN);
      if (!tc::mbar_wait_bounded(&tfull[acc], acc_phase[acc], abort_flag, err, 4)) break;
      tc::tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      if constexpr (EPI == EPI_PARTIAL) {
        // fp32 partial of this piece -> part[slot][t][col] (consecutive lanes: consecutive columns)
        float* dst = p.part + (size_t)w.slot * p.M * p.N;
        const int col = x.n_tile * 128 + row;
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tc::tmem_ld16(t_row + c0, v);
          if (col < p.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (x.a_row0 + c0 + j < t_end) dst[(size_t)(x.a_row0 + c0 + j) * p.N + col] = v[j];
          }
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[acc]);
      } else if (p.splits == 1) {
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tc::tmem_ld16(t_row + c0, v);
          epilogue_store<EPI>(p, v, row, x.n_tile, x.a_row0 + c0, t_end, xchg, quad, lane);
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[acc]);
        if constexpr (EPI == EPI_PUSH) {
          if (!p.lamport) publish_tile(p, last_flag);
        }
      } else if (p.cluster_red) {
        // partial tile -> this CTA's shared memory (the drained stage ring), reduced after the
        // cluster barrier below
        float* red = reinterpret_cast<float*>(smem);
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tc::tmem_ld16(t_row + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) red[(c0 + j) * 128 + row] = v[j];
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[acc]);
      } else {
        // partial tile -> workspace [split][tile][BN][128] (coalesced over the 128 features)
        float* ws_mine = p.ws + ((size_t)x.split * total_tiles + x.tile) * BN * 128;
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tc::tmem_ld16(t_row + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) ws_mine[(size_t)(c0 + j) * 128 + row] = v[j];
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[acc]);
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const int old = atomicAdd(&p.counters[x.tile], 1);
          *last_flag = (old == p.splits - 1);
        }
        epi_bar();
        const bool last = *last_flag != 0;
        epi_bar();  // everyone has read last_flag before it is rewritten
        if (last) {
          // every split of this tile has arrived: reset its counter before the epilogue's stores
          // (a flag-free consumer may let the next GEMM start as soon as those stores land)
          if (threadIdx.x == 64) p.counters[x.tile] = 0;
          __threadfence();
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = 0.f;
            // 4 splits per batch, 16 independent loads each: keeps ~64 L2 reads in flight per thread
            for (int sp0 = 0; sp0 < p.splits; sp0 += 4) {
              float t[4][16];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int sp = sp0 + q;
                const float* src = p.ws + ((size_t)min(sp, p.splits - 1) * total_tiles + x.tile) * BN * 128 +
                                   (size_t)c0 * 128 + row;
#pragma unroll
                for (int j = 0; j < 16; ++j) t[q][j] = sp < p.splits ? __ldcg(src + (size_t)j * 128) : 0.f;
              }
#pragma unroll
              for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] += t[q][j];
            }
            epilogue_store<EPI>(p, v, row, x.n_tile, x.a_row0 + c0, t_end, xchg, quad, lane);
          }
          if constexpr (EPI == EPI_PUSH) {
            if (!p.lamport) publish_tile(p, last_flag);
          }
        }
      }
      acc_phase[acc] ^= 1;
      acc ^= 1;
    }
  }
  if (threadIdx.x == 64) trace_mark(p, 5);
  if constexpr (BN <= 64 && EPI != EPI_PUSH) {
    if (p.cluster_red) {
      // every CTA reaches both barriers, also after a timed-out wait (no cluster member may
      // exit while a peer still reads its shared memory)
      tc::cluster_sync();
      if (warp >= 2 && !*abort_flag) {
        const int quad = warp & 3;
        cluster_reduce_store<BN, EPI>(p, smem, xchg, quad * 32 + lane, quad, lane);
      }
      tc::cluster_sync();
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_mark(p, 6);
  if (threadIdx.x == 32) trace_mark(p, 7);
  if (*abort_flag) {
    // error path: give TMA copies that may still be landing in shared memory time to finish
    const uint64_t until = globaltimer_ns() + 100000ull;
    while (globaltimer_ns() < until) {
    }
  }
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}


template <int BN, int EPI>
void launch_gemm(const CUtensorMap& tw, const CUtensorMap& ta, const GemmParams& p, int grid, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    B200_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024));
    attr_set = true;
  }
  TORCH_CHECK(p.stages >= 2 && p.stages <= Cfg::MAX_STAGES && Cfg::smem(p.stages, EPI) <= 227 * 1024,
              "GEMM stage count out of range");
  if (p.cluster_red)
    launch_pdl_cluster(gemm_tc_kernel<BN, EPI>, dim3(grid), dim3(192), Cfg::smem(p.stages, EPI), stream, p.splits, tw,
                       ta, p);
  else
    launch_pdl(gemm_tc_kernel<BN, EPI>, dim3(grid), dim3(192), Cfg::smem(p.stages, EPI), stream, tw, ta, p);
}

// one translation unit per BN (gemm_tc_bn*.cu) instantiates this for every epilogue
template <int BN>
void launch_gemm_bn(int epi, const CUtensorMap& tw, const CUtensorMap& ta, const GemmParams& p, int grid,
                    cudaStream_t stream);

}  // namespace b200
