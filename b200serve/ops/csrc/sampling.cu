// Greedy argmax over vocabulary rows (restates argmax.wgsl:58,80: maximum value,
// lowest index on ties), plus the merge step of a vocabulary-parallel argmax
// across tensor-parallel ranks.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

// One row per cluster of C CTAs (512 threads each): CTA r scans its slice of the vocabulary
// (slice starts rounded down to 4 values), fp32 logits read as float4 where aligned; the slices'
// winners meet in CTA 0 through distributed shared memory (ties: the lowest index, as with C = 1).
template <int C>
__global__ void __launch_bounds__(512) argmax_rows_kernel(const float* __restrict__ logits, int V, int ld,
                                                          int* __restrict__ out_idx, float* __restrict__ out_val,
                                                          int index_offset) {
  pdl_wait();
  pdl_trigger();
  const int rowid = blockIdx.x / C;
  const int rank = C == 1 ? 0 : (int)cluster_rank();
  const int lo = C == 1 ? 0 : ((int)((long long)V * rank / C) & ~3);
  const int hi = C == 1 ? V : (rank == C - 1 ? V : ((int)((long long)V * (rank + 1) / C) & ~3));
  const float* row = logits + (size_t)rowid * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0 && (ld & 3) == 0;
  const int n4 = vec ? (hi - lo) / 4 : 0;
  const float4* r4 = reinterpret_cast<const float4*>(row + lo);
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 v = r4[i];
    const int c = lo + 4 * i;
    better(bv, bi, v.x, c);
    better(bv, bi, v.y, c + 1);
    better(bv, bi, v.z, c + 2);
    better(bv, bi, v.w, c + 3);
  }
  for (int i = lo + n4 * 4 + threadIdx.x; i < hi; i += blockDim.x) better(bv, bi, row[i], i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __shared__ float sv[16];
  __shared__ int si[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      better(bv, bi, ov, oi);
    }
    if (C == 1 && lane == 0) {
      out_idx[rowid] = bi + index_offset;
      if (out_val) out_val[rowid] = bv;
    }
    if (C > 1 && lane == 0) { sv[0] = bv; si[0] = bi; }
  }
  if constexpr (C > 1) {
    cluster_barrier();
    if (rank == 0 && threadIdx.x == 0) {
      for (int r = 1; r < C; ++r) better(bv, bi, cluster_ld_f32(&sv[0], (uint32_t)r), cluster_ld_i32(&si[0], (uint32_t)r));
      out_idx[rowid] = bi + index_offset;
      if (out_val) out_val[rowid] = bv;
    }
    cluster_barrier();                    // CTA 0 has read every slice's winner
  }
}

// Merge per-rank (value, index) candidates [R, B] -> index [B].
__global__ void argmax_merge_kernel(const float* __restrict__ vals, const int* __restrict__ idx, int R, int B,
                                    int* __restrict__ out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int r = 0; r < R; ++r) better(bv, bi, vals[r * B + b], idx[r * B + b]);
  out[b] = bi;
}

}  // namespace b200

using namespace b200;

void argmax_rows(torch::Tensor logits, torch::Tensor out_idx, torch::Tensor out_val, int64_t index_offset) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1);
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  // rows split over clusters so that B x C CTAs fill the SMs (one CTA per row would leave most idle)
  const int C = V < 4096 * 8 ? 1 : B <= 18 ? 8 : B <= 37 ? 4 : B <= 74 ? 2 : 1;
  auto stream = at::cuda::getCurrentCUDAStream();
  const float* lp = logits.data_ptr<float>();
  float* vp = out_val.numel() ? out_val.data_ptr<float>() : (float*)nullptr;
  const int ld = (int)logits.stride(0), off = (int)index_offset;
  int* ip = out_idx.data_ptr<int>();
  switch (C) {
    case 8: launch_pdl_cluster(argmax_rows_kernel<8>, dim3(B * 8), dim3(512), 0, stream, 8, lp, V, ld, ip, vp, off); break;
    case 4: launch_pdl_cluster(argmax_rows_kernel<4>, dim3(B * 4), dim3(512), 0, stream, 4, lp, V, ld, ip, vp, off); break;
    case 2: launch_pdl_cluster(argmax_rows_kernel<2>, dim3(B * 2), dim3(512), 0, stream, 2, lp, V, ld, ip, vp, off); break;
    default: launch_pdl(argmax_rows_kernel<1>, dim3(B), dim3(512), 0, stream, lp, V, ld, ip, vp, off); break;
  }
}

void argmax_merge(torch::Tensor vals, torch::Tensor idx, torch::Tensor out) {
  const int R = vals.size(0), B = vals.size(1);
  if (B == 0) return;
  argmax_merge_kernel<<<(B + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      vals.data_ptr<float>(), idx.data_ptr<int>(), R, B, out.data_ptr<int>());
  B200_CHECK_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Full sampler: penalties, temperature, top-k, top-p, min-p, seeded draw.
// Semantics follow the reference CPU sampler (webgpu/src/engine/generate.ts:274-510)
// and HF logits processors; the draw is a Gumbel-max over the kept tokens,
// which samples exactly from the softmax restricted to them.
// ---------------------------------------------------------------------------
namespace b200 {

// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC 2011): 10 rounds of two 32x32->64
// multiplies with the paper's multipliers and Weyl key increments.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += W0;
    k.y += W1;
  }
  return c;
}

struct SampleRow {
  float temperature, top_p, min_p;
  int top_k;
  uint64_t seed;
  uint32_t step;
};

// ---- filter thresholds in "distance" space -------------------------------------------------
// Every filter keeps an upper set of the row: top-k the k largest logits, top-p the
// largest ones up to a probability mass, min-p those with p >= min_p * p_max. With
// d = (m - x) / t (m = row max, t = temperature) each is a threshold on d, and
// exp(-d) is the unnormalised probability. Thresholds are found with histograms of d:
// level 1 bins [0, R] into 256 equal bins; if the bins up to the boundary hold at most
// kSCand tokens they are compacted and finished exactly (sort + prefix sums), else
// the boundary bin is split again into 256 sub-bins (level 2, resolution R / 65536).
// Tokens with d > 32 (probability below 1.3e-14 of the maximum) are excluded whenever
// top-k or top-p is active.
constexpr int kSThreads = 512, kSWarps = kSThreads / 32, kSBins = 256, kSCand = 4096;
constexpr float kDFar = 32.f;

struct DThr {          // keep d iff bin1(d) < b1, or bin1(d) == b1 and bin2(d) <= b2
  float s1, lo2, s2;
  int b1, b2;
};
struct DPred {
  float dcap;          // min-p / far-tail cap: keep only d <= dcap
  int n;
  DThr t[3];
};

__device__ __forceinline__ int dbin1(float d, float s1) { return min((int)(d * s1), kSBins - 1); }
__device__ __forceinline__ int dbin2(float d, float lo2, float s2) {
  return max(0, min((int)((d - lo2) * s2), kSBins - 1));
}
__device__ __forceinline__ bool dkeep(float d, const DPred& p) {
  if (!(d <= p.dcap)) return false;
  for (int j = 0; j < p.n; ++j) {
    const int b = dbin1(d, p.t[j].s1);
    if (b > p.t[j].b1) return false;
    if (b == p.t[j].b1 && p.t[j].b2 < kSBins - 1 && dbin2(d, p.t[j].lo2, p.t[j].s2) > p.t[j].b2) return false;
  }
  return true;
}

struct SampShared {
  union {
    struct { uint32_t cnt[kSWarps][kSBins]; float mass[kSWarps][kSBins]; } h;   // per-warp histograms
    struct { float v[kSCand]; int i[kSCand]; } c;                                 // compacted candidates
  } u;
  uint32_t tot_cnt[kSBins];
  float tot_mass[kSBins];
  uint32_t g_cnt[kSBins];      // cluster sums of tot_* (several CTAs per row)
  float g_mass[kSBins];
  float red[32];
  int redi[32];
  float wmin[32];
  float f[4];
  int n[4];
};

// This CTA's share of a row: [lo, hi), lo a multiple of 4.
struct Slice {
  int lo, hi;
};

// Calls f(x, i) for every element of the slice (float4 loads when aligned).
template <class F>
__device__ __forceinline__ void for_row(const float* row, Slice sl, bool vec, F&& f) {
  const int n4 = vec ? (sl.hi - sl.lo) / 4 : 0;
  const float4* r4 = reinterpret_cast<const float4*>(row + sl.lo);
  for (int q = threadIdx.x; q < n4; q += blockDim.x) {
    const float4 v = r4[q];
    const int i = sl.lo + 4 * q;
    f(v.x, i);
    f(v.y, i + 1);
    f(v.z, i + 2);
    f(v.w, i + 3);
  }
  for (int i = sl.lo + n4 * 4 + threadIdx.x; i < sl.hi; i += blockDim.x) f(row[i], i);
}

// ---- thread-block cluster helpers (C CTAs share one row) ----
__device__ __forceinline__ void cl_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cl_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(r)
               : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ uint32_t cl_ld_u32(const void* p, uint32_t rank) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cl_addr(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ float cl_ld_f32(const void* p, uint32_t rank) {
  return __uint_as_float(cl_ld_u32(p, rank));
}

// Histogram of the surviving tokens' d: level 1 (bsel < 0) over bin1 with scale s1, level 2
// over the sub-bins of bin1 == bsel. Counts are aggregated per warp (match_any), masses use
// per-warp shared atomics. Leaves totals in S.tot_cnt / S.tot_mass.
template <int C>
__device__ void d_histogram(const float* row, Slice sl, bool vec, float m, float inv_t, const DPred& P, float s1,
                            int bsel, float lo2, float s2, SampShared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kSWarps * kSBins; i += blockDim.x) {
    (&S.u.h.cnt[0][0])[i] = 0u;
    (&S.u.h.mass[0][0])[i] = 0.f;
  }
  __syncthreads();
  uint32_t* cnt = S.u.h.cnt[warp];
  float* mass = S.u.h.mass[warp];
  for_row(row, sl, vec, [&](float x, int) {
    const float d = (m - x) * inv_t;
    int b = -1;
    if (dkeep(d, P)) {
      b = dbin1(d, s1);
      if (bsel >= 0) b = (b == bsel) ? dbin2(d, lo2, s2) : -1;
    }
    const unsigned act = __activemask();
    const unsigned grp = __match_any_sync(act, b);
    if (b >= 0) {
      if (lane == __ffs(grp) - 1) atomicAdd(&cnt[b], (uint32_t)__popc(grp));
      atomicAdd(&mass[b], __expf(-d));
    }
  });
  __syncthreads();
  for (int b = threadIdx.x; b < kSBins; b += blockDim.x) {
    uint32_t c = 0;
    float w = 0.f;
#pragma unroll
    for (int k = 0; k < kSWarps; ++k) {
      c += S.u.h.cnt[k][b];
      w += S.u.h.mass[k][b];
    }
    S.tot_cnt[b] = c;
    S.tot_mass[b] = w;
  }
  __syncthreads();
  if constexpr (C > 1) {
    // every CTA of the row sums the C local histograms in rank order (same totals everywhere)
    cl_sync();
    for (int b = threadIdx.x; b < kSBins; b += blockDim.x) {
      uint32_t c = 0;
      float w = 0.f;
      for (int r = 0; r < C; ++r) {
        c += cl_ld_u32(&S.tot_cnt[b], (uint32_t)r);
        w += cl_ld_f32(&S.tot_mass[b], (uint32_t)r);
      }
      S.g_cnt[b] = c;
      S.g_mass[b] = w;
    }
    cl_sync();                    // no CTA overwrites its totals while another still reads them
    for (int b = threadIdx.x; b < kSBins; b += blockDim.x) {
      S.tot_cnt[b] = S.g_cnt[b];
      S.tot_mass[b] = S.g_mass[b];
    }
    __syncthreads();
  }
}

// Warp 0: first bin whose inclusive cumulative count (MASS: mass) reaches the target, which is
// frac * total when frac >= 0, else `target`. Writes S.n[0] = bin (kSBins if never reached),
// S.f[0] = cumulative before the bin, S.n[1] = tokens through the bin, S.f[2] = the target.
template <bool MASS>
__device__ void d_find(float target, float frac, SampShared& S) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float w[8], c[8];
    float ws = 0.f, cs = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      c[k] = (float)S.tot_cnt[lane * 8 + k];
      w[k] = MASS ? S.tot_mass[lane * 8 + k] : c[k];
      ws += w[k];
      cs += c[k];
    }
    float wi = ws, ci = cs;   // inclusive scans over lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float a = __shfl_up_sync(0xffffffffu, wi, o), b = __shfl_up_sync(0xffffffffu, ci, o);
      if (lane >= o) { wi += a; ci += b; }
    }
    const float total_w = __shfl_sync(0xffffffffu, wi, 31), total_c = __shfl_sync(0xffffffffu, ci, 31);
    const float tgt = frac >= 0.f ? frac * total_w : target;
    const unsigned hit = __ballot_sync(0xffffffffu, wi >= tgt);
    const int L = hit ? __ffs(hit) - 1 : -1;
    if (lane == 0 && !hit) { S.n[0] = kSBins; S.f[0] = total_w; S.n[1] = (int)total_c; }
    if (lane == L) {
      float cum = wi - ws, cc = ci - cs;
      int bin = lane * 8 + 7;
      for (int k = 0; k < 8; ++k) {
        cc += c[k];
        if (cum + w[k] >= tgt) { bin = lane * 8 + k; break; }
        cum += w[k];
      }
      S.n[0] = bin;
      S.f[0] = cum;
      S.n[1] = (int)cc;
    }
    if (lane == 0) S.f[2] = tgt;
  }
  __syncthreads();
}

__device__ __forceinline__ void block_best(float& bv, int& bi, SampShared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __syncthreads();
  if (lane == 0) { S.red[warp] = bv; S.redi[warp] = bi; }
  __syncthreads();
  bv = lane < nw ? S.red[lane] : -INFINITY;
  bi = lane < nw ? S.redi[lane] : 0x7fffffff;
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
}

__device__ __forceinline__ float gumbel(int i, uint32_t step, uint32_t row, uint2 key) {
  const uint4 r = philox4x32_10(make_uint4((uint32_t)i, step, row, 0x5A4D504Cu), key);
  const float u = ((float)(r.x >> 8) + 0.5f) * (1.f / 16777216.f);
  return -__logf(-__logf(u));
}

// Sorted (descending value, ascending index) candidates: exact top-k, then exact top-p
// (keep j while the mass before it is <= target; target = top_p * mass of the top-k
// survivors when mass_target < 0), then the Gumbel-max draw. Returns the vocabulary id.
__device__ int finish_candidates(int n, int top_k, float top_p, float mass_target, float m, float inv_t,
                                 uint32_t step, uint2 key, int rowid, SampShared& S) {
  int N2 = 32;
  while (N2 < n) N2 <<= 1;
  for (int i = n + threadIdx.x; i < N2; i += blockDim.x) { S.u.c.v[i] = -INFINITY; S.u.c.i[i] = 0x7fffffff; }
  __syncthreads();
  for (int k = 2; k <= N2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int t = threadIdx.x; t < N2; t += blockDim.x) {
        const int u = t ^ j;
        if (u > t) {
          const float vt = S.u.c.v[t], vu = S.u.c.v[u];
          const int it = S.u.c.i[t], iu = S.u.c.i[u];
          const bool u_first = vu > vt || (vu == vt && iu < it);
          if (((t & k) == 0) == u_first) {
            S.u.c.v[t] = vu; S.u.c.v[u] = vt;
            S.u.c.i[t] = iu; S.u.c.i[u] = it;
          }
        }
      }
      __syncthreads();
    }
  }
  int keep = n;
  if (top_k > 0 && top_k < n) {
    const float vk = S.u.c.v[top_k - 1];
    keep = top_k;
    while (keep < n && S.u.c.v[keep] == vk) ++keep;   // ties at the boundary stay
  }
  if (top_p < 1.f && keep > 1) {
    // chunked block scan of the weights over [0, keep)
    const int per = (keep + blockDim.x - 1) / blockDim.x;
    const int j0 = min(keep, (int)threadIdx.x * per), j1 = min(keep, j0 + per);
    float loc = 0.f;
    for (int j = j0; j < j1; ++j) loc += __expf((S.u.c.v[j] - m) * inv_t);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float inc = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float a = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += a;
    }
    if (lane == 31) S.red[warp] = inc;
    if (threadIdx.x == 0) S.n[2] = keep;
    __syncthreads();
    float wbase = 0.f, total = 0.f;
    for (int w = 0; w < nw; ++w) {
      if (w < warp) wbase += S.red[w];
      total += S.red[w];
    }
    const float tgt = mass_target >= 0.f ? mass_target : top_p * total;
    float before = wbase + inc - loc;
    for (int j = j0; j < j1; ++j) {
      if (before > tgt) { atomicMin(&S.n[2], j); break; }
      before += __expf((S.u.c.v[j] - m) * inv_t);
    }
    __syncthreads();
    keep = max(1, S.n[2]);
    __syncthreads();
  }
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = threadIdx.x; j < keep; j += blockDim.x) {
    const int id = S.u.c.i[j];
    better(bv, bi, S.u.c.v[j] * inv_t + gumbel(id, step, (uint32_t)rowid, key), id);
  }
  block_best(bv, bi, S);
  return bi;
}

// Cluster-wide (value, index) best and minimum: each CTA publishes its own in S.red/S.redi/S.wmin
// slot 0..2, then every CTA combines the C entries in rank order.
template <int C>
__device__ __forceinline__ void cl_best(float& bv, int& bi, float& mn, SampShared& S) {
  if constexpr (C > 1) {
    if (threadIdx.x == 0) { S.f[1] = bv; S.n[1] = bi; S.f[3] = mn; }
    cl_sync();
    float v = -INFINITY, m2 = INFINITY;
    int ix = 0x7fffffff;
    for (int r = 0; r < C; ++r) {
      better(v, ix, cl_ld_f32(&S.f[1], (uint32_t)r), (int)cl_ld_u32(&S.n[1], (uint32_t)r));
      m2 = fminf(m2, cl_ld_f32(&S.f[3], (uint32_t)r));
    }
    cl_sync();
    bv = v;
    bi = ix;
    mn = m2;
  }
}

// C CTAs per row (a thread-block cluster when C > 1): CTA rank r of row b works on the slice
// [r*V/C, (r+1)*V/C) (multiples of 4); histograms, maxima and candidate sets are merged through
// distributed shared memory, and rank 0 finishes the draw.
template <int C>
__global__ void __launch_bounds__(kSThreads) sample_rows_kernel(float* __restrict__ logits, int V, int ld,
                                                                const SampleRow* __restrict__ params,
                                                                const int* __restrict__ pen_ids,
                                                                const float* __restrict__ pen_counts, int P,
                                                                const float* __restrict__ pen_vals,
                                                                int* __restrict__ out) {
  __shared__ SampShared S;
  pdl_wait();                       // the logits come from the previous kernel
  pdl_trigger();
  const int rowid = blockIdx.x / C, rank = blockIdx.x % C;
  float* row = logits + (size_t)rowid * ld;
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0) && (ld & 3) == 0;
  Slice sl;
  sl.lo = C == 1 ? 0 : ((int)((long long)V * rank / C) & ~3);
  sl.hi = C == 1 ? V : (rank == C - 1 ? V : ((int)((long long)V * (rank + 1) / C) & ~3));
  const SampleRow pr = params[rowid];
  // ---- penalties (ids unique per row) on this CTA's slice: repetition, presence, frequency ----
  if (P > 0) {
    const float rp = pen_vals[rowid * 3 + 0], pres = pen_vals[rowid * 3 + 1], freq = pen_vals[rowid * 3 + 2];
    for (int j = threadIdx.x; j < P; j += blockDim.x) {
      const int id = pen_ids[rowid * P + j];
      if (id < sl.lo || id >= sl.hi) continue;
      float x = row[id];
      if (rp != 1.f) x = x > 0.f ? x / rp : x * rp;
      x -= pres + freq * pen_counts[rowid * P + j];
      row[id] = x;
    }
    __syncthreads();
  }
  // ---- row max (the greedy answer) and min ----
  float bv = -INFINITY, mn = INFINITY;
  int bi = 0x7fffffff;
  for_row(row, sl, vec, [&](float x, int i) { better(bv, bi, x, i); mn = fminf(mn, x); });
  mn = -warp_max(-mn);
  if ((threadIdx.x & 31) == 0) S.wmin[threadIdx.x >> 5] = mn;
  block_best(bv, bi, S);
  float xmin = INFINITY;
  __syncthreads();
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) xmin = fminf(xmin, S.wmin[w]);
  __syncthreads();
  cl_best<C>(bv, bi, xmin, S);
  if (threadIdx.x == 0) { S.f[0] = bv; S.n[0] = bi; }
  __syncthreads();
  const float m = S.f[0];
  const int greedy = S.n[0];
  __syncthreads();
  if (!(pr.temperature > 0.f)) {
    if (threadIdx.x == 0 && rank == 0) out[rowid] = greedy;
    return;
  }
  const float inv_t = 1.f / pr.temperature;
  const uint2 key = make_uint2((uint32_t)pr.seed, (uint32_t)(pr.seed >> 32));
  const bool use_k = pr.top_k > 0 && pr.top_k < V, use_p = pr.top_p < 1.f;
  DPred Pd;
  Pd.n = 0;
  Pd.dcap = pr.min_p > 0.f ? -__logf(pr.min_p) : INFINITY;
  int result = -1;
  if (use_k || use_p) {
    Pd.dcap = fminf(Pd.dcap, kDFar);
    float R = fminf((m - xmin) * inv_t, Pd.dcap);
    if (!(R > 0.f)) R = 1.f;
    int exact_k = 0;
    float mass_target = -1.f;
    bool cand = false;
    for (int stage = 0; stage < 2 && !cand; ++stage) {
      const bool mass = stage == 1;
      if (mass ? !use_p : !use_k) continue;
      const float s1 = (float)kSBins / R;
      d_histogram<C>(row, sl, vec, m, inv_t, Pd, s1, -1, 0.f, 0.f, S);
      if (mass) d_find<true>(0.f, pr.top_p, S);
      else d_find<false>((float)pr.top_k, -1.f, S);
      const int b1 = S.n[0];
      const float before1 = S.f[0], tgt = S.f[2];
      const int through = S.n[1];
      __syncthreads();
      if (b1 >= kSBins) continue;                       // filter keeps every survivor
      DThr t{s1, 0.f, 0.f, b1, kSBins - 1};
      if (through <= kSCand) {
        Pd.t[Pd.n++] = t;
        cand = true;
        if (!mass) exact_k = pr.top_k;
        else mass_target = tgt;
        break;
      }
      const float lo2 = (float)b1 / s1, s2 = s1 * (float)kSBins;
      d_histogram<C>(row, sl, vec, m, inv_t, Pd, s1, b1, lo2, s2, S);
      if (mass) d_find<true>(tgt - before1, -1.f, S);   // the mass still needed inside bin b1
      else d_find<false>((float)pr.top_k - before1, -1.f, S);
      t.lo2 = lo2;
      t.s2 = s2;
      t.b2 = min(S.n[0], kSBins - 1);
      Pd.t[Pd.n++] = t;
      R = ((float)b1 + (float)(t.b2 + 1) / (float)kSBins) / s1;
      __syncthreads();
    }
    if (cand) {
      if (threadIdx.x == 0) S.n[2] = 0;
      __syncthreads();
      const int lane = threadIdx.x & 31;
      for_row(row, sl, vec, [&](float x, int i) {
        const bool k = dkeep((m - x) * inv_t, Pd);
        const unsigned act = __activemask();
        const unsigned bal = __ballot_sync(act, k);
        const int leader = __ffs(act) - 1;
        int base = 0;
        if (lane == leader && bal) base = atomicAdd(&S.n[2], __popc(bal));
        base = __shfl_sync(act, base, leader);
        if (k) {
          const int slot = base + __popc(bal & ((1u << lane) - 1u));
          if (slot < kSCand) { S.u.c.v[slot] = x; S.u.c.i[slot] = i; }
        }
      });
      __syncthreads();
      int n = min(S.n[2], kSCand);
      if constexpr (C > 1) {
        // rank 0 appends the other CTAs' candidates (the global count is <= kSCand)
        cl_sync();
        if (rank == 0) {
          for (int r = 1; r < C; ++r) {
            const int nr = min((int)cl_ld_u32(&S.n[2], (uint32_t)r), kSCand);
            for (int j = threadIdx.x; j < nr && n + j < kSCand; j += blockDim.x) {
              S.u.c.v[n + j] = cl_ld_f32(&S.u.c.v[j], (uint32_t)r);
              S.u.c.i[n + j] = (int)cl_ld_u32(&S.u.c.i[j], (uint32_t)r);
            }
            n = min(kSCand, n + nr);
          }
        }
        cl_sync();                  // the other CTAs keep their shared memory until rank 0 has read it
        if (rank != 0) return;
      }
      __syncthreads();
      result = finish_candidates(n, exact_k, use_p ? pr.top_p : 1.f, mass_target, m, inv_t, pr.step, key, rowid, S);
    }
  }
  if (result < 0) {
    // ---- Gumbel-max draw over every surviving token ----
    float best = -INFINITY, unused = INFINITY;
    int best_i = 0x7fffffff;
    for_row(row, sl, vec, [&](float x, int i) {
      if (!dkeep((m - x) * inv_t, Pd)) return;
      better(best, best_i, x * inv_t + gumbel(i, pr.step, (uint32_t)rowid, key), i);
    });
    block_best(best, best_i, S);
    __syncthreads();
    cl_best<C>(best, best_i, unused, S);
    result = best_i;
  }
  if (threadIdx.x == 0 && rank == 0) out[rowid] = result == 0x7fffffff ? greedy : result;
}

}  // namespace b200

// logits [B, V] fp32 (modified in place by penalties); params: int64 [B, 6] packed as
// (temperature bits, top_p bits, min_p bits, top_k, seed, step); pen_ids [B, P] int32 (-1 pad),
// pen_counts [B, P] fp32, pen_vals [B, 3] fp32 (repeat, presence, frequency).
void sample_rows(torch::Tensor logits, torch::Tensor params, torch::Tensor pen_ids, torch::Tensor pen_counts,
                 torch::Tensor pen_vals, torch::Tensor out, int64_t cluster) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1);
  TORCH_CHECK(params.scalar_type() == at::kByte && params.numel() == logits.size(0) * (int64_t)sizeof(b200::SampleRow));
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const int P = pen_ids.numel() ? pen_ids.size(1) : 0;
  // CTAs per row: a thread-block cluster splits each row so that small batches still fill the SMs
  static int cl = -1;
  if (cl < 0) {
    const char* e = getenv("B200_SAMPLER_CLUSTER");
    cl = e ? atoi(e) : 0;
  }
  int C = cluster > 0 ? (int)cluster : cl > 0 ? cl : (B <= 18 ? 8 : B <= 74 ? 4 : 1);
  if (C != 1 && C != 2 && C != 4 && C != 8) C = 4;
  if (V < 4096 * C) C = 1;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto lp = reinterpret_cast<const b200::SampleRow*>(params.data_ptr());
  const int* pi = P ? pen_ids.data_ptr<int>() : nullptr;
  const float* pc = P ? pen_counts.data_ptr<float>() : nullptr;
  const float* pv = P ? pen_vals.data_ptr<float>() : nullptr;
  float* lg = logits.data_ptr<float>();
  const int ld = logits.stride(0);
  int* o = out.data_ptr<int>();
  switch (C) {
    case 8: b200::launch_pdl_cluster(b200::sample_rows_kernel<8>, dim3(B * 8), dim3(b200::kSThreads), 0, stream, 8,
                                     lg, V, ld, lp, pi, pc, P, pv, o); break;
    case 4: b200::launch_pdl_cluster(b200::sample_rows_kernel<4>, dim3(B * 4), dim3(b200::kSThreads), 0, stream, 4,
                                     lg, V, ld, lp, pi, pc, P, pv, o); break;
    case 2: b200::launch_pdl_cluster(b200::sample_rows_kernel<2>, dim3(B * 2), dim3(b200::kSThreads), 0, stream, 2,
                                     lg, V, ld, lp, pi, pc, P, pv, o); break;
    default:
      b200::sample_rows_kernel<1><<<B, b200::kSThreads, 0, stream>>>(lg, V, ld, lp, pi, pc, P, pv, o);
      B200_CHECK_CUDA(cudaGetLastError());
  }
}
