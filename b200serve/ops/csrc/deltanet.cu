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
//            warps also turn (a, b) into the log decay g = A softplus(a + dt) and
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
    __nv_bfloat16* __restrict__ xc, float* __restrict__ gb, int T, int S, int nk, int nv, int nstates) {
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
  if (!B200_IN_RANGE(slots[s], nstates, 0x501)) return;
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
    gb[((size_t)t * nv + h) * 2 + 0] = g;          // log decay (<= 0)
    gb[((size_t)t * nv + h) * 2 + 1] = 1.f / (1.f + __expf(-b));
  }
}

template <int D, int K>
__global__ void __launch_bounds__(2 * D) dn_scan_kernel(
    const __nv_bfloat16* __restrict__ y, int ystride, const __nv_bfloat16* __restrict__ xc,
    const float* __restrict__ gb, const __nv_bfloat16* __restrict__ norm_w, float* __restrict__ conv_state,
    float* __restrict__ rec_state, const int* __restrict__ cu_q, const int* __restrict__ q_start,
    const int* __restrict__ slots, __nv_bfloat16* __restrict__ out, int nk, int nv, float eps, int nstates) {
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
  if (!B200_IN_RANGE(slot, nstates, 0x502)) return;            // whole CTA, before any barrier
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
    const float decay = __expf(gb[((size_t)t * nv + h) * 2 + 0]), beta = gb[((size_t)t * nv + h) * 2 + 1];
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

// ---------------------------------------------------------------------------------
// Chunked form of the same recurrence for prefill (sequences of many tokens). Within a
// chunk of C tokens with in-chunk cumulative log decay b_t (Gamma_t = exp(b_t)) and the
// state S0 entering it, the pseudo-values U solve (I + A) U = R with
//   A[t][s] = beta_t exp(b_t - b_s) k_t.k_s  (s < t),   R_t = beta_t (v_t - Gamma_t S0^T k_t),
// and then
//   o_t = Gamma_t S0^T q_t + sum_{s<=t} exp(b_t - b_s) (q_t.k_s) u_s,
//   S_C = Gamma_C S0 + sum_s exp(b_C - b_s) k_s u_s^T
// (the WY-style chunking of the (gated) delta rule, Yang et al., "Parallelizing Linear
// Transformers with the Delta Rule over Sequence Length", 2024). One CTA of 256 threads per
// (sequence, value head, group of CW state columns): columns of S evolve independently given
// k and q, so the CW-column groups split the work; A and q.k are recomputed per group. The
// sequential part is a 64-step forward substitution done warp-locally (each warp owns 4
// columns). fp32 throughout; the raw o (before the gated RMSNorm) goes to o_raw.
constexpr int kDnC = 64;    // chunk length
constexpr int kDnCW = 32;   // state columns per CTA

template <int D>
struct DnChunkSmem {
  static constexpr int LDK = D + 1;                 // padded rows: conflict-free column walks
  static constexpr int S = 0;                       // [D][CW]
  static constexpr int K = S + D * kDnCW;           // [C][LDK]
  static constexpr int Q = K + kDnC * LDK;          // [C][LDK]
  static constexpr int V = Q + kDnC * LDK;          // [C][CW]  v, then R, then U
  static constexpr int QS = V + kDnC * kDnCW;       // [C][CW]
  static constexpr int A = QS + kDnC * kDnCW;       // [C][C+1] strictly lower A
  static constexpr int QK = A + kDnC * (kDnC + 1);  // [C][C+1] exp(b_t-b_s) q_t.k_s, s<=t
  static constexpr int B = QK + kDnC * (kDnC + 1);  // [C] cumulative log decay
  static constexpr int BETA = B + kDnC;             // [C]
  static constexpr int TOTAL = BETA + kDnC;         // floats
};

template <int D, int K>
__global__ void __launch_bounds__(256) dn_chunk_kernel(
    const __nv_bfloat16* __restrict__ y, int ystride, const __nv_bfloat16* __restrict__ xc,
    const float* __restrict__ gb, float* __restrict__ conv_state, float* __restrict__ rec_state,
    const int* __restrict__ cu_q, const int* __restrict__ q_start, const int* __restrict__ slots,
    float* __restrict__ o_raw, int nk, int nv, int nstates) {
  using L = DnChunkSmem<D>;
  extern __shared__ __align__(16) float sm[];
  float* Ss = sm + L::S;
  float* Ks = sm + L::K;
  float* Qs = sm + L::Q;
  float* Vs = sm + L::V;
  float* QSs = sm + L::QS;
  float* As = sm + L::A;
  float* QKs = sm + L::QK;
  float* Bs = sm + L::B;
  float* BETAs = sm + L::BETA;
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x, h = blockIdx.y, c0 = blockIdx.z * kDnCW;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ratio = nv / nk, kh = h / ratio;
  const int conv_dim = (2 * nk + nv) * D;
  const int t0 = cu_q[s], n = cu_q[s + 1] - t0;
  const int slot = slots[s];
  if (!B200_IN_RANGE(slot, nstates, 0x503)) return;            // whole CTA, before any barrier
  const bool hist = q_start[s] > 0;
  const float scale = rsqrtf((float)D);
  float* rs = rec_state + ((size_t)slot * nv + h) * D * D;
  for (int e = tid; e < D * kDnCW; e += 256) {
    const int i = e / kDnCW, j = e % kDnCW;
    Ss[e] = hist ? rs[(size_t)i * D + c0 + j] : 0.f;
  }
  for (int cs = 0; cs < n; cs += kDnC) {
    const int nc = min(kDnC, n - cs);
    __syncthreads();   // previous chunk done with K/Q/V/A
    for (int e = tid; e < kDnC * D; e += 256) {
      const int t = e / D, i = e % D;
      float kv = 0.f, qv = 0.f;
      if (t < nc) {
        const __nv_bfloat16* xr = xc + (size_t)(t0 + cs + t) * conv_dim;
        qv = __bfloat162float(xr[kh * D + i]) * scale;
        kv = __bfloat162float(xr[nk * D + kh * D + i]);
      }
      Ks[t * L::LDK + i] = kv;
      Qs[t * L::LDK + i] = qv;
    }
    for (int e = tid; e < kDnC * kDnCW; e += 256) {
      const int t = e / kDnCW, j = e % kDnCW;
      Vs[e] = t < nc ? __bfloat162float(xc[(size_t)(t0 + cs + t) * conv_dim + 2 * nk * D + h * D + c0 + j]) : 0.f;
    }
    if (tid < kDnC) {
      const bool ok = tid < nc;
      Bs[tid] = ok ? gb[((size_t)(t0 + cs + tid) * nv + h) * 2 + 0] : 0.f;
      BETAs[tid] = ok ? gb[((size_t)(t0 + cs + tid) * nv + h) * 2 + 1] : 0.f;
    }
    __syncthreads();
    if (warp == 0) {   // inclusive prefix sum of the log decays (2 per lane)
      float a0 = Bs[2 * lane], a1 = Bs[2 * lane + 1];
      a1 += a0;
      float run = a1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o) run += v;
      }
      const float before = run - a1;
      Bs[2 * lane] = before + a0;
      Bs[2 * lane + 1] = run;
    }
    __syncthreads();
    // A (strictly lower) and the masked, decay-weighted q.k: warp w rows t = w + 8r, lane cols s = lane, lane+32
    {
      float ak[8][2], aq[8][2];
#pragma unroll
      for (int r = 0; r < 8; ++r) ak[r][0] = ak[r][1] = aq[r][0] = aq[r][1] = 0.f;
      for (int i = 0; i < D; ++i) {
        const float k0 = Ks[lane * L::LDK + i], k1 = Ks[(lane + 32) * L::LDK + i];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int t = warp + 8 * r;
          const float kt = Ks[t * L::LDK + i], qt = Qs[t * L::LDK + i];
          ak[r][0] += kt * k0;
          ak[r][1] += kt * k1;
          aq[r][0] += qt * k0;
          aq[r][1] += qt * k1;
        }
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int t = warp + 8 * r;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int sc = lane + 32 * c;
          const float w = sc <= t ? __expf(Bs[t] - Bs[sc]) : 0.f;
          As[t * (kDnC + 1) + sc] = sc < t ? BETAs[t] * w * ak[r][c] : 0.f;
          QKs[t * (kDnC + 1) + sc] = w * aq[r][c];
        }
      }
    }
    // S0^T k and S0^T q for this CTA's columns: warp w rows t = w + 8r, lane = column
    {
      float ks[8], qs[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) ks[r] = qs[r] = 0.f;
      for (int i = 0; i < D; ++i) {
        const float sv = Ss[i * kDnCW + lane];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int t = warp + 8 * r;
          ks[r] += Ks[t * L::LDK + i] * sv;
          qs[r] += Qs[t * L::LDK + i] * sv;
        }
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int t = warp + 8 * r;
        const float g = __expf(Bs[t]);
        Vs[t * kDnCW + lane] = BETAs[t] * (Vs[t * kDnCW + lane] - g * ks[r]);   // R
        QSs[t * kDnCW + lane] = g * qs[r];
      }
    }
    __syncthreads();
    // forward substitution (I + A) U = R, warp-local: warp w owns columns 4w..4w+3,
    // lane = 8 * column-in-warp + s-group
    {
      const int j = warp * 4 + (lane >> 3), sg = lane & 7;
      for (int t = 0; t < nc; ++t) {
        float part = 0.f;
        for (int s2 = sg; s2 < t; s2 += 8) part += As[t * (kDnC + 1) + s2] * Vs[s2 * kDnCW + j];
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        if (sg == 0) Vs[t * kDnCW + j] -= part;
        __syncwarp();
      }
    }
    __syncthreads();
    // o_t = Gamma_t S0^T q_t + sum_{s<=t} QK[t][s] u_s
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int t = warp + 8 * r;
      if (t >= nc) continue;
      float o = QSs[t * kDnCW + lane];
      for (int s2 = 0; s2 <= t; ++s2) o += QKs[t * (kDnC + 1) + s2] * Vs[s2 * kDnCW + lane];
      o_raw[(size_t)(t0 + cs + t) * nv * D + h * D + c0 + lane] = o;
    }
    // S <- Gamma_C S + sum_t exp(b_C - b_t) k_t u_t^T: warp w rows i = w + 8r (16 rows), lane = column
    {
      const float bl = Bs[nc - 1];
      const float gl = __expf(bl);
      float acc[D / 8];
#pragma unroll
      for (int r = 0; r < D / 8; ++r) acc[r] = gl * Ss[(warp + 8 * r) * kDnCW + lane];
      for (int t = 0; t < nc; ++t) {
        const float wu = __expf(bl - Bs[t]) * Vs[t * kDnCW + lane];
#pragma unroll
        for (int r = 0; r < D / 8; ++r) acc[r] += Ks[t * L::LDK + warp + 8 * r] * wu;
      }
      __syncthreads();   // every warp has read the old S
#pragma unroll
      for (int r = 0; r < D / 8; ++r) Ss[(warp + 8 * r) * kDnCW + lane] = acc[r];
    }
  }
  __syncthreads();
  for (int e = tid; e < D * kDnCW; e += 256) {
    const int i = e / kDnCW, j = e % kDnCW;
    rs[(size_t)i * D + c0 + j] = Ss[e];
  }
  // column group 0 rolls the conv state of this head's channels (as dn_scan does)
  if (blockIdx.z == 0 && tid < D) {
    auto roll = [&](int c) {
      float* cst = conv_state + ((size_t)slot * conv_dim + c) * (K - 1);
      float old[K - 1];
#pragma unroll
      for (int q = 0; q < K - 1; ++q) old[q] = hist ? cst[q] : 0.f;
#pragma unroll
      for (int q = 0; q < K - 1; ++q) {
        const int p = n - (K - 1) + q;
        cst[q] = p >= 0 ? __bfloat162float(y[(size_t)(t0 + p) * ystride + c]) : old[(K - 1) + p];
      }
    };
    roll(2 * nk * D + h * D + tid);
    if (h % ratio == 0) {
      roll(kh * D + tid);
      roll(nk * D + kh * D + tid);
    }
  }
}

// The gated RMSNorm of dn_scan applied to o_raw: one warp per (token, value head).
template <int D>
__global__ void dn_gnorm_kernel(const float* __restrict__ o_raw, const __nv_bfloat16* __restrict__ y, int ystride,
                                const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ out, int T,
                                int nk, int nv, float eps) {
  constexpr int E = D / 32;
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T * nv) return;
  const int t = warp / nv, h = warp % nv;
  const int conv_dim = (2 * nk + nv) * D;
  float o[E];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    o[e] = bf16r(o_raw[(size_t)t * nv * D + h * D + lane * E + e]);
    ss += o[e] * o[e];
  }
  const float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int j = lane * E + e;
    const float z = __bfloat162float(y[(size_t)t * ystride + conv_dim + h * D + j]);
    const float res = bf16r(__bfloat162float(norm_w[j]) * bf16r(o[e] * inv)) * silu(z);
    out[(size_t)t * nv * D + h * D + j] = __float2bfloat16_rn(res);
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
                    torch::Tensor gb, torch::Tensor out, int64_t nk, int64_t nv, int64_t D, double eps,
                    c10::optional<torch::Tensor> o_raw) {
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
  const int nstates = (int)std::min(conv_state.size(0), rec_state.size(0));
  auto stream = at::cuda::getCurrentCUDAStream();
  const int* cu = cu_q ? cu_q->data_ptr<int>() : nullptr;
  const int warps = T * (2 * nk + nv);
  const int blocks = (warps * 32 + 255) / 256;
  const int ys = (int)y.stride(0);
#define B200_DN(DV)                                                                                            \
  launch_pdl(dn_prep_kernel<DV, 4>, dim3(blocks), dim3(256), 0, stream,                                         \
             (const __nv_bfloat16*)y.data_ptr(), ys, (const float*)conv_w.data_ptr(), (const float*)A.data_ptr(), \
             (const float*)dt_bias.data_ptr(), (const float*)conv_state.data_ptr(), cu, q_start.data_ptr<int>(),  \
             slots.data_ptr<int>(), (__nv_bfloat16*)xc.data_ptr(), gb.data_ptr<float>(), T, S, (int)nk, (int)nv,   \
             nstates);                                                                                          \
  launch_pdl(dn_scan_kernel<DV, 4>, dim3(S, nv), dim3(2 * DV), 0, stream, (const __nv_bfloat16*)y.data_ptr(), ys, \
             (const __nv_bfloat16*)xc.data_ptr(), (const float*)gb.data_ptr(),                                  \
             (const __nv_bfloat16*)norm_w.data_ptr(), conv_state.data_ptr<float>(), rec_state.data_ptr<float>(),  \
             cu, q_start.data_ptr<int>(), slots.data_ptr<int>(), (__nv_bfloat16*)out.data_ptr(), (int)nk,        \
             (int)nv, (float)eps, nstates)
  // chunked path (prefill): prep, then the chunk kernel writes raw o, then the gated norm
#define B200_DNC(DV)                                                                                           \
  {                                                                                                            \
    launch_pdl(dn_prep_kernel<DV, 4>, dim3(blocks), dim3(256), 0, stream,                                       \
               (const __nv_bfloat16*)y.data_ptr(), ys, (const float*)conv_w.data_ptr(),                          \
               (const float*)A.data_ptr(), (const float*)dt_bias.data_ptr(),                                     \
               (const float*)conv_state.data_ptr(), cu, q_start.data_ptr<int>(), slots.data_ptr<int>(),          \
               (__nv_bfloat16*)xc.data_ptr(), gb.data_ptr<float>(), T, S, (int)nk, (int)nv, nstates);            \
    const size_t smem = DnChunkSmem<DV>::TOTAL * sizeof(float);                                                \
    static bool attr = false;                                                                                   \
    if (!attr) {                                                                                                \
      B200_CHECK_CUDA(cudaFuncSetAttribute(dn_chunk_kernel<DV, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                           (int)smem));                                                        \
      attr = true;                                                                                              \
    }                                                                                                           \
    launch_pdl(dn_chunk_kernel<DV, 4>, dim3(S, nv, DV / kDnCW), dim3(256), smem, stream,                       \
               (const __nv_bfloat16*)y.data_ptr(), ys, (const __nv_bfloat16*)xc.data_ptr(),                      \
               (const float*)gb.data_ptr(), conv_state.data_ptr<float>(), rec_state.data_ptr<float>(), cu,        \
               q_start.data_ptr<int>(), slots.data_ptr<int>(), o_raw->data_ptr<float>(), (int)nk, (int)nv,       \
               nstates);                                                                                        \
    launch_pdl(dn_gnorm_kernel<DV>, dim3((T * nv * 32 + 255) / 256), dim3(256), 0, stream,                     \
               (const float*)o_raw->data_ptr<float>(), (const __nv_bfloat16*)y.data_ptr(), ys,                   \
               (const __nv_bfloat16*)norm_w.data_ptr(), (__nv_bfloat16*)out.data_ptr(), T, (int)nk, (int)nv,     \
               (float)eps);                                                                                     \
  }
  if (o_raw) {
    TORCH_CHECK(cu != nullptr, "the chunked path is for prefill batches (cu_q)");
    TORCH_CHECK(o_raw->scalar_type() == torch::kFloat32 && o_raw->is_contiguous() && o_raw->numel() >= (long)T * nv * D);
    if (D == 128) B200_DNC(128)
    else if (D == 64) B200_DNC(64)
    else if (D == 32) B200_DNC(32)
    else TORCH_CHECK(false, "DeltaNet head dim must be 32, 64 or 128");
  } else if (D == 128) { B200_DN(128); }
  else if (D == 64) { B200_DN(64); }
  else if (D == 32) { B200_DN(32); }
  else TORCH_CHECK(false, "DeltaNet head dim must be 32, 64 or 128");
#undef B200_DN
#undef B200_DNC
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

B200_BOUNDS_ACCESSOR(deltanet)
