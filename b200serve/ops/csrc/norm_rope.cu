// Row-wise kernels of the decoder: fused (partials + residual) RMSNorm, the QKV
// post-processing step (bias, per-head q/k RMSNorm, rotate-half RoPE, paged KV
// write), SwiGLU on the tile-interleaved gate/up layout, and the embedding gather.
//
// Reference kernels restated here: rmsnorm.wgsl:20 (RMSNorm), rope.wgsl:29
// (rotate-half RoPE), elementwise.wgsl:96 (gate_silu), embed.wgsl:26 (embed).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "common.cuh"

namespace b200 {

struct PartPtrs {
  const __nv_bfloat16* p[8];
};

// Norm output as an all-gather: row i of this launch is global row row0 + i; rows < T are stored
// into dst[r] on every rank r (P2P), then the last CTA raises flag[r] = *epoch on every rank.
struct AgArgs {
  __nv_bfloat16* dst[8];
  int* flag[8];
  int world, row0, T;
  int* done;                 // local counter of finished CTAs, zero on entry and exit
  const int* epoch;
};

// y = rmsnorm(sum(parts) [+ residual_in]) * w ; residual_out = the pre-norm sum.
// One CTA per row, 8 bf16 per thread per step, at most 4 steps (H <= 32768 with 1024 threads).
// Wait (one thread per CTA) until every rank has published this step's epoch
// for the site; bounded by `wait_ns`, after which an error code is
// recorded and the CTA proceeds (the host raises on the error word).
__device__ __forceinline__ void wait_peer_flags(const int* flags, const int* epoch, int n, int* err,
                                                uint64_t wait_ns) {
  if (threadIdx.x == 0) {
    const int e = *epoch;
    const uint64_t deadline = globaltimer_ns() + wait_ns;
    for (int r = 0; r < n; ++r) {
      uint32_t it = 0;
      while (true) {
        int v;
        asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
        if (v == e) break;
        if ((++it & 1023u) == 0 && globaltimer_ns() > deadline) {
          if (err) atomicExch(err, 100 + r);
          r = n;
          break;
        }
      }
    }
    // relaxed polls + one acquire fence (pairs with the writer's fence before its relaxed flags)
    asm volatile("fence.acq_rel.sys;" ::: "memory");
  }
  __syncthreads();
}

// Flag-free receive slots: a 16-byte vector of 8 bf16 is complete once none of its elements
// holds the empty-slot pattern 0xFFFF (producers never store that pattern).
__device__ __forceinline__ bool lamport_empty(const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  bool e = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) e |= (w[i] & 0xFFFFu) == 0xFFFFu || (w[i] >> 16) == 0xFFFFu;
  return e;
}

// Poll one vector of a flag-free slot until a peer's store has landed (bounded: after
// `wait_ns` an error code is recorded, `gave_up` is set and zeros are returned without further
// spinning), then put the empty pattern back for the slot's next use.
__device__ __forceinline__ uint4 lamport_take(const __nv_bfloat16* ptr, uint64_t wait_ns, int* err, bool& gave_up) {
  uint4 v;
  uint64_t deadline = 0;
  for (uint32_t it = 1;; ++it) {
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(ptr) : "memory");
    if (!lamport_empty(v)) break;
    if (gave_up) { v = make_uint4(0, 0, 0, 0); break; }
    if ((it & 255u) == 0) {
      const uint64_t now = globaltimer_ns();
      if (deadline == 0) {
        deadline = now + wait_ns;
      } else if (now > deadline) {
        if (err) atomicExch(err, 160);
        gave_up = true;
        v = make_uint4(0, 0, 0, 0);
        break;
      }
    }
  }
  asm volatile("st.global.v4.u32 [%0], {%1, %1, %1, %1};" ::"l"(ptr), "r"(0xFFFFFFFFu) : "memory");
  return v;
}

template <int VPT>
__global__ void __launch_bounds__(1024) rmsnorm_fused_kernel(
    PartPtrs parts, int nparts, const __nv_bfloat16* residual_in, __nv_bfloat16* residual_out,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H, float eps,
    const int* wait_flags, const int* epoch, int* err, const AgArgs ag, uint64_t wait_ns, int lamport,
    const PartialIn pin, int nflags) {
  __shared__ float red[32];
  // lamport == 2: the partials come from a flag-free push GEMM launched right before this kernel,
  // which let it start only after that GEMM's own prerequisites completed; the partials are
  // polled, so the wait for the GEMM's grid to drain is skipped
  if (lamport != 2) pdl_wait();
  pdl_trigger();
  if (wait_flags) wait_peer_flags(wait_flags, epoch, nflags, err, wait_ns);
  bool gave_up = false;
  const int row = blockIdx.x;
  const size_t base = (size_t)row * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int s = 0; s < VPT; ++s) {
    const int col = (threadIdx.x + s * blockDim.x) * 8;
    if (col < H) {
      float acc[8];
      if (pin.part) {
        // the GEMM's fp32 stream-K partials of this row (one "part"), summed here (a small batch:
        // this kernel runs up to 1024 threads and keeps VPT x 8 values per thread)
        partial_sum<8, 2>(pin, row, col, acc);
      } else {
      // partials may have been written by other GPUs: read through L2, not L1
      uint4 a4 = lamport ? lamport_take(parts.p[0] + base + col, wait_ns, err, gave_up)
                         : __ldcg(reinterpret_cast<const uint4*>(parts.p[0] + base + col));
      unpack8(*reinterpret_cast<bf16x8*>(&a4), acc);
      for (int k = 1; k < nparts; ++k) {
        float t[8];
        uint4 t4 = lamport ? lamport_take(parts.p[k] + base + col, wait_ns, err, gave_up)
                           : __ldcg(reinterpret_cast<const uint4*>(parts.p[k] + base + col));
        unpack8(*reinterpret_cast<bf16x8*>(&t4), t);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += t[i];
      }
      }
      if (residual_in) {
        float r[8];
        unpack8(*reinterpret_cast<const bf16x8*>(residual_in + base + col), r);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += r[i];
      }
      // the residual stream is stored in bf16; normalise the rounded value
      bf16x8 rounded = pack8(acc);
      unpack8(rounded, v[s]);
      if (residual_out) *reinterpret_cast<bf16x8*>(residual_out + base + col) = rounded;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[s][i] * v[s][i];
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
#pragma unroll
  for (int s = 0; s < VPT; ++s) {
    const int col = (threadIdx.x + s * blockDim.x) * 8;
    if (col < H) {
      float wf[8], o[8];
      unpack8(*reinterpret_cast<const bf16x8*>(w + col), wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // round the normalised value to bf16 before the weight multiply
        const float n = __bfloat162float(__float2bfloat16_rn(v[s][i] * inv));
        o[i] = n * wf[i];
      }
      const bf16x8 ov = pack8(o);
      if (ag.world > 0) {
        const int g = ag.row0 + row;
        if (g < ag.T)
          for (int r = 0; r < ag.world; ++r)
            *reinterpret_cast<bf16x8*>(ag.dst[r] + (size_t)g * H + col) = ov;
      } else {
        *reinterpret_cast<bf16x8*>(out + base + col) = ov;
      }
    }
  }
  if (ag.world > 0) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int old = atomicAdd(ag.done, 1);
      if (old == (int)gridDim.x - 1) {
        *ag.done = 0;
        __threadfence_system();
        const int e = *ag.epoch;
        for (int r = 0; r < ag.world; ++r)   // ordered by the fence above; relaxed stores pipeline
          asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(ag.flag[r]), "r"(e) : "memory");
      }
    }
  }
}

// Add + RMSNorm of decode-sized batches without cross-GPU waits, one row per thread-block cluster
// of C CTAs: CTA r of a row takes columns [r H / C, (r + 1) H / C) (8 per thread), and the row's sum
// of squares is reduced across the cluster through distributed shared memory. With one CTA per row
// only T SMs would work (T = 32 decode rows against 148 SMs). Inputs: the bf16 parts summed, or the
// fp32 stream-K partials (PartialIn), or the flag-free all-reduce slots of every rank (lamport 1 /
// 2, as in rmsnorm_fused_kernel: each CTA polls only its own columns, bounded by wait_ns); the
// same rounding as rmsnorm_fused_kernel.
template <int C>
__global__ void __launch_bounds__(256) rmsnorm_cluster_kernel(
    PartPtrs parts, int nparts, const __nv_bfloat16* residual_in, __nv_bfloat16* residual_out,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H, float eps, const PartialIn pin,
    int lamport, uint64_t wait_ns, int* err) {
  __shared__ float red[32];
  __shared__ float cl_ss;
  if (lamport != 2) pdl_wait();
  pdl_trigger();
  bool gave_up = false;
  const int row = blockIdx.x / C;
  const uint32_t rank = cluster_rank();
  const int col = (int)rank * (H / C) + threadIdx.x * 8;
  const size_t base = (size_t)row * H;
  float v[8];
  float ss = 0.f;
  const bool on = col < (int)(rank + 1) * (H / C);
  if (on) {
    float acc[8];
    if (pin.part) {
      partial_sum<8>(pin, row, col, acc);
    } else if (lamport) {
      uint4 a4 = lamport_take(parts.p[0] + base + col, wait_ns, err, gave_up);
      unpack8(*reinterpret_cast<bf16x8*>(&a4), acc);
      for (int k = 1; k < nparts; ++k) {           // rank order: the same sum on every rank
        float t[8];
        uint4 t4 = lamport_take(parts.p[k] + base + col, wait_ns, err, gave_up);
        unpack8(*reinterpret_cast<bf16x8*>(&t4), t);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += t[i];
      }
    } else {
      unpack8(*reinterpret_cast<const bf16x8*>(parts.p[0] + base + col), acc);
      for (int k = 1; k < nparts; ++k) {
        float t[8];
        unpack8(*reinterpret_cast<const bf16x8*>(parts.p[k] + base + col), t);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += t[i];
      }
    }
    if (residual_in) {
      float r[8];
      unpack8(*reinterpret_cast<const bf16x8*>(residual_in + base + col), r);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += r[i];
    }
    const bf16x8 rounded = pack8(acc);
    unpack8(rounded, v);
    if (residual_out) *reinterpret_cast<bf16x8*>(residual_out + base + col) = rounded;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) cl_ss = ss;
  cluster_barrier();
  float tot = 0.f;
#pragma unroll
  for (int r = 0; r < C; ++r) tot += cluster_ld_f32(&cl_ss, (uint32_t)r);   // the same order in every CTA
  cluster_barrier();                        // no CTA leaves while another still reads its total
  const float inv = rsqrtf(tot / (float)H + eps);
  if (on) {
    float wf[8], o[8];
    unpack8(*reinterpret_cast<const bf16x8*>(w + col), wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __bfloat162float(__float2bfloat16_rn(v[i] * inv)) * wf[i];
    *reinterpret_cast<bf16x8*>(out + base + col) = pack8(o);
  }
}

// QKV post-processing of one (token, head slot) by one warp; head slots are
// [0, nq) query heads, [nq, nq+nkv) key heads, [nq+nkv, nq+2nkv) value heads.
// E = HD/32 elements per lane; the rotate-half partner of lane l is lane l^16.
// KVQ = 0: bf16 cache [blocks][nkv][16][HD]; KVQ = 1: int4g128 cache, codes
// [blocks][nkv][16][HD/2] (two 4-bit offset-binary values per byte, even dim in
// the low nibble) + fp16 scale per (token, head) in k_scale/v_scale [blocks][nkv][16].
template <int HD, int KVQ>
__device__ __forceinline__ void qkv_post_one(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ bias,
                                             const __nv_bfloat16* __restrict__ qn_w,
                                             const __nv_bfloat16* __restrict__ kn_w, const float* __restrict__ cos_sin,
                                             const int* __restrict__ positions, const int* __restrict__ slots,
                                             __nv_bfloat16* __restrict__ q_out, void* __restrict__ k_cache,
                                             void* __restrict__ v_cache, __half* __restrict__ k_scale,
                                             __half* __restrict__ v_scale, int nq, int nkv, float eps, int width,
                                             int rot, const PartialIn& pin, int cache_slots, int max_pos, int t, int h,
                                             int lane) {
  constexpr int E = HD / 32;
  const __nv_bfloat16* src = qkv + (size_t)t * width + h * HD + lane * E;
  float x[E];
  if (pin.part) partial_sum<E>(pin, t, h * HD + lane * E, x);
#pragma unroll
  for (int i = 0; i < E; ++i) {
    if (!pin.part) x[i] = __bfloat162float(src[i]);
    if (bias) x[i] = __bfloat162float(__float2bfloat16_rn(x[i] + __bfloat162float(bias[h * HD + lane * E + i])));
  }
  const bool is_q = h < nq, is_k = !is_q && h < nq + nkv;
  if (is_q || is_k) {
    const __nv_bfloat16* nw = is_q ? qn_w : kn_w;
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < E; ++i) ss += x[i] * x[i];
      const float inv = rsqrtf(warp_sum(ss) / (float)HD + eps);
#pragma unroll
      for (int i = 0; i < E; ++i)
        x[i] = __bfloat162float(__float2bfloat16_rn(x[i] * inv)) * __bfloat162float(nw[lane * E + i]);
#pragma unroll
      for (int i = 0; i < E; ++i) x[i] = __bfloat162float(__float2bfloat16_rn(x[i]));
    }
    // rotate-half RoPE over the first `rot` dims (pairs (d, d + rot/2)); the rest pass through.
    // The partner of dim d sits rot/2 dims away, i.e. in lane ^ (rot/2/E) (a power of two).
    const int pos = positions[t];
    if (!B200_IN_RANGE(pos, max_pos, 0x101)) return;
    const int hr = rot >> 1, xo = hr / E;
    const float* cs = cos_sin + (size_t)pos * rot;  // [cos(rot/2) | sin(rot/2)]
    float y[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[i], xo);
      const int d = lane * E + i;
      if (d < rot) {
        const int f = d & (hr - 1);
        const float c = cs[f], s = cs[hr + f];
        y[i] = d < hr ? x[i] * c - partner * s : x[i] * c + partner * s;
      } else {
        y[i] = x[i];
      }
    }
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = y[i];
  }
  if (is_q) {
    __nv_bfloat16* dst = q_out + ((size_t)t * nq + h) * HD + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = __float2bfloat16_rn(x[i]);
  } else {
    const int slot = slots[t];
    if (slot < 0 || !B200_IN_RANGE(slot, cache_slots, 0x102)) return;
    const int kvh = is_k ? h - nq : h - nq - nkv;
    const size_t row = ((size_t)(slot >> 4) * nkv + kvh) * 16 + (slot & 15);
    if constexpr (KVQ == 0) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(is_k ? k_cache : v_cache) + row * HD + lane * E;
#pragma unroll
      for (int i = 0; i < E; ++i) dst[i] = __float2bfloat16_rn(x[i]);
    } else {
      // symmetric 4-bit: scale = amax / 7, q = clamp(round(x / scale), -8, 7), stored as q + 8
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < E; ++i) amax = fmaxf(amax, fabsf(x[i]));
      amax = warp_max(amax);
      const float scale = amax > 0.f ? amax / 7.f : 1.f;
      const __half scale_h = __float2half_rn(scale);
      const float inv = 1.f / __half2float(scale_h);
      // (host side allows head_dim 128 only; this branch is compiled but unused for 64)
      // 8 dims per 32-bit word; dims (2p, 2p+1) of the group go to nibbles (p, p + 4) so the
      // reader turns a nibble pair into a bf16 pair with one mask-and-or
      uint32_t part = 0;
      const int base = (lane & 1) * 4;   // this lane holds dims 4l..4l+3 = group offsets base..base+3
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const uint32_t q = (uint32_t)(max(-8, min(7, __float2int_rn(x[i] * inv))) + 8);
        const int o = base + i, pr = o >> 1, hi = o & 1;
        part |= q << (4 * (pr + 4 * hi));
      }
      const uint32_t word = part | __shfl_xor_sync(0xffffffffu, part, 1);
      uint32_t* codes = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(is_k ? k_cache : v_cache) +
                                                    row * (HD / 2));
      if ((lane & 1) == 0) codes[lane >> 1] = word;
      if (lane == 0) (is_k ? k_scale : v_scale)[row] = scale_h;
    }
  }
}

// One warp per (token, HPW consecutive head slots): HPW = 1 for decode-sized steps (most warps in
// flight), 8 for prefill chunks (the token's position and rotary table are read once per warp and
// the heads' loads overlap).
template <int HD, int KVQ, int HPW>
__global__ void qkv_post_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ bias,
                                const __nv_bfloat16* __restrict__ qn_w, const __nv_bfloat16* __restrict__ kn_w,
                                const float* __restrict__ cos_sin, const int* __restrict__ positions,
                                const int* __restrict__ slots, __nv_bfloat16* __restrict__ q_out,
                                void* __restrict__ k_cache, void* __restrict__ v_cache, __half* __restrict__ k_scale,
                                __half* __restrict__ v_scale, int T, int nq, int nkv, float eps, int width, int rot,
                                const PartialIn pin, int cache_slots, int max_pos) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nslots = nq + 2 * nkv;
  const int groups = (nslots + HPW - 1) / HPW;
  if (warp >= T * groups) return;
  const int t = warp / groups, h0 = (warp % groups) * HPW;
#pragma unroll
  for (int i = 0; i < HPW; ++i)
    if (h0 + i < nslots)
      qkv_post_one<HD, KVQ>(qkv, bias, qn_w, kn_w, cos_sin, positions, slots, q_out, k_cache, v_cache, k_scale,
                            v_scale, nq, nkv, eps, width, rot, pin, cache_slots, max_pos, t, h0 + i, lane);
}

// act[t, j] = silu(g) * u where the gate/up GEMM output interleaves 64-wide
// column blocks: [g(0..63) u(0..63) g(64..127) u(64..127) ...].
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ act, int T,
                                int I) {
  pdl_wait();
  pdl_trigger();
  const size_t n8 = (size_t)T * I / 8;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < n8; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    const size_t t = e / I;
    const int j = (int)(e % I);
    const int blk = j >> 6, within = j & 63;
    const __nv_bfloat16* row = gu + t * 2 * (size_t)I;
    float g[8], u[8], o[8];
    unpack8(*reinterpret_cast<const bf16x8*>(row + blk * 128 + within), g);
    unpack8(*reinterpret_cast<const bf16x8*>(row + blk * 128 + 64 + within), u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float gg = __bfloat162float(__float2bfloat16_rn(g[i] / (1.f + __expf(-g[i]))));
      o[i] = gg * u[i];
    }
    *reinterpret_cast<bf16x8*>(act + e) = pack8(o);
  }
}

__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int H, int vocab) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int id = ids[t];
  (void)B200_IN_RANGE(id, vocab, 0x103);
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const bf16x8* src = reinterpret_cast<const bf16x8*>(table + (size_t)id * H);
  bf16x8* dst = reinterpret_cast<bf16x8*>(out + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

}  // namespace b200

using namespace b200;

void rmsnorm_fused_impl(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                        c10::optional<torch::Tensor> residual_out, torch::Tensor w, torch::Tensor out, double eps,
                        const int* wait_flags, const int* epoch, int* err, const AgArgs& ag, int lamport = 0,
                        const PartialIn& pin = PartialIn{}, int nflags = -1) {
  TORCH_CHECK(!parts.empty() && parts.size() <= 8, "1..8 partial inputs");
  const int H = parts[0].size(-1);
  const int T = parts[0].numel() / H;
  TORCH_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  PartPtrs pp{};
  for (size_t i = 0; i < parts.size(); ++i) {
    TORCH_CHECK(parts[i].is_contiguous() && parts[i].scalar_type() == at::kBFloat16);
    pp.p[i] = reinterpret_cast<const __nv_bfloat16*>(parts[i].data_ptr());
  }
  if (T == 0) return;
  int threads = std::min(1024, ((H / 8 + 31) / 32) * 32);
  const int vpt = (H / 8 + threads - 1) / threads;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto rin = residual_in ? reinterpret_cast<const __nv_bfloat16*>(residual_in->data_ptr()) : nullptr;
  auto rout = residual_out ? reinterpret_cast<__nv_bfloat16*>(residual_out->data_ptr()) : nullptr;
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  // decode-sized batches without cross-GPU waits: a cluster of C CTAs per row (see the kernel);
  // B200_NORM_CLUSTER overrides C (1: one CTA per row)
  static const int cl_env = [] { const char* e = getenv("B200_NORM_CLUSTER"); return e ? atoi(e) : -1; }();
  int C = T <= 18 ? 8 : T <= 37 ? 4 : T <= 74 ? 2 : 1;
  if (cl_env >= 0) C = cl_env;
  // the flag-free (lamport) receive slots take the cluster path only with B200_NORM_CLUSTER_LAMPORT=1:
  // measured at TP2 (8B, batch 32) it was 1.4% slower (7743 against 7850 tok/s), four times as many
  // CTAs polling the slots while the pushing GEMM still runs
  static const bool cl_lamport = [] { const char* e = getenv("B200_NORM_CLUSTER_LAMPORT"); return e && atoi(e) != 0; }();
  if (!wait_flags && (!lamport || cl_lamport) && ag.world == 0 && (C == 2 || C == 4 || C == 8) &&
      H % (8 * C) == 0 && H / (8 * C) <= 256) {
    const dim3 grid(T * C), block(((H / (8 * C)) + 31) / 32 * 32);
    const int np = (int)parts.size();
    const uint64_t wns = flag_wait_ns();
    switch (C) {
      case 8: launch_pdl_cluster(rmsnorm_cluster_kernel<8>, grid, block, 0, stream, 8, pp, np, rin, rout, wp, op, H, (float)eps, pin, lamport, wns, err); break;
      case 4: launch_pdl_cluster(rmsnorm_cluster_kernel<4>, grid, block, 0, stream, 4, pp, np, rin, rout, wp, op, H, (float)eps, pin, lamport, wns, err); break;
      default: launch_pdl_cluster(rmsnorm_cluster_kernel<2>, grid, block, 0, stream, 2, pp, np, rin, rout, wp, op, H, (float)eps, pin, lamport, wns, err); break;
    }
    B200_CHECK_CUDA(cudaGetLastError());
    return;
  }
  switch (vpt) {
    case 1: launch_pdl(rmsnorm_fused_kernel<1>, dim3(T), dim3(threads), 0, stream, pp, (int)parts.size(), rin, rout, wp, op, H, (float)eps, wait_flags, epoch, err, ag, flag_wait_ns(), lamport, pin, nflags < 0 ? (int)parts.size() : nflags); break;
    case 2: launch_pdl(rmsnorm_fused_kernel<2>, dim3(T), dim3(threads), 0, stream, pp, (int)parts.size(), rin, rout, wp, op, H, (float)eps, wait_flags, epoch, err, ag, flag_wait_ns(), lamport, pin, nflags < 0 ? (int)parts.size() : nflags); break;
    case 3:
    case 4: launch_pdl(rmsnorm_fused_kernel<4>, dim3(T), dim3(threads), 0, stream, pp, (int)parts.size(), rin, rout, wp, op, H, (float)eps, wait_flags, epoch, err, ag, flag_wait_ns(), lamport, pin, nflags < 0 ? (int)parts.size() : nflags); break;
    default: TORCH_CHECK(false, "hidden size too large");
  }
  B200_CHECK_CUDA(cudaGetLastError());
}

void rmsnorm_fused(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                   c10::optional<torch::Tensor> residual_out, torch::Tensor w, torch::Tensor out, double eps) {
  rmsnorm_fused_impl(parts, residual_in, residual_out, w, out, eps, nullptr, nullptr, nullptr, AgArgs{});
}

// Same, after waiting for the peers' flags of a fused all-reduce site
// (flags_ptr: this rank's [world] flag words of the site; one per part).
void rmsnorm_fused_wait(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                        c10::optional<torch::Tensor> residual_out, torch::Tensor w, torch::Tensor out, double eps,
                        int64_t flags_ptr, int64_t epoch_ptr, int64_t err_ptr, int64_t n_flags) {
  rmsnorm_fused_impl(parts, residual_in, residual_out, w, out, eps, reinterpret_cast<const int*>(flags_ptr),
                     reinterpret_cast<const int*>(epoch_ptr), reinterpret_cast<int*>(err_ptr), AgArgs{}, 0,
                     PartialIn{}, (int)n_flags);
}

// out = RMSNorm(sum of a stream-K GEMM's fp32 partials + residual) * w (see PartialIn);
// `like` is a bf16 [T, H] tensor that gives the row geometry (its data is not read).
void rmsnorm_partial(torch::Tensor like, torch::Tensor part, int64_t kb, int64_t ctas, int64_t total, int64_t tile,
                     c10::optional<torch::Tensor> residual_in, c10::optional<torch::Tensor> residual_out,
                     torch::Tensor w, torch::Tensor out, double eps) {
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous(), "partials: contiguous fp32");
  TORCH_CHECK(tile == 16 || tile == 128, "partial tiles are 16 or 128 columns wide");
  TORCH_CHECK((uint64_t)((like.size(1) + tile - 1) / tile) * (uint64_t)kb * (uint64_t)ctas < (1ull << 32),
              "stream-K plan too large for 32-bit slot arithmetic");
  PartialIn pin{part.data_ptr<float>(), (int)kb, (int)ctas, (long long)total, (int)like.size(0), (int)like.size(1),
                (int)tile};
  rmsnorm_fused_impl({like}, residual_in, residual_out, w, out, eps, nullptr, nullptr, nullptr, AgArgs{}, 0, pin);
}

// Consumer of a flag-free all-reduce site: parts are this rank's receive slots (one per source
// rank, filled with 0xFFFF while empty); every vector is polled until it has landed, summed in
// rank order and reset to empty. skip_prior_wait: the push GEMM was the launch right before.
void rmsnorm_lamport(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                     c10::optional<torch::Tensor> residual_out, torch::Tensor w, torch::Tensor out, double eps,
                     int64_t err_ptr, bool skip_prior_wait) {
  rmsnorm_fused_impl(parts, residual_in, residual_out, w, out, eps, nullptr, nullptr,
                     reinterpret_cast<int*>(err_ptr), AgArgs{}, skip_prior_wait ? 2 : 1);
}

// Reduce-scatter consumer + all-gather producer: waits for the partial rows of this rank's
// token shard (flags_ptr, 0 = no wait), normalises them, and stores row i as global row row0 + i
// (< T) into dst_ptrs[r] (int64 [world], every rank's gathered buffer), then raises
// ag_flag_ptrs[r] = epoch on every rank. done: int32 [1] counter, zero on entry.
void rmsnorm_rs_ag(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                   c10::optional<torch::Tensor> residual_out, torch::Tensor w, double eps, int64_t flags_ptr,
                   int64_t epoch_ptr, int64_t err_ptr, torch::Tensor dst_ptrs, torch::Tensor ag_flag_ptrs,
                   int64_t row0, int64_t T, torch::Tensor done, int64_t n_flags) {
  const int world = dst_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= 8 && ag_flag_ptrs.numel() == world && dst_ptrs.device().is_cpu() &&
                  ag_flag_ptrs.device().is_cpu(), "dst/flag pointer lists: host int64 [world]");
  AgArgs ag{};
  ag.world = world;
  ag.row0 = (int)row0;
  ag.T = (int)T;
  ag.done = done.data_ptr<int>();
  ag.epoch = reinterpret_cast<const int*>(epoch_ptr);
  for (int r = 0; r < world; ++r) {
    ag.dst[r] = reinterpret_cast<__nv_bfloat16*>(dst_ptrs.data_ptr<int64_t>()[r]);
    ag.flag[r] = reinterpret_cast<int*>(ag_flag_ptrs.data_ptr<int64_t>()[r]);
  }
  rmsnorm_fused_impl(parts, residual_in, residual_out, w, parts[0], eps,
                     flags_ptr ? reinterpret_cast<const int*>(flags_ptr) : nullptr,
                     reinterpret_cast<const int*>(epoch_ptr), reinterpret_cast<int*>(err_ptr), ag, 0, PartialIn{},
                     (int)n_flags);
}

void qkv_post_impl(torch::Tensor qkv, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> qn_w,
                   c10::optional<torch::Tensor> kn_w, torch::Tensor cos_sin, torch::Tensor positions,
                   torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache,
                   __half* k_scale, __half* v_scale, int64_t nq, int64_t nkv, double eps, int kvq,
                   const PartialIn& pin = PartialIn{}) {
  const int T = qkv.size(0);
  const int HD = q_out.size(2), rot = cos_sin.size(1);
  const int width = (int)qkv.stride(0);
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.size(1) >= (nq + 2 * nkv) * HD, "qkv width mismatch");
  const int hr = rot / 2, E = HD / 32;
  TORCH_CHECK(rot <= HD && rot % 2 == 0 && hr % E == 0 && ((hr / E) & (hr / E - 1)) == 0,
              "rotary dims must be <= head_dim with (rot/2)/(head_dim/32) a power of two");
  TORCH_CHECK(positions.scalar_type() == at::kInt && slots.scalar_type() == at::kInt);
  if (T == 0) return;
  const int hpw = T >= 128 ? 8 : 1;          // heads per warp: see qkv_post_kernel
  const int warps = T * ((int)(nq + 2 * nkv + hpw - 1) / hpw);
  const int threads = 256;
  const int blocks = (warps * 32 + threads - 1) / threads;
  auto stream = at::cuda::getCurrentCUDAStream();
#define B200_QKV(KERNEL)                                                                                   \
  launch_pdl(KERNEL, dim3(blocks), dim3(threads), 0, stream,                                                \
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),                                               \
      bias ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr,                            \
      qn_w ? reinterpret_cast<const __nv_bfloat16*>(qn_w->data_ptr()) : nullptr,                            \
      kn_w ? reinterpret_cast<const __nv_bfloat16*>(kn_w->data_ptr()) : nullptr, cos_sin.data_ptr<float>(), \
      positions.data_ptr<int>(), slots.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), \
      k_cache.data_ptr(), v_cache.data_ptr(), k_scale, v_scale, T, (int)nq, (int)nkv, (float)eps, width, rot, pin, \
      (int)(k_cache.size(0) * 16), (int)cos_sin.size(0))
#define B200_QKV2(HDV, KQV) { if (hpw == 8) B200_QKV((qkv_post_kernel<HDV, KQV, 8>)); else B200_QKV((qkv_post_kernel<HDV, KQV, 1>)); }
  if (HD == 128) { if (kvq) B200_QKV2(128, 1) else B200_QKV2(128, 0) }
  else if (HD == 64 && !kvq) B200_QKV2(64, 0)
  else if (HD == 256 && !kvq) B200_QKV2(256, 0)
  else TORCH_CHECK(false, "head_dim must be 64, 128 or 256 (int4 KV: 128)");
#undef B200_QKV2
#undef B200_QKV
  B200_CHECK_CUDA(cudaGetLastError());
}

void qkv_post(torch::Tensor qkv, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> qn_w,
              c10::optional<torch::Tensor> kn_w, torch::Tensor cos_sin, torch::Tensor positions,
              torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache, int64_t nq,
              int64_t nkv, double eps) {
  qkv_post_impl(qkv, bias, qn_w, kn_w, cos_sin, positions, slots, q_out, k_cache, v_cache, nullptr, nullptr, nq, nkv,
                eps, 0);
}

// qkv_post whose input rows are the fp32 stream-K partials of the QKV GEMM (see PartialIn);
// `like` [T, width] bf16 only gives the geometry. Scales given: int4g128 KV cache.
void qkv_post_partial(torch::Tensor like, torch::Tensor part, int64_t kb, int64_t ctas, int64_t total,
                      int64_t tile, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> qn_w,
                      c10::optional<torch::Tensor> kn_w, torch::Tensor cos_sin, torch::Tensor positions,
                      torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache,
                      c10::optional<torch::Tensor> k_scale, c10::optional<torch::Tensor> v_scale, int64_t nq,
                      int64_t nkv, double eps) {
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous(), "partials: contiguous fp32");
  TORCH_CHECK(like.stride(0) == like.size(1), "partials have the row stride of a dense [T, width] output");
  TORCH_CHECK(tile == 16 || tile == 128, "partial tiles are 16 or 128 columns wide");
  TORCH_CHECK((uint64_t)((like.size(1) + tile - 1) / tile) * (uint64_t)kb * (uint64_t)ctas < (1ull << 32),
              "stream-K plan too large for 32-bit slot arithmetic");
  PartialIn pin{part.data_ptr<float>(), (int)kb, (int)ctas, (long long)total, (int)like.size(0), (int)like.size(1),
                (int)tile};
  const bool q4 = k_scale.has_value();
  qkv_post_impl(like, bias, qn_w, kn_w, cos_sin, positions, slots, q_out, k_cache, v_cache,
                q4 ? reinterpret_cast<__half*>(k_scale->data_ptr()) : nullptr,
                q4 ? reinterpret_cast<__half*>(v_scale->data_ptr()) : nullptr, nq, nkv, eps, q4 ? 1 : 0, pin);
}

// Same, writing K/V into an int4g128 cache (codes + fp16 scales).
void qkv_post_q4(torch::Tensor qkv, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> qn_w,
                 c10::optional<torch::Tensor> kn_w, torch::Tensor cos_sin, torch::Tensor positions,
                 torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_codes, torch::Tensor v_codes,
                 torch::Tensor k_scale, torch::Tensor v_scale, int64_t nq, int64_t nkv, double eps) {
  TORCH_CHECK(cos_sin.size(1) == 128, "int4g128 KV cache needs head_dim 128");
  qkv_post_impl(qkv, bias, qn_w, kn_w, cos_sin, positions, slots, q_out, k_codes, v_codes,
                reinterpret_cast<__half*>(k_scale.data_ptr()), reinterpret_cast<__half*>(v_scale.data_ptr()), nq, nkv,
                eps, 1);
}

void silu_mul(torch::Tensor gu, torch::Tensor act) {
  const int I = act.size(-1);
  const int T = act.numel() / I;
  TORCH_CHECK(I % 64 == 0 && gu.size(-1) == 2 * I);
  if (T == 0) return;
  const size_t n8 = (size_t)T * I / 8;
  const int threads = 256;
  const int blocks = (int)std::min<size_t>((n8 + threads - 1) / threads, 148 * 16);
  launch_pdl(silu_mul_kernel, dim3(blocks), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<__nv_bfloat16*>(act.data_ptr()), T, I);
  B200_CHECK_CUDA(cudaGetLastError());
}

void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out) {
  const int T = ids.numel();
  const int H = table.size(1);
  if (T == 0) return;
  launch_pdl(embedding_kernel, dim3(T), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
             (const int*)ids.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H, (int)table.size(0));
  B200_CHECK_CUDA(cudaGetLastError());
}

B200_BOUNDS_ACCESSOR(norm_rope)
