// GGUF block-quantised GEMV for decode batches of 1..16 tokens.
//
// The unit of work is a warp task: one 16-row slice of the weight times a contiguous range of
// 256-column chunks of K (k split s of S). A warp streams its slice's fragment-ordered codes
// (the repack of models/gguf.py: one 32-bit word of 4-bit codes, or two of 8-bit codes, per
// lane per 16-column k-step) with two chunks of loads in flight, dequantises them in registers
// (gguf_common.cuh) and runs mma.sync m16n8k16 with the activations as the B operand, read
// straight from global memory (a decode batch is a few KB and stays in L1/L2): no shared-memory
// staging and no barrier between loading and computing. Outputs:
//   QV_BF16 / QV_F32  S == 1, out[t][col0 + n]
//   QV_PARTIAL       fp32 part[s][t][col0 + n]; the consuming row kernel (RMSNorm, qkv_post,
//                    silu_mul_partial) sums the S slots (PartialIn with S slots per tile)
//   QV_PUSH          S == 1, bf16 tile stored into every rank's flag-free all-reduce slot
//                    (P2P, or one multimem store through an NVLink multicast object)
//
// Reference kernels restated: webgpu/src/shaders/matmul_gguf.wgsl:2103-3310 (q4_k / q6_k / q8_0
// matmuls), with the weight repack of webgpu/src/model/gguf-dequant.ts:152-406.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "gguf_common.cuh"

namespace b200 {

enum QvOut : int { QV_BF16 = 0, QV_F32 = 1, QV_PARTIAL = 2, QV_PUSH = 4 };

constexpr int kVWarps = 8;          // warps (tasks) per CTA
constexpr int kVSteps = 16;         // k-steps of 16 columns per chunk (one 256-column super-block)

struct QvArgs {
  const uint32_t* codes;
  const uint32_t* meta;
  const __nv_bfloat16* x;
  int ldx, M, N, K, group, S;
  void* out;
  int ldo, col0;                    // output row stride (elements) and first column of this matrix
  float* part;
  long long part_slot;              // floats between partial slots (M * ldo)
  __nv_bfloat16* push[8];           // QV_PUSH: this rank's slot base on every rank (row stride ldo)
  int world;
  __nv_bfloat16* mc;                // QV_PUSH through multicast: this rank's slot, multicast address
};

// B fragment of m16n8k16 for token `tok`: columns k + 2*t4 (+1) and k + 8 + 2*t4 (+1)
__device__ __forceinline__ void x_frag(const QvArgs& a, int tok, int k, uint32_t& b0, uint32_t& b1) {
  if (tok < a.M) {
    const __nv_bfloat16* p = a.x + (size_t)tok * a.ldx + k;
    b0 = __ldg(reinterpret_cast<const uint32_t*>(p));
    b1 = __ldg(reinterpret_cast<const uint32_t*>(p + 8));
  } else {
    b0 = b1 = 0u;
  }
}

// ---- 4-bit (Q4_K): codes [slices][K/16][32] u32, meta [slices][K/32][16 rows][2] (scale, -min)
struct Q4Regs {
  uint32_t cw[kVSteps];
  uint32_t mt[kVSteps / 2][4];
};

__device__ __forceinline__ void q4_load(const QvArgs& a, int slice, int chunk, int lane, Q4Regs& r) {
  const int g = lane >> 2;
  const int ksteps = a.K / 16, ks0 = chunk * kVSteps;
#pragma unroll
  for (int ks = 0; ks < kVSteps; ++ks) r.cw[ks] = __ldg(a.codes + ((size_t)slice * ksteps + ks0 + ks) * 32 + lane);
#pragma unroll
  for (int sb = 0; sb < kVSteps / 2; ++sb) {
    const uint32_t* mp = a.meta + ((size_t)slice * (a.K / 32) + ks0 / 2 + sb) * 32;
    r.mt[sb][0] = __ldg(mp + g * 2);
    r.mt[sb][1] = __ldg(mp + g * 2 + 1);
    r.mt[sb][2] = __ldg(mp + (g + 8) * 2);
    r.mt[sb][3] = __ldg(mp + (g + 8) * 2 + 1);
  }
}

template <int NB>
__device__ __forceinline__ void q4_mma(const QvArgs& a, const Q4Regs& r, int chunk, int lane, float (&acc)[NB][4]) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int ks = 0; ks < kVSteps; ++ks) {
    uint32_t w[4];
    dequant_u4(r.cw[ks], r.mt[ks / 2][0], r.mt[ks / 2][1], r.mt[ks / 2][2], r.mt[ks / 2][3], w);
    const int k = (chunk * kVSteps + ks) * 16 + 2 * t4;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      uint32_t b0, b1;
      x_frag(a, j * 8 + g, k, b0, b1);
      qmma(acc[j], w, b0, b1);
    }
  }
}

// ---- 8-bit (Q6_K / Q8_0 repacked): codes [slices][K/16][32] uint2, scales [slices][K/group][16]
struct Q8Regs {
  uint2 cw[kVSteps];
  uint32_t sc[kVSteps][2];
};

__device__ __forceinline__ void q8_load(const QvArgs& a, int slice, int chunk, int lane, Q8Regs& r) {
  const int g = lane >> 2;
  const int ksteps = a.K / 16, ks0 = chunk * kVSteps;
#pragma unroll
  for (int ks = 0; ks < kVSteps; ++ks)
    r.cw[ks] = __ldg(reinterpret_cast<const uint2*>(a.codes) + ((size_t)slice * ksteps + ks0 + ks) * 32 + lane);
#pragma unroll
  for (int ks = 0; ks < kVSteps; ++ks) {
    // the group holding k-step ks (group 16: one per step; group 32: one per two steps)
    const int gi = (ks0 * 16 + ks * 16) / a.group;
    if (a.group == 16 || (ks & 1) == 0) {
      const uint32_t* sp = a.meta + ((size_t)slice * (a.K / a.group) + gi) * 16;
      r.sc[ks][0] = __ldg(sp + g);
      r.sc[ks][1] = __ldg(sp + g + 8);
    } else {
      r.sc[ks][0] = r.sc[ks - 1][0];
      r.sc[ks][1] = r.sc[ks - 1][1];
    }
  }
}

template <int NB>
__device__ __forceinline__ void q8_mma(const QvArgs& a, const Q8Regs& r, int chunk, int lane, float (&acc)[NB][4]) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int ks = 0; ks < kVSteps; ++ks) {
    uint32_t w[4];
    dequant_s8(r.cw[ks].x, r.cw[ks].y, r.sc[ks][0], r.sc[ks][1], w);
    const int k = (chunk * kVSteps + ks) * 16 + 2 * t4;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      uint32_t b0, b1;
      x_frag(a, j * 8 + g, k, b0, b1);
      qmma(acc[j], w, b0, b1);
    }
  }
}

// Chunks [c0, c1) of one slice, two chunks of loads in flight.
template <int BITS, int NB>
__device__ __forceinline__ void run_chunks(const QvArgs& a, int slice, int c0, int c1, int lane,
                                           float (&acc)[NB][4]) {
  if constexpr (BITS == 4) {
    Q4Regs r0, r1;
    int c = c0;
    if (c < c1) q4_load(a, slice, c, lane, r0);
    while (c < c1) {
      if (c + 1 < c1) q4_load(a, slice, c + 1, lane, r1);
      q4_mma<NB>(a, r0, c, lane, acc);
      if (++c >= c1) break;
      if (c + 1 < c1) q4_load(a, slice, c + 1, lane, r0);
      q4_mma<NB>(a, r1, c, lane, acc);
      ++c;
    }
  } else {
    Q8Regs r0, r1;
    int c = c0;
    if (c < c1) q8_load(a, slice, c, lane, r0);
    while (c < c1) {
      if (c + 1 < c1) q8_load(a, slice, c + 1, lane, r1);
      q8_mma<NB>(a, r0, c, lane, acc);
      if (++c >= c1) break;
      if (c + 1 < c1) q8_load(a, slice, c + 1, lane, r0);
      q8_mma<NB>(a, r1, c, lane, acc);
      ++c;
    }
  }
}

template <int BITS, int NB, int MODE>
__global__ void __launch_bounds__(kVWarps * 32) gguf_gemv_kernel(const QvArgs a) {
  __shared__ __align__(16) __nv_bfloat16 stage[kVWarps][16][16];   // QV_PUSH: [token][col] of a warp's tile
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int slices = a.N / 16, nchunks = a.K / 256;
  const int task = blockIdx.x * kVWarps + warp;
  if (task >= slices * a.S) return;
  const int slice = task / a.S, s = task % a.S;
  const int c0 = (int)((long long)s * nchunks / a.S), c1 = (int)((long long)(s + 1) * nchunks / a.S);
  float acc[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  run_chunks<BITS, NB>(a, slice, c0, c1, lane, acc);
  // acc[j]: rows (g, g, g+8, g+8) of the slice, tokens (j*8 + 2*t4, +1, +0, +1)
  const int n0 = a.col0 + slice * 16;
  if constexpr (MODE == QV_PUSH) {
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = j * 8 + 2 * t4 + (e & 1), row = g + (e >> 1) * 8;
        __nv_bfloat16 h = __float2bfloat16_rn(acc[j][e]);
        // 0xFFFF marks an empty flag-free slot; a NaN with that payload is stored as 0x7FFF
        if (__bfloat16_as_ushort(h) == 0xFFFFu) h = __ushort_as_bfloat16((unsigned short)0x7FFFu);
        stage[warp][tok][row] = h;
      }
    }
    __syncwarp();
    // 16 columns x 2 bytes = two 16-byte pieces per token
    if (lane < 2 * a.M) {
      const int tok = lane >> 1, half = lane & 1;
      const uint4 v = *reinterpret_cast<const uint4*>(&stage[warp][tok][half * 8]);
      const size_t off = (size_t)tok * a.ldo + n0 + half * 8;
      if (a.mc) {
        asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};"
                     ::"l"(a.mc + off), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
      } else {
        for (int r = 0; r < a.world; ++r) *reinterpret_cast<uint4*>(a.push[r] + off) = v;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = j * 8 + 2 * t4 + (e & 1), n = n0 + g + (e >> 1) * 8;
        if (tok >= a.M) continue;
        if constexpr (MODE == QV_PARTIAL)
          a.part[(size_t)s * a.part_slot + (size_t)tok * a.ldo + n] = acc[j][e];
        else if constexpr (MODE == QV_F32)
          reinterpret_cast<float*>(a.out)[(size_t)tok * a.ldo + n] = acc[j][e];
        else
          reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)tok * a.ldo + n] = __float2bfloat16_rn(acc[j][e]);
      }
    }
  }
}

// Block-quantised weight -> bf16 in the tile-packed layout of the tcgen05 GEMM
// ([N/128][K/64][128][64]), for prefill-sized batches: one warp per (slice, k-step), each lane
// dequantises its fragment (rows g, g+8 x columns 2t, 2t+1, 2t+8, 2t+9) and stores four bf16 pairs.
template <int BITS>
__global__ void gguf_dequant_packed_kernel(const uint32_t* __restrict__ codes, const uint32_t* __restrict__ meta,
                                           int N, int K, int group, __nv_bfloat16* __restrict__ out,
                                           const uint32_t* __restrict__ e8cb) {   // E8 codebook or IQ4 pair table
  // No early launch of the dependent: the GEMM that reads this weight streams its first weight
  // tiles before its own dependency wait, so it must start only after this grid has finished.
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int ksteps = K / 16;
  const long long task = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (task >= (long long)(N / 16) * ksteps) return;
  const int slice = (int)(task / ksteps), ks = (int)(task % ksteps);
  uint32_t a[4];
  if constexpr (BITS == 2) {
    // E8: the four codebook indices of the lane's row pair, (s, o) of rows g and g + 8
    const uint32_t q = __ldg(codes + ((size_t)slice * ksteps + ks) * 8 + g);
    const uint2* mp = reinterpret_cast<const uint2*>(meta) + ((size_t)slice * (K / group) + (ks * 16) / group) * 16;
    const uint2 ma = __ldg(mp + g), mc = __ldg(mp + g + 8);
    const uint32_t idx[4] = {q & 255u, (q >> 8) & 255u, (q >> 16) & 255u, q >> 24};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      a[i] = bf2_fma(__ldg(e8cb + idx[i] * 4 + t4), (i & 1) ? mc.x : ma.x, (i & 1) ? mc.y : ma.y);
  } else if constexpr (BITS == 5) {
    // IQ4: byte i = register i's pair of indices into the pair table (e8cb here), times the scale
    const uint32_t w = __ldg(codes + ((size_t)slice * ksteps + ks) * 32 + lane);
    const uint32_t* mp = meta + ((size_t)slice * (K / 32) + ks / 2) * 32;
    const uint32_t sa = __ldg(mp + g * 2), sb = __ldg(mp + (g + 8) * 2);
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = bf2_fma(__ldg(e8cb + ((w >> (8 * i)) & 255u)), (i & 1) ? sb : sa, 0u);
  } else if constexpr (BITS == 4) {
    const uint32_t w = __ldg(codes + ((size_t)slice * ksteps + ks) * 32 + lane);
    const uint32_t* mp = meta + ((size_t)slice * (K / 32) + ks / 2) * 32;
    dequant_u4(w, __ldg(mp + g * 2), __ldg(mp + g * 2 + 1), __ldg(mp + (g + 8) * 2), __ldg(mp + (g + 8) * 2 + 1), a);
  } else {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(codes) + ((size_t)slice * ksteps + ks) * 32 + lane);
    const uint32_t* sp = meta + ((size_t)slice * (K / group) + (ks * 16) / group) * 16;
    dequant_s8(w.x, w.y, __ldg(sp + g), __ldg(sp + g + 8), a);
  }
  const int kblocks = K / 64;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = slice * 16 + g + (i & 1) * 8;
    const int k = ks * 16 + 2 * t4 + (i >> 1) * 8;
    const size_t idx = ((size_t)(n / 128) * kblocks + k / 64) * (128 * 64) + (size_t)(n % 128) * 64 + (k % 64);
    *reinterpret_cast<uint32_t*>(out + idx) = a[i];
  }
}

}  // namespace b200

using namespace b200;

// codes/meta (N x K, N % 128 == 0, K % 64 == 0) -> out bf16 [N/128 * K/64 * 128, 64] tile-packed.
void gguf_dequant_packed(torch::Tensor codes, torch::Tensor meta, int64_t N, int64_t K, int64_t bits, int64_t group,
                         torch::Tensor out, int64_t table) {
  TORCH_CHECK(N % 128 == 0 && K % 256 == 0, "tile-packed dequantisation needs N % 128 == 0 and K % 256 == 0");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.numel() >= N * K, "output too small");
  const long long tasks = (N / 16) * (K / 16);
  const int threads = 256;
  const dim3 grid((unsigned)((tasks + 7) / 8));
  auto cp = reinterpret_cast<const uint32_t*>(codes.data_ptr());
  auto mp = reinterpret_cast<const uint32_t*>(meta.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto cbp = reinterpret_cast<const uint32_t*>(table);
  if (bits == 2) {
    TORCH_CHECK(cbp != nullptr && (group == 32 || group == 64 || group == 128 || group == 256), "E8: codebook, group");
    launch_pdl(gguf_dequant_packed_kernel<2>, grid, dim3(threads), 0, at::cuda::getCurrentCUDAStream(), cp, mp,
               (int)N, (int)K, (int)group, op, cbp);
  } else if (bits == 5) {
    TORCH_CHECK(cbp != nullptr, "IQ4: pair table");
    launch_pdl(gguf_dequant_packed_kernel<5>, grid, dim3(threads), 0, at::cuda::getCurrentCUDAStream(), cp, mp,
               (int)N, (int)K, (int)group, op, cbp);
  } else if (bits == 4)
    launch_pdl(gguf_dequant_packed_kernel<4>, grid, dim3(threads), 0, at::cuda::getCurrentCUDAStream(), cp, mp,
               (int)N, (int)K, (int)group, op, cbp);
  else
    launch_pdl(gguf_dequant_packed_kernel<8>, grid, dim3(threads), 0, at::cuda::getCurrentCUDAStream(), cp, mp,
               (int)N, (int)K, (int)group, op, cbp);
}

// K splits for a matrix of N / 16 slices and K / 256 chunks: about two waves of warp tasks over
// 148 SMs x 8 resident warps, with at least two chunks per task so that the two-chunk load
// pipeline has something to overlap.
int64_t gguf_gemv_splits(int64_t N, int64_t K) {
  const int64_t slices = N / 16, nchunks = K / 256;
  const int64_t want = 2 * 148 * kVWarps;
  return std::max<int64_t>(1, std::min<int64_t>(nchunks / 2, (want + slices - 1) / slices));
}

// mode: 0 bf16, 1 fp32 (S must be 1), 2 partial (out = fp32 part [S][M][ldo]), 4 push.
// x [M, K] bf16 (M <= 16); codes/meta from the repack; col0/ldo place this matrix's columns.
void gguf_gemv(torch::Tensor x, torch::Tensor codes, torch::Tensor meta, int64_t N, int64_t bits, int64_t group,
               int64_t mode, int64_t S, torch::Tensor out, int64_t ldo, int64_t col0, torch::Tensor push_ptrs,
               int64_t mc_ptr) {
  const int M = x.size(0), K = x.size(1);
  TORCH_CHECK(M >= 1 && M <= 16, "gguf_gemv serves decode batches of 1..16 tokens");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && (x.stride(0) % 8) == 0,
              "x: bf16 rows, 16-byte aligned");
  TORCH_CHECK(K % 256 == 0 && N % 16 == 0, "K must be a multiple of 256 and N of 16");
  TORCH_CHECK(group == 16 || group == 32, "group must be 16 or 32");
  TORCH_CHECK(S >= 1 && S <= K / 256 && (mode == QV_PARTIAL || S == 1), "bad k split");
  QvArgs a{};
  a.codes = reinterpret_cast<const uint32_t*>(codes.data_ptr());
  a.meta = reinterpret_cast<const uint32_t*>(meta.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = (int)x.stride(0);
  a.M = M; a.N = (int)N; a.K = K; a.group = (int)group; a.S = (int)S;
  a.ldo = (int)ldo; a.col0 = (int)col0;
  if (mode == QV_PARTIAL) {
    TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() >= S * (int64_t)M * ldo, "partial buffer too small");
    a.part = out.data_ptr<float>();
    a.part_slot = (long long)M * ldo;
  } else if (mode == QV_PUSH) {
    const int world = push_ptrs.numel();
    TORCH_CHECK(world >= 1 && world <= 8 && push_ptrs.device().is_cpu(), "push pointers: host int64 [world]");
    TORCH_CHECK((ldo % 8) == 0 && (col0 % 8) == 0, "push rows must stay 16-byte aligned");
    a.world = world;
    for (int r = 0; r < world; ++r) a.push[r] = reinterpret_cast<__nv_bfloat16*>(push_ptrs.data_ptr<int64_t>()[r]);
    a.mc = reinterpret_cast<__nv_bfloat16*>(mc_ptr);
  } else {
    TORCH_CHECK(out.scalar_type() == (mode == QV_F32 ? at::kFloat : at::kBFloat16), "output dtype");
    a.out = out.data_ptr();
  }
  const int tasks = (int)(N / 16) * (int)S;
  const dim3 grid((tasks + kVWarps - 1) / kVWarps), block(kVWarps * 32);
  auto stream = at::cuda::getCurrentCUDAStream();
#define B200_QV(BITSV, NBV, MODEV) launch_pdl(gguf_gemv_kernel<BITSV, NBV, MODEV>, grid, block, 0, stream, a)
#define B200_QV_MODES(BITSV, NBV)                                      \
  switch (mode) {                                                     \
    case QV_BF16: B200_QV(BITSV, NBV, QV_BF16); break;                \
    case QV_F32: B200_QV(BITSV, NBV, QV_F32); break;                  \
    case QV_PARTIAL: B200_QV(BITSV, NBV, QV_PARTIAL); break;          \
    case QV_PUSH: B200_QV(BITSV, NBV, QV_PUSH); break;                \
    default: TORCH_CHECK(false, "bad gguf_gemv mode");                \
  }
  if (bits == 4) {
    if (M <= 8) { B200_QV_MODES(4, 1) } else { B200_QV_MODES(4, 2) }
  } else {
    TORCH_CHECK(bits == 8, "bits must be 4 or 8");
    if (M <= 8) { B200_QV_MODES(8, 1) } else { B200_QV_MODES(8, 2) }
  }
#undef B200_QV_MODES
#undef B200_QV
  B200_CHECK_CUDA(cudaGetLastError());
}

