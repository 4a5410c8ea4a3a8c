// GGUF block-quantised GEMM for decode-sized batches (M <= 32 tokens):
//   out[m, n] = sum_k x[m, k] * W[n, k],  W in Q4_K (4-bit, scale+min per 32)
//   or in 8-bit codes with a scale per 16/32 (Q6_K, Q8_0 repacked).
//
// Restates the arithmetic of the reference's GGUF matmul shaders
// (webgpu/src/shaders/matmul_gguf.wgsl:2103-3310, q4_k/q6_k/q8_0 variants) on
// tensor cores: weights are repacked once at load time into "fragment order":
// for every 16-row x 16-column tile, lane (g, t) of a warp owns the 8 weights
// (rows g, g+8) x (cols 2t, 2t+1, 2t+8, 2t+9) of the m16n8k16 A operand, stored
// as one 32-bit word of codes (4-bit) or two (8-bit). The kernel loads that
// word, dequantises it in registers (bf16 magic-number conversion, then
// q * scale - min with one HFMA2 per register) and issues mma.sync with the
// activations (staged in shared memory) as the B operand, tokens on the N side.
// Each warp covers 16 output rows and a 256-wide K chunk; the warps of a CTA
// split K and are reduced through shared memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "gguf_common.cuh"

namespace b200 {

constexpr int kQWarps = 8;       // K chunks per CTA pass
constexpr int kQChunk = 256;     // K per warp chunk = 16 MMA k-steps
constexpr int kQStage = 2048;    // K columns of the activations staged in shared memory at a time

// Chunk of 256 K columns for one warp: all codes and scales are loaded into registers before the
// MMAs, so a warp keeps ~1 KB of independent loads in flight.
template <int BITS, int NB>
__device__ __forceinline__ void gguf_chunk(const uint32_t* __restrict__ codes, const uint32_t* __restrict__ smeta,
                                           const __nv_bfloat16* xs, int LDX, int slice, int ksteps, int K, int group,
                                           int k0, int kc0, int lane, float (&acc)[NB][4]) {
  constexpr int KS = kQChunk / 16;                           // 16 k-steps per chunk
  const int g = lane >> 2, t4 = lane & 3;
  const int ks0 = k0 / 16;
  if constexpr (BITS == 4) {
    uint32_t cw[KS];
    uint32_t mt[KS / 2][4];                                  // per 32-wide sub-block: sA, mA, sB, mB
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) cw[ks] = __ldg(codes + ((size_t)slice * ksteps + ks0 + ks) * 32 + lane);
#pragma unroll
    for (int sb = 0; sb < KS / 2; ++sb) {
      const uint32_t* mp = smeta + ((size_t)slice * (K / 32) + (ks0 / 2 + sb)) * 32;
      mt[sb][0] = __ldg(mp + g * 2);
      mt[sb][1] = __ldg(mp + g * 2 + 1);
      mt[sb][2] = __ldg(mp + (g + 8) * 2);
      mt[sb][3] = __ldg(mp + (g + 8) * 2 + 1);
    }
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t a[4];
      dequant_u4(cw[ks], mt[ks / 2][0], mt[ks / 2][1], mt[ks / 2][2], mt[ks / 2][3], a);
      const int kk = (ks0 + ks) * 16 - kc0 + 2 * t4;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const __nv_bfloat16* xr = xs + (size_t)(j * 8 + g) * LDX + kk;
        qmma(acc[j], a, *reinterpret_cast<const uint32_t*>(xr), *reinterpret_cast<const uint32_t*>(xr + 8));
      }
    }
  } else {
    uint2 cw[KS];
    constexpr int GPC = kQChunk / 16;                        // max groups per chunk (group >= 16)
    uint32_t sc[GPC][2];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
      cw[ks] = __ldg(reinterpret_cast<const uint2*>(codes) + ((size_t)slice * ksteps + ks0 + ks) * 32 + lane);
    const int ngr = kQChunk / group;
#pragma unroll
    for (int gi = 0; gi < GPC; ++gi) {
      if (gi < ngr) {
        const uint32_t* sp = smeta + ((size_t)slice * (K / group) + (k0 / group + gi)) * 16;
        sc[gi][0] = __ldg(sp + g);
        sc[gi][1] = __ldg(sp + g + 8);
      }
    }
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t a[4];
      const bool g16 = group == 16;                          // both indices are compile-time
      dequant_s8(cw[ks].x, cw[ks].y, g16 ? sc[ks][0] : sc[ks / 2][0], g16 ? sc[ks][1] : sc[ks / 2][1], a);
      const int kk = (ks0 + ks) * 16 - kc0 + 2 * t4;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const __nv_bfloat16* xr = xs + (size_t)(j * 8 + g) * LDX + kk;
        qmma(acc[j], a, *reinterpret_cast<const uint32_t*>(xr), *reinterpret_cast<const uint32_t*>(xr + 8));
      }
    }
  }
}

// BITS = 4 (Q4_K: codes [N/16][K/16][32] u32, scale/min [N/16][K/32][16 rows] bf16x2 (s, -m))
// BITS = 8 (codes [N/16][K/16][32][2] u32, scales [N/16][K/GROUP][16] bf16)
// A CTA covers NB 16-row slices (more tokens -> more slices share one staged activation block);
// warp w works on slice w % NB and every (8/NB)-th 256-column chunk of each staged block.
template <int BITS, int NB>
__global__ void __launch_bounds__(kQWarps * 32) gguf_gemm_kernel(
    const uint32_t* __restrict__ codes, const uint32_t* __restrict__ smeta, const __nv_bfloat16* __restrict__ x,
    int M, int N, int K, int group, __nv_bfloat16* __restrict__ out, int ldo) {
  constexpr int SPC = NB, NPH = kQWarps / SPC;
  extern __shared__ __align__(16) uint8_t smem[];
  const int KC = min(K, kQStage);                          // K columns of x staged at a time
  const int LDX = KC + 8;                                  // padded row: conflict-free B fragments
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);   // [NB*8][LDX]
  float* red = reinterpret_cast<float*>(smem + (size_t)NB * 8 * LDX * 2);   // [warps][16][NB*8]
  const int rows_tok = NB * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int nslices = N / 16;
  const int slice = blockIdx.x * SPC + warp % SPC;          // 16 output rows
  const int phase = warp / SPC;
  const bool live = slice < nslices;
  const int ksteps = K / 16;
  float acc[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  pdl_wait();
  pdl_trigger();
  for (int kc0 = 0; kc0 < K; kc0 += KC) {
    const int kcn = min(KC, K - kc0);
    if (kc0 > 0) __syncthreads();                          // previous x block fully consumed
    // stage x[:, kc0:kc0+kcn) with asynchronous 16-byte copies (rows >= M zero-filled)
    const uint32_t xs_base = (uint32_t)__cvta_generic_to_shared(xs);
    for (int i = threadIdx.x; i < rows_tok * (kcn / 8); i += blockDim.x) {
      const int r = i / (kcn / 8), c = (i % (kcn / 8)) * 8;
      const uint32_t dst = xs_base + (uint32_t)(((size_t)r * LDX + c) * 2);
      const __nv_bfloat16* src = x + (size_t)min(r, M - 1) * K + kc0 + c;
      const int bytes = r < M ? 16 : 0;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (live) {
      for (int c = phase; c < kcn / kQChunk; c += NPH)
        gguf_chunk<BITS, NB>(codes, smeta, xs, LDX, slice, ksteps, K, group, kc0 + c * kQChunk, kc0, lane, acc);
    }
  }
  // acc[j]: rows g / g+8 of the slice, tokens j*8 + 2t, +1 -> reduce over the warps of each slice
  __syncthreads();
  float* mine = red + (size_t)warp * 16 * rows_tok;
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    mine[g * rows_tok + j * 8 + 2 * t4] = acc[j][0];
    mine[g * rows_tok + j * 8 + 2 * t4 + 1] = acc[j][1];
    mine[(g + 8) * rows_tok + j * 8 + 2 * t4] = acc[j][2];
    mine[(g + 8) * rows_tok + j * 8 + 2 * t4 + 1] = acc[j][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < SPC * 16 * rows_tok; i += blockDim.x) {
    const int sl = i / (16 * rows_tok), rem = i % (16 * rows_tok);
    const int r = rem / rows_tok, tk = rem % rows_tok;
    float s = 0.f;
#pragma unroll
    for (int ph = 0; ph < NPH; ++ph) s += red[(size_t)(ph * SPC + sl) * 16 * rows_tok + rem];
    const int n = (blockIdx.x * SPC + sl) * 16 + r;
    if (tk < M && n < N) out[(size_t)tk * ldo + n] = __float2bfloat16_rn(s);
  }
}

}  // namespace b200

using namespace b200;

// codes/meta from models.gguf repack_*; x [M, K] bf16; out [M, N] bf16.
void gguf_gemm(torch::Tensor x, torch::Tensor codes, torch::Tensor meta, int64_t N, int64_t bits, int64_t group,
               torch::Tensor out) {
  const int M = x.size(0), K = x.size(1);
  TORCH_CHECK(M <= 32, "gguf_gemm handles decode batches up to 32 tokens");
  TORCH_CHECK(K % 256 == 0 && N % 16 == 0, "K must be a multiple of 256 and N of 16");
  TORCH_CHECK(group == 16 || group == 32, "group must be 16 or 32");
  if (M == 0) return;
  const int NB = M <= 8 ? 1 : M <= 16 ? 2 : 4;
  const size_t smem = (size_t)NB * 8 * (std::min<int>(K, kQStage) + 8) * 2 + (size_t)kQWarps * 16 * NB * 8 * 4;
  auto stream = at::cuda::getCurrentCUDAStream();
  const dim3 grid((N / 16 + NB - 1) / NB), block(kQWarps * 32);
  auto cp = reinterpret_cast<const uint32_t*>(codes.data_ptr());
  auto mp = reinterpret_cast<const uint32_t*>(meta.data_ptr());
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
#define B200_GG(BITSV, NBV)                                                                                  \
  {                                                                                                           \
    static bool attr = false;                                                                                 \
    if (!attr) {                                                                                              \
      B200_CHECK_CUDA(cudaFuncSetAttribute(gguf_gemm_kernel<BITSV, NBV>,                                      \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));         \
      attr = true;                                                                                            \
    }                                                                                                         \
    launch_pdl(gguf_gemm_kernel<BITSV, NBV>, grid, block, smem, stream, cp, mp, xp, M, (int)N, K, (int)group, op, \
               (int)out.stride(0));                                                                           \
  }
  TORCH_CHECK(smem <= 220 * 1024, "activation tile too large for shared memory");
  if (bits == 4) {
    if (NB == 1) B200_GG(4, 1) else if (NB == 2) B200_GG(4, 2) else B200_GG(4, 4)
  } else {
    if (NB == 1) B200_GG(8, 1) else if (NB == 2) B200_GG(8, 2) else B200_GG(8, 4)
  }
#undef B200_GG
}
