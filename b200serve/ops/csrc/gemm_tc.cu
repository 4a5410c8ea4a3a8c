// Host side of the tcgen05 GEMM: tile/split planning, TMA descriptors, launch.
#include <mutex>
#include "gemm_tc.cuh"

namespace b200 {

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    B200_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor [rows, cols] with row stride `ld` elements; box = 64 cols x box_rows, 128B swizzle.
static CUtensorMap make_tmap_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

static int g_num_sms = 0;

// error word of the bounded waits (device memory, allocated once per process)
static int* g_err_dev = nullptr;
static int* gemm_err_word() {
  if (g_err_dev == nullptr) {
    B200_CHECK_CUDA(cudaMalloc(&g_err_dev, sizeof(int)));
    B200_CHECK_CUDA(cudaMemset(g_err_dev, 0, sizeof(int)));
  }
  return g_err_dev;
}

// Shared-memory budget of the stage ring. Decode-sized token tiles (BN <= 64) default to
// ~104 KB, which leaves room for a neighbouring kernel's CTA on the SM (programmatic dependent
// launch overlap); B200_GEMM_DECODE_SMEM_KB overrides it. Larger tiles use 200 KB.
static int ring_stages(int BN) {
  static int decode_kb = -1;
  if (decode_kb < 0) {
    const char* e = getenv("B200_GEMM_DECODE_SMEM_KB");
    decode_kb = e ? std::max(40, std::min(220, atoi(e))) : 104;
  }
  const int budget = (BN <= 64 ? decode_kb : 200) * 1024;
  const int stage = 128 * 64 * 2 + BN * 64 * 2;
  return std::max(2, std::min(12, budget / stage));
}

static void launch_by_bn(int BN, int epi, const CUtensorMap& tw, const CUtensorMap& ta, const GemmParams& p0,
                         int grid, cudaStream_t stream) {
  GemmParams p = p0;
  if (p.stages <= 0) p.stages = ring_stages(BN);
  static int l2_kb = -1;
  if (l2_kb < 0) {
    const char* e = getenv("B200_GEMM_L2_PREFETCH_KB");
    l2_kb = e ? std::max(0, atoi(e)) : 0;
  }
  if (p.w_packed && !p.grouped) p.l2_prefetch_blocks = l2_kb / 16;
  else p.w_ptr = nullptr;
  switch (BN) {
    case 16: launch_gemm_bn<16>(epi, tw, ta, p, grid, stream); break;
    case 32: launch_gemm_bn<32>(epi, tw, ta, p, grid, stream); break;
    case 64: launch_gemm_bn<64>(epi, tw, ta, p, grid, stream); break;
    case 128: launch_gemm_bn<128>(epi, tw, ta, p, grid, stream); break;
    case 256: launch_gemm_bn<256>(epi, tw, ta, p, grid, stream); break;
    default: TORCH_CHECK(false, "bad BN");
  }
}

}  // namespace b200

using namespace b200;

// Tile/split plan: returns {BN, m_tiles, n_tiles, splits, kb_per_split, units, grid}.
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t num_sms) {
  int BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const int m_tiles = (int)((M + BN - 1) / BN);
  const int n_tiles = (int)((N + 127) / 128);
  const int kb_total = (int)((K + 63) / 64);
  const int tiles = m_tiles * n_tiles;
  int best_s = 1, best_kbp = kb_total;
  static int planner = -1;
  if (planner < 0) {
    const char* e = getenv("B200_GEMM_PLANNER");
    planner = e ? atoi(e) : 1;
  }
  if (m_tiles * BN <= 256 && planner == 1) {
    // decode-sized M, latency model: the kernel takes as long as its busiest CTA streams its
    // weight tiles, at the smaller of an equal share of HBM bandwidth and what one CTA's
    // stage ring sustains (ring bytes per ~1.5 us round trip), plus the split-K reduction
    // (~1.5 us + 0.15 us per split) and ~1 us per extra unit a persistent CTA runs.
    const double hbm = 6.5e3;                                   // bytes per ns
    const double stage = 128.0 * 64 * 2 + BN * 64 * 2;
    const double ring = (double)ring_stages(BN) * stage;
    const double cta_bw = ring / 1800.0;                        // bytes per ns (with margin)
    double best = 1e30;
    for (int s = 1; s <= 32; ++s) {
      const int kbp = (kb_total + s - 1) / s;
      if (kbp < 2 && s > 1) break;
      const int se = (kb_total + kbp - 1) / kbp;
      const long units = (long)tiles * se;
      if (se > 1 && units > 4 * num_sms) break;
      const long ctas = std::min<long>(units, num_sms);
      const long waves = (units + num_sms - 1) / num_sms;
      const double bytes = (double)waves * kbp * stage;
      const double bw = std::min(hbm / (double)ctas, cta_bw);
      const double t = bytes / bw + (se > 1 ? 1500.0 + 150.0 * se : 0.0) + 1000.0 * (double)(waves - 1);
      if (t < best - 1e-6) { best = t; best_s = se; best_kbp = kbp; }
    }
  } else if (m_tiles * BN <= 256) {
    // decode-sized M: weight streaming, balance the busiest SM with split-K
    double best = -1.0;
    for (int s = 1; s <= 32; ++s) {
      const int kbp = (kb_total + s - 1) / s;
      if (kbp < 4 && s > 1) break;
      const int se = (kb_total + kbp - 1) / kbp;
      const long units = (long)tiles * se;
      const long waves = (units + num_sms - 1) / num_sms;
      // balance of the busiest CTA, discounted by the partial-tile traffic of more splits
      const double eff = (double)units / (double)(waves * num_sms) - 0.01 * se;
      if (eff > best + 1e-9) { best = eff; best_s = se; best_kbp = kbp; }
    }
  }
  const long units = (long)tiles * best_s;
  const int grid = (int)std::min<long>(units, num_sms);
  return {BN, m_tiles, n_tiles, best_s, best_kbp, units, grid};
}

// act [M, K] (row stride lda), w [N, K] contiguous; out [M, ldo] bf16/fp32 or [M, N/2] for SwiGLU.
// ws: fp32 workspace >= splits*m_tiles*BN*N, counters: int32 >= m_tiles*n_tiles (zeroed once).
// Weight geometry: plain [N, K] (packed_n == 0) or tile-packed with logical N = packed_n.
static CUtensorMap weight_tmap(const torch::Tensor& w, int N, int K, bool packed) {
  if (!packed) return make_tmap_bf16(w.data_ptr(), N, K, K, 128);
  TORCH_CHECK(w.size(1) == 64 && w.size(0) == (int64_t)((N + 127) / 128) * ((K + 63) / 64) * 128,
              "packed weight has the wrong shape");
  return make_tmap_bf16(w.data_ptr(), w.size(0), 64, 64, 128);
}

// Per-CTA timeline capture (diagnostics only): launch i writes [2048 CTAs][8] stamps at
// g_trace + (i % g_trace_slots) * 2048 * 8.
static unsigned long long* g_trace = nullptr;
static int g_trace_slots = 1, g_trace_next = 0;
static unsigned long long* next_trace() {
  if (!g_trace) return nullptr;
  unsigned long long* t = g_trace + (size_t)(g_trace_next % g_trace_slots) * 2048 * 8;
  ++g_trace_next;
  return t;
}

void gemm_set_trace(int64_t ptr, int64_t slots) {
  g_trace = reinterpret_cast<unsigned long long*>(ptr);
  g_trace_slots = (int)std::max<int64_t>(1, slots);
  g_trace_next = 0;
}

static void gemm_tc_impl(torch::Tensor act, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> bias,
                         c10::optional<torch::Tensor> residual, torch::Tensor ws, torch::Tensor counters, int64_t epi,
                         int64_t force_splits, int64_t packed_n, const int* ag_flags, int ag_n,
                         const int* ag_epoch, const GemmParams* qkv = nullptr) {
  TORCH_CHECK(act.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16);
  TORCH_CHECK(act.dim() == 2 && w.dim() == 2 && act.stride(1) == 1 && w.is_contiguous());
  const bool packed = packed_n > 0;
  const int M = act.size(0), K = act.size(1), N = packed ? (int)packed_n : w.size(0);
  TORCH_CHECK(packed || w.size(1) == K, "K mismatch");
  TORCH_CHECK(K % 8 == 0, "K must be a multiple of 8");
  if (M == 0) return;
  if (g_num_sms == 0) {
    int dev;
    B200_CHECK_CUDA(cudaGetDevice(&dev));
    B200_CHECK_CUDA(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  auto plan = gemm_plan(M, N, K, epi, g_num_sms);
  int BN = plan[0];
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.m_tiles = plan[1]; p.n_tiles = plan[2]; p.splits = plan[3]; p.kb_per_split = plan[4];
  p.kb_total = (K + 63) / 64;
  if (force_splits > 0) {
    p.kb_per_split = (p.kb_total + force_splits - 1) / force_splits;
    p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  }
  // Cluster split-K for decode-sized tiles: one CTA per (tile, split), the splits of a tile
  // (<= 8) form a thread-block cluster and reduce through distributed shared memory.
  static int cluster_mode = -1;
  if (cluster_mode < 0) {
    const char* e = getenv("B200_GEMM_CLUSTER");
    cluster_mode = e ? atoi(e) : 0;   // measured slower than the workspace fixup at decode sizes
  }
  if (cluster_mode && force_splits <= 0 && BN <= 64 && p.m_tiles == 1 && epi != EPI_PUSH) {
    const int tiles = p.n_tiles;
    int s = std::min(8, std::max(1, (2 * g_num_sms) / tiles));
    while (s > 1 && (p.kb_total + s - 1) / s < 4) --s;
    if (s > 1) {
      p.kb_per_split = (p.kb_total + s - 1) / s;
      p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
      p.cluster_red = p.splits > 1 ? 1 : 0;
    }
  }
  p.units = p.m_tiles * p.n_tiles * p.splits;
  static int raster = -1;
  if (raster < 0) {
    const char* e = getenv("B200_GEMM_RASTER");
    raster = e ? atoi(e) : 8;
  }
  if (p.splits == 1 && p.m_tiles > 1 && raster > 1) p.raster = raster;
  const int grid = p.cluster_red ? p.units : std::min(p.units, g_num_sms);
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.bias = bias ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.residual = residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  p.ldr = residual ? residual->stride(0) : 0;
  if (epi == EPI_F32) {
    TORCH_CHECK(out.scalar_type() == at::kFloat);
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16);
  }
  if (epi == EPI_SWIGLU) TORCH_CHECK(N % 128 == 0 && out.size(1) == N / 2, "SwiGLU needs N % 128 == 0");
  if (p.splits > 1 && !p.cluster_red) {
    TORCH_CHECK(ws.scalar_type() == at::kFloat &&
                    ws.numel() >= (int64_t)p.splits * p.m_tiles * p.n_tiles * BN * 128,
                "GEMM workspace too small");
    TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= p.m_tiles * p.n_tiles,
                "GEMM counters too small");
    p.ws = ws.data_ptr<float>();
    p.counters = counters.data_ptr<int>();
  }
  p.err = gemm_err_word();
  p.w_packed = packed ? 1 : 0;
  p.w_ptr = packed ? reinterpret_cast<const uint8_t*>(w.data_ptr()) : nullptr;
  p.ag_flags = ag_flags;
  p.ag_n = ag_n;
  p.ag_epoch = ag_epoch;
  p.ag_wait_ns = flag_wait_ns();
  if (qkv) {
    p.qkv_nq = qkv->qkv_nq; p.qkv_nkv = qkv->qkv_nkv; p.q_norm = qkv->q_norm; p.k_norm = qkv->k_norm;
    p.cos_sin = qkv->cos_sin; p.positions = qkv->positions; p.slots = qkv->slots; p.q_out = qkv->q_out;
    p.k_cache = qkv->k_cache; p.v_cache = qkv->v_cache; p.qkv_eps = qkv->qkv_eps;
  }
  p.trace = next_trace();
  CUtensorMap tw = weight_tmap(w, N, K, packed);
  CUtensorMap ta = make_tmap_bf16(act.data_ptr(), M, K, act.stride(0), BN);
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_by_bn(BN, (int)epi, tw, ta, p, grid, stream);
}

void gemm_tc(torch::Tensor act, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> bias,
             c10::optional<torch::Tensor> residual, torch::Tensor ws, torch::Tensor counters, int64_t epi,
             int64_t force_splits, int64_t packed_n) {
  gemm_tc_impl(act, w, out, bias, residual, ws, counters, epi, force_splits, packed_n, nullptr, 0, nullptr);
}

// All-gather -> GEMM: the activation rows are written by the ranks' norm kernels (P2P pushes);
// the kernel streams its weights right away and loads activations once every rank's flag at
// ag_flags_ptr[0..ag_n) holds the step epoch at ag_epoch_ptr.
void gemm_tc_ag(torch::Tensor act, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> bias,
                torch::Tensor ws, torch::Tensor counters, int64_t epi, int64_t packed_n, int64_t ag_flags_ptr,
                int64_t ag_n, int64_t ag_epoch_ptr) {
  TORCH_CHECK(ag_flags_ptr && ag_epoch_ptr && ag_n >= 1 && ag_n <= kMaxPeers, "bad all-gather flags");
  gemm_tc_impl(act, w, out, bias, c10::nullopt, ws, counters, epi, 0, packed_n,
               reinterpret_cast<const int*>(ag_flags_ptr), (int)ag_n, reinterpret_cast<const int*>(ag_epoch_ptr));
}

// Fused QKV projection: x [T, H] @ W_qkv^T (+bias) with the per-head q/k RMSNorm, RoPE and
// the paged bf16 KV write in the epilogue (head_dim 128): q -> q_out [T, nq, 128], k/v rows ->
// k_cache / v_cache [blocks][nkv][16][128] at slots (-1 = skip). ag_* as in gemm_tc_ag (0 = none).
void gemm_tc_qkv(torch::Tensor act, torch::Tensor w, int64_t packed_n, c10::optional<torch::Tensor> bias,
                 c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, torch::Tensor cos_sin,
                 torch::Tensor positions, torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_cache,
                 torch::Tensor v_cache, int64_t nq, int64_t nkv, double eps, torch::Tensor ws,
                 torch::Tensor counters, int64_t ag_flags_ptr, int64_t ag_n, int64_t ag_epoch_ptr) {
  TORCH_CHECK(cos_sin.size(1) == 128 && k_cache.size(-1) == 128 && k_cache.scalar_type() == at::kBFloat16,
              "fused QKV epilogue needs head_dim 128 and a bf16 KV cache");
  TORCH_CHECK(packed_n == (nq + 2 * nkv) * 128, "QKV weight rows must be (nq + 2 nkv) x 128");
  TORCH_CHECK(q_out.is_contiguous() && q_out.size(0) == act.size(0));
  GemmParams q{};
  q.qkv_nq = (int)nq; q.qkv_nkv = (int)nkv;
  q.q_norm = q_norm ? reinterpret_cast<const __nv_bfloat16*>(q_norm->data_ptr()) : nullptr;
  q.k_norm = k_norm ? reinterpret_cast<const __nv_bfloat16*>(k_norm->data_ptr()) : nullptr;
  q.cos_sin = cos_sin.data_ptr<float>();
  q.positions = positions.data_ptr<int>();
  q.slots = slots.data_ptr<int>();
  q.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  q.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  q.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  q.qkv_eps = (float)eps;
  gemm_tc_impl(act, w, q_out.view({act.size(0), -1}), bias, c10::nullopt, ws, counters, EPI_QKV, 0, packed_n,
               ag_flags_ptr ? reinterpret_cast<const int*>(ag_flags_ptr) : nullptr, (int)ag_n,
               ag_epoch_ptr ? reinterpret_cast<const int*>(ag_epoch_ptr) : nullptr, &q);
}

// Tensor-parallel GEMM whose epilogue pushes the bf16 output tile into the
// receive slot of every rank (P2P stores) and raises per-rank flags once the
// whole output is pushed. dst_ptrs/flag_ptrs: int64 [world] device addresses.
void gemm_tc_push(torch::Tensor act, torch::Tensor w, torch::Tensor dst_ptrs, int64_t ldo, torch::Tensor flag_ptrs,
                  int64_t epoch_ptr, torch::Tensor tile_done, c10::optional<torch::Tensor> bias, torch::Tensor ws,
                  torch::Tensor counters, int64_t err_ptr, int64_t packed_n, int64_t rs_rows, int64_t lamport,
                  int64_t mc_ptr) {
  TORCH_CHECK(act.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16);
  const bool packed = packed_n > 0;
  const int M = act.size(0), K = act.size(1), N = packed ? (int)packed_n : w.size(0);
  const int world = dst_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && flag_ptrs.numel() == world);
  if (M == 0) return;
  if (g_num_sms == 0) {
    int dev;
    B200_CHECK_CUDA(cudaGetDevice(&dev));
    B200_CHECK_CUDA(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  auto plan = gemm_plan(M, N, K, EPI_PUSH, g_num_sms);
  const int BN = plan[0];
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.m_tiles = plan[1]; p.n_tiles = plan[2]; p.splits = plan[3]; p.kb_per_split = plan[4];
  p.kb_total = (K + 63) / 64;
  p.units = p.m_tiles * p.n_tiles * p.splits;
  const int grid = std::min(p.units, g_num_sms);
  p.ldo = ldo;
  p.bias = bias ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  if (p.splits > 1) {
    TORCH_CHECK(ws.numel() >= (int64_t)p.splits * p.m_tiles * p.n_tiles * BN * 128, "GEMM workspace too small");
    TORCH_CHECK(counters.numel() >= p.m_tiles * p.n_tiles, "GEMM counters too small");
    p.ws = ws.data_ptr<float>();
    p.counters = counters.data_ptr<int>();
  }
  p.world = world;
  auto dp = dst_ptrs.cpu();
  auto fp = flag_ptrs.cpu();
  for (int r = 0; r < world; ++r) {
    p.push_dst[r] = reinterpret_cast<__nv_bfloat16*>(dp[r].item<int64_t>());
    p.push_flag[r] = reinterpret_cast<int*>(fp[r].item<int64_t>());
  }
  p.epoch = reinterpret_cast<const int*>(epoch_ptr);
  p.tile_done = tile_done.data_ptr<int>();
  p.rs_rows = (int)rs_rows;
  p.lamport = lamport ? 1 : 0;
  p.mc_dst = reinterpret_cast<__nv_bfloat16*>(mc_ptr);
  TORCH_CHECK(!mc_ptr || (lamport && (mc_ptr % 16) == 0 && (ldo % 8) == 0),
              "multicast push: flag-free mode, 16-byte aligned slot and row stride");
  TORCH_CHECK(!(lamport && rs_rows), "the flag-free push is an all-reduce (rs_rows must be 0)");
  TORCH_CHECK(rs_rows == 0 || (int64_t)rs_rows * world >= M, "reduce-scatter rows do not cover the tokens");
  p.err = err_ptr ? reinterpret_cast<int*>(err_ptr) : gemm_err_word();
  p.w_packed = packed ? 1 : 0;
  p.w_ptr = packed ? reinterpret_cast<const uint8_t*>(w.data_ptr()) : nullptr;
  CUtensorMap tw = weight_tmap(w, N, K, packed);
  CUtensorMap ta = make_tmap_bf16(act.data_ptr(), M, K, act.stride(0), BN);
  launch_by_bn(BN, EPI_PUSH, tw, ta, p, grid, at::cuda::getCurrentCUDAStream());
}

// Decode-sized GEMM (M <= 64) as stream-K with consumer-side reduction: every CTA streams an
// equal share of the flattened (n tile, k block) space and stores the fp32 partial of each
// piece to part[slot][M][N]; the row kernel that consumes the output (RMSNorm, qkv_post) sums
// the slots (PartialIn). No split-K counters and no fixup pass. Returns {kb, ctas, total,
// slots}; part must hold slots * M * N floats (gemm_partial_slots gives the size up front).
std::vector<int64_t> gemm_partial_plan(int64_t M, int64_t N, int64_t K, int64_t num_sms) {
  const int64_t kb = (K + 63) / 64, tiles = (N + 127) / 128, total = tiles * kb;
  // CTAs per SM (B200_GEMM_PARTIAL_PER_SM, 1 or 2; the decode ring of ~104 KB lets two share an SM).
  // Two measured no better on the 8B decode step (6084 against 6055 tok/s, within run-to-run noise),
  // so one is the default.
  static const int per_sm = [] { const char* e = getenv("B200_GEMM_PARTIAL_PER_SM"); return e && atoi(e) == 2 ? 2 : 1; }();
  // at least 4 k-blocks (64 KB of weights) per CTA, so every piece amortises its pipeline start
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(per_sm * num_sms, total / 4));
  const int64_t slots = (kb * ctas + total - 1) / total + 1;
  return {kb, ctas, total, slots};
}

std::vector<int64_t> gemm_tc_partial(torch::Tensor act, torch::Tensor w, int64_t packed_n, torch::Tensor part) {
  TORCH_CHECK(act.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16);
  TORCH_CHECK(act.dim() == 2 && act.stride(1) == 1 && w.is_contiguous());
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous(), "partials: contiguous fp32");
  const bool packed = packed_n > 0;
  const int M = act.size(0), K = act.size(1), N = packed ? (int)packed_n : w.size(0);
  TORCH_CHECK(M >= 1 && M <= 64, "the stream-K partial GEMM serves decode sizes (1..64 tokens)");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "K and N must be multiples of 8");
  if (g_num_sms == 0) {
    int dev;
    B200_CHECK_CUDA(cudaGetDevice(&dev));
    B200_CHECK_CUDA(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  auto plan = gemm_partial_plan(M, N, K, g_num_sms);
  const int BN = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  TORCH_CHECK(part.numel() >= plan[3] * M * N, "partial buffer too small: need ", plan[3] * M * N, " floats");
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.m_tiles = 1; p.n_tiles = (N + 127) / 128; p.splits = 1;
  p.kb_total = (int)plan[0]; p.kb_per_split = p.kb_total;
  p.units = (int)plan[1];
  p.streamk = 1;
  p.sk_total = plan[2];
  p.part = part.data_ptr<float>();
  p.err = gemm_err_word();
  p.w_packed = packed ? 1 : 0;
  p.w_ptr = packed ? reinterpret_cast<const uint8_t*>(w.data_ptr()) : nullptr;
  p.trace = next_trace();
  CUtensorMap tw = weight_tmap(w, N, K, packed);
  CUtensorMap ta = make_tmap_bf16(act.data_ptr(), M, K, act.stride(0), BN);
  launch_by_bn(BN, EPI_PARTIAL, tw, ta, p, (int)plan[1], at::cuda::getCurrentCUDAStream());
  return plan;
}

// Grouped expert GEMM: act [R, K] rows sorted by expert, offsets [E+1] (device), w packed
// [E][n_tiles][k_blocks][128][64] (logical per-expert [N, K]); out [R, N] bf16 or [R, N/2] (SwiGLU).
// max_rows bounds the rows of one expert (sizes the m-tile grid without reading offsets on the host).
void gemm_grouped(torch::Tensor act, torch::Tensor w_packed, int64_t N, int64_t E, torch::Tensor offsets,
                  int64_t max_rows, torch::Tensor out, torch::Tensor ws, torch::Tensor counters, int64_t epi) {
  TORCH_CHECK(act.scalar_type() == at::kBFloat16 && w_packed.scalar_type() == at::kBFloat16);
  TORCH_CHECK(epi == EPI_BF16 || epi == EPI_SWIGLU, "grouped GEMM epilogue must be bf16 or SwiGLU");
  const int R = act.size(0), K = act.size(1);
  if (R == 0 || E == 0) return;
  if (g_num_sms == 0) {
    int dev;
    B200_CHECK_CUDA(cudaGetDevice(&dev));
    B200_CHECK_CUDA(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int BN = max_rows <= 16 ? 16 : max_rows <= 32 ? 32 : max_rows <= 64 ? 64 : max_rows <= 128 ? 128 : 256;
  GemmParams p{};
  p.M = R; p.N = N; p.K = K;
  p.n_tiles = (N + 127) / 128;
  p.m_tiles = (max_rows + BN - 1) / BN;
  p.kb_total = (K + 63) / 64;
  p.splits = 1;
  p.kb_per_split = p.kb_total;
  p.units = E * p.m_tiles * p.n_tiles;
  p.grouped = 1;
  p.g_offsets = offsets.data_ptr<int>();
  p.g_E = E;
  p.w_packed = 1;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.err = gemm_err_word();
  TORCH_CHECK(w_packed.size(1) == 64 && w_packed.size(0) == E * p.n_tiles * p.kb_total * 128, "bad packed expert weight");
  CUtensorMap tw = make_tmap_bf16(w_packed.data_ptr(), w_packed.size(0), 64, 64, 128);
  CUtensorMap ta = make_tmap_bf16(act.data_ptr(), R, K, act.stride(0), BN);
  const int grid = std::min(p.units, g_num_sms);
  launch_by_bn(BN, (int)epi, tw, ta, p, grid, at::cuda::getCurrentCUDAStream());
}

// Grouped expert GEMM of the expert-parallel all-to-all: like gemm_grouped, plus
//  * ag_flags_ptr/ag_n (0 = none): the activation rows arrive from peers; the producer waits
//    until those flags hold the step epoch before loading any row;
//  * comb_meta (empty = none): EPI_PUSH combine epilogue (GemmParams::comb_meta) into the home
//    ranks' slots comb_dst_ptrs[rank] (row stride ldo), then the site flags flag_ptrs[rank]
//    raised once all push_tiles tiles are stored.
void gemm_grouped_ep(torch::Tensor act, torch::Tensor w_packed, int64_t N, int64_t E, torch::Tensor offsets,
                     int64_t max_rows, torch::Tensor out, torch::Tensor ws, torch::Tensor counters, int64_t epi,
                     int64_t ag_flags_ptr, int64_t ag_n, int64_t ag_epoch_ptr, torch::Tensor comb_meta,
                     int64_t comb_k, int64_t comb_rows, torch::Tensor comb_dst_ptrs, int64_t ldo,
                     torch::Tensor flag_ptrs, torch::Tensor tile_done, int64_t push_tiles, int64_t err_ptr) {
  TORCH_CHECK(act.scalar_type() == at::kBFloat16 && w_packed.scalar_type() == at::kBFloat16);
  const bool comb = comb_meta.numel() > 0;
  TORCH_CHECK(comb ? epi == EPI_PUSH : (epi == EPI_BF16 || epi == EPI_SWIGLU), "bad epilogue for the grouped GEMM");
  const int R = act.size(0), K = act.size(1);
  if (R == 0 || E == 0 || max_rows == 0) return;
  if (g_num_sms == 0) {
    int dev;
    B200_CHECK_CUDA(cudaGetDevice(&dev));
    B200_CHECK_CUDA(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int BN = max_rows <= 16 ? 16 : max_rows <= 32 ? 32 : max_rows <= 64 ? 64 : max_rows <= 128 ? 128 : 256;
  GemmParams p{};
  p.M = R; p.N = N; p.K = K;
  p.n_tiles = (N + 127) / 128;
  p.m_tiles = (max_rows + BN - 1) / BN;
  p.kb_total = (K + 63) / 64;
  p.splits = 1;
  p.kb_per_split = p.kb_total;
  p.units = E * p.m_tiles * p.n_tiles;
  p.grouped = 1;
  p.g_offsets = offsets.data_ptr<int>();
  p.g_E = E;
  p.w_packed = 1;
  p.err = err_ptr ? reinterpret_cast<int*>(err_ptr) : gemm_err_word();
  p.ag_flags = ag_flags_ptr ? reinterpret_cast<const int*>(ag_flags_ptr) : nullptr;
  p.ag_n = (int)ag_n;
  p.ag_epoch = reinterpret_cast<const int*>(ag_epoch_ptr);
  p.ag_wait_ns = flag_wait_ns();
  if (comb) {
    const int world = comb_dst_ptrs.numel();
    TORCH_CHECK(world >= 1 && world <= kMaxPeers && flag_ptrs.numel() == world && comb_k >= 1 && push_tiles > 0,
                "combine: pointers, k and tile count");
    TORCH_CHECK(comb_meta.scalar_type() == at::kInt && comb_meta.numel() >= (int64_t)R * 4, "combine metadata");
    p.comb_meta = reinterpret_cast<const int4*>(comb_meta.data_ptr<int>());
    p.comb_k = (int)comb_k;
    p.comb_rows = (int)comb_rows;
    p.push_tiles = (int)push_tiles;
    p.world = world;
    for (int r = 0; r < world; ++r) {
      p.push_dst[r] = reinterpret_cast<__nv_bfloat16*>(comb_dst_ptrs.data_ptr<int64_t>()[r]);
      p.push_flag[r] = reinterpret_cast<int*>(flag_ptrs.data_ptr<int64_t>()[r]);
    }
    p.epoch = reinterpret_cast<const int*>(ag_epoch_ptr);
    p.tile_done = tile_done.data_ptr<int>();
    p.ldo = (int)ldo;
  } else {
    p.out = out.data_ptr();
    p.ldo = out.stride(0);
  }
  TORCH_CHECK(w_packed.size(1) == 64 && w_packed.size(0) == E * p.n_tiles * p.kb_total * 128, "bad packed expert weight");
  CUtensorMap tw = make_tmap_bf16(w_packed.data_ptr(), w_packed.size(0), 64, 64, 128);
  CUtensorMap ta = make_tmap_bf16(act.data_ptr(), R, K, act.stride(0), BN);
  const int grid = std::min(p.units, g_num_sms);
  launch_by_bn(BN, (int)epi, tw, ta, p, grid, at::cuda::getCurrentCUDAStream());
}

int64_t gemm_error_flag(bool reset) {
  int v = 0;
  B200_CHECK_CUDA(cudaMemcpy(&v, gemm_err_word(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) B200_CHECK_CUDA(cudaMemset(gemm_err_word(), 0, sizeof(int)));
  return v;
}
