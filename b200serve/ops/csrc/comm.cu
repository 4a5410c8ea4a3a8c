// Cross-GPU plumbing for the fused tensor-parallel kernels: CUDA IPC buffers
// shared between the ranks of one node, the per-step epoch counter, and the
// bounded flag wait used by consumers of peer-pushed data.
//
// Protocol of one fused all-reduce site (decode-sized row-parallel output):
//  * every rank's GEMM epilogue stores its partial tile into slot
//    [site % 2][its own rank] of EVERY rank's receive buffer (NVLink P2P stores);
//  * when all tiles of the GEMM are pushed, the rank's last CTA publishes
//    flag[site][its rank] = epoch on every peer: one system-scope fence, then
//    relaxed system-scope stores (a release store per peer would serialise);
//  * the consumer kernel on each rank polls until flag[site][r] == epoch for all
//    r (relaxed loads, bounded by a deadline), issues one acquire fence, then sums
//    the world slots locally.
// Two slots alternate by site parity; a rank can only overwrite slot (site % 2)
// after every peer has pushed site+1, which each peer does only after it has
// finished reading site (stream order), so no slot is overwritten while read.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <algorithm>
#include <cstdlib>
#include "common.cuh"

namespace b200 {

struct FlagPtrs {
  int* p[8];
};

__global__ void epoch_inc_kernel(int* epoch) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) *epoch += 1;
}

// One thread waits (bounded by wait_ns) until flags[0..n) all hold *epoch: orders a consumer
// that cannot wait by itself (a library kernel) after the peers' all-gather pushes. On expiry
// it records 140 + r in *err and returns, so the context stays usable.
__global__ void flag_wait_kernel(const int* flags, int n, const int* epoch, int* err, uint64_t wait_ns) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  const int e = *epoch;
  const uint64_t deadline = globaltimer_ns() + wait_ns;
  for (int r = 0; r < n; ++r) {
    uint32_t it = 0;
    while (true) {
      int v;
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
      if (v == e) break;
      if ((++it & 1023u) == 0 && globaltimer_ns() > deadline) {
        if (err) atomicExch(err, 140 + r);
        return;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Raise flag[r] = *epoch on every rank (a producer with nothing to send still releases its
// consumers); one system fence first.
__global__ void publish_flags_kernel(const FlagPtrs f, int world, const int* epoch) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  __threadfence_system();
  const int e = *epoch;
  for (int r = 0; r < world; ++r)
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f.p[r]), "r"(e) : "memory");
}

// Cross-GPU flag round trip (diagnostics): the initiator stores i into the peer's flag and waits
// for the peer to echo i into its own flag, `iters` times; every wait is bounded (1 s in total).
// Writes the elapsed ns (or -1 on a timeout) to *out.
// mode 0: st.release.sys / ld.acquire.sys; 1: st.relaxed.sys / ld.relaxed.sys; 2: volatile.
__device__ __forceinline__ void pp_store(int* p, int v, int mode) {
  if (mode == 0) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
  else if (mode == 1) asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
  else asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int pp_load(volatile int* p, int mode) {
  int v;
  if (mode == 0) asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  else if (mode == 1) asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  else asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void flag_pingpong_kernel(volatile int* mine, int* peer, int iters, int initiator, int mode,
                                     long long* out) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t deadline = t0 + 1000000000ull;
  for (int i = 1; i <= iters; ++i) {
    if (initiator) pp_store(peer, i, mode);
    uint32_t it = 0;
    while (pp_load(mine, mode) < i) {
      if ((++it & 255u) == 0 && globaltimer_ns() > deadline) {
        *out = -1;
        return;
      }
    }
    if (!initiator) pp_store(peer, i, mode);
  }
  *out = (long long)(globaltimer_ns() - t0);
}

static uint64_t g_flag_wait_ns = 0;

uint64_t flag_wait_ns() {
  if (g_flag_wait_ns == 0) {
    const char* e = getenv("B200_FLAG_WAIT_MS");
    const long ms = e ? atol(e) : 2000;
    g_flag_wait_ns = (uint64_t)std::max(1L, ms) * 1000000ull;
  }
  return g_flag_wait_ns;
}

}  // namespace b200

using namespace b200;

// Deadline of the cross-GPU flag waits for kernels launched (or graphs captured) from now on.
void set_flag_wait_ms(double ms) {
  TORCH_CHECK(ms > 0, "flag wait deadline must be positive");
  g_flag_wait_ns = (uint64_t)(ms * 1e6);
}

double get_flag_wait_ms() { return (double)flag_wait_ns() / 1e6; }

void flag_pingpong(int64_t mine_ptr, int64_t peer_ptr, int64_t iters, int64_t initiator, int64_t mode,
                   torch::Tensor out) {
  flag_pingpong_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<volatile int*>(mine_ptr), reinterpret_cast<int*>(peer_ptr), (int)iters, (int)initiator,
      (int)mode, reinterpret_cast<long long*>(out.data_ptr<int64_t>()));
  B200_CHECK_CUDA(cudaGetLastError());
}

// timeout_ms <= 0: the process-wide deadline (flag_wait_ns)
void flag_wait(int64_t flags_ptr, int64_t n, int64_t epoch_ptr, int64_t err_ptr, double timeout_ms) {
  const uint64_t ns = timeout_ms > 0 ? (uint64_t)(timeout_ms * 1e6) : flag_wait_ns();
  launch_pdl(flag_wait_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const int*>(flags_ptr), (int)n, reinterpret_cast<const int*>(epoch_ptr),
             reinterpret_cast<int*>(err_ptr), ns);
}

void publish_flags(torch::Tensor flag_ptrs, int64_t epoch_ptr) {
  const int world = flag_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= 8 && flag_ptrs.device().is_cpu(), "flag pointers: host int64 [world]");
  FlagPtrs f{};
  for (int r = 0; r < world; ++r) f.p[r] = reinterpret_cast<int*>(flag_ptrs.data_ptr<int64_t>()[r]);
  launch_pdl(publish_flags_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(), f, world,
             reinterpret_cast<const int*>(epoch_ptr));
}

int64_t ipc_malloc(int64_t bytes) {
  void* p = nullptr;
  B200_CHECK_CUDA(cudaMalloc(&p, bytes));
  B200_CHECK_CUDA(cudaMemset(p, 0, bytes));
  return reinterpret_cast<int64_t>(p);
}

void ipc_free(int64_t ptr) { B200_CHECK_CUDA(cudaFree(reinterpret_cast<void*>(ptr))); }

torch::Tensor ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  B200_CHECK_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t ipc_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  B200_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { B200_CHECK_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

// Host-mapped error word: kernels that give up a bounded wait write a code here;
// the host reads it after each step without a device synchronisation.
torch::Tensor host_error_word() {
  int* h = nullptr;
  B200_CHECK_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h), 64, cudaHostAllocMapped));
  memset(h, 0, 64);
  int* d = nullptr;
  B200_CHECK_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0));
  auto t = torch::empty({2}, torch::kInt64);
  t[0] = reinterpret_cast<int64_t>(h);
  t[1] = reinterpret_cast<int64_t>(d);
  return t;
}

int64_t read_host_word(int64_t host_ptr, int64_t index, bool reset) {
  volatile int* h = reinterpret_cast<volatile int*>(host_ptr);
  const int v = h[index];
  if (reset) h[index] = 0;
  return v;
}

void epoch_inc(int64_t epoch_ptr) {
  launch_pdl(epoch_inc_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<int*>(epoch_ptr));
}
