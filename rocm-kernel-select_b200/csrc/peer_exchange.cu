// Peer-memory exchange of the T-sharded conv stack: GroupNorm statistics
// gather and halo frames written straight into the peers' memory over
// NVLink (CUDA IPC windows), ordered by release/acquire flags at system
// scope.  Replaces an NCCL all-gather + an NCCL send/recv pair per block.
//
// Window layout (bytes; identical on every rank below xp):
//   0      u32 epoch (local: advanced by publish, read by the other kernels)
//   256    u32 stats flags [2 parities][B200_PEER_MAX_RANKS]
//   1024   u32 halo arrivals: [0] bottom halo (pushed by the previous rank),
//          1024 + 128: [1] top halo (pushed by the next rank)
//   2048   fp32 statistics slots [2][ranks][entries][3]
//   xp     64 KiB aligned: the haloed conv operand
//
// Every wait is bounded by kWaitLimitNs; on running out it records a code in
// the device fault word and the kernel returns (the merge writes NaN).
#include <cstring>

#include "common.cuh"

namespace b200 {
namespace {

constexpr int64_t kFlagOff = 256;
constexpr int64_t kCntOff = 1024;
constexpr int64_t kCntStride = 128;
constexpr int64_t kStatsOff = 2048;
constexpr int64_t kXpAlign = 65536;
constexpr int kFaultStats = 3;
constexpr int kFaultHalo = 4;

static_assert(sizeof(cudaIpcMemHandle_t) == B200_PEER_HANDLE_BYTES, "IPC handle size");
static_assert(kFlagOff + 2 * B200_PEER_MAX_RANKS * 4 <= kCntOff, "flag area overlaps");

__device__ bool poll_bounded(const uint32_t* p, uint32_t target) {
  if (counter_reached(ld_acquire_sys(p), target)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (counter_reached(ld_acquire_sys(p), target)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    __nanosleep(32);
  }
}
__device__ __forceinline__ uint32_t local_epoch(const char* local) {
  return *reinterpret_cast<const volatile uint32_t*>(local);
}

__global__ void __launch_bounds__(256)
peer_stats_publish_kernel(const float* __restrict__ stats, void* const* __restrict__ windows,
                          int ranks, int rank, int entries, char* local) {
  __shared__ uint32_t s_e;
  if (threadIdx.x == 0) {
    uint32_t* ep = reinterpret_cast<uint32_t*>(local);
    const uint32_t e = *ep + 1u;
    *ep = e;
    s_e = e;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int p = static_cast<int>(e & 1u);
  const int n = entries * 3;
  for (int q = 0; q < ranks; ++q) {
    float* dst = reinterpret_cast<float*>(static_cast<char*>(windows[q]) + kStatsOff) +
                 (static_cast<int64_t>(p) * ranks + rank) * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = stats[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < ranks) {
    uint32_t* f = reinterpret_cast<uint32_t*>(static_cast<char*>(windows[threadIdx.x]) + kFlagOff) +
                  p * B200_PEER_MAX_RANKS + rank;
    st_release_sys(f, e);
  }
}

// Rank-order Chan merge, the same arithmetic as gn_merge_ranks_kernel, so
// the peer exchange and the all-gather route give bit-identical statistics.
__global__ void __launch_bounds__(256)
peer_stats_merge_kernel(const char* local, float* __restrict__ out, int ranks, int entries,
                        int* gflags) {
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  const uint32_t e = local_epoch(local);
  const int p = static_cast<int>(e & 1u);
  if (static_cast<int>(threadIdx.x) < ranks) {
    const uint32_t* f =
        reinterpret_cast<const uint32_t*>(local + kFlagOff) + p * B200_PEER_MAX_RANKS + threadIdx.x;
    if (!poll_bounded(f, e)) {
      s_bad = 1;
      if (gflags) atomicExch(gflags, kFaultStats);
    }
  }
  __syncthreads();
  const float* slots =
      reinterpret_cast<const float*>(local + kStatsOff) + static_cast<int64_t>(p) * ranks * entries * 3;
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= entries) return;
  if (s_bad) {
    out[g * 3 + 0] = out[g * 3 + 1] = out[g * 3 + 2] = __int_as_float(0x7fc00000);
    return;
  }
  double n = 0.0, mean = 0.0, m2 = 0.0;
  for (int r = 0; r < ranks; ++r) {
    const float* s = slots + (static_cast<int64_t>(r) * entries + g) * 3;
    const double nb = __ldcg(s);
    if (nb <= 0.0) continue;
    const double tot = n + nb;
    const double d = static_cast<double>(__ldcg(s + 1)) - mean;
    mean += d * nb / tot;
    m2 += static_cast<double>(__ldcg(s + 2)) + d * d * n * nb / tot;
    n = tot;
  }
  out[g * 3 + 0] = static_cast<float>(n);
  out[g * 3 + 1] = static_cast<float>(mean);
  out[g * 3 + 2] = static_cast<float>(m2);
}

struct PushSide {
  const char* src;
  char* dst;
  char* window;    // receiver's window (NULL: side absent)
  int64_t src_stride, dst_stride;
  int counter;     // receiver's arrival counter index
};

constexpr int kPushThreads = 256;
constexpr int kPushUnroll = 4;

// blockIdx.y selects the side.  Every CTA of a present side adds exactly one
// to the receiver's counter, after its stores are fenced at system scope.
__global__ void __launch_bounds__(kPushThreads)
peer_halo_push_kernel(PushSide lo, PushSide hi, int64_t items, int64_t bytes) {
  const PushSide s = blockIdx.y == 0 ? lo : hi;
  if (!s.window) return;
  const int64_t per_item = bytes / 16;
  const int64_t total = items * per_item;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kPushThreads;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kPushThreads * kPushUnroll + threadIdx.x;
       base < total; base += step * kPushUnroll) {
    uint4 v[kPushUnroll];
    int64_t idx[kPushUnroll];
#pragma unroll
    for (int k = 0; k < kPushUnroll; ++k) {
      idx[k] = base + static_cast<int64_t>(k) * kPushThreads;
      if (idx[k] < total) {
        const int64_t it = idx[k] / per_item, o = idx[k] - it * per_item;
        v[k] = __ldcg(reinterpret_cast<const uint4*>(s.src + it * s.src_stride) + o);
      }
    }
#pragma unroll
    for (int k = 0; k < kPushUnroll; ++k) {
      if (idx[k] < total) {
        const int64_t it = idx[k] / per_item, o = idx[k] - it * per_item;
        reinterpret_cast<uint4*>(s.dst + it * s.dst_stride)[o] = v[k];
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    red_release_sys_add(reinterpret_cast<uint32_t*>(s.window + kCntOff + s.counter * kCntStride), 1u);
}

__global__ void peer_halo_wait_kernel(const char* local, int expect_lo, int expect_hi,
                                      int* gflags) {
  const int side = threadIdx.x;
  if (side > 1 || !(side == 0 ? expect_lo : expect_hi)) return;
  const uint32_t target = local_epoch(local) * static_cast<uint32_t>(B200_PEER_PUSH_CTAS);
  const uint32_t* c = reinterpret_cast<const uint32_t*>(local + kCntOff + side * kCntStride);
  if (!poll_bounded(c, target) && gflags) atomicExch(gflags, kFaultHalo);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int64_t b200_peer_window_xp_offset(int64_t ranks, int64_t entries) {
  if (ranks < 1 || ranks > B200_PEER_MAX_RANKS || entries < 1) return -1;
  const int64_t end = kStatsOff + 2 * ranks * entries * 3 * static_cast<int64_t>(sizeof(float));
  return (end + kXpAlign - 1) / kXpAlign * kXpAlign;
}

int64_t b200_peer_window_bytes(int64_t ranks, int64_t entries, int64_t xp_bytes) {
  const int64_t off = b200_peer_window_xp_offset(ranks, entries);
  if (off < 0 || xp_bytes < 0) return -1;
  return off + (xp_bytes + kXpAlign - 1) / kXpAlign * kXpAlign;
}

int b200_peer_window_alloc(int64_t bytes, void** window, void* handle) {
  if (bytes <= 0 || !window || !handle) return fail_arg("bytes/window/handle");
  void* p = nullptr;
  B200_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)));
  cudaError_t err = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return fail_cuda(err, "b200_peer_window_alloc");
  }
  std::memcpy(handle, &h, sizeof(h));
  *window = p;
  return B200_OK;
}

int b200_peer_window_open(const void* handle, void** window) {
  if (!handle || !window) return fail_arg("handle/window");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  B200_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *window = p;
  return B200_OK;
}

int b200_peer_window_close(void* window) {
  if (!window) return fail_arg("window");
  B200_CUDA_CHECK(cudaIpcCloseMemHandle(window));
  return B200_OK;
}

int b200_peer_window_free(void* window) {
  if (!window) return fail_arg("window");
  B200_CUDA_CHECK(cudaFree(window));
  return B200_OK;
}

int b200_peer_stats_publish(const float* stats, void* const* windows, int64_t ranks,
                            int64_t rank, int64_t entries, void* local_window, void* stream) {
  if (!stats || !windows || !local_window) return fail_arg("stats/windows/local_window");
  if (ranks < 1 || ranks > B200_PEER_MAX_RANKS || rank < 0 || rank >= ranks)
    return fail_arg("ranks/rank");
  if (entries < 1 || entries * 3 > (1 << 24)) return fail_arg("entries");
  peer_stats_publish_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      stats, windows, static_cast<int>(ranks), static_cast<int>(rank), static_cast<int>(entries),
      static_cast<char*>(local_window));
  B200_LAUNCH_CHECK("peer_stats_publish_kernel");
  return B200_OK;
}

int b200_peer_stats_merge(void* local_window, float* out, int64_t ranks, int64_t entries,
                          void* stream) {
  if (!local_window || !out) return fail_arg("local_window/out");
  if (ranks < 1 || ranks > B200_PEER_MAX_RANKS) return fail_arg("ranks");
  if (entries < 1 || entries * 3 > (1 << 24)) return fail_arg("entries");
  const unsigned blocks = static_cast<unsigned>((entries + 255) / 256);
  peer_stats_merge_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(local_window), out, static_cast<int>(ranks),
      static_cast<int>(entries), device_flags_ptr());
  B200_LAUNCH_CHECK("peer_stats_merge_kernel");
  return B200_OK;
}

int b200_peer_halo_push(void* local_window, const void* src_lo, void* dst_lo, void* lo_window,
                        int64_t src_lo_stride, int64_t dst_lo_stride, const void* src_hi,
                        void* dst_hi, void* hi_window, int64_t src_hi_stride,
                        int64_t dst_hi_stride, int64_t items, int64_t bytes, void* stream) {
  (void)local_window;
  if (items < 1 || bytes < 16 || bytes % 16) return fail_arg("items/bytes");
  if (lo_window && (!src_lo || !dst_lo || !aligned16(src_lo) || !aligned16(dst_lo) ||
                    src_lo_stride % 16 || dst_lo_stride % 16))
    return fail_arg("lo side pointers/strides");
  if (hi_window && (!src_hi || !dst_hi || !aligned16(src_hi) || !aligned16(dst_hi) ||
                    src_hi_stride % 16 || dst_hi_stride % 16))
    return fail_arg("hi side pointers/strides");
  if (!lo_window && !hi_window) return B200_OK;
  // lo: this rank's first frames -> the previous rank's top halo (its counter 1);
  // hi: the last frames -> the next rank's bottom halo (its counter 0).
  PushSide lo{static_cast<const char*>(src_lo), static_cast<char*>(dst_lo),
              static_cast<char*>(lo_window), src_lo_stride, dst_lo_stride, 1};
  PushSide hi{static_cast<const char*>(src_hi), static_cast<char*>(dst_hi),
              static_cast<char*>(hi_window), src_hi_stride, dst_hi_stride, 0};
  peer_halo_push_kernel<<<dim3(B200_PEER_PUSH_CTAS, 2), kPushThreads, 0,
                          static_cast<cudaStream_t>(stream)>>>(lo, hi, items, bytes);
  B200_LAUNCH_CHECK("peer_halo_push_kernel");
  return B200_OK;
}

int b200_peer_halo_wait(void* local_window, int expect_lo, int expect_hi, void* stream) {
  if (!local_window) return fail_arg("local_window");
  if (!expect_lo && !expect_hi) return B200_OK;
  peer_halo_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(local_window), expect_lo, expect_hi, device_flags_ptr());
  B200_LAUNCH_CHECK("peer_halo_wait_kernel");
  return B200_OK;
}

}  // extern "C"
