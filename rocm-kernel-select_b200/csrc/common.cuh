// Shared helpers for the sm_100a kernels of libb200conv.so: dtype handling,
// status plumbing for the C ABI, vector memory access and bounded waits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/b200conv.h"

namespace b200 {

// ---------------------------------------------------------------- status ---
void set_last_error(const std::string& msg);
int fail_arg(const char* what);
int fail_unsupported(const char* what);
int fail_cuda(cudaError_t err, const char* where);

#define B200_CUDA_CHECK(expr)                                 \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::b200::fail_cuda(_e, #expr); \
  } while (0)

#define B200_LAUNCH_CHECK(where)                                   \
  do {                                                             \
    cudaError_t _e = cudaGetLastError();                           \
    if (_e != cudaSuccess) return ::b200::fail_cuda(_e, where);    \
  } while (0)

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

inline size_t dtype_size(int dt) { return dt == B200_DTYPE_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) {
  return dt == B200_DTYPE_F32 || dt == B200_DTYPE_F16 || dt == B200_DTYPE_BF16;
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count();
int max_smem_optin();

// Device-side fault word: bounded waits set it instead of spinning forever.
// Codes: 1 = pipeline wait timed out in conv3d; 3 = peer statistics wait,
// 4 = peer halo wait (b200_peer_* and the gated conv3d) timed out.  Kernels receive its device
// address as a plain pointer (no relocatable device code needed).
int* device_flags_ptr();

// ----------------------------------------------------------------- dtypes ---
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// fp32 -> bit pattern of a 16-bit float (register-only, no address taken).
template <typename T>
__device__ __forceinline__ uint16_t f32_to_bits16(float v);
template <>
__device__ __forceinline__ uint16_t f32_to_bits16<__half>(float v) {
  return __half_as_ushort(__float2half_rn(v));
}
template <>
__device__ __forceinline__ uint16_t f32_to_bits16<__nv_bfloat16>(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Loads one parameter (gamma/beta/bias/weight) of runtime dtype `dt` as fp32.
__device__ __forceinline__ float load_param(const void* p, int dt, int64_t i) {
  if (dt == B200_DTYPE_F32) return __ldg(reinterpret_cast<const float*>(p) + i);
  if (dt == B200_DTYPE_F16) return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
  return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(p) + i));
}

// 16-byte vector of T: 4 fp32 or 8 fp16/bf16 lanes.
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& r, float (&v)[Vec16<T>::N]);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& r, float (&v)[4]) {
  v[0] = __uint_as_float(r.x);
  v[1] = __uint_as_float(r.y);
  v[2] = __uint_as_float(r.z);
  v[3] = __uint_as_float(r.w);
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& r, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& r, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float (&v)[Vec16<T>::N]);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float (&v)[4]) {
  return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                    __float_as_uint(v[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<__half>(const float (&v)[8]) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  return r;
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float (&v)[8]) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return r;
}

// Streaming 16-byte global load (read once: no L1 allocation).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Streaming 16-byte global store (evict-first).
__device__ __forceinline__ void st_stream16(void* p, const uint4& r) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(r.x), "r"(r.y),
               "r"(r.z), "r"(r.w)
               : "memory");
}

// Programmatic dependent launch.  launch_dependents lets the next grid in the
// stream (launched with the programmatic-serialization attribute) start its
// prologue early; wait blocks until every grid this one depends on has
// completed and its memory is visible.  Both are no-ops without PDL.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// System-scope ordering for flags that other GPUs write over NVLink.
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Wrap-safe "counter has reached target" for monotonically advancing words.
__device__ __forceinline__ bool counter_reached(uint32_t v, uint32_t target) {
  return static_cast<int32_t>(v - target) >= 0;
}

// Upper bound for any device-side wait (ns).  Normal waits are microseconds;
// running out means a broken pipeline, and the kernel then records the fault
// in g_device_flags and returns instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; result valid in every thread.  `scratch` holds >= 33 floats.
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (warp == 0) {
    t = lane < W ? scratch[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) scratch[32] = t;
  }
  __syncthreads();
  t = scratch[32];
  __syncthreads();
  return t;
}

}  // namespace b200
