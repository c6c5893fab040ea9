// Depthwise conv1d forward (stride 1, dilation 1, zero padding) for sm_100a.
//
// Same contract as the reference's vendored conv1d_kernel
// (amd_tuned_torch/_vendor/flashfftconv_depthwise_conv1d/conv1d_bhl.cu:53-98):
//   y[b,c,l] = bias[c] + sum_k w[c,k] * x[b,c,l - pad + k],
//   L_out = L + 2*pad - K + 1, bias always added (zeros when absent).
// Differences by design: fp32 accumulation for every dtype (the reference
// accumulates in the input dtype with __hfma), any K (the reference requires
// odd K and mis-indexes the batch stride for K != 3 when L_out != L, see
// conv1d_bhl.cu:89), and launches on the caller's stream (the reference uses
// the default stream, conv1d_bhl.cu:124).
//
// One CTA computes a tile of kTile outputs of one (b, c) row: it stages the
// input window [o0 - pad, o0 - pad + kTile + K - 1) in shared memory as fp32
// with 16-byte global loads (zero outside [0, L)), then each thread produces
// outputs o = tid, tid + 256, ... so shared-memory reads and global stores
// are contiguous across a warp.  HBM-bound: each input element is read once
// (plus a K-1 halo per tile) and each output written once.
#include "common.cuh"

namespace b200 {
namespace {

constexpr int kDwThreads = 256;
constexpr int kDwTile = 2048;

template <typename T, int KS>
__global__ void __launch_bounds__(kDwThreads)
dwconv1d_kernel(const T* __restrict__ x, const void* __restrict__ w, const void* __restrict__ bias,
                T* __restrict__ y, int wdt, int64_t C, int64_t L, int K_dyn, int64_t pad,
                int64_t Lout, int64_t tiles_per_row, bool vec_in) {
  const int K = KS > 0 ? KS : K_dyn;
  extern __shared__ float smem[];
  float* sw = smem;                          // K weights
  float* sx = smem + ((K + 3) & ~3);         // input window (16-byte aligned)
  const int64_t row = blockIdx.x / tiles_per_row;
  const int64_t tile = blockIdx.x % tiles_per_row;
  const int64_t c = row % C;
  const int64_t o0 = tile * kDwTile;
  const int nout = static_cast<int>(min64(kDwTile, Lout - o0));
  const int win = nout + K - 1;
  const T* xr = x + row * L;

  for (int k = threadIdx.x; k < K; k += kDwThreads) sw[k] = load_param(w, wdt, c * K + k);
  const float b = bias ? load_param(bias, wdt, c) : 0.f;

  const int64_t lbeg = o0 - pad;  // global index of sx[0]
  constexpr int V = Vec16<T>::N;
  if (vec_in) {
    // Vectors aligned to V elements covering [lbeg, lbeg + win); `sh` is the
    // offset of lbeg inside the first vector.
    const int64_t abeg = (lbeg >= 0 ? lbeg / V : -((-lbeg + V - 1) / V)) * V;
    const int sh = static_cast<int>(lbeg - abeg);
    const int nvec = (sh + win + V - 1) / V;
    for (int q = threadIdx.x; q < nvec; q += kDwThreads) {
      const int64_t l = abeg + static_cast<int64_t>(q) * V;
      float v[V];
      if (l >= 0 && l + V <= L) {
        unpack16<T>(ld_stream16(xr + l), v);
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const int64_t le = l + e;
          v[e] = (le >= 0 && le < L) ? to_f32(xr[le]) : 0.f;
        }
      }
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const int j = q * V + e - sh;
        if (j >= 0 && j < win) sx[j] = v[e];
      }
    }
  } else {
    for (int j = threadIdx.x; j < win; j += kDwThreads) {
      const int64_t l = lbeg + j;
      sx[j] = (l >= 0 && l < L) ? to_f32(xr[l]) : 0.f;
    }
  }
  __syncthreads();

  T* yr = y + row * Lout + o0;
  for (int o = threadIdx.x; o < nout; o += kDwThreads) {
    float acc = b;
    if (KS > 0) {
#pragma unroll
      for (int k = 0; k < KS; ++k) acc = fmaf(sw[k], sx[o + k], acc);
    } else {
      int k = 0;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (; k + 4 <= K; k += 4) {
        a0 = fmaf(sw[k], sx[o + k], a0);
        a1 = fmaf(sw[k + 1], sx[o + k + 1], a1);
        a2 = fmaf(sw[k + 2], sx[o + k + 2], a2);
        a3 = fmaf(sw[k + 3], sx[o + k + 3], a3);
      }
      for (; k < K; ++k) a0 = fmaf(sw[k], sx[o + k], a0);
      acc += (a0 + a1) + (a2 + a3);
    }
    yr[o] = from_f32<T>(acc);
  }
}

template <typename T>
int launch(const void* xv, const void* w, const void* bias, void* yv, int wdt, int64_t B,
           int64_t C, int64_t L, int64_t K, int64_t pad, int64_t Lout, cudaStream_t stream) {
  const T* x = static_cast<const T*>(xv);
  T* y = static_cast<T*>(yv);
  const int64_t tiles = (Lout + kDwTile - 1) / kDwTile;
  const int64_t blocks = B * C * tiles;
  if (blocks > 0x7fffffffLL) return fail_unsupported("grid too large");
  const size_t smem = (static_cast<size_t>((K + 3) & ~3LL) + kDwTile + K + 16) * sizeof(float);
  if (smem > static_cast<size_t>(max_smem_optin())) return fail_unsupported("kernel too wide");
  constexpr int V = Vec16<T>::N;
  const bool vec_in = aligned16(x) && (L % V == 0);
  const unsigned grid = static_cast<unsigned>(blocks);
  const int Ki = static_cast<int>(K);
#define B200_DW_LAUNCH(KS)                                                                   \
  do {                                                                                      \
    auto kern = dwconv1d_kernel<T, KS>;                                                     \
    if (smem > 48 * 1024)                                                                   \
      B200_CUDA_CHECK(                                                                      \
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    kern<<<grid, kDwThreads, smem, stream>>>(x, w, bias, y, wdt, C, L, Ki, pad, Lout, tiles, \
                                             vec_in);                                       \
  } while (0)
  switch (Ki) {
    case 3: B200_DW_LAUNCH(3); break;
    case 5: B200_DW_LAUNCH(5); break;
    case 7: B200_DW_LAUNCH(7); break;
    case 4: B200_DW_LAUNCH(4); break;
    default: B200_DW_LAUNCH(0); break;
  }
#undef B200_DW_LAUNCH
  B200_LAUNCH_CHECK("dwconv1d_kernel");
  return B200_OK;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_dwconv1d_fwd(const void* x, const void* w, const void* bias, void* y,
                                 int dtype, int w_dtype, int64_t B, int64_t C, int64_t L,
                                 int64_t K, int64_t pad, int64_t L_out, int variant,
                                 void* stream) {
  (void)variant;
  if (!x || !w || !y) return fail_arg("x/w/y is NULL");
  if (!dtype_ok(dtype) || !dtype_ok(w_dtype)) return fail_arg("bad dtype");
  if (B <= 0 || C <= 0 || L <= 0 || K <= 0 || pad < 0) return fail_arg("bad size");
  if (L_out != L + 2 * pad - K + 1 || L_out <= 0) return fail_arg("L_out != L + 2*pad - K + 1");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_DTYPE_F32) return launch<float>(x, w, bias, y, w_dtype, B, C, L, K, pad, L_out, s);
  if (dtype == B200_DTYPE_F16) return launch<__half>(x, w, bias, y, w_dtype, B, C, L, K, pad, L_out, s);
  return launch<__nv_bfloat16>(x, w, bias, y, w_dtype, B, C, L, K, pad, L_out, s);
}
