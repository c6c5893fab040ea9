// Backward kernels for sm_100a: depthwise conv1d weight/bias gradients and
// GroupNorm input/affine gradients.
//
// Depthwise conv1d (forward y[b,c,o] = bias[c] + sum_k w[c,k] x[b,c,o-pad+k]):
//   dx is a depthwise correlation of dy with the reversed taps at padding
//   K-1-pad, so it runs on the forward kernels (b200_dwconv1d_fwd with
//   B200_DWCONV1D_FLIP_TAPS); this file adds
//     dw[c,k] = sum_{b,o} dy[b,c,o] * x[b,c,o-pad+k],  db[c] = sum_{b,o} dy[b,c,o]
//   as per-(row, tile) partial sums (one CTA stages a tile of dy and the
//   matching x window in shared memory) followed by a per-channel reduction
//   in a fixed order (fp64), so the result does not depend on scheduling.
//   The reference computes the same three gradients with its vendored
//   backward kernel (amd_tuned_torch/_vendor/flashfftconv_depthwise_conv1d/
//   conv1d_bwd_cuda_bhl.cu:19-114).
//
// GroupNorm (forward y = (x - mu_g) * rstd_g * gamma_c + beta_c, biased
// variance, eps inside the square root): with the group statistics of the
// forward recomputed by the caller (b200_gn_partial_stats), per (n, c) row
//   r1[n,c] = sum_s dy,   r2[n,c] = sum_s dy * (x - mu_g)
// and per (n, g), with M = C/G * S elements,
//   c1 = sum_{c in g} gamma_c r1 / M,   c2 = rstd * sum_{c in g} gamma_c r2 / M
// the gradients are
//   dx = rstd * (gamma_c dy - c1 - (x - mu) rstd c2)
//   dgamma[c] = sum_n rstd_{n,g} r2[n,c],   dbeta[c] = sum_n r1[n,c].
// Centring on the group mean before the product keeps r2 free of the
// E[dy x] - mu E[dy] cancellation.  Role of the reference's torch-ops
// derivative _group_norm_backward (amd_tuned_torch/_dispatch.py:2212-2302).
#include "common.cuh"

namespace b200 {
namespace {

constexpr int kBwThreads = 256;
constexpr int kBwTile = 2048;   // outputs of one row handled by one CTA (conv1d dw)
constexpr int kBwSmallK = 16;   // taps held in registers per thread

__device__ __forceinline__ void store_param(void* p, int dt, int64_t i, float v) {
  if (dt == B200_DTYPE_F32) {
    static_cast<float*>(p)[i] = v;
  } else if (dt == B200_DTYPE_F16) {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  } else {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
}

// ------------------------------------------------ conv1d weight gradient ---
// part[(c * P + b * tiles + tile) * (K + 1) + k], P = B * tiles; slot K holds
// the tile's sum of dy (bias gradient).
template <typename T, int KS>
__global__ void __launch_bounds__(kBwThreads)
dw_partial_kernel(const T* __restrict__ x, const T* __restrict__ dy, float* __restrict__ part,
                  int64_t B, int64_t C, int64_t L, int K_dyn, int64_t pad, int64_t Lout,
                  int64_t tiles) {
  const int K = KS > 0 ? KS : K_dyn;
  extern __shared__ float smem[];
  float* sdy = smem;             // kBwTile
  float* sx = smem + kBwTile;    // kBwTile + K - 1
  __shared__ float red[kBwThreads / 32][kBwSmallK + 1];
  const int64_t row = blockIdx.x / tiles;
  const int64_t tile = blockIdx.x % tiles;
  const int64_t b = row / C, c = row % C;
  const int64_t o0 = tile * kBwTile;
  const int n = static_cast<int>(min64(kBwTile, Lout - o0));
  const T* dyr = dy + row * Lout + o0;
  const T* xr = x + row * L;
  for (int j = threadIdx.x; j < n; j += kBwThreads) sdy[j] = to_f32(dyr[j]);
  const int64_t lbeg = o0 - pad;
  for (int j = threadIdx.x; j < n + K - 1; j += kBwThreads) {
    const int64_t l = lbeg + j;
    sx[j] = (l >= 0 && l < L) ? to_f32(xr[l]) : 0.f;
  }
  __syncthreads();
  const int P = static_cast<int>(B * tiles);
  float* out = part + (c * P + b * tiles + tile) * static_cast<int64_t>(K + 1);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (KS > 0) {
    float acc[KS + 1];
#pragma unroll
    for (int k = 0; k <= KS; ++k) acc[k] = 0.f;
    for (int o = threadIdx.x; o < n; o += kBwThreads) {
      const float d = sdy[o];
      acc[KS] += d;
#pragma unroll
      for (int k = 0; k < KS; ++k) acc[k] = fmaf(d, sx[o + k], acc[k]);
    }
#pragma unroll
    for (int k = 0; k <= KS; ++k) {
      const float v = warp_sum(acc[k]);
      if (lane == 0) red[warp][k] = v;
    }
    __syncthreads();
    if (threadIdx.x <= KS) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kBwThreads / 32; ++w) s += red[w][threadIdx.x];
      out[threadIdx.x] = s;
    }
  } else {
    // Wide filters: one thread per tap, dy broadcast from shared memory.
    for (int k = threadIdx.x; k < K; k += kBwThreads) {
      float a0 = 0.f, a1 = 0.f;
      int o = 0;
      for (; o + 2 <= n; o += 2) {
        a0 = fmaf(sdy[o], sx[o + k], a0);
        a1 = fmaf(sdy[o + 1], sx[o + 1 + k], a1);
      }
      if (o < n) a0 = fmaf(sdy[o], sx[o + k], a0);
      out[k] = a0 + a1;
    }
    float s = 0.f;
    for (int o = threadIdx.x; o < n; o += kBwThreads) s += sdy[o];
    s = warp_sum(s);
    if (lane == 0) red[warp][0] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kBwThreads / 32; ++w) t += red[w][0];
      out[K] = t;
    }
  }
}

// One CTA per channel: fixed-order fp64 sums of the P partials of each tap.
__global__ void __launch_bounds__(kBwThreads)
dw_reduce_kernel(const float* __restrict__ part, void* __restrict__ dw, void* __restrict__ db,
                 int wdt, int K, int64_t P) {
  const int64_t c = blockIdx.x;
  const float* base = part + c * P * (K + 1);
  for (int k = threadIdx.x; k <= K; k += kBwThreads) {
    double s = 0.0;
    for (int64_t p = 0; p < P; ++p) s += base[p * (K + 1) + k];
    if (k < K)
      store_param(dw, wdt, c * K + k, static_cast<float>(s));
    else if (db != nullptr)
      store_param(db, wdt, c, static_cast<float>(s));
  }
}

int64_t dw_tiles(int64_t Lout) { return (Lout + kBwTile - 1) / kBwTile; }

size_t dw_ws_bytes(int64_t B, int64_t C, int64_t K, int64_t Lout) {
  return static_cast<size_t>(C * B * dw_tiles(Lout) * (K + 1)) * sizeof(float);
}

template <typename T>
int launch_dw(const void* xv, const void* dyv, void* dw, void* db, int wdt, int64_t B, int64_t C,
              int64_t L, int64_t K, int64_t pad, int64_t Lout, float* part, cudaStream_t s) {
  const T* x = static_cast<const T*>(xv);
  const T* dy = static_cast<const T*>(dyv);
  const int64_t tiles = dw_tiles(Lout);
  const int64_t blocks = B * C * tiles;
  if (blocks > 0x7fffffffLL || C > 0x7fffffffLL) return fail_unsupported("grid too large");
  const size_t smem = static_cast<size_t>(2 * kBwTile + K) * sizeof(float);
  if (smem > static_cast<size_t>(max_smem_optin())) return fail_unsupported("filter too wide");
  const unsigned grid = static_cast<unsigned>(blocks);
  const int Ki = static_cast<int>(K);
#define B200_DW_PART(KS)                                                                      \
  do {                                                                                       \
    auto kern = dw_partial_kernel<T, KS>;                                                    \
    if (smem > 48 * 1024)                                                                    \
      B200_CUDA_CHECK(                                                                       \
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    kern<<<grid, kBwThreads, smem, s>>>(x, dy, part, B, C, L, Ki, pad, Lout, tiles);         \
  } while (0)
  switch (Ki) {
    case 1: B200_DW_PART(1); break;
    case 2: B200_DW_PART(2); break;
    case 3: B200_DW_PART(3); break;
    case 4: B200_DW_PART(4); break;
    case 5: B200_DW_PART(5); break;
    case 7: B200_DW_PART(7); break;
    case 9: B200_DW_PART(9); break;
    default: B200_DW_PART(0); break;
  }
#undef B200_DW_PART
  B200_LAUNCH_CHECK("dw_partial_kernel");
  dw_reduce_kernel<<<static_cast<unsigned>(C), kBwThreads, 0, s>>>(part, dw, db, wdt, Ki,
                                                                   B * tiles);
  B200_LAUNCH_CHECK("dw_reduce_kernel");
  return B200_OK;
}

// ------------------------------------------------------- GroupNorm bwd ---
constexpr int64_t kGnBwChunk = 16384;   // elements of one row per partial-sum CTA

int64_t gn_bw_chunk(int64_t S) { return S < kGnBwChunk ? S : kGnBwChunk; }

// part[row * chunks + ch] = (sum dy, sum dy * (x - mu_g)) over one chunk of a row.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
gn_bwd_partial_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                      const float* __restrict__ stats, float2* __restrict__ part, int64_t C,
                      int64_t S, int Cg, int G, int64_t chunk, int chunks) {
  __shared__ float scratch[33];
  const int64_t row = blockIdx.x / chunks;
  const int ch = blockIdx.x % chunks;
  const int64_t n = row / C, c = row % C;
  const int64_t ng = n * G + c / Cg;
  const float mean = stats[ng * 3 + 1];
  const int64_t beg = static_cast<int64_t>(ch) * chunk;
  const int64_t cnt = max64(0, min64(chunk, S - beg));
  const T* xs = x + row * S + beg;
  const T* ds = dy + row * S + beg;
  float s1 = 0.f, s2 = 0.f;
  constexpr int V = Vec16<T>::N;
  if (VEC) {
    const int64_t nv = cnt / V;
    for (int64_t i = threadIdx.x; i < nv; i += 256) {
      float xv[V], dv[V];
      unpack16<T>(ld_stream16(reinterpret_cast<const uint4*>(xs) + i), xv);
      unpack16<T>(ld_stream16(reinterpret_cast<const uint4*>(ds) + i), dv);
#pragma unroll
      for (int e = 0; e < V; ++e) {
        s1 += dv[e];
        s2 = fmaf(dv[e], xv[e] - mean, s2);
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < cnt; i += 256) {
      const float d = to_f32(ds[i]);
      s1 += d;
      s2 = fmaf(d, to_f32(xs[i]) - mean, s2);
    }
  }
  s1 = block_sum<256>(s1, scratch);
  s2 = block_sum<256>(s2, scratch);
  if (threadIdx.x == 0) part[row * chunks + ch] = make_float2(s1, s2);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One 128-thread CTA per (n, g): row totals rows[n*C + c] = (r1, r2) and the
// group's (rstd, mean, c1, c2).
__global__ void __launch_bounds__(128)
gn_bwd_group_kernel(const float2* __restrict__ part, const float* __restrict__ stats,
                    const void* __restrict__ gamma, int adt, float2* __restrict__ rows,
                    float4* __restrict__ coef, int64_t C, int G, int Cg, int chunks, float eps) {
  __shared__ double red[2][4];
  const int64_t ng = blockIdx.x;
  const int64_t n = ng / G;
  const int g = static_cast<int>(ng % G);
  double a1 = 0.0, a2 = 0.0;
  for (int j = threadIdx.x; j < Cg; j += 128) {
    const int64_t c = static_cast<int64_t>(g) * Cg + j;
    const int64_t row = n * C + c;
    double r1 = 0.0, r2 = 0.0;
    for (int ch = 0; ch < chunks; ++ch) {
      const float2 p = part[row * chunks + ch];
      r1 += p.x;
      r2 += p.y;
    }
    rows[row] = make_float2(static_cast<float>(r1), static_cast<float>(r2));
    const double gm = gamma ? static_cast<double>(load_param(gamma, adt, c)) : 1.0;
    a1 += gm * r1;
    a2 += gm * r2;
  }
  a1 = warp_sum_d(a1);
  a2 = warp_sum_d(a2);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    red[0][warp] = a1;
    red[1][warp] = a2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const double t1 = red[0][0] + red[0][1] + red[0][2] + red[0][3];
    const double t2 = red[1][0] + red[1][1] + red[1][2] + red[1][3];
    const double cnt = stats[ng * 3 + 0];
    const double mean = stats[ng * 3 + 1];
    const double rstd = 1.0 / sqrt(static_cast<double>(stats[ng * 3 + 2]) / cnt + eps);
    coef[ng] = make_float4(static_cast<float>(rstd), static_cast<float>(mean),
                           static_cast<float>(t1 / cnt), static_cast<float>(rstd * t2 / cnt));
  }
}

// dx = rstd * (gamma_c dy - c1 - (x - mean) rstd c2) over chunks of each group.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
gn_bwd_dx_kernel(const T* __restrict__ x, const T* __restrict__ dy, const float4* __restrict__ coef,
                 const void* __restrict__ gamma, int adt, T* __restrict__ dx, int64_t S, int G,
                 int Cg, int64_t chunk, int chunks) {
  const int64_t ng = blockIdx.x / chunks;
  const int ch = blockIdx.x % chunks;
  const int64_t M = static_cast<int64_t>(Cg) * S;
  const int64_t beg = static_cast<int64_t>(ch) * chunk;
  const int64_t cnt = max64(0, min64(chunk, M - beg));
  const float4 k = coef[ng];
  const float rstd = k.x, mean = k.y, c1 = k.z, c2 = k.w;
  const float xs = rstd * c2;        // coefficient of (x - mean) inside the bracket
  const int c0 = static_cast<int>(ng % G) * Cg;
  const T* xp = x + ng * M + beg;
  const T* dp = dy + ng * M + beg;
  T* op = dx + ng * M + beg;
  constexpr int V = Vec16<T>::N;
  if (VEC) {
    const int64_t nv = cnt / V;
    for (int64_t i = threadIdx.x; i < nv; i += 256) {
      const int c = c0 + static_cast<int>((beg + i * V) / S);
      const float gm = gamma ? load_param(gamma, adt, c) : 1.f;
      float xv[V], dv[V];
      unpack16<T>(ld_stream16(reinterpret_cast<const uint4*>(xp) + i), xv);
      unpack16<T>(ld_stream16(reinterpret_cast<const uint4*>(dp) + i), dv);
#pragma unroll
      for (int e = 0; e < V; ++e) xv[e] = rstd * (fmaf(gm, dv[e], -c1) - (xv[e] - mean) * xs);
      st_stream16(reinterpret_cast<uint4*>(op) + i, pack16<T>(xv));
    }
  } else {
    for (int64_t i = threadIdx.x; i < cnt; i += 256) {
      const int c = c0 + static_cast<int>((beg + i) / S);
      const float gm = gamma ? load_param(gamma, adt, c) : 1.f;
      const float v = rstd * (fmaf(gm, to_f32(dp[i]), -c1) - (to_f32(xp[i]) - mean) * xs);
      op[i] = from_f32<T>(v);
    }
  }
}

// dgamma[c] = sum_n rstd_{n,g} r2[n,c], dbeta[c] = sum_n r1[n,c] (fixed order, fp64).
__global__ void gn_bwd_param_kernel(const float2* __restrict__ rows, const float4* __restrict__ coef,
                                    void* __restrict__ dgamma, void* __restrict__ dbeta, int adt,
                                    int64_t N, int64_t C, int G, int Cg) {
  const int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (c >= C) return;
  const int64_t g = c / Cg;
  double sg = 0.0, sb = 0.0;
  for (int64_t n = 0; n < N; ++n) {
    const float2 r = rows[n * C + c];
    sg += static_cast<double>(coef[n * G + g].x) * r.y;
    sb += r.x;
  }
  if (dgamma) store_param(dgamma, adt, c, static_cast<float>(sg));
  if (dbeta) store_param(dbeta, adt, c, static_cast<float>(sb));
}

struct GnBwLayout {
  int64_t chunk, chunks;
  size_t part_off, rows_off, coef_off, total;
};

GnBwLayout gn_bw_layout(int64_t N, int64_t C, int64_t S, int64_t G) {
  GnBwLayout l;
  l.chunk = gn_bw_chunk(S);
  l.chunks = (S + l.chunk - 1) / l.chunk;
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  l.part_off = 0;
  l.rows_off = up(static_cast<size_t>(N * C * l.chunks) * sizeof(float2));
  l.coef_off = l.rows_off + up(static_cast<size_t>(N * C) * sizeof(float2));
  l.total = l.coef_off + up(static_cast<size_t>(N * G) * sizeof(float4));
  return l;
}

template <typename T>
int launch_gn_bwd(const void* xv, const void* dyv, const float* stats, const void* gamma,
                  void* dxv, void* dgamma, void* dbeta, int adt, int64_t N, int64_t C, int64_t S,
                  int64_t G, float eps, void* ws, const GnBwLayout& lay, cudaStream_t s) {
  const T* x = static_cast<const T*>(xv);
  const T* dy = static_cast<const T*>(dyv);
  T* dx = static_cast<T*>(dxv);
  constexpr int V = Vec16<T>::N;
  const int Cg = static_cast<int>(C / G);
  const bool vec = aligned16(x) && aligned16(dy) && (dx == nullptr || aligned16(dx)) && S % V == 0;
  unsigned char* base = static_cast<unsigned char*>(ws);
  float2* part = reinterpret_cast<float2*>(base + lay.part_off);
  float2* rows = reinterpret_cast<float2*>(base + lay.rows_off);
  float4* coef = reinterpret_cast<float4*>(base + lay.coef_off);
  if (N * C * lay.chunks > 0x7fffffffLL || N * G > 0x7fffffffLL)
    return fail_unsupported("grid too large");
  const unsigned g1 = static_cast<unsigned>(N * C * lay.chunks);
  const int nc = static_cast<int>(lay.chunks);
  if (vec)
    gn_bwd_partial_kernel<T, true><<<g1, 256, 0, s>>>(x, dy, stats, part, C, S, Cg, (int)G,
                                                      lay.chunk, nc);
  else
    gn_bwd_partial_kernel<T, false><<<g1, 256, 0, s>>>(x, dy, stats, part, C, S, Cg, (int)G,
                                                       lay.chunk, nc);
  B200_LAUNCH_CHECK("gn_bwd_partial_kernel");
  gn_bwd_group_kernel<<<static_cast<unsigned>(N * G), 128, 0, s>>>(part, stats, gamma, adt, rows,
                                                                   coef, C, (int)G, Cg, nc, eps);
  B200_LAUNCH_CHECK("gn_bwd_group_kernel");
  if (dx != nullptr) {
    const int64_t M = static_cast<int64_t>(Cg) * S;
    int64_t chunk = M < 65536 ? M : 65536;
    chunk = (chunk + V - 1) / V * V;
    const int64_t chunks = (M + chunk - 1) / chunk;
    if (N * G * chunks > 0x7fffffffLL) return fail_unsupported("grid too large");
    const unsigned g3 = static_cast<unsigned>(N * G * chunks);
    if (vec)
      gn_bwd_dx_kernel<T, true><<<g3, 256, 0, s>>>(x, dy, coef, gamma, adt, dx, S, (int)G, Cg,
                                                   chunk, (int)chunks);
    else
      gn_bwd_dx_kernel<T, false><<<g3, 256, 0, s>>>(x, dy, coef, gamma, adt, dx, S, (int)G, Cg,
                                                    chunk, (int)chunks);
    B200_LAUNCH_CHECK("gn_bwd_dx_kernel");
  }
  if (dgamma != nullptr || dbeta != nullptr) {
    gn_bwd_param_kernel<<<static_cast<unsigned>((C + 127) / 128), 128, 0, s>>>(
        rows, coef, dgamma, dbeta, adt, N, C, (int)G, Cg);
    B200_LAUNCH_CHECK("gn_bwd_param_kernel");
  }
  return B200_OK;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

size_t b200_dwconv1d_bwd_workspace_bytes(int64_t B, int64_t C, int64_t K, int64_t L_out) {
  if (B <= 0 || C <= 0 || K <= 0 || L_out <= 0) return 0;
  return dw_ws_bytes(B, C, K, L_out);
}

int b200_dwconv1d_bwd_weight(const void* x, const void* dy, void* dw, void* dbias, int dtype,
                             int w_dtype, int64_t B, int64_t C, int64_t L, int64_t K, int64_t pad,
                             int64_t L_out, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (!x || !dy || !dw) return fail_arg("x/dy/dw is NULL");
  if (!dtype_ok(dtype) || !dtype_ok(w_dtype)) return fail_arg("bad dtype");
  if (B <= 0 || C <= 0 || L <= 0 || K <= 0 || pad < 0) return fail_arg("bad size");
  if (L_out != L + 2 * pad - K + 1 || L_out <= 0) return fail_arg("L_out != L + 2*pad - K + 1");
  if (workspace == nullptr || workspace_bytes < dw_ws_bytes(B, C, K, L_out))
    return fail_arg("dwconv1d backward workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  if (dtype == B200_DTYPE_F32)
    return launch_dw<float>(x, dy, dw, dbias, w_dtype, B, C, L, K, pad, L_out, part, s);
  if (dtype == B200_DTYPE_F16)
    return launch_dw<__half>(x, dy, dw, dbias, w_dtype, B, C, L, K, pad, L_out, part, s);
  return launch_dw<__nv_bfloat16>(x, dy, dw, dbias, w_dtype, B, C, L, K, pad, L_out, part, s);
}

size_t b200_gn_bwd_workspace_bytes(int64_t N, int64_t C, int64_t S, int64_t G) {
  if (N <= 0 || C <= 0 || S <= 0 || G <= 0 || C % G != 0) return 0;
  return gn_bw_layout(N, C, S, G).total;
}

int b200_gn_bwd(const void* x, const void* dy, const float* stats, const void* gamma, void* dx,
                void* dgamma, void* dbeta, int dtype, int affine_dtype, int64_t N, int64_t C,
                int64_t S, int64_t G, float eps, void* workspace, size_t workspace_bytes,
                void* stream) {
  if (!x || !dy || !stats) return fail_arg("x/dy/stats is NULL");
  if (!dtype_ok(dtype) || ((gamma || dgamma || dbeta) && !dtype_ok(affine_dtype)))
    return fail_arg("bad dtype");
  if (N <= 0 || C <= 0 || S <= 0 || G <= 0) return fail_arg("non-positive GroupNorm size");
  if (C % G != 0) return fail_arg("C must be divisible by num_groups");
  const GnBwLayout lay = gn_bw_layout(N, C, S, G);
  if (workspace == nullptr || workspace_bytes < lay.total)
    return fail_arg("GroupNorm backward workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_DTYPE_F32)
    return launch_gn_bwd<float>(x, dy, stats, gamma, dx, dgamma, dbeta, affine_dtype, N, C, S,
                                G, eps, workspace, lay, s);
  if (dtype == B200_DTYPE_F16)
    return launch_gn_bwd<__half>(x, dy, stats, gamma, dx, dgamma, dbeta, affine_dtype, N, C, S,
                                 G, eps, workspace, lay, s);
  return launch_gn_bwd<__nv_bfloat16>(x, dy, stats, gamma, dx, dgamma, dbeta, affine_dtype, N,
                                      C, S, G, eps, workspace, lay, s);
}

}  // extern "C"
