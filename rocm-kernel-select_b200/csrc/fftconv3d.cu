// Dense conv3d through the FFT (large kernels), sm_100a.
//
// Reference: fftconv_ops.fft_conv3d -> fft_conv (amd_tuned_torch/fftconv_ops.py
// :603-746, :749-781): zero-pad, rfftn (fp32), multiply by the conjugated
// kernel spectrum and contract over input channels per frequency bin
// (complex_matmul, :480-543), irfftn, crop, + bias.
//
// Layout of the computation (Fd x Fh x Fw transform, 2/3/5-smooth, each <= 256):
//  * Batch items are packed in pairs as the real and imaginary parts of one
//    complex volume (P = ceil(N/2) pairs).  Because the contraction is linear
//    and the kernel real, the inverse transform of
//    U = sum_ci (X_a + i X_b) H = Y_a + i Y_b returns y_a + i y_b.
//  * K1 plane_fwd: one CTA per (pair, ci, input plane): the zero-padded
//    Fh x Fw plane through row then column FFTs in shared memory -> G.
//  * K2 depth_fwd: one CTA per (pair, 4 columns): Fd-point FFTs along depth
//    for all ci -> Z[bin][pair][ci] (natural frequency order).
//  * K3 contract: one warp per STORED bin of the weight spectrum, which keeps
//    only fw <= Fw/2 (the kernel is real, so H[-f] = conj(H[f])): the warp
//    produces U[f] = sum_ci Z[f] H[f] and U[-f] = sum_ci Z[-f] conj(H[f]),
//    reading each weight-spectrum element once.  This kernel streams the
//    cached weight spectrum and bounds the route.
//  * K4 depth_inv / K5 plane_inv: the inverse transforms, crop to the output
//    volume, 1/(Fd Fh Fw) scale, bias, dtype conversion.
// The weight spectrum H[hb][ci][co] (conjugated) is built once per weight by
// the same K1/K2 on pairs of output channels plus a Hermitian separation
// (K_sep) and cached by the caller.
#include "fft_core.cuh"

namespace b200 {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxDim = 256;
constexpr int kCols = 4;   // transform columns per depth-FFT CTA

struct Plan3 {
  fft::Plan d, h, w;
};

// Position of natural frequency f after a forward DIF with plan p.
__device__ __forceinline__ int dpos(int f, const fft::Plan& p) {
  int pos = 0, span = p.n;
  for (int i = 0; i < p.passes; ++i) {
    const int r = p.radix[i];
    span /= r;
    pos += (f % r) * span;
    f /= r;
  }
  return pos;
}

__device__ __forceinline__ void build_small_tw(float2* tw, int n) {
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    double s, c;
    sincospi(-2.0 * t / static_cast<double>(n), &s, &c);
    tw[t] = make_float2(static_cast<float>(c), static_cast<float>(s));
  }
}

// One pass over nseq sequences; element j of sequence s at buf[s*ss + j*es].
template <int R, bool INV>
__device__ __forceinline__ void bpass(float2* buf, int n, int span, int nseq, int ss, int es,
                                      const float2* tw) {
  const int stride = span / R, per = n / R, total = nseq * per, tscale = n / span;
  for (int b = threadIdx.x; b < total; b += blockDim.x) {
    const int s = b / per, bb = b - s * per;
    const int g = bb / stride, k = bb - g * stride;
    float2* base = buf + s * ss + (g * span + k) * es;
    float2 v[R];
#pragma unroll
    for (int m = 0; m < R; ++m) v[m] = base[m * stride * es];
    if (!INV) {
      fft::Dft<R, false>::run(v);
      if (k != 0) {
#pragma unroll
        for (int m = 1; m < R; ++m) v[m] = fft::cmul(v[m], tw[k * m * tscale]);
      }
    } else {
      if (k != 0) {
#pragma unroll
        for (int m = 1; m < R; ++m) v[m] = fft::cmulc(v[m], tw[k * m * tscale]);
      }
      fft::Dft<R, true>::run(v);
    }
#pragma unroll
    for (int m = 0; m < R; ++m) base[m * stride * es] = v[m];
  }
}

template <bool INV>
__device__ __forceinline__ void bpass_r(int r, float2* buf, int n, int span, int nseq, int ss,
                                        int es, const float2* tw) {
  switch (r) {
    case 16: bpass<16, INV>(buf, n, span, nseq, ss, es, tw); break;
    case 8: bpass<8, INV>(buf, n, span, nseq, ss, es, tw); break;
    case 4: bpass<4, INV>(buf, n, span, nseq, ss, es, tw); break;
    case 2: bpass<2, INV>(buf, n, span, nseq, ss, es, tw); break;
    case 9: bpass<9, INV>(buf, n, span, nseq, ss, es, tw); break;
    case 3: bpass<3, INV>(buf, n, span, nseq, ss, es, tw); break;
    default: bpass<5, INV>(buf, n, span, nseq, ss, es, tw); break;
  }
}

// Batched forward (DIF, digit-reversed out) or inverse (DIT, natural out).
template <bool INV>
__device__ __forceinline__ void bfft(float2* buf, const fft::Plan& p, int nseq, int ss, int es,
                                     const float2* tw) {
  if (!INV) {
    int span = p.n;
    for (int i = 0; i < p.passes; ++i) {
      bpass_r<false>(p.radix[i], buf, p.n, span, nseq, ss, es, tw);
      span /= p.radix[i];
      __syncthreads();
    }
  } else {
    int span = p.radix[p.passes - 1];
    for (int i = p.passes - 1; i >= 0; --i) {
      bpass_r<true>(p.radix[i], buf, p.n, span, nseq, ss, es, tw);
      if (i > 0) span *= p.radix[i - 1];
      __syncthreads();
    }
  }
}

// --------------------------------------------------------------- K1 -----
// items [n_items][C][Dz][H][W] real (T); pair p packs items item0+2p, +2p+1.
// Output G[p][c][dz][Fh][Fw] complex, natural order.  Placement offset
// (oh, ow) of the real data inside the transform plane.
template <typename T>
__global__ void __launch_bounds__(kThreads)
plane_fwd_kernel(const T* __restrict__ x, float2* __restrict__ G, int64_t n_items, int64_t item0,
                 int C, int Dz, int H, int W, int oh, int ow, const Plan3 pl) {
  extern __shared__ float2 sm[];
  const int Fh = pl.h.n, Fw = pl.w.n, RS = Fw + 1;
  float2* twh = sm;
  float2* tww = twh + Fh;
  float2* buf = tww + Fw;
  const int64_t per_pair = static_cast<int64_t>(C) * Dz;
  const int64_t p = blockIdx.x / per_pair;
  const int c = static_cast<int>((blockIdx.x / Dz) % C);
  const int dz = static_cast<int>(blockIdx.x % Dz);
  const int64_t i0 = item0 + 2 * p, i1 = i0 + 1;
  const bool has1 = i1 < n_items;
  const int64_t plane = static_cast<int64_t>(H) * W;
  const T* x0 = x + ((i0 * C + c) * Dz + dz) * plane;
  const T* x1 = x + ((min64(i1, n_items - 1) * C + c) * Dz + dz) * plane;
  build_small_tw(twh, Fh);
  build_small_tw(tww, Fw);
  for (int idx = threadIdx.x; idx < Fh * Fw; idx += blockDim.x) {
    const int hh = idx / Fw, ww = idx - hh * Fw;
    const int h = hh - oh, w = ww - ow;
    const bool in = h >= 0 && h < H && w >= 0 && w < W;
    const float re = in ? to_f32(x0[h * W + w]) : 0.f;
    const float im = (in && has1) ? to_f32(x1[h * W + w]) : 0.f;
    buf[hh * RS + ww] = make_float2(re, im);
  }
  __syncthreads();
  bfft<false>(buf, pl.w, Fh, RS, 1, tww);   // rows
  bfft<false>(buf, pl.h, Fw, 1, RS, twh);   // columns
  float2* g = G + ((p * C + c) * Dz + dz) * static_cast<int64_t>(Fh) * Fw;
  for (int idx = threadIdx.x; idx < Fh * Fw; idx += blockDim.x) {
    const int fh = idx / Fw, fw = idx - fh * Fw;
    g[idx] = buf[dpos(fh, pl.h) * RS + dpos(fw, pl.w)];
  }
}

// --------------------------------------------------------------- K2 -----
// G[p][c][dz][Fh*Fw] (Dz planes at depth offset od) -> Z[bin][p][c].
__global__ void __launch_bounds__(kThreads)
depth_fwd_kernel(const float2* __restrict__ G, float2* __restrict__ Z, int P, int C, int Dz,
                 int od, const Plan3 pl) {
  extern __shared__ float2 sm[];
  const int Fd = pl.d.n, cols = pl.h.n * pl.w.n, SS = Fd + 1;
  float2* twd = sm;
  float2* buf = twd + Fd;
  const int tiles = (cols + kCols - 1) / kCols;
  const int p = blockIdx.x / tiles;
  const int col0 = (blockIdx.x % tiles) * kCols;
  build_small_tw(twd, Fd);
  const int nseq = C * kCols;
  for (int idx = threadIdx.x; idx < nseq * Fd; idx += blockDim.x) {
    const int c = idx / (Fd * kCols);
    const int r = idx - c * Fd * kCols;
    const int j = r / kCols, q = r - j * kCols;   // q fastest: contiguous columns
    const int d = j - od, col = col0 + q;
    float2 v = make_float2(0.f, 0.f);
    if (d >= 0 && d < Dz && col < cols)
      v = G[((static_cast<int64_t>(p) * C + c) * Dz + d) * cols + col];
    buf[(c * kCols + q) * SS + j] = v;
  }
  __syncthreads();
  bfft<false>(buf, pl.d, nseq, SS, 1, twd);
  for (int idx = threadIdx.x; idx < nseq * Fd; idx += blockDim.x) {
    const int c = idx % C;                        // c fastest: contiguous output
    const int r = idx / C;
    const int q = r % kCols, fd = r / kCols;
    const int col = col0 + q;
    if (col >= cols) continue;
    Z[((static_cast<int64_t>(fd) * cols + col) * P + p) * C + c] =
        buf[(c * kCols + q) * SS + dpos(fd, pl.d)];
  }
}

// --------------------------------------------------------------- K3 -----
// U[f][p][co] = sum_ci Z[f][p][ci] H[hb][ci][co], and the partner -f with
// conj(H).  One warp per stored bin, lanes over output channels.
__global__ void __launch_bounds__(kThreads)
contract_kernel(const float2* __restrict__ Z, const float2* __restrict__ Hs,
                float2* __restrict__ U, int P, int Cin, int Cout, int Fd, int Fh, int Fw,
                int64_t hbins) {
  const int lane = threadIdx.x & 31;
  const int64_t hb = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  if (hb >= hbins) return;
  const int Fw2 = Fw / 2 + 1;
  const int fw = static_cast<int>(hb % Fw2);
  const int fh = static_cast<int>((hb / Fw2) % Fh);
  const int fd = static_cast<int>(hb / (static_cast<int64_t>(Fw2) * Fh));
  const int64_t f = (static_cast<int64_t>(fd) * Fh + fh) * Fw + fw;
  const bool neg = fw > 0 && 2 * fw != Fw;
  const int64_t fn = (static_cast<int64_t>((Fd - fd) % Fd) * Fh + (Fh - fh) % Fh) * Fw + (Fw - fw);
  const float2* h = Hs + hb * Cin * Cout;
  for (int p = 0; p < P; ++p) {
    const float2* zf = Z + (f * P + p) * Cin;
    const float2* zn = Z + (fn * P + p) * Cin;
    for (int co0 = 0; co0 < Cout; co0 += 64) {
      const int c0 = co0 + lane, c1 = co0 + 32 + lane;
      float2 a0 = make_float2(0.f, 0.f), a1 = a0, b0 = a0, b1 = a0;
      for (int ci = 0; ci < Cin; ++ci) {
        const float2 z = __ldg(zf + ci);
        const float2 zz = neg ? __ldg(zn + ci) : make_float2(0.f, 0.f);
        const float2 h0 = c0 < Cout ? __ldg(h + static_cast<int64_t>(ci) * Cout + c0) : z;
        const float2 h1 = c1 < Cout ? __ldg(h + static_cast<int64_t>(ci) * Cout + c1) : z;
        a0.x = fmaf(z.x, h0.x, fmaf(-z.y, h0.y, a0.x));
        a0.y = fmaf(z.x, h0.y, fmaf(z.y, h0.x, a0.y));
        a1.x = fmaf(z.x, h1.x, fmaf(-z.y, h1.y, a1.x));
        a1.y = fmaf(z.x, h1.y, fmaf(z.y, h1.x, a1.y));
        // zz * conj(h)
        b0.x = fmaf(zz.x, h0.x, fmaf(zz.y, h0.y, b0.x));
        b0.y = fmaf(zz.y, h0.x, fmaf(-zz.x, h0.y, b0.y));
        b1.x = fmaf(zz.x, h1.x, fmaf(zz.y, h1.y, b1.x));
        b1.y = fmaf(zz.y, h1.x, fmaf(-zz.x, h1.y, b1.y));
      }
      float2* uf = U + (f * P + p) * Cout;
      float2* un = U + (fn * P + p) * Cout;
      if (c0 < Cout) uf[c0] = a0;
      if (c1 < Cout) uf[c1] = a1;
      if (neg) {
        if (c0 < Cout) un[c0] = b0;
        if (c1 < Cout) un[c1] = b1;
      }
    }
  }
}

// --------------------------------------------------------------- K4 -----
// U[bin][p][co] -> G2[p][co][od < Do][Fh*Fw] (inverse depth FFT).
__global__ void __launch_bounds__(kThreads)
depth_inv_kernel(const float2* __restrict__ U, float2* __restrict__ G2, int P, int C, int Do,
                 const Plan3 pl) {
  extern __shared__ float2 sm[];
  const int Fd = pl.d.n, cols = pl.h.n * pl.w.n, SS = Fd + 1;
  float2* twd = sm;
  float2* buf = twd + Fd;
  const int tiles = (cols + kCols - 1) / kCols;
  const int p = blockIdx.x / tiles;
  const int col0 = (blockIdx.x % tiles) * kCols;
  build_small_tw(twd, Fd);
  const int nseq = C * kCols;
  for (int idx = threadIdx.x; idx < nseq * Fd; idx += blockDim.x) {
    const int c = idx % C;
    const int r = idx / C;
    const int q = r % kCols, fd = r / kCols;
    const int col = col0 + q;
    float2 v = make_float2(0.f, 0.f);
    if (col < cols) v = U[((static_cast<int64_t>(fd) * cols + col) * P + p) * C + c];
    buf[(c * kCols + q) * SS + dpos(fd, pl.d)] = v;
  }
  __syncthreads();
  bfft<true>(buf, pl.d, nseq, SS, 1, twd);
  for (int idx = threadIdx.x; idx < C * Do * kCols; idx += blockDim.x) {
    const int c = idx / (Do * kCols);
    const int r = idx - c * Do * kCols;
    const int o = r / kCols, q = r - o * kCols;
    const int col = col0 + q;
    if (col >= cols) continue;
    G2[((static_cast<int64_t>(p) * C + c) * Do + o) * cols + col] = buf[(c * kCols + q) * SS + o];
  }
}

// --------------------------------------------------------------- K5 -----
// G2[p][co][od][Fh*Fw] -> y[n][co][od][Ho][Wo] (inverse plane FFT, crop,
// scale, bias).
template <typename T>
__global__ void __launch_bounds__(kThreads)
plane_inv_kernel(const float2* __restrict__ G2, T* __restrict__ y, const void* __restrict__ bias,
                 int bias_dt, int64_t N, int C, int Do, int Ho, int Wo, float scale,
                 const Plan3 pl) {
  extern __shared__ float2 sm[];
  const int Fh = pl.h.n, Fw = pl.w.n, RS = Fw + 1;
  float2* twh = sm;
  float2* tww = twh + Fh;
  float2* buf = tww + Fw;
  const int64_t per_pair = static_cast<int64_t>(C) * Do;
  const int64_t p = blockIdx.x / per_pair;
  const int c = static_cast<int>((blockIdx.x / Do) % C);
  const int od = static_cast<int>(blockIdx.x % Do);
  build_small_tw(twh, Fh);
  build_small_tw(tww, Fw);
  const float2* g = G2 + ((p * C + c) * Do + od) * static_cast<int64_t>(Fh) * Fw;
  for (int idx = threadIdx.x; idx < Fh * Fw; idx += blockDim.x) {
    const int fh = idx / Fw, fw = idx - fh * Fw;
    buf[dpos(fh, pl.h) * RS + dpos(fw, pl.w)] = g[idx];
  }
  __syncthreads();
  bfft<true>(buf, pl.h, Fw, 1, RS, twh);
  bfft<true>(buf, pl.w, Fh, RS, 1, tww);
  const float bv = bias ? load_param(bias, bias_dt, c) : 0.f;
  const int64_t n0 = 2 * p, n1 = n0 + 1;
  const int64_t vol = static_cast<int64_t>(Do) * Ho * Wo;
  T* y0 = y + (n0 * C + c) * vol + static_cast<int64_t>(od) * Ho * Wo;
  T* y1 = y + (min64(n1, N - 1) * C + c) * vol + static_cast<int64_t>(od) * Ho * Wo;
  for (int idx = threadIdx.x; idx < Ho * Wo; idx += blockDim.x) {
    const int h = idx / Wo, w = idx - h * Wo;
    const float2 v = buf[h * RS + w];
    y0[idx] = from_f32<T>(fmaf(v.x, scale, bv));
    if (n1 < N) y1[idx] = from_f32<T>(fmaf(v.y, scale, bv));
  }
}

// ------------------------------------------------------------ K_sep -----
// Weight spectrum: Zw[bin][0][ci] packs output channels (co0, co0 + 1) as
// real/imag; split them by Hermitian symmetry and store the conjugates for
// the stored half (fw <= Fw/2) as Hs[hb][ci][co].
__global__ void separate_kernel(const float2* __restrict__ Zw, float2* __restrict__ Hs, int Cin,
                                int Cout, int co0, int Fd, int Fh, int Fw, int64_t hbins) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= hbins * Cin) return;
  const int ci = static_cast<int>(idx % Cin);
  const int64_t hb = idx / Cin;
  const int Fw2 = Fw / 2 + 1;
  const int fw = static_cast<int>(hb % Fw2);
  const int fh = static_cast<int>((hb / Fw2) % Fh);
  const int fd = static_cast<int>(hb / (static_cast<int64_t>(Fw2) * Fh));
  const int64_t f = (static_cast<int64_t>(fd) * Fh + fh) * Fw + fw;
  const int64_t fn = (static_cast<int64_t>((Fd - fd) % Fd) * Fh + (Fh - fh) % Fh) * Fw +
                     (Fw - fw) % Fw;
  const float2 a = Zw[f * Cin + ci], b = Zw[fn * Cin + ci];
  // A = (a + conj(b)) / 2, B = (a - conj(b)) / (2i); store conj(A), conj(B).
  const float2 A = make_float2(0.5f * (a.x + b.x), 0.5f * (a.y - b.y));
  const float2 Bv = make_float2(0.5f * (a.y + b.y), 0.5f * (b.x - a.x));
  float2* out = Hs + (hb * Cin + ci) * Cout;
  out[co0] = make_float2(A.x, -A.y);
  if (co0 + 1 < Cout) out[co0 + 1] = make_float2(Bv.x, -Bv.y);
}

// ------------------------------------------------------------ host ------
struct Sizes {
  int64_t bins, hbins, P;
  size_t g_bytes, z_bytes, u_bytes;
};

bool plan3(int64_t fd, int64_t fh, int64_t fw, Plan3* p) {
  if (fd > kMaxDim || fh > kMaxDim || fw > kMaxDim || fw % 2 != 0) return false;
  return fft::make_plan(fd, &p->d) && fft::make_plan(fh, &p->h) && fft::make_plan(fw, &p->w);
}

Sizes sizes(int64_t N, int64_t Cin, int64_t Cout, int64_t fd, int64_t fh, int64_t fw) {
  Sizes s;
  s.P = (N + 1) / 2;
  s.bins = fd * fh * fw;
  s.hbins = fd * fh * (fw / 2 + 1);
  const int64_t cmax = Cin > Cout ? Cin : Cout;
  s.g_bytes = static_cast<size_t>(s.P * cmax * fd * fh * fw) * sizeof(float2);
  s.z_bytes = static_cast<size_t>(s.bins * s.P * Cin) * sizeof(float2);
  s.u_bytes = static_cast<size_t>(s.bins * s.P * Cout) * sizeof(float2);
  return s;
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

size_t plane_smem(const Plan3& p) {
  return static_cast<size_t>(p.h.n + p.w.n + p.h.n * (p.w.n + 1)) * sizeof(float2);
}
size_t depth_smem(const Plan3& p, int C) {
  return static_cast<size_t>(p.d.n + C * kCols * (p.d.n + 1)) * sizeof(float2);
}

template <typename K>
int set_smem(K kern, size_t smem) {
  if (smem > static_cast<size_t>(max_smem_optin())) return fail_unsupported("transform too large for shared memory");
  B200_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
  return B200_OK;
}

// K1 + K2 over pairs [pair0, pair0 + npairs) of `items`.
template <typename T>
int forward_volume(const T* x, float2* G, float2* Z, int64_t n_items, int64_t item0,
                   int64_t npairs, int C, int Dz, int H, int W, int od, int oh, int ow,
                   const Plan3& pl, cudaStream_t s) {
  int rc;
  const size_t ps = plane_smem(pl), ds = depth_smem(pl, C);
  if ((rc = set_smem(plane_fwd_kernel<T>, ps)) != B200_OK) return rc;
  if ((rc = set_smem(depth_fwd_kernel, ds)) != B200_OK) return rc;
  const int64_t g1 = npairs * C * Dz;
  if (g1 > 0x7fffffffLL) return fail_unsupported("grid too large");
  plane_fwd_kernel<T><<<(unsigned)g1, kThreads, ps, s>>>(x, G, n_items, item0, C, Dz, H, W, oh,
                                                         ow, pl);
  B200_LAUNCH_CHECK("plane_fwd_kernel");
  const int cols = pl.h.n * pl.w.n;
  const int64_t g2 = npairs * ((cols + kCols - 1) / kCols);
  depth_fwd_kernel<<<(unsigned)g2, kThreads, ds, s>>>(G, Z, (int)npairs, C, Dz, od, pl);
  B200_LAUNCH_CHECK("depth_fwd_kernel");
  return B200_OK;
}

template <typename T>
int prepare_typed(const void* wv, float2* Hs, int64_t Cout, int64_t Cin, int64_t KD, int64_t KH,
                  int64_t KW, const Plan3& pl, void* ws, size_t ws_bytes, cudaStream_t s) {
  const Sizes sz = sizes(1, Cin, Cout, pl.d.n, pl.h.n, pl.w.n);
  const size_t need = align256(sz.g_bytes) + align256(sz.z_bytes);
  if (!ws || ws_bytes < need) return fail_arg("fftconv3d prepare workspace too small");
  float2* G = static_cast<float2*>(ws);
  float2* Zw = reinterpret_cast<float2*>(static_cast<char*>(ws) + align256(sz.g_bytes));
  const T* w = static_cast<const T*>(wv);
  for (int64_t co0 = 0; co0 < Cout; co0 += 2) {
    int rc = forward_volume<T>(w, G, Zw, Cout, co0, 1, (int)Cin, (int)KD, (int)KH, (int)KW, 0, 0,
                               0, pl, s);
    if (rc != B200_OK) return rc;
    const int64_t n = sz.hbins * Cin;
    separate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(Zw, Hs, (int)Cin, (int)Cout,
                                                                (int)co0, pl.d.n, pl.h.n,
                                                                pl.w.n, sz.hbins);
    B200_LAUNCH_CHECK("separate_kernel");
  }
  return B200_OK;
}

template <typename T>
int fwd_typed(const void* xv, const float2* Hs, const void* bias, int bias_dt, void* yv,
              int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t Cout, int64_t Do,
              int64_t Ho, int64_t Wo, const int64_t* pad3, const Plan3& pl, void* ws,
              size_t ws_bytes, cudaStream_t s) {
  const Sizes sz = sizes(N, Cin, Cout, pl.d.n, pl.h.n, pl.w.n);
  const size_t need = align256(sz.g_bytes) + align256(sz.z_bytes) + align256(sz.u_bytes);
  if (!ws || ws_bytes < need) return fail_arg("fftconv3d workspace too small");
  float2* G = static_cast<float2*>(ws);
  float2* Z = reinterpret_cast<float2*>(static_cast<char*>(ws) + align256(sz.g_bytes));
  float2* U = reinterpret_cast<float2*>(reinterpret_cast<char*>(Z) + align256(sz.z_bytes));
  int rc = forward_volume<T>(static_cast<const T*>(xv), G, Z, N, 0, sz.P, (int)Cin, (int)D,
                             (int)H, (int)W, (int)pad3[0], (int)pad3[1], (int)pad3[2], pl, s);
  if (rc != B200_OK) return rc;
  const int64_t warps = sz.hbins;
  contract_kernel<<<(unsigned)((warps * 32 + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      Z, Hs, U, (int)sz.P, (int)Cin, (int)Cout, pl.d.n, pl.h.n, pl.w.n, sz.hbins);
  B200_LAUNCH_CHECK("contract_kernel");
  const size_t ds = depth_smem(pl, (int)Cout), ps = plane_smem(pl);
  if ((rc = set_smem(depth_inv_kernel, ds)) != B200_OK) return rc;
  if ((rc = set_smem(plane_inv_kernel<T>, ps)) != B200_OK) return rc;
  const int cols = pl.h.n * pl.w.n;
  float2* G2 = G;   // G is dead once Z is built
  depth_inv_kernel<<<(unsigned)(sz.P * ((cols + kCols - 1) / kCols)), kThreads, ds, s>>>(
      U, G2, (int)sz.P, (int)Cout, (int)Do, pl);
  B200_LAUNCH_CHECK("depth_inv_kernel");
  const float scale = 1.0f / static_cast<float>(static_cast<double>(pl.d.n) * pl.h.n * pl.w.n);
  const int64_t g5 = sz.P * Cout * Do;
  if (g5 > 0x7fffffffLL) return fail_unsupported("grid too large");
  plane_inv_kernel<T><<<(unsigned)g5, kThreads, ps, s>>>(G2, static_cast<T*>(yv), bias, bias_dt,
                                                         N, (int)Cout, (int)Do, (int)Ho, (int)Wo,
                                                         scale, pl);
  B200_LAUNCH_CHECK("plane_inv_kernel");
  return B200_OK;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

size_t b200_fftconv3d_spectrum_bytes(int64_t Cout, int64_t Cin, int64_t fd, int64_t fh,
                                     int64_t fw) {
  return static_cast<size_t>(Cout * Cin * fd * fh * (fw / 2 + 1)) * sizeof(float2);
}

size_t b200_fftconv3d_workspace_bytes(int64_t N, int64_t Cin, int64_t Cout, int64_t fd,
                                      int64_t fh, int64_t fw) {
  const Sizes s = sizes(N, Cin, Cout, fd, fh, fw);
  return align256(s.g_bytes) + align256(s.z_bytes) + align256(s.u_bytes);
}

int b200_fftconv3d_prepare(const void* w, void* spectrum, int w_dtype, int64_t Cout,
                           int64_t Cin, int64_t KD, int64_t KH, int64_t KW, int64_t fd,
                           int64_t fh, int64_t fw, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (!w || !spectrum) return fail_arg("NULL pointer");
  if (!dtype_ok(w_dtype)) return fail_arg("bad dtype");
  if (Cout <= 0 || Cin <= 0 || KD <= 0 || KH <= 0 || KW <= 0) return fail_arg("bad size");
  if (KD > fd || KH > fh || KW > fw) return fail_arg("kernel larger than the transform");
  Plan3 pl;
  if (!plan3(fd, fh, fw, &pl)) return fail_unsupported("transform extents unsupported");
  if (Cin > 4096 || Cout > 65535) return fail_unsupported("too many channels");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float2* H = static_cast<float2*>(spectrum);
  if (w_dtype == B200_DTYPE_F32)
    return prepare_typed<float>(w, H, Cout, Cin, KD, KH, KW, pl, workspace, workspace_bytes, s);
  if (w_dtype == B200_DTYPE_F16)
    return prepare_typed<__half>(w, H, Cout, Cin, KD, KH, KW, pl, workspace, workspace_bytes, s);
  return prepare_typed<__nv_bfloat16>(w, H, Cout, Cin, KD, KH, KW, pl, workspace,
                                      workspace_bytes, s);
}

int b200_fftconv3d_fwd(const void* x, const void* spectrum, const void* bias, void* y,
                       int dtype, int bias_dtype, int64_t N, int64_t Cin, int64_t D,
                       int64_t H, int64_t W, int64_t Cout, int64_t KD, int64_t KH, int64_t KW,
                       const int64_t* pad3, int64_t fd, int64_t fh, int64_t fw,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !spectrum || !y || !pad3) return fail_arg("NULL pointer");
  if (!dtype_ok(dtype) || (bias && !dtype_ok(bias_dtype))) return fail_arg("bad dtype");
  if (N <= 0 || Cin <= 0 || D <= 0 || H <= 0 || W <= 0 || Cout <= 0) return fail_arg("bad size");
  if (pad3[0] < 0 || pad3[1] < 0 || pad3[2] < 0) return fail_arg("negative padding");
  const int64_t Dp = D + 2 * pad3[0], Hp = H + 2 * pad3[1], Wp = W + 2 * pad3[2];
  if (Dp > fd || Hp > fh || Wp > fw) return fail_arg("transform shorter than the padded input");
  const int64_t Do = Dp - KD + 1, Ho = Hp - KH + 1, Wo = Wp - KW + 1;
  if (Do <= 0 || Ho <= 0 || Wo <= 0) return fail_arg("kernel larger than the padded input");
  Plan3 pl;
  if (!plan3(fd, fh, fw, &pl)) return fail_unsupported("transform extents unsupported");
  if (Cin > 4096 || Cout > 4096) return fail_unsupported("too many channels");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float2* Hs = static_cast<const float2*>(spectrum);
  if (dtype == B200_DTYPE_F32)
    return fwd_typed<float>(x, Hs, bias, bias_dtype, y, N, Cin, D, H, W, Cout, Do, Ho, Wo, pad3,
                            pl, workspace, workspace_bytes, s);
  if (dtype == B200_DTYPE_F16)
    return fwd_typed<__half>(x, Hs, bias, bias_dtype, y, N, Cin, D, H, W, Cout, Do, Ho, Wo, pad3,
                             pl, workspace, workspace_bytes, s);
  return fwd_typed<__nv_bfloat16>(x, Hs, bias, bias_dtype, y, N, Cin, D, H, W, Cout, Do, Ho, Wo,
                                  pad3, pl, workspace, workspace_bytes, s);
}

}  // extern "C"
