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
// Residency: every kernel here is latency-bound at low occupancy, so each
// carries a launch bound picked by measurement: the transforms three CTAs per
// SM (the 80 x 80 forward plane kernel four, at 64 registers), the
// contraction three for fp16 spectra and narrow outputs, two for fp32.  At
// the unbounded register counts (90-147) they ran one or two CTAs, too few
// warps to hide shared-memory and HBM latency.
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

// Digit-reversed position table of a plan (dpos for f = 0 .. n-1) in shared
// memory; the caller synchronises before use.
__device__ __forceinline__ void build_pos(int* pos, const fft::Plan& p) {
  for (int f = threadIdx.x; f < p.n; f += blockDim.x) pos[f] = dpos(f, p);
}

__device__ __forceinline__ void build_small_tw(float2* tw, int n) {
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    double s, c;
    sincospi(-2.0 * t / static_cast<double>(n), &s, &c);
    tw[t] = make_float2(static_cast<float>(c), static_cast<float>(s));
  }
}

// a / d for 0 <= a < 2^24 and 0 < d, from a float reciprocal of d plus one
// correction step (the float quotient is within 1 of the true one).
__device__ __forceinline__ int qdiv(int a, int d, float inv_d) {
  int q = __float2int_rz(__int2float_rz(a) * inv_d);
  const int r = a - q * d;
  if (r < 0) --q;
  else if (r >= d) ++q;
  return q;
}

// Gathers total elements into shared memory with kGather independent global
// loads in flight per thread: load(i) returns element i, slot(i) its
// shared-memory index.  (A plain loop leaves one load in flight per thread,
// and these kernels then wait out one memory latency per element.)
constexpr int kGather = 8;
template <int GD = kGather, typename LoadF, typename SlotF>
__device__ __forceinline__ void gather_smem(float2* buf, int total, LoadF load, SlotF slot) {
  for (int base = threadIdx.x; base < total; base += blockDim.x * GD) {
    float2 v[GD];
#pragma unroll
    for (int u = 0; u < GD; ++u) {
      const int i = base + u * static_cast<int>(blockDim.x);
      v[u] = i < total ? load(i) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < GD; ++u) {
      const int i = base + u * static_cast<int>(blockDim.x);
      if (i < total) buf[slot(i)] = v[u];
    }
  }
}

// Row stride (float2) of a plane in shared memory.  For rows of a multiple
// of 16 points the first radix-16 pass has 5 (or 4) butterflies per row, so
// a half-warp spans about four rows; a stride of 5 mod 16 puts those rows on
// distinct banks (measured at 80 x 80 planes: 632 -> 608 us for cfg 4a),
// where Fw + 1 (1 mod 16) made the rows collide.
__host__ __device__ __forceinline__ int plane_row_stride(int Fw) {
  return Fw % 16 == 0 ? Fw + 5 : Fw + 1;
}

// One pass over nseq sequences; element j of sequence s at buf[s*ss + j*es].
template <int R, bool INV>
__device__ __forceinline__ void bpass(float2* buf, int n, int span, int nseq, int ss, int es,
                                      const float2* tw) {
  const int stride = span / R, per = n / R, total = nseq * per, tscale = n / span;
  const float inv_per = 1.0f / static_cast<float>(per), inv_stride = 1.0f / static_cast<float>(stride);
  for (int b = threadIdx.x; b < total; b += blockDim.x) {
    const int s = qdiv(b, per, inv_per), bb = b - s * per;
    const int g = qdiv(bb, stride, inv_stride), k = bb - g * stride;
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

// Two-pass transforms of a compile-time plan RA x RB (the 80-point plane
// rows and columns of cfg 4a: 16 x 5): the pass geometry and the index
// divisions become constants (bpass divides by runtime pass sizes through
// qdiv and picks the radix with a switch per pass).
template <int R, bool INV, int N, int SPAN>
__device__ __forceinline__ void bpass_ct(float2* buf, int nseq, int ss, int es,
                                         const float2* tw) {
  constexpr int stride = SPAN / R, per = N / R, tscale = N / SPAN;
  const int total = nseq * per;
  for (int b = threadIdx.x; b < total; b += blockDim.x) {
    const int s = b / per, bb = b - s * per;
    const int g = bb / stride, k = bb - g * stride;
    float2* base = buf + s * ss + (g * SPAN + k) * es;
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

// bfft for a plan of exactly two passes RA, RB (same order and output as
// bfft with that plan).
template <bool INV, int RA, int RB>
__device__ __forceinline__ void bfft2_ct(float2* buf, int nseq, int ss, int es,
                                         const float2* tw) {
  constexpr int N = RA * RB;
  if (!INV) {
    bpass_ct<RA, false, N, N>(buf, nseq, ss, es, tw);
    __syncthreads();
    bpass_ct<RB, false, N, RB>(buf, nseq, ss, es, tw);
    __syncthreads();
  } else {
    bpass_ct<RB, true, N, RB>(buf, nseq, ss, es, tw);
    __syncthreads();
    bpass_ct<RA, true, N, N>(buf, nseq, ss, es, tw);
    __syncthreads();
  }
}

// Plane transforms: NP = 80 is the 80 x 80 plane with the 16 x 5 plan in
// both directions (compile-time), NP = 0 any plan.
template <bool INV, int NP>
__device__ __forceinline__ void plane_fft(float2* buf, const fft::Plan& p, int nseq, int ss,
                                          int es, const float2* tw) {
  if constexpr (NP == 80) {
    bfft2_ct<INV, 16, 5>(buf, nseq, ss, es, tw);
  } else {
    bfft<INV>(buf, p, nseq, ss, es, tw);
  }
}

template <int NP>
__device__ __forceinline__ int div_np(int a, int n, float inv_n) {
  if constexpr (NP != 0) {
    return a / NP;
  } else {
    return qdiv(a, n, inv_n);
  }
}

// Whether both plane plans are 80 = 16 x 5 (the NP = 80 plane kernels).
inline bool plane80(const fft::Plan& h, const fft::Plan& w) {
  auto is80 = [](const fft::Plan& p) {
    return p.n == 80 && p.passes == 2 && p.radix[0] == 16 && p.radix[1] == 5;
  };
  return is80(h) && is80(w);
}

// --------------------------------------------------------------- K1 -----
// items [n_items][C][Dz][H][W] real (T); pair p packs items item0+2p, +2p+1.
// Output G[p][c][dz][Fh][Fw] complex, natural order.  Placement offset
// (oh, ow) of the real data inside the transform plane.
// The 80 x 80 variant fits in 64 registers without spills and runs four CTAs
// per SM (cfg 4a: 66.5 -> 53.7 us; the inverse spills at 64 and stays at three).
template <typename T, int NP>
__global__ void __launch_bounds__(kThreads, NP ? 4 : 3)
plane_fwd_kernel(const T* __restrict__ x, float2* __restrict__ G, int64_t n_items, int64_t item0,
                 int C, int Dz, int H, int W, int oh, int ow, const Plan3 pl) {
  extern __shared__ float2 sm[];
  const int Fh = NP ? NP : pl.h.n, Fw = NP ? NP : pl.w.n, RS = plane_row_stride(Fw);
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
  const float inv_fw0 = 1.0f / static_cast<float>(Fw);
  gather_smem(
      buf, Fh * Fw,
      [&](int idx) {
        const int hh = div_np<NP>(idx, Fw, inv_fw0), ww = idx - hh * Fw;
        const int h = hh - oh, w = ww - ow;
        const bool in = h >= 0 && h < H && w >= 0 && w < W;
        return make_float2(in ? to_f32(x0[h * W + w]) : 0.f,
                           (in && has1) ? to_f32(x1[h * W + w]) : 0.f);
      },
      [&](int idx) {
        const int hh = div_np<NP>(idx, Fw, inv_fw0);
        return hh * RS + (idx - hh * Fw);
      });
  __syncthreads();
  int* posh = reinterpret_cast<int*>(buf + Fh * RS);
  int* posw = posh + Fh;
  build_pos(posh, pl.h);
  build_pos(posw, pl.w);
  // Rows (their barriers also publish posh / posw); rows outside the data are
  // zero and stay zero, so only the H data rows are transformed.
  {
    const int r0 = oh > 0 ? oh : 0, r1 = oh + H < Fh ? oh + H : Fh;
    if (r1 > r0) {
      plane_fft<false, NP>(buf + r0 * RS, pl.w, r1 - r0, RS, 1, tww);
    } else {
      __syncthreads();
    }
  }
  plane_fft<false, NP>(buf, pl.h, Fw, 1, RS, twh);   // columns
  float2* g = G + ((p * C + c) * Dz + dz) * static_cast<int64_t>(Fh) * Fw;
  const float inv_fw = 1.0f / static_cast<float>(Fw);
  for (int idx = threadIdx.x; idx < Fh * Fw; idx += blockDim.x) {
    const int fh = div_np<NP>(idx, Fw, inv_fw), fw = idx - fh * Fw;
    g[idx] = buf[posh[fh] * RS + posw[fw]];
  }
}

// --------------------------------------------------------------- K2 -----
// G[p][c][dz][Fh*Fw] (Dz planes at depth offset od) -> Z[bin][p][c].
__global__ void __launch_bounds__(kThreads, 3)
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
  int* posd = reinterpret_cast<int*>(buf + nseq * SS);
  build_pos(posd, pl.d);
  const int fk = Fd * kCols;
  const float inv_fk = 1.0f / static_cast<float>(fk);
  gather_smem(
      buf, nseq * Fd,
      [&](int idx) {
        const int c = qdiv(idx, fk, inv_fk);
        const int r = idx - c * fk;
        const int j = r / kCols, q = r - j * kCols;   // q fastest: contiguous columns
        const int d = j - od, col = col0 + q;
        return (d >= 0 && d < Dz && col < cols)
                   ? G[((static_cast<int64_t>(p) * C + c) * Dz + d) * cols + col]
                   : make_float2(0.f, 0.f);
      },
      [&](int idx) {
        const int c = qdiv(idx, fk, inv_fk);
        const int r = idx - c * fk;
        const int j = r / kCols, q = r - j * kCols;
        return (c * kCols + q) * SS + j;
      });
  __syncthreads();
  bfft<false>(buf, pl.d, nseq, SS, 1, twd);
  const float inv_c = 1.0f / static_cast<float>(C);
  for (int idx = threadIdx.x; idx < nseq * Fd; idx += blockDim.x) {
    const int r = qdiv(idx, C, inv_c);
    const int c = idx - r * C;                    // c fastest: contiguous output
    const int q = r % kCols, fd = r / kCols;
    const int col = col0 + q;
    if (col >= cols) continue;
    Z[((static_cast<int64_t>(fd) * cols + col) * P + p) * C + c] =
        buf[(c * kCols + q) * SS + posd[fd]];
  }
}

// ------------------------------------------------ K2 / K4, in registers ---
// Depth transforms of a compile-time length FD (30 for the cfg 4a shapes)
// with each sequence in one thread's registers (fft::Dft<FD>, natural order
// in and out).  A CTA takes 16 columns x 16 channels of one pair: the loads
// read 16 consecutive columns (128 bytes) per (channel, depth); the switch to
// the channel-fastest spectrum layout goes through shared memory, so the
// stores (K2) / loads (K4) move 16 consecutive channels per (bin, column).
// ~10x fewer instructions per point than the shared-memory pass engine.
constexpr int kDCols = 16, kDCh = 16;

template <int FD>
size_t depth_reg_smem() { return static_cast<size_t>(FD) * kDCols * (kDCh + 1) * sizeof(float2); }

// Three CTAs per SM (80 registers, no spills; cfg 4a op 484 -> 479 us), as
// the inverse below.
template <int FD>
__global__ void __launch_bounds__(kDCols * kDCh, 3)
depth_fwd_reg_kernel(const float2* __restrict__ G, float2* __restrict__ Z, int P, int C, int Dz,
                     int od, int cols) {
  extern __shared__ float2 sm[];   // [FD][kDCols][kDCh + 1]
  const int tcol = threadIdx.x % kDCols, tch = threadIdx.x / kDCols;
  const int ctiles = (cols + kDCols - 1) / kDCols, chtiles = (C + kDCh - 1) / kDCh;
  int b = blockIdx.x;
  const int coltile = b % ctiles;
  b /= ctiles;
  const int chtile = b % chtiles, p = b / chtiles;
  const int col = coltile * kDCols + tcol, c = chtile * kDCh + tch;
  float2 v[FD];
#pragma unroll
  for (int j = 0; j < FD; ++j) v[j] = make_float2(0.f, 0.f);
  if (col < cols && c < C) {
    const float2* g = G + (static_cast<int64_t>(p) * C + c) * Dz * cols + col;
#pragma unroll
    for (int j = 0; j < FD; ++j) {
      const int d = j - od;
      if (d >= 0 && d < Dz) v[j] = g[static_cast<int64_t>(d) * cols];
    }
  }
  fft::Dft<FD, false>::run(v);
#pragma unroll
  for (int f = 0; f < FD; ++f) sm[(f * kDCols + tcol) * (kDCh + 1) + tch] = v[f];
  __syncthreads();
  for (int i = threadIdx.x; i < FD * kDCols * kDCh; i += kDCols * kDCh) {
    const int cc = i % kDCh, r = i / kDCh, q = r % kDCols, f = r / kDCols;
    const int colw = coltile * kDCols + q, cw = chtile * kDCh + cc;
    if (colw < cols && cw < C)
      Z[((static_cast<int64_t>(f) * cols + colw) * P + p) * C + cw] =
          sm[(f * kDCols + q) * (kDCh + 1) + cc];
  }
}

template <int FD>
__global__ void __launch_bounds__(kDCols * kDCh, 3)
depth_inv_reg_kernel(const float2* __restrict__ U, float2* __restrict__ G2, int P, int C, int Do,
                     int cols) {
  extern __shared__ float2 sm[];   // [FD][kDCols][kDCh + 1]
  const int tcol = threadIdx.x % kDCols, tch = threadIdx.x / kDCols;
  const int ctiles = (cols + kDCols - 1) / kDCols, chtiles = (C + kDCh - 1) / kDCh;
  int b = blockIdx.x;
  const int coltile = b % ctiles;
  b /= ctiles;
  const int chtile = b % chtiles, p = b / chtiles;
  // Half of a thread's FD loads in flight at once (two batches): all FD at
  // once needed 128 registers (two CTAs per SM, 47 us at cfg 4a); two batches
  // fit three CTAs per SM at 80 (op 479 -> 474 us).
  gather_smem<(FD + 1) / 2>(
      sm, FD * kDCols * kDCh,
      [&](int i) {
        const int cc = i % kDCh, r = i / kDCh, q = r % kDCols, f = r / kDCols;
        const int colr = coltile * kDCols + q, cr = chtile * kDCh + cc;
        return (colr < cols && cr < C)
                   ? U[((static_cast<int64_t>(f) * cols + colr) * P + p) * C + cr]
                   : make_float2(0.f, 0.f);
      },
      [&](int i) {
        const int cc = i % kDCh, r = i / kDCh;
        return r * (kDCh + 1) + cc;
      });
  __syncthreads();
  const int col = coltile * kDCols + tcol, c = chtile * kDCh + tch;
  float2 v[FD];
#pragma unroll
  for (int f = 0; f < FD; ++f) v[f] = sm[(f * kDCols + tcol) * (kDCh + 1) + tch];
  fft::Dft<FD, true>::run(v);
  if (col < cols && c < C) {
    float2* g = G2 + (static_cast<int64_t>(p) * C + c) * Do * cols + col;
#pragma unroll
    for (int o = 0; o < FD; ++o)
      if (o < Do) g[static_cast<int64_t>(o) * cols] = v[o];
  }
}

// --------------------------------------------------------------- K3 -----
// U[f][p][co] = sum_ci Z[f][p][ci] H[hb][ci][co], and the partner -f with
// conj(H).  One warp per stored bin; the lane mapping (groups of lanes over
// input channels, 4 output channels per lane, one 16-byte weight load) is
// described in the kernel.  Every weight load of a step is issued before
// the step's arithmetic.  H is stored scaled by `hscale` (a power of two, see
// the spectrum header); the sums are scaled back before they are written.
// Weight loads per lane per step at KDIV = 1 (the kernel takes ci_step /
// KDIV): 16 for fp16-complex weights, 8 for fp32-complex.
template <typename S>
constexpr int ci_step() { return sizeof(S) == 4 ? 16 : 8; }

// Packed fp32 pairs (sm_100 fma.rn.f32x2: two fp32 FMAs per instruction).
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 up2(unsigned long long v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b,
                                                   unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ void cmac(float2& acc, float2 z, float2 h) {
  acc.x = fmaf(z.x, h.x, fmaf(-z.y, h.y, acc.x));
  acc.y = fmaf(z.x, h.y, fmaf(z.y, h.x, acc.y));
}
__device__ __forceinline__ void cmac_conj(float2& acc, float2 z, float2 h) {   // z * conj(h)
  acc.x = fmaf(z.x, h.x, fmaf(z.y, h.y, acc.x));
  acc.y = fmaf(z.y, h.x, fmaf(-z.x, h.y, acc.y));
}

// Spectrum element: complex fp32 (float2) for fp32 weights, complex fp16
// (__half2, scaled by the header value) for fp16 / bf16 weights.
__device__ __forceinline__ float2 spec_f2(float2 v) { return v; }
__device__ __forceinline__ float2 spec_f2(__half2 v) { return __half22float2(v); }
__device__ __forceinline__ void spec_zero(float2& v) { v = make_float2(0.f, 0.f); }
__device__ __forceinline__ void spec_zero(__half2& v) { v = __floats2half2_rn(0.f, 0.f); }
__device__ __forceinline__ void spec_put(float2* o, float a, float b) { *o = make_float2(a, b); }
__device__ __forceinline__ void spec_put(__half2* o, float a, float b) { *o = __floats2half2_rn(a, b); }

// 8-byte global -> shared copy; bytes past src_bytes are zero-filled.
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem, int src_bytes) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(sa), "l"(gmem),
               "r"(src_bytes) : "memory");
}

// KDIV: the step holds ci_step / KDIV weight loads per lane.  KDIV = 1 runs
// two CTAs per SM at 128 registers; KDIV = 2 and 4 run three at <= 85, which
// keeps more bins in flight per SM: KDIV = 4 for Cout <= 16 (NG >= 8 lane
// groups cover a 64-channel block in a few short steps; a bin is ~2 KB of
// weights and the kernel latency-bound), KDIV = 2 for wider fp16 spectra.
template <typename S, int KDIV>
__global__ void __launch_bounds__(kThreads, KDIV == 1 ? 2 : 3)
contract_kernel(const float2* __restrict__ Z, const S* __restrict__ Hs,
                const float* __restrict__ hdr, float2* __restrict__ U, int P, int Cin, int Cout,
                int Fd, int Fh, int Fw, int64_t hbins) {
  const int lane = threadIdx.x & 31;
  // Bin indices fit 32 bits (extents <= 256, so hbins < 2^24): 32-bit
  // division here, not the 64-bit routine (~10% of this kernel's instructions).
  const int hbi = static_cast<int>((blockIdx.x * static_cast<unsigned>(kThreads) + threadIdx.x) >> 5);
  if (hbi >= hbins) return;
  const int64_t hb = hbi;
  const float inv = 1.0f / __ldg(hdr);
  const int Fw2 = Fw / 2 + 1;
  const int q2 = hbi / Fw2;
  const int fw = hbi - q2 * Fw2;
  const int fd = q2 / Fh;
  const int fh = q2 - fd * Fh;
  const int64_t f = (static_cast<int64_t>(fd) * Fh + fh) * Fw + fw;
  const bool neg = fw > 0 && 2 * fw != Fw;
  const int64_t fn = (static_cast<int64_t>((Fd - fd) % Fd) * Fh + (Fh - fh) % Fh) * Fw + (Fw - fw);
  const S* h = Hs + hb * Cin * Cout;
  // The warp splits into NG groups of LPG lanes (LPG = 16 for Cout >= 64;
  // fewer for narrow outputs, e.g. a rank's slice of a channel-sharded conv,
  // so that no lane idles): group g takes input channels ci = g (mod NG),
  // lane q of a group owns output channels 4q .. 4q + 3 of each 4 * LPG
  // channel block (one 16-byte load of fp16 complex, two of fp32 complex).
  // The groups' sums are added at the end.
  // The bin's input spectrum (f and -f) is staged per 64-channel block in
  // the warp's shared memory, so the registers hold kCi weight loads in flight.
  constexpr int kCi = ci_step<S>() / KDIV;
  __shared__ float2 zs_all[kThreads / 32][2][64];
  float2 (*zs)[64] = zs_all[threadIdx.x >> 5];
  const int LPG = Cout > 32 ? 16 : (Cout > 16 ? 8 : (Cout > 8 ? 4 : (Cout > 4 ? 2 : 1)));
  const int NG = 32 / LPG;
  const int grp = lane / LPG, q = lane % LPG;
  constexpr int kPer = 16 / static_cast<int>(sizeof(S));   // values per 16-byte load
  const bool vec = (Cout % 4) == 0;
  const bool dense = Cout % (4 * LPG) == 0;   // every lane's 4 channels exist
  for (int p = 0; p < P; ++p) {
    const float2* zf = Z + (f * P + p) * Cin;
    const float2* zn = Z + (fn * P + p) * Cin;
    for (int co0 = 0; co0 < Cout; co0 += 4 * LPG) {
      const int c0 = co0 + 4 * q;
      float2 a[4], bsum[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) a[j] = bsum[j] = make_float2(0.f, 0.f);
      for (int cb = 0; cb < Cin; cb += 64) {
        const int cend = min(Cin, cb + 64);
        // The block's input spectrum is copied straight into shared memory
        // while the first step's weight loads are in flight (one memory
        // round trip per step, not two; no registers held by the copy).
        __syncwarp();   // the previous block's values are no longer read
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ci = cb + lane + 32 * u;
          const bool in = ci < Cin;
          cp_async8(&zs[0][lane + 32 * u], in ? zf + ci : zf, in ? 8 : 0);
          cp_async8(&zs[1][lane + 32 * u], (in && neg) ? zn + ci : zf, (in && neg) ? 8 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        for (int ci0 = cb; ci0 < cend; ci0 += NG * kCi) {
          S hv[kCi][4];
          if (dense && ci0 + NG * kCi <= cend) {
            // Whole step in range (warp-uniform): plain strided 16-byte loads.
            const S* hp = h + static_cast<int64_t>(ci0 + grp) * Cout + c0;
            const int st = NG * Cout;
#pragma unroll
            for (int k = 0; k < kCi; ++k) {
#pragma unroll
              for (int v = 0; v < 4; v += kPer) {
                const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(hp + k * st + v));
                const S* e = reinterpret_cast<const S*>(&w4);
#pragma unroll
                for (int u = 0; u < kPer; ++u) hv[k][v + u] = e[u];
              }
            }
            if (ci0 == cb) {
              asm volatile("cp.async.wait_group 0;" ::: "memory");
              __syncwarp();
            }
            // Packed pairs: a += (hx, hy) (zx, zx) + (hy, hx) (-zy, zy) is z h;
            // b += (hx, hy) (zzx, -zzx) + (hy, hx) (zzy, zzy) is zz conj(h).
            unsigned long long A[4], B[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              A[j] = pk2(a[j].x, a[j].y);
              B[j] = pk2(bsum[j].x, bsum[j].y);
            }
#pragma unroll
            for (int k = 0; k < kCi; ++k) {
              const int cl = ci0 - cb + NG * k + grp;
              const float2 z = zs[0][cl], zz = zs[1][cl];
              const unsigned long long zxx = pk2(z.x, z.x), zyn = pk2(-z.y, z.y);
              const unsigned long long wxn = pk2(zz.x, -zz.x), wyy = pk2(zz.y, zz.y);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 g = spec_f2(hv[k][j]);
                const unsigned long long hp = pk2(g.x, g.y), hs = pk2(g.y, g.x);
                A[j] = fma2(hs, zyn, fma2(hp, zxx, A[j]));
                B[j] = fma2(hs, wyy, fma2(hp, wxn, B[j]));
              }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              a[j] = up2(A[j]);
              bsum[j] = up2(B[j]);
            }
            continue;
          }
#pragma unroll
          for (int k = 0; k < kCi; ++k) {
            const int ci = ci0 + NG * k + grp;
            const bool in = ci < cend;
            const S* hr = h + static_cast<int64_t>(in ? ci : 0) * Cout + c0;
            if (!in) {
#pragma unroll
              for (int j = 0; j < 4; ++j) spec_zero(hv[k][j]);
            } else if (vec && c0 + 3 < Cout) {
#pragma unroll
              for (int v = 0; v < 4; v += kPer) {
                const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(hr + v));
                const S* e = reinterpret_cast<const S*>(&w4);
#pragma unroll
                for (int u = 0; u < kPer; ++u) hv[k][v + u] = e[u];
              }
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if (c0 + j < Cout) hv[k][j] = __ldg(hr + j);
                else spec_zero(hv[k][j]);
              }
            }
          }
          if (ci0 == cb) {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            __syncwarp();
          }
#pragma unroll
          for (int k = 0; k < kCi; ++k) {
            if (ci0 + NG * k >= cend) break;   // warp-uniform: no group has channels left
            const int cl = ci0 - cb + NG * k + grp;         // weights are zero past cend
            const float2 z = zs[0][cl & 63], zz = zs[1][cl & 63];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 g = spec_f2(hv[k][j]);
              cmac(a[j], z, g);
              cmac_conj(bsum[j], zz, g);
            }
          }
        }
      }
      for (int o = LPG; o < 32; o <<= 1) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          a[j].x += __shfl_xor_sync(0xffffffffu, a[j].x, o);
          a[j].y += __shfl_xor_sync(0xffffffffu, a[j].y, o);
          bsum[j].x += __shfl_xor_sync(0xffffffffu, bsum[j].x, o);
          bsum[j].y += __shfl_xor_sync(0xffffffffu, bsum[j].y, o);
        }
      }
      if (grp == 0) {
        float2* uf = U + (f * P + p) * Cout;
        float2* un = U + (fn * P + p) * Cout;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (c0 + j < Cout) {
            uf[c0 + j] = make_float2(a[j].x * inv, a[j].y * inv);
            if (neg) un[c0 + j] = make_float2(bsum[j].x * inv, bsum[j].y * inv);
          }
        }
      }
    }
  }
}

// --------------------------------------------------------------- K4 -----
// U[bin][p][co] -> G2[p][co][od < Do][Fh*Fw] (inverse depth FFT).
__global__ void __launch_bounds__(kThreads, 3)
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
  int* posd = reinterpret_cast<int*>(buf + nseq * SS);
  build_pos(posd, pl.d);
  __syncthreads();
  const float inv_c = 1.0f / static_cast<float>(C);
  gather_smem(
      buf, nseq * Fd,
      [&](int idx) {
        const int r = qdiv(idx, C, inv_c);
        const int c = idx - r * C;
        const int q = r % kCols, fd = r / kCols;
        const int col = col0 + q;
        return col < cols ? U[((static_cast<int64_t>(fd) * cols + col) * P + p) * C + c]
                          : make_float2(0.f, 0.f);
      },
      [&](int idx) {
        const int r = qdiv(idx, C, inv_c);
        const int c = idx - r * C;
        return (c * kCols + r % kCols) * SS + posd[r / kCols];
      });
  __syncthreads();
  bfft<true>(buf, pl.d, nseq, SS, 1, twd);
  const int dk = Do * kCols;
  const float inv_dk = 1.0f / static_cast<float>(dk);
  for (int idx = threadIdx.x; idx < C * Do * kCols; idx += blockDim.x) {
    const int c = qdiv(idx, dk, inv_dk);
    const int r = idx - c * dk;
    const int o = r / kCols, q = r - o * kCols;
    const int col = col0 + q;
    if (col >= cols) continue;
    G2[((static_cast<int64_t>(p) * C + c) * Do + o) * cols + col] = buf[(c * kCols + q) * SS + o];
  }
}

// --------------------------------------------------------------- K5 -----
// G2[p][co][od][Fh*Fw] -> y[n][co][od][Ho][Wo] (inverse plane FFT, crop,
// scale, bias).
template <typename T, int NP>
__global__ void __launch_bounds__(kThreads, 3)
plane_inv_kernel(const float2* __restrict__ G2, T* __restrict__ y, const void* __restrict__ bias,
                 int bias_dt, int64_t N, int C, int Do, int Ho, int Wo, float scale,
                 const Plan3 pl) {
  extern __shared__ float2 sm[];
  const int Fh = NP ? NP : pl.h.n, Fw = NP ? NP : pl.w.n, RS = plane_row_stride(Fw);
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
  int* posh = reinterpret_cast<int*>(buf + Fh * RS);
  int* posw = posh + Fh;
  build_pos(posh, pl.h);
  build_pos(posw, pl.w);
  __syncthreads();
  const float inv_fw = 1.0f / static_cast<float>(Fw);
  gather_smem<16>(
      buf, Fh * Fw, [&](int idx) { return g[idx]; },
      [&](int idx) {
        const int fh = div_np<NP>(idx, Fw, inv_fw);
        return posh[fh] * RS + posw[idx - fh * Fw];
      });
  __syncthreads();
  plane_fft<true, NP>(buf, pl.h, Fw, 1, RS, twh);
  plane_fft<true, NP>(buf, pl.w, Ho < Fh ? Ho : Fh, RS, 1, tww);   // only the output rows
  const float bv = bias ? load_param(bias, bias_dt, c) : 0.f;
  const int64_t n0 = 2 * p, n1 = n0 + 1;
  const int64_t vol = static_cast<int64_t>(Do) * Ho * Wo;
  T* y0 = y + (n0 * C + c) * vol + static_cast<int64_t>(od) * Ho * Wo;
  T* y1 = y + (min64(n1, N - 1) * C + c) * vol + static_cast<int64_t>(od) * Ho * Wo;
  const float inv_wo = 1.0f / static_cast<float>(Wo);
  for (int idx = threadIdx.x; idx < Ho * Wo; idx += blockDim.x) {
    const int h = qdiv(idx, Wo, inv_wo), w = idx - h * Wo;
    const float2 v = buf[h * RS + w];
    y0[idx] = from_f32<T>(fmaf(v.x, scale, bv));
    if (n1 < N) y1[idx] = from_f32<T>(fmaf(v.y, scale, bv));
  }
}

// ------------------------------------------------------------ K_sep -----
// Weight spectrum: Zw[bin][0][ci] packs output channels (co0, co0 + 1) as
// real/imag; split them by Hermitian symmetry and store the conjugates for
// the stored half (fw <= Fw/2) as Hs[hb][ci][co].
template <typename S>
__global__ void separate_kernel(const float2* __restrict__ Zw, S* __restrict__ Hs,
                                const float* __restrict__ hdr, int Cin, int Cout, int co0, int Fd,
                                int Fh, int Fw, int64_t hbins) {
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
  const float sc = __ldg(hdr);
  S* out = Hs + (hb * Cin + ci) * Cout;
  spec_put(out + co0, A.x * sc, -A.y * sc);
  if (co0 + 1 < Cout) spec_put(out + co0 + 1, Bv.x * sc, -Bv.y * sc);
}

// Spectrum scale: the largest power of two s with s * max|w| * taps <= 2^15,
// so every stored |H| (at most sum |w| <= max|w| * taps) stays inside fp16
// and the typical values keep full fp16 precision.  One CTA; the weight is
// small (read once per weight).
template <typename T>
__global__ void __launch_bounds__(256)
spectrum_scale_kernel(const T* __restrict__ w, int64_t n, int64_t taps, int unit,
                      float* __restrict__ hdr) {
  __shared__ float red[32];
  float m = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += 256) m = fmaxf(m, fabsf(to_f32(w[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = 0.f;
    for (int k = 0; k < 8; ++k) mm = fmaxf(mm, red[k]);
    const float bound = mm * static_cast<float>(taps);
    int e = 0;
    if (bound > 0.f && isfinite(bound)) {
      frexpf(32768.0f / bound, &e);   // 32768 / bound = f * 2^e, f in [0.5, 1)
      e -= 1;                          // 2^e <= 32768 / bound
    }
    e = e > 60 ? 60 : (e < -60 ? -60 : e);
    hdr[0] = unit ? 1.0f : ldexpf(1.0f, e);
  }
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

// twiddles + transform buffer + digit-reversed position tables (int)
size_t plane_smem(const Plan3& p) {
  return static_cast<size_t>(p.h.n + p.w.n + p.h.n * plane_row_stride(p.w.n)) * sizeof(float2) +
         static_cast<size_t>(p.h.n + p.w.n) * sizeof(int);
}
size_t depth_smem(const Plan3& p, int C) {
  return static_cast<size_t>(p.d.n + C * kCols * (p.d.n + 1)) * sizeof(float2) +
         static_cast<size_t>(p.d.n) * sizeof(int);
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
  const bool p80 = plane80(pl.h, pl.w);
  auto plane_fwd = p80 ? plane_fwd_kernel<T, 80> : plane_fwd_kernel<T, 0>;
  if ((rc = set_smem(plane_fwd, ps)) != B200_OK) return rc;
  if ((rc = set_smem(depth_fwd_kernel, ds)) != B200_OK) return rc;
  const int64_t g1 = npairs * C * Dz;
  if (g1 > 0x7fffffffLL) return fail_unsupported("grid too large");
  plane_fwd<<<(unsigned)g1, kThreads, ps, s>>>(x, G, n_items, item0, C, Dz, H, W, oh, ow, pl);
  B200_LAUNCH_CHECK("plane_fwd_kernel");
  const int cols = pl.h.n * pl.w.n;
  if (pl.d.n == 30) {
    const size_t rs = depth_reg_smem<30>();
    if ((rc = set_smem(depth_fwd_reg_kernel<30>, rs)) != B200_OK) return rc;
    const int64_t g2 = npairs * ((C + kDCh - 1) / kDCh) * ((cols + kDCols - 1) / kDCols);
    if (g2 > 0x7fffffffLL) return fail_unsupported("grid too large");
    depth_fwd_reg_kernel<30><<<(unsigned)g2, kDCols * kDCh, rs, s>>>(G, Z, (int)npairs, C, Dz,
                                                                      od, cols);
    B200_LAUNCH_CHECK("depth_fwd_reg_kernel");
    return B200_OK;
  }
  const int64_t g2 = npairs * ((cols + kCols - 1) / kCols);
  depth_fwd_kernel<<<(unsigned)g2, kThreads, ds, s>>>(G, Z, (int)npairs, C, Dz, od, pl);
  B200_LAUNCH_CHECK("depth_fwd_kernel");
  return B200_OK;
}

// Spectrum buffer: a 256-byte header (float scale at offset 0) followed by
// Hs[hbin][Cin][Cout]: complex fp32 for fp32 weights (scale 1), complex fp16
// scaled by the header value for fp16 / bf16 weights.
constexpr size_t kSpecHeader = 256;
template <typename T>
using SpecT = typename std::conditional<std::is_same<T, float>::value, float2, __half2>::type;

template <typename T>
int prepare_typed(const void* wv, void* spec, int64_t Cout, int64_t Cin, int64_t KD, int64_t KH,
                  int64_t KW, const Plan3& pl, void* ws, size_t ws_bytes, cudaStream_t s) {
  const Sizes sz = sizes(1, Cin, Cout, pl.d.n, pl.h.n, pl.w.n);
  const size_t need = align256(sz.g_bytes) + align256(sz.z_bytes);
  if (!ws || ws_bytes < need) return fail_arg("fftconv3d prepare workspace too small");
  float2* G = static_cast<float2*>(ws);
  float2* Zw = reinterpret_cast<float2*>(static_cast<char*>(ws) + align256(sz.g_bytes));
  const T* w = static_cast<const T*>(wv);
  float* hdr = static_cast<float*>(spec);
  SpecT<T>* Hs = reinterpret_cast<SpecT<T>*>(static_cast<char*>(spec) + kSpecHeader);
  spectrum_scale_kernel<T><<<1, 256, 0, s>>>(w, Cout * Cin * KD * KH * KW, KD * KH * KW,
                                             std::is_same<T, float>::value ? 1 : 0, hdr);
  B200_LAUNCH_CHECK("spectrum_scale_kernel");
  for (int64_t co0 = 0; co0 < Cout; co0 += 2) {
    int rc = forward_volume<T>(w, G, Zw, Cout, co0, 1, (int)Cin, (int)KD, (int)KH, (int)KW, 0, 0,
                               0, pl, s);
    if (rc != B200_OK) return rc;
    const int64_t n = sz.hbins * Cin;
    separate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(Zw, Hs, hdr, (int)Cin, (int)Cout,
                                                                (int)co0, pl.d.n, pl.h.n,
                                                                pl.w.n, sz.hbins);
    B200_LAUNCH_CHECK("separate_kernel");
  }
  return B200_OK;
}

template <typename T>
int fwd_typed(const void* xv, const void* spec, const void* bias, int bias_dt, void* yv,
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
  const float* hdr = static_cast<const float*>(spec);
  const SpecT<T>* Hs =
      reinterpret_cast<const SpecT<T>*>(static_cast<const char*>(spec) + kSpecHeader);
  const unsigned cgrid = (unsigned)((warps * 32 + kThreads - 1) / kThreads);
  // Weight loads in flight per lane against CTAs per SM (measured at cfg 4a,
  // Cout = 64, fp16 spectrum, whole op: kCi 16 at two CTAs 541 us, kCi 8 at
  // three 530 us, kCi 4 at three 554 us).
  const int kd = Cout <= 16 ? 4 : (sizeof(SpecT<T>) == 4 ? 2 : 1);
  if (kd == 4)
    contract_kernel<SpecT<T>, 4><<<cgrid, kThreads, 0, s>>>(
        Z, Hs, hdr, U, (int)sz.P, (int)Cin, (int)Cout, pl.d.n, pl.h.n, pl.w.n, sz.hbins);
  else if (kd == 2)
    contract_kernel<SpecT<T>, 2><<<cgrid, kThreads, 0, s>>>(
        Z, Hs, hdr, U, (int)sz.P, (int)Cin, (int)Cout, pl.d.n, pl.h.n, pl.w.n, sz.hbins);
  else
    contract_kernel<SpecT<T>, 1><<<cgrid, kThreads, 0, s>>>(
        Z, Hs, hdr, U, (int)sz.P, (int)Cin, (int)Cout, pl.d.n, pl.h.n, pl.w.n, sz.hbins);
  B200_LAUNCH_CHECK("contract_kernel");
  const size_t ds = depth_smem(pl, (int)Cout), ps = plane_smem(pl);
  if ((rc = set_smem(depth_inv_kernel, ds)) != B200_OK) return rc;
  auto plane_inv = plane80(pl.h, pl.w) ? plane_inv_kernel<T, 80> : plane_inv_kernel<T, 0>;
  if ((rc = set_smem(plane_inv, ps)) != B200_OK) return rc;
  const int cols = pl.h.n * pl.w.n;
  float2* G2 = G;   // G is dead once Z is built
  if (pl.d.n == 30) {
    const size_t rs = depth_reg_smem<30>();
    if ((rc = set_smem(depth_inv_reg_kernel<30>, rs)) != B200_OK) return rc;
    const int64_t g4 = sz.P * ((Cout + kDCh - 1) / kDCh) * ((cols + kDCols - 1) / kDCols);
    if (g4 > 0x7fffffffLL) return fail_unsupported("grid too large");
    depth_inv_reg_kernel<30><<<(unsigned)g4, kDCols * kDCh, rs, s>>>(U, G2, (int)sz.P,
                                                                      (int)Cout, (int)Do, cols);
    B200_LAUNCH_CHECK("depth_inv_reg_kernel");
  } else {
    depth_inv_kernel<<<(unsigned)(sz.P * ((cols + kCols - 1) / kCols)), kThreads, ds, s>>>(
        U, G2, (int)sz.P, (int)Cout, (int)Do, pl);
    B200_LAUNCH_CHECK("depth_inv_kernel");
  }
  const float scale = 1.0f / static_cast<float>(static_cast<double>(pl.d.n) * pl.h.n * pl.w.n);
  const int64_t g5 = sz.P * Cout * Do;
  if (g5 > 0x7fffffffLL) return fail_unsupported("grid too large");
  plane_inv<<<(unsigned)g5, kThreads, ps, s>>>(G2, static_cast<T*>(yv), bias, bias_dt, N,
                                               (int)Cout, (int)Do, (int)Ho, (int)Wo, scale, pl);
  B200_LAUNCH_CHECK("plane_inv_kernel");
  return B200_OK;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

size_t b200_fftconv3d_spectrum_bytes(int64_t Cout, int64_t Cin, int64_t fd, int64_t fh,
                                     int64_t fw, int w_dtype) {
  const size_t elem = w_dtype == B200_DTYPE_F32 ? sizeof(float2) : sizeof(__half2);
  return kSpecHeader + static_cast<size_t>(Cout * Cin * fd * fh * (fw / 2 + 1)) * elem;
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
  if (!aligned16(spectrum)) return fail_arg("spectrum must be 16-byte aligned");
  if (w_dtype == B200_DTYPE_F32)
    return prepare_typed<float>(w, spectrum, Cout, Cin, KD, KH, KW, pl, workspace,
                                workspace_bytes, s);
  if (w_dtype == B200_DTYPE_F16)
    return prepare_typed<__half>(w, spectrum, Cout, Cin, KD, KH, KW, pl, workspace,
                                 workspace_bytes, s);
  return prepare_typed<__nv_bfloat16>(w, spectrum, Cout, Cin, KD, KH, KW, pl, workspace,
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
  if (!aligned16(spectrum)) return fail_arg("spectrum must be 16-byte aligned");
  const void* Hs = spectrum;
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
