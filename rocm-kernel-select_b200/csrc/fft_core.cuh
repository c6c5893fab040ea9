// In-place mixed-radix FFT in shared memory (complex fp32), used by the FFT
// convolution kernels.
//
// Forward transform: decimation in frequency (Gentleman-Sande).  Pass p of
// radix R and span S takes the R elements {base + m * S/R}, applies an R-point
// DFT in registers and multiplies output m by W_S^(k m) (W_S = e^{-2 pi i/S},
// k = the butterfly's offset inside its span), writing back to the SAME
// positions.  After all passes the spectrum sits in mixed-radix digit-reversed
// order.  Inverse transform: the exact reverse (decimation in time): passes
// in reverse order, each multiplying by the conjugate twiddles and applying
// the inverse R-point DFT.  A spectral product computed position by position
// between two spectra produced by the same forward plan is therefore a
// product of matching frequencies, and the inverse returns natural order:
// no reordering pass is ever needed (the kernel spectrum is produced by the
// same forward plan).  The inverse is unnormalised (result * N).
//
// Butterflies touch only their own positions, so a pass needs no barrier
// between its reads and writes -- only between passes.  Shared-memory
// indices are padded by one element every 16 (pidx) so the small-span
// passes (stride 1) do not serialise on banks.  Twiddles W_N^t come from a
// two-level table built per CTA in double precision: W_N^t =
// hi[t >> 8] * lo[t & 255].
#pragma once

#include "common.cuh"

namespace b200 {
namespace fft {

constexpr int kMaxPasses = 12;
constexpr int kLoBits = 8;
constexpr int kLo = 1 << kLoBits;

struct Plan {
  int n;
  int passes;
  int radix[kMaxPasses];
};

__device__ __forceinline__ int pidx(int i) { return i + (i >> 4); }
inline int padded_len(int n) { return n + (n >> 4) + 16; }

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ float2 cmulc(float2 a, float2 b) {  // a * conj(b)
  return make_float2(fmaf(a.x, b.x, a.y * b.y), fmaf(a.y, b.x, -a.x * b.y));
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }

// e^{-2 pi i e / R} for the radices used by the small DFTs (e folded mod R).
template <int R>
__device__ __forceinline__ float2 root(int e);
template <>
__device__ __forceinline__ float2 root<16>(int e) {
  switch (e & 15) {
    case 0: return make_float2(1.f, 0.f);
    case 1: return make_float2(0.923879533f, -0.382683432f);
    case 2: return make_float2(0.707106781f, -0.707106781f);
    case 3: return make_float2(0.382683432f, -0.923879533f);
    case 4: return make_float2(0.f, -1.f);
    case 5: return make_float2(-0.382683432f, -0.923879533f);
    case 6: return make_float2(-0.707106781f, -0.707106781f);
    case 7: return make_float2(-0.923879533f, -0.382683432f);
    case 8: return make_float2(-1.f, 0.f);
    case 9: return make_float2(-0.923879533f, 0.382683432f);
    case 10: return make_float2(-0.707106781f, 0.707106781f);
    case 11: return make_float2(-0.382683432f, 0.923879533f);
    case 12: return make_float2(0.f, 1.f);
    case 13: return make_float2(0.382683432f, 0.923879533f);
    case 14: return make_float2(0.707106781f, 0.707106781f);
    default: return make_float2(0.923879533f, 0.382683432f);
  }
}
template <>
__device__ __forceinline__ float2 root<32>(int e) {
  e &= 31;
  if ((e & 1) == 0) return root<16>(e >> 1);
  switch (e) {
    case 1: return make_float2(0.980785280f, -0.195090322f);
    case 3: return make_float2(0.831469612f, -0.555570233f);
    case 5: return make_float2(0.555570233f, -0.831469612f);
    case 7: return make_float2(0.195090322f, -0.980785280f);
    case 9: return make_float2(-0.195090322f, -0.980785280f);
    case 11: return make_float2(-0.555570233f, -0.831469612f);
    case 13: return make_float2(-0.831469612f, -0.555570233f);
    case 15: return make_float2(-0.980785280f, -0.195090322f);
    case 17: return make_float2(-0.980785280f, 0.195090322f);
    case 19: return make_float2(-0.831469612f, 0.555570233f);
    case 21: return make_float2(-0.555570233f, 0.831469612f);
    case 23: return make_float2(-0.195090322f, 0.980785280f);
    case 25: return make_float2(0.195090322f, 0.980785280f);
    case 27: return make_float2(0.555570233f, 0.831469612f);
    case 29: return make_float2(0.831469612f, 0.555570233f);
    default: return make_float2(0.980785280f, 0.195090322f);
  }
}
template <>
__device__ __forceinline__ float2 root<30>(int e) {
  switch (((e % 30) + 30) % 30) {
    case 0: return make_float2(1.000000000f, 0.f);
    case 1: return make_float2(0.978147601f, -0.207911691f);
    case 2: return make_float2(0.913545458f, -0.406736643f);
    case 3: return make_float2(0.809016994f, -0.587785252f);
    case 4: return make_float2(0.669130606f, -0.743144825f);
    case 5: return make_float2(0.500000000f, -0.866025404f);
    case 6: return make_float2(0.309016994f, -0.951056516f);
    case 7: return make_float2(0.104528463f, -0.994521895f);
    case 8: return make_float2(-0.104528463f, -0.994521895f);
    case 9: return make_float2(-0.309016994f, -0.951056516f);
    case 10: return make_float2(-0.500000000f, -0.866025404f);
    case 11: return make_float2(-0.669130606f, -0.743144825f);
    case 12: return make_float2(-0.809016994f, -0.587785252f);
    case 13: return make_float2(-0.913545458f, -0.406736643f);
    case 14: return make_float2(-0.978147601f, -0.207911691f);
    case 15: return make_float2(-1.000000000f, 0.f);
    case 16: return make_float2(-0.978147601f, 0.207911691f);
    case 17: return make_float2(-0.913545458f, 0.406736643f);
    case 18: return make_float2(-0.809016994f, 0.587785252f);
    case 19: return make_float2(-0.669130606f, 0.743144825f);
    case 20: return make_float2(-0.500000000f, 0.866025404f);
    case 21: return make_float2(-0.309016994f, 0.951056516f);
    case 22: return make_float2(-0.104528463f, 0.994521895f);
    case 23: return make_float2(0.104528463f, 0.994521895f);
    case 24: return make_float2(0.309016994f, 0.951056516f);
    case 25: return make_float2(0.500000000f, 0.866025404f);
    case 26: return make_float2(0.669130606f, 0.743144825f);
    case 27: return make_float2(0.809016994f, 0.587785252f);
    case 28: return make_float2(0.913545458f, 0.406736643f);
    default: return make_float2(0.978147601f, 0.207911691f);
  }
}
template <>
__device__ __forceinline__ float2 root<15>(int e) { return root<30>(2 * e); }
template <>
__device__ __forceinline__ float2 root<6>(int e) { return root<30>(5 * e); }
template <>
__device__ __forceinline__ float2 root<8>(int e) { return root<16>(2 * e); }
template <>
__device__ __forceinline__ float2 root<4>(int e) { return root<16>(4 * e); }
template <>
__device__ __forceinline__ float2 root<2>(int e) { return root<16>(8 * e); }
template <>
__device__ __forceinline__ float2 root<9>(int e) {
  switch (e % 9) {
    case 0: return make_float2(1.f, 0.f);
    case 1: return make_float2(0.766044443f, -0.642787610f);
    case 2: return make_float2(0.173648178f, -0.984807753f);
    case 3: return make_float2(-0.5f, -0.866025404f);
    case 4: return make_float2(-0.939692621f, -0.342020143f);
    case 5: return make_float2(-0.939692621f, 0.342020143f);
    case 6: return make_float2(-0.5f, 0.866025404f);
    case 7: return make_float2(0.173648178f, 0.984807753f);
    default: return make_float2(0.766044443f, 0.642787610f);
  }
}
template <>
__device__ __forceinline__ float2 root<3>(int e) { return root<9>(3 * e); }
template <>
__device__ __forceinline__ float2 root<5>(int e) {
  switch (e % 5) {
    case 0: return make_float2(1.f, 0.f);
    case 1: return make_float2(0.309016994f, -0.951056516f);
    case 2: return make_float2(-0.809016994f, -0.587785252f);
    case 3: return make_float2(-0.809016994f, 0.587785252f);
    default: return make_float2(0.309016994f, 0.951056516f);
  }
}
template <int R, bool INV>
__device__ __forceinline__ float2 rootd(int e) {
  const float2 w = root<R>(e);
  return INV ? make_float2(w.x, -w.y) : w;
}

// v * W_R^{+-e} for an exponent known after unrolling: multiples of a quarter
// turn are swaps and negations, the rest a complex multiply.
template <int R, bool INV>
__device__ __forceinline__ float2 twiddle_const(float2 v, int e) {
  e %= R;
  if (e == 0) return v;
  if (2 * e == R) return make_float2(-v.x, -v.y);
  if (4 * e == R)  // W_R^{R/4} = -i forward, +i inverse
    return INV ? make_float2(-v.y, v.x) : make_float2(v.y, -v.x);
  if (4 * e == 3 * R) return INV ? make_float2(v.y, -v.x) : make_float2(-v.y, v.x);
  return cmul(v, rootd<R, INV>(e));
}

// R-point DFT in registers: out[k] = sum_n v[n] W_R^{+-nk}.
template <int R, bool INV>
struct Dft {
  static __device__ __forceinline__ void run(float2 (&v)[R]) {  // direct (R = 3, 5)
    float2 out[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      float2 acc = v[0];
#pragma unroll
      for (int n = 1; n < R; ++n) {
        const float2 w = rootd<R, INV>(n * k);
        acc.x = fmaf(v[n].x, w.x, fmaf(-v[n].y, w.y, acc.x));
        acc.y = fmaf(v[n].x, w.y, fmaf(v[n].y, w.x, acc.y));
      }
      out[k] = acc;
    }
#pragma unroll
    for (int k = 0; k < R; ++k) v[k] = out[k];
  }
};

template <bool INV>
struct Dft<2, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[2]) {
    const float2 a = cadd(v[0], v[1]), b = csub(v[0], v[1]);
    v[0] = a;
    v[1] = b;
  }
};

template <bool INV>
struct Dft<4, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[4]) {
    const float2 a = cadd(v[0], v[2]), b = csub(v[0], v[2]);
    const float2 c = cadd(v[1], v[3]), d = csub(v[1], v[3]);
    // d * (-i) forward, d * (+i) inverse
    const float2 dj = INV ? make_float2(-d.y, d.x) : make_float2(d.y, -d.x);
    v[0] = cadd(a, c);
    v[2] = csub(a, c);
    v[1] = cadd(b, dj);
    v[3] = csub(b, dj);
  }
};

// R = R1 * R2 by one Cooley-Tukey split: n = R2 n1 + n2, k = k1 + R1 k2.
template <int R1, int R2, bool INV>
struct DftSplit {
  static __device__ __forceinline__ void run(float2 (&v)[R1 * R2]) {
    constexpr int R = R1 * R2;
    float2 y[R];
#pragma unroll
    for (int n2 = 0; n2 < R2; ++n2) {
      float2 t[R1];
#pragma unroll
      for (int n1 = 0; n1 < R1; ++n1) t[n1] = v[R2 * n1 + n2];
      Dft<R1, INV>::run(t);
#pragma unroll
      for (int k1 = 0; k1 < R1; ++k1)
        y[n2 * R1 + k1] = twiddle_const<R, INV>(t[k1], n2 * k1);
    }
#pragma unroll
    for (int k1 = 0; k1 < R1; ++k1) {
      float2 t[R2];
#pragma unroll
      for (int n2 = 0; n2 < R2; ++n2) t[n2] = y[n2 * R1 + k1];
      Dft<R2, INV>::run(t);
#pragma unroll
      for (int k2 = 0; k2 < R2; ++k2) v[k1 + R1 * k2] = t[k2];
    }
  }
};
template <bool INV>
struct Dft<8, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[8]) { DftSplit<2, 4, INV>::run(v); }
};
template <bool INV>
struct Dft<16, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[16]) { DftSplit<4, 4, INV>::run(v); }
};
template <bool INV>
struct Dft<32, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[32]) { DftSplit<2, 16, INV>::run(v); }
};
template <bool INV>
struct Dft<6, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[6]) { DftSplit<2, 3, INV>::run(v); }
};
template <bool INV>
struct Dft<15, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[15]) { DftSplit<3, 5, INV>::run(v); }
};
template <bool INV>
struct Dft<30, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[30]) { DftSplit<2, 15, INV>::run(v); }
};
template <bool INV>
struct Dft<9, INV> {
  static __device__ __forceinline__ void run(float2 (&v)[9]) { DftSplit<3, 3, INV>::run(v); }
};

// ---------------------------------------------------------------- tables ---
// lo[j] = W_N^j (j < 256), hi[h] = W_N^(256 h); built by the calling CTA.
__device__ __forceinline__ void build_twiddles(float2* lo, float2* hi, int n) {
  const int nhi = (n + kLo - 1) >> kLoBits;
  for (int j = threadIdx.x; j < kLo + nhi; j += blockDim.x) {
    const int t = j < kLo ? j : (j - kLo) << kLoBits;
    double s, c;
    sincospi(-2.0 * static_cast<double>(t % n) / static_cast<double>(n), &s, &c);
    const float2 w = make_float2(static_cast<float>(c), static_cast<float>(s));
    if (j < kLo)
      lo[j] = w;
    else
      hi[j - kLo] = w;
  }
}
__device__ __forceinline__ float2 twiddle(const float2* lo, const float2* hi, int t) {
  return cmul(hi[t >> kLoBits], lo[t & (kLo - 1)]);
}

// One DIF (forward) or DIT (inverse) pass of radix R over span S.
template <int R, bool INV>
__device__ __forceinline__ void pass(float2* buf, int n, int span, const float2* lo,
                                     const float2* hi) {
  const int stride = span / R;
  const int nbf = n / R;
  const int tscale = n / span;
  for (int b = threadIdx.x; b < nbf; b += blockDim.x) {
    const int g = b / stride, k = b - g * stride;
    const int base = g * span + k;
    float2 v[R];
#pragma unroll
    for (int m = 0; m < R; ++m) v[m] = buf[pidx(base + m * stride)];
    if (!INV) {
      Dft<R, false>::run(v);
      if (k != 0) {
#pragma unroll
        for (int m = 1; m < R; ++m) v[m] = cmul(v[m], twiddle(lo, hi, k * m * tscale));
      }
    } else {
      if (k != 0) {
#pragma unroll
        for (int m = 1; m < R; ++m) v[m] = cmulc(v[m], twiddle(lo, hi, k * m * tscale));
      }
      Dft<R, true>::run(v);
    }
#pragma unroll
    for (int m = 0; m < R; ++m) buf[pidx(base + m * stride)] = v[m];
  }
}

template <bool INV>
__device__ __forceinline__ void run_pass(int radix, float2* buf, int n, int span,
                                         const float2* lo, const float2* hi) {
  switch (radix) {
    case 16: pass<16, INV>(buf, n, span, lo, hi); break;
    case 8: pass<8, INV>(buf, n, span, lo, hi); break;
    case 4: pass<4, INV>(buf, n, span, lo, hi); break;
    case 2: pass<2, INV>(buf, n, span, lo, hi); break;
    case 9: pass<9, INV>(buf, n, span, lo, hi); break;
    case 3: pass<3, INV>(buf, n, span, lo, hi); break;
    default: pass<5, INV>(buf, n, span, lo, hi); break;
  }
}

// Full forward transform (natural order in, digit-reversed order out).
__device__ __forceinline__ void forward(float2* buf, const Plan& p, const float2* lo,
                                        const float2* hi) {
  int span = p.n;
  for (int i = 0; i < p.passes; ++i) {
    run_pass<false>(p.radix[i], buf, p.n, span, lo, hi);
    span /= p.radix[i];
    __syncthreads();
  }
}

// Full inverse transform (digit-reversed in, natural out, unnormalised).
__device__ __forceinline__ void inverse(float2* buf, const Plan& p, const float2* lo,
                                        const float2* hi) {
  int span = p.radix[p.passes - 1];
  for (int i = p.passes - 1; i >= 0; --i) {
    run_pass<true>(p.radix[i], buf, p.n, span, lo, hi);
    if (i > 0) span *= p.radix[i - 1];
    __syncthreads();
  }
}

// ------------------------------------------------ per-pass twiddle tables ---
// Pass p (span S_p, radix R_p) needs W_{S_p}^(k m) for k < S_p / R_p, m < R_p.
// The table holds only W_{S_p}^k (contiguous in k, so a warp's lookups hit
// distinct banks); the powers m are formed in registers by repeated complex
// multiplication (R - 2 products, error ~R ulps).
__device__ __forceinline__ int pass_tw_count(const Plan& p) {
  int total = 0, span = p.n;
  for (int i = 0; i < p.passes; ++i) {
    total += span / p.radix[i];
    span /= p.radix[i];
  }
  return total;
}

__device__ __forceinline__ void build_pass_twiddles(float2* tw, const Plan& p) {
  int off = 0, span = p.n;
  for (int i = 0; i < p.passes; ++i) {
    const int cnt = span / p.radix[i];
    for (int k = threadIdx.x; k < cnt; k += blockDim.x) {
      double s, c;
      sincospi(-2.0 * static_cast<double>(k) / static_cast<double>(span), &s, &c);
      tw[off + k] = make_float2(static_cast<float>(c), static_cast<float>(s));
    }
    off += cnt;
    span /= p.radix[i];
  }
}

// Multiplies v[m] (m >= 1) by w^m (forward) or conj(w)^m (inverse).
template <int R, bool INV>
__device__ __forceinline__ void apply_twiddle_powers(float2 (&v)[R], float2 w) {
  if (INV) w.y = -w.y;
  // Powers as a product tree, w^m = w^(m/2) * w^(m - m/2): the same R - 2
  // multiplications as a running product, but log2(R) deep instead of R - 2.
  float2 wp[R];
  wp[1] = w;
#pragma unroll
  for (int m = 2; m < R; ++m) wp[m] = cmul(wp[m / 2], wp[m - m / 2]);
#pragma unroll
  for (int m = 1; m < R; ++m) v[m] = cmul(v[m], wp[m]);
}

// Middle pass (shared memory in and out), per-pass table `tw`.
template <int R, bool INV>
__device__ __forceinline__ void pass_t(float2* buf, int n, int span, const float2* tw) {
  const int stride = span / R;
  const int nbf = n / R;
  for (int b = threadIdx.x; b < nbf; b += blockDim.x) {
    const int g = b / stride, k = b - g * stride;
    const int base = g * span + k;
    float2 v[R];
#pragma unroll
    for (int m = 0; m < R; ++m) v[m] = buf[pidx(base + m * stride)];
    if (!INV) {
      Dft<R, false>::run(v);
      if (k != 0) apply_twiddle_powers<R, false>(v, tw[k]);
    } else {
      if (k != 0) apply_twiddle_powers<R, true>(v, tw[k]);
      Dft<R, true>::run(v);
    }
#pragma unroll
    for (int m = 0; m < R; ++m) buf[pidx(base + m * stride)] = v[m];
  }
}

// MAXR: largest radix the caller's plans use (radix-16 code is only
// instantiated when MAXR >= 16).
template <bool INV, int MAXR = 16>
__device__ __forceinline__ void run_pass_t(int radix, float2* buf, int n, int span,
                                           const float2* tw) {
  if constexpr (MAXR >= 16) {
    if (radix == 16) {
      pass_t<16, INV>(buf, n, span, tw);
      return;
    }
  }
  switch (radix) {
    case 8: pass_t<8, INV>(buf, n, span, tw); break;
    case 4: pass_t<4, INV>(buf, n, span, tw); break;
    case 2: pass_t<2, INV>(buf, n, span, tw); break;
    case 9: pass_t<9, INV>(buf, n, span, tw); break;
    case 3: pass_t<3, INV>(buf, n, span, tw); break;
    default: pass_t<5, INV>(buf, n, span, tw); break;
  }
}

// Host: radix plan for n = 2^a 3^b 5^c (largest radices first); false if n
// has another prime factor or needs too many passes.
// max_radix 16 (default) or 8: a radix-8 plan has more passes but its
// butterflies need half the registers, for kernels that run more threads.
inline bool make_plan(int64_t n, Plan* p, int max_radix = 16) {
  if (n < 2 || n > (1 << 24)) return false;
  p->n = static_cast<int>(n);
  p->passes = 0;
  int64_t m = n;
  const int order[] = {16, 8, 4, 2, 9, 3, 5};
  for (int r : order) {
    if (r > max_radix) continue;
    while (m % r == 0) {
      if (r == 2 && m % 4 == 0) break;  // prefer 4 over 2 x 2
      if (p->passes == kMaxPasses) return false;
      p->radix[p->passes++] = r;
      m /= r;
    }
  }
  return m == 1;
}

}  // namespace fft
}  // namespace b200
