// Register-resident FFT of N = R1 * R2 * R3 points for one CTA of
// T = R2 * R3 threads, each thread holding R1 points in registers.
//
// Three passes, all butterflies in registers, two shared-memory exchanges
// per direction (the four-step factorisation applied twice):
//   n = M1 n1 + m1 (M1 = R2 R3), m1 = R3 n2 + m2; k = k1 + R1 (k2 + R2 k3)
//   pass 1  thread m1:      DFT-R1 over n1, times W_N^(m1 k1)
//   pass 2  combo (k1, m2): DFT-R2 over n2, times W_M1^(m2 k2)
//   pass 3  combo (k1, k2): DFT-R3 over m2  -> X[k1 + R1 (k2 + R2 k3)]
// The forward result stays in pass 3's registers in that permuted order;
// the spectral product is taken there against a kernel spectrum produced by
// the same passes (stored in the same per-thread order), and the inverse is
// the adjoint of the forward run backwards (inverse DFTs, conjugate
// twiddles), which returns natural order, unnormalised (x N).
//
// Shared memory holds one float2 per point in rows of R3 + 1 (one pad
// element per row), so every exchange is a conflict-free 64-bit access:
// element (k1, j, m2) with j = n2 or k2 sits at k1 * S + j * (R3 + 1) + m2.
// Pass 2 reads and writes the SAME positions of its combo (n2 in, k2 out),
// and so does pass 3 (m2 in and out): no barrier inside a pass.
//
// Per point and direction this costs two 64-bit shared-memory stores and
// loads, against one store and load per radix pass (plus a twiddle-table
// load) for the shared-memory pass-per-radix transform in fft_core.cuh.
#pragma once

#include "fft_core.cuh"

namespace b200 {
namespace fftr {

using fft::cmul;

template <int R1, int R2, int R3>
struct Shape {
  static constexpr int N = R1 * R2 * R3;
  static constexpr int M1 = R2 * R3;  // sub-transform length after pass 1
  static constexpr int T = M1;        // threads per transform
  static constexpr int G2 = R1 / R2;  // pass-2 DFTs per thread
  static constexpr int G3 = R1 / R3;  // pass-3 DFTs per thread
  static constexpr int P = R3 + 1;    // padded row
  static constexpr int S = R2 * P;    // one k1 block
  static constexpr int SMEM = R1 * S; // float2 elements of the exchange buffer
  static_assert(R1 % R2 == 0 && R1 % R3 == 0, "pass DFTs must tile the thread's points");
  static_assert(T % R2 == 0 && T % R3 == 0, "combo index arithmetic");
};

// v[k] *= w^k (forward) or conj(w)^k (inverse) for k >= 1, by a running
// product (R - 2 extra multiplies; error ~R ulps, far below the fp32 data).
template <int R, bool INV>
__device__ __forceinline__ void twiddle_run(float2 (&v)[R], float2 w) {
  if (INV) w.y = -w.y;
  float2 p = w;
#pragma unroll
  for (int k = 1; k < R; ++k) {
    v[k] = cmul(v[k], p);
    if (k + 1 < R) p = cmul(p, w);
  }
}

// e^{-2 pi i j / n} for an exact fraction j / n (n a power of two here).
__device__ __forceinline__ float2 unit_root(int j, int n) {
  float s, c;
  sincospif(-2.f * static_cast<float>(j) / static_cast<float>(n), &s, &c);
  return make_float2(c, s);
}

// Per-thread twiddle bases: W_N^(m1) for pass 1 (m1 = t) and W_M1^(m2) for
// pass 2 (every pass-2 combo of thread t has m2 = t mod R3).
template <int R1, int R2, int R3>
struct Bases {
  float2 w1, w2;
  __device__ __forceinline__ explicit Bases(int t) {
    using Sh = Shape<R1, R2, R3>;
    w1 = unit_root(t, Sh::N);
    w2 = unit_root(t % R3, Sh::M1);
  }
};

// Pass 1 forward: a[n1] = x[M1 n1 + t] in, spectrum slice to shared memory.
template <int R1, int R2, int R3>
__device__ __forceinline__ void fwd_pass1(float2 (&a)[R1], float2* sm, int t, float2 w1) {
  using Sh = Shape<R1, R2, R3>;
  fft::Dft<R1, false>::run(a);
  twiddle_run<R1, false>(a, w1);
  float2* p = sm + (t / R3) * Sh::P + (t % R3);
#pragma unroll
  for (int k1 = 0; k1 < R1; ++k1) p[k1 * Sh::S] = a[k1];
}

template <int R1, int R2, int R3, bool INV>
__device__ __forceinline__ void pass2(float2* sm, int t, float2 w2) {
  using Sh = Shape<R1, R2, R3>;
#pragma unroll
  for (int g = 0; g < Sh::G2; ++g) {
    const int k1 = g * (Sh::T / R3) + t / R3;
    float2* p = sm + k1 * Sh::S + (t % R3);
    float2 b[R2];
#pragma unroll
    for (int j = 0; j < R2; ++j) b[j] = p[j * Sh::P];
    if (!INV) {
      fft::Dft<R2, false>::run(b);
      twiddle_run<R2, false>(b, w2);
    } else {
      twiddle_run<R2, true>(b, w2);
      fft::Dft<R2, true>::run(b);
    }
#pragma unroll
    for (int j = 0; j < R2; ++j) p[j * Sh::P] = b[j];
  }
}

// Shared-memory row of pass-3 combo g of thread t (R3 consecutive values:
// m2 before the pass-3 DFT, k3 after it).
template <int R1, int R2, int R3>
__device__ __forceinline__ float2* pass3_row(float2* sm, int t, int g) {
  using Sh = Shape<R1, R2, R3>;
  const int k1 = g * (Sh::T / R2) + t / R2;
  return sm + k1 * Sh::S + (t % R2) * Sh::P;
}

// Pass 1 inverse: shared memory in, a[n1] = N x[M1 n1 + t] out.
template <int R1, int R2, int R3>
__device__ __forceinline__ void inv_pass1(float2 (&a)[R1], const float2* sm, int t, float2 w1) {
  using Sh = Shape<R1, R2, R3>;
  const float2* p = sm + (t / R3) * Sh::P + (t % R3);
#pragma unroll
  for (int k1 = 0; k1 < R1; ++k1) a[k1] = p[k1 * Sh::S];
  twiddle_run<R1, true>(a, w1);
  fft::Dft<R1, true>::run(a);
}

// Index of spectrum value k3 of pass-3 combo g of thread t in a channel's
// stored spectrum (lanes of a warp read consecutive elements).
template <int R1, int R2, int R3>
__device__ __forceinline__ int spec_index(int g, int k3, int t) {
  using Sh = Shape<R1, R2, R3>;
  return (k3 * Sh::G3 + g) * Sh::T + t;
}

}  // namespace fftr
}  // namespace b200
