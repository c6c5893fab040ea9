// FFT convolution for sm_100a: long-filter depthwise conv1d and large-kernel
// dense conv3d.
//
// Reference: amd_tuned_torch/fftconv_ops.py -- fft_conv (:603-746) pads the
// signal, rfftn's signal and kernel in fp32, multiplies by the conjugated
// kernel spectrum (elementwise for depthwise, complex_matmul :480-543 for
// dense), irfftn's, crops and adds the bias, output in the input dtype.  The
// reference runs the vendor FFT and recomputes the kernel spectrum per call.
//
// conv1d (depthwise).  One transform per (channel, pair of batch rows,
// segment): the two real rows are the real and imaginary parts of ONE
// complex sequence (linearity: IFFT(FFT(a + i b) * H) = (a corr w) +
// i (b corr w) for a real filter), so each complex transform serves two
// rows.  Two transform engines:
//  - nfft = 2048 ... 16384: the register-resident three-pass transform
//    (fft_reg.cuh) in persistent CTAs, the next item's input rows staged by
//    cp.async during the current item (measured at cfg 4b, 8192-point
//    segments: 1.15 ms against 2.35 ms for the shared-memory engine);
//  - other 2^a 3^b 5^c lengths: the whole transform in shared memory
//    (fft_core.cuh: in-place DIF forward, spectral product in digit-reversed
//    order, DIT inverse back to natural order).
// Either way the spectral product is taken against a kernel spectrum
// produced by the same forward passes, then crop + bias + dtype conversion
// on the way out.  HBM traffic: the two input rows, the channel's spectrum
// (shared by the CTAs of a channel through L2) and the two output rows.
#include "fft_core.cuh"
#include "fft_reg.cuh"

namespace b200 {
namespace {

// One CTA of kFftThreads per (channel, row pair), plans of radices <= 16.
// (1024 threads with radix <= 8 plans -- twice the resident warps -- measured
// no faster: the kernel is not occupancy-bound.)
constexpr int kFftThreads = 512;
constexpr int kFftMaxRadix = 16;
constexpr int64_t kMaxFftN = 24576;

size_t fft1d_smem(int n) {
  const int nhi = (n + fft::kLo - 1) >> fft::kLoBits;
  return static_cast<size_t>(fft::kLo + nhi + fft::padded_len(n)) * sizeof(float2);
}

// Forward pass 0 (span n, stride n/R) fed straight from the two input rows:
// transform position i holds input position q0 + i (zero outside [0, L)).
template <typename T, int R>
__device__ __forceinline__ void first_pass_from_rows(float2* buf, int n, const float2* tw0,
                                                     const T* x0, const T* x1, bool has1,
                                                     int64_t q0, int64_t L) {
  const int stride = n / R;
  for (int k = threadIdx.x; k < stride; k += blockDim.x) {
    float2 v[R];
#pragma unroll
    for (int m = 0; m < R; ++m) {
      const int64_t l = static_cast<int64_t>(k + m * stride) + q0;
      const bool in = l >= 0 && l < L;
      v[m] = make_float2(in ? to_f32(x0[l]) : 0.f, (in && has1) ? to_f32(x1[l]) : 0.f);
    }
    fft::Dft<R, false>::run(v);
    if (k != 0) fft::apply_twiddle_powers<R, false>(v, tw0[k]);
#pragma unroll
    for (int m = 0; m < R; ++m) buf[fft::pidx(k + m * stride)] = v[m];
  }
}

// Last forward pass (span R: R consecutive positions, no twiddles), the
// spectral product, and the first inverse pass over the same positions --
// all in registers, one shared-memory round trip.
template <int R>
__device__ __forceinline__ void last_fwd_product_first_inv(float2* buf, int n,
                                                            const float2* __restrict__ h) {
  const int ng = n / R;
  for (int g = threadIdx.x; g < ng; g += blockDim.x) {
    const int base = g * R;
    float2 v[R];
#pragma unroll
    for (int m = 0; m < R; ++m) v[m] = buf[fft::pidx(base + m)];
    fft::Dft<R, false>::run(v);
#pragma unroll
    for (int m = 0; m < R; ++m) v[m] = fft::cmul(v[m], __ldg(h + base + m));
    fft::Dft<R, true>::run(v);
#pragma unroll
    for (int m = 0; m < R; ++m) buf[fft::pidx(base + m)] = v[m];
  }
}

// Inverse pass 0 (span n) written straight to the two output rows:
// transform position i < vlen is output position o0 + i (cropped to L_out),
// scale 1/n, + bias, dtype conversion.
template <typename T, int R>
__device__ __forceinline__ void last_pass_to_rows(const float2* buf, int n, const float2* tw0,
                                                  T* y0, T* y1, bool has1, int64_t o0,
                                                  int64_t vlen, int64_t Lout, float scale,
                                                  float bv) {
  const int stride = n / R;
  for (int k = threadIdx.x; k < stride; k += blockDim.x) {
    float2 v[R];
#pragma unroll
    for (int m = 0; m < R; ++m) v[m] = buf[fft::pidx(k + m * stride)];
    if (k != 0) fft::apply_twiddle_powers<R, true>(v, tw0[k]);
    fft::Dft<R, true>::run(v);
#pragma unroll
    for (int m = 0; m < R; ++m) {
      const int64_t i = k + m * stride, l = o0 + i;
      if (i < vlen && l < Lout) {
        y0[l] = from_f32<T>(fmaf(v[m].x, scale, bv));
        if (has1) y1[l] = from_f32<T>(fmaf(v[m].y, scale, bv));
      }
    }
  }
}

#define B200_FFT_RADIX_SWITCH(r, CALL) \
  switch (r) {                         \
    case 16: CALL(16); break;          \
    case 8: CALL(8); break;            \
    case 4: CALL(4); break;            \
    case 2: CALL(2); break;            \
    case 9: CALL(9); break;            \
    case 3: CALL(3); break;            \
    default: CALL(5); break;           \
  }

// One CTA per (channel, row pair, segment).  Segment s of seg_len outputs
// (overlap-save): the transform holds inputs [s * seg_len - pad, + n) and its
// first seg_len circular-correlation outputs are exact when
// seg_len <= n - K + 1.  One segment covering L_out = the whole padded row.
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS, THREADS >= 512 ? 1 : 3)
fftconv1d_kernel(const T* __restrict__ x, const float2* __restrict__ spec,
                 const void* __restrict__ bias, int bias_dt, T* __restrict__ y, int64_t B,
                 int64_t C, int64_t L, int64_t pad, int64_t Lout, int64_t seg_len, int64_t segs,
                 const fft::Plan plan, int tw_count) {
  extern __shared__ float2 sm[];
  const int n = plan.n;
  float2* tw = sm;
  float2* buf = tw + ((tw_count + 1) & ~1);

  const int64_t pairs = (B + 1) / 2;
  const int64_t seg = blockIdx.x % segs;
  const int64_t rest = blockIdx.x / segs;
  const int64_t c = rest / pairs;
  const int64_t b0 = 2 * (rest % pairs), b1 = b0 + 1;
  const int64_t o0 = seg * seg_len;
  const bool has1 = b1 < B;
  const T* x0 = x + (b0 * C + c) * L;
  const T* x1 = x + (min64(b1, B - 1) * C + c) * L;
  T* y0 = y + (b0 * C + c) * Lout;
  T* y1 = y + (min64(b1, B - 1) * C + c) * Lout;

  fft::build_pass_twiddles(tw, plan);
  __syncthreads();
  // Span and twiddle-table offset of every pass.
  int span[fft::kMaxPasses], off[fft::kMaxPasses];
  {
    int s = n, o = 0;
    for (int i = 0; i < plan.passes; ++i) {
      span[i] = s;
      off[i] = o;
      o += s / plan.radix[i];
      s /= plan.radix[i];
    }
  }
  const int P = plan.passes;

#define B200_FIRST(R) first_pass_from_rows<T, R>(buf, n, tw, x0, x1, has1, o0 - pad, L)
  B200_FFT_RADIX_SWITCH(plan.radix[0], B200_FIRST)
#undef B200_FIRST
  __syncthreads();
  for (int i = 1; i < P - 1; ++i) {
    fft::run_pass_t<false, kFftMaxRadix>(plan.radix[i], buf, n, span[i], tw + off[i]);
    __syncthreads();
  }
  const float2* h = spec + c * n;
#define B200_MID(R) last_fwd_product_first_inv<R>(buf, n, h)
  B200_FFT_RADIX_SWITCH(plan.radix[P - 1], B200_MID)
#undef B200_MID
  __syncthreads();
  for (int i = P - 2; i >= 1; --i) {
    fft::run_pass_t<true, kFftMaxRadix>(plan.radix[i], buf, n, span[i], tw + off[i]);
    __syncthreads();
  }
  const float scale = 1.0f / static_cast<float>(n);
  const float bv = bias ? load_param(bias, bias_dt, c) : 0.f;
#define B200_LAST(R) \
  last_pass_to_rows<T, R>(buf, n, tw, y0, y1, has1, o0, seg_len, Lout, scale, bv)
  B200_FFT_RADIX_SWITCH(plan.radix[0], B200_LAST)
#undef B200_LAST
}

template <typename K>
int prep_smem(K kern, size_t smem) {
  B200_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
  return B200_OK;
}

// ------------------------------------------------ register-resident path ---
// Transform lengths with a register-resident plan (fft_reg.cuh).  Persistent
// CTAs of R2 * R3 threads walk the (channel, row pair, segment) items, every
// point in registers between the two shared-memory exchanges of each
// direction.  The channel's spectrum is stored in the plan's per-thread
// order (written by fftconv1d_reg_prepare_kernel, which runs the same
// forward passes).  When the rows are 16-byte aligned the next item's two
// input segments are copied into a staging buffer by cp.async while the
// current item is transformed, so the load latency is off the critical path.

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// One work item: channel c, batch rows b0 and b0 + 1 (has1), outputs from o0.
struct FftItem {
  int64_t c, b0, o0;
  bool has1;
};
// (32-bit division: the host keeps the item count below 2^31, and a 64-bit
// division is a subroutine call that forces the live points to spill.)
__device__ __forceinline__ FftItem fft_item(int item, int segs, int pairs, int64_t B,
                                            int64_t seg_len) {
  FftItem it;
  const int rest = item / segs, seg = item - rest * segs;
  const int c = rest / pairs;
  it.c = c;
  it.b0 = 2 * (rest - c * pairs);
  it.has1 = it.b0 + 1 < B;
  it.o0 = seg * seg_len;
  return it;
}

// Elements of T per 16-byte chunk, and staged elements per row: the row
// segment [q0, q0 + N) copied from the chunk boundary at or below q0.
template <typename T, int N>
struct FftStage {
  static constexpr int VE = 16 / static_cast<int>(sizeof(T));
  static constexpr int CHUNKS = N / VE + 1;
  static constexpr int ROW = CHUNKS * VE;
  static constexpr size_t BYTES = 2 * ROW * sizeof(T);
};

// Issues the cp.async copies of item `it`'s two row segments (zero fill
// outside [0, L) and for a missing second row).
template <typename T, int N, int THREADS>
__device__ __forceinline__ void fft_stage_issue(T* stage, const T* x, const FftItem& it, int64_t C,
                                                int64_t L, int64_t pad) {
  using St = FftStage<T, N>;
  const int64_t q0 = it.o0 - pad;
  const int64_t base = q0 & ~static_cast<int64_t>(St::VE - 1);  // VE is a power of two
  for (int j = threadIdx.x; j < 2 * St::CHUNKS; j += THREADS) {
    const int r = j >= St::CHUNKS;
    const int k = j - r * St::CHUNKS;
    const T* row = x + ((it.b0 + r) * C + it.c) * L;
    const int64_t l = base + static_cast<int64_t>(k) * St::VE;
    int bytes = 0;
    const T* src = x;
    if ((r == 0 || it.has1) && l >= 0 && l < L) {
      bytes = static_cast<int>(min64(St::VE, L - l) * sizeof(T));
      src = row + l;
    }
    cp_async16(stage + r * St::ROW + k * St::VE, src, bytes);
  }
  cp_async_commit();
}

template <typename T, int R1, int R2, int R3>
__global__ void __launch_bounds__(R2 * R3, (R2 * R3 <= 256) ? 2 : 1)
fftconv1d_reg_kernel(const T* __restrict__ x, const float2* __restrict__ spec,
                     const void* __restrict__ bias, int bias_dt, T* __restrict__ y, int64_t B,
                     int64_t C, int64_t L, int64_t pad, int64_t Lout, int64_t seg_len,
                     int64_t segs, int staged) {
  using Sh = fftr::Shape<R1, R2, R3>;
  using St = FftStage<T, Sh::N>;
  extern __shared__ float2 sm[];
  T* stage = reinterpret_cast<T*>(sm + Sh::SMEM);
  const int t = threadIdx.x;
  const int pairs = static_cast<int>((B + 1) / 2);
  const int nseg = static_cast<int>(segs);
  const int items = static_cast<int>(C) * pairs * nseg;
  int item = blockIdx.x;
  if (item >= items) return;
  const fftr::Bases<R1, R2, R3> tw(t);
  const float scale = 1.0f / static_cast<float>(Sh::N);
  if (staged)
    fft_stage_issue<T, Sh::N, Sh::T>(stage, x, fft_item(item, nseg, pairs, B, seg_len), C, L,
                                     pad);

  for (; item < items; item += static_cast<int>(gridDim.x)) {
    const FftItem it = fft_item(item, nseg, pairs, B, seg_len);
    const int64_t q0 = it.o0 - pad;  // input position of transform point 0
    const float2* h = spec + it.c * Sh::N;
    float2 a[R1];
    if (staged) {
      cp_async_wait_all();
      __syncthreads();  // staged rows visible; the previous item's exchange reads done
      const int off = static_cast<int>(q0 & (St::VE - 1));
      const T* s0 = stage + off + t;
      const T* s1 = s0 + St::ROW;
#pragma unroll
      for (int n1 = 0; n1 < R1; ++n1)
        a[n1] = make_float2(to_f32(s0[n1 * Sh::M1]), to_f32(s1[n1 * Sh::M1]));
    } else {
      __syncthreads();  // the previous item's exchange reads done
      const T* x0 = x + (it.b0 * C + it.c) * L;
      const T* x1 = x + (min64(it.b0 + 1, B - 1) * C + it.c) * L;
#pragma unroll
      for (int n1 = 0; n1 < R1; ++n1) {
        const int64_t l = q0 + n1 * Sh::M1 + t;
        const bool in = l >= 0 && l < L;
        a[n1] = make_float2(in ? to_f32(x0[l]) : 0.f, (in && it.has1) ? to_f32(x1[l]) : 0.f);
      }
    }
    fftr::fwd_pass1<R1, R2, R3>(a, sm, t, tw.w1);
    __syncthreads();  // exchange written; every thread is past its staging reads
    if (staged) {
      const int next = item + static_cast<int>(gridDim.x);
      if (next < items)
        fft_stage_issue<T, Sh::N, Sh::T>(stage, x, fft_item(next, nseg, pairs, B, seg_len), C,
                                         L, pad);
    }
    // Spectrum values of the first pass-3 combo, in flight during pass 2.
    float2 hv[R3];
#pragma unroll
    for (int k = 0; k < R3; ++k) hv[k] = __ldg(h + fftr::spec_index<R1, R2, R3>(0, k, t));
    fftr::pass2<R1, R2, R3, false>(sm, t, tw.w2);
    __syncthreads();
#pragma unroll
    for (int g = 0; g < Sh::G3; ++g) {
      float2* p = fftr::pass3_row<R1, R2, R3>(sm, t, g);
      float2 d[R3];
#pragma unroll
      for (int m = 0; m < R3; ++m) d[m] = p[m];
      fft::Dft<R3, false>::run(d);
#pragma unroll
      for (int k = 0; k < R3; ++k) d[k] = fft::cmul(d[k], hv[k]);
      if (g + 1 < Sh::G3) {
#pragma unroll
        for (int k = 0; k < R3; ++k)
          hv[k] = __ldg(h + fftr::spec_index<R1, R2, R3>(g + 1, k, t));
      }
      fft::Dft<R3, true>::run(d);
#pragma unroll
      for (int m = 0; m < R3; ++m) p[m] = d[m];
    }
    __syncthreads();
    fftr::pass2<R1, R2, R3, true>(sm, t, tw.w2);
    __syncthreads();
    fftr::inv_pass1<R1, R2, R3>(a, sm, t, tw.w1);

    const float bv = bias ? load_param(bias, bias_dt, it.c) : 0.f;
    const int64_t lim = min64(seg_len, Lout - it.o0);
    T* y0 = y + (it.b0 * C + it.c) * Lout + it.o0;
    T* y1 = y + (min64(it.b0 + 1, B - 1) * C + it.c) * Lout + it.o0;
#pragma unroll
    for (int n1 = 0; n1 < R1; ++n1) {
      const int i = n1 * Sh::M1 + t;
      if (i < lim) {
        y0[i] = from_f32<T>(fmaf(a[n1].x, scale, bv));
        if (it.has1) y1[i] = from_f32<T>(fmaf(a[n1].y, scale, bv));
      }
    }
  }
}

// Kernel spectrum for the register-resident plan, one CTA per channel: the
// zero-padded real filter through the same forward passes, conjugated.
template <typename T, int R1, int R2, int R3>
__global__ void __launch_bounds__(R2 * R3, 1)
fftconv1d_reg_prepare_kernel(const T* __restrict__ w, float2* __restrict__ spec, int64_t K) {
  using Sh = fftr::Shape<R1, R2, R3>;
  extern __shared__ float2 sm[];
  const int t = threadIdx.x;
  const int64_t c = blockIdx.x;
  const fftr::Bases<R1, R2, R3> tw(t);
  float2 a[R1];
#pragma unroll
  for (int n1 = 0; n1 < R1; ++n1) {
    const int i = n1 * Sh::M1 + t;
    a[n1] = make_float2(i < K ? to_f32(w[c * K + i]) : 0.f, 0.f);
  }
  fftr::fwd_pass1<R1, R2, R3>(a, sm, t, tw.w1);
  __syncthreads();
  fftr::pass2<R1, R2, R3, false>(sm, t, tw.w2);
  __syncthreads();
  float2* out = spec + c * Sh::N;
#pragma unroll
  for (int g = 0; g < Sh::G3; ++g) {
    const float2* p = fftr::pass3_row<R1, R2, R3>(sm, t, g);
    float2 d[R3];
#pragma unroll
    for (int m = 0; m < R3; ++m) d[m] = p[m];
    fft::Dft<R3, false>::run(d);
#pragma unroll
    for (int k = 0; k < R3; ++k)
      out[fftr::spec_index<R1, R2, R3>(g, k, t)] = make_float2(d[k].x, -d[k].y);
  }
}

// Lengths with a register-resident plan, and their radices.
bool reg_plan(int64_t n) { return n == 2048 || n == 4096 || n == 8192 || n == 16384; }

#define B200_REG_SHAPES(n, CALL)   \
  switch (n) {                     \
    case 2048: CALL(16, 16, 8); break;  \
    case 4096: CALL(16, 16, 16); break; \
    case 8192: CALL(32, 16, 16); break; \
    default: CALL(32, 32, 16); break;   \
  }

// Persistent grid: as many CTAs as fit on the device at once (at most one
// per item).  Rows are staged by cp.async when every row start is 16-byte
// aligned.
template <typename T>
int launch_fftconv1d_reg(const T* x, const float2* sp, const void* bias, int bias_dt, T* y,
                         int64_t B, int64_t C, int64_t L, int64_t pad, int64_t Lout,
                         int64_t seg_len, int64_t segs, int n, cudaStream_t s) {
  const int64_t items = C * ((B + 1) / 2) * segs;
  int staged = (reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                      (L * static_cast<int64_t>(sizeof(T))) % 16 == 0) ? 1 : 0;
  int rc = B200_OK;
#define B200_REG_LAUNCH(R1, R2, R3)                                                           \
  {                                                                                          \
    using Sh = fftr::Shape<R1, R2, R3>;                                                      \
    auto kern = fftconv1d_reg_kernel<T, R1, R2, R3>;                                         \
    const size_t xbytes = static_cast<size_t>(Sh::SMEM) * sizeof(float2);                    \
    if (xbytes + FftStage<T, Sh::N>::BYTES > static_cast<size_t>(max_smem_optin()))          \
      staged = 0;                                                                            \
    const size_t smem = xbytes + (staged ? FftStage<T, Sh::N>::BYTES : 0);                   \
    if ((rc = prep_smem(kern, smem)) != B200_OK) return rc;                                  \
    int per_sm = 0;                                                                          \
    B200_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, Sh::T, smem)); \
    const int64_t grid = min64(items, static_cast<int64_t>(sm_count()) * max(per_sm, 1));    \
    kern<<<static_cast<unsigned>(grid), Sh::T, smem, s>>>(x, sp, bias, bias_dt, y, B, C, L,  \
                                                          pad, Lout, seg_len, segs, staged); \
  }
  B200_REG_SHAPES(n, B200_REG_LAUNCH)
#undef B200_REG_LAUNCH
  B200_LAUNCH_CHECK("fftconv1d_reg_kernel");
  return rc;
}

template <typename T>
int launch_fftconv1d_reg_prepare(const T* w, float2* spec, int64_t C, int64_t K, int n,
                                 cudaStream_t s) {
  int rc = B200_OK;
#define B200_REG_PREP(R1, R2, R3)                                                            \
  {                                                                                         \
    using Sh = fftr::Shape<R1, R2, R3>;                                                     \
    const size_t smem = static_cast<size_t>(Sh::SMEM) * sizeof(float2);                     \
    if ((rc = prep_smem(fftconv1d_reg_prepare_kernel<T, R1, R2, R3>, smem)) != B200_OK)     \
      return rc;                                                                            \
    fftconv1d_reg_prepare_kernel<T, R1, R2, R3><<<static_cast<unsigned>(C), Sh::T, smem, s>>>( \
        w, spec, K);                                                                        \
  }
  B200_REG_SHAPES(n, B200_REG_PREP)
#undef B200_REG_PREP
  B200_LAUNCH_CHECK("fftconv1d_reg_prepare_kernel");
  return rc;
}

// Host mirror of fft::pass_tw_count.
int host_tw_count(const fft::Plan& p) {
  int total = 0, span = p.n;
  for (int i = 0; i < p.passes; ++i) {
    total += span / p.radix[i];
    span /= p.radix[i];
  }
  return total;
}

// Kernel spectrum, one CTA per channel: the zero-padded real filter through
// the same forward plan, stored conjugated in transform-position order.
template <typename T>
__global__ void __launch_bounds__(kFftThreads, 1)
fftconv1d_prepare_kernel(const T* __restrict__ w, float2* __restrict__ spec, int64_t K,
                         const fft::Plan plan) {
  extern __shared__ float2 sm[];
  const int n = plan.n;
  const int nhi = (n + fft::kLo - 1) >> fft::kLoBits;
  float2* lo = sm;
  float2* hi = lo + fft::kLo;
  float2* buf = hi + nhi;
  const int64_t c = blockIdx.x;
  fft::build_twiddles(lo, hi, n);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    buf[fft::pidx(i)] = make_float2(i < K ? to_f32(w[c * K + i]) : 0.f, 0.f);
  __syncthreads();
  fft::forward(buf, plan, lo, hi);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float2 v = buf[fft::pidx(i)];
    spec[c * n + i] = make_float2(v.x, -v.y);
  }
}

bool plan1d(int64_t n, fft::Plan* p) {
  return n >= 2 && n <= kMaxFftN && fft::make_plan(n, p, kFftMaxRadix);
}

// Short transforms (segments) run as CTAs of 256 threads, three per SM (80
// registers; an 8192-point segment takes ~70 KB of shared memory); the
// whole-row transform as one 512-thread CTA per SM.
template <typename T, int THREADS>
int launch_fftconv1d_t(const T* x, const float2* sp, const void* bias, int bias_dt, T* y,
                       int64_t B, int64_t C, int64_t L, int64_t pad, int64_t Lout,
                       int64_t seg_len, int64_t segs, const fft::Plan& plan, cudaStream_t s) {
  const int twc = host_tw_count(plan);
  const size_t smem =
      static_cast<size_t>(((twc + 1) & ~1) + fft::padded_len(plan.n)) * sizeof(float2);
  int rc;
  if ((rc = prep_smem(fftconv1d_kernel<T, THREADS>, smem)) != B200_OK) return rc;
  const int64_t blocks = C * ((B + 1) / 2) * segs;
  fftconv1d_kernel<T, THREADS><<<static_cast<unsigned>(blocks), THREADS, smem, s>>>(
      x, sp, bias, bias_dt, y, B, C, L, pad, Lout, seg_len, segs, plan, twc);
  B200_LAUNCH_CHECK("fftconv1d_kernel");
  return B200_OK;
}

template <typename T>
int launch_fftconv1d_typed(const void* x, const void* spectrum, const void* bias, int bias_dt,
                           void* y, int64_t B, int64_t C, int64_t L, int64_t pad, int64_t Lout,
                           int64_t seg_len, int64_t segs, const fft::Plan& plan, cudaStream_t s) {
  const T* xt = static_cast<const T*>(x);
  T* yt = static_cast<T*>(y);
  const float2* sp = static_cast<const float2*>(spectrum);
  if (reg_plan(plan.n))
    return launch_fftconv1d_reg<T>(xt, sp, bias, bias_dt, yt, B, C, L, pad, Lout, seg_len, segs,
                                   plan.n, s);
  if (plan.n <= 8192)
    return launch_fftconv1d_t<T, 256>(xt, sp, bias, bias_dt, yt, B, C, L, pad, Lout, seg_len,
                                      segs, plan, s);
  return launch_fftconv1d_t<T, kFftThreads>(xt, sp, bias, bias_dt, yt, B, C, L, pad, Lout,
                                            seg_len, segs, plan, s);
}

int launch_fftconv1d(const void* x, const void* spectrum, const void* bias, void* y, int dtype,
                     int bias_dt, int64_t B, int64_t C, int64_t L, int64_t pad, int64_t Lout,
                     int64_t seg_len, int64_t segs, const fft::Plan& plan, cudaStream_t s) {
  if (dtype == B200_DTYPE_F32)
    return launch_fftconv1d_typed<float>(x, spectrum, bias, bias_dt, y, B, C, L, pad, Lout,
                                         seg_len, segs, plan, s);
  if (dtype == B200_DTYPE_F16)
    return launch_fftconv1d_typed<__half>(x, spectrum, bias, bias_dt, y, B, C, L, pad, Lout,
                                          seg_len, segs, plan, s);
  return launch_fftconv1d_typed<__nv_bfloat16>(x, spectrum, bias, bias_dt, y, B, C, L, pad,
                                               Lout, seg_len, segs, plan, s);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int b200_fft_supported_length(int64_t n) {
  fft::Plan p;
  return plan1d(n, &p) ? 1 : 0;
}

size_t b200_fftconv1d_spectrum_bytes(int64_t C, int64_t nfft) {
  return static_cast<size_t>(C * nfft) * sizeof(float2);
}

int b200_fftconv1d_prepare(const void* w, void* spectrum, int w_dtype, int64_t C, int64_t K,
                           int64_t nfft, void* stream) {
  if (!w || !spectrum) return fail_arg("NULL pointer");
  if (!dtype_ok(w_dtype)) return fail_arg("bad dtype");
  fft::Plan plan;
  if (!plan1d(nfft, &plan)) return fail_unsupported("FFT length not 2^a 3^b 5^c or too long");
  if (C <= 0 || K <= 0 || K > nfft) return fail_arg("bad size");
  if (C > 0x7fffffffLL) return fail_unsupported("too many channels");
  const size_t smem = fft1d_smem(plan.n);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float2* sp = static_cast<float2*>(spectrum);
  if (reg_plan(plan.n)) {
    if (w_dtype == B200_DTYPE_F32)
      return launch_fftconv1d_reg_prepare(static_cast<const float*>(w), sp, C, K, plan.n, s);
    if (w_dtype == B200_DTYPE_F16)
      return launch_fftconv1d_reg_prepare(static_cast<const __half*>(w), sp, C, K, plan.n, s);
    return launch_fftconv1d_reg_prepare(static_cast<const __nv_bfloat16*>(w), sp, C, K, plan.n,
                                        s);
  }
  int rc;
  if (w_dtype == B200_DTYPE_F32) {
    if ((rc = prep_smem(fftconv1d_prepare_kernel<float>, smem)) != B200_OK) return rc;
    fftconv1d_prepare_kernel<float><<<(unsigned)C, kFftThreads, smem, s>>>(
        static_cast<const float*>(w), static_cast<float2*>(spectrum), K, plan);
  } else if (w_dtype == B200_DTYPE_F16) {
    if ((rc = prep_smem(fftconv1d_prepare_kernel<__half>, smem)) != B200_OK) return rc;
    fftconv1d_prepare_kernel<__half><<<(unsigned)C, kFftThreads, smem, s>>>(
        static_cast<const __half*>(w), static_cast<float2*>(spectrum), K, plan);
  } else {
    if ((rc = prep_smem(fftconv1d_prepare_kernel<__nv_bfloat16>, smem)) != B200_OK) return rc;
    fftconv1d_prepare_kernel<__nv_bfloat16><<<(unsigned)C, kFftThreads, smem, s>>>(
        static_cast<const __nv_bfloat16*>(w), static_cast<float2*>(spectrum), K, plan);
  }
  B200_LAUNCH_CHECK("fftconv1d_prepare_kernel");
  return B200_OK;
}

int b200_fftconv1d_fwd_os(const void* x, const void* spectrum, const void* bias, void* y,
                          int dtype, int bias_dtype, int64_t B, int64_t C, int64_t L, int64_t K,
                          int64_t pad, int64_t L_out, int64_t nfft, void* stream) {
  if (!x || !spectrum || !y) return fail_arg("NULL pointer");
  if (!dtype_ok(dtype) || (bias && !dtype_ok(bias_dtype))) return fail_arg("bad dtype");
  if (B <= 0 || C <= 0 || L <= 0 || K <= 0 || pad < 0 || L_out <= 0) return fail_arg("bad size");
  if (L_out != L + 2 * pad - K + 1) return fail_arg("L_out != L + 2 * pad - K + 1");
  fft::Plan plan;
  if (!plan1d(nfft, &plan)) return fail_unsupported("FFT length not 2^a 3^b 5^c or too long");
  if (K > nfft) return fail_arg("nfft shorter than the filter");
  if (plan.passes < 2) return fail_unsupported("FFT length too short for the fused kernel");
  const int64_t seg_len = nfft - K + 1;
  const int64_t segs = (L_out + seg_len - 1) / seg_len;
  const int64_t blocks = C * ((B + 1) / 2) * segs;
  if (blocks > 0x7fffffffLL) return fail_unsupported("grid too large");
  return launch_fftconv1d(x, spectrum, bias, y, dtype, bias_dtype, B, C, L, pad, L_out, seg_len,
                          segs, plan, static_cast<cudaStream_t>(stream));
}

int b200_fftconv1d_fwd(const void* x, const void* spectrum, const void* bias, void* y,
                       int dtype, int bias_dtype, int64_t B, int64_t C, int64_t L,
                       int64_t pad, int64_t L_out, int64_t nfft, void* stream) {
  if (!x || !spectrum || !y) return fail_arg("NULL pointer");
  if (!dtype_ok(dtype) || (bias && !dtype_ok(bias_dtype))) return fail_arg("bad dtype");
  if (B <= 0 || C <= 0 || L <= 0 || pad < 0 || L_out <= 0) return fail_arg("bad size");
  fft::Plan plan;
  if (!plan1d(nfft, &plan)) return fail_unsupported("FFT length not 2^a 3^b 5^c or too long");
  if (L + 2 * pad > nfft) return fail_arg("nfft shorter than the padded signal");
  if (L_out > L + 2 * pad) return fail_arg("L_out too long");
  const int64_t blocks = C * ((B + 1) / 2);
  if (blocks > 0x7fffffffLL) return fail_unsupported("grid too large");
  if (plan.passes < 2) return fail_unsupported("FFT length too short for the fused kernel");
  return launch_fftconv1d(x, spectrum, bias, y, dtype, bias_dtype, B, C, L, pad, L_out, L_out, 1,
                          plan, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
