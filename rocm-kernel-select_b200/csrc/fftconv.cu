// FFT convolution for sm_100a: long-filter depthwise conv1d and large-kernel
// dense conv3d.
//
// Reference: amd_tuned_torch/fftconv_ops.py -- fft_conv (:603-746) pads the
// signal, rfftn's signal and kernel in fp32, multiplies by the conjugated
// kernel spectrum (elementwise for depthwise, complex_matmul :480-543 for
// dense), irfftn's, crops and adds the bias, output in the input dtype.  The
// reference runs the vendor FFT and recomputes the kernel spectrum per call.
//
// conv1d (depthwise).  One CTA per (channel, pair of batch rows): the two real
// rows are the real and imaginary parts of ONE complex sequence (linearity:
// IFFT(FFT(a + i b) * H) = (a corr w) + i (b corr w) for a real filter), so
// each complex transform serves two rows.  The whole transform lives in
// shared memory (fft_core.cuh: in-place DIF forward, spectral product in
// digit-reversed order against a kernel spectrum produced by the same
// forward plan, DIT inverse back to natural order), then crop + bias +
// dtype conversion on the way out.  HBM traffic: the two input rows, the
// channel's spectrum (shared by the B/2 CTAs of a channel through L2) and
// the two output rows.
#include "fft_core.cuh"

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

template <typename K>
int prep_smem(K kern, size_t smem) {
  B200_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
  return B200_OK;
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
