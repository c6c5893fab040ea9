// FFT convolution entry points (long-filter depthwise conv1d, large-kernel
// dense conv3d).  Placeholder: every call declines until the kernels land.
#include "common.cuh"

using namespace b200;

extern "C" {

int b200_fft_supported_length(int64_t n) {
  (void)n;
  return 0;
}
size_t b200_fftconv1d_spectrum_bytes(int64_t C, int64_t nfft) {
  return static_cast<size_t>(C * (nfft / 2 + 1)) * 8;
}
int b200_fftconv1d_prepare(const void*, void*, int, int64_t, int64_t, int64_t, void*) {
  return fail_unsupported("fftconv1d not built");
}
int b200_fftconv1d_fwd(const void*, const void*, const void*, void*, int, int, int64_t, int64_t,
                       int64_t, int64_t, int64_t, int64_t, void*) {
  return fail_unsupported("fftconv1d not built");
}
size_t b200_fftconv3d_spectrum_bytes(int64_t Cout, int64_t Cin, int64_t fd, int64_t fh,
                                     int64_t fw) {
  return static_cast<size_t>(Cout * Cin * fd * fh * (fw / 2 + 1)) * 8;
}
int b200_fftconv3d_prepare(const void*, void*, int, int64_t, int64_t, int64_t, int64_t, int64_t,
                           int64_t, int64_t, int64_t, void*, size_t, void*) {
  return fail_unsupported("fftconv3d not built");
}
size_t b200_fftconv3d_workspace_bytes(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t) {
  return 0;
}
int b200_fftconv3d_fwd(const void*, const void*, const void*, void*, int, int, int64_t, int64_t,
                       int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                       const int64_t*, int64_t, int64_t, int64_t, void*, size_t, void*) {
  return fail_unsupported("fftconv3d not built");
}

}  // extern "C"
