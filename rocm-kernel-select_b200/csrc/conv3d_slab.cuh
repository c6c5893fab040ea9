// Shifted-window ("slab") implicit-GEMM conv3d on tcgen05: host entry points
// shared between conv3d_tc.cu (the C ABI and the box-per-tap kernel) and
// conv3d_slab.cu (the slab kernel and its input staging).
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"

namespace b200 {

// cuTensorMapEncodeTiled through the runtime's driver entry point (nullptr
// when the driver does not provide it).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Geometry of a slab-path problem (stride, padding and dilation already
// folded into phase grids); computed by slab_plan().
struct SlabPlan {
  bool ok = false;
  int64_t phases = 1, s_d = 1, s_h = 1, s_w = 1;   // stride = phases per dim
  int64_t Dq = 0, Hq = 0, Wq = 0;                  // phase-grid extents
  int64_t Do = 0, Ho = 0, Wo = 0;
  int64_t Cp = 0;                                  // staged channels (multiple of 8)
  int64_t rows = 0;                                // rows of the staged buffer
  size_t staging_bytes = 0;
};

// Plans the slab path for x [N, Cin, D, H, W] (16-bit) and a KD x KH x KW
// filter with params9 = (stride, padding, dilation) x (d, h, w).
// split: fp32 input staged as bf16 [hi | lo | hi] channel blocks.
SlabPlan slab_plan(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t KD,
                   int64_t KH, int64_t KW, const int64_t* params9, bool split);

// fp32 weights [Cout, Cin, KD, KH, KW] -> bf16 [taps][Cout][3 Cq] as
// [hi | hi | lo] blocks (Cq = Cin rounded up to 64), the operand that pairs
// with the split staging of an fp32 input.
int pack_weight_split(const float* w, __nv_bfloat16* wp, int64_t Cout, int64_t Cin, int64_t KD,
                      int64_t KH, int64_t KW, cudaStream_t stream);

// Stages x into the phase grids and runs the slab kernel (TIN = float: the
// split fp32 form with fp32 output).  Returns
// B200_UNSUPPORTED when the problem does not fit the kernel (the caller then
// uses the box-per-tap kernel).  `pair` selects CTA pairs (cta_group::2);
// `staged` skips the staging pass (the workspace already holds this x
// staged by an earlier call).
template <typename TIN>
int conv3d_slab(const void* x, const void* wp, const void* bias, void* y, int bias_dt,
                int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t Cout,
                int64_t KD, int64_t KH, int64_t KW, const int64_t* params9, int x_cl, int y_cl,
                int bn_code, bool pair, bool staged, void* ws, size_t ws_bytes,
                cudaStream_t stream);

}  // namespace b200
