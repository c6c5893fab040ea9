/*
 * b200conv.h -- C ABI of libb200conv.so, the sm_100a kernels behind the
 * amd_tuned_torch conv/norm hot path (F.conv1d depthwise, F.conv3d,
 * F.group_norm).
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are raw DEVICE pointers owned by the caller; the
 *     library never allocates or frees caller memory.  Where an op needs
 *     scratch, a *_workspace_bytes() query tells the caller how much to pass.
 *   - Sizes are int64_t element counts; dtypes are B200_DTYPE_* codes.
 *   - `stream` is a cudaStream_t passed as void* (torch's
 *     torch.cuda.current_stream().cuda_stream); every launch goes on it.
 *   - Return value: 0 = launched, > 0 = B200_UNSUPPORTED (the call is outside
 *     what the kernel handles -- the Python candidate declines and the contest
 *     moves on), < 0 = error (-1 bad argument, -(1000 + cudaError_t) for a
 *     CUDA runtime error).  b200_last_error() returns a message for the
 *     calling thread's last non-zero status.
 *
 * Each declaration cites the reference interface it replaces
 * (WifiLast/rocm-kernel-select, path:line).
 */
#ifndef B200CONV_H
#define B200CONV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_DTYPE_F32 0
#define B200_DTYPE_F16 1
#define B200_DTYPE_BF16 2

#define B200_OK 0
#define B200_UNSUPPORTED 1
#define B200_ERR_ARG (-1)

/* Library version (major*10000 + minor*100 + patch). No reference
 * counterpart: the reference ships pybind11 modules, see
 * amd_tuned_torch/_native_loader.py:56-147 for its loader. */
int b200_version(void);

/* Message for the calling thread's last non-zero status. */
const char* b200_last_error(void);

/* Reads and clears the device-side fault word that bounded waits inside the
 * kernels set when a wait runs out (0 = none).  Synchronizes `stream`. */
int b200_read_device_flags(void* stream, int* flags_out);

/* Number of SMs on the current device (grid sizing). */
int b200_sm_count(void);

/* ------------------------------------------------------------------ */
/* GroupNorm forward.
 * Replaces _C.group_norm(input, num_groups, weight?, bias?, eps)
 * (src/main_rocm.cpp:556-599) and its kernel group_norm_kernel
 * (src/cuda/group_norm.cu:40-104).  x, y: contiguous [N, C, S] with
 * S = product of spatial dims; gamma/beta: [C] of `affine_dtype` or NULL.
 * variant: 0 auto (streaming for 16-byte rows that fit the L2 keep budget,
 *            else the cluster kernel for small groups, else split),
 *          1 split (stats + apply, uses workspace),
 *          2 two-pass: statistics pass, then a normalise pass that re-reads
 *            x (from L2 when the tensor fits), both 16-byte vectorised,
 *          3 streaming: statistics on a persistent grid (next chunk's loads
 *            in flight while the current one is reduced), a per-channel
 *            scale/shift kernel, and a persistent normalise pass over the
 *            whole tensor (16-byte rows required),
 *          16 + k: single-read cluster kernel with k CTAs per group
 *          (k in {1, 2, 4, 8, 16}; group slice held in shared memory). */
size_t b200_gn_workspace_bytes(int64_t N, int64_t C, int64_t S, int64_t G, int dtype,
                               int variant);
int b200_gn_fwd(const void* x, const void* gamma, const void* beta, void* y, int dtype,
                int affine_dtype, int64_t N, int64_t C, int64_t S, int64_t G, float eps,
                int variant, void* workspace, size_t workspace_bytes, void* stream);

/* GroupNorm forward that allocates nothing: same result as b200_gn_fwd's
 * split variant, with its scratch in a fixed 256 KiB device array inside the
 * library instead of a caller workspace.  For callers that cannot allocate
 * device memory (their device memory belongs to their own pool or arena, or
 * they run in a loop where an allocation is not acceptable).  Limit:
 * 3 * N * G * (ceil(C/G * S / 65536) + 1) floats <= 65536, else B200_ERR_ARG.
 * Calls share the array: calls that may overlap on the GPU race.  The first
 * call on a device resolves the array's address (make it before any stream
 * capture); it is resolved again if the device's context is re-created
 * (cudaDeviceReset).  No counterpart in the reference. */
int b200_gn_fwd_static_scratch(const void* x, const void* gamma, const void* beta, void* y,
                               int dtype, int affine_dtype, int64_t N, int64_t C, int64_t S,
                               int64_t G, float eps, void* stream);

/* Merges per-rank (count, mean, M2) triples parts [ranks][groups][3] (fp32)
 * in rank order (Chan et al., fp64) into out [groups][3]: the statistics
 * exchange of the T-sharded GroupNorm (all-gather of b200_gn_partial_stats,
 * then this, identical on every rank).  No counterpart in the reference (it
 * has no sharded GroupNorm). */
int b200_gn_merge_ranks(const float* parts, float* out, int64_t ranks, int64_t groups,
                        void* stream);

/* GroupNorm statistics only: per (n, g) mean and rstd (fp32, [N*G] each).
 * Used by the fused GroupNorm->SiLU->conv3d producer and by the T-sharded
 * stack, which merges per-rank partial statistics.  Partial form: writes
 * (count, mean, M2) triples per (n, g) of THIS tensor without finalising.
 * No single reference counterpart: it is the first pass of
 * src/cuda/group_norm.cu:55-90 exposed on its own. */
size_t b200_gn_stats_workspace_bytes(int64_t N, int64_t C, int64_t S, int64_t G, int dtype);
int b200_gn_partial_stats(const void* x, float* partial_out, int dtype, int64_t N, int64_t C,
                          int64_t S, int64_t G, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Normalise + affine + optional SiLU, reading x NCDHW ([N, C, S]) and writing
 * y either NCDHW (to_channels_last = 0) or channels-last [N, S, C]
 * (to_channels_last = 1, the conv3d operand layout).  stats: (count, mean,
 * M2) triples per (n, g) as produced by b200_gn_partial_stats (possibly merged
 * across ranks).  Reference analogue: ck_norm_ops.group_norm_silu
 * (amd_tuned_torch/ck_norm_ops.py:93-103) and the GN->SiLU prologue of
 * conv_fusion_ops.group_norm_silu (amd_tuned_torch/conv_fusion_ops.py:245-353). */
int b200_gn_apply(const void* x, const float* stats, const void* gamma, const void* beta,
                  void* y, int dtype, int affine_dtype, int64_t N, int64_t C, int64_t S,
                  int64_t G, float eps, int silu, int to_channels_last, void* stream);

/* ------------------------------------------------------------------ */
/* Depthwise conv1d forward, stride 1, dilation 1, zero padding:
 *   y[b,c,l] = bias[c] + sum_k w[c,k] * x[b,c,l - pad + k],  l < L_out.
 * Replaces _native_depthwise_conv1d.conv1d_forward(u, weight[C,K], bias[C],
 * padding, is_bhl=True) (amd_tuned_torch/_vendor/flashfftconv_depthwise_conv1d/
 * host.cpp:7-11 -> conv1d.h:56-83 -> conv1d_bhl.cu:100-140).  x: [B, C, L],
 * w: [C, K], bias: [C] or NULL (w_dtype for both), y: [B, C, L_out].
 * variant: 0, or B200_DWCONV1D_FLIP_TAPS to use w[c, K-1-k] for tap k -- the
 * input gradient of the forward at padding p is this op applied to dy with
 * the flipped taps at padding K-1-p (no bias), output length L. */
#define B200_DWCONV1D_FLIP_TAPS 1
int b200_dwconv1d_fwd(const void* x, const void* w, const void* bias, void* y, int dtype,
                      int w_dtype, int64_t B, int64_t C, int64_t L, int64_t K, int64_t pad,
                      int64_t L_out, int variant, void* stream);

/* Depthwise conv1d weight and bias gradients of the forward above:
 *   dw[c,k] = sum_{b,o} dy[b,c,o] * x[b,c,o-pad+k],  dbias[c] = sum_{b,o} dy[b,c,o]
 * x: [B, C, L], dy: [B, C, L_out] (dtype), dw: [C, K], dbias: [C] or NULL
 * (w_dtype).  Fixed-order reduction (deterministic).  workspace: at least
 * b200_dwconv1d_bwd_workspace_bytes() bytes.  Replaces the weight/bias half
 * of conv1d_bwd (amd_tuned_torch/_vendor/flashfftconv_depthwise_conv1d/
 * conv1d.h:85-104 -> conv1d_bwd_cuda_bhl.cu:19-114); the input half is
 * b200_dwconv1d_fwd with B200_DWCONV1D_FLIP_TAPS. */
size_t b200_dwconv1d_bwd_workspace_bytes(int64_t B, int64_t C, int64_t K, int64_t L_out);
int b200_dwconv1d_bwd_weight(const void* x, const void* dy, void* dw, void* dbias, int dtype,
                             int w_dtype, int64_t B, int64_t C, int64_t L, int64_t K, int64_t pad,
                             int64_t L_out, void* workspace, size_t workspace_bytes,
                             void* stream);

/* GroupNorm backward: dx [N, C, S] (dtype; NULL to skip), dgamma / dbeta [C]
 * (affine_dtype; NULL to skip) of y = (x - mean) * rstd * gamma + beta.
 * stats: (count, mean, M2) per (n, g) of x as written by
 * b200_gn_partial_stats.  gamma NULL = no affine scale.  Reductions in fp32
 * per chunk, fp64 across chunks and channels (fixed order).  workspace: at
 * least b200_gn_bwd_workspace_bytes() bytes.  Replaces the torch-ops
 * derivative _group_norm_backward (amd_tuned_torch/_dispatch.py:2212-2302). */
size_t b200_gn_bwd_workspace_bytes(int64_t N, int64_t C, int64_t S, int64_t G);
int b200_gn_bwd(const void* x, const void* dy, const float* stats, const void* gamma, void* dx,
                void* dgamma, void* dbeta, int dtype, int affine_dtype, int64_t N, int64_t C,
                int64_t S, int64_t G, float eps, void* workspace, size_t workspace_bytes,
                void* stream);

/* ------------------------------------------------------------------ */
/* Dense conv3d (groups = 1) as an implicit GEMM on tcgen05 tensor cores.
 * Replaces _C.conv3d(input, weight, bias?, stride, padding, dilation)
 * (src/main_rocm.cpp:798-854 -> run_conv3d_fp16 :514-548 ->
 * src/cuda/generated/conv3d_fp16_bm256_bn128_bk32_s2.cu:84-380).
 *
 * b200_conv3d_pack_weight: w [Cout, Cin, KD, KH, KW] -> packed
 *   [KD*KH*KW, Cout_pad, Cin_pad] (K-major GEMM B operand, zero padded).
 * b200_conv3d_fwd: x [N, Cin, D, H, W] (x_channels_last = 0) or
 *   [N, D, H, W, Cin] (x_channels_last = 1); y [N, Cout, Do, Ho, Wo] or
 *   channels-last.  params: {stride d,h,w, pad d,h,w, dil d,h,w}.
 *   fp16/bf16, and fp32 through the slab kernel on bf16 hi/lo splits of x
 *   and w (x_hi w_hi + x_lo w_hi + x_hi w_lo, fp32 accumulation and output;
 *   about 16 significant bits kept per operand, rel-L2 ~5e-6 against fp32
 *   on unit-scale data; weights packed by b200_conv3d_pack_weight with
 *   dtype fp32, b200_conv3d_packed_weight_bytes_for bytes).  Two kernels: the box-per-tap kernel (stride 1, Cin a
 *   multiple of 8; scratch = the channels-last copy of an NCDHW x) and the
 *   slab kernel (any stride <= 4, any Cin; scratch = x staged into zero-
 *   padded channels-last phase grids, one per stride phase, so every filter
 *   tap reads the staged rows at a constant offset).  The slab kernel is
 *   chosen for strides and Cin % 8 != 0.  variant bits: 0-3 Cout tile (0 auto, 1/2/3 = 64/128/256),
 *   20 force the slab kernel, 21 never use it, 22 slab kernel without CTA
 *   pairs, 23 (with 20) the workspace already holds x staged by an earlier
 *   call on the same shapes (the staging pass is skipped: for timing the
 *   GEMM alone and for callers that keep the staged layout); the other bits
 *   select box-kernel options (see conv3d_tc.cu).
 * b200_conv3d_fwd_workspace_bytes: scratch b200_conv3d_fwd may need for
 *   this problem (either kernel).
 * b200_conv3d_uses_slab: 1 when b200_conv3d_fwd with this variant runs the
 *   slab kernel (ungated calls), else 0. */
size_t b200_conv3d_packed_weight_bytes(int64_t Cout, int64_t Cin, int64_t KD, int64_t KH,
                                       int64_t KW);
/* Packed size for a weight of `dtype`: fp32 weights pack as three bf16
 * K blocks [hi | hi | lo] per tap (3x the 16-bit size). */
size_t b200_conv3d_packed_weight_bytes_for(int64_t Cout, int64_t Cin, int64_t KD, int64_t KH,
                                           int64_t KW, int dtype);
int b200_conv3d_pack_weight(const void* w, void* wp, int dtype, int64_t Cout, int64_t Cin,
                            int64_t KD, int64_t KH, int64_t KW, void* stream);
size_t b200_conv3d_workspace_bytes(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                                   int x_channels_last);
int b200_conv3d_uses_slab(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                          int64_t Cout, int64_t KD, int64_t KH, int64_t KW,
                          const int64_t* params9, int dtype, int variant);
size_t b200_conv3d_fwd_workspace_bytes(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                                       int64_t KD, int64_t KH, int64_t KW, const int64_t* params9,
                                       int dtype, int x_channels_last);
int b200_conv3d_fwd(const void* x, const void* wp, const void* bias, void* y, int dtype,
                    int bias_dtype, int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                    int64_t Cout, int64_t KD, int64_t KH, int64_t KW, const int64_t* params9,
                    int x_channels_last, int y_channels_last, int variant, void* workspace,
                    size_t workspace_bytes, void* stream);
/* The same call with the per-problem arguments packed once: hosts that call
 * one conv shape repeatedly (the patched F.conv3d after its contest) build a
 * B200Conv3dProblem per shape and pass only the per-call pointers, which
 * keeps the per-call binding cost of a foreign-function interface (ctypes:
 * ~8 us for the 22-argument form) to a few arguments.  Fields mean what the
 * b200_conv3d_fwd arguments of the same names mean; workspace_bytes is the
 * size of `workspace`.  Replaces the same reference call as b200_conv3d_fwd. */
typedef struct B200Conv3dProblem {
  int64_t N, Cin, D, H, W, Cout, KD, KH, KW;
  int64_t params9[9];
  int32_t dtype, bias_dtype, x_channels_last, y_channels_last, variant, reserved;
  uint64_t workspace_bytes;
} B200Conv3dProblem;
int b200_conv3d_fwd_call(const B200Conv3dProblem* problem, const void* x, const void* wp,
                         const void* bias, void* y, void* workspace, void* stream);
/* b200_conv3d_fwd with a halo gate for the T-sharded stack (no reference
 * counterpart): x is a haloed operand whose first and last frames other GPUs
 * write (b200_peer_halo_push).  Tiles of output frame 0 / Do - 1 are
 * scheduled last, and before loading one the producer waits (bounded, fault
 * code 4) until *gate_lo / *gate_hi reach *gate_epoch * gate_scale (u32
 * device words; a NULL counter means that side needs no wait).  With
 * gate_epoch NULL this is b200_conv3d_fwd.  Needs KD = 3, T padding 0,
 * T dilation 1. */
int b200_conv3d_fwd_gated(const void* x, const void* wp, const void* bias, void* y, int dtype,
                          int bias_dtype, int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                          int64_t Cout, int64_t KD, int64_t KH, int64_t KW,
                          const int64_t* params9, int x_channels_last, int y_channels_last,
                          int variant, void* workspace, size_t workspace_bytes,
                          const void* gate_epoch, const void* gate_lo, const void* gate_hi,
                          int64_t gate_scale, void* stream);

/* NCDHW -> channels-last copy ([N, C, S] -> [N, S, C]); conv3d operand layout. */
int b200_to_channels_last(const void* x, void* y, int dtype, int64_t N, int64_t C, int64_t S,
                          void* stream);

/* ------------------------------------------------------------------ */
/* Long-filter depthwise conv1d through the FFT (cross-correlation with a
 * zero-padded transform of length nfft, nfft >= L + 2*pad, nfft in
 * 2^a 3^b 5^c).  Replaces fftconv_ops.fftconv1d_candidate -> fft_conv
 * (amd_tuned_torch/fftconv_ops.py:889-942, :603-746) for groups == C.
 * b200_fftconv1d_prepare: w [C, K] -> spectrum [C, nfft] complex fp32,
 *   conjugated (ready to multiply), in an order private to the kernels that
 *   depends only on nfft: for nfft = 2048, 4096, 8192 and 16384 the
 *   register-resident transform's per-thread order, otherwise the
 *   shared-memory transform's digit-reversed order.  b200_fftconv1d_fwd and
 *   b200_fftconv1d_fwd_os with the same nfft consume it. */
int b200_fft_supported_length(int64_t n);
size_t b200_fftconv1d_spectrum_bytes(int64_t C, int64_t nfft);
int b200_fftconv1d_prepare(const void* w, void* spectrum, int w_dtype, int64_t C, int64_t K,
                           int64_t nfft, void* stream);
int b200_fftconv1d_fwd(const void* x, const void* spectrum, const void* bias, void* y,
                       int dtype, int bias_dtype, int64_t B, int64_t C, int64_t L,
                       int64_t pad, int64_t L_out, int64_t nfft, void* stream);
/* Overlap-save form: the row is cut into segments of nfft - K + 1 outputs,
 * each one transform of length nfft >= K over inputs [start - pad, + nfft)
 * (one transform per channel, row pair and segment); spectrum from
 * b200_fftconv1d_prepare with the same nfft.  L_out = L + 2*pad - K + 1.
 * Same result as b200_fftconv1d_fwd (same fft_conv semantics), with short
 * transforms that several CTAs per SM can hold. */
int b200_fftconv1d_fwd_os(const void* x, const void* spectrum, const void* bias, void* y,
                          int dtype, int bias_dtype, int64_t B, int64_t C, int64_t L, int64_t K,
                          int64_t pad, int64_t L_out, int64_t nfft, void* stream);

/* Dense (groups = 1) conv3d through the FFT for large kernels:
 * rfft3(x) . conj(rfft3(w)) summed over Cin per frequency bin, irfft3,
 * crop, + bias.  Replaces fftconv_ops.fft_conv3d (fftconv_ops.py:749-781)
 * with complex_matmul (:480-543).  Transform extents (fd, fh, fw) are
 * chosen by the caller (fw even).
 * b200_fftconv3d_prepare: w [Cout, Cin, KD, KH, KW] -> conjugated spectrum:
 *   a 256-byte header (fp32 scale s at offset 0) followed by [bins][Cin][Cout]
 *   complex values s * conj(W), bins = fd*fh*(fw/2+1), 16-byte aligned.  fp32
 *   weights: complex fp32, s = 1.  fp16 / bf16 weights: complex fp16 (re, im),
 *   s the power of two with s * max|w| * KD*KH*KW <= 2^15 (half the bytes the
 *   contraction streams per call).  b200_fftconv3d_fwd must be called with
 *   dtype == the w_dtype the spectrum was prepared with.
 * Workspace: input spectrum [bins][N][Cin] + output spectrum [bins][N][Cout]
 *   + a real staging volume. */
size_t b200_fftconv3d_spectrum_bytes(int64_t Cout, int64_t Cin, int64_t fd, int64_t fh,
                                     int64_t fw, int w_dtype);
int b200_fftconv3d_prepare(const void* w, void* spectrum, int w_dtype, int64_t Cout,
                           int64_t Cin, int64_t KD, int64_t KH, int64_t KW, int64_t fd,
                           int64_t fh, int64_t fw, void* workspace, size_t workspace_bytes,
                           void* stream);
size_t b200_fftconv3d_workspace_bytes(int64_t N, int64_t Cin, int64_t Cout, int64_t fd,
                                      int64_t fh, int64_t fw);
int b200_fftconv3d_fwd(const void* x, const void* spectrum, const void* bias, void* y,
                       int dtype, int bias_dtype, int64_t N, int64_t Cin, int64_t D,
                       int64_t H, int64_t W, int64_t Cout, int64_t KD, int64_t KH, int64_t KW,
                       const int64_t* pad3, int64_t fd, int64_t fh, int64_t fw,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ */
/* Peer-memory exchange of the T-sharded conv stack (one process per GPU).
 * No counterpart in the reference (it is single-GPU); these replace the
 * NCCL all-gather of GroupNorm partial statistics and the NCCL send/recv of
 * halo frames with stores into the peers' memory over NVLink, ordered by
 * flags that bounded device waits poll.
 *
 * A window is one device allocation per rank, mapped into every other rank
 * with CUDA IPC:
 *   [control | statistics flags | halo arrival counters |
 *    statistics slots [2][ranks][entries * 3] fp32 | pad | xp]
 * where xp is the rank's haloed channels-last conv operand
 * [N, T_local + 2, H, W, C] at b200_peer_window_xp_offset().  Every rank
 * uses the same ranks / entries, so the offsets below xp agree.
 *
 * Per block, in stream order on every rank:
 *   b200_peer_stats_publish  advances the window's epoch e and stores this
 *                            rank's (count, mean, M2) triples into slot
 *                            [e & 1][rank] of every window, then raises
 *                            flag [e & 1][rank] = e in each;
 *   b200_peer_stats_merge    waits for flags [e & 1][*] == e in the local
 *                            window and merges the slots in rank order (fp64,
 *                            Chan) -- identical statistics on every rank;
 *   (GroupNorm apply writes the xp interior)
 *   b200_peer_halo_push      copies the first interior frame(s) into the
 *                            previous rank's top halo and the last into the
 *                            next rank's bottom halo, then adds 1 per CTA to
 *                            the receiver's arrival counter;
 *   b200_peer_halo_wait      waits until the local counters reach
 *                            e * B200_PEER_PUSH_CTAS.
 * Two slot parities suffice: a rank cannot publish block e + 2 before every
 * rank has merged block e (it needs their block e + 1 statistics, computed
 * after their merge of e).  One xp buffer suffices for the same reason.
 * Every wait gives up after 2 s, records code 3 (statistics) or 4 (halo) in
 * the device fault word (b200_read_device_flags) and returns; the merge then
 * writes NaN statistics so that a broken exchange cannot pass unnoticed. */
#define B200_PEER_MAX_RANKS 64
#define B200_PEER_HANDLE_BYTES 64
#define B200_PEER_PUSH_CTAS 64
int64_t b200_peer_window_xp_offset(int64_t ranks, int64_t entries);
int64_t b200_peer_window_bytes(int64_t ranks, int64_t entries, int64_t xp_bytes);
/* cudaMalloc + zero fill + IPC handle (B200_PEER_HANDLE_BYTES into `handle`). */
int b200_peer_window_alloc(int64_t bytes, void** window, void* handle);
/* Maps a peer's window (cudaIpcOpenMemHandle); b200_peer_window_close unmaps. */
int b200_peer_window_open(const void* handle, void** window);
int b200_peer_window_close(void* window);
int b200_peer_window_free(void* window);
/* windows: DEVICE array of `ranks` window addresses as seen by this process
 * (windows[rank] = the local window). */
int b200_peer_stats_publish(const float* stats, void* const* windows, int64_t ranks,
                            int64_t rank, int64_t entries, void* local_window, void* stream);
int b200_peer_stats_merge(void* local_window, float* out, int64_t ranks, int64_t entries,
                          void* stream);
/* Side "lo" sends `items` blocks of `bytes` from src_lo (+ i * src_lo_stride)
 * to dst_lo (+ i * dst_lo_stride) inside window `lo_window` (the previous
 * rank's) and counts the arrival there; "hi" likewise to the next rank.
 * A side with a NULL window is skipped.  bytes and strides are multiples of
 * 16, pointers 16-byte aligned. */
int b200_peer_halo_push(void* local_window, const void* src_lo, void* dst_lo, void* lo_window,
                        int64_t src_lo_stride, int64_t dst_lo_stride, const void* src_hi,
                        void* dst_hi, void* hi_window, int64_t src_hi_stride,
                        int64_t dst_hi_stride, int64_t items, int64_t bytes, void* stream);
/* expect_lo: the previous rank pushes into this window (bottom halo);
 * expect_hi: the next rank does (top halo). */
int b200_peer_halo_wait(void* local_window, int expect_lo, int expect_hi, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200CONV_H */
