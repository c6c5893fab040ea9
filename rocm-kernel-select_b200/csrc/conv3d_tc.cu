// Dense conv3d (groups = 1, stride 1, any padding/dilation) as an implicit
// GEMM on the sm_100a tensor cores.
//
// Reference role: custom_conv3d_forward -> run_conv3d_fp16 ->
// conv3d_fp16_kernel_bm256_bn128_bk32_s2 (src/main_rocm.cpp:798-854, :514-548;
// src/cuda/generated/conv3d_fp16_bm256_bn128_bk32_s2.cu:84-380), an rocWMMA
// implicit GEMM with M = N*Do*Ho*Wo, N = Cout, K = Cin*KD*KH*KW, fp32
// accumulation and a bias epilogue.  Same GEMM view here, built for Blackwell:
//
//  * Operand A comes from a channels-last copy of the input ([N, D, H, W, C],
//    made by b200_to_channels_last or the fused GroupNorm producer).  For
//    every filter tap (kd, kh, kw) and 64-channel chunk, ONE TMA tiled load
//    fetches the box {64 channels, BW, BH, 1, 1} at the tap-shifted output
//    coordinates.  The innermost coordinate is the channel offset (a multiple
//    of 64, so always 16-byte aligned); the spatial shift lands on W/H/D,
//    which carry no alignment rule, and the padding is the TMA zero fill of
//    out-of-range coordinates.  The 128 rows of the box are the 128 output
//    positions of the tile, each a 128-byte K-major row, SWIZZLE_128B.
//  * Operand B is the weight packed as [tap][Cout][Cin_pad] (K-major), one
//    TMA box {64, BN, 1} per k-block.
//  * tcgen05.mma (kind::f16, M = 128, N = BN, K = 16) issued by one thread,
//    fp32 accumulators in TMEM, double-buffered so the epilogue of tile i
//    overlaps the MMAs of tile i + 1 in a persistent CTA.
//  * Warp roles (6 warps): 0 = TMA producer, 1 = MMA issuer (+ TMEM
//    allocation), 2-5 = epilogue (tcgen05.ld -> + bias -> fp16/bf16 store,
//    NCDHW or channels-last).
//  * Every mbarrier wait is bounded (kWaitLimitNs); running out records a
//    fault code and unwinds: the MMA thread drains its in-flight MMAs through
//    a final commit before TMEM is released.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "conv3d_slab.cuh"
#include "sm100_ptx.cuh"

namespace b200 {
namespace {

constexpr int kConvThreads = 192;       // 6 warps
constexpr int kBM = 128;
constexpr int kBK = 64;            // weight packing granule: Cin is padded to a multiple of 64
constexpr int kMaxStages = 8;

struct ConvParams {
  int Do, Ho, Wo, Cout;
  int KH, KW;
  int pd, ph, pw, dd, dh, dw;
  int BW, BH;
  int MT;                       // M tiles (of 128 positions) per CTA tile, stacked along H
  int pair;                     // CTA pairs (cta_group::2): a tile is 2 x MT M tiles
  int tiles_w, tiles_h, tiles_n, num_tiles;
  int cchunks, kblocks;
  int khg, khb;                 // kh taps per k-block (1 or KH), kh blocks = KH / khg
  int a_bytes, stage_bytes, stages;
  int rotate;
  void* y;
  const void* bias;
  int bias_dt;
  int y_cl;
  int out_tma;
  int* flags;
  // Halo gate (T-sharded stack): output frame 0 reads input frame 0 and
  // frame Do - 1 reads frame Do + 1, which other GPUs write.  Before loading
  // a tile of such a frame the producer waits until *gate_lo / *gate_hi
  // (arrival counters, NULL = no wait) reach *gate_epoch * gate_scale; the
  // tile order puts those frames last.  gate_epoch NULL = no gate.
  int Nb;
  const uint32_t* gate_epoch;
  const uint32_t* gate_lo;
  const uint32_t* gate_hi;
  uint32_t gate_scale;
};

struct TileCoord {
  int n, od, oh0, ow0, n0;
  uint32_t lin;   // schedule-independent tile id (n, od, th, tw, nt order)
};

__device__ __forceinline__ TileCoord decode_tile(int t, const ConvParams& p, int BN) {
  TileCoord c;
  const int nt = t % p.tiles_n;
  t /= p.tiles_n;
  const int tw = t % p.tiles_w;
  t /= p.tiles_w;
  const int th = t % p.tiles_h;
  t /= p.tiles_h;
  if (p.gate_epoch) {
    // (n, od) pairs: interior frames first, then the gated frames 0, Do - 1.
    const int inner = p.Do > 2 ? p.Do - 2 : 0;
    const int I = p.Nb * inner;
    if (t < I) {
      c.n = t / inner;
      c.od = 1 + t % inner;
    } else {
      const int B = p.Do < 2 ? p.Do : 2;
      const int j = t - I;
      c.n = j / B;
      c.od = (j % B) ? p.Do - 1 : 0;
    }
  } else {
    c.od = t % p.Do;
    c.n = t / p.Do;
  }
  c.lin = ((((static_cast<uint32_t>(c.n) * p.Do + c.od) * p.tiles_h + th) * p.tiles_w + tw) *
           p.tiles_n) + nt;
  c.oh0 = th * p.BH * p.MT * (p.pair ? 2 : 1);
  c.ow0 = tw * p.BW;
  c.n0 = nt * BN;
  return c;
}

// Waits (bounded) until the halo frames output frame `od` reads have arrived;
// false (fault code 4 recorded) when the wait runs out.  The proxy fence
// orders the peers' generic stores before this CTA's TMA reads of them.
__device__ bool halo_gate_wait(const ConvParams& p, int od) {
  const uint32_t target =
      *reinterpret_cast<const volatile uint32_t*>(p.gate_epoch) * p.gate_scale;
  const uint64_t t0 = globaltimer_ns();
  for (int side = 0; side < 2; ++side) {
    const uint32_t* c = side == 0 ? (od == 0 ? p.gate_lo : nullptr)
                                  : (od == p.Do - 1 ? p.gate_hi : nullptr);
    if (!c) continue;
    while (!counter_reached(ld_acquire_sys(c), target)) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (p.flags) atomicExch(p.flags, 4);
        return false;
      }
      __nanosleep(64);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// MT: M tiles per CTA tile (1, 2 or 4); they share every weight box and the
// A rows of neighbouring taps.  KB: channels per k-block -- 64 (128-byte
// K-major rows, SWIZZLE_128B) or 32 (64-byte rows, SWIZZLE_64B, half the
// stage size so that MT = 4 still leaves three stages).
//
// PAIR: a cluster of two CTAs on two SMs computes 2 x MT M tiles with MMAs
// of M = 256 (tcgen05 cta_group::2): each CTA loads its own A rows and HALF
// of the weight box (BN / 2 output channels), so the pair streams the
// weights once instead of twice.  The even CTA (leader) issues the MMAs;
// both producers' copies count on the leader's stage barriers; the leader's
// MMA completions are committed to both CTAs' barriers; each CTA's epilogue
// drains its own TMEM and tells the leader (one arrival per warp).
template <typename T, int BN, int MT, int KB, bool PAIR = false>
__global__ void __launch_bounds__(kConvThreads, 1)
conv3d_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                 const __grid_constant__ CUtensorMap tmy, const ConvParams p) {
  static_assert(KB == 64 || KB == 32, "k-block of 32 or 64 channels");
  constexpr int kRow = KB * 2;               // bytes per K-major operand row
  constexpr int kBNl = PAIR ? BN / 2 : BN;   // weight rows (output channels) this CTA loads
  constexpr int kBTap = kBNl * kRow;         // this CTA's share of one tap's weight box
  constexpr int kAcc = MT * BN;              // TMEM columns of one tile's accumulators
  constexpr int kBufs = (2 * kAcc <= 512) ? 2 : 1;
  constexpr uint32_t kTmemCols = kBufs * kAcc < 32 ? 32u : static_cast<uint32_t>(kBufs * kAcc);
  static_assert(kBufs * kAcc <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM columns");
  constexpr uint32_t kIdesc = umma_idesc_f16(sizeof(T) == 2 && std::is_same<T, __half>::value ? 0 : 1,
                                             PAIR ? 2 * kBM : kBM, BN);
  const int STAGES = p.stages;
  // Tile walk: per CTA, or per CTA pair (both CTAs walk the same tiles).
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const int tile0 = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int tstep = PAIR ? static_cast<int>(nclusters_x()) : static_cast<int>(gridDim.x);
  const bool leader = crank == 0u;
  const int oh_rank = PAIR ? static_cast<int>(crank) * p.BH * MT : 0;   // this CTA's first row

  // Stage s = [A box: a_bytes][B boxes: khg * kBTap], every piece 1024-byte
  // aligned, then the output staging tile (present when out_tma is set).
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sOut = smem + STAGES * p.stage_bytes;                   // [BN][128] staging
  float* sBias = reinterpret_cast<float*>(sOut + (p.out_tma ? kBM * BN * 2 : 0));  // [BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(sBias + BN + 4);   // + 16-byte scratch
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;  // [2]
  uint64_t* tempty = tfull + 2;      // [2]
  uint64_t* drain = tempty + 2;      // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmx);
    prefetch_tmap(&tmw);
    if (p.out_tma) prefetch_tmap(&tmy);
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      // PAIR: one arrival per epilogue warp of both CTAs (on the leader's).
      mbar_init(&tempty[a], PAIR ? 8 : 128);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if (PAIR)
      tmem_alloc_pair(tmem_slot, kTmemCols);
    else
      tmem_alloc(tmem_slot, kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  // Both CTAs' barriers exist before either CTA touches the other's.
  if (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialisation: everything above (barrier
  // set-up, TMEM allocation, descriptor prefetch) overlaps the previous
  // kernel; no global memory is touched before it has completed.
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    // The whole warp walks the loop (waits included) so it stays converged;
    // one lane issues the copies.
    {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // k-block = (kd, kh block, kw, 64-channel chunk).  One A box of
      // BH + (khg - 1) * dh input rows serves the khg kh-taps of the block
      // (tap j reads the rows starting j * dh rows down); one weight box per
      // tap.  Neighbouring tiles start their K walk at different k-blocks:
      // CTAs in lockstep would all fetch the same weight box at once (an L2
      // hot spot).  The start depends on the tile, not on the CTA, so a
      // tile's accumulation order (and its rounding) is the same whatever
      // the schedule or grid.
      for (int t = tile0; t < p.num_tiles && ok; t += tstep) {
        const TileCoord tc = decode_tile(t, p, BN);
        // Both CTAs of a pair walk the k-blocks in the same order (the
        // rotation depends on the tile only): stage s holds the same k-block
        // in both.
        const int rot = p.rotate ? static_cast<int>((tc.lin * 7u) % p.kblocks) : 0;
        if (p.gate_epoch && (tc.od == 0 || tc.od == p.Do - 1)) {
          int open = 1;
          if (lane == 0) open = halo_gate_wait(p, tc.od) ? 1 : 0;
          open = __shfl_sync(0xffffffffu, open, 0);
          if (!open) {
            if (lane == 0) *abort = 1;
            ok = false;
            break;
          }
        }
        for (int kk = 0; kk < p.kblocks; ++kk) {
          int kb = kk + rot;
          if (kb >= p.kblocks) kb -= p.kblocks;
          const int cc = kb % p.cchunks;
          int r = kb / p.cchunks;
          const int kw = r % p.KW;
          r /= p.KW;
          const int hb = r % p.khb, kd = r / p.khb;
          const bool got = mbar_wait_bounded(&empty[stage], phase ^ 1u, abort, p.flags, 1);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            uint8_t* st = smem + stage * p.stage_bytes;
            if (PAIR) {
              // The leader's barrier counts both CTAs' bytes; only the leader
              // arrives on it.
              if (leader) mbar_expect_tx(&full[stage], 2u * static_cast<uint32_t>(p.stage_bytes));
              const uint32_t fb = mapa_u32(&full[stage], 0);
              tma_load_5d_pair(st, &tmx, fb, cc * KB, tc.ow0 - p.pw + kw * p.dw,
                               tc.oh0 + oh_rank - p.ph + hb * p.khg * p.dh,
                               tc.od - p.pd + kd * p.dd, tc.n);
              for (int j = 0; j < p.khg; ++j) {
                const int tap = (kd * p.KH + hb * p.khg + j) * p.KW + kw;
                tma_load_3d_pair(st + p.a_bytes + j * kBTap, &tmw, fb, cc * KB,
                                 tc.n0 + static_cast<int>(crank) * kBNl, tap);
              }
            } else {
              mbar_expect_tx(&full[stage], p.stage_bytes);
              tma_load_5d(st, &tmx, &full[stage], cc * KB, tc.ow0 - p.pw + kw * p.dw,
                          tc.oh0 - p.ph + hb * p.khg * p.dh, tc.od - p.pd + kd * p.dd, tc.n);
              for (int j = 0; j < p.khg; ++j) {
                const int tap = (kd * p.KH + hb * p.khg + j) * p.KW + kw;
                tma_load_3d(st + p.a_bytes + j * kBTap, &tmw, &full[stage], cc * KB, tc.n0, tap);
              }
            }
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && lane == 0 && leader) {
        // Let the loads already issued land before shared memory goes away
        // (a pair's loads all count on the leader's barriers).
        const int last = (stage + STAGES - 1) % STAGES;
        mbar_wait_bounded(&full[last], (stage == 0 ? phase ^ 1u : phase), nullptr, nullptr, 0);
      }
      __syncwarp();
    }
  } else if (warp == 1 && PAIR && !leader) {
    // The pair's MMAs are issued by the leader only.
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer
    // Converged warp; lane 0 issues the MMAs and commits.
    {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = tile0; t < p.num_tiles && ok; t += tstep, ++it) {
        const int acc = kBufs == 2 ? (it & 1) : 0;
        const uint32_t aphase = static_cast<uint32_t>(kBufs == 2 ? (it >> 1) : it) & 1u;
        const bool free_acc = mbar_wait_bounded(&tempty[acc], aphase ^ 1u, abort, p.flags, 1);
        if (!__all_sync(0xffffffffu, free_acc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kAcc);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          const bool got = mbar_wait_bounded(&full[stage], phase, abort, p.flags, 1);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint8_t* st = smem + stage * p.stage_bytes;
            // One input row of the box = BW positions x kRow bytes.
            const uint32_t row_bytes = static_cast<uint32_t>(p.BW * kRow);
            for (int j = 0; j < p.khg; ++j) {
              const uint32_t b_addr = smem_u32(st + p.a_bytes + j * kBTap);
              const uint64_t bdesc = KB == 64 ? umma_desc_sw128(b_addr) : umma_desc_sw64(b_addr);
#pragma unroll
              for (int i = 0; i < MT; ++i) {
                // M tile i of tap j: its A rows start i * BH + j * dh input
                // rows down (BW >= 8, so a whole number of 8-row swizzle
                // atoms); the weight box is shared by the MT tiles.
                const uint32_t a_addr =
                    smem_u32(st) + static_cast<uint32_t>(i * p.BH + j * p.dh) * row_bytes;
                const uint64_t adesc = KB == 64 ? umma_desc_sw128(a_addr) : umma_desc_sw64(a_addr);
#pragma unroll
                for (int k = 0; k < KB / 16; ++k) {
                  // +32 bytes along K inside the swizzled row = +2 in the
                  // descriptor's address field.
                  const uint32_t accum = (kb > 0 || j > 0 || k > 0) ? 1u : 0u;
                  if (PAIR)
                    umma_f16_ss_pair(d_tmem + static_cast<uint32_t>(i * BN),
                                     adesc + static_cast<uint64_t>(2 * k),
                                     bdesc + static_cast<uint64_t>(2 * k), kIdesc, accum);
                  else
                    umma_f16_ss(d_tmem + static_cast<uint32_t>(i * BN),
                                adesc + static_cast<uint64_t>(2 * k),
                                bdesc + static_cast<uint64_t>(2 * k), kIdesc, accum);
                }
              }
            }
            if (PAIR) {
              // The stage is free in both CTAs once these MMAs are done.
              umma_commit_pair(smem_u32(&empty[stage]));
              umma_commit_pair(mapa_u32(&empty[stage], 1));
            } else {
              umma_commit(&empty[stage]);
            }
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok && lane == 0) {
          if (PAIR) {
            umma_commit_pair(smem_u32(&tfull[acc]));
            umma_commit_pair(mapa_u32(&tfull[acc], 1));
          } else {
            umma_commit(&tfull[acc]);
          }
        }
        __syncwarp();
      }
      // Drain: every MMA issued above has completed once `drain` flips.
      if (lane == 0) {
        if (PAIR)
          umma_commit_pair(smem_u32(drain));
        else
          umma_commit(drain);
      }
      __syncwarp();
      mbar_wait_bounded(drain, 0, nullptr, nullptr, 0);
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------- epilogue
    // TMEM -> registers (+ bias) -> either a shared staging tile written by
    // one TMA tensor store (NCDHW output whose rows TMA can address), or
    // direct global stores.  Warps 2-5 synchronise on named barrier 1.
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;
    const int etid = threadIdx.x - 64;
    int it = 0;
    T* y = static_cast<T*>(p.y);
    uint16_t* stage16 = reinterpret_cast<uint16_t*>(sOut);
    const int64_t plane = static_cast<int64_t>(p.Ho) * p.Wo;
    for (int t = tile0; t < p.num_tiles; t += tstep, ++it) {
      const int acc = kBufs == 2 ? (it & 1) : 0;
      const uint32_t aphase = static_cast<uint32_t>(kBufs == 2 ? (it >> 1) : it) & 1u;
      // All 128 threads leave together or not at all (a named barrier
      // follows); the vote also orders this tile after the previous tile's
      // readers of sBias / staging.
      const bool got = mbar_wait_bounded(&tfull[acc], aphase, abort, p.flags, 1);
      if (!epi_bar_and(got)) break;
      tc_fence_after();
      const TileCoord tc = decode_tile(t, p, BN);
      for (int j = etid; j < BN; j += 128) {
        const int co = tc.n0 + j;
        sBias[j] = (p.bias && co < p.Cout) ? load_param(p.bias, p.bias_dt, co) : 0.f;
      }
      if (p.out_tma && etid == 0) bulk_wait_read0();  // staging free again
      epi_bar();
#pragma unroll 1
      for (int i = 0; i < MT; ++i) {
        if (i > 0 && p.out_tma) {
          if (etid == 0) bulk_wait_read0();
          epi_bar();
        }
        const int oh0 = tc.oh0 + oh_rank + i * p.BH;
        const int oh = oh0 + row / p.BW, ow = tc.ow0 + row % p.BW;
        const bool valid = oh < p.Ho && ow < p.Wo;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(acc * kAcc + i * BN);
        const int64_t pos = (static_cast<int64_t>(tc.od) * p.Ho + oh) * p.Wo + ow;
#pragma unroll 1
        for (int j0 = 0; j0 < BN; j0 += 32) {
          float v0[16], v1[16], v[32];
          tmem_ld16(taddr + j0, v0);
          tmem_ld16(taddr + j0 + 16, v1);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = (j < 16 ? v0[j] : v1[j - 16]) + sBias[j0 + j];
          if (p.out_tma) {
#pragma unroll
            for (int j = 0; j < 32; ++j) stage16[(j0 + j) * kBM + row] = f32_to_bits16<T>(v[j]);
          } else if (valid && p.y_cl) {
            T* dst = y + (static_cast<int64_t>(tc.n) * p.Do * plane + pos) * p.Cout + tc.n0 + j0;
            const bool vec = tc.n0 + j0 + 32 <= p.Cout && (p.Cout & 7) == 0;
            if (vec) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = v[8 * q + e];
                *reinterpret_cast<uint4*>(dst + 8 * q) = pack16<T>(f);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (tc.n0 + j0 + j < p.Cout) dst[j] = from_f32<T>(v[j]);
            }
          } else if (valid) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int co = tc.n0 + j0 + j;
              if (co < p.Cout)
                y[((static_cast<int64_t>(tc.n) * p.Cout + co) * p.Do) * plane + pos] =
                    from_f32<T>(v[j]);
            }
          }
        }
        if (i == MT - 1) {
          // Accumulators drained: the MMA warp may reuse them.
          tc_fence_before();
          if (PAIR) {
            __syncwarp();
            if (lane == 0) {
              if (leader)
                mbar_arrive(&tempty[acc]);
              else
                mbar_arrive_remote(mapa_u32(&tempty[acc], 0));
            }
          } else {
            mbar_arrive(&tempty[acc]);
          }
        }
        if (p.out_tma) {
          fence_proxy_async();        // staging writes -> visible to the TMA engine
          epi_bar();
          if (etid == 0) {
            tma_store_5d(&tmy, sOut, tc.ow0, oh0, tc.od, tc.n0, tc.n);
            bulk_commit();
          }
        }
      }
    }
    if (p.out_tma && etid == 0) bulk_wait_all0();
  }

  tc_fence_before();
  __syncthreads();
  // A pair's CTAs exchange barrier arrivals until the end: neither leaves
  // (and gives up its shared memory) before the other is done.
  if (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

// --------------------------------------------------------- weight packing ---
// w [Cout][Cin][taps] -> wp [taps][Cout][Cin_pad], zero beyond Cin.
template <typename T>
__global__ void pack_weight_kernel(const T* __restrict__ w, T* __restrict__ wp, int64_t Cout,
                                   int64_t Cin, int64_t Cin_pad, int64_t taps) {
  const int64_t total = taps * Cout * Cin_pad;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t ci = i % Cin_pad;
    const int64_t co = (i / Cin_pad) % Cout;
    const int64_t tap = i / (Cin_pad * Cout);
    wp[i] = ci < Cin ? w[(co * Cin + ci) * taps + tap] : from_f32<T>(0.f);
  }
}

// ------------------------------------------------------ NCDHW -> N[S]C ---
// 16-bit elements, 64 channels x 64 positions per CTA: 16-byte loads along
// the positions of a channel row, 16-byte stores along the channels of a
// position.  Shared rows are 66 elements (33 words) so both the 32-bit
// writes and the 8-channel column gathers spread over the banks.
template <typename T>
__global__ void __launch_bounds__(256)
to_cl16_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t C, int64_t S) {
  static_assert(sizeof(T) == 2, "16-bit elements");
  __shared__ uint32_t tile[64 * 33];
  // Launched with programmatic serialisation behind the previous kernel
  // (which may still read the workspace this copy writes): wait for it first.
  pdl_wait();
  pdl_launch_dependents();  // the conv kernel's prologue may overlap this copy
  const int64_t n = blockIdx.z;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 64;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int v = threadIdx.x & 7;
  const bool full = (c0 + 64 <= C) && (p0 + 64 <= S);
  for (int r = threadIdx.x >> 3; r < 64; r += 32) {
    const int64_t c = c0 + r;
    uint4 q = make_uint4(0, 0, 0, 0);
    const int64_t p = p0 + 8 * v;
    const T* src = x + (n * C + c) * S + p;
    if (full && (S & 7) == 0) {
      q = ld_stream16(src);
    } else if (c < C) {
      uint16_t e[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        e[k] = (p + k < S) ? reinterpret_cast<const uint16_t*>(src)[k] : uint16_t(0);
      q = make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16),
                     e[4] | (uint32_t(e[5]) << 16), e[6] | (uint32_t(e[7]) << 16));
    }
    uint32_t* row = tile + r * 33 + 4 * v;
    row[0] = q.x;
    row[1] = q.y;
    row[2] = q.z;
    row[3] = q.w;
  }
  __syncthreads();
  const uint16_t* t16 = reinterpret_cast<const uint16_t*>(tile);
  for (int qp = threadIdx.x >> 3; qp < 64; qp += 32) {
    const int64_t p = p0 + qp;
    if (p >= S) continue;
    uint16_t e[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = t16[(8 * v + k) * 66 + qp];
    T* dst = y + (n * S + p) * C + c0 + 8 * v;
    if (full && (C & 7) == 0) {
      *reinterpret_cast<uint4*>(dst) =
          make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16),
                     e[4] | (uint32_t(e[5]) << 16), e[6] | (uint32_t(e[7]) << 16));
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (c0 + 8 * v + k < C) reinterpret_cast<uint16_t*>(dst)[k] = e[k];
    }
  }
}

// Generic element type (fp32): 64 x 64 tile of scalars.
template <typename T>
__global__ void __launch_bounds__(256)
to_cl_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t C, int64_t S) {
  __shared__ T tile[64][66];
  pdl_wait();  // as to_cl16_kernel
  pdl_launch_dependents();
  const int64_t n = blockIdx.z;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 64;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  for (int cc = ty; cc < 64; cc += 4) {
    const int64_t c = c0 + cc, q = p0 + tx;
    tile[cc][tx] = (c < C && q < S) ? x[(n * C + c) * S + q] : from_f32<T>(0.f);
  }
  __syncthreads();
  for (int pp = ty; pp < 64; pp += 4) {
    const int64_t q = p0 + pp, c = c0 + tx;
    if (q < S && c < C) y[(n * S + q) * C + c] = tile[tx][pp];
  }
}

// ------------------------------------------------------------ host side ---
// Shared memory besides the stages: output staging (when the output goes out
// through TMA stores), bias, barriers, and the slack for aligning the dynamic
// base to 1024 bytes.
constexpr size_t fixed_smem(int BN, bool staging) {
  return (staging ? static_cast<size_t>(kBM) * BN * 2 : 0) + BN * 4 + 16 + (2 * kMaxStages + 9) * 8 +
         8 + 1024;
}
constexpr size_t kSmemBudget = 232448;  // sm_100 opt-in maximum per CTA

template <typename T, int BN, int MT, int KB, bool PAIR = false>
int launch_conv(const CUtensorMap& tmx, const CUtensorMap& tmw, const CUtensorMap& tmy,
                const ConvParams& prm, bool staging, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(prm.stages) * prm.stage_bytes + fixed_smem(BN, staging);
  if (smem > kSmemBudget) return fail_unsupported("conv3d stage geometry exceeds shared memory");
  if (prm.out_tma && !staging) return fail_arg("conv3d TMA output without staging");
  auto kern = conv3d_tc_kernel<T, BN, MT, KB, PAIR>;
  B200_CUDA_CHECK(
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  // Pairs: clusters of two CTAs, one tile per cluster per turn.
  const int grid = PAIR ? 2 * std::min(prm.num_tiles, std::max(1, sm_count() / 2))
                        : std::min(prm.num_tiles, sm_count());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kConvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = PAIR ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 2 : 1;
  B200_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tmx, tmw, tmy, prm));
  return B200_OK;
}

int pick_bn(int64_t Cout, int code) {
  if (code == 1) return 64;
  if (code == 2) return 128;
  if (code == 3) return 256;
  if (Cout <= 64) return 64;
  if (Cout <= 128) return 128;
  return 256;
}

struct HaloGate {
  const uint32_t* epoch;
  const uint32_t* lo;
  const uint32_t* hi;
  uint32_t scale;
};

// Whether b200_conv3d_fwd takes the slab path: variant bit 20 forces it and
// bit 21 rules it out; otherwise only strides and channel counts that are
// not a multiple of 8, which only it handles.  (On stride-1 problems it is
// not faster than the box kernel: with 64 output channels both are bound by
// the operand bytes every M = 128, N = 64 MMA reads from shared memory, and
// its staging pass and 13% of discarded rows cost more than the input bytes
// it saves; the kernel_select contest times both where both apply.)  Never
// with a halo gate.
bool slab_wanted(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t Cout,
                 int64_t KD, int64_t KH, int64_t KW, const int64_t* prm9, int variant,
                 bool gated) {
  (void)N, (void)D, (void)H, (void)W, (void)Cout, (void)KD, (void)KH, (void)KW;
  if (gated || ((variant >> 21) & 1) != 0) return false;
  if (((variant >> 20) & 1) != 0) return true;
  return prm9[0] != 1 || prm9[1] != 1 || prm9[2] != 1 || Cin % 8 != 0;
}

template <typename T>
int conv3d_typed(const void* x, const void* wp, const void* bias, void* y, int bias_dt,
                 int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t Cout,
                 int64_t KD, int64_t KH, int64_t KW, const int64_t* prm9, int x_cl, int y_cl,
                 int variant, void* ws, size_t ws_bytes, cudaStream_t stream,
                 const HaloGate* gate) {
  const int64_t sd = prm9[0], sh = prm9[1], sw = prm9[2];
  const int64_t pd = prm9[3], ph = prm9[4], pw = prm9[5];
  const int64_t dd = prm9[6], dh = prm9[7], dw = prm9[8];
  if (pd < 0 || ph < 0 || pw < 0 || dd < 1 || dh < 1 || dw < 1) return fail_arg("bad padding/dilation");
  if (sd < 1 || sh < 1 || sw < 1) return fail_arg("bad stride");
  // Slab path (conv3d_slab.cu): strides, any channel count, and the small
  // problems where one tile per SM leaves the box kernel latency-bound.
  if (slab_wanted(N, Cin, D, H, W, Cout, KD, KH, KW, prm9, variant, gate && gate->epoch)) {
    const bool only = ((variant >> 20) & 1) != 0 || sd != 1 || sh != 1 || sw != 1 || Cin % 8 != 0;
    const int rc = conv3d_slab<T>(x, wp, bias, y, bias_dt, N, Cin, D, H, W, Cout, KD, KH, KW,
                                  prm9, x_cl, y_cl, variant & 0xF, ((variant >> 22) & 1) == 0,
                                  ((variant >> 23) & 1) != 0, ws, ws_bytes, stream);
    if (rc <= 0 || only) return rc;
  }
  if (sd != 1 || sh != 1 || sw != 1) return fail_unsupported("conv3d tensor-core path: stride != 1");
  if (Cin % 8 != 0) return fail_unsupported("conv3d tensor-core path: Cin % 8 != 0");
  const int64_t Do = D + 2 * pd - dd * (KD - 1);
  const int64_t Ho = H + 2 * ph - dh * (KH - 1);
  const int64_t Wo = W + 2 * pw - dw * (KW - 1);
  if (Do <= 0 || Ho <= 0 || Wo <= 0) return fail_arg("conv3d output size must be positive");
  const int64_t lim = 1LL << 30;
  if (N >= 65536 || D >= lim || H >= lim || W >= lim || Cout >= lim || Cin >= lim)
    return fail_unsupported("conv3d size out of range");
  auto encode = tensor_map_encoder();
  if (!encode) return fail_unsupported("cuTensorMapEncodeTiled unavailable");

  if (!aligned16(wp)) return fail_unsupported("operands not 16-byte aligned");

  if (((variant >> 14) & 3) != 0) return fail_arg("conv3d variant bits 14-15 are not defined");
  const int BN = pick_bn(Cout, variant & 0xF);
  int BW;
  const int bw_code = (variant >> 4) & 0xF;
  if (bw_code) {
    BW = 1 << bw_code;
    if (BW > 128) return fail_arg("conv3d tile width code");
  } else {
    BW = 8;
    while (BW < Wo && BW < 128) BW *= 2;
  }
  if (BW < 8) return fail_arg("conv3d tile width must be >= 8");
  const int BH = kBM / BW;
  const int64_t taps = KD * KH * KW;
  const int64_t Cin_pad = (Cin + kBK - 1) / kBK * kBK;   // packed weight row length
  const int64_t tiles_w = (Wo + BW - 1) / BW, tiles_n = (Cout + BN - 1) / BN;
  // Variant bit 16: CTA pairs (cta_group::2 MMAs of M = 256; each CTA of the
  // pair loads half of the weight box).  A pair tile is 2 x MT M tiles.
  const bool pair = ((variant >> 16) & 1) != 0;
  if (pair && BN > 128) return fail_unsupported("conv3d CTA pairs: Cout tiles <= 128");
  const int BNl = pair ? BN / 2 : BN;   // weight rows one CTA loads
  const int prow = pair ? 2 : 1;
  auto tiles_for = [&](int mt) {
    return N * Do * ((Ho + BH * mt * prow - 1) / (BH * mt * prow)) * tiles_w * tiles_n;
  };
  // NCDHW output through TMA stores when TMA can address it: 16-byte aligned
  // base, rows of Wo elements a multiple of 16 bytes (variant bit 9 disables).
  const bool tma_out_ok = !y_cl && aligned16(y) && (Wo % 8) == 0 && ((variant >> 9) & 1) == 0;

  // Tile geometry.  MT M tiles per CTA tile share each weight box: per MMA
  // clock the CTA then streams ~1/MT of the weight bytes; with MT > 1 the
  // k-block is 32 channels so that three stages still fit.  kh grouping: one
  // A box of MT * BH + (KH - 1) * dh rows serves all KH taps of a (kd, kw)
  // pair.  Variant bits 10-11: 1 = one tap per k-block, 2 = grouped whenever
  // it fits; bits 12-13: 1/2/3 force MT = 1/2/4 (0 = choose).
  struct Geo {
    int mt = 1, kb = kBK, khg = 1, stages = 0, a_bytes = 0, stage_bytes = 0;
    bool staging = false;
  };
  // A gated conv may spin on halo arrivals while the push kernel that
  // delivers this GPU's own halo to a peer still has to run: keep 8 KiB of
  // each SM's shared memory free so a push CTA can always be resident beside
  // a conv CTA (it needs none but the per-CTA reservation).
  const size_t smem_cap = (gate && gate->epoch) ? kSmemBudget - 8192 : kSmemBudget;
  auto geom = [&](int mt, int kb, int khg, bool staging, Geo* g) {
    const int64_t rows = static_cast<int64_t>(mt) * BH + (khg - 1) * dh;
    if (rows > 256) return false;
    const size_t budget = smem_cap - fixed_smem(BN, staging);
    g->mt = mt;
    g->kb = kb;
    g->khg = khg;
    g->staging = staging;
    g->a_bytes = static_cast<int>(rows * BW * kb * 2);
    g->stage_bytes = g->a_bytes + khg * BNl * kb * 2;
    g->stages = static_cast<int>(std::min<size_t>(kMaxStages, budget / g->stage_bytes));
    return g->stages >= 2;
  };
  const int kgmode = (variant >> 10) & 3;
  const int mt_code = (variant >> 12) & 3;
  // Geometry for a given MT: kh-grouped when that leaves >= 3 stages (any
  // number >= 2 when forced), else one tap per k-block; the output staging
  // tile only when three stages remain beside it.
  auto plan = [&](int mt, Geo* g) {
    const int kb = mt == 1 ? kBK : 32;
    const bool group = kgmode != 1 && KH > 1;
    const int nopt = group ? 2 : 1;
    for (int o = 0; o < nopt; ++o) {
      const int khg = (group && o == 0) ? static_cast<int>(KH) : 1;
      const bool last = o == nopt - 1;
      const int need = (last || kgmode == 2) ? 2 : 3;
      if (tma_out_ok && geom(mt, kb, khg, true, g) && g->stages >= std::max(need, 3)) return true;
      if (geom(mt, kb, khg, false, g) && g->stages >= need) return true;
    }
    return false;
  };
  Geo g;
  bool planned = false;
  if (mt_code != 0) {
    const int mt = mt_code == 1 ? 1 : (mt_code == 2 ? 2 : 4);
    if (mt > 1 && BN > 128) return fail_unsupported("conv3d: MT > 1 needs Cout tiles <= 128");
    planned = plan(mt, &g);
  } else {
    // Several M tiles per CTA when there are still >= 2 tiles per SM and the
    // accumulators stay double-buffered in TMEM (2 * MT * BN <= 512 columns,
    // so the epilogue of one tile overlaps the MMAs of the next): MT = 4 for
    // BN = 64, MT = 2 for BN = 128.  (MT = 4 at BN = 128 single-buffers and
    // measured slower than MT = 2 on the video stack's conv.)
    const int64_t want = 2LL * sm_count() / prow;
    for (int mt : {4, 2}) {
      if (planned || BN > 128 || 2 * mt * BN > 512 || tiles_for(mt) < want) continue;
      if (pair && mt > 2) continue;
      Geo c;
      if (plan(mt, &c) && c.stages >= 3) {
        g = c;
        planned = true;
      }
    }
    if (!planned) planned = plan(1, &g);
  }
  if (!planned) return fail_unsupported("conv3d tile does not fit in shared memory");

  // NCDHW input: transposed into the workspace first (a separate
  // bandwidth-bound kernel that triggers this kernel's dependent launch).
  const void* xcl = x;
  if (!x_cl) {
    const size_t need = static_cast<size_t>(N * D * H * W * Cin) * sizeof(T);
    if (ws == nullptr || ws_bytes < need) return fail_arg("conv3d workspace too small");
    const int64_t S = D * H * W;
    dim3 grid(static_cast<unsigned>((S + 63) / 64), static_cast<unsigned>((Cin + 63) / 64),
              static_cast<unsigned>(N));
    if ((S + 63) / 64 > 0x7fffffffLL || (Cin + 63) / 64 > 65535)
      return fail_unsupported("transpose grid too large");
    if (aligned16(x) && aligned16(ws))
    {
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      at[0].val.programmaticStreamSerializationAllowed = 1;
      cudaLaunchConfig_t lc = {};
      lc.gridDim = grid;
      lc.blockDim = dim3(256);
      lc.stream = stream;
      lc.attrs = at;
      lc.numAttrs = 1;
      const T* xs = static_cast<const T*>(x);
      T* wsd = static_cast<T*>(ws);
      if (aligned16(x) && aligned16(ws))
        B200_CUDA_CHECK(cudaLaunchKernelEx(&lc, to_cl16_kernel<T>, xs, wsd, Cin, S));
      else
        B200_CUDA_CHECK(cudaLaunchKernelEx(&lc, to_cl_kernel<T>, xs, wsd, Cin, S));
    }
    xcl = ws;
  }
  if (!aligned16(xcl)) return fail_unsupported("operands not 16-byte aligned");
  const int khg = g.khg, stages = g.stages, a_bytes = g.a_bytes, stage_bytes = g.stage_bytes;
  const int KB = g.kb, MT = g.mt;
  const int a_rows_h = MT * BH + (khg - 1) * static_cast<int>(dh);

  CUtensorMap tmx, tmw;
  const CUtensorMapSwizzle swz = KB == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  {
    cuuint64_t dims[5] = {(cuuint64_t)Cin, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)D, (cuuint64_t)N};
    cuuint64_t strides[4] = {(cuuint64_t)(Cin * 2), (cuuint64_t)(W * Cin * 2),
                             (cuuint64_t)(H * W * Cin * 2), (cuuint64_t)(D * H * W * Cin * 2)};
    // Channels-last: one A box {KB, BW, rows, 1, 1} per (kd, kw).
    cuuint32_t box[5] = {(cuuint32_t)KB, (cuuint32_t)BW, (cuuint32_t)a_rows_h, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = encode(&tmx, dt, 5, const_cast<void*>(xcl), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail_unsupported("input tensor map rejected");
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)Cin_pad, (cuuint64_t)Cout, (cuuint64_t)taps};
    cuuint64_t strides[2] = {(cuuint64_t)(Cin_pad * 2), (cuuint64_t)(Cout * Cin_pad * 2)};
    cuuint32_t box[3] = {(cuuint32_t)KB, (cuuint32_t)BNl, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(&tmw, dt, 3, const_cast<void*>(wp), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail_unsupported("weight tensor map rejected");
  }

  ConvParams prm;
  prm.Do = (int)Do;
  prm.Ho = (int)Ho;
  prm.Wo = (int)Wo;
  prm.Cout = (int)Cout;
  prm.KH = (int)KH;
  prm.KW = (int)KW;
  prm.pd = (int)pd;
  prm.ph = (int)ph;
  prm.pw = (int)pw;
  prm.dd = (int)dd;
  prm.dh = (int)dh;
  prm.dw = (int)dw;
  prm.BW = BW;
  prm.BH = BH;
  prm.MT = MT;
  prm.tiles_w = (int)tiles_w;
  prm.tiles_h = (int)((Ho + BH * MT * prow - 1) / (BH * MT * prow));
  prm.pair = pair ? 1 : 0;
  prm.tiles_n = (int)tiles_n;
  const int64_t nt = tiles_for(MT);
  if (nt > 0x7fffffffLL) return fail_unsupported("too many tiles");
  prm.num_tiles = (int)nt;
  prm.cchunks = (int)((Cin + KB - 1) / KB);
  prm.khg = khg;
  prm.khb = static_cast<int>(KH) / khg;
  prm.a_bytes = a_bytes;
  prm.stage_bytes = stage_bytes;
  prm.stages = stages;
  prm.kblocks = static_cast<int>(KD * prm.khb * KW * prm.cchunks);
  (void)taps;
  prm.rotate = ((variant >> 8) & 1) ? 0 : 1;   // variant bit 8 disables the k rotation
  prm.y = y;
  prm.bias = bias;
  prm.bias_dt = bias_dt;
  prm.y_cl = y_cl;
  prm.flags = device_flags_ptr();
  prm.Nb = (int)N;
  prm.gate_epoch = nullptr;
  prm.gate_lo = prm.gate_hi = nullptr;
  prm.gate_scale = 0;
  if (gate && gate->epoch) {
    // The gate assumes one halo frame each side read only by the edge
    // output frames: KD = 3, no T padding, no T dilation.
    if (KD != 3 || pd != 0 || dd != 1)
      return fail_unsupported("halo gate: needs KD = 3, T padding 0, T dilation 1");
    prm.gate_epoch = gate->epoch;
    prm.gate_lo = gate->lo;
    prm.gate_hi = gate->hi;
    prm.gate_scale = gate->scale;
  }

  // NCDHW output through one TMA store per tile when TMA can address it:
  // 16-byte aligned base, rows of Wo elements a multiple of 16 bytes.  The
  // store clips positions and channels outside the output.
  CUtensorMap tmy;
  std::memset(&tmy, 0, sizeof(tmy));
  prm.out_tma = 0;
  if (tma_out_ok && g.staging) {
    cuuint64_t dims[5] = {(cuuint64_t)Wo, (cuuint64_t)Ho, (cuuint64_t)Do, (cuuint64_t)Cout,
                          (cuuint64_t)N};
    cuuint64_t strides[4] = {(cuuint64_t)(Wo * 2), (cuuint64_t)(Ho * Wo * 2),
                             (cuuint64_t)(Do * Ho * Wo * 2), (cuuint64_t)(Cout * Do * Ho * Wo * 2)};
    cuuint32_t box[5] = {(cuuint32_t)BW, (cuuint32_t)BH, 1, (cuuint32_t)BN, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = encode(&tmy, dt, 5, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    prm.out_tma = (r == CUDA_SUCCESS) ? 1 : 0;
  }
  const bool stg = g.staging;
  if (pair) {
    if (MT == 1) {
      if (BN == 64) return launch_conv<T, 64, 1, 64, true>(tmx, tmw, tmy, prm, stg, stream);
      return launch_conv<T, 128, 1, 64, true>(tmx, tmw, tmy, prm, stg, stream);
    }
    if (MT == 2) {
      if (BN == 64) return launch_conv<T, 64, 2, 32, true>(tmx, tmw, tmy, prm, stg, stream);
      return launch_conv<T, 128, 2, 32, true>(tmx, tmw, tmy, prm, stg, stream);
    }
    return fail_unsupported("conv3d CTA pairs: MT <= 2");
  }
  if (MT == 1) {
    if (BN == 64) return launch_conv<T, 64, 1, 64>(tmx, tmw, tmy, prm, stg, stream);
    if (BN == 128) return launch_conv<T, 128, 1, 64>(tmx, tmw, tmy, prm, stg, stream);
    return launch_conv<T, 256, 1, 64>(tmx, tmw, tmy, prm, stg, stream);
  }
  if (MT == 2) {
    if (BN == 64) return launch_conv<T, 64, 2, 32>(tmx, tmw, tmy, prm, stg, stream);
    return launch_conv<T, 128, 2, 32>(tmx, tmw, tmy, prm, stg, stream);
  }
  if (BN == 64) return launch_conv<T, 64, 4, 32>(tmx, tmw, tmy, prm, stg, stream);
  return launch_conv<T, 128, 4, 32>(tmx, tmw, tmy, prm, stg, stream);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

size_t b200_conv3d_packed_weight_bytes(int64_t Cout, int64_t Cin, int64_t KD, int64_t KH,
                                       int64_t KW) {
  const int64_t Cin_pad = (Cin + kBK - 1) / kBK * kBK;
  return static_cast<size_t>(KD * KH * KW * Cout * Cin_pad) * 2;
}

size_t b200_conv3d_packed_weight_bytes_for(int64_t Cout, int64_t Cin, int64_t KD, int64_t KH,
                                           int64_t KW, int dtype) {
  const size_t b16 = b200_conv3d_packed_weight_bytes(Cout, Cin, KD, KH, KW);
  return dtype == B200_DTYPE_F32 ? 3 * b16 : b16;
}

int b200_conv3d_pack_weight(const void* w, void* wp, int dtype, int64_t Cout, int64_t Cin,
                            int64_t KD, int64_t KH, int64_t KW, void* stream) {
  if (!w || !wp) return fail_arg("w/wp is NULL");
  if (Cout <= 0 || Cin <= 0 || KD <= 0 || KH <= 0 || KW <= 0) return fail_arg("bad size");
  if (dtype == B200_DTYPE_F32)
    return pack_weight_split(static_cast<const float*>(w), static_cast<__nv_bfloat16*>(wp), Cout,
                             Cin, KD, KH, KW, static_cast<cudaStream_t>(stream));
  if (dtype != B200_DTYPE_F16 && dtype != B200_DTYPE_BF16) return fail_arg("bad dtype");
  const int64_t Cin_pad = (Cin + kBK - 1) / kBK * kBK;
  const int64_t taps = KD * KH * KW;
  const int64_t total = taps * Cout * Cin_pad;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 65536));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_DTYPE_F16)
    pack_weight_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(w),
                                                    static_cast<__half*>(wp), Cout, Cin, Cin_pad, taps);
  else
    pack_weight_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(wp), Cout, Cin, Cin_pad, taps);
  B200_LAUNCH_CHECK("pack_weight_kernel");
  return B200_OK;
}

size_t b200_conv3d_workspace_bytes(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                                   int x_channels_last) {
  if (x_channels_last) return 0;
  return static_cast<size_t>(N * Cin * D * H * W) * 2;
}

int b200_conv3d_uses_slab(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                          int64_t Cout, int64_t KD, int64_t KH, int64_t KW,
                          const int64_t* params9, int dtype, int variant) {
  if (!params9) return 0;
  if (dtype == B200_DTYPE_F32) return 1;
  return slab_wanted(N, Cin, D, H, W, Cout, KD, KH, KW, params9, variant, false) ? 1 : 0;
}

size_t b200_conv3d_fwd_workspace_bytes(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                                       int64_t KD, int64_t KH, int64_t KW, const int64_t* params9,
                                       int dtype, int x_channels_last) {
  if (!params9 || N <= 0 || Cin <= 0 || D <= 0 || H <= 0 || W <= 0) return 0;
  const bool split = dtype == B200_DTYPE_F32;
  size_t need = split ? 0 : b200_conv3d_workspace_bytes(N, Cin, D, H, W, x_channels_last);
  const SlabPlan sp = slab_plan(N, Cin, D, H, W, KD, KH, KW, params9, split);
  if (sp.ok && sp.staging_bytes > need) need = sp.staging_bytes;
  return need;
}

int b200_conv3d_fwd(const void* x, const void* wp, const void* bias, void* y, int dtype,
                    int bias_dtype, int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                    int64_t Cout, int64_t KD, int64_t KH, int64_t KW, const int64_t* params9,
                    int x_channels_last, int y_channels_last, int variant, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return b200_conv3d_fwd_gated(x, wp, bias, y, dtype, bias_dtype, N, Cin, D, H, W, Cout, KD, KH,
                               KW, params9, x_channels_last, y_channels_last, variant, workspace,
                               workspace_bytes, nullptr, nullptr, nullptr, 0, stream);
}

int b200_conv3d_fwd_call(const B200Conv3dProblem* pr, const void* x, const void* wp,
                         const void* bias, void* y, void* workspace, void* stream) {
  if (!pr) return fail_arg("NULL problem");
  return b200_conv3d_fwd_gated(x, wp, bias, y, pr->dtype, pr->bias_dtype, pr->N, pr->Cin, pr->D,
                               pr->H, pr->W, pr->Cout, pr->KD, pr->KH, pr->KW, pr->params9,
                               pr->x_channels_last, pr->y_channels_last, pr->variant, workspace,
                               static_cast<size_t>(pr->workspace_bytes), nullptr, nullptr,
                               nullptr, 0, stream);
}

int b200_conv3d_fwd_gated(const void* x, const void* wp, const void* bias, void* y, int dtype,
                          int bias_dtype, int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W,
                          int64_t Cout, int64_t KD, int64_t KH, int64_t KW,
                          const int64_t* params9, int x_channels_last, int y_channels_last,
                          int variant, void* workspace, size_t workspace_bytes,
                          const void* gate_epoch, const void* gate_lo, const void* gate_hi,
                          int64_t gate_scale, void* stream) {
  if (!x || !wp || !y || !params9) return fail_arg("NULL pointer");
  if (gate_epoch && (gate_scale < 1 || gate_scale > 0xffff)) return fail_arg("gate_scale");
  const HaloGate gate{static_cast<const uint32_t*>(gate_epoch),
                      static_cast<const uint32_t*>(gate_lo),
                      static_cast<const uint32_t*>(gate_hi), static_cast<uint32_t>(gate_scale)};
  if (!dtype_ok(dtype)) return fail_arg("bad dtype");
  if (bias && !dtype_ok(bias_dtype)) return fail_arg("bad bias dtype");
  if (N <= 0 || Cin <= 0 || D <= 0 || H <= 0 || W <= 0 || Cout <= 0 || KD <= 0 || KH <= 0 ||
      KW <= 0)
    return fail_arg("bad size");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_DTYPE_F32) {
    // fp32: the slab kernel on bf16 hi/lo splits of x and w (packed by
    // b200_conv3d_pack_weight with dtype fp32).
    if (gate.epoch) return fail_unsupported("conv3d fp32: no halo gate");
    const int64_t p9[9] = {params9[0], params9[1], params9[2], params9[3], params9[4],
                           params9[5], params9[6], params9[7], params9[8]};
    if (p9[3] < 0 || p9[4] < 0 || p9[5] < 0 || p9[6] < 1 || p9[7] < 1 || p9[8] < 1 || p9[0] < 1 ||
        p9[1] < 1 || p9[2] < 1)
      return fail_arg("bad stride/padding/dilation");
    return conv3d_slab<float>(x, wp, bias, y, bias_dtype, N, Cin, D, H, W, Cout, KD, KH, KW, p9,
                              x_channels_last, y_channels_last, variant & 0xF,
                              ((variant >> 22) & 1) == 0, ((variant >> 23) & 1) != 0, workspace,
                              workspace_bytes, s);
  }
  if (dtype == B200_DTYPE_F16)
    return conv3d_typed<__half>(x, wp, bias, y, bias_dtype, N, Cin, D, H, W, Cout, KD, KH, KW,
                                params9, x_channels_last, y_channels_last, variant, workspace,
                                workspace_bytes, s, &gate);
  return conv3d_typed<__nv_bfloat16>(x, wp, bias, y, bias_dtype, N, Cin, D, H, W, Cout, KD, KH,
                                     KW, params9, x_channels_last, y_channels_last, variant,
                                     workspace, workspace_bytes, s, &gate);
}

int b200_to_channels_last(const void* x, void* y, int dtype, int64_t N, int64_t C, int64_t S,
                          void* stream) {
  if (!x || !y) return fail_arg("NULL pointer");
  if (N <= 0 || C <= 0 || S <= 0) return fail_arg("bad size");
  if ((S + 63) / 64 > 0x7fffffffLL || (C + 63) / 64 > 65535 || N > 65535)
    return fail_unsupported("transpose grid too large");
  dim3 grid(static_cast<unsigned>((S + 63) / 64), static_cast<unsigned>((C + 63) / 64),
            static_cast<unsigned>(N));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool al = aligned16(x) && aligned16(y);
  if (dtype == B200_DTYPE_F32)
    to_cl_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), static_cast<float*>(y), C, S);
  else if (dtype == B200_DTYPE_F16 && al)
    to_cl16_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(y), C, S);
  else if (dtype == B200_DTYPE_F16)
    to_cl_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(y), C, S);
  else if (dtype == B200_DTYPE_BF16 && al)
    to_cl16_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                      static_cast<__nv_bfloat16*>(y), C, S);
  else if (dtype == B200_DTYPE_BF16)
    to_cl_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                    static_cast<__nv_bfloat16*>(y), C, S);
  else
    return fail_arg("bad dtype");
  B200_LAUNCH_CHECK("to_cl_kernel");
  return B200_OK;
}

}  // extern "C"
