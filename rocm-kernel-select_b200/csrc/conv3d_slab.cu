// Dense conv3d as a shifted-window ("slab") implicit GEMM on sm_100a.
//
// The box-per-tap kernel (conv3d_tc.cu) loads one TMA box of the input per
// filter tap group and per M tile, so a CTA streams its input halo once per
// (kd, kw) pair and the whole weight tensor once per tile.  Here the input
// is first staged (one pass, same stream) into PHASE GRIDS: for stride s the
// padded input splits into s^3 grids x_r[d', h', w'] = x_pad[s d' + rd,
// s h' + rh, s w' + rw] (one grid for stride 1), channels-last, channels
// padded to a multiple of 8, zeros in the halo.  Every filter tap (kd, kh,
// kw) then reads ONE phase grid at a constant offset from the output
// position:  tap offset kd*dd = s*qd + rd (same per dim), so output
// position q = (od*Hq + oh)*Wq + ow of the grid reads row
// q + (qd*Hq + qh)*Wq + qw of grid r.  A CTA's M tile is 128 consecutive
// positions q (rows with oh >= Ho or ow >= Wo are computed and dropped), so
// the A operand of a tap is 128 consecutive 128-byte rows of a staged
// buffer: for all taps of one (phase, qd) group, a single TMA load of
// 128 + max(qh*Wq + qw) rows (a "slab") holds every tap's A tile, and the
// MMA of tap (qh, qw) starts its descriptor (qh*Wq + qw) rows into the slab.
// The 128-byte swizzle of both TMA and tcgen05 is a function of the shared-
// memory address alone, so such a start needs no base offset and no copy.
//
// CTA pairs (tcgen05 cta_group::2): two CTAs on two SMs compute 256
// consecutive positions with M = 256 MMAs; each loads its own slab and HALF
// of every weight box, so the weights cross L2 -> SM once per pair instead
// of once per CTA.  TMA loads only ever land in the issuing CTA.
//
// Roles (6 warps): 0 = TMA producer, 1 = MMA issuer (the pair leader's),
// 2-5 = epilogue (TMEM -> + bias -> 16-bit stores, NCDHW or channels-last).
// A ring of slab slots and a ring of weight slots decouple the producer
// from the MMAs; accumulators are double-buffered in TMEM so a persistent
// CTA's epilogue overlaps its next tile.  Every wait is bounded
// (kWaitLimitNs): on expiry the fault word gets code 1 and the CTA unwinds.
#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>
#include <vector>

#include "conv3d_slab.cuh"
#include "sm100_ptx.cuh"

namespace b200 {
namespace {

constexpr int kSlabThreads = 192;
constexpr int kSlabMaxGroups = 128;
constexpr int kSlabMaxTaps = 1024;
constexpr int kSlabMaxA = 4;
constexpr int kSlabMaxW = 32;
constexpr int kSlabStageTaps = 12;     // most weight boxes behind one W barrier
constexpr int kSlabM = 128;            // output positions per CTA tile
constexpr int kSlabMaxRows = 256;      // TMA box limit along a dimension
constexpr size_t kSlabSmemBudget = 232448;

struct SlabGroup {
  int a_off;       // staged-buffer row of this group for batch 0, position 0
  int tap_begin;   // first entry in taps[]
  int tap_count;
  int rows;        // slab rows this group loads (128 + largest tap offset)
};
struct SlabTap {
  int off;    // rows into the slab where this tap's A tile starts
  int wtap;   // tap index in the packed weights
};

struct SlabParams {
  int n_groups, n_taps, n_chunks;
  int slab_rows;                       // rows of every slab load (the TMA box height)
  int a_slot_bytes, a_slots, w_slot_bytes, w_slots;
  int w_box_bytes, w_taps;             // one tap's weight box; taps per W slot (one barrier)
  int tiles_per_batch, tiles_n, num_tiles;
  int batch_rows;                      // staged rows per batch inside one phase grid
  int Hq, Wq, Do, Ho, Wo, Cout, positions;
  int hoist_w;                         // weight loads may precede griddepcontrol.wait
  void* y;
  const void* bias;
  int bias_dt, y_cl;
  int* flags;
  SlabGroup groups[kSlabMaxGroups];
  SlabTap taps[kSlabMaxTaps];
};

// Order of work inside a tile.  Tiles start their walk at different units
// and taps: CTAs in lockstep would otherwise all request the same weight box
// at the same moment, and those few L2 lines become a hot spot every CTA
// queues on.  The order depends on the tile only, so a tile's accumulation
// order (and rounding) does not depend on the grid or the schedule.
__device__ __forceinline__ int unit_start(int t, int units) {
  return static_cast<int>((static_cast<uint32_t>(t) * 7u) % static_cast<uint32_t>(units));
}
__device__ __forceinline__ int tap_start(int t, int count) {
  return static_cast<int>((static_cast<uint32_t>(t) * 5u + 3u * (static_cast<uint32_t>(t) >> 3)) %
                          static_cast<uint32_t>(count));
}

// Slot and phase of a ring of barriers, advanced without divisions (the
// producer and MMA loops are short enough that integer division by a
// runtime ring size would dominate them).
struct Ring {
  int slot;
  uint32_t phase;
  int n;
  __device__ __forceinline__ void advance() {
    if (++slot == n) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Rows a pair-tile / CTA-tile covers.
template <bool PAIR>
__device__ __forceinline__ int tile_rows() { return PAIR ? 2 * kSlabM : kSlabM; }

template <typename T, typename TO, int BN, bool PAIR>
__global__ void __launch_bounds__(kSlabThreads, 1)
conv3d_slab_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmw,
                   const __grid_constant__ SlabParams p) {
  constexpr int kBNl = PAIR ? BN / 2 : BN;      // weight rows this CTA loads
  constexpr int kBufs = 2;
  constexpr uint32_t kTmemCols = static_cast<uint32_t>(kBufs * BN) < 32u ? 32u
                                                                        : static_cast<uint32_t>(kBufs * BN);
  static_assert((kTmemCols & (kTmemCols - 1)) == 0 && kTmemCols <= 512, "TMEM columns");
  constexpr uint32_t kIdesc =
      umma_idesc_f16(std::is_same<T, __half>::value ? 0 : 1, PAIR ? 2 * kSlabM : kSlabM, BN);

  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = crank == 0u;
  const int tile0 = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int tstep = PAIR ? static_cast<int>(nclusters_x()) : static_cast<int>(gridDim.x);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sW = sA + p.a_slots * p.a_slot_bytes;
  float* sBias = reinterpret_cast<float*>(sW + p.w_slots * p.w_slot_bytes);   // [BN]
  uint64_t* afull = reinterpret_cast<uint64_t*>(sBias + BN);
  uint64_t* aempty = afull + kSlabMaxA;
  uint64_t* wfull = aempty + kSlabMaxA;
  uint64_t* wempty = wfull + kSlabMaxW;
  uint64_t* tfull = wempty + kSlabMaxW;    // [2]
  uint64_t* tempty = tfull + 2;            // [2]
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // The group / tap tables, copied out of the parameter block once: read
  // through a pointer, the parameter space costs a long-latency load per
  // access, and the producer and MMA loops read them on every tap.
  SlabGroup* groups = reinterpret_cast<SlabGroup*>(tmem_slot + 4);
  SlabTap* taps = reinterpret_cast<SlabTap*>(groups + p.n_groups);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tma);
    prefetch_tmap(&tmw);
    for (int s = 0; s < kSlabMaxA; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < kSlabMaxW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 8 : 4);   // one arrival per epilogue warp (both CTAs)
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < p.n_groups; i += kSlabThreads) groups[i] = p.groups[i];
  for (int i = threadIdx.x; i < p.n_taps; i += kSlabThreads) taps[i] = p.taps[i];
  if (warp == 1) {
    if (PAIR)
      tmem_alloc_pair(tmem_slot, kTmemCols);
    else
      tmem_alloc(tmem_slot, kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int units = p.n_groups * p.n_chunks;

  if (warp == 0) {
    // -------------------------------------------------------- TMA producer
    // Unit = (group, channel chunk): one slab into an A slot, then one
    // weight box per tap of the group into W slots.  Every copy of a pair
    // completes on the leader's barriers (the leader's MMAs read both CTAs).
    // Weight boxes do not depend on the previous kernel: when the host allows
    // it, those of the very first unit (as many as the ring holds) are
    // requested before griddepcontrol.wait, while the staging kernel is
    // still finishing.
    Ring ar{0, 0u, p.a_slots}, wr{0, 0u, p.w_slots};
    int a_issued = 0, w_issued = 0;
    bool ok = true, waited = p.hoist_w == 0;
    if (waited) pdl_wait();
    for (int t = tile0; t < p.num_tiles && ok; t += tstep) {
      const int nt = t % p.tiles_n;
      const int pt = (t / p.tiles_n) % p.tiles_per_batch;
      const int nb = t / (p.tiles_n * p.tiles_per_batch);
      const int n0w = nt * BN + static_cast<int>(crank) * kBNl;
      const int base = nb * p.batch_rows + pt * tile_rows<PAIR>() + static_cast<int>(crank) * kSlabM;
      const int u0 = unit_start(t, units);
      int gi = u0 / p.n_chunks, ci = u0 - (u0 / p.n_chunks) * p.n_chunks;
      for (int uk = 0; uk < units && ok; ++uk) {
        const SlabGroup g = groups[gi];
        int j = tap_start(t, g.tap_count);
        // W stages of this unit: up to w_taps weight boxes on one barrier.
        const int stages = (g.tap_count + p.w_taps - 1) / p.w_taps;
        const int early = waited ? 0 : (stages < p.w_slots ? stages : p.w_slots);
        for (int k = 0; k <= stages && ok; ++k) {
          if (k == early) {
            // The slab of this unit, after the early weight stages.
            if (!waited) {
              pdl_wait();
              waited = true;
            }
            const bool got = mbar_wait_bounded(&aempty[ar.slot], ar.phase ^ 1u, abort, p.flags, 1);
            if (!__all_sync(0xffffffffu, got)) {
              ok = false;
              break;
            }
            if (lane == 0) {
              uint8_t* dst = sA + ar.slot * p.a_slot_bytes;
              const uint32_t bytes = static_cast<uint32_t>(p.slab_rows) * 128u;
              if (PAIR) {
                if (leader) mbar_expect_tx(&afull[ar.slot], 2u * bytes);
                tma_load_2d_pair(dst, &tma, mapa_u32(&afull[ar.slot], 0), ci * 64, g.a_off + base);
              } else {
                mbar_expect_tx(&afull[ar.slot], bytes);
                tma_load_2d(dst, &tma, &afull[ar.slot], ci * 64, g.a_off + base);
              }
            }
            __syncwarp();
            ar.advance();
            ++a_issued;
          }
          if (k == stages) break;
          const int nb_taps = (k == stages - 1) ? g.tap_count - k * p.w_taps : p.w_taps;
          const bool got = mbar_wait_bounded(&wempty[wr.slot], wr.phase ^ 1u, abort, p.flags, 1);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            uint8_t* dst = sW + wr.slot * p.w_slot_bytes;
            const uint32_t bytes = static_cast<uint32_t>(nb_taps * p.w_box_bytes);
            if (PAIR) {
              if (leader) mbar_expect_tx(&wfull[wr.slot], 2u * bytes);
            } else {
              mbar_expect_tx(&wfull[wr.slot], bytes);
            }
            int jj = j;
            for (int e = 0; e < nb_taps; ++e) {
              const int wtap = taps[g.tap_begin + jj].wtap;
              if (PAIR)
                tma_load_3d_pair(dst + e * p.w_box_bytes, &tmw, mapa_u32(&wfull[wr.slot], 0),
                                 ci * 64, n0w, wtap);
              else
                tma_load_3d(dst + e * p.w_box_bytes, &tmw, &wfull[wr.slot], ci * 64, n0w, wtap);
              if (++jj == g.tap_count) jj = 0;
            }
          }
          __syncwarp();
          j += nb_taps;
          if (j >= g.tap_count) j -= g.tap_count;
          wr.advance();
          ++w_issued;
        }
        if (++ci == p.n_chunks) {
          ci = 0;
          if (++gi == p.n_groups) gi = 0;
        }
      }
    }
    if (!waited) pdl_wait();
    if (!ok && lane == 0 && leader) {
      // Let every copy already issued land before shared memory goes away
      // (a pair's copies all complete on the leader's barriers): for each
      // slot, the phase of the last load issued into it.
      for (int s = 0; s < p.a_slots && s < a_issued; ++s) {
        const int cnt = (a_issued - 1 - s) / p.a_slots + 1;
        mbar_wait_bounded(&afull[s], static_cast<uint32_t>(cnt - 1) & 1u, nullptr, nullptr, 0);
      }
      for (int s = 0; s < p.w_slots && s < w_issued; ++s) {
        const int cnt = (w_issued - 1 - s) / p.w_slots + 1;
        mbar_wait_bounded(&wfull[s], static_cast<uint32_t>(cnt - 1) & 1u, nullptr, nullptr, 0);
      }
    }
    __syncwarp();
  } else if (warp == 1 && PAIR && !leader) {
    pdl_wait();   // the pair's MMAs are issued by the leader only
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    pdl_wait();
    Ring ar{0, 0u, p.a_slots}, wr{0, 0u, p.w_slots};
    int it = 0;
    bool ok = true;
    for (int t = tile0; t < p.num_tiles && ok; t += tstep, ++it) {
      const int acc = it & 1;
      const uint32_t aph = static_cast<uint32_t>(it >> 1) & 1u;
      const bool free_acc = mbar_wait_bounded(&tempty[acc], aph ^ 1u, abort, p.flags, 1);
      if (!__all_sync(0xffffffffu, free_acc)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      uint32_t accum = 0u;
      const int u0 = unit_start(t, units);
      int gi = u0 / p.n_chunks, ci = u0 - (u0 / p.n_chunks) * p.n_chunks;
      for (int uk = 0; uk < units && ok; ++uk) {
        const SlabGroup g = groups[gi];
        const bool got_a = mbar_wait_bounded(&afull[ar.slot], ar.phase, abort, p.flags, 1);
        if (!__all_sync(0xffffffffu, got_a)) {
          ok = false;
          break;
        }
        const uint32_t a_base = smem_u32(sA + ar.slot * p.a_slot_bytes);
        int j = tap_start(t, g.tap_count);
        const int stages = (g.tap_count + p.w_taps - 1) / p.w_taps;
        for (int k = 0; k < stages; ++k) {
          const int nb_taps = (k == stages - 1) ? g.tap_count - k * p.w_taps : p.w_taps;
          const bool got_w = mbar_wait_bounded(&wfull[wr.slot], wr.phase, abort, p.flags, 1);
          if (!__all_sync(0xffffffffu, got_w)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            // Every descriptor of the stage first (the tap table lives in
            // shared memory), then the MMAs back to back.
            const uint32_t w_base = smem_u32(sW + wr.slot * p.w_slot_bytes);
            uint32_t a_at[kSlabStageTaps];
#pragma unroll
            for (int e = 0; e < kSlabStageTaps; ++e) {
              a_at[e] = a_base + static_cast<uint32_t>(taps[g.tap_begin + j].off) * 128u;
              if (e < nb_taps && ++j == g.tap_count) j = 0;
            }
#pragma unroll
            for (int e = 0; e < kSlabStageTaps; ++e) {
              if (e < nb_taps) {
                const uint64_t adesc = umma_desc_sw128(a_at[e]);
                const uint64_t bdesc =
                    umma_desc_sw128(w_base + static_cast<uint32_t>(e * p.w_box_bytes));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  if (PAIR)
                    umma_f16_ss_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, kIdesc, accum);
                  else
                    umma_f16_ss(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, kIdesc, accum);
                  accum = 1u;
                }
              }
            }
            if (PAIR) {
              umma_commit_pair(smem_u32(&wempty[wr.slot]));
              umma_commit_pair(mapa_u32(&wempty[wr.slot], 1));
            } else {
              umma_commit(&wempty[wr.slot]);
            }
          } else {
            j += nb_taps;
            if (j >= g.tap_count) j -= g.tap_count;
          }
          __syncwarp();
          accum = 1u;
          wr.advance();
        }
        if (!ok) break;
        if (lane == 0) {
          if (PAIR) {
            umma_commit_pair(smem_u32(&aempty[ar.slot]));
            umma_commit_pair(mapa_u32(&aempty[ar.slot], 1));
          } else {
            umma_commit(&aempty[ar.slot]);
          }
        }
        __syncwarp();
        ar.advance();
        if (++ci == p.n_chunks) {
          ci = 0;
          if (++gi == p.n_groups) gi = 0;
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
    if (lane == 0) {
      if (PAIR)
        umma_commit_pair(smem_u32(drain));
      else
        umma_commit(drain);
    }
    __syncwarp();
    mbar_wait_bounded(drain, 0, nullptr, nullptr, 0);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int etid = threadIdx.x - 64;
    TO* y = static_cast<TO*>(p.y);
    const int64_t HWq = static_cast<int64_t>(p.Hq) * p.Wq;
    const int64_t plane = static_cast<int64_t>(p.Ho) * p.Wo;
    int it = 0;
    for (int t = tile0; t < p.num_tiles; t += tstep, ++it) {
      const int acc = it & 1;
      const uint32_t aph = static_cast<uint32_t>(it >> 1) & 1u;
      const bool got = mbar_wait_bounded(&tfull[acc], aph, abort, p.flags, 1);
      if (!epi_bar_and(got)) break;
      tc_fence_after();
      const int nt = t % p.tiles_n;
      const int pt = (t / p.tiles_n) % p.tiles_per_batch;
      const int64_t nb = t / (p.tiles_n * p.tiles_per_batch);
      const int n0 = nt * BN;
      for (int j = etid; j < BN; j += 128) {
        const int co = n0 + j;
        sBias[j] = (p.bias && co < p.Cout) ? load_param(p.bias, p.bias_dt, co) : 0.f;
      }
      epi_bar();
      const int64_t q = static_cast<int64_t>(pt) * tile_rows<PAIR>() + crank * kSlabM + row;
      const int64_t od = q / HWq;
      const int64_t rem = q - od * HWq;
      const int64_t oh = rem / p.Wq, ow = rem - (rem / p.Wq) * p.Wq;
      const bool valid = q < p.positions && oh < p.Ho && ow < p.Wo;
      const int64_t pos = (od * p.Ho + oh) * p.Wo + ow;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 32) {
        float v0[16], v1[16], v[32];
        tmem_ld16(taddr + j0, v0);
        tmem_ld16(taddr + j0 + 16, v1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (j < 16 ? v0[j] : v1[j - 16]) + sBias[j0 + j];
        if (!valid) continue;
        if (p.y_cl) {
          TO* dst = y + (nb * p.Do * plane + pos) * p.Cout + n0 + j0;
          constexpr int V = Vec16<TO>::N;
          if (n0 + j0 + 32 <= p.Cout && p.Cout % V == 0) {
#pragma unroll
            for (int g8 = 0; g8 < 32 / V; ++g8) {
              float f[V];
#pragma unroll
              for (int e = 0; e < V; ++e) f[e] = v[V * g8 + e];
              *reinterpret_cast<uint4*>(dst + V * g8) = pack16<TO>(f);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j0 + j < p.Cout) dst[j] = from_f32<TO>(v[j]);
          }
        } else {
          const int64_t cstride = static_cast<int64_t>(p.Do) * plane;
          TO* dst = y + (nb * p.Cout + n0 + j0) * cstride + pos;
          const int nco = p.Cout - (n0 + j0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < nco) *dst = from_f32<TO>(v[j]);
            dst += cstride;
          }
        }
      }
      // Accumulators drained: the MMA warp may reuse them.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (!PAIR || leader)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_remote(mapa_u32(&tempty[acc], 0));
      }
      epi_bar();   // sBias is rewritten by the next tile
    }
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------ staging ---
// x (NCDHW, or channels-last [N, D, H, W, C]) -> phase grids
// [phase][N][Dq][Hq][Wq][Cp], zero where the padded position is outside the
// input or the channel is >= C.  One CTA: 64 consecutive positions of one
// (phase, n, d', h') row x 64 channels, through shared memory for NCDHW
// (reads along w, writes 16-byte channel vectors).
template <typename T, bool CL_IN>
__global__ void __launch_bounds__(256)
slab_stage_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t N, int64_t C,
                  int64_t D, int64_t H, int64_t W, int64_t Cp, int64_t Dq, int64_t Hq,
                  int64_t Wq, int sd, int sh, int sw, int pd, int ph, int pw, int wblocks) {
  static_assert(sizeof(T) == 2, "16-bit elements");
  __shared__ uint16_t tile[64][66];
  pdl_launch_dependents();   // the conv kernel's prologue may overlap this pass
  const int64_t rowblk = blockIdx.x;
  const int wb = static_cast<int>(rowblk % wblocks);
  int64_t r = rowblk / wblocks;            // (phase, n, d', h') row
  const int64_t hq = r % Hq;
  r /= Hq;
  const int64_t dq = r % Dq;
  r /= Dq;
  const int64_t n = r % N;
  const int64_t phase = r / N;
  const int rw = static_cast<int>(phase % sw);
  const int rh = static_cast<int>((phase / sw) % sh);
  const int rd = static_cast<int>(phase / (sw * sh));
  const int64_t d = dq * sd + rd - pd, h = hq * sh + rh - ph;
  const bool row_in = d >= 0 && d < D && h >= 0 && h < H;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 64;
  const int64_t w0 = static_cast<int64_t>(wb) * 64;
  const int64_t npos = min64(64, Wq - w0);
  const int64_t orow = ((phase * N + n) * Dq + dq) * Hq * Wq + hq * Wq + w0;   // first out position
  if (CL_IN) {
    // 16-byte vectors of 8 channels (scalar when C is not a multiple of 8):
    // both vectors of a thread are loaded before either is stored.
    uint4 q[2];
    int64_t dst[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = threadIdx.x + 256 * k;
      const int pi = i >> 3, v = i & 7;
      const int64_t c = c0 + 8 * v;
      const int64_t w = (w0 + pi) * sw + rw - pw;
      q[k] = make_uint4(0, 0, 0, 0);
      dst[k] = (pi < npos && c < Cp) ? (orow + pi) * Cp + c : -1;
      if (dst[k] >= 0 && row_in && w >= 0 && w < W && c < C) {
        const T* src = x + (((n * D + d) * H + h) * W + w) * C + c;
        if ((C & 7) == 0) {
          q[k] = *reinterpret_cast<const uint4*>(src);
        } else {
          uint16_t e[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            e[j] = (c + j < C) ? reinterpret_cast<const uint16_t*>(src)[j] : uint16_t(0);
          q[k] = make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16),
                            e[4] | (uint32_t(e[5]) << 16), e[6] | (uint32_t(e[7]) << 16));
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (dst[k] >= 0) *reinterpret_cast<uint4*>(out + dst[k]) = q[k];
    return;
  }
  // NCDHW: channel rows of the input along w into tile[c][pos] -- all 16
  // loads of a thread in flight before the first shared-memory store ...
  const uint16_t* x16 = reinterpret_cast<const uint16_t*>(x);
  const int pi = threadIdx.x & 63;
  const int64_t w = (w0 + pi) * sw + rw - pw;
  const bool col_in = row_in && pi < npos && w >= 0 && w < W;
  const int64_t plane_in = D * H * W;
  const int64_t src0 = ((n * C + c0) * D + d) * H * W + h * W + w;
  uint16_t v[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int cc = (threadIdx.x >> 6) + 4 * k;
    v[k] = (col_in && c0 + cc < C) ? x16[src0 + cc * plane_in] : uint16_t(0);
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) tile[(threadIdx.x >> 6) + 4 * k][pi] = v[k];
  __syncthreads();
  // ... then 16-byte vectors of 8 channels per position.
  for (int i = threadIdx.x; i < npos * 8; i += 256) {
    const int pi = i >> 3, v = i & 7;
    const int64_t c = c0 + 8 * v;
    if (c >= Cp) continue;
    uint16_t e[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = tile[8 * v + k][pi];
    *reinterpret_cast<uint4*>(out + (orow + pi) * Cp + c) =
        make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16),
                   e[4] | (uint32_t(e[5]) << 16), e[6] | (uint32_t(e[7]) << 16));
  }
}

// fp32 x -> phase grids of bf16 pairs: each staged position holds three
// channel blocks of Cq = Cin rounded up to 64, [hi | lo | hi] with hi =
// bf16(x) and lo = bf16(x - hi).  Against weights packed as [hi | hi | lo]
// (pack_weight_split_kernel) the GEMM over the concatenated K computes
// x_hi w_hi + x_lo w_hi + x_hi w_lo: x and w each kept to about 16
// significant bits, fp32 accumulation, the x_lo w_lo term (2^-16 relative)
// dropped.  Same CTA geometry as slab_stage_kernel.
template <bool CL_IN>
__global__ void __launch_bounds__(256)
slab_stage_split_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ out, int64_t N,
                        int64_t C, int64_t D, int64_t H, int64_t W, int64_t Cq, int64_t Dq,
                        int64_t Hq, int64_t Wq, int sd, int sh, int sw, int pd, int ph, int pw,
                        int wblocks) {
  __shared__ float tile[64][65];
  pdl_launch_dependents();
  const int64_t rowblk = blockIdx.x;
  const int wb = static_cast<int>(rowblk % wblocks);
  int64_t r = rowblk / wblocks;
  const int64_t hq = r % Hq;
  r /= Hq;
  const int64_t dq = r % Dq;
  r /= Dq;
  const int64_t n = r % N;
  const int64_t phase = r / N;
  const int rw = static_cast<int>(phase % sw);
  const int rh = static_cast<int>((phase / sw) % sh);
  const int rd = static_cast<int>(phase / (sw * sh));
  const int64_t d = dq * sd + rd - pd, h = hq * sh + rh - ph;
  const bool row_in = d >= 0 && d < D && h >= 0 && h < H;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 64;
  const int64_t w0 = static_cast<int64_t>(wb) * 64;
  const int64_t npos = min64(64, Wq - w0);
  const int64_t orow = ((phase * N + n) * Dq + dq) * Hq * Wq + hq * Wq + w0;
  float v[16];
  if (CL_IN) {
    // consecutive threads read consecutive channels of one position
    const int cc = threadIdx.x & 63;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int pi = (threadIdx.x >> 6) + 4 * k;
      const int64_t w = (w0 + pi) * sw + rw - pw;
      v[k] = (row_in && pi < npos && w >= 0 && w < W && c0 + cc < C)
                 ? x[(((n * D + d) * H + h) * W + w) * C + c0 + cc]
                 : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) tile[cc][(threadIdx.x >> 6) + 4 * k] = v[k];
  } else {
    const int pi = threadIdx.x & 63;
    const int64_t w = (w0 + pi) * sw + rw - pw;
    const bool col_in = row_in && pi < npos && w >= 0 && w < W;
    const int64_t plane_in = D * H * W;
    const int64_t src0 = ((n * C + c0) * D + d) * H * W + h * W + w;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int cc = (threadIdx.x >> 6) + 4 * k;
      v[k] = (col_in && c0 + cc < C) ? x[src0 + cc * plane_in] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) tile[(threadIdx.x >> 6) + 4 * k][pi] = v[k];
  }
  __syncthreads();
  const int64_t Ct = 3 * Cq;
  for (int i = threadIdx.x; i < npos * 8; i += 256) {
    const int pi = i >> 3, vg = i & 7;
    const int64_t c = c0 + 8 * vg;
    if (c >= Cq) continue;
    float hi[8], lo[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float f = tile[8 * vg + k][pi];
      hi[k] = __bfloat162float(__float2bfloat16_rn(f));
      lo[k] = f - hi[k];
    }
    __nv_bfloat16* dst = out + (orow + pi) * Ct + c;
    const uint4 qh = pack16<__nv_bfloat16>(hi), ql = pack16<__nv_bfloat16>(lo);
    *reinterpret_cast<uint4*>(dst) = qh;
    *reinterpret_cast<uint4*>(dst + Cq) = ql;
    *reinterpret_cast<uint4*>(dst + 2 * Cq) = qh;
  }
}

// w [Cout][Cin][taps] fp32 -> [taps][Cout][3 Cq] bf16 as [hi | hi | lo]
// (zero beyond Cin in each block).
__global__ void pack_weight_split_kernel(const float* __restrict__ w, __nv_bfloat16* __restrict__ wp,
                                         int64_t Cout, int64_t Cin, int64_t Cq, int64_t taps) {
  const int64_t Ct = 3 * Cq;
  const int64_t total = taps * Cout * Ct;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t k3 = i % Ct;
    const int64_t co = (i / Ct) % Cout;
    const int64_t tap = i / (Ct * Cout);
    const int64_t part = k3 / Cq, ci = k3 - part * Cq;
    const float v = ci < Cin ? w[(co * Cin + ci) * taps + tap] : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    wp[i] = part == 2 ? __float2bfloat16_rn(v - __bfloat162float(hi)) : hi;
  }
}

size_t slab_fixed_smem(int BN, int n_groups, int n_taps) {
  return static_cast<size_t>(BN) * 4 + (2 * kSlabMaxA + 2 * kSlabMaxW + 5) * 8 + 16 +
         static_cast<size_t>(n_groups) * sizeof(SlabGroup) +
         static_cast<size_t>(n_taps) * sizeof(SlabTap) + 1024;
}

}  // namespace

int pack_weight_split(const float* w, __nv_bfloat16* wp, int64_t Cout, int64_t Cin, int64_t KD,
                      int64_t KH, int64_t KW, cudaStream_t stream) {
  const int64_t Cq = (Cin + 63) / 64 * 64;
  const int64_t taps = KD * KH * KW;
  const int64_t total = taps * Cout * 3 * Cq;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 65536));
  pack_weight_split_kernel<<<grid, 256, 0, stream>>>(w, wp, Cout, Cin, Cq, taps);
  B200_LAUNCH_CHECK("pack_weight_split_kernel");
  return B200_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

SlabPlan slab_plan(int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t KD,
                   int64_t KH, int64_t KW, const int64_t* prm, bool split) {
  SlabPlan s;
  const int64_t sd = prm[0], sh = prm[1], sw = prm[2];
  const int64_t pd = prm[3], ph = prm[4], pw = prm[5];
  const int64_t dd = prm[6], dh = prm[7], dw = prm[8];
  if (sd < 1 || sh < 1 || sw < 1 || sd > 4 || sh > 4 || sw > 4) return s;
  if (pd < 0 || ph < 0 || pw < 0 || dd < 1 || dh < 1 || dw < 1) return s;
  const int64_t Dp = D + 2 * pd, Hp = H + 2 * ph, Wp = W + 2 * pw;
  if (Dp < dd * (KD - 1) + 1 || Hp < dh * (KH - 1) + 1 || Wp < dw * (KW - 1) + 1) return s;
  s.s_d = sd;
  s.s_h = sh;
  s.s_w = sw;
  s.phases = sd * sh * sw;
  s.Do = (Dp - dd * (KD - 1) - 1) / sd + 1;
  s.Ho = (Hp - dh * (KH - 1) - 1) / sh + 1;
  s.Wo = (Wp - dw * (KW - 1) - 1) / sw + 1;
  s.Dq = (Dp + sd - 1) / sd;
  s.Hq = (Hp + sh - 1) / sh;
  s.Wq = (Wp + sw - 1) / sw;
  s.Cp = split ? 3 * ((Cin + 63) / 64 * 64) : (Cin + 7) / 8 * 8;
  s.rows = s.phases * N * s.Dq * s.Hq * s.Wq;
  if (s.rows + 2 * kSlabMaxRows >= (1LL << 31)) return s;
  s.staging_bytes = static_cast<size_t>(s.rows * s.Cp) * 2;
  s.ok = true;
  return s;
}

template <typename TIN>
int conv3d_slab(const void* x, const void* wp, const void* bias, void* y, int bias_dt,
                int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t Cout,
                int64_t KD, int64_t KH, int64_t KW, const int64_t* prm, int x_cl, int y_cl,
                int bn_code, bool pair, bool staged, void* ws, size_t ws_bytes,
                cudaStream_t stream) {
  // fp32: bf16 hi/lo operands (three K blocks), fp32 output.
  constexpr bool kSplit = std::is_same<TIN, float>::value;
  using T = typename std::conditional<kSplit, __nv_bfloat16, TIN>::type;
  using TO = TIN;
  const SlabPlan sp = slab_plan(N, Cin, D, H, W, KD, KH, KW, prm, kSplit);
  if (!sp.ok) return fail_unsupported("conv3d slab path: geometry");
  auto encode = tensor_map_encoder();
  if (!encode) return fail_unsupported("cuTensorMapEncodeTiled unavailable");
  if (ws == nullptr || ws_bytes < sp.staging_bytes || !aligned16(ws) || !aligned16(wp))
    return fail_unsupported("conv3d slab path: staging workspace");
  if (!aligned16(x) && (x_cl && Cin % 8 == 0))
    return fail_unsupported("conv3d slab path: unaligned channels-last input");
  const int64_t dd = prm[6], dh = prm[7], dw = prm[8];

  // Tap groups: (phase, qd) -- split by qh when the slab would exceed the
  // TMA box limit.
  const int64_t HWq = sp.Hq * sp.Wq;
  std::map<std::tuple<int64_t, int64_t, int64_t>, std::vector<std::pair<int64_t, int64_t>>> byg;
  int64_t max_off_whole = 0;
  for (int64_t kd = 0; kd < KD; ++kd)
    for (int64_t kh = 0; kh < KH; ++kh)
      for (int64_t kw = 0; kw < KW; ++kw) {
        const int64_t qh = kh * dh / sp.s_h, qw = kw * dw / sp.s_w;
        max_off_whole = std::max(max_off_whole, qh * sp.Wq + qw);
      }
  const bool split_h = kSlabM + max_off_whole > kSlabMaxRows;
  for (int64_t kd = 0; kd < KD; ++kd)
    for (int64_t kh = 0; kh < KH; ++kh)
      for (int64_t kw = 0; kw < KW; ++kw) {
        const int64_t td = kd * dd, th = kh * dh, tw = kw * dw;
        const int64_t rd = td % sp.s_d, qd = td / sp.s_d;
        const int64_t rh = th % sp.s_h, qh = th / sp.s_h;
        const int64_t rw = tw % sp.s_w, qw = tw / sp.s_w;
        const int64_t phase = (rd * sp.s_h + rh) * sp.s_w + rw;
        const int64_t a_off = (phase * N * sp.Dq + qd) * HWq + (split_h ? qh * sp.Wq : 0);
        const int64_t off = (split_h ? 0 : qh * sp.Wq) + qw;
        const int64_t wtap = (kd * KH + kh) * KW + kw;
        byg[std::make_tuple(phase, qd, split_h ? qh : 0)].push_back({off, wtap});
        (void)a_off;
      }
  static thread_local SlabParams p;
  std::memset(&p, 0, sizeof(p));
  int ng = 0, nt = 0, max_rows = 0, max_taps = 0;
  for (auto& kv : byg) {
    const int64_t phase = std::get<0>(kv.first), qd = std::get<1>(kv.first),
                  qh = std::get<2>(kv.first);
    if (ng >= kSlabMaxGroups || nt + static_cast<int>(kv.second.size()) > kSlabMaxTaps)
      return fail_unsupported("conv3d slab path: too many taps");
    int64_t mo = 0;
    for (auto& e : kv.second) mo = std::max(mo, e.first);
    const int64_t a_off = (phase * N * sp.Dq + qd) * HWq + qh * sp.Wq;
    SlabGroup& g = p.groups[ng++];
    g.a_off = static_cast<int>(a_off);
    g.tap_begin = nt;
    g.tap_count = static_cast<int>(kv.second.size());
    g.rows = static_cast<int>(kSlabM + mo);
    if (g.rows > kSlabMaxRows) return fail_unsupported("conv3d slab path: slab too tall");
    for (auto& e : kv.second) p.taps[nt++] = SlabTap{static_cast<int>(e.first), static_cast<int>(e.second)};
    max_rows = std::max(max_rows, g.rows);
    max_taps = std::max(max_taps, g.tap_count);
  }
  p.n_groups = ng;
  p.n_taps = nt;
  p.n_chunks = static_cast<int>((sp.Cp + 63) / 64);
  p.slab_rows = max_rows;

  int BN = bn_code == 1 ? 64 : bn_code == 2 ? 128 : bn_code == 3 ? 256 : (Cout <= 64 ? 64 : Cout <= 128 ? 128 : 256);
  if (pair && BN > 128) BN = 128;
  const int BNl = pair ? BN / 2 : BN;
  p.a_slot_bytes = (max_rows * 128 + 1023) / 1024 * 1024;
  p.w_box_bytes = BNl * 128;
  // Taps per W slot: a whole group when it fits in about a fifth of shared
  // memory (one barrier round trip per group), else fewer.
  p.w_taps = std::max(1, std::min({max_taps, static_cast<int>(44 * 1024 / p.w_box_bytes),
                                    kSlabStageTaps}));
  p.w_slot_bytes = p.w_taps * p.w_box_bytes;
  const size_t budget = kSlabSmemBudget - slab_fixed_smem(BN, ng, nt);
  const int units = p.n_groups * p.n_chunks;
  int total_w = 0;
  for (int gg = 0; gg < ng; ++gg)
    total_w += (p.groups[gg].tap_count + p.w_taps - 1) / p.w_taps * p.n_chunks;
  p.a_slots = std::min(kSlabMaxA, std::max(2, std::min(units, 3)));
  if (units == 1) p.a_slots = 1;
  while (p.a_slots > 1 && static_cast<size_t>(p.a_slots) * p.a_slot_bytes + 2ull * p.w_slot_bytes > budget)
    --p.a_slots;
  const size_t left = budget - static_cast<size_t>(p.a_slots) * p.a_slot_bytes;
  p.w_slots = static_cast<int>(std::min<size_t>({static_cast<size_t>(kSlabMaxW),
                                                 left / p.w_slot_bytes,
                                                 static_cast<size_t>(std::max(total_w, 2))}));
  if (p.w_slots < 2 || (units > 1 && p.a_slots < 2))
    return fail_unsupported("conv3d slab path: shared memory");

  // Stage the input (same stream; the conv overlaps its tail through PDL),
  // unless the caller staged it into the workspace already.
  if (!staged) {
    const int wblocks = static_cast<int>((sp.Wq + 63) / 64);
    const int64_t rowsblk = sp.phases * N * sp.Dq * sp.Hq * wblocks;
    if (rowsblk > 0x7fffffffLL || (sp.Cp + 63) / 64 > 65535)
      return fail_unsupported("conv3d slab path: staging grid");
    const int64_t cq = kSplit ? sp.Cp / 3 : sp.Cp;   // input channels staged per block
    dim3 grid(static_cast<unsigned>(rowsblk), static_cast<unsigned>((cq + 63) / 64));
    T* out = static_cast<T*>(ws);
    const int isd = static_cast<int>(sp.s_d), ish = static_cast<int>(sp.s_h),
              isw = static_cast<int>(sp.s_w);
    const int ipd = static_cast<int>(prm[3]), iph = static_cast<int>(prm[4]),
              ipw = static_cast<int>(prm[5]);
    if constexpr (kSplit) {
      const float* xs = static_cast<const float*>(x);
      if (x_cl)
        slab_stage_split_kernel<true><<<grid, 256, 0, stream>>>(
            xs, out, N, Cin, D, H, W, cq, sp.Dq, sp.Hq, sp.Wq, isd, ish, isw, ipd, iph, ipw, wblocks);
      else
        slab_stage_split_kernel<false><<<grid, 256, 0, stream>>>(
            xs, out, N, Cin, D, H, W, cq, sp.Dq, sp.Hq, sp.Wq, isd, ish, isw, ipd, iph, ipw, wblocks);
    } else {
      const T* xs = static_cast<const T*>(x);
      if (x_cl)
        slab_stage_kernel<T, true><<<grid, 256, 0, stream>>>(xs, out, N, Cin, D, H, W, sp.Cp,
                                                             sp.Dq, sp.Hq, sp.Wq, isd, ish, isw,
                                                             ipd, iph, ipw, wblocks);
      else
        slab_stage_kernel<T, false><<<grid, 256, 0, stream>>>(xs, out, N, Cin, D, H, W, sp.Cp,
                                                              sp.Dq, sp.Hq, sp.Wq, isd, ish, isw,
                                                              ipd, iph, ipw, wblocks);
    }
    B200_LAUNCH_CHECK("slab_stage_kernel");
  }

  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tma, tmw;
  {
    cuuint64_t dims[2] = {(cuuint64_t)sp.Cp, (cuuint64_t)sp.rows};
    cuuint64_t strides[1] = {(cuuint64_t)(sp.Cp * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)max_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&tma, dt, 2, ws, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail_unsupported("conv3d slab path: staged tensor map rejected");
  }
  {
    const int64_t Cin_pad = kSplit ? sp.Cp : (Cin + 63) / 64 * 64;   // packed K per tap
    const int64_t taps = KD * KH * KW;
    cuuint64_t dims[3] = {(cuuint64_t)Cin_pad, (cuuint64_t)Cout, (cuuint64_t)taps};
    cuuint64_t strides[2] = {(cuuint64_t)(Cin_pad * 2), (cuuint64_t)(Cout * Cin_pad * 2)};
    cuuint32_t box[3] = {64, (cuuint32_t)BNl, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(&tmw, dt, 3, const_cast<void*>(wp), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail_unsupported("conv3d slab path: weight tensor map rejected");
  }
  // The staged box must not start beyond the buffer: rows are int, and the
  // group offsets plus a tile base stay below rows + 256 (the tail beyond the
  // buffer reads as zeros).
  const int64_t positions = sp.Do * HWq;
  const int64_t trows = pair ? 2 * kSlabM : kSlabM;
  p.tiles_per_batch = static_cast<int>((positions + trows - 1) / trows);
  p.tiles_n = static_cast<int>((Cout + BN - 1) / BN);
  const int64_t ntiles = N * p.tiles_per_batch * p.tiles_n;
  if (ntiles > 0x7fffffffLL) return fail_unsupported("conv3d slab path: too many tiles");
  p.num_tiles = static_cast<int>(ntiles);
  p.batch_rows = static_cast<int>(sp.Dq * HWq);
  p.Hq = static_cast<int>(sp.Hq);
  p.Wq = static_cast<int>(sp.Wq);
  p.Do = static_cast<int>(sp.Do);
  p.Ho = static_cast<int>(sp.Ho);
  p.Wo = static_cast<int>(sp.Wo);
  p.Cout = static_cast<int>(Cout);
  p.positions = static_cast<int>(positions);
  // Weight loads may run ahead of griddepcontrol.wait only when this call's
  // own staging kernel is the conv's predecessor in the stream.
  p.hoist_w = staged ? 0 : 1;
  p.y = y;
  p.bias = bias;
  p.bias_dt = bias_dt;
  p.y_cl = y_cl;
  p.flags = device_flags_ptr();

  const size_t smem = static_cast<size_t>(p.a_slots) * p.a_slot_bytes +
                      static_cast<size_t>(p.w_slots) * p.w_slot_bytes + slab_fixed_smem(BN, ng, nt);
  if (smem > kSlabSmemBudget) return fail_unsupported("conv3d slab path: shared memory");
  cudaLaunchConfig_t cfg = {};
  const int sms = sm_count();
  const int grid = pair ? 2 * std::min(p.num_tiles, std::max(1, sms / 2)) : std::min(p.num_tiles, sms);
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kSlabThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = pair ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pair ? 2 : 1;
#define B200_SLAB_LAUNCH(BNV, PR)                                                               \
  do {                                                                                         \
    auto kern = conv3d_slab_kernel<T, TO, BNV, PR>;                                                \
    B200_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,     \
                                         static_cast<int>(smem)));                             \
    B200_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tma, tmw, p));                              \
  } while (0)
  if (pair) {
    if (BN == 64)
      B200_SLAB_LAUNCH(64, true);
    else
      B200_SLAB_LAUNCH(128, true);
  } else {
    if (BN == 64)
      B200_SLAB_LAUNCH(64, false);
    else if (BN == 128)
      B200_SLAB_LAUNCH(128, false);
    else
      B200_SLAB_LAUNCH(256, false);
  }
#undef B200_SLAB_LAUNCH
  return B200_OK;
}

template int conv3d_slab<float>(const void*, const void*, const void*, void*, int, int64_t,
                                int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                int64_t, const int64_t*, int, int, int, bool, bool, void*,
                                size_t, cudaStream_t);
template int conv3d_slab<__half>(const void*, const void*, const void*, void*, int, int64_t,
                                 int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                 int64_t, const int64_t*, int, int, int, bool, bool, void*,
                                 size_t, cudaStream_t);
template int conv3d_slab<__nv_bfloat16>(const void*, const void*, const void*, void*, int,
                                        int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                        int64_t, int64_t, int64_t, const int64_t*, int, int, int,
                                        bool, bool, void*, size_t, cudaStream_t);

}  // namespace b200
