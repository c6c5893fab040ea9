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
  int n_groups, n_chunks;
  int slab_rows;                       // rows of every slab load (the TMA box height)
  int a_slot_bytes, a_slots, w_slot_bytes, w_slots;
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

// Rows a pair-tile / CTA-tile covers.
template <bool PAIR>
__device__ __forceinline__ int tile_rows() { return PAIR ? 2 * kSlabM : kSlabM; }

template <typename T, int BN, bool PAIR>
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
    // Unit u = (group g, channel chunk c): one slab into an A slot, then one
    // weight box per tap of the group into W slots.  Every copy of a pair
    // completes on the leader's barriers (the leader's MMAs read both CTAs).
    int a_it = 0, w_it = 0;
    bool ok = true, waited = false;
    // Weight boxes of the first unit do not depend on the previous kernel:
    // when the host allows it they are requested before griddepcontrol.wait
    // (while the staging kernel is still finishing).
    int pre = 0, pre0 = 0;
    if (p.hoist_w && tile0 < p.num_tiles) {
      const int n0 = (tile0 % p.tiles_n) * BN;
      const SlabGroup& g0 = p.groups[0];
      pre = g0.tap_count < p.w_slots ? g0.tap_count : p.w_slots;
      pre0 = pre;
      if (lane == 0) {
        for (int j = 0; j < pre; ++j) {
          const int slot = j;
          uint8_t* dst = sW + slot * p.w_slot_bytes;
          if (PAIR) {
            if (leader) mbar_expect_tx(&wfull[slot], 2u * p.w_slot_bytes);
            tma_load_3d_pair(dst, &tmw, mapa_u32(&wfull[slot], 0), 0,
                             n0 + static_cast<int>(crank) * kBNl, p.taps[g0.tap_begin + j].wtap);
          } else {
            mbar_expect_tx(&wfull[slot], p.w_slot_bytes);
            tma_load_3d(dst, &tmw, &wfull[slot], 0, n0, p.taps[g0.tap_begin + j].wtap);
          }
        }
      }
      __syncwarp();
    }
    for (int t = tile0; t < p.num_tiles && ok; t += tstep) {
      const int nt = t % p.tiles_n;
      const int pt = (t / p.tiles_n) % p.tiles_per_batch;
      const int nb = t / (p.tiles_n * p.tiles_per_batch);
      const int n0 = nt * BN;
      const int q0 = pt * tile_rows<PAIR>() + static_cast<int>(crank) * kSlabM;
      const int base = nb * p.batch_rows + q0;
      for (int u = 0; u < units && ok; ++u) {
        const SlabGroup& g = p.groups[u / p.n_chunks];
        const int c = u % p.n_chunks;
        {
          const int slot = a_it % p.a_slots;
          const uint32_t ph = static_cast<uint32_t>(a_it / p.a_slots) & 1u;
          const bool got = mbar_wait_bounded(&aempty[slot], ph ^ 1u, abort, p.flags, 1);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          if (!waited) {
            pdl_wait();
            waited = true;
          }
          if (lane == 0) {
            uint8_t* dst = sA + slot * p.a_slot_bytes;
            const uint32_t bytes = static_cast<uint32_t>(p.slab_rows) * 128u;
            if (PAIR) {
              if (leader) mbar_expect_tx(&afull[slot], 2u * bytes);
              tma_load_2d_pair(dst, &tma, mapa_u32(&afull[slot], 0), c * 64, g.a_off + base);
            } else {
              mbar_expect_tx(&afull[slot], bytes);
              tma_load_2d(dst, &tma, &afull[slot], c * 64, g.a_off + base);
            }
          }
          __syncwarp();
          ++a_it;
        }
        for (int j = 0; j < g.tap_count && ok; ++j) {
          if (pre > 0) {   // issued before the wait
            --pre;
            ++w_it;
            continue;
          }
          const int slot = w_it % p.w_slots;
          const uint32_t ph = static_cast<uint32_t>(w_it / p.w_slots) & 1u;
          const bool got = mbar_wait_bounded(&wempty[slot], ph ^ 1u, abort, p.flags, 1);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            uint8_t* dst = sW + slot * p.w_slot_bytes;
            const int wtap = p.taps[g.tap_begin + j].wtap;
            if (PAIR) {
              if (leader) mbar_expect_tx(&wfull[slot], 2u * p.w_slot_bytes);
              tma_load_3d_pair(dst, &tmw, mapa_u32(&wfull[slot], 0), c * 64,
                               n0 + static_cast<int>(crank) * kBNl, wtap);
            } else {
              mbar_expect_tx(&wfull[slot], p.w_slot_bytes);
              tma_load_3d(dst, &tmw, &wfull[slot], c * 64, n0, wtap);
            }
          }
          __syncwarp();
          ++w_it;
        }
      }
    }
    if (!waited) pdl_wait();
    if (!ok && lane == 0 && leader) {
      // Let every copy already issued land before shared memory goes away
      // (a pair's copies all complete on the leader's barriers): for each
      // slot, the phase of the last load issued into it.
      for (int s = 0; s < p.a_slots && s < a_it; ++s) {
        const int cnt = (a_it - 1 - s) / p.a_slots + 1;
        mbar_wait_bounded(&afull[s], static_cast<uint32_t>(cnt - 1) & 1u, nullptr, nullptr, 0);
      }
      const int w_issued = w_it > pre0 ? w_it : pre0;
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
    int a_it = 0, w_it = 0, it = 0;
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
      bool first = true;
      for (int u = 0; u < units && ok; ++u) {
        const SlabGroup& g = p.groups[u / p.n_chunks];
        const int aslot = a_it % p.a_slots;
        const bool got_a = mbar_wait_bounded(&afull[aslot],
                                             static_cast<uint32_t>(a_it / p.a_slots) & 1u, abort,
                                             p.flags, 1);
        if (!__all_sync(0xffffffffu, got_a)) {
          ok = false;
          break;
        }
        const uint32_t a_base = smem_u32(sA + aslot * p.a_slot_bytes);
        for (int j = 0; j < g.tap_count; ++j) {
          const int wslot = w_it % p.w_slots;
          const bool got_w = mbar_wait_bounded(&wfull[wslot],
                                               static_cast<uint32_t>(w_it / p.w_slots) & 1u, abort,
                                               p.flags, 1);
          if (!__all_sync(0xffffffffu, got_w)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint64_t adesc =
                umma_desc_sw128(a_base + static_cast<uint32_t>(p.taps[g.tap_begin + j].off) * 128u);
            const uint64_t bdesc = umma_desc_sw128(smem_u32(sW + wslot * p.w_slot_bytes));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t accum = (first && k == 0) ? 0u : 1u;
              if (PAIR)
                umma_f16_ss_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, kIdesc, accum);
              else
                umma_f16_ss(d_tmem, adesc + 2 * k, bdesc + 2 * k, kIdesc, accum);
            }
            if (PAIR) {
              umma_commit_pair(smem_u32(&wempty[wslot]));
              umma_commit_pair(mapa_u32(&wempty[wslot], 1));
            } else {
              umma_commit(&wempty[wslot]);
            }
          }
          __syncwarp();
          first = false;
          ++w_it;
        }
        if (!ok) break;
        if (lane == 0) {
          if (PAIR) {
            umma_commit_pair(smem_u32(&aempty[aslot]));
            umma_commit_pair(mapa_u32(&aempty[aslot], 1));
          } else {
            umma_commit(&aempty[aslot]);
          }
        }
        __syncwarp();
        ++a_it;
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
    T* y = static_cast<T*>(p.y);
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
          T* dst = y + (nb * p.Do * plane + pos) * p.Cout + n0 + j0;
          if (n0 + j0 + 32 <= p.Cout && (p.Cout & 7) == 0) {
#pragma unroll
            for (int g8 = 0; g8 < 4; ++g8) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = v[8 * g8 + e];
              *reinterpret_cast<uint4*>(dst + 8 * g8) = pack16<T>(f);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j0 + j < p.Cout) dst[j] = from_f32<T>(v[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int co = n0 + j0 + j;
            if (co < p.Cout) y[((nb * p.Cout + co) * p.Do) * plane + pos] = from_f32<T>(v[j]);
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
    // 16-byte vectors of 8 channels; scalar when C is not a multiple of 8.
    for (int i = threadIdx.x; i < npos * 8; i += 256) {
      const int pi = i >> 3, v = i & 7;
      const int64_t c = c0 + 8 * v;
      if (c >= Cp) continue;
      const int64_t w = (w0 + pi) * sw + rw - pw;
      uint4 q = make_uint4(0, 0, 0, 0);
      if (row_in && w >= 0 && w < W && c < C) {
        const T* src = x + (((n * D + d) * H + h) * W + w) * C + c;
        if ((C & 7) == 0) {
          q = *reinterpret_cast<const uint4*>(src);
        } else {
          uint16_t e[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            e[k] = (c + k < C) ? reinterpret_cast<const uint16_t*>(src)[k] : uint16_t(0);
          q = make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16),
                         e[4] | (uint32_t(e[5]) << 16), e[6] | (uint32_t(e[7]) << 16));
        }
      }
      *reinterpret_cast<uint4*>(out + (orow + pi) * Cp + c) = q;
    }
    return;
  }
  // NCDHW: channel rows of the input along w into tile[c][pos] ...
  for (int i = threadIdx.x; i < 64 * 64; i += 256) {
    const int cc = i >> 6, pi = i & 63;
    const int64_t c = c0 + cc;
    const int64_t w = (w0 + pi) * sw + rw - pw;
    uint16_t v = 0;
    if (row_in && pi < npos && c < C && w >= 0 && w < W)
      v = reinterpret_cast<const uint16_t*>(x)[(((n * C + c) * D + d) * H + h) * W + w];
    tile[cc][pi] = v;
  }
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

size_t slab_fixed_smem(int BN) {
  return static_cast<size_t>(BN) * 4 + (2 * kSlabMaxA + 2 * kSlabMaxW + 5) * 8 + 16 + 1024;
}

}  // namespace

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
                   int64_t KH, int64_t KW, const int64_t* prm) {
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
  s.Cp = (Cin + 7) / 8 * 8;
  s.rows = s.phases * N * s.Dq * s.Hq * s.Wq;
  if (s.rows + 2 * kSlabMaxRows >= (1LL << 31)) return s;
  s.staging_bytes = static_cast<size_t>(s.rows * s.Cp) * 2;
  s.ok = true;
  return s;
}

template <typename T>
int conv3d_slab(const void* x, const void* wp, const void* bias, void* y, int bias_dt,
                int64_t N, int64_t Cin, int64_t D, int64_t H, int64_t W, int64_t Cout,
                int64_t KD, int64_t KH, int64_t KW, const int64_t* prm, int x_cl, int y_cl,
                int bn_code, bool pair, bool staged, void* ws, size_t ws_bytes,
                cudaStream_t stream) {
  const SlabPlan sp = slab_plan(N, Cin, D, H, W, KD, KH, KW, prm);
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
  p.n_chunks = static_cast<int>((sp.Cp + 63) / 64);
  p.slab_rows = max_rows;

  int BN = bn_code == 1 ? 64 : bn_code == 2 ? 128 : bn_code == 3 ? 256 : (Cout <= 64 ? 64 : Cout <= 128 ? 128 : 256);
  if (pair && BN > 128) BN = 128;
  const int BNl = pair ? BN / 2 : BN;
  p.a_slot_bytes = (max_rows * 128 + 1023) / 1024 * 1024;
  p.w_slot_bytes = BNl * 128;
  const size_t budget = kSlabSmemBudget - slab_fixed_smem(BN);
  const int units = p.n_groups * p.n_chunks;
  const int total_w = ng > 0 ? nt * p.n_chunks : 0;
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
  (void)max_taps;

  // Stage the input (same stream; the conv overlaps its tail through PDL),
  // unless the caller staged it into the workspace already.
  if (!staged) {
    const int wblocks = static_cast<int>((sp.Wq + 63) / 64);
    const int64_t rowsblk = sp.phases * N * sp.Dq * sp.Hq * wblocks;
    if (rowsblk > 0x7fffffffLL || (sp.Cp + 63) / 64 > 65535)
      return fail_unsupported("conv3d slab path: staging grid");
    dim3 grid(static_cast<unsigned>(rowsblk), static_cast<unsigned>((sp.Cp + 63) / 64));
    const T* xs = static_cast<const T*>(x);
    T* out = static_cast<T*>(ws);
    const int isd = static_cast<int>(sp.s_d), ish = static_cast<int>(sp.s_h),
              isw = static_cast<int>(sp.s_w);
    const int ipd = static_cast<int>(prm[3]), iph = static_cast<int>(prm[4]),
              ipw = static_cast<int>(prm[5]);
    if (x_cl)
      slab_stage_kernel<T, true><<<grid, 256, 0, stream>>>(xs, out, N, Cin, D, H, W, sp.Cp, sp.Dq,
                                                           sp.Hq, sp.Wq, isd, ish, isw, ipd, iph,
                                                           ipw, wblocks);
    else
      slab_stage_kernel<T, false><<<grid, 256, 0, stream>>>(xs, out, N, Cin, D, H, W, sp.Cp, sp.Dq,
                                                            sp.Hq, sp.Wq, isd, ish, isw, ipd, iph,
                                                            ipw, wblocks);
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
    const int64_t Cin_pad = (Cin + 63) / 64 * 64;
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
                      static_cast<size_t>(p.w_slots) * p.w_slot_bytes + slab_fixed_smem(BN);
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
    auto kern = conv3d_slab_kernel<T, BNV, PR>;                                                \
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

template int conv3d_slab<__half>(const void*, const void*, const void*, void*, int, int64_t,
                                 int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                 int64_t, const int64_t*, int, int, int, bool, bool, void*,
                                 size_t, cudaStream_t);
template int conv3d_slab<__nv_bfloat16>(const void*, const void*, const void*, void*, int,
                                        int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                        int64_t, int64_t, int64_t, const int64_t*, int, int, int,
                                        bool, bool, void*, size_t, cudaStream_t);

}  // namespace b200
