// GroupNorm forward for sm_100a.
//
// Semantics follow the reference kernel group_norm_kernel
// (src/cuda/group_norm.cu:40-104): one (n, g) group = Cg = C/G consecutive
// channels x S spatial elements, contiguous in an NCHW/NCDHW tensor; biased
// variance, eps inside the square root, per-channel affine; fp32 statistics.
// The reference computes var = E[x^2] - mean^2 in two strided passes over
// global memory with one 256-thread block per group.  Here:
//
//  * gn_cluster_kernel -- single HBM read.  A thread-block cluster of k CTAs
//    owns one group; each CTA streams its slice of the group into shared
//    memory with 16-byte loads while summing it, the cluster exchanges
//    partial sums through distributed shared memory (DSMEM), each CTA then
//    computes sum((x - mean)^2) from shared memory (exact two-pass variance,
//    no E[x^2] - mean^2 cancellation), exchanges again, and writes the
//    normalised slice back with 16-byte streaming stores.  HBM traffic is
//    the algorithmic minimum: one read + one write.
//  * gn_partial_stats_kernel + gn_apply_kernel -- the general fallback for
//    groups too large for a cluster's shared memory: per-chunk shifted sums
//    merged with Chan's formula, then a normalising pass (one extra read).
//    The same pair serves the fused GroupNorm -> SiLU -> channels-last
//    producer of the conv3d stack, and the cross-rank statistics merge of
//    the T-sharded stack (partials are (count, mean, M2) triples).
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace b200 {
namespace {

constexpr int kGnThreads = 512;
constexpr int kGnUnroll = 4;

// x * sigmoid(x) with the fast exponential and a reciprocal-based divide
// (two special-function operations; ~1e-6 relative error).  A divide by
// 1 + e^-x that overflows gives -0, the limit of x * sigmoid(x).
__device__ __forceinline__ float silu(float v) { return __fdividef(v, 1.f + __expf(-v)); }

// ------------------------------------------------------------ cluster ----
template <typename T, bool VEC>
__global__ void __launch_bounds__(kGnThreads)
gn_cluster_kernel(const T* __restrict__ x, const void* __restrict__ gamma,
                  const void* __restrict__ beta, T* __restrict__ y, int affine_dt, int64_t S,
                  int G, int Cg, float eps, int slice, int csize) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float scratch[33];
  __shared__ float part[2];   // this CTA's partial sum and partial M2 (read by peers)
  __shared__ float stat[2];   // mean, rstd

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t ng = blockIdx.x / csize;
  const int g = static_cast<int>(ng % G);
  const int64_t M = static_cast<int64_t>(Cg) * S;
  const int64_t beg = static_cast<int64_t>(rank) * slice;
  const int cnt = static_cast<int>(max64(0, min64(slice, M - beg)));
  const T* src = x + ng * M + beg;
  T* dst = y + ng * M + beg;
  T* sx = reinterpret_cast<T*>(smem_raw);
  constexpr int V = Vec16<T>::N;

  // Pass 0: HBM -> shared memory, summing on the way.
  float s = 0.f;
  if (VEC) {
    const int nv = cnt / V;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(sx);
    for (int i0 = threadIdx.x; i0 < nv; i0 += kGnThreads * kGnUnroll) {
      uint4 r[kGnUnroll];
#pragma unroll
      for (int u = 0; u < kGnUnroll; ++u) {
        const int i = i0 + u * kGnThreads;
        if (i < nv) r[u] = ld_stream16(s4 + i);
      }
#pragma unroll
      for (int u = 0; u < kGnUnroll; ++u) {
        const int i = i0 + u * kGnThreads;
        if (i < nv) {
          d4[i] = r[u];
          float v[V];
          unpack16<T>(r[u], v);
#pragma unroll
          for (int e = 0; e < V; ++e) s += v[e];
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < cnt; i += kGnThreads) {
      const T v = src[i];
      sx[i] = v;
      s += to_f32(v);
    }
  }
  s = block_sum<kGnThreads>(s, scratch);
  if (threadIdx.x == 0) part[0] = s;
  cluster.sync();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int r = 0; r < csize; ++r) tot += *cluster.map_shared_rank(&part[0], r);
    stat[0] = tot / static_cast<float>(M);
  }
  __syncthreads();
  const float mean = stat[0];

  // Pass 1: sum of squared deviations from shared memory.
  float q = 0.f;
  if (VEC) {
    const int nv = cnt / V;
    const uint4* d4 = reinterpret_cast<const uint4*>(sx);
    for (int i = threadIdx.x; i < nv; i += kGnThreads) {
      float v[V];
      unpack16<T>(d4[i], v);
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const float d = v[e] - mean;
        q = fmaf(d, d, q);
      }
    }
  } else {
    for (int i = threadIdx.x; i < cnt; i += kGnThreads) {
      const float d = to_f32(sx[i]) - mean;
      q = fmaf(d, d, q);
    }
  }
  q = block_sum<kGnThreads>(q, scratch);
  if (threadIdx.x == 0) part[1] = q;
  cluster.sync();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int r = 0; r < csize; ++r) tot += *cluster.map_shared_rank(&part[1], r);
    stat[1] = 1.0f / sqrtf(tot / static_cast<float>(M) + eps);
  }
  // Peers may still be reading part[] of this CTA: arrive now, wait at exit.
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  __syncthreads();
  const float rstd = stat[1];

  // Pass 2: normalise + affine from shared memory -> HBM.
  const int c0 = g * Cg;
  if (VEC) {
    const int nv = cnt / V;
    const uint4* d4 = reinterpret_cast<const uint4*>(sx);
    for (int i = threadIdx.x; i < nv; i += kGnThreads) {
      const int64_t idx = beg + static_cast<int64_t>(i) * V;
      const int c = c0 + static_cast<int>(idx / S);
      // (x - mean) * (rstd * gamma) + beta: subtracting first keeps full
      // precision when rstd is large (near-constant groups).
      const float a = gamma ? rstd * load_param(gamma, affine_dt, c) : rstd;
      const float b = beta ? load_param(beta, affine_dt, c) : 0.f;
      float v[V];
      unpack16<T>(d4[i], v);
#pragma unroll
      for (int e = 0; e < V; ++e) v[e] = fmaf(v[e] - mean, a, b);
      st_stream16(reinterpret_cast<uint4*>(dst) + i, pack16<T>(v));
    }
  } else {
    for (int i = threadIdx.x; i < cnt; i += kGnThreads) {
      const int c = c0 + static_cast<int>((beg + i) / S);
      const float a = gamma ? rstd * load_param(gamma, affine_dt, c) : rstd;
      const float b = beta ? load_param(beta, affine_dt, c) : 0.f;
      dst[i] = from_f32<T>(fmaf(to_f32(sx[i]) - mean, a, b));
    }
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Unsigned 32-bit division by a runtime constant without a divide
// instruction: q = (umulhi(n, m) + n) >> l with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1 (Granlund and Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994).
struct FastDiv {
  uint32_t m, l;
};

inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{static_cast<uint32_t>(m), l};
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, FastDiv f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, f.m)) + n) >> f.l);
}

// ------------------------------------------------------- split: stats ----
// One CTA per (group, chunk).  Shifted sums around the chunk's first value
// keep the single-pass variance well conditioned; the chunk's (count, mean,
// M2) triple goes to `part`.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
gn_partial_stats_kernel(const T* __restrict__ x, float* __restrict__ part, int64_t M,
                        int64_t chunk, int chunks) {
  __shared__ float scratch[33];
  const int64_t ng = blockIdx.x / chunks;
  const int ch = blockIdx.x % chunks;
  const int64_t beg = static_cast<int64_t>(ch) * chunk;
  const int64_t cnt = max64(0, min64(chunk, M - beg));
  const T* src = x + ng * M + beg;
  const float shift = cnt > 0 ? to_f32(src[0]) : 0.f;
  float s1 = 0.f, s2 = 0.f;
  constexpr int V = Vec16<T>::N;
  if (VEC) {
    const int64_t nv = cnt / V;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    for (int64_t i0 = threadIdx.x; i0 < nv; i0 += 256 * kGnUnroll) {
      uint4 r[kGnUnroll];
#pragma unroll
      for (int u = 0; u < kGnUnroll; ++u) {
        const int64_t i = i0 + u * 256;
        if (i < nv) r[u] = ld_stream16(s4 + i);
      }
#pragma unroll
      for (int u = 0; u < kGnUnroll; ++u) {
        const int64_t i = i0 + u * 256;
        if (i < nv) {
          float v[V];
          unpack16<T>(r[u], v);
#pragma unroll
          for (int e = 0; e < V; ++e) {
            const float d = v[e] - shift;
            s1 += d;
            s2 = fmaf(d, d, s2);
          }
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < cnt; i += 256) {
      const float d = to_f32(src[i]) - shift;
      s1 += d;
      s2 = fmaf(d, d, s2);
    }
  }
  s1 = block_sum<256>(s1, scratch);
  s2 = block_sum<256>(s2, scratch);
  if (threadIdx.x == 0) {
    const float n = static_cast<float>(cnt);
    float* o = part + (ng * chunks + ch) * 3;
    o[0] = n;
    o[1] = cnt > 0 ? shift + s1 / n : 0.f;
    o[2] = cnt > 0 ? fmaxf(s2 - s1 * s1 / n, 0.f) : 0.f;
  }
}

// Merges `chunks` (count, mean, M2) triples of each group into one (Chan et
// al. pairwise update, fixed order, fp64).  One thread per group.
__global__ void gn_merge_kernel(const float* __restrict__ part, float* __restrict__ out,
                                int64_t groups, int chunks) {
  const int64_t ng = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (ng >= groups) return;
  double n = 0.0, mean = 0.0, m2 = 0.0;
  for (int c = 0; c < chunks; ++c) {
    const float* p = part + (ng * chunks + c) * 3;
    const double nb = p[0];
    if (nb <= 0.0) continue;
    const double mb = p[1], qb = p[2];
    const double tot = n + nb;
    const double d = mb - mean;
    mean += d * nb / tot;
    m2 += qb + d * d * n * nb / tot;
    n = tot;
  }
  out[ng * 3 + 0] = static_cast<float>(n);
  out[ng * 3 + 1] = static_cast<float>(mean);
  out[ng * 3 + 2] = static_cast<float>(m2);
}

// Merges per-rank triples parts[r][g][3] in rank order (fp64) -> out[g][3]:
// the statistics exchange of a sharded GroupNorm (every rank runs it on the
// same gathered array and gets identical statistics).  One thread per group.
__global__ void gn_merge_ranks_kernel(const float* __restrict__ parts, float* __restrict__ out,
                                      int64_t groups, int ranks) {
  const int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (g >= groups) return;
  double n = 0.0, mean = 0.0, m2 = 0.0;
  for (int r = 0; r < ranks; ++r) {
    const float* p = parts + (static_cast<int64_t>(r) * groups + g) * 3;
    const double nb = p[0];
    if (nb <= 0.0) continue;
    const double tot = n + nb;
    const double d = static_cast<double>(p[1]) - mean;
    mean += d * nb / tot;
    m2 += static_cast<double>(p[2]) + d * d * n * nb / tot;
    n = tot;
  }
  out[g * 3 + 0] = static_cast<float>(n);
  out[g * 3 + 1] = static_cast<float>(mean);
  out[g * 3 + 2] = static_cast<float>(m2);
}

// ------------------------------------------------------- split: apply ----
// y = (x - mean) * rstd * gamma + beta, optional SiLU; NC[S] layout out.
template <typename T, bool VEC, bool SILU>
__global__ void __launch_bounds__(256)
gn_apply_kernel(const T* __restrict__ x, const float* __restrict__ stats,
                const void* __restrict__ gamma, const void* __restrict__ beta,
                T* __restrict__ y, int affine_dt, int64_t S, int G, int Cg, float eps,
                int64_t chunk, int chunks) {
  const int64_t ng = blockIdx.x / chunks;
  const int ch = blockIdx.x % chunks;
  const int64_t M = static_cast<int64_t>(Cg) * S;
  const int64_t beg = static_cast<int64_t>(ch) * chunk;
  const int64_t cnt = max64(0, min64(chunk, M - beg));
  const float n = stats[ng * 3 + 0];
  const float mean = stats[ng * 3 + 1];
  const float rstd = 1.0f / sqrtf(stats[ng * 3 + 2] / n + eps);
  const int c0 = static_cast<int>(ng % G) * Cg;
  const T* src = x + ng * M + beg;
  T* dst = y + ng * M + beg;
  constexpr int V = Vec16<T>::N;
  if (VEC) {
    const int64_t nv = cnt / V;
    for (int64_t i = threadIdx.x; i < nv; i += 256) {
      const int64_t idx = beg + i * V;
      const int c = c0 + static_cast<int>(idx / S);
      const float a = gamma ? rstd * load_param(gamma, affine_dt, c) : rstd;
      const float b = beta ? load_param(beta, affine_dt, c) : 0.f;
      float v[V];
      unpack16<T>(ld_stream16(reinterpret_cast<const uint4*>(src) + i), v);
#pragma unroll
      for (int e = 0; e < V; ++e) {
        v[e] = fmaf(v[e] - mean, a, b);
        if (SILU) v[e] = silu(v[e]);
      }
      st_stream16(reinterpret_cast<uint4*>(dst) + i, pack16<T>(v));
    }
  } else {
    for (int64_t i = threadIdx.x; i < cnt; i += 256) {
      const int c = c0 + static_cast<int>((beg + i) / S);
      const float a = gamma ? rstd * load_param(gamma, affine_dt, c) : rstd;
      const float b = beta ? load_param(beta, affine_dt, c) : 0.f;
      float v = fmaf(to_f32(src[i]) - mean, a, b);
      if (SILU) v = silu(v);
      dst[i] = from_f32<T>(v);
    }
  }
}

// Normalise (+SiLU) and transpose NC[S] -> N[S]C in one pass: the conv3d
// operand producer of the fused GroupNorm -> SiLU -> conv3d path.  Tile of
// 32 channels x 64 positions through shared memory; grid (S/64, C/32, N).
template <typename T, bool SILU>
__global__ void __launch_bounds__(256)
gn_apply_cl_kernel(const T* __restrict__ x, const float* __restrict__ stats,
                   const void* __restrict__ gamma, const void* __restrict__ beta,
                   T* __restrict__ y, int affine_dt, int64_t C, int64_t S, int G, int Cg,
                   float eps) {
  __shared__ float tile[32][65];
  pdl_launch_dependents();  // the consuming conv kernel's prologue may overlap
  const int64_t n = blockIdx.z;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
  for (int cc = ty; cc < 32; cc += 4) {
    const int64_t c = c0 + cc;
    const int64_t p = p0 + tx;
    float v = 0.f;
    if (c < C && p < S) {
      const int64_t ng = n * G + c / Cg;
      const float cntf = stats[ng * 3 + 0];
      const float mean = stats[ng * 3 + 1];
      const float rstd = 1.0f / sqrtf(stats[ng * 3 + 2] / cntf + eps);
      const float a = gamma ? rstd * load_param(gamma, affine_dt, c) : rstd;
      const float b = beta ? load_param(beta, affine_dt, c) : 0.f;
      v = fmaf(to_f32(x[(n * C + c) * S + p]) - mean, a, b);
      if (SILU) v = silu(v);
    }
    tile[cc][tx] = v;
  }
  __syncthreads();
  const int lc = threadIdx.x & 31, lp = threadIdx.x >> 5;  // 32 x 8
  for (int pp = lp; pp < 64; pp += 8) {
    const int64_t p = p0 + pp, c = c0 + lc;
    if (p < S && c < C) y[(n * S + p) * C + c] = from_f32<T>(tile[lc][pp]);
  }
}

// -------------------------------------------- two-pass, L2-resident ----
// For tensors that fit in L2 (126 MB): pass 1 reads x from HBM once, marking
// the lines evict_last, and writes per-chunk shifted sums; pass 2 re-reads x
// (now from L2), merges its group's partial sums in fp64, and streams y out.
// HBM traffic stays at one read and one write of the tensor, and no cluster
// lock-step is needed.  Each thread moves kL2Vec 16-byte vectors per pass,
// all loads issued before the first use.
constexpr int kL2Threads = 256;
constexpr int kL2Vec = 8;
constexpr int kL2MaxCh = 1024;   // channels of one chunk staged in shared memory

__device__ __forceinline__ uint64_t l2_policy_evict_last(float fraction) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, %1;" : "=l"(pol) : "f"(fraction));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint4 ld16_hint(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ void st16_hint(void* p, const uint4& r, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.u32 [%0], {%1, %2, %3, %4}, %5;"
               ::"l"(p), "r"(r.x), "r"(r.y), "r"(r.z), "r"(r.w), "l"(pol)
               : "memory");
}

// Pass 1: one CTA per (group, chunk of kL2Threads * kL2Vec vectors).  Sums
// are shifted by the group's first element (the same shift for every chunk
// of a group, so the merge is a plain fp64 sum).
template <typename T>
__global__ void __launch_bounds__(kL2Threads)
gn_l2_stats_kernel(const T* __restrict__ x, float2* __restrict__ part, int64_t M, int chunks,
                   float keep_fraction) {
  constexpr int V = Vec16<T>::N;
  constexpr int64_t kChunk = static_cast<int64_t>(kL2Threads) * kL2Vec * V;
  __shared__ float scratch[33];
  const int64_t ng = blockIdx.x / chunks;
  const int ch = blockIdx.x % chunks;
  const T* grp = x + ng * M;
  const int64_t beg = static_cast<int64_t>(ch) * kChunk;
  const uint64_t pol = l2_policy_evict_last(keep_fraction);
  uint4 r[kL2Vec];
#pragma unroll
  for (int u = 0; u < kL2Vec; ++u) {
    const int64_t e = beg + (static_cast<int64_t>(u) * kL2Threads + threadIdx.x) * V;
    if (e < M) r[u] = ld16_hint(grp + e, pol);
  }
  const float shift = to_f32(grp[0]);
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int u = 0; u < kL2Vec; ++u) {
    const int64_t e = beg + (static_cast<int64_t>(u) * kL2Threads + threadIdx.x) * V;
    if (e < M) {
      float v[V];
      unpack16<T>(r[u], v);
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float d = v[k] - shift;
        s1 += d;
        s2 = fmaf(d, d, s2);
      }
    }
  }
  s1 = block_sum<kL2Threads>(s1, scratch);
  s2 = block_sum<kL2Threads>(s2, scratch);
  if (threadIdx.x == 0) part[ng * chunks + ch] = make_float2(s1, s2);
  pdl_launch_dependents();
}

// Pass 2: same chunking, walked in reverse (the chunks pass 1 read last are
// the likeliest still in L2).  The x loads are issued before waiting on pass 1
// (x is not written by it), so they overlap pass 1's tail.  The channels the
// chunk spans get their gamma / beta staged in shared memory once.
template <typename T, bool SILU>
__global__ void __launch_bounds__(kL2Threads, 4)
gn_l2_apply_kernel(const T* __restrict__ x, const float2* __restrict__ part,
                   const void* __restrict__ gamma, const void* __restrict__ beta,
                   T* __restrict__ y, int affine_dt, int64_t S, int G, int Cg, int64_t M,
                   int chunks, float eps) {
  constexpr int V = Vec16<T>::N;
  constexpr int64_t kChunk = static_cast<int64_t>(kL2Threads) * kL2Vec * V;
  __shared__ float stat[2];
  __shared__ float sG[kL2MaxCh], sB[kL2MaxCh];
  const int64_t t = static_cast<int64_t>(gridDim.x) - 1 - blockIdx.x;
  const int64_t ng = t / chunks;
  const int ch = static_cast<int>(t % chunks);
  const T* grp = x + ng * M;
  T* out = y + ng * M;
  const int64_t beg = static_cast<int64_t>(ch) * kChunk;
  const uint64_t pol = l2_policy_evict_first();
  uint4 r[kL2Vec];
#pragma unroll
  for (int u = 0; u < kL2Vec; ++u) {
    const int64_t e = beg + (static_cast<int64_t>(u) * kL2Threads + threadIdx.x) * V;
    if (e < M) r[u] = ld16_hint(grp + e, pol);
  }
  // Channels [c_lo, c_hi] of the group hold this chunk.
  const int64_t last = min64(M, beg + kChunk) - 1;
  const int c_lo = static_cast<int>(beg / S);
  const int nch = static_cast<int>(last / S) - c_lo + 1;
  const bool staged = nch <= kL2MaxCh;
  const int c0 = static_cast<int>(ng % G) * Cg;
  if (staged) {
    for (int c = threadIdx.x; c < nch; c += kL2Threads) {
      sG[c] = gamma ? load_param(gamma, affine_dt, c0 + c_lo + c) : 1.f;
      sB[c] = beta ? load_param(beta, affine_dt, c0 + c_lo + c) : 0.f;
    }
  }
  pdl_wait();
  if (threadIdx.x < 32) {
    // Fixed-order fp64 merge of the group's partial sums (lane-strided, then
    // a butterfly): every CTA of the group computes identical statistics.
    double a = 0.0, b = 0.0;
    for (int c = threadIdx.x; c < chunks; c += 32) {
      const float2 q = part[ng * chunks + c];
      a += q.x;
      b += q.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (threadIdx.x == 0) {
      const double n = static_cast<double>(M);
      const double mean_d = a / n;
      const double var = fmax(b / n - mean_d * mean_d, 0.0);
      stat[0] = static_cast<float>(mean_d + static_cast<double>(to_f32(grp[0])));
      stat[1] = 1.0f / sqrtf(static_cast<float>(var) + eps);
    }
  }
  __syncthreads();
  const float mean = stat[0], rstd = stat[1];
  // Channel of this thread's first vector; later vectors are kL2Threads * V
  // elements further on.
  const int64_t e0 = beg + static_cast<int64_t>(threadIdx.x) * V;
  int64_t q = e0 / S, rem = e0 - q * S;
  constexpr int64_t kStep = static_cast<int64_t>(kL2Threads) * V;
#pragma unroll
  for (int u = 0; u < kL2Vec; ++u) {
    const int64_t e = e0 + u * kStep;
    if (u > 0) {
      rem += kStep;
      if (rem >= S) {
        if (rem < 2 * S) {
          rem -= S;
          q += 1;
        } else {
          q += rem / S;
          rem %= S;
        }
      }
    }
    if (e < M) {
      const int c = static_cast<int>(q);
      float a, b;
      if (staged) {
        a = rstd * sG[c - c_lo];
        b = sB[c - c_lo];
      } else {
        a = gamma ? rstd * load_param(gamma, affine_dt, c0 + c) : rstd;
        b = beta ? load_param(beta, affine_dt, c0 + c) : 0.f;
      }
      float v[V];
      unpack16<T>(r[u], v);
#pragma unroll
      for (int k = 0; k < V; ++k) {
        v[k] = fmaf(v[k] - mean, a, b);
        if (SILU) v[k] = silu(v[k]);
      }
      st16_hint(out + e, pack16<T>(v), pol);
    }
  }
}

// Channels-last normalise (+SiLU) with the transposition in registers (16-bit
// types, C % 8 == 0, S % 8 == 0, aligned pointers).  A thread owns an
// 8-channel x 8-position block: eight 16-byte loads (one per channel row),
// normalise, an 8 x 8 transpose of 16-bit values by byte permutes, eight
// 16-byte stores (8 consecutive channels of one position).  A warp holds CGW
// channel groups x 32 / CGW position blocks, so a load instruction reads
// whole 32-byte sectors of CGW channel rows and a store instruction writes
// 16 * CGW contiguous bytes of each position's channel vector.  A CTA (8
// warps) keeps its 8 * CGW channels' (mean, scale, shift) in shared memory
// and walks `tiles` position tiles, the next tile's rows requested before
// the current one is processed.  (Measured at the cfg 5 shape: 116 us
// against 212 us for a shared-memory tile transpose it replaced; a plain copy
// of the same bytes takes 84 us.)
template <typename T, int CGW, bool SILU>
__global__ void __launch_bounds__(256)
gn_apply_clt_kernel(const T* __restrict__ x, const float* __restrict__ stats,
                    const void* __restrict__ gamma, const void* __restrict__ beta,
                    T* __restrict__ y, int affine_dt, int64_t C, int64_t S, int G, int Cg,
                    float eps, int tiles) {
  static_assert(sizeof(T) == 2, "16-bit elements");
  constexpr int PB = 32 / CGW;               // position blocks per warp
  constexpr int TILE_P = 8 * PB * 8;         // positions per CTA tile (8 warps)
  __shared__ float4 coef[8 * CGW];           // mean, scale, shift per channel of the tile
  pdl_launch_dependents();                   // the consuming conv kernel's prologue may overlap
  const int64_t n = blockIdx.z;
  const int64_t c_tile = static_cast<int64_t>(blockIdx.y) * 8 * CGW;
  if (threadIdx.x < 8 * CGW) {
    const int64_t c = c_tile + threadIdx.x;
    float4 k = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < C) {
      const int64_t ng = n * G + c / Cg;
      const float cnt = stats[ng * 3 + 0];
      k.x = stats[ng * 3 + 1];
      const float rstd = rsqrtf(stats[ng * 3 + 2] / cnt + eps);
      k.y = gamma ? rstd * load_param(gamma, affine_dt, c) : rstd;
      k.z = beta ? load_param(beta, affine_dt, c) : 0.f;
    }
    // Stored channel-within-group major, so that the lanes of a warp (one
    // channel group each) read consecutive entries below.
    coef[(threadIdx.x & 7) * CGW + (threadIdx.x >> 3)] = k;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cg = lane % CGW, pb = lane / CGW;
  const int64_t c0 = c_tile + 8 * cg;
  if (c0 >= C) return;
  float4 k[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) k[i] = coef[i * CGW + cg];
  const T* xr = x + (n * C + c0) * S;
  T* yn = y + n * S * C + c0;
  auto pos = [&](int t) {
    return (static_cast<int64_t>(blockIdx.x) * tiles + t) * TILE_P + (warp * PB + pb) * 8;
  };
  uint4 nx[8];
  if (pos(0) < S) {
#pragma unroll
    for (int i = 0; i < 8; ++i) nx[i] = ld_stream16(xr + i * S + pos(0));
  }
  for (int t = 0; t < tiles; ++t) {
    const int64_t p = pos(t);
    if (p >= S) break;
    uint4 r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = nx[i];
    if (t + 1 < tiles && pos(t + 1) < S) {
#pragma unroll
      for (int i = 0; i < 8; ++i) nx[i] = ld_stream16(xr + i * S + pos(t + 1));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float f[8];
      unpack16<T>(r[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        f[e] = fmaf(f[e] - k[i].x, k[i].y, k[i].z);
        if (SILU) f[e] = silu(f[e]);
      }
      r[i] = pack16<T>(f);
    }
    // r[i].word j = positions (2j, 2j+1) of channel i  ->  o[e].word m =
    // channels (2m, 2m+1) of position e.
    uint32_t o[8][4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t a[4] = {r[2 * m].x, r[2 * m].y, r[2 * m].z, r[2 * m].w};
      const uint32_t b[4] = {r[2 * m + 1].x, r[2 * m + 1].y, r[2 * m + 1].z, r[2 * m + 1].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[2 * j][m] = __byte_perm(a[j], b[j], 0x5410);
        o[2 * j + 1][m] = __byte_perm(a[j], b[j], 0x7632);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e)
      st_stream16(yn + (p + e) * C, make_uint4(o[e][0], o[e][1], o[e][2], o[e][3]));
  }
}

// ----------------------------------------------------------- host side ---
struct GnShape {
  int64_t N, C, S, G, Cg, M, groups;
};

int check_shape(int64_t N, int64_t C, int64_t S, int64_t G, GnShape* sh) {
  if (N <= 0 || C <= 0 || S <= 0 || G <= 0) return fail_arg("non-positive GroupNorm size");
  if (C % G != 0) return fail_arg("C must be divisible by num_groups");
  sh->N = N;
  sh->C = C;
  sh->S = S;
  sh->G = G;
  sh->Cg = C / G;
  sh->M = sh->Cg * S;
  sh->groups = N * G;
  return B200_OK;
}

// Split-path chunking: ~64K elements per CTA, at least one chunk.
int64_t split_chunk(const GnShape& sh, int V) {
  int64_t chunk = 65536;
  if (sh.M < chunk) chunk = sh.M;
  chunk = (chunk + V - 1) / V * V;
  return chunk;
}

template <typename T>
bool vec_ok(const void* x, const void* y, const GnShape& sh) {
  constexpr int V = Vec16<T>::N;
  return aligned16(x) && (y == nullptr || aligned16(y)) && sh.S % V == 0;
}

template <typename T>
int launch_cluster(const T* x, const void* gamma, const void* beta, T* y, int affine_dt,
                   const GnShape& sh, float eps, int csize, cudaStream_t stream) {
  constexpr int V = Vec16<T>::N;
  const bool vec = vec_ok<T>(x, y, sh);
  int64_t slice = (sh.M + csize - 1) / csize;
  slice = (slice + V - 1) / V * V;
  const int64_t smem = slice * static_cast<int64_t>(sizeof(T));
  if (smem > max_smem_optin() - 4096) return fail_unsupported("group slice exceeds shared memory");
  if (sh.groups * csize > 0x7fffffffLL) return fail_unsupported("grid too large");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sh.groups * csize));
  cfg.blockDim = dim3(kGnThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kern = vec ? gn_cluster_kernel<T, true> : gn_cluster_kernel<T, false>;
  B200_CUDA_CHECK(
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  if (csize > 8)
    B200_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    return fail_unsupported("cluster configuration cannot be scheduled");
  }
  B200_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, x, gamma, beta, y, affine_dt, sh.S,
                                     static_cast<int>(sh.G), static_cast<int>(sh.Cg), eps,
                                     static_cast<int>(slice), csize));
  return B200_OK;
}

template <typename T>
int launch_stats(const T* x, float* stats_out, const GnShape& sh, void* ws, size_t ws_bytes,
                 cudaStream_t stream) {
  constexpr int V = Vec16<T>::N;
  const bool vec = vec_ok<T>(x, nullptr, sh);
  const int64_t chunk = split_chunk(sh, vec ? V : 1);
  const int64_t chunks = (sh.M + chunk - 1) / chunk;
  const size_t need = static_cast<size_t>(sh.groups * chunks * 3) * sizeof(float);
  if (ws_bytes < need || ws == nullptr) return fail_arg("GroupNorm workspace too small");
  if (sh.groups * chunks > 0x7fffffffLL) return fail_unsupported("grid too large");
  float* part = static_cast<float*>(ws);
  const unsigned grid = static_cast<unsigned>(sh.groups * chunks);
  if (vec)
    gn_partial_stats_kernel<T, true><<<grid, 256, 0, stream>>>(x, part, sh.M, chunk, (int)chunks);
  else
    gn_partial_stats_kernel<T, false><<<grid, 256, 0, stream>>>(x, part, sh.M, chunk, (int)chunks);
  B200_LAUNCH_CHECK("gn_partial_stats_kernel");
  gn_merge_kernel<<<static_cast<unsigned>((sh.groups + 127) / 128), 128, 0, stream>>>(
      part, stats_out, sh.groups, static_cast<int>(chunks));
  B200_LAUNCH_CHECK("gn_merge_kernel");
  return B200_OK;
}

size_t stats_ws_bytes(const GnShape& sh, int dtype) {
  // Sized for the scalar chunking (the larger of the two).
  const int64_t chunk = split_chunk(sh, 1);
  const int64_t chunks = (sh.M + chunk - 1) / chunk;
  (void)dtype;
  return static_cast<size_t>(sh.groups * (chunks + 1) * 3) * sizeof(float) + 256;
}

template <typename T>
int launch_apply(const T* x, const float* stats, const void* gamma, const void* beta, T* y,
                 int affine_dt, const GnShape& sh, float eps, bool silu, bool to_cl,
                 cudaStream_t stream) {
  if constexpr (sizeof(T) == 2) {
    if (to_cl && sh.C % 8 == 0 && sh.S % 8 == 0 && aligned16(x) && aligned16(y) &&
        sh.N <= 65535 && (sh.C + 31) / 32 <= 65535 && sh.S / 8 < 0x7fffffffLL) {
      // Register-transpose kernel: channel groups per warp by C.
      const int cgw = sh.C % 128 == 0 ? 16 : (sh.C % 64 == 0 ? 8 : 4);
      const int64_t tile_p = 8 * (32 / cgw) * 8;
      const int tiles = 4;
      const int64_t ptiles = (sh.S + tile_p * tiles - 1) / (tile_p * tiles);
      if (ptiles <= 0x7fffffffLL) {
        dim3 grid(static_cast<unsigned>(ptiles),
                  static_cast<unsigned>((sh.C + 8 * cgw - 1) / (8 * cgw)),
                  static_cast<unsigned>(sh.N));
#define B200_CLT(CGW, SL)                                                                   \
  gn_apply_clt_kernel<T, CGW, SL><<<grid, 256, 0, stream>>>(x, stats, gamma, beta, y, affine_dt, \
                                                            sh.C, sh.S, (int)sh.G, (int)sh.Cg, \
                                                            eps, tiles)
        if (cgw == 16) {
          if (silu) B200_CLT(16, true); else B200_CLT(16, false);
        } else if (cgw == 8) {
          if (silu) B200_CLT(8, true); else B200_CLT(8, false);
        } else {
          if (silu) B200_CLT(4, true); else B200_CLT(4, false);
        }
#undef B200_CLT
        B200_LAUNCH_CHECK("gn_apply_clt_kernel");
        return B200_OK;
      }
    }
  }
  if (to_cl) {
    if (sh.S > 0x7fffffffLL * 64 || (sh.C + 31) / 32 > 65535 || sh.N > 65535)
      return fail_unsupported("channels-last apply grid too large");
    dim3 grid(static_cast<unsigned>((sh.S + 63) / 64), static_cast<unsigned>((sh.C + 31) / 32),
              static_cast<unsigned>(sh.N));
    if (silu)
      gn_apply_cl_kernel<T, true><<<grid, 256, 0, stream>>>(x, stats, gamma, beta, y, affine_dt,
                                                            sh.C, sh.S, (int)sh.G, (int)sh.Cg, eps);
    else
      gn_apply_cl_kernel<T, false><<<grid, 256, 0, stream>>>(x, stats, gamma, beta, y, affine_dt,
                                                             sh.C, sh.S, (int)sh.G, (int)sh.Cg, eps);
    B200_LAUNCH_CHECK("gn_apply_cl_kernel");
    return B200_OK;
  }
  constexpr int V = Vec16<T>::N;
  const bool vec = vec_ok<T>(x, y, sh);
  const int64_t chunk = split_chunk(sh, vec ? V : 1);
  const int64_t chunks = (sh.M + chunk - 1) / chunk;
  if (sh.groups * chunks > 0x7fffffffLL) return fail_unsupported("grid too large");
  const unsigned grid = static_cast<unsigned>(sh.groups * chunks);
  const int G = static_cast<int>(sh.G), Cg = static_cast<int>(sh.Cg), nc = static_cast<int>(chunks);
  if (vec && silu)
    gn_apply_kernel<T, true, true><<<grid, 256, 0, stream>>>(x, stats, gamma, beta, y, affine_dt, sh.S, G, Cg, eps, chunk, nc);
  else if (vec)
    gn_apply_kernel<T, true, false><<<grid, 256, 0, stream>>>(x, stats, gamma, beta, y, affine_dt, sh.S, G, Cg, eps, chunk, nc);
  else if (silu)
    gn_apply_kernel<T, false, true><<<grid, 256, 0, stream>>>(x, stats, gamma, beta, y, affine_dt, sh.S, G, Cg, eps, chunk, nc);
  else
    gn_apply_kernel<T, false, false><<<grid, 256, 0, stream>>>(x, stats, gamma, beta, y, affine_dt, sh.S, G, Cg, eps, chunk, nc);
  B200_LAUNCH_CHECK("gn_apply_kernel");
  return B200_OK;
}

// Two-pass L2-resident path (variant 2).  Declines (> 0) unless x/y are
// 16-byte aligned with S a multiple of the vector width.
constexpr double kL2KeepBytes = 80e6;  // evict_last budget, well inside the 126 MB L2

int64_t l2_chunks(const GnShape& sh, size_t esize) {
  const int64_t chunk = static_cast<int64_t>(kL2Threads) * kL2Vec * (16 / static_cast<int64_t>(esize));
  return (sh.M + chunk - 1) / chunk;
}

size_t l2_ws_bytes(const GnShape& sh, size_t esize) {
  return static_cast<size_t>(sh.groups * l2_chunks(sh, esize)) * sizeof(float2);
}

// Whole tensor within the L2 keep budget: the re-read of pass 2 hits L2.
bool l2_fits(const GnShape& sh, size_t esize) {
  return static_cast<double>(sh.N) * sh.C * sh.S * esize <= kL2KeepBytes;
}

template <typename T>
int launch_l2(const T* x, const void* gamma, const void* beta, T* y, int affine_dt,
              const GnShape& sh, float eps, bool silu, void* ws, size_t ws_bytes,
              cudaStream_t stream) {
  if (!vec_ok<T>(x, y, sh)) return fail_unsupported("two-pass GroupNorm needs 16-byte rows");
  const int64_t chunks = l2_chunks(sh, sizeof(T));
  const int64_t blocks = sh.groups * chunks;
  if (blocks > 0x7fffffffLL) return fail_unsupported("grid too large");
  if (ws == nullptr || ws_bytes < l2_ws_bytes(sh, sizeof(T)))
    return fail_arg("GroupNorm workspace too small");
  float2* part = static_cast<float2*>(ws);
  const double bytes = static_cast<double>(sh.N) * sh.C * sh.S * sizeof(T);
  const float keep = static_cast<float>(std::min(1.0, kL2KeepBytes / bytes));
  const unsigned grid = static_cast<unsigned>(blocks);
  gn_l2_stats_kernel<T><<<grid, kL2Threads, 0, stream>>>(x, part, sh.M, (int)chunks, keep);
  B200_LAUNCH_CHECK("gn_l2_stats_kernel");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kL2Threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kern = silu ? gn_l2_apply_kernel<T, true> : gn_l2_apply_kernel<T, false>;
  const float2* cpart = part;
  B200_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, x, cpart, gamma, beta, y, affine_dt, sh.S,
                                     static_cast<int>(sh.G), static_cast<int>(sh.Cg), sh.M,
                                     static_cast<int>(chunks), eps));
  return B200_OK;
}

// ------------------------------------------------------ streaming path ---
// Variant 3: three kernels on a persistent grid of 256-thread CTAs.
//  1. gn_s_stats_kernel: chunks of kSChunk elements (4 16-byte vectors per
//     thread) walked with a grid stride; the next chunk's loads are issued
//     before the current chunk is reduced, so every thread keeps 8 vectors in
//     flight.  Loads mark x evict_last (the apply pass re-reads it from L2).
//     Per chunk: sums shifted by the group's first element -> part[g][chunk].
//  2. gn_s_coef_kernel: one warp per (n, g) merges its chunks in fp64 and
//     writes each channel's (scale, shift) = (rstd gamma, beta - mean rstd
//     gamma).
//  3. gn_s_apply_kernel: y = x * scale_c + shift_c (+ SiLU) over the whole
//     tensor as 16-byte vectors, grid stride walked from the end (the lines
//     pass 1 read last are the likeliest still in L2), 4 vectors in flight
//     per thread, streaming stores.
// 2 and 3 are launched with programmatic dependent launch; 3 issues its
// first loads of x before waiting.
constexpr int kSThreads = 256;
constexpr int kSVec = 4;   // 16-byte vectors per thread per chunk / iteration

template <typename T>
constexpr int64_t s_chunk() { return static_cast<int64_t>(kSThreads) * kSVec * Vec16<T>::N; }
inline int64_t s_chunk_elems(size_t esize) {
  return static_cast<int64_t>(kSThreads) * kSVec * (16 / static_cast<int64_t>(esize));
}

template <typename T>
__global__ void __launch_bounds__(kSThreads)
gn_s_stats_kernel(const T* __restrict__ x, float2* __restrict__ part, int64_t M, int chunks,
                  int64_t total_chunks, float keep_fraction) {
  constexpr int V = Vec16<T>::N;
  constexpr int64_t kChunk = s_chunk<T>();
  __shared__ float2 red[kSThreads / 32];
  const uint64_t pol = l2_policy_evict_last(keep_fraction);
  uint4 cur[kSVec], nxt[kSVec];
  auto issue = [&](int64_t c, uint4 (&r)[kSVec]) {
    const int64_t g = c / chunks, ch = c - (c / chunks) * chunks;
    const T* grp = x + g * M;
#pragma unroll
    for (int u = 0; u < kSVec; ++u) {
      const int64_t e = ch * kChunk + (static_cast<int64_t>(u) * kSThreads + threadIdx.x) * V;
      r[u] = e < M ? ld16_hint(grp + e, pol) : make_uint4(0, 0, 0, 0);
    }
  };
  int64_t c = blockIdx.x;
  pdl_wait();  // launched with programmatic serialisation behind the previous kernel
  if (c < total_chunks) issue(c, cur);
  for (; c < total_chunks; c += gridDim.x) {
    const int64_t cn = c + gridDim.x;
    if (cn < total_chunks) issue(cn, nxt);
    const int64_t g = c / chunks, ch = c - (c / chunks) * chunks;
    const float shift = to_f32(x[g * M]);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int u = 0; u < kSVec; ++u) {
      const int64_t e = ch * kChunk + (static_cast<int64_t>(u) * kSThreads + threadIdx.x) * V;
      if (e < M) {
        float v[V];
        unpack16<T>(cur[u], v);
#pragma unroll
        for (int k = 0; k < V; ++k) {
          const float d = v[k] - shift;
          s1 += d;
          s2 = fmaf(d, d, s2);
        }
      }
    }
    // One block reduction of the (sum, sum of squares) pair.
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(s1, s2);
    __syncthreads();
    if (threadIdx.x == 0) {
      float2 tot = red[0];
#pragma unroll
      for (int w = 1; w < kSThreads / 32; ++w) {
        tot.x += red[w].x;
        tot.y += red[w].y;
      }
      part[c] = tot;
    }
#pragma unroll
    for (int u = 0; u < kSVec; ++u) cur[u] = nxt[u];
    __syncthreads();  // red[] is rewritten by the next chunk
  }
  pdl_launch_dependents();
}

// One warp per (n, g): fixed-order fp64 merge of the group's chunk sums,
// then per channel scale = rstd * gamma, shift = beta - mean * scale.
__global__ void __launch_bounds__(128)
gn_s_coef_kernel(const float2* __restrict__ part, const void* __restrict__ gamma,
                 const void* __restrict__ beta, int affine_dt, float2* __restrict__ coef,
                 const void* __restrict__ x, int xdt, int64_t groups, int G, int Cg, int64_t M,
                 int chunks, float eps) {
  pdl_wait();
  const int64_t ng = blockIdx.x * 4LL + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (ng >= groups) return;
  double a = 0.0, b = 0.0;
  for (int c = lane; c < chunks; c += 32) {
    const float2 q = part[ng * chunks + c];
    a += q.x;
    b += q.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const double n = static_cast<double>(M);
  const double mean_d = a / n;
  const double var = fmax(b / n - mean_d * mean_d, 0.0);
  const float mean = static_cast<float>(mean_d + static_cast<double>(load_param(x, xdt, ng * M)));
  const float rstd = 1.0f / sqrtf(static_cast<float>(var) + eps);
  const int64_t c0 = (ng % G) * Cg;
  for (int j = lane; j < Cg; j += 32) {
    const float gm = gamma ? load_param(gamma, affine_dt, c0 + j) : 1.f;
    const float bt = beta ? load_param(beta, affine_dt, c0 + j) : 0.f;
    const float sc = rstd * gm;
    coef[(ng / G) * G * Cg + c0 + j] = make_float2(sc, bt - mean * sc);
  }
  pdl_launch_dependents();
}

template <typename T, bool SILU>
__global__ void __launch_bounds__(kSThreads)
gn_s_apply_kernel(const T* __restrict__ x, const float2* __restrict__ coef, T* __restrict__ y,
                  int nvec, FastDiv per_row) {
  constexpr int V = Vec16<T>::N;
  const uint64_t pol = l2_policy_evict_first();
  const int step = static_cast<int>(gridDim.x) * kSThreads * kSVec;
  // Walk from the end of the tensor: vector index i = last - (base + u * stride).
  const int last = nvec - 1;
  int base = static_cast<int>(blockIdx.x) * kSThreads * kSVec + static_cast<int>(threadIdx.x);
  uint4 r[kSVec];
#pragma unroll
  for (int u = 0; u < kSVec; ++u) {
    const int i = last - (base + u * kSThreads);
    if (i >= 0) r[u] = ld16_hint(x + static_cast<int64_t>(i) * V, pol);
  }
  pdl_wait();
  for (; base <= last; base += step) {
    uint4 q[kSVec];
#pragma unroll
    for (int u = 0; u < kSVec; ++u) {   // next iteration's loads first
      const int i = last - (base + step + u * kSThreads);
      if (i >= 0) q[u] = ld16_hint(x + static_cast<int64_t>(i) * V, pol);
    }
#pragma unroll
    for (int u = 0; u < kSVec; ++u) {
      const int i = last - (base + u * kSThreads);
      if (i >= 0) {
        // (n, c) row of this vector: S / V vectors per row (S % V == 0).
        const float2 k = coef[fast_div(static_cast<uint32_t>(i), per_row)];
        float v[V];
        unpack16<T>(r[u], v);
#pragma unroll
        for (int e = 0; e < V; ++e) {
          v[e] = fmaf(v[e], k.x, k.y);
          if (SILU) v[e] = silu(v[e]);
        }
        st_stream16(y + static_cast<int64_t>(i) * V, pack16<T>(v));
      }
    }
#pragma unroll
    for (int u = 0; u < kSVec; ++u) r[u] = q[u];
  }
}

// (count, mean, M2) per group from the streaming statistics pass's shifted
// chunk sums (one warp per group, fixed-order fp64 merge): the
// b200_gn_partial_stats output for 16-byte rows.
__global__ void __launch_bounds__(128)
gn_s_triples_kernel(const float2* __restrict__ part, const void* __restrict__ x, int xdt,
                    float* __restrict__ out, int64_t groups, int64_t M, int chunks) {
  pdl_wait();
  const int64_t ng = blockIdx.x * 4LL + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (ng >= groups) return;
  double a = 0.0, b = 0.0;
  for (int c = lane; c < chunks; c += 32) {
    const float2 q = part[ng * chunks + c];
    a += q.x;
    b += q.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if (lane == 0) {
    const double n = static_cast<double>(M);
    const double md = a / n;
    out[ng * 3 + 0] = static_cast<float>(n);
    out[ng * 3 + 1] = static_cast<float>(md + static_cast<double>(load_param(x, xdt, ng * M)));
    out[ng * 3 + 2] = static_cast<float>(fmax(b - a * md, 0.0));
  }
}

// b200_gn_partial_stats for 16-byte rows: the persistent streaming
// statistics kernel (two chunks of loads in flight per thread), then the
// triples.  Declines (> 0) for other shapes.
template <typename T>
int launch_stats_stream(const T* x, float* stats_out, const GnShape& sh, void* ws,
                        size_t ws_bytes, cudaStream_t stream) {
  if (!vec_ok<T>(x, nullptr, sh)) return fail_unsupported("streaming statistics need 16-byte rows");
  constexpr int64_t kChunk = s_chunk<T>();
  const int64_t chunks = (sh.M + kChunk - 1) / kChunk;
  const int64_t total = sh.groups * chunks;
  if (chunks > 0x7fffffffLL || total > 0x7fffffffLL) return fail_unsupported("too many chunks");
  if (ws == nullptr || ws_bytes < static_cast<size_t>(total) * sizeof(float2))
    return fail_unsupported("workspace too small for the streaming statistics");
  float2* part = static_cast<float2*>(ws);
  const double bytes = static_cast<double>(sh.N) * sh.C * sh.S * sizeof(T);
  const float keep = static_cast<float>(std::min(1.0, kL2KeepBytes / bytes));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c1 = {};
  c1.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(total, 8LL * sm_count())));
  c1.blockDim = dim3(kSThreads);
  c1.stream = stream;
  c1.attrs = attr;
  c1.numAttrs = 1;
  B200_CUDA_CHECK(cudaLaunchKernelEx(&c1, gn_s_stats_kernel<T>, x, part, sh.M,
                                     static_cast<int>(chunks), total, keep));
  cudaLaunchConfig_t c2 = c1;
  c2.gridDim = dim3(static_cast<unsigned>((sh.groups + 3) / 4));
  c2.blockDim = dim3(128);
  const int xdt = sizeof(T) == 4 ? B200_DTYPE_F32
                                 : (std::is_same<T, __half>::value ? B200_DTYPE_F16 : B200_DTYPE_BF16);
  const float2* cpart = part;
  B200_CUDA_CHECK(cudaLaunchKernelEx(&c2, gn_s_triples_kernel, cpart,
                                     static_cast<const void*>(x), xdt, stats_out, sh.groups,
                                     sh.M, static_cast<int>(chunks)));
  return B200_OK;
}

size_t s_ws_bytes(const GnShape& sh, size_t esize) {
  const int64_t chunk = static_cast<int64_t>(kSThreads) * kSVec * (16 / static_cast<int64_t>(esize));
  const int64_t chunks = (sh.M + chunk - 1) / chunk;
  const size_t part = static_cast<size_t>(sh.groups * chunks) * sizeof(float2);
  return (part + 255) / 256 * 256 + static_cast<size_t>(sh.N * sh.C) * sizeof(float2);
}

template <typename T>
int launch_stream(const T* x, const void* gamma, const void* beta, T* y, int affine_dt,
                  const GnShape& sh, float eps, bool silu, void* ws, size_t ws_bytes,
                  cudaStream_t stream) {
  if (!vec_ok<T>(x, y, sh)) return fail_unsupported("streaming GroupNorm needs 16-byte rows");
  if (sh.S / Vec16<T>::N >= (1LL << 31)) return fail_unsupported("streaming GroupNorm: rows too long");
  constexpr int64_t kChunk = s_chunk<T>();
  const int64_t chunks = (sh.M + kChunk - 1) / kChunk;
  const int64_t total = sh.groups * chunks;
  if (ws == nullptr || ws_bytes < s_ws_bytes(sh, sizeof(T)))
    return fail_arg("GroupNorm workspace too small");
  if (chunks > 0x7fffffffLL || sh.groups > 0x7fffffffLL) return fail_unsupported("too large");
  float2* part = static_cast<float2*>(ws);
  const size_t part_bytes = (static_cast<size_t>(total) * sizeof(float2) + 255) / 256 * 256;
  float2* coef = reinterpret_cast<float2*>(static_cast<char*>(ws) + part_bytes);
  const double bytes = static_cast<double>(sh.N) * sh.C * sh.S * sizeof(T);
  const float keep = static_cast<float>(std::min(1.0, kL2KeepBytes / bytes));
  const int sms = sm_count();
  const unsigned g1 = static_cast<unsigned>(std::min<int64_t>(total, 8LL * sms));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  {
    cudaLaunchConfig_t c1 = {};
    c1.gridDim = dim3(g1);
    c1.blockDim = dim3(kSThreads);
    c1.stream = stream;
    c1.attrs = attr;
    c1.numAttrs = 1;
    B200_CUDA_CHECK(cudaLaunchKernelEx(&c1, gn_s_stats_kernel<T>, x, part, sh.M,
                                       static_cast<int>(chunks), total, keep));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((sh.groups + 3) / 4));
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int xdt = sizeof(T) == 4 ? B200_DTYPE_F32 : (std::is_same<T, __half>::value ? B200_DTYPE_F16 : B200_DTYPE_BF16);
  const float2* cpart = part;
  B200_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gn_s_coef_kernel, cpart, gamma, beta, affine_dt, coef,
                                     static_cast<const void*>(x), xdt, sh.groups,
                                     static_cast<int>(sh.G), static_cast<int>(sh.Cg), sh.M,
                                     static_cast<int>(chunks), eps));
  constexpr int V = Vec16<T>::N;
  const int64_t nvec = sh.N * sh.C * sh.S / V;
  if (nvec + 2LL * kSThreads * kSVec * 8 * sms >= (1LL << 31))
    return fail_unsupported("streaming GroupNorm: more than 2^31 vectors");
  cudaLaunchConfig_t cfg3 = cfg;
  cfg3.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>((nvec + kSThreads * kSVec - 1) / (kSThreads * kSVec), 8LL * sms)));
  cfg3.blockDim = dim3(kSThreads);
  const float2* ccoef = coef;
  auto kern = silu ? gn_s_apply_kernel<T, true> : gn_s_apply_kernel<T, false>;
  const FastDiv per_row = make_fastdiv(static_cast<uint32_t>(sh.S / V));
  B200_CUDA_CHECK(cudaLaunchKernelEx(&cfg3, kern, x, ccoef, y, static_cast<int>(nvec), per_row));
  return B200_OK;
}

// Smallest power-of-two cluster whose per-CTA slice fits `target` bytes.
int auto_cluster(const GnShape& sh, size_t esize) {
  const int64_t bytes = sh.M * static_cast<int64_t>(esize);
  const int64_t target = 64 * 1024;
  for (int k = 1; k <= 8; k *= 2)
    if ((bytes + k - 1) / k <= target) return k;
  if ((bytes + 15) / 16 <= 200 * 1024) return 16;
  return 0;
}

template <typename T>
int gn_fwd_typed(const void* xv, const void* gamma, const void* beta, void* yv, int affine_dt,
                 const GnShape& sh, float eps, int variant, void* ws, size_t ws_bytes,
                 cudaStream_t stream) {
  const T* x = static_cast<const T*>(xv);
  T* y = static_cast<T*>(yv);
  // Auto: the streaming variant for 16-byte rows that fit the L2 keep budget
  // (measured 35.5-36.0 us vs 36.6 us for the two-kernel L2 variant at cfg 3).
  if (variant == 0 && l2_fits(sh, sizeof(T)) && vec_ok<T>(x, y, sh) &&
      sh.S / Vec16<T>::N < (1LL << 31))
    variant = 3;
  if (variant == 2) return launch_l2<T>(x, gamma, beta, y, affine_dt, sh, eps, false, ws, ws_bytes, stream);
  if (variant == 3)
    return launch_stream<T>(x, gamma, beta, y, affine_dt, sh, eps, false, ws, ws_bytes, stream);
  if (variant == 0) {
    const int k = auto_cluster(sh, sizeof(T));
    if (k > 0) {
      const int rc = launch_cluster<T>(x, gamma, beta, y, affine_dt, sh, eps, k, stream);
      if (rc <= 0) return rc;
    }
    variant = 1;
  }
  if (variant >= 16) {
    const int k = variant - 16;
    if (k != 1 && k != 2 && k != 4 && k != 8 && k != 16)
      return fail_arg("GroupNorm cluster size must be 1, 2, 4, 8 or 16");
    return launch_cluster<T>(x, gamma, beta, y, affine_dt, sh, eps, k, stream);
  }
  if (variant != 1) return fail_arg("unknown GroupNorm variant");
  // Split path: partials + merged stats in the workspace, then apply.
  const int64_t chunk = split_chunk(sh, 1);
  const int64_t chunks = (sh.M + chunk - 1) / chunk;
  const size_t stats_bytes = static_cast<size_t>(sh.groups * 3) * sizeof(float);
  const size_t part_bytes = static_cast<size_t>(sh.groups * chunks * 3) * sizeof(float);
  if (ws == nullptr || ws_bytes < stats_bytes + part_bytes + 16)
    return fail_arg("GroupNorm workspace too small");
  float* stats = static_cast<float*>(ws);
  void* part = static_cast<char*>(ws) + ((stats_bytes + 15) / 16) * 16;
  const int rc = launch_stats<T>(x, stats, sh, part, ws_bytes - ((stats_bytes + 15) / 16) * 16,
                                 stream);
  if (rc != B200_OK) return rc;
  return launch_apply<T>(x, stats, gamma, beta, y, affine_dt, sh, eps, false, false, stream);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

size_t b200_gn_workspace_bytes(int64_t N, int64_t C, int64_t S, int64_t G, int dtype,
                               int variant) {
  GnShape sh;
  if (check_shape(N, C, S, G, &sh) != B200_OK) return 0;
  if (variant >= 16) return 0;
  if (variant == 0 && auto_cluster(sh, dtype_size(dtype)) > 0) {
    // The cluster path may still decline (scheduling); keep the split
    // fallback's scratch available.
  }
  const size_t stats_bytes = ((static_cast<size_t>(sh.groups * 3) * sizeof(float) + 15) / 16) * 16;
  const size_t split = stats_bytes + stats_ws_bytes(sh, dtype);
  const size_t l2 = l2_ws_bytes(sh, dtype_size(dtype));
  const size_t st = s_ws_bytes(sh, dtype_size(dtype));
  return std::max(split, std::max(l2, st));
}

int b200_gn_fwd(const void* x, const void* gamma, const void* beta, void* y, int dtype,
                int affine_dtype, int64_t N, int64_t C, int64_t S, int64_t G, float eps,
                int variant, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !y) return fail_arg("x/y is NULL");
  if (!dtype_ok(dtype) || ((gamma || beta) && !dtype_ok(affine_dtype)))
    return fail_arg("bad dtype");
  GnShape sh;
  int rc = check_shape(N, C, S, G, &sh);
  if (rc != B200_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_DTYPE_F32)
    return gn_fwd_typed<float>(x, gamma, beta, y, affine_dtype, sh, eps, variant, workspace,
                               workspace_bytes, s);
  if (dtype == B200_DTYPE_F16)
    return gn_fwd_typed<__half>(x, gamma, beta, y, affine_dtype, sh, eps, variant, workspace,
                                workspace_bytes, s);
  return gn_fwd_typed<__nv_bfloat16>(x, gamma, beta, y, affine_dtype, sh, eps, variant,
                                     workspace, workspace_bytes, s);
}

size_t b200_gn_stats_workspace_bytes(int64_t N, int64_t C, int64_t S, int64_t G, int dtype) {
  GnShape sh;
  if (check_shape(N, C, S, G, &sh) != B200_OK) return 0;
  const int64_t ck = s_chunk_elems(dtype_size(dtype));
  const size_t stream_bytes =
      static_cast<size_t>(sh.groups * ((sh.M + ck - 1) / ck)) * sizeof(float2);
  return std::max(stats_ws_bytes(sh, dtype), stream_bytes);
}

int b200_gn_partial_stats(const void* x, float* partial_out, int dtype, int64_t N, int64_t C,
                          int64_t S, int64_t G, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (!x || !partial_out) return fail_arg("x/partial_out is NULL");
  if (!dtype_ok(dtype)) return fail_arg("bad dtype");
  GnShape sh;
  int rc = check_shape(N, C, S, G, &sh);
  if (rc != B200_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // 16-byte rows: the persistent streaming pass; otherwise (or when the
  // caller's workspace is sized for the chunked pass only) the chunked one.
  if (dtype == B200_DTYPE_F32)
    rc = launch_stats_stream<float>(static_cast<const float*>(x), partial_out, sh, workspace,
                                    workspace_bytes, s);
  else if (dtype == B200_DTYPE_F16)
    rc = launch_stats_stream<__half>(static_cast<const __half*>(x), partial_out, sh, workspace,
                                     workspace_bytes, s);
  else
    rc = launch_stats_stream<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), partial_out,
                                            sh, workspace, workspace_bytes, s);
  if (rc <= 0) return rc;
  if (dtype == B200_DTYPE_F32)
    return launch_stats<float>(static_cast<const float*>(x), partial_out, sh, workspace,
                               workspace_bytes, s);
  if (dtype == B200_DTYPE_F16)
    return launch_stats<__half>(static_cast<const __half*>(x), partial_out, sh, workspace,
                                workspace_bytes, s);
  return launch_stats<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), partial_out, sh,
                                     workspace, workspace_bytes, s);
}

int b200_gn_merge_ranks(const float* parts, float* out, int64_t ranks, int64_t groups,
                        void* stream) {
  if (!parts || !out) return fail_arg("parts/out is NULL");
  if (ranks <= 0 || groups <= 0 || ranks > 0x7fffffffLL) return fail_arg("bad size");
  const int64_t blocks = (groups + 127) / 128;
  if (blocks > 0x7fffffffLL) return fail_unsupported("grid too large");
  gn_merge_ranks_kernel<<<static_cast<unsigned>(blocks), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      parts, out, groups, static_cast<int>(ranks));
  B200_LAUNCH_CHECK("gn_merge_ranks_kernel");
  return B200_OK;
}

int b200_gn_apply(const void* x, const float* stats, const void* gamma, const void* beta,
                  void* y, int dtype, int affine_dtype, int64_t N, int64_t C, int64_t S,
                  int64_t G, float eps, int silu, int to_channels_last, void* stream) {
  if (!x || !y || !stats) return fail_arg("x/y/stats is NULL");
  if (!dtype_ok(dtype) || ((gamma || beta) && !dtype_ok(affine_dtype)))
    return fail_arg("bad dtype");
  GnShape sh;
  int rc = check_shape(N, C, S, G, &sh);
  if (rc != B200_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_DTYPE_F32)
    return launch_apply<float>(static_cast<const float*>(x), stats, gamma, beta,
                               static_cast<float*>(y), affine_dtype, sh, eps, silu != 0,
                               to_channels_last != 0, s);
  if (dtype == B200_DTYPE_F16)
    return launch_apply<__half>(static_cast<const __half*>(x), stats, gamma, beta,
                                static_cast<__half*>(y), affine_dtype, sh, eps, silu != 0,
                                to_channels_last != 0, s);
  return launch_apply<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), stats, gamma, beta,
                                     static_cast<__nv_bfloat16*>(y), affine_dtype, sh, eps,
                                     silu != 0, to_channels_last != 0, s);
}

}  // extern "C"

// ---------------------------------------------- allocation-free variant ---
// GroupNorm forward for callers that cannot allocate device memory: an
// application whose device memory is owned entirely by its own pool or
// arena (a serving engine's memory planner, a plugin host that forbids
// third-party allocations), or a latency-critical loop where an allocation
// and the synchronisation it can imply are not acceptable.  The per-chunk
// partial statistics and the merged per-group statistics of the split path
// live in the file-scope device array below instead of a caller workspace.
//
// Limits and sharing rules:
//  * kStaticScratchFloats floats (256 KiB) per device, held by every GPU that
//    loads this library until the process exits.  The split path needs
//    3 * N * G * (chunks + 1) floats, chunks = ceil(Cg * S / 65536); calls
//    that need more are rejected with B200_ERR_ARG and a message.
//  * Every call uses the same array.  Each slot a call reads was written
//    earlier by that same call (partials by the statistics kernel, merged
//    statistics by the merge kernel), so nothing has to start at zero and
//    a previous call's leftovers are never read.  Calls whose kernels can
//    overlap on the GPU (different streams without ordering between them)
//    race on the array and must not be issued.
//  * The first call on each device resolves the array's device address
//    with cudaGetSymbolAddress while that device is current; make that
//    first call before any stream capture begins.  The address is resolved
//    again when the device's current context is no longer the one it was
//    resolved in (after a cudaDeviceReset the module is reloaded into a new
//    context); the first call after such a reset also belongs before any
//    capture.
namespace b200 {
namespace {
constexpr int64_t kStaticScratchFloats = 65536;
}  // namespace
}  // namespace b200

static __device__ __align__(256) float g_gn_static_scratch[b200::kStaticScratchFloats];

namespace b200 {
namespace {

// The calling thread's current driver context (nullptr when none is bound
// or the driver entry point is unavailable).
CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(ptr);
  });
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Device address of g_gn_static_scratch on the current device (host code
// cannot use the symbol itself as a device pointer).  Resolved on the first
// call per device and again whenever that device's current context differs
// from the one the address was resolved in (the module is loaded afresh
// into a context re-created after cudaDeviceReset, possibly elsewhere).
// nullptr on failure.
float* static_scratch_address(cudaError_t* err) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  static CUcontext owner[64] = {nullptr};
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr || ctx == nullptr || ctx != owner[dev]) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_gn_static_scratch);
    if (*err != cudaSuccess) return nullptr;
    addr[dev] = static_cast<float*>(p);
    owner[dev] = current_context();   // bound now, if it was not before the lookup
  }
  return addr[dev];
}

template <typename T>
int gn_static_typed(const void* xv, const void* gamma, const void* beta, void* yv, int affine_dt,
                    const GnShape& sh, float eps, float* scratch, cudaStream_t stream) {
  const T* x = static_cast<const T*>(xv);
  T* y = static_cast<T*>(yv);
  const int64_t stats_floats = sh.groups * 3;
  const int64_t stats_pad = (stats_floats + 3) / 4 * 4;   // keep partials 16-byte aligned
  const size_t part_bytes =
      static_cast<size_t>(kStaticScratchFloats - stats_pad) * sizeof(float);
  const int rc = launch_stats<T>(x, scratch, sh, scratch + stats_pad, part_bytes, stream);
  if (rc != B200_OK) return rc;
  return launch_apply<T>(x, scratch, gamma, beta, y, affine_dt, sh, eps, false, false, stream);
}

}  // namespace
}  // namespace b200

extern "C" int b200_gn_fwd_static_scratch(const void* x, const void* gamma, const void* beta,
                                          void* y, int dtype, int affine_dtype, int64_t N,
                                          int64_t C, int64_t S, int64_t G, float eps,
                                          void* stream) {
  using namespace b200;
  if (!x || !y) return fail_arg("x/y is NULL");
  if (!dtype_ok(dtype) || ((gamma || beta) && !dtype_ok(affine_dtype)))
    return fail_arg("bad dtype");
  GnShape sh;
  int rc = check_shape(N, C, S, G, &sh);
  if (rc != B200_OK) return rc;
  // Scratch demand of the split path (scalar chunking is the larger case).
  const int64_t chunk = split_chunk(sh, 1);
  const int64_t chunks = (sh.M + chunk - 1) / chunk;
  const int64_t need = (sh.groups * 3 + 3) / 4 * 4 + sh.groups * chunks * 3;
  if (need > kStaticScratchFloats) {
    set_last_error("b200_gn_fwd_static_scratch: needs " + std::to_string(need) +
                   " scratch floats (N*G*(chunks+1)*3), the static array holds " +
                   std::to_string(kStaticScratchFloats));
    return B200_ERR_ARG;
  }
  cudaError_t err = cudaSuccess;
  float* scratch = static_scratch_address(&err);
  if (scratch == nullptr) return fail_cuda(err, "cudaGetSymbolAddress(g_gn_static_scratch)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_DTYPE_F32)
    return gn_static_typed<float>(x, gamma, beta, y, affine_dtype, sh, eps, scratch, s);
  if (dtype == B200_DTYPE_F16)
    return gn_static_typed<__half>(x, gamma, beta, y, affine_dtype, sh, eps, scratch, s);
  return gn_static_typed<__nv_bfloat16>(x, gamma, beta, y, affine_dtype, sh, eps, scratch, s);
}
