// Nearest-centroid assignment on the 5th-generation tensor cores
// (skcq/codebook/kmeans.py:25-66, assign_cosine / assign_l2).
//
// Kernel 1 -- one persistent CTA per SM, warp-specialised:
//   warp 0      producer: 1-D bulk copies (TMA engine) of the point tile
//               (256 points, double buffered across work units) and a ring
//               of centroid tiles (128 centroids each, up to 16 deep);
//   warp 1      issues tcgen05.mma kind::tf32 (M=128, N=128, K=8) into one of
//               two tensor-memory accumulator sets (double buffered);
//   warps 2-17  epilogue: tcgen05.ld 64 columns of the fp32 scores of one
//               (row tile, lane quarter), release the accumulator, then keep
//               a running (best value, best group of 32 centroids) per point
//               with 3-input max; the distance matrix never leaves the SM.
// Operands are split-tf32 (hi/lo) so A.B reproduces the fp32 dot product to
// ~2^-21 relative.
// Kernel 2 -- refine: one thread per point re-scores the 32 centroids of its
// winning group with the exact fp32 reference formula (first maximum wins),
// reading the problem's centroid table from shared-memory slices.
#include <algorithm>

#include "common.cuh"

namespace skcq {

constexpr int TC_BM = 128;                       // points per MMA (TMEM lanes)
constexpr int TC_RT = 2;                         // row tiles per work unit
constexpr int TC_ROWS = TC_BM * TC_RT;           // points per work unit
constexpr int TC_BN = 128;                       // centroids per tile
constexpr int TC_STAGES = 16;                    // max centroid tile ring depth (as many as shared memory holds)
constexpr int TC_ABUF = 2;                       // point tiles in flight (next unit loads during this one)
constexpr int TC_EPI_WARPS = 8 * TC_RT;          // one warp per (row tile, lane quarter, column half)
constexpr int TC_THREADS = (2 + TC_EPI_WARPS) * 32;
constexpr int TC_TMEM_COLS = 2 * TC_RT * TC_BN;  // 512: two accumulator sets
constexpr size_t TC_MIN_SMEM = 116 * 1024;       // keeps one CTA (and one TMEM owner) per SM
constexpr int TC_MAX_KSTEPS = 8;                 // kp <= 64: bs <= 20 (l2) / 21 (cosine)
constexpr int GROUP = 32;                        // centroids per re-scored group

static_assert(TC_ROWS == SKCQ_ROWS_PER_UNIT, "work unit size is part of the ABI");
static_assert(TC_BN == SKCQ_CENT_TILE, "centroid tile size is part of the ABI");

struct TcParams {
  const float* A;  // [nblk][n_pad/8][kp/4][8][4]
  const float* B;  // [nblk][k_pad/8][kp/4][8][4]
  int nblk, n_pad, k_pad, kp, stages;
  const int32_t* n;
  const int32_t* k;
  const int32_t* active;
  int32_t* group;  // out: winning 32-centroid group per point
  int* err;
};

struct TcSmem {
  float* a;
  float* b;
  uint64_t* a_full;
  uint64_t* a_empty;
  uint64_t* b_full;
  uint64_t* b_empty;
  uint64_t* acc_full;
  uint64_t* acc_empty;
  uint32_t* tmem_slot;
  uint32_t a_bytes, b_bytes;
};

__device__ __forceinline__ bool unit_live(const TcParams& p, int64_t u, int upb, int* b, int* r0) {
  *b = (int)(u / upb);
  *r0 = (int)(u % upb) * TC_ROWS;
  if (p.active && !p.active[*b]) return false;
  return *r0 < p.n[*b];
}

// Position in a ring of n barrier-guarded slots: slot index and the parity of
// the slot's current use. Advancing never divides (the issuing threads are
// single-thread critical paths).
struct Ring {
  uint32_t idx = 0, phase = 0;
  __device__ __forceinline__ void next(uint32_t n) {
    if (++idx == n) {
      idx = 0;
      phase ^= 1;
    }
  }
};

__device__ void tc_producer(const TcParams& p, const TcSmem& s) {
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  const uint32_t b_floats = (uint32_t)TC_BN * p.kp;
  Ring ar, br;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int nbt = ceil_div(p.k[b], TC_BN);
    if (!mbar_wait(s.a_empty + ar.idx, ar.phase ^ 1, p.err, 11)) return;
    mbar_arrive_expect_tx(s.a_full + ar.idx, s.a_bytes);
    bulk_g2s(s.a + ar.idx * (TC_ROWS * p.kp), p.A + ((int64_t)b * p.n_pad + r0) * p.kp, s.a_bytes,
             s.a_full + ar.idx);
    ar.next(TC_ABUF);
    const float* bsrc = p.B + (int64_t)b * p.k_pad * p.kp;
    for (int j = 0; j < nbt; ++j, bsrc += b_floats) {
      if (!mbar_wait(s.b_empty + br.idx, br.phase ^ 1, p.err, 12)) return;
      mbar_arrive_expect_tx(s.b_full + br.idx, s.b_bytes);
      bulk_g2s(s.b + br.idx * b_floats, bsrc, s.b_bytes, s.b_full + br.idx);
      br.next(p.stages);
    }
  }
}

template <int KSTEPS>
__device__ void tc_mma(const TcParams& p, const TcSmem& s, uint32_t tmem_base) {
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  constexpr uint32_t idesc = idesc_tf32(TC_BM, TC_BN);
  const uint32_t sbo = (uint32_t)p.kp * 32;  // bytes between 8-row core-matrix groups
  // Descriptors advance by (bytes >> 4) in their start-address field.
  const uint64_t a0 = smem_desc(smem_u32(s.a), 128, sbo);
  const uint64_t b0 = smem_desc(smem_u32(s.b), 128, sbo);
  const uint64_t a_rt = (uint64_t)(TC_BM * p.kp * 4) >> 4;
  const uint64_t a_buf = (uint64_t)s.a_bytes >> 4;
  const uint64_t b_st = (uint64_t)s.b_bytes >> 4;
  Ring ar, br, cr;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int nbt = ceil_div(p.k[b], TC_BN);
    if (!mbar_wait(s.a_full + ar.idx, ar.phase, p.err, 13)) return;
    tc_fence_after();
    const uint64_t a_unit = a0 + ar.idx * a_buf;
    uint64_t bd = b0 + br.idx * b_st;
    for (int j = 0; j < nbt; ++j) {
      if (!mbar_wait(s.b_full + br.idx, br.phase, p.err, 14)) return;
      if (!mbar_wait(s.acc_empty + cr.idx, cr.phase ^ 1, p.err, 15)) return;
      tc_fence_after();
      const uint32_t d0 = tmem_base + cr.idx * (TC_RT * TC_BN);
#pragma unroll
      for (int rt = 0; rt < TC_RT; ++rt) {
        const uint64_t ad = a_unit + rt * a_rt;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) mma_tf32(d0 + rt * TC_BN, ad + 16 * ks, bd + 16 * ks, idesc, ks > 0 ? 1u : 0u);
      }
      tc_commit(s.b_empty + br.idx);
      tc_commit(s.acc_full + cr.idx);
      cr.next(2);
      br.next(p.stages);
      bd = br.idx == 0 ? b0 : bd + b_st;
    }
    tc_commit(s.a_empty + ar.idx);
    ar.next(TC_ABUF);
  }
}

__device__ __forceinline__ float group_max32(const float (&v)[32]) {
  float m0 = max3f(v[0], v[1], v[2]);
  float m1 = max3f(v[3], v[4], v[5]);
  float m2 = max3f(v[6], v[7], v[8]);
  float m3 = max3f(v[9], v[10], v[11]);
  m0 = max3f(m0, v[12], v[13]);
  m1 = max3f(m1, v[14], v[15]);
  m2 = max3f(m2, v[16], v[17]);
  m3 = max3f(m3, v[18], v[19]);
  m0 = max3f(m0, v[20], v[21]);
  m1 = max3f(m1, v[22], v[23]);
  m2 = max3f(m2, v[24], v[25]);
  m3 = max3f(m3, v[26], v[27]);
  m0 = max3f(m0, v[28], v[29]);
  m1 = max3f(m1, v[30], v[31]);
  return max3f(max3f(m0, m1, m2), m3, m3);
}

// Epilogue warp e = warp - 2 owns TMEM lane quarter warp % 4 (hardware rule),
// row tile (e >> 2) & 1 and column half e >> 3 of every 128-column tile. The
// two halves of a row keep separate (best, group) pairs, merged through shared
// memory at the end of each work unit (larger value, then lower group, wins).
__device__ void tc_epilogue(const TcParams& p, const TcSmem& s, uint32_t tmem_base, int warp, int lane,
                            float* m_best, int* m_group) {
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  const int e = warp - 2;
  const int q = warp & 3;
  const int rt = (e >> 2) & 1;
  const int half = e >> 3;
  const int lrow = rt * TC_BM + q * 32 + lane;  // row within the unit
  const uint32_t lane_off = (uint32_t)(q * 32) << 16;
  Ring cr;
  // After a failed wait a warp stops touching tensor memory but keeps joining
  // the named barriers below, so its partner warps are never left waiting.
  bool failed = false;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int kb = p.k[b], nb = p.n[b];
    const int nbt = ceil_div(kb, TC_BN);
    float best = -INFINITY;
    int bestg = 0x7fffffff;
    for (int j = 0; j < nbt; ++j) {
      if (failed) continue;
      const uint32_t acc = cr.idx;
      const bool ok = mbar_wait(s.acc_full + acc, cr.phase, p.err, 16);
      cr.next(2);
      if (!__all_sync(0xffffffffu, ok)) {
        failed = true;
        continue;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_off + (acc * TC_RT + rt) * TC_BN + half * 64;
      float v0[32], v1[32];
      tmem_ld32(taddr + 0, v0);
      tmem_ld32(taddr + 32, v1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s.acc_empty + acc);  // one arrival per warp
      const int cbase = j * TC_BN + half * 64;
      if (cbase + 64 > kb) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (cbase + i >= kb) v0[i] = -INFINITY;
          if (cbase + 32 + i >= kb) v1[i] = -INFINITY;
        }
      }
      const int g0 = cbase / GROUP;
      float m;
      m = group_max32(v0);
      if (m > best) { best = m; bestg = g0; }
      m = group_max32(v1);
      if (m > best) { best = m; bestg = g0 + 1; }
    }
    // merge the two column halves of each row (epilogue warps only: named barrier 1)
    if (half == 1) {
      m_best[lrow] = best;
      m_group[lrow] = bestg;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(TC_EPI_WARPS * 32) : "memory");
    if (half == 0) {
      const float ob = m_best[lrow];
      const int og = m_group[lrow];
      if (ob > best || (ob == best && og < bestg)) {
        best = ob;
        bestg = og;
      }
      const int row = r0 + lrow;
      if (row < nb && !failed) p.group[(int64_t)b * p.n_pad + row] = -(bestg + 1);  // negative: not yet refined
    }
    asm volatile("bar.sync 1, %0;" ::"n"(TC_EPI_WARPS * 32) : "memory");
  }
}

template <int KSTEPS>
__global__ void __launch_bounds__(TC_THREADS, 1) assign_tc_kernel(TcParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  TcSmem s;
  s.a_bytes = (uint32_t)TC_ROWS * p.kp * 4;
  s.b_bytes = (uint32_t)TC_BN * p.kp * 4;
  s.a = reinterpret_cast<float*>(smem_raw);
  s.b = reinterpret_cast<float*>(smem_raw + (size_t)TC_ABUF * s.a_bytes);
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem_raw + (size_t)TC_ABUF * s.a_bytes + (size_t)p.stages * s.b_bytes);
  s.a_full = bars;
  s.a_empty = bars + TC_ABUF;
  s.b_full = bars + 2 * TC_ABUF;
  s.b_empty = s.b_full + TC_STAGES;
  s.acc_full = s.b_empty + TC_STAGES;
  s.acc_empty = s.acc_full + 2;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.acc_empty + 2);
  float* m_best = reinterpret_cast<float*>(s.tmem_slot + 4);  // [TC_ROWS] half-row merge
  int* m_group = reinterpret_cast<int*>(m_best + TC_ROWS);      // [TC_ROWS]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_ABUF; ++i) {
      mbar_init(s.a_full + i, 1);
      mbar_init(s.a_empty + i, 1);
    }
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(s.b_full + i, 1);
      mbar_init(s.b_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s.acc_full + i, 1);
      mbar_init(s.acc_empty + i, TC_EPI_WARPS);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(s.tmem_slot, TC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_slot;

  if (warp == 0) {
    if (lane == 0) tc_producer(p, s);
  } else if (warp == 1) {
    if (lane == 0) tc_mma<KSTEPS>(p, s, tmem_base);
  } else {
    tc_epilogue(p, s, tmem_base, warp, lane, m_best, m_group);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC_TMEM_COLS);
  }
}

// Exact re-score of the winning group. On entry labels[b][i] = -(g + 1) for
// the winning group g of 32 centroids; on exit labels[b][i] = the argmax over
// c in [32 g, 32 g + 32) of the exact fp32 reference score (first maximum
// wins). One CTA owns a range of points of one problem and walks the
// problem's centroid table in shared-memory slices (each group padded by one
// float so that threads of a warp working on different groups hit different
// banks); L2 traffic is one table read per CTA instead of 32 centroids per point.
constexpr int RF_THREADS = 512;
constexpr int RF_SMEM = 200 * 1024;

template <int BS>
__global__ void __launch_bounds__(RF_THREADS)
refine_kernel(int metric, const float* __restrict__ X, const float* __restrict__ C,
              const float* __restrict__ cnorm, int n_pad, int k_pad, int bs_rt, int groups_per_slice,
              int chunk_rows, const int32_t* __restrict__ n, const int32_t* __restrict__ kvec,
              const int32_t* __restrict__ active, int32_t* __restrict__ labels) {
  extern __shared__ float tab[];
  const int bs = BS > 0 ? BS : bs_rt;
  constexpr int XN = BS > 0 ? BS : 64;
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b], kb = kvec[b];
  const int r0 = blockIdx.x * chunk_rows;
  if (r0 >= nb) return;
  const int r1 = min(nb, r0 + chunk_rows);
  const int gstride = GROUP * bs + 1;
  float* cn = tab + (size_t)groups_per_slice * gstride;
  const int n_groups = ceil_div(kb, GROUP);
  const float* Cb = C + (int64_t)b * k_pad * bs;
  const float* Nb = cnorm + (int64_t)b * k_pad;
  int32_t* Lb = labels + (int64_t)b * n_pad;
  const float* Xb = X + (int64_t)b * n_pad * bs;
  for (int g0 = 0; g0 < n_groups; g0 += groups_per_slice) {
    const int g1 = min(n_groups, g0 + groups_per_slice);
    __syncthreads();
    const int words = (g1 - g0) * GROUP * bs;
    for (int t = threadIdx.x; t < words; t += RF_THREADS) {
      const int gl = t / (GROUP * bs), rem = t - gl * GROUP * bs;
      const int c = (g0 + gl) * GROUP + rem / bs;
      tab[gl * gstride + rem] = c < kb ? Cb[(int64_t)g0 * GROUP * bs + t] : 0.f;
    }
    for (int t = threadIdx.x; t < (g1 - g0) * GROUP; t += RF_THREADS) {
      const int c = g0 * GROUP + t;
      cn[t] = c < kb ? Nb[c] : 0.f;
    }
    __syncthreads();
    for (int i = r0 + threadIdx.x; i < r1; i += RF_THREADS) {
      const int v = Lb[i];
      if (v >= 0) continue;
      const int g = -v - 1;
      if (g < g0 || g >= g1) continue;
      float x[XN];
      const float* xr = Xb + (int64_t)i * bs;
#pragma unroll
      for (int j = 0; j < XN; ++j)
        if (BS > 0 || j < bs) x[j] = xr[j];
      const float* T = tab + (g - g0) * gstride;
      const float* TN = cn + (g - g0) * GROUP;
      const int cnt = min(GROUP, kb - g * GROUP);
      float sbest = -INFINITY;
      int ibest = 0;
      for (int ii = 0; ii < cnt; ++ii) {
        const float* cc = T + ii * bs;
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < XN; ++j)
          if (BS > 0 || j < bs) dot = __fmaf_rn(x[j], cc[j], dot);
        const float sc = metric == SKCQ_METRIC_COSINE ? dot : -__fadd_rn(__fmul_rn(dot, -2.0f), TN[ii]);
        if (sc > sbest) {
          sbest = sc;
          ibest = ii;
        }
      }
      Lb[i] = g * GROUP + ibest;
    }
  }
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

template <int KSTEPS>
static cudaError_t launch_tc(const TcParams& p, int grid, size_t smem, cudaStream_t s) {
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e =
        cudaFuncSetAttribute(assign_tc_kernel<KSTEPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  assign_tc_kernel<KSTEPS><<<grid, TC_THREADS, smem, s>>>(p);
  return cudaGetLastError();
}

template <int BS>
static cudaError_t launch_refine(int metric, const float* X, const float* C, const float* cnorm, int nblk, int n_pad,
                                 int k_pad, int bs, const int32_t* n, const int32_t* k, const int32_t* active,
                                 int32_t* labels, cudaStream_t s) {
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(refine_kernel<BS>, cudaFuncAttributeMaxDynamicSharedMemorySize, RF_SMEM);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  const size_t group_bytes = (size_t)(GROUP * bs + 1 + GROUP) * sizeof(float);
  const int n_groups = k_pad / GROUP;
  int gps = (int)std::min<size_t>(RF_SMEM / group_bytes, (size_t)n_groups);
  if (gps < 1) gps = 1;
  const size_t smem = (size_t)gps * group_bytes;
  // enough CTAs for two waves, each owning >= 4096 points so the table load amortises
  const int64_t target = (int64_t)num_sms() * 2;
  int64_t chunks = (target + nblk - 1) / nblk;
  int64_t chunk_rows = (n_pad + chunks - 1) / chunks;
  if (chunk_rows < 4096) chunk_rows = std::min<int64_t>(4096, n_pad);
  chunks = (n_pad + chunk_rows - 1) / chunk_rows;
  dim3 grid((unsigned)chunks, (unsigned)nblk);
  refine_kernel<BS><<<grid, RF_THREADS, smem, s>>>(metric, X, C, cnorm, n_pad, k_pad, bs, gps, (int)chunk_rows, n, k,
                                                   active, labels);
  return cudaGetLastError();
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_assign(int metric, const float* A, const float* B, const float* X, const float* C,
                           const float* cnorm, int nblk, int n_pad, int k_pad, int bs, const int32_t* n,
                           const int32_t* k, const int32_t* active, int32_t* labels, void* stream) {
  SKCQ_REQUIRE(A && B && X && C && cnorm && n && k && labels, SKCQ_ERR_INVALID, "assign: null pointer");
  SKCQ_REQUIRE(metric == SKCQ_METRIC_COSINE || metric == SKCQ_METRIC_L2, SKCQ_ERR_INVALID, "assign: bad metric");
  SKCQ_REQUIRE(bs > 0 && bs <= 64, SKCQ_ERR_INVALID, "assign: block size %d outside [1, 64]", bs);
  SKCQ_REQUIRE(n_pad > 0 && n_pad % TC_ROWS == 0, SKCQ_ERR_INVALID, "assign: n_pad %d not a multiple of %d", n_pad,
               TC_ROWS);
  SKCQ_REQUIRE(k_pad > 0 && k_pad % TC_BN == 0, SKCQ_ERR_INVALID, "assign: k_pad %d not a multiple of %d", k_pad,
               TC_BN);
  SKCQ_REQUIRE((((uintptr_t)A | (uintptr_t)B) & 15) == 0, SKCQ_ERR_INVALID, "assign: operands not 16-byte aligned");
  const int kp = skcq_packed_width(metric, bs);
  SKCQ_REQUIRE(kp / 8 <= TC_MAX_KSTEPS, SKCQ_ERR_INVALID,
               "assign: block size %d too wide for the tensor-core path (use skcq_assign_exact)", bs);
  const size_t bar_bytes = (2 * TC_ABUF + 2 * TC_STAGES + 4) * sizeof(uint64_t) + 16 + 2 * TC_ROWS * 4;
  int stages = TC_STAGES;
  auto smem_for = [&](int st) {
    return (size_t)TC_ABUF * TC_ROWS * kp * 4 + (size_t)st * TC_BN * kp * 4 + bar_bytes;
  };
  while (stages > 2 && smem_for(stages) > 227 * 1024) --stages;
  size_t smem = smem_for(stages);
  SKCQ_REQUIRE(smem <= 227 * 1024, SKCQ_ERR_INVALID, "assign: block size %d needs too much shared memory", bs);
  if (smem < TC_MIN_SMEM) smem = TC_MIN_SMEM;
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "assign: no device error word");
  TcParams p{A, B, nblk, n_pad, k_pad, kp, stages, n, k, active, labels, err};
  const int64_t n_units = (int64_t)nblk * (n_pad / TC_ROWS);
  const int grid = (int)(n_units < num_sms() ? n_units : num_sms());
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  switch (kp / 8) {
    case 1: e = launch_tc<1>(p, grid, smem, s); break;
    case 2: e = launch_tc<2>(p, grid, smem, s); break;
    case 3: e = launch_tc<3>(p, grid, smem, s); break;
    case 4: e = launch_tc<4>(p, grid, smem, s); break;
    case 5: e = launch_tc<5>(p, grid, smem, s); break;
    case 6: e = launch_tc<6>(p, grid, smem, s); break;
    case 7: e = launch_tc<7>(p, grid, smem, s); break;
    default: e = launch_tc<8>(p, grid, smem, s); break;
  }
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "assign: %s", cudaGetErrorString(e));
  SKCQ_REQUIRE(nblk <= 65535, SKCQ_ERR_INVALID, "assign: %d problems exceed 65535", nblk);
  switch (bs) {
    case 4: e = launch_refine<4>(metric, X, C, cnorm, nblk, n_pad, k_pad, bs, n, k, active, labels, s); break;
    case 6: e = launch_refine<6>(metric, X, C, cnorm, nblk, n_pad, k_pad, bs, n, k, active, labels, s); break;
    case 8: e = launch_refine<8>(metric, X, C, cnorm, nblk, n_pad, k_pad, bs, n, k, active, labels, s); break;
    case 12: e = launch_refine<12>(metric, X, C, cnorm, nblk, n_pad, k_pad, bs, n, k, active, labels, s); break;
    case 16: e = launch_refine<16>(metric, X, C, cnorm, nblk, n_pad, k_pad, bs, n, k, active, labels, s); break;
    default: e = launch_refine<0>(metric, X, C, cnorm, nblk, n_pad, k_pad, bs, n, k, active, labels, s); break;
  }
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "assign (refine): %s", cudaGetErrorString(e));
  return SKCQ_OK;
}
