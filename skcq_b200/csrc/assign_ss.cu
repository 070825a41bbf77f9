// Nearest-centroid assignment, shared-memory-operand form (kernel 1 of
// skcq/codebook/kmeans.py:25-66, assign_cosine / assign_l2, for packed widths
// of three or more MMA k-steps; the tensor-memory-operand form in
// assign_tc.cu serves narrower ones).
//
// One persistent CTA per SM, warp-specialised:
//   warp 0      producer: 1-D bulk copies (TMA engine) of the point tile
//               (256 points, double buffered across work units) and a ring
//               of centroid tiles (128 centroids each, up to 16 deep);
//   warp 1      issues tcgen05.mma kind::tf32 (M=128, N=128, K=8, both
//               operands from shared memory) into one of two tensor-memory
//               accumulator sets (double buffered);
//   warps 2-17  epilogue: tcgen05.ld 64 columns of the fp32 scores of one
//               (row tile, lane quarter), release the accumulator, then keep
//               a running (best value, best group of 32 centroids) per point
//               with 3-input max; the distance matrix never leaves the SM.
// With four accumulator slots (two sets of two row tiles) the MMA thread
// never waits on the epilogue, which makes this form faster than the
// two-slot tensor-memory-operand form once each tile's MMA chain is long.
// Operands are split-tf32 (hi/lo) so A.B reproduces the fp32 dot product to
// ~2^-21 relative. The winning group is re-scored exactly by refine_kernel.
#include <algorithm>

#include "assign_ss.cuh"
#include "common.cuh"

namespace skcq {
namespace ss {


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
      if (row < nb && !failed && nbt > 0) p.group[(int64_t)b * p.n_pad + row] = -(bestg + 1);  // negative: not yet refined
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


template <int KSTEPS>
static cudaError_t launch(const TcParams& p, int grid, size_t smem, cudaStream_t s) {
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

}  // namespace ss

cudaError_t assign_ss_launch(const float* A, const float* B, int nblk, int n_pad, int k_pad, int kp,
                             const int32_t* n, const int32_t* k, const int32_t* active, int32_t* group, int* err,
                             int grid, cudaStream_t s) {
  using namespace ss;
  const size_t bar_bytes = (2 * TC_ABUF + 2 * TC_STAGES + 4) * sizeof(uint64_t) + 16 + 2 * TC_ROWS * 4;
  int stages = TC_STAGES;
  auto smem_for = [&](int st) {
    return (size_t)TC_ABUF * TC_ROWS * kp * 4 + (size_t)st * TC_BN * kp * 4 + bar_bytes;
  };
  while (stages > 2 && smem_for(stages) > 227 * 1024) --stages;
  size_t smem = smem_for(stages);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem < TC_MIN_SMEM) smem = TC_MIN_SMEM;
  TcParams p{A, B, nblk, n_pad, k_pad, kp, stages, n, k, active, group, err};
  switch (kp / 8) {
    case 1: return launch<1>(p, grid, smem, s);
    case 2: return launch<2>(p, grid, smem, s);
    case 3: return launch<3>(p, grid, smem, s);
    case 4: return launch<4>(p, grid, smem, s);
    case 5: return launch<5>(p, grid, smem, s);
    case 6: return launch<6>(p, grid, smem, s);
    case 7: return launch<7>(p, grid, smem, s);
    default: return launch<8>(p, grid, smem, s);
  }
}

}  // namespace skcq
