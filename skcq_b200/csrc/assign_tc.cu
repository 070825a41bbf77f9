// Nearest-centroid assignment on the 5th-generation tensor cores
// (skcq/codebook/kmeans.py:25-66, assign_cosine / assign_l2).
//
// One persistent CTA per SM, warp-specialised:
//   warp 0      producer: 1-D bulk copies (TMA engine) of the point tile
//               (256 points, resident for the whole centroid sweep) and a
//               4-stage ring of centroid tiles (128 centroids each);
//   warp 1      issues tcgen05.mma kind::tf32 (M=128, N=128, K=8) into one of
//               two tensor-memory accumulator sets (double buffered);
//   warps 2-9   epilogue: tcgen05.ld the 128x128 fp32 scores of one row tile
//               and lane quarter, release the accumulator, then keep a
//               running (best value, best group of 32 centroids) per point
//               with 3-input max; the distance matrix never leaves the SM.
// Operands are split-tf32 (hi/lo) so A.B reproduces the fp32 dot product to
// ~2^-21 relative; the winning 32-centroid group is re-scored with the exact
// fp32 reference formula, which also resolves ties to the first index.
#include "common.cuh"

namespace skcq {

constexpr int TC_BM = 128;                       // points per MMA (TMEM lanes)
constexpr int TC_RT = 2;                         // row tiles per work unit
constexpr int TC_ROWS = TC_BM * TC_RT;           // points per work unit
constexpr int TC_BN = 128;                       // centroids per tile
constexpr int TC_STAGES = 4;                     // centroid tile ring depth
constexpr int TC_EPI_WARPS = 4 * TC_RT;          // one warp per (row tile, lane quarter)
constexpr int TC_THREADS = (2 + TC_EPI_WARPS) * 32;
constexpr int TC_TMEM_COLS = 2 * TC_RT * TC_BN;  // 512: two accumulator sets
constexpr size_t TC_MIN_SMEM = 116 * 1024;       // keeps one CTA (and one TMEM owner) per SM

static_assert(TC_ROWS == SKCQ_ROWS_PER_UNIT, "work unit size is part of the ABI");
static_assert(TC_BN == SKCQ_CENT_TILE, "centroid tile size is part of the ABI");

struct TcParams {
  int metric;
  const float* A;  // [nblk][n_pad/8][kp/4][8][4]
  const float* B;  // [nblk][k_pad/8][kp/4][8][4]
  const float* X;  // [nblk][n_pad][bs]
  const float* C;  // [nblk][k_pad][bs]
  const float* cnorm;
  int nblk, n_pad, k_pad, bs, kp;
  const int32_t* n;
  const int32_t* k;
  const int32_t* active;
  int32_t* labels;
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

__device__ void tc_producer(const TcParams& p, const TcSmem& s) {
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  uint32_t a_use = 0, b_cnt = 0;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int nbt = ceil_div(p.k[b], TC_BN);
    if (!mbar_wait(s.a_empty, (a_use & 1) ^ 1, p.err, 11)) return;
    mbar_arrive_expect_tx(s.a_full, s.a_bytes);
    bulk_g2s(s.a, p.A + ((int64_t)b * p.n_pad + r0) * p.kp, s.a_bytes, s.a_full);
    ++a_use;
    for (int j = 0; j < nbt; ++j, ++b_cnt) {
      const uint32_t st = b_cnt % TC_STAGES, use = b_cnt / TC_STAGES;
      if (!mbar_wait(s.b_empty + st, (use & 1) ^ 1, p.err, 12)) return;
      mbar_arrive_expect_tx(s.b_full + st, s.b_bytes);
      bulk_g2s(s.b + (size_t)st * TC_BN * p.kp, p.B + ((int64_t)b * p.k_pad + (int64_t)j * TC_BN) * p.kp, s.b_bytes,
               s.b_full + st);
    }
  }
}

__device__ void tc_mma(const TcParams& p, const TcSmem& s, uint32_t tmem_base) {
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  const uint32_t idesc = idesc_tf32(TC_BM, TC_BN);
  const uint32_t sbo = (uint32_t)p.kp * 32;  // bytes between 8-row core-matrix groups
  const int ksteps = p.kp / 8;
  const uint32_t a_base = smem_u32(s.a), b_base = smem_u32(s.b);
  uint32_t a_use = 0, b_cnt = 0, t_cnt = 0;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int nbt = ceil_div(p.k[b], TC_BN);
    if (!mbar_wait(s.a_full, a_use & 1, p.err, 13)) return;
    tc_fence_after();
    ++a_use;
    for (int j = 0; j < nbt; ++j, ++b_cnt, ++t_cnt) {
      const uint32_t st = b_cnt % TC_STAGES, use = b_cnt / TC_STAGES;
      const uint32_t acc = t_cnt & 1, ause = t_cnt >> 1;
      if (!mbar_wait(s.b_full + st, use & 1, p.err, 14)) return;
      if (!mbar_wait(s.acc_empty + acc, (ause & 1) ^ 1, p.err, 15)) return;
      tc_fence_after();
      const uint32_t b_tile = b_base + st * s.b_bytes;
#pragma unroll
      for (int rt = 0; rt < TC_RT; ++rt) {
        const uint32_t d = tmem_base + (acc * TC_RT + rt) * TC_BN;
        const uint32_t a_tile = a_base + rt * (TC_BM * p.kp * 4);
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint64_t ad = smem_desc(a_tile + ks * 256, 128, sbo);
          const uint64_t bd = smem_desc(b_tile + ks * 256, 128, sbo);
          mma_tf32(d, ad, bd, idesc, ks > 0 ? 1u : 0u);
        }
      }
      tc_commit(s.b_empty + st);
      tc_commit(s.acc_full + acc);
    }
    tc_commit(s.a_empty);
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

__device__ void tc_epilogue(const TcParams& p, const TcSmem& s, uint32_t tmem_base, int warp, int lane) {
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  const int q = warp & 3;             // tensor-memory lane quarter this warp may access
  const int rt = (warp - 2) >> 2;     // row tile handled by this warp
  const uint32_t lane_off = (uint32_t)(q * 32) << 16;
  uint32_t t_cnt = 0;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int kb = p.k[b], nb = p.n[b];
    const int nbt = ceil_div(kb, TC_BN);
    float best = -INFINITY;
    int bestg = 0;
    for (int j = 0; j < nbt; ++j, ++t_cnt) {
      const uint32_t acc = t_cnt & 1, ause = t_cnt >> 1;
      bool ok = mbar_wait(s.acc_full + acc, ause & 1, p.err, 16);
      if (!__all_sync(0xffffffffu, ok)) return;
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_off + (acc * TC_RT + rt) * TC_BN;
      float v0[32], v1[32], v2[32], v3[32];
      tmem_ld32(taddr + 0, v0);
      tmem_ld32(taddr + 32, v1);
      tmem_ld32(taddr + 64, v2);
      tmem_ld32(taddr + 96, v3);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s.acc_empty + acc);
      const int cbase = j * TC_BN;
      if (cbase + TC_BN > kb) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (cbase + i >= kb) v0[i] = -INFINITY;
          if (cbase + 32 + i >= kb) v1[i] = -INFINITY;
          if (cbase + 64 + i >= kb) v2[i] = -INFINITY;
          if (cbase + 96 + i >= kb) v3[i] = -INFINITY;
        }
      }
      const int g0 = cbase >> 5;
      float m;
      m = group_max32(v0);
      if (m > best) { best = m; bestg = g0; }
      m = group_max32(v1);
      if (m > best) { best = m; bestg = g0 + 1; }
      m = group_max32(v2);
      if (m > best) { best = m; bestg = g0 + 2; }
      m = group_max32(v3);
      if (m > best) { best = m; bestg = g0 + 3; }
    }
    // Exact fp32 re-score of the winning group (first maximum wins).
    const int row = r0 + rt * TC_BM + q * 32 + lane;
    if (row < nb) {
      float x[64];
      const float* xr = p.X + ((int64_t)b * p.n_pad + row) * p.bs;
      for (int jj = 0; jj < p.bs; ++jj) x[jj] = xr[jj];
      const int c0 = bestg * 32;
      const int c1 = min(c0 + 32, kb);
      const float* Cb = p.C + (int64_t)b * p.k_pad * p.bs;
      const float* nb_ = p.cnorm + (int64_t)b * p.k_pad;
      float sbest = -INFINITY;
      int cbest = c0;
      for (int c = c0; c < c1; ++c) {
        const float sc = exact_score(p.metric, x, Cb + (int64_t)c * p.bs, nb_[c], p.bs);
        if (sc > sbest) {
          sbest = sc;
          cbest = c;
        }
      }
      p.labels[(int64_t)b * p.n_pad + row] = cbest;
    }
  }
}

__global__ void __launch_bounds__(TC_THREADS, 1) assign_tc_kernel(TcParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  TcSmem s;
  s.a_bytes = (uint32_t)TC_ROWS * p.kp * 4;
  s.b_bytes = (uint32_t)TC_BN * p.kp * 4;
  s.a = reinterpret_cast<float*>(smem_raw);
  s.b = reinterpret_cast<float*>(smem_raw + s.a_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + s.a_bytes + (size_t)TC_STAGES * s.b_bytes);
  s.a_full = bars;
  s.a_empty = bars + 1;
  s.b_full = bars + 2;
  s.b_empty = bars + 2 + TC_STAGES;
  s.acc_full = bars + 2 + 2 * TC_STAGES;
  s.acc_empty = s.acc_full + 2;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(s.a_full, 1);
    mbar_init(s.a_empty, 1);
    for (int i = 0; i < TC_STAGES; ++i) {
      mbar_init(s.b_full + i, 1);
      mbar_init(s.b_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s.acc_full + i, 1);
      mbar_init(s.acc_empty + i, TC_EPI_WARPS * 32);
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
    if (lane == 0) tc_mma(p, s, tmem_base);
  } else {
    tc_epilogue(p, s, tmem_base, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC_TMEM_COLS);
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
  size_t smem = (size_t)TC_ROWS * kp * 4 + (size_t)TC_STAGES * TC_BN * kp * 4 + 16 * sizeof(uint64_t);
  SKCQ_REQUIRE(smem <= 227 * 1024, SKCQ_ERR_INVALID, "assign: block size %d needs too much shared memory", bs);
  if (smem < TC_MIN_SMEM) smem = TC_MIN_SMEM;
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "assign: no device error word");
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(assign_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "assign: %s", cudaGetErrorString(e));
    configured_dev = dev;
  }
  TcParams p{metric, A, B, X, C, cnorm, nblk, n_pad, k_pad, bs, kp, n, k, active, labels, err};
  const int64_t n_units = (int64_t)nblk * (n_pad / TC_ROWS);
  const int grid = (int)(n_units < num_sms() ? n_units : num_sms());
  assign_tc_kernel<<<grid, TC_THREADS, smem, (cudaStream_t)stream>>>(p);
  return check_launch("assign");
}
