// Nearest-centroid assignment on the 5th-generation tensor cores
// (skcq/codebook/kmeans.py:25-66, assign_cosine / assign_l2).
//
// Kernel 1 -- one persistent CTA per SM, warp-specialised:
//   warp 0      producer: 1-D bulk copies (TMA engine) of the work unit's
//               256 points and a ring of centroid tiles;
//   warps 1, 2  issue the tensor-core work, one thread per row tile: at the
//               start of each unit tcgen05.cp moves the thread's 128-point row
//               tile from shared into tensor memory, then for every centroid
//               tile one chain of tcgen05.mma kind::tf32 (M=128, N, K=8, A
//               from tensor memory, B from shared memory) into the next of
//               three accumulator slots (items alternate between the two
//               threads: (tile 0, row tile 0), (tile 0, row tile 1), ...);
//   warps 3..   epilogue, one set of warps per row tile: a warp owns a TMEM
//               lane quarter and a pair of 32-centroid groups of every tile
//               of its row tile. For every item it tcgen05.lds its 64 scores
//               per point, releases the slot at once and folds the groups
//               into a running (best value, best group) per point with
//               3-input max; the distance matrix never leaves the SM.
// What bounds this kernel is issue and hand-off latency, not the tensor
// pipe. Measured on B200: a tcgen05.mma issue stalls its thread ~64 clocks,
// a tcgen05.commit ~90 and an mbarrier try_wait ~130, so one thread needs
// ~350 clocks per item while a 128 x 128 item at two k-steps is 128 clocks
// of tensor work. Two issuing threads halve that; every slot is released
// after one tcgen05.ld round per epilogue warp (no ALU work in between); and
// three slots of N = 128 keep the tensor core busy while the epilogue drains
// the others.
// Operands are split-tf32 (hi/lo) so A.B reproduces the fp32 dot product to
// ~2^-21 relative.
// Kernel 2 -- refine: one warp per point re-scores the 32 centroids of its
// winning group, one centroid per lane, with the exact fp32 reference formula
// (first maximum wins), reading the problem's centroid table from transposed
// shared-memory slices.
#include <algorithm>

#include "common.cuh"

namespace skcq {

constexpr int TC_BM = 128;                // points per MMA (TMEM lanes)
constexpr int TC_RT = 2;                  // row tiles per work unit
constexpr int TC_ROWS = TC_BM * TC_RT;    // points per work unit
constexpr int TC_STAGES = 16;             // max centroid tile ring depth (as many as shared memory holds)
constexpr int TC_SLOTS = 3;               // accumulators in flight
constexpr int TC_TMEM_COLS = 512;
constexpr size_t TC_MIN_SMEM = 116 * 1024;  // keeps one CTA (and one TMEM owner) per SM
constexpr int TC_MAX_KSTEPS = 8;          // kp <= 64: bs <= 20 (l2) / 21 (cosine)
constexpr int GROUP = 32;                 // centroids per re-scored group

static_assert(TC_ROWS == SKCQ_ROWS_PER_UNIT, "work unit size is part of the ABI");

// Shapes of the kernel for KSTEPS k-steps (kp = 8 KSTEPS): N centroids per
// tile, the accumulator slots at tensor-memory columns [0, SLOTS N) and the
// unit's two A tiles at [SLOTS N, SLOTS N + 2 kp).
template <int KSTEPS>
struct TcShape {
  static constexpr int KP = KSTEPS * 8;
  static constexpr int N = 128;
  static constexpr int NG = N / GROUP;             // groups per tile
  static constexpr int GPW = 2;                    // groups one epilogue warp loads per item
  static constexpr int WPQ = NG / GPW;             // warps per lane quarter per row tile
  static constexpr int EPI_PER_RT = 4 * WPQ;       // epilogue warps of one row tile
  static constexpr int EPI_WARPS = TC_RT * EPI_PER_RT;
  static constexpr int EPI_WARP0 = 1 + TC_RT;       // producer, one MMA warp per row tile, epilogue
  static constexpr int THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
  static constexpr int A_COL = TC_SLOTS * N;
  static_assert(A_COL + TC_RT * KP <= TC_TMEM_COLS, "slots and A tiles must fit tensor memory");
  static_assert(N % GROUP == 0 && N % 16 == 0 && N <= 256, "MMA N");
  static_assert(NG % GPW == 0, "whole group pairs");
};

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
  uint64_t* a_tmem_free;  // [TC_RT] the row tile's MMAs of the previous unit done: its A columns reusable
  uint64_t* b_full;
  uint64_t* b_empty;
  // [TC_SLOTS][2]: use u of slot s signals on barrier (s, u & 1). Consecutive
  // uses of a slot belong to alternating row tiles (three slots, two row
  // tiles), so each barrier object has one signalling and one waiting party
  // and sees its phases strictly in order; with one barrier per slot a party
  // running ahead could meet a barrier two phases behind and pass its parity
  // test early.
  uint64_t* acc_full;
  uint64_t* acc_empty;
  uint32_t* tmem_slot;
  float* m_best;        // [TC_RT][NG][TC_BM] per-warp candidates, merged per unit
  int* m_group;
  uint32_t a_bytes, b_stage_bytes;
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

// D(tmem) = A(tmem) * B(smem desc), kind::tf32, fp32 accumulate; the
// accumulate flag is a constant of the instruction (first k-step overwrites).
__device__ __forceinline__ void mma_tf32_ts_first(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
  asm volatile("tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, 0;" ::"r"(d_tmem), "r"(a_tmem),
               "l"(b_desc), "r"(idesc)
               : "memory");
}
__device__ __forceinline__ void mma_tf32_ts_acc(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
  asm volatile("tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, 1;" ::"r"(d_tmem), "r"(a_tmem),
               "l"(b_desc), "r"(idesc)
               : "memory");
}

// 128 rows x 256 bits (eight fp32 columns) of a no-swizzle K-major shared
// image into tensor memory, row i to lane i. Ordered before later
// tcgen05.mma issued by the same thread.
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t s_desc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(s_desc) : "memory");
}

template <int KSTEPS>
__device__ void tc_producer(const TcParams& p, const TcSmem& s) {
  constexpr int N = TcShape<KSTEPS>::N;
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  const int64_t tile_floats = (int64_t)N * p.kp;
  Ring ar, br;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int nbt = ceil_div(p.k[b], N);
    if (!mbar_wait(s.a_empty, ar.phase ^ 1, p.err, 11)) return;
    mbar_arrive_expect_tx(s.a_full, s.a_bytes);
    bulk_g2s(s.a, p.A + ((int64_t)b * p.n_pad + r0) * p.kp, s.a_bytes, s.a_full);
    ar.next(1);
    const float* bsrc = p.B + (int64_t)b * p.k_pad * p.kp;
    for (int j = 0; j < nbt; ++j, bsrc += tile_floats) {
      // the last tile may run past k_pad (a multiple of 128): copy only the
      // rows that exist; the epilogue masks every column >= k
      const int rows = min(N, p.k_pad - j * N);
      const uint32_t bytes = (uint32_t)rows * p.kp * 4;
      if (!mbar_wait(s.b_empty + br.idx, br.phase ^ 1, p.err, 12)) return;
      mbar_arrive_expect_tx(s.b_full + br.idx, bytes);
      bulk_g2s(s.b + (size_t)br.idx * tile_floats, bsrc, bytes, s.b_full + br.idx);
      br.next(p.stages);
    }
  }
}

// Issues row tile rt's items. Item t = 2 * (tiles issued so far by this
// CTA) + rt goes to accumulator slot t % 3, on that slot's (t / 3)-th use;
// the epilogue consumes items in t order.
template <int KSTEPS>
__device__ void tc_mma(const TcParams& p, const TcSmem& s, uint32_t tmem_base, int rt) {
  using S = TcShape<KSTEPS>;
  constexpr int N = S::N;
  constexpr int KP = S::KP;
  constexpr uint32_t idesc = idesc_tf32(TC_BM, N);
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  const uint32_t sbo = (uint32_t)KP * 32;  // bytes between 8-row core-matrix groups
  // Descriptors advance by (bytes >> 4) in their start-address field.
  const uint64_t a0 = smem_desc(smem_u32(s.a), 128, sbo) + (((uint64_t)(TC_BM * KP * 4) >> 4) * rt);
  const uint64_t b0 = smem_desc(smem_u32(s.b), 128, sbo);
  const uint64_t b_st = (uint64_t)s.b_stage_bytes >> 4;
  const uint32_t a_tm = tmem_base + S::A_COL + rt * KP;
  Ring ar, br;
  uint32_t item = (uint32_t)rt;
  uint32_t a_free_phase = 0;
  bool first = true;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int nbt = ceil_div(p.k[b], N);
    if (!mbar_wait(s.a_full, ar.phase, p.err, 13)) return;
    if (!first) {
      // this row tile's MMAs of the previous unit read the A columns until they complete
      if (!mbar_wait(s.a_tmem_free + rt, a_free_phase, p.err, 17)) return;
      a_free_phase ^= 1;
    }
    first = false;
    tc_fence_after();
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) tmem_cp_128x256b(a_tm + ks * 8, a0 + 16 * ks);
    tc_commit(s.a_empty);  // one of the two arrivals that free the shared copy
    for (int i = 0; i < nbt; ++i, item += TC_RT) {
      if (!mbar_wait(s.b_full + br.idx, br.phase, p.err, 14)) return;
      const uint32_t slot = item % TC_SLOTS;
      const uint32_t use = item / TC_SLOTS;
      if (use > 0) {
        // the slot's previous use (the other row tile's item) has been read
        const uint32_t prev = use - 1;
        if (!mbar_wait(s.acc_empty + 2 * slot + (prev & 1), (prev >> 1) & 1, p.err, 15)) return;
      }
      tc_fence_after();
      const uint64_t bd = b0 + br.idx * b_st;
      const uint32_t d = tmem_base + slot * N;
      mma_tf32_ts_first(d, a_tm, bd, idesc);
#pragma unroll
      for (int ks = 1; ks < KSTEPS; ++ks) mma_tf32_ts_acc(d, a_tm + ks * 8, bd + 16 * ks, idesc);
      tc_commit(s.acc_full + 2 * slot + (use & 1));
      tc_commit(s.b_empty + br.idx);  // one of the two arrivals that free the stage
      br.next(p.stages);
    }
    tc_commit(s.a_tmem_free + rt);
    ar.next(1);
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

// Mask the columns of one 32-centroid group at or past the problem's k.
__device__ __forceinline__ void mask_group(float (&v)[32], int cbase, int kb) {
  if (cbase + GROUP > kb) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (cbase + i >= kb) v[i] = -INFINITY;
  }
}

// Epilogue warps 3.. form one set per row tile; warp e = warp - 3 serves row
// tile rt = e / EPI_PER_RT, TMEM lane quarter warp % 4 (hardware rule) and
// the group pair h = (e / 4) % WPQ of every tile, i.e. the items
// t = 2 j + rt of tiles j, which arrive in accumulator slot t % 3. For each
// it loads both groups' scores, waits for the loads, releases the slot (one
// arrival per warp) and only then reduces, so a slot is held for one
// tensor-memory load round; the two row tiles' sets work on alternate items,
// one loading while the other reduces. Each thread keeps a running (best,
// group) per point; tiles arrive in index order, so a strictly larger
// maximum is needed to move to a later group. At the end of a work unit the
// WPQ candidates of each row are merged through shared memory (larger value,
// then lower group, wins).
template <int KSTEPS>
__device__ void tc_epilogue(const TcParams& p, const TcSmem& s, uint32_t tmem_base, int warp, int lane) {
  using S = TcShape<KSTEPS>;
  constexpr int N = S::N;
  constexpr int NG = S::NG;
  constexpr int GPW = S::GPW;
  constexpr int WPQ = S::WPQ;
  const int upb = p.n_pad / TC_ROWS;
  const int64_t n_units = (int64_t)p.nblk * upb;
  const int e = warp - S::EPI_WARP0;
  const int rt = e / S::EPI_PER_RT;
  const int q = warp & 3;
  const int h = (e >> 2) % WPQ;
  const int qrow = q * 32 + lane;  // row within the row tile
  const uint32_t tq = tmem_base + ((uint32_t)(q * 32) << 16) + h * GPW * GROUP;
  uint32_t item = (uint32_t)rt;
  // After a failed wait a warp stops touching tensor memory but keeps joining
  // the named barriers below, so its partner warps are never left waiting.
  bool failed = false;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    int b, r0;
    if (!unit_live(p, u, upb, &b, &r0)) continue;
    const int kb = p.k[b], nb = p.n[b];
    const int nbt = ceil_div(kb, N);
    float best = -INFINITY;
    int bestg = 0x7fffffff;
    for (int j = 0; j < nbt; ++j, item += TC_RT) {
      if (failed) continue;
      const uint32_t slot = item % TC_SLOTS;
      const uint32_t use = item / TC_SLOTS;
      const uint32_t bar = 2 * slot + (use & 1);
      const bool ok = mbar_wait(s.acc_full + bar, (use >> 1) & 1, p.err, 16);
      if (!__all_sync(0xffffffffu, ok)) {
        failed = true;
        continue;
      }
      tc_fence_after();
      float v0[32], v1[32];
      tmem_ld32(tq + slot * N, v0);
      tmem_ld32(tq + slot * N + GROUP, v1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s.acc_empty + bar);  // one arrival per warp
      const int gg = j * NG + h * GPW;  // global index of the first group
      if ((j + 1) * N > kb) {  // only the problem's last tile has columns past k
        mask_group(v0, gg * GROUP, kb);
        mask_group(v1, (gg + 1) * GROUP, kb);
      }
      // one compare per group pair; the pair's winner (lower group on a tie,
      // NaN never wins) only when the running best moves, as two sequential
      // strictly-greater updates would choose
      const float m0 = group_max32(v0), m1 = group_max32(v1);
      const float m = fmaxf(m0, m1);
      if (m > best) {
        best = m;
        bestg = m0 >= m1 ? gg : gg + 1;
      }
    }
    // merge the WPQ candidates of each row (epilogue warps only: named barrier 1)
    s.m_best[(rt * WPQ + h) * TC_BM + qrow] = best;
    s.m_group[(rt * WPQ + h) * TC_BM + qrow] = bestg;
    asm volatile("bar.sync 1, %0;" ::"n"(S::EPI_WARPS * 32) : "memory");
    if (h == 0) {
      float bv = best;
      int bg = bestg;
#pragma unroll
      for (int o = 1; o < WPQ; ++o) {
        const float ov = s.m_best[(rt * WPQ + o) * TC_BM + qrow];
        const int og = s.m_group[(rt * WPQ + o) * TC_BM + qrow];
        if (ov > bv || (ov == bv && og < bg)) {
          bv = ov;
          bg = og;
        }
      }
      if (bg == 0x7fffffff) bg = 0;  // no finite score in any group (all masked or NaN)
      const int row = r0 + rt * TC_BM + qrow;
      if (row < nb && !failed && nbt > 0) p.group[(int64_t)b * p.n_pad + row] = -(bg + 1);  // negative: not yet refined
    }
    asm volatile("bar.sync 1, %0;" ::"n"(S::EPI_WARPS * 32) : "memory");
  }
}

template <int KSTEPS>
__global__ void __launch_bounds__(TcShape<KSTEPS>::THREADS, 1) assign_tc_kernel(TcParams p) {
  using S = TcShape<KSTEPS>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  TcSmem s;
  s.a_bytes = (uint32_t)TC_ROWS * p.kp * 4;
  s.b_stage_bytes = (uint32_t)S::N * p.kp * 4;
  s.a = reinterpret_cast<float*>(smem_raw);
  s.b = reinterpret_cast<float*>(smem_raw + (size_t)s.a_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + (size_t)s.a_bytes + (size_t)p.stages * s.b_stage_bytes);
  s.a_full = bars;
  s.a_empty = bars + 1;
  s.a_tmem_free = bars + 2;
  s.b_full = bars + 2 + TC_RT;
  s.b_empty = s.b_full + TC_STAGES;
  s.acc_full = s.b_empty + TC_STAGES;
  s.acc_empty = s.acc_full + 2 * TC_SLOTS;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.acc_empty + 2 * TC_SLOTS);
  s.m_best = reinterpret_cast<float*>(s.tmem_slot + 4);
  s.m_group = reinterpret_cast<int*>(s.m_best + TC_RT * S::WPQ * TC_BM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(s.a_full, 1);
    mbar_init(s.a_empty, TC_RT);  // both MMA threads' copies
    for (int i = 0; i < TC_RT; ++i) mbar_init(s.a_tmem_free + i, 1);
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(s.b_full + i, 1);
      mbar_init(s.b_empty + i, TC_RT);  // both row tiles' MMAs
    }
    for (int i = 0; i < 2 * TC_SLOTS; ++i) {
      mbar_init(s.acc_full + i, 1);
      mbar_init(s.acc_empty + i, S::EPI_PER_RT);  // the warps of the item's row tile
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
    if (lane == 0) tc_producer<KSTEPS>(p, s);
  } else if (warp < S::EPI_WARP0) {
    if (lane == 0) tc_mma<KSTEPS>(p, s, tmem_base, warp - 1);
  } else {
    tc_epilogue<KSTEPS>(p, s, tmem_base, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC_TMEM_COLS);
  }
}

// Shared memory of one CTA for `stages` centroid tiles.
template <int KSTEPS>
static size_t tc_smem_bytes(int kp, int stages) {
  using S = TcShape<KSTEPS>;
  const size_t bars = (2 + TC_RT + 2 * TC_STAGES + 4 * TC_SLOTS) * sizeof(uint64_t) + 16;
  const size_t merge = (size_t)2 * TC_RT * S::WPQ * TC_BM * 4;
  return (size_t)TC_ROWS * kp * 4 + (size_t)stages * S::N * kp * 4 + bars + merge;
}

// Exact re-score of the winning group. On entry labels[b][i] = -(g + 1) for
// the winning group g of 32 centroids; on exit labels[b][i] = the argmax over
// c in [32 g, 32 g + 32) of the exact fp32 reference score (first maximum
// wins). One CTA owns a range of points of one problem and walks the
// problem's centroid table in shared-memory slices stored transposed
// ([group][coordinate][32 centroids]), so that one warp re-scores one point
// with lane l holding centroid 32 g + l: every table read is 32 consecutive
// words (no bank conflicts) and the point's coordinates are broadcast. Each
// lane accumulates its dot product in coordinate order with fused
// multiply-adds, exactly as a sequential loop would; the winner is the
// largest score (NaN never wins), lowest lane among equals, found with a
// warp max over order-preserving keys and a ballot.
// A warp takes its points 32 at a time: lane l loads the label and the
// coordinates of point base + l (one coalesced batch) and stages the
// coordinates in the warp's shared-memory slot; a ballot picks the points
// whose group lies in the current slice, and each of those is scored with its
// coordinates read as broadcast vector loads, so no global-memory latency
// sits between one point and the next. Two CTAs fit an SM, so one CTA's table
// fill overlaps the other's scoring.
constexpr int RF_THREADS = 512;
constexpr int RF_WARPS = RF_THREADS / 32;
constexpr int RF_SMEM = 100 * 1024;

template <int BS>
__device__ __forceinline__ void rf_load_point(const float* xr, int bs, float (&x)[BS > 0 ? BS : 64]) {
  constexpr int XN = BS > 0 ? BS : 64;
  if constexpr (BS > 0 && BS % 4 == 0) {
#pragma unroll
    for (int j = 0; j < BS; j += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xr + j));
      x[j] = v.x; x[j + 1] = v.y; x[j + 2] = v.z; x[j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < XN; ++j)
      if (BS > 0 || j < bs) x[j] = __ldg(xr + j);
  }
}

template <int BS>
__global__ void __launch_bounds__(RF_THREADS, 2)
refine_kernel(int metric, const float* __restrict__ X, const float* __restrict__ C,
              const float* __restrict__ cnorm, int n_pad, int k_pad, int bs_rt, int groups_per_slice,
              int chunk_rows, const int32_t* __restrict__ n, const int32_t* __restrict__ kvec,
              const int32_t* __restrict__ active, int32_t* __restrict__ labels) {
  extern __shared__ float tab[];
  constexpr int XN = BS > 0 ? BS : 64;
  const int bs = BS > 0 ? BS : bs_rt;
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b], kb = kvec[b];
  const int r0 = blockIdx.x * chunk_rows;
  if (r0 >= nb) return;
  const int r1 = min(nb, r0 + chunk_rows);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* cn = tab + (size_t)groups_per_slice * bs * GROUP;
  float* xs = cn + (size_t)groups_per_slice * GROUP + (size_t)warp * GROUP * bs;  // this warp's 32 points
  const int n_groups = ceil_div(kb, GROUP);
  const float* Cb = C + (int64_t)b * k_pad * bs;
  const float* Nb = cnorm + (int64_t)b * k_pad;
  int32_t* Lb = labels + (int64_t)b * n_pad;
  const float* Xb = X + (int64_t)b * n_pad * bs;
  for (int g0 = 0; g0 < n_groups; g0 += groups_per_slice) {
    const int g1 = min(n_groups, g0 + groups_per_slice);
    __syncthreads();
    // one thread per centroid of the slice: its row in, one column of the
    // transposed table out (consecutive threads write consecutive words).
    // Every centroid index here is below k_pad; rows at or past k read as 0.
    const int cents = (g1 - g0) * GROUP;
#pragma unroll 2
    for (int t = threadIdx.x; t < cents; t += RF_THREADS) {
      const int c = g0 * GROUP + t;
      const bool ok = c < kb;
      float row[XN];
      rf_load_point<BS>(Cb + (int64_t)c * bs, bs, row);
      float* dst = tab + (size_t)(t >> 5) * bs * GROUP + (t & 31);
#pragma unroll
      for (int j = 0; j < XN; ++j)
        if (BS > 0 || j < bs) dst[j * GROUP] = ok ? row[j] : 0.f;
      cn[t] = ok ? __ldg(Nb + c) : 0.f;
    }
    __syncthreads();
    for (int base = r0 + warp * 32; base < r1; base += RF_WARPS * 32) {
      const int i_own = base + lane;
      const int v = i_own < r1 ? Lb[i_own] : 0;
      const int g_own = -v - 1;
      const bool mine = v < 0 && g_own >= g0 && g_own < g1;
      uint32_t todo = __ballot_sync(0xffffffffu, mine);
      if (!todo) continue;
      // each lane stages its own point (consecutive points: coalesced loads) in
      // this warp's shared-memory slot; the point being scored is then read by
      // all lanes at one address (broadcast), four coordinates per load when
      // bs % 4 == 0
      __syncwarp();
      if (mine) {
        float xo[XN];
        rf_load_point<BS>(Xb + (int64_t)i_own * bs, bs, xo);
#pragma unroll
        for (int j = 0; j < XN; ++j)
          if (BS > 0 || j < bs) xs[lane * bs + j] = xo[j];
      }
      __syncwarp();
      while (todo) {
        const int k = __ffs(todo) - 1;
        todo &= todo - 1;
        const int g = __shfl_sync(0xffffffffu, g_own, k);
        const float* T = tab + (size_t)(g - g0) * bs * GROUP + lane;
        float x[XN];
        if constexpr (BS > 0 && BS % 4 == 0) {
#pragma unroll
          for (int j = 0; j < BS; j += 4) {
            const float4 q = *reinterpret_cast<const float4*>(xs + k * BS + j);
            x[j] = q.x; x[j + 1] = q.y; x[j + 2] = q.z; x[j + 3] = q.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < XN; ++j)
            if (BS > 0 || j < bs) x[j] = xs[k * bs + j];
        }
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < XN; ++j)
          if (BS > 0 || j < bs) dot = __fmaf_rn(x[j], T[j * GROUP], dot);
        float sc = metric == SKCQ_METRIC_COSINE ? dot : -__fadd_rn(__fmul_rn(dot, -2.0f), cn[(g - g0) * GROUP + lane]);
        if (g * GROUP + lane >= kb || sc != sc) sc = -INFINITY;
        const uint32_t key = float_key(sc + 0.0f);  // -0 and +0 compare equal
        const uint32_t top = __reduce_max_sync(0xffffffffu, key);
        const uint32_t win = __ballot_sync(0xffffffffu, key == top);
        if (lane == 0) Lb[base + k] = g * GROUP + (__ffs(win) - 1);
      }
    }
  }
}

// Re-score for short centroid lists (at most RSO_MAX_GROUPS groups of 32): a
// CTA takes RSO_CHUNK points of one problem, sorts them by winning group in
// shared memory (counting sort), and a warp then holds one group's 32
// centroids in registers (lane = centroid) while it scores every point of
// that group, each point's coordinates read as a broadcast from the warp's
// staging slot. The table is read once per group and chunk instead of once
// per point, which is what bounds refine_kernel (shared-memory reads of the
// group table for every point). Same arithmetic and tie rule as refine_kernel.
constexpr int RSO_CHUNK = 4096;
constexpr int RSO_THREADS = 256;
constexpr int RSO_WARPS = RSO_THREADS / 32;
constexpr int RSO_MAX_GROUPS = 256;

template <int BS>
__global__ void __launch_bounds__(RSO_THREADS) refine_sorted_kernel(
    int metric, const float* __restrict__ X, const float* __restrict__ C, const float* __restrict__ cnorm, int n_pad,
    int k_pad, const int32_t* __restrict__ n, const int32_t* __restrict__ kvec, const int32_t* __restrict__ active,
    int32_t* __restrict__ labels) {
  __shared__ int idx[RSO_CHUNK];
  __shared__ int off[RSO_MAX_GROUPS + 1];
  __shared__ int pos[RSO_MAX_GROUPS];
  __shared__ __align__(16) float xs[RSO_WARPS][32][BS];
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b], kb = kvec[b];
  const int i0 = blockIdx.x * RSO_CHUNK;
  if (i0 >= nb) return;
  const int i1 = min(nb, i0 + RSO_CHUNK);
  const int G = k_pad / GROUP;  // <= RSO_MAX_GROUPS (host check)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int32_t* Lb = labels + (int64_t)b * n_pad;
  for (int g = tid; g < RSO_MAX_GROUPS; g += RSO_THREADS) pos[g] = 0;
  __syncthreads();
  for (int i = i0 + tid; i < i1; i += RSO_THREADS) {
    const int v = Lb[i];
    if (v < 0 && -v - 1 < G) atomicAdd(&pos[-v - 1], 1);
  }
  __syncthreads();
  int tot;
  const int c0 = tid < G ? pos[tid] : 0;
  const int ex = block_exclusive_scan(c0, &tot);  // RSO_THREADS >= RSO_MAX_GROUPS
  if (tid < G) {
    off[tid] = ex;
    pos[tid] = ex;
  }
  if (tid == 0) off[G] = tot;
  __syncthreads();
  for (int i = i0 + tid; i < i1; i += RSO_THREADS) {
    const int v = Lb[i];
    if (v < 0 && -v - 1 < G) idx[atomicAdd(&pos[-v - 1], 1)] = i;
  }
  __syncthreads();
  const float* Cb = C + (int64_t)b * k_pad * BS;
  const float* Nb = cnorm + (int64_t)b * k_pad;
  const float* Xb = X + (int64_t)b * n_pad * BS;
  for (int g = warp; g < G; g += RSO_WARPS) {
    const int p0 = off[g], cnt = off[g + 1] - p0;
    if (cnt == 0) continue;
    const int c = g * GROUP + lane;
    const bool ok = c < kb;
    float cr[BS];
    rf_load_point<BS>(Cb + (int64_t)c * BS, BS, cr);  // c < k_pad: in bounds; values past k unused
    const float cn = ok ? __ldg(Nb + c) : 0.f;
    for (int base = 0; base < cnt; base += 32) {
      const int m = min(32, cnt - base);
      __syncwarp();
      if (lane < m) {
        float xo[BS];
        rf_load_point<BS>(Xb + (int64_t)idx[p0 + base + lane] * BS, BS, xo);
#pragma unroll
        for (int j = 0; j < BS; ++j) xs[warp][lane][j] = xo[j];
      }
      __syncwarp();
      for (int k = 0; k < m; ++k) {
        float x[BS];
        if constexpr (BS % 4 == 0) {
#pragma unroll
          for (int j = 0; j < BS; j += 4) {
            const float4 q = *reinterpret_cast<const float4*>(&xs[warp][k][j]);
            x[j] = q.x; x[j + 1] = q.y; x[j + 2] = q.z; x[j + 3] = q.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < BS; ++j) x[j] = xs[warp][k][j];
        }
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < BS; ++j) dot = __fmaf_rn(x[j], cr[j], dot);
        float sc = metric == SKCQ_METRIC_COSINE ? dot : -__fadd_rn(__fmul_rn(dot, -2.0f), cn);
        if (!ok || sc != sc) sc = -INFINITY;
        const uint32_t key = float_key(sc + 0.0f);
        const uint32_t top = __reduce_max_sync(0xffffffffu, key);
        const uint32_t win = __ballot_sync(0xffffffffu, key == top);
        if (lane == 0) Lb[idx[p0 + base + k]] = g * GROUP + (__ffs(win) - 1);
      }
    }
  }
}

template <int BS>
static cudaError_t launch_refine_sorted(int metric, const float* X, const float* C, const float* cnorm, int nblk,
                                        int n_pad, int k_pad, const int32_t* n, const int32_t* k,
                                        const int32_t* active, int32_t* labels, cudaStream_t s) {
  dim3 grid((unsigned)((n_pad + RSO_CHUNK - 1) / RSO_CHUNK), (unsigned)nblk);
  refine_sorted_kernel<BS><<<grid, RSO_THREADS, 0, s>>>(metric, X, C, cnorm, n_pad, k_pad, n, k, active, labels);
  return cudaGetLastError();
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
static cudaError_t launch_tc(const TcParams& p0, int grid, cudaStream_t s) {
  using S = TcShape<KSTEPS>;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e =
        cudaFuncSetAttribute(assign_tc_kernel<KSTEPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  TcParams p = p0;
  int stages = TC_STAGES;
  while (stages > 2 && tc_smem_bytes<KSTEPS>(p.kp, stages) > 227 * 1024) --stages;
  size_t smem = tc_smem_bytes<KSTEPS>(p.kp, stages);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem < TC_MIN_SMEM) smem = TC_MIN_SMEM;
  p.stages = stages;
  assign_tc_kernel<KSTEPS><<<grid, S::THREADS, smem, s>>>(p);
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
  const size_t group_bytes = (size_t)(GROUP * bs + GROUP) * sizeof(float);
  const size_t stage_bytes = (size_t)RF_WARPS * GROUP * bs * sizeof(float);  // per-warp point slots
  if (stage_bytes + group_bytes > (size_t)RF_SMEM) return cudaErrorInvalidValue;  // bs > 21 never gets here
  const int n_groups = k_pad / GROUP;
  int gps = (int)std::min<size_t>((RF_SMEM - stage_bytes) / group_bytes, (size_t)n_groups);
  if (gps < 1) gps = 1;
  const size_t smem = (size_t)gps * group_bytes + stage_bytes;
  // about four CTAs per SM (two resident at a time), each owning >= 4096
  // points so that the table load amortises
  const int64_t target = (int64_t)num_sms() * 4;
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
  SKCQ_REQUIRE(k_pad > 0 && k_pad % SKCQ_CENT_TILE == 0, SKCQ_ERR_INVALID, "assign: k_pad %d not a multiple of %d",
               k_pad, SKCQ_CENT_TILE);
  SKCQ_REQUIRE((((uintptr_t)A | (uintptr_t)B) & 15) == 0, SKCQ_ERR_INVALID, "assign: operands not 16-byte aligned");
  const int kp = skcq_packed_width(metric, bs);
  SKCQ_REQUIRE(kp / 8 <= TC_MAX_KSTEPS, SKCQ_ERR_INVALID,
               "assign: block size %d too wide for the tensor-core path (use skcq_assign_exact)", bs);
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "assign: no device error word");
  const int64_t n_units = (int64_t)nblk * (n_pad / TC_ROWS);
  const int grid = (int)(n_units < num_sms() ? n_units : num_sms());
  cudaStream_t s = (cudaStream_t)stream;
  TcParams p{A, B, nblk, n_pad, k_pad, kp, 0, n, k, active, labels, err};
  cudaError_t e;
  switch (kp / 8) {
    case 1: e = launch_tc<1>(p, grid, s); break;
    case 2: e = launch_tc<2>(p, grid, s); break;
    case 3: e = launch_tc<3>(p, grid, s); break;
    case 4: e = launch_tc<4>(p, grid, s); break;
    case 5: e = launch_tc<5>(p, grid, s); break;
    case 6: e = launch_tc<6>(p, grid, s); break;
    case 7: e = launch_tc<7>(p, grid, s); break;
    default: e = launch_tc<8>(p, grid, s); break;
  }
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "assign: %s", cudaGetErrorString(e));
  SKCQ_REQUIRE(nblk <= 65535, SKCQ_ERR_INVALID, "assign: %d problems exceed 65535", nblk);
  const bool sorted = k_pad / GROUP <= RSO_MAX_GROUPS && (bs == 4 || bs == 6 || bs == 8 || bs == 12 || bs == 16);
  if (sorted) {
    switch (bs) {
      case 4: e = launch_refine_sorted<4>(metric, X, C, cnorm, nblk, n_pad, k_pad, n, k, active, labels, s); break;
      case 6: e = launch_refine_sorted<6>(metric, X, C, cnorm, nblk, n_pad, k_pad, n, k, active, labels, s); break;
      case 8: e = launch_refine_sorted<8>(metric, X, C, cnorm, nblk, n_pad, k_pad, n, k, active, labels, s); break;
      case 12: e = launch_refine_sorted<12>(metric, X, C, cnorm, nblk, n_pad, k_pad, n, k, active, labels, s); break;
      default: e = launch_refine_sorted<16>(metric, X, C, cnorm, nblk, n_pad, k_pad, n, k, active, labels, s); break;
    }
    if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "assign (refine): %s", cudaGetErrorString(e));
    return SKCQ_OK;
  }
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
